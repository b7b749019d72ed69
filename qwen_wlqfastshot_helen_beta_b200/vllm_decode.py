"""A random-initialised Qwen2.5-7B-shaped WLQ model decoding inside vLLM
batch 32, 1024 random prompt tokens each, 256 generated
tokens, every linear through this package's quantisation method.

The checkpoint comes from checkpoint.write_checkpoint (the reference's
on-disk format, loaded by vLLM's own Qwen2 loader).  The engine runs in this
process (VLLM_ENABLE_V1_MULTIPROCESSING=0), so importing the package is what
registers ``wlq_fastShot`` with vLLM, as the reference's ``register`` entry
point does.  Decode steps run as full CUDA graphs without torch.compile.

Prints one JSON line: output tokens per second over the whole generate call
(prefill included), and the decode rate alone from the difference with a
1-token run.

    python -m qwen_wlqfastshot_helen_beta_b200.vllm_decode --model /tmp/wlq_qwen7b --write
"""
from __future__ import annotations

import argparse
import json
import os
import time


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--model", required=True, help="checkpoint directory")
    ap.add_argument("--write", action="store_true", help="write the synthetic checkpoint first (if absent)")
    ap.add_argument("--layers", type=int, default=None, help="layer count override when writing (default 28)")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--prompt", type=int, default=1024)
    ap.add_argument("--gen", type=int, default=256)
    ap.add_argument("--gpu-mem", type=float, default=0.80)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)

    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    from . import checkpoint
    if a.write and not os.path.isfile(os.path.join(a.model, "config.json")):
        t0 = time.time()
        checkpoint.write_checkpoint(a.model, num_layers=a.layers, seed=a.seed)
        print(f"checkpoint written in {time.time() - t0:.0f} s", flush=True)

    import numpy as np
    from vllm import LLM, SamplingParams
    from . import register
    register()  # WLQFastShotConfig -> vLLM's quantization registry

    llm = LLM(model=a.model, dtype="bfloat16", skip_tokenizer_init=True, seed=a.seed,
              max_model_len=a.prompt + a.gen + 16, max_num_seqs=a.batch, gpu_memory_utilization=a.gpu_mem,
              enable_prefix_caching=False,  # every run prefills its prompts
              compilation_config={"mode": 0, "cudagraph_mode": "FULL_DECODE_ONLY"})
    with open(os.path.join(a.model, "config.json")) as f:
        vocab = json.load(f)["vocab_size"]
    rng = np.random.default_rng(a.seed)
    prompts = [{"prompt_token_ids": rng.integers(0, vocab, size=a.prompt).tolist()} for _ in range(a.batch)]

    def run(n):
        sp = SamplingParams(max_tokens=n, min_tokens=n, ignore_eos=True, temperature=0.0, detokenize=False)
        t = time.perf_counter()
        outs = llm.generate(prompts, sp, use_tqdm=False)
        dt = time.perf_counter() - t
        ntok = sum(len(o.outputs[0].token_ids) for o in outs)
        return dt, ntok

    run(4)  # warm-up
    t1, _ = run(1)
    tg, ntok = run(a.gen)
    decode_tok = a.batch * (a.gen - 1)
    print(json.dumps({
        "metric": "Qwen2.5-7B decode tok/s (vLLM, every linear WLQ)",
        "value": round(ntok / tg, 1), "unit": "tok/s",
        "decode_tok_s": round(decode_tok / max(tg - t1, 1e-9), 1),
        "prefill_s": round(t1, 3), "generate_s": round(tg, 3), "tokens": ntok,
        "config": {"model": os.path.basename(os.path.normpath(a.model)), "batch": a.batch, "prompt": a.prompt,
                   "gen": a.gen, "dtype": "bf16", "parallelism": "single",
                   "cudagraph_mode": "FULL_DECODE_ONLY", "compile": "off"},
    }), flush=True)


if __name__ == "__main__":
    main()
