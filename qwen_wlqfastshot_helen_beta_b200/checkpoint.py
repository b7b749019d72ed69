"""Synthetic WLQ checkpoints in the reference's on-disk format, for running a
random-initialised model inside vLLM (BASELINE configs 3 and 4).

vLLM's dummy loader cannot create WLQ layers (it fills only floating-point
parameters of known shape), so the model is written to disk the way the
reference's checkpoints are laid out and then loaded through the normal
path, ``WLQLinearMethod.create_weights`` / ``process_weights_after_loading``
(vllm_wlq/linear_method.py:376-408, 413-935):

* per quantised projection (``q_proj`` ... ``down_proj``): ``q_packed``
  (int32 words, the row-major [N, K] 4-bit indices packed 8 per word,
  least significant nibble first, continuous across rows), ``lut_c`` (fp16
  codebooks, [N, 16] or [N, groups, 16] with ``lut_group_size``), ``bits``,
  ``outlier_mask_1bit`` (np.packbits of the [N, K] outlier mask) and
  ``outlier_values`` (fp16, in mask order);
* the DoRA adapter in ``lora_adapter_distilled/adapter_model.safetensors``
  (``lora_A`` [r, K], ``lora_B`` [N, r], ``lora_magnitude_vector`` [N] per
  projection) with its ``adapter_config.json`` (vllm_wlq/linear_method.py:21-120);
* everything else (embeddings, norms, qkv biases, lm_head) in bf16; the
  embedding and lm_head tables repeat a block of 4096 random rows.

Values follow the BASELINE recipe: codebook levels sigma * Phi^-1((i + 0.5) / 16)
* (1 + U(-0.05, 0.05)) sorted per (row, group), indices uniform (the quantile
levels make every level equally likely for Gaussian weights), 0.5 % outliers at
uniform positions with N(0, 0.1) values, A, B ~ N(0, 0.01) and magnitudes the
row norm of N(0, 0.02) weights times (1 + U(-0.1, 0.1)).  Written layer by
layer with numpy, so a 7B model needs no GPU and a few GB of host memory.
"""
from __future__ import annotations

import json
import os
from statistics import NormalDist
from typing import Dict, Optional

import numpy as np

QWEN25_7B = {
    "hidden_size": 3584, "intermediate_size": 18944, "num_hidden_layers": 28, "num_attention_heads": 28,
    "num_key_value_heads": 4, "vocab_size": 152064, "rope_theta": 1000000.0, "rms_norm_eps": 1e-6,
    "max_position_embeddings": 32768,
}

_Q16 = np.array([NormalDist().inv_cdf((i + 0.5) / 16) for i in range(16)], np.float64)


def _projections(arch: Dict) -> Dict[str, tuple]:
    """(K in, N out, module) of every quantised projection of one layer."""
    h, inter = arch["hidden_size"], arch["intermediate_size"]
    hd = h // arch["num_attention_heads"]
    kv = arch["num_key_value_heads"] * hd
    return {"q_proj": (h, h, "self_attn"), "k_proj": (h, kv, "self_attn"), "v_proj": (h, kv, "self_attn"),
            "o_proj": (h, h, "self_attn"), "gate_proj": (h, inter, "mlp"), "up_proj": (h, inter, "mlp"),
            "down_proj": (inter, h, "mlp")}


def quantised_projection(rng: np.random.Generator, N: int, K: int, group_size: int, density: float,
                         sigma: float = 0.02) -> Dict[str, np.ndarray]:
    """One projection's checkpoint tensors in the reference's layout."""
    total = N * K
    nwords = -(-total // 8)
    q = rng.integers(0, 1 << 32, size=nwords, dtype=np.uint64).astype(np.uint32)
    tail = total - (nwords - 1) * 8  # symbols in the last word
    if tail < 8:
        q[-1] &= np.uint32((1 << (4 * tail)) - 1)
    ng = -(-K // group_size) if group_size > 0 else 1
    shape = (N, ng, 16) if group_size > 0 else (N, 16)
    std = sigma * (1.0 + rng.uniform(-0.02, 0.02, size=shape[:-1] + (1,)))
    jit = 1.0 + rng.uniform(-0.05, 0.05, size=shape)
    lut = np.sort(std * _Q16 * jit, axis=-1).astype(np.float16)
    nnz = int(round(total * density))
    pos = np.unique(rng.integers(0, total, size=int(nnz * 1.02) + 16, dtype=np.int64))
    pos = np.sort(rng.permutation(pos)[:nnz])
    mask = np.zeros(-(-total // 8), np.uint8)
    np.bitwise_or.at(mask, pos >> 3, (0x80 >> (pos & 7)).astype(np.uint8))
    vals = (rng.standard_normal(pos.size) * 0.1).astype(np.float16)
    return {"q_packed": q.view(np.int32), "lut_c": lut, "bits": np.array([4], np.int32),
            "outlier_mask_1bit": mask, "outlier_values": vals}


def _table(rng: np.random.Generator, rows: int, cols: int, block: int = 4096) -> np.ndarray:
    """[rows, cols] float32 N(0, 0.02) table (embeddings, lm_head): a block of
    random rows repeated, which is all a throughput run needs and keeps a
    150k-row vocabulary from dominating the write time."""
    b = rng.standard_normal((min(rows, block), cols), np.float32) * 0.02
    return np.resize(b, (rows, cols))


def _save(tensors: Dict[str, np.ndarray], path: str, bf16_names=()) -> None:
    """safetensors file; arrays named in bf16_names (float32) stored as bf16."""
    import torch
    from safetensors.torch import save_file
    out = {}
    for k, v in tensors.items():
        t = torch.from_numpy(np.ascontiguousarray(v))
        out[k] = t.to(torch.bfloat16) if k in bf16_names else t
    save_file(out, path)


def write_checkpoint(out_dir: str, arch: Optional[Dict] = None, num_layers: Optional[int] = None, *,
                     group_size: int = 128, density: float = 0.005, rank: int = 16, lora_alpha: Optional[int] = None,
                     seed: int = 0, shard_bytes: int = 2 << 30) -> str:
    """Writes a random-initialised Qwen2-architecture WLQ checkpoint to
    out_dir (config.json, safetensors shards + index, DoRA adapter) and
    returns out_dir.  num_layers overrides the architecture's layer count."""
    arch = dict(QWEN25_7B if arch is None else arch)
    if num_layers is not None:
        arch["num_hidden_layers"] = int(num_layers)
    os.makedirs(out_dir, exist_ok=True)
    out_dir = os.path.abspath(out_dir)
    rng = np.random.default_rng(seed)
    h, vocab = arch["hidden_size"], arch["vocab_size"]
    hd = h // arch["num_attention_heads"]
    kv = arch["num_key_value_heads"] * hd
    weight_map: Dict[str, str] = {}
    shard: Dict[str, np.ndarray] = {}
    shard_bf16 = set()
    shard_size = 0
    shard_files = []

    def flush():
        nonlocal shard, shard_size, shard_bf16
        if not shard:
            return
        name = f"model-{len(shard_files) + 1:05d}.safetensors"
        _save(shard, os.path.join(out_dir, name), shard_bf16)
        for k in shard:
            weight_map[k] = name
        shard_files.append(name)
        shard, shard_size, shard_bf16 = {}, 0, set()

    def put(name, arr, bf16=False):
        nonlocal shard_size
        shard[name] = arr
        if bf16:  # float32 here, bf16 on disk
            shard_bf16.add(name)
        shard_size += arr.nbytes // 2 if bf16 else arr.nbytes
        if shard_size >= shard_bytes:
            flush()

    put("model.embed_tokens.weight", _table(rng, vocab, h), bf16=True)
    adapter: Dict[str, np.ndarray] = {}
    for li in range(arch["num_hidden_layers"]):
        pre = f"model.layers.{li}"
        put(f"{pre}.input_layernorm.weight", np.ones(h, np.float32), bf16=True)
        put(f"{pre}.post_attention_layernorm.weight", np.ones(h, np.float32), bf16=True)
        for proj, (K, N, mod) in _projections(arch).items():
            for k, v in quantised_projection(rng, N, K, group_size, density).items():
                put(f"{pre}.{mod}.{proj}.{k}", v)
            if proj in ("q_proj", "k_proj", "v_proj"):
                put(f"{pre}.{mod}.{proj}.bias", rng.standard_normal(N, np.float32) * 0.02, bf16=True)
            if rank > 0:
                ak = f"base_model.model.{pre}.{mod}.{proj}"
                adapter[f"{ak}.lora_A.weight"] = (rng.standard_normal((rank, K), np.float32) * 0.01).astype(np.float16)
                adapter[f"{ak}.lora_B.weight"] = (rng.standard_normal((N, rank), np.float32) * 0.01).astype(np.float16)
                mag = 0.02 * np.sqrt(K) * (1.0 + rng.uniform(-0.1, 0.1, size=N))
                adapter[f"{ak}.lora_magnitude_vector"] = mag.astype(np.float16)
    put("model.norm.weight", np.ones(h, np.float32), bf16=True)
    put("lm_head.weight", _table(rng, vocab, h), bf16=True)
    flush()
    with open(os.path.join(out_dir, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f)

    config = {
        "architectures": ["Qwen2ForCausalLM"], "model_type": "qwen2", "hidden_act": "silu",
        "hidden_size": h, "intermediate_size": arch["intermediate_size"],
        "num_hidden_layers": arch["num_hidden_layers"], "num_attention_heads": arch["num_attention_heads"],
        "num_key_value_heads": arch["num_key_value_heads"], "head_dim": hd, "vocab_size": vocab,
        "max_position_embeddings": arch["max_position_embeddings"], "rope_theta": arch["rope_theta"],
        "rms_norm_eps": arch["rms_norm_eps"], "tie_word_embeddings": False, "torch_dtype": "bfloat16",
        "use_sliding_window": False, "sliding_window": None, "max_window_layers": arch["num_hidden_layers"],
        "attention_dropout": 0.0, "bos_token_id": 0, "eos_token_id": 1, "use_cache": True,
        "quantization_config": {"quant_method": "wlq_fastShot", "bits": 4, "lut_group_size": group_size,
                                "use_dora": rank > 0, "_name_or_path": out_dir},
    }
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(config, f, indent=1)
    if rank > 0:
        ad = os.path.join(out_dir, "lora_adapter_distilled")
        os.makedirs(ad, exist_ok=True)
        _save(adapter, os.path.join(ad, "adapter_model.safetensors"))
        with open(os.path.join(ad, "adapter_config.json"), "w") as f:
            json.dump({"r": rank, "lora_alpha": lora_alpha if lora_alpha is not None else rank, "use_dora": True,
                       "target_modules": list(_projections(arch))}, f)
    return out_dir


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("out_dir")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count (default: 28)")
    ap.add_argument("--group-size", type=int, default=128)
    ap.add_argument("--density", type=float, default=0.005)
    ap.add_argument("--rank", type=int, default=16)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args()
    print(write_checkpoint(a.out_dir, num_layers=a.layers, group_size=a.group_size, density=a.density,
                           rank=a.rank, seed=a.seed))
