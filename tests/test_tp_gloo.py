"""Tensor-parallel sharding of the WLQ linear, world size 2 on CPU (gloo).

Each rank loads its shard of one full checkpoint through WLQLinearMethod's
load path (the reference's slicing, vllm_wlq/linear_method.py:676-935):
row-parallel layers split K (and the chunk-CSR / index columns), column-
parallel layers split N.  Each rank evaluates its shard with the oracle and
the ranks combine the partial outputs the way vLLM does (all-reduce for
row-parallel, all-gather for column-parallel); the result must equal the
unsharded layer.  No GPU: this checks the host-side sharding and the
collective composition that bench.py --gpus N runs over NCCL."""
import os
import socket
from types import SimpleNamespace

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _checkpoint(seed, N, K, dens):
    """One shard in the reference's on-disk format (continuous 4-bit words,
    per-row fp16 codebooks, 1-bit outlier mask + fp16 values)."""
    rng = np.random.default_rng(seed)
    lut = np.sort(rng.standard_normal((N, 16)) * 0.02, axis=1).astype(np.float16)
    idx = rng.integers(0, 16, size=(N, K), dtype=np.uint32).reshape(-1)
    idx = np.concatenate([idx, np.zeros((-idx.size) % 8, np.uint32)]).reshape(-1, 8)
    words = np.bitwise_or.reduce(idx << (np.arange(8, dtype=np.uint32) * 4)[None, :], axis=1)
    mask = rng.random((N, K)) < dens
    vals = (rng.standard_normal(int(mask.sum())) * 0.1).astype(np.float16)
    return {"q_packed": words.view(np.int32), "lut_c": lut, "bits": np.array([4], np.int32),
            "outlier_values": vals, "outlier_mask_1bit": np.packbits(mask.reshape(-1))}


def _load(lm, ck, rank, tp, row_par, N, K):
    lm.get_tp_info = lambda: (rank, tp)
    torch.cuda.is_available = lambda: False
    method = lm.WLQLinearMethod(SimpleNamespace(bits=4, model_id=None, lut_group_size=0))
    layer = torch.nn.Module()
    layer.is_row_parallel = row_par
    K_part = K // tp if row_par else K
    N_part = N if row_par else N // tp
    method.create_weights(layer, K_part, [N_part], K, N, torch.float16)
    layer.vllm_prefix = "model.layers.0.mlp.down_proj" if row_par else "model.layers.0.mlp.gate_up_proj"
    for nm, arr in ck.items():
        prm = getattr(layer, nm)
        prm.weight_loader(prm, torch.from_numpy(np.ascontiguousarray(arr)))
    method.process_weights_after_loading(layer)
    return layer


def _dense(O, layer):
    return O.dequant(layer.q_packed_aligned.numpy().view(np.uint32).reshape(-1), layer.words_per_row,
                     layer.lut_c.numpy(), layer.N, layer.K, 4, 0, 0, layer.chunk_offsets.numpy(),
                     layer.chunk_cols.numpy(), layer.chunk_vals.numpy())


def _rank_main(rank, port, results):
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    from oracle import oracle as O
    from qwen_wlqfastshot_helen_beta_b200 import linear_method as lm
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
    try:
        N, K, M = 96, 1536, 5
        x = np.random.default_rng(3).standard_normal((M, K)).astype(np.float16).astype(np.float64)
        out = {}
        for row_par in (True, False):
            ck = _checkpoint(11 if row_par else 12, N, K, 0.01)
            full = _load(lm, ck, 0, 1, row_par, N, K)
            ref = O.forward_f64(_dense(O, full), x)
            shard = _load(lm, ck, rank, 2, row_par, N, K)
            if row_par:
                xs = x[:, rank * (K // 2):(rank + 1) * (K // 2)]
                y = torch.from_numpy(np.ascontiguousarray(O.forward_f64(_dense(O, shard), xs)))
                dist.all_reduce(y)  # the row-parallel all-reduce after o / down
            else:
                part = torch.from_numpy(np.ascontiguousarray(O.forward_f64(_dense(O, shard), x)))
                parts = [torch.empty_like(part) for _ in range(2)]
                dist.all_gather(parts, part)  # column-parallel outputs are concatenated
                y = torch.cat(parts, dim=1)
            out["row" if row_par else "col"] = float(np.max(np.abs(y.numpy() - ref)) / np.max(np.abs(ref)))
        results[rank] = out
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_tp2_shards_recombine_to_the_full_layer():
    pytest.importorskip("vllm")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(2):
        assert results[r]["row"] <= 1e-12 and results[r]["col"] <= 1e-12, dict(results[r])
