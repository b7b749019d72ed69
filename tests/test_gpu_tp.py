"""Fused row-parallel all-reduce (wlq_gemv_allreduce) across 2, 4 and 8 GPUs
(each size runs when that many GPUs are present): every rank takes its K
shard of one layer -- cut the way vLLM's row-parallel layers shard K,
codebook groups carried with their offset -- through the GEMV with the sum
over ranks done inside the kernel over NVLink peer memory.  The ranks'
outputs must be identical bit for bit, and match the oracle's float64 forward
of the UNSHARDED layer.  Eager calls (h given, and h = A x of the rank's
columns computed in the kernel), a down-proj shard with a forced 11-CTA K
split feeding the exchange, and CUDA-graph replays (the per-tile epochs
advance on the device)."""
import os
import socket

import numpy as np
import pytest
import torch

from _layers import make_np_parts, rel_err
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TOL = 2e-2  # bf16 activations, normwise max relative error


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


# (name, N, K, tokens, forced K split of each rank's GEMV or 0)
CASES = [("o", 512, 3584, (1, 5, 16), 0), ("down", 256, 18944, (1, 16), 11)]


def _inputs(seed, K, M):
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(torch.bfloat16)


def _rank_main(rank, world, port, results):
    import sys
    import ctypes
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from datetime import timedelta
    import torch.distributed as dist
    from _gpu import dev_layer
    from qwen_wlqfastshot_helen_beta_b200 import _C, _lib
    from qwen_wlqfastshot_helen_beta_b200.tp import TPComm
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    comm = None
    out = {}
    try:
        comm = TPComm(max_N=max(c[1] for c in CASES))
        for ci, (name, N, K, Ms, split) in enumerate(CASES):
            P = make_np_parts(np.random.default_rng(100 + ci), N, K, 128, 0.005, 16)
            Kp = K // world
            S = P.shard(rank * Kp, (rank + 1) * Kp)
            T = dev_layer(S)
            lut = _C.prepack_lut(T["lut"], torch.bfloat16)
            cols, vals = _C.prepack_outliers(T["q"], T["lut"], T["off"], T["cols"], T["vals"], N, Kp, 4,
                                             torch.bfloat16, S.G, S.goff)
            A = T["A"].to(torch.bfloat16).contiguous()

            def fused(x, y, h=None):
                _C.gemv_allreduce(comm, x, T["q"], lut, y, N, Kp, 4, S.wpr, T["off"], cols, vals, h, T["B"],
                                  T["gamma"], S.scale, S.G, S.goff, 1, lora_A=None if h is not None else A)

            if split:
                _lib.check(_lib.lib.wlq_gemv_set_split(split), "wlq_gemv_set_split")
            try:
                for M in Ms:
                    for i in range(3):  # repeated calls: epochs and slot parity advance
                        x = _inputs(1000 * ci + 10 * M + i, K, M)[:, rank * Kp:(rank + 1) * Kp].contiguous().to(dev)
                        y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
                        if i % 2 == 0:  # h = A x of this rank's columns inside the kernel
                            fused(x, y)
                        else:           # h given
                            fused(x, y, _C.lora_h(x, A))
                        torch.cuda.synchronize()
                        out[(name, M, i)] = y.float().cpu().numpy()
                if split:
                    out[(name, "split")] = int(_lib.lib.wlq_gemv_last_split())
            finally:
                _lib.check(_lib.lib.wlq_gemv_set_split(0), "wlq_gemv_set_split")
        # a CUDA graph of the o shard, replayed with new inputs
        name, N, K, _, _ = CASES[0]
        P = make_np_parts(np.random.default_rng(100), N, K, 128, 0.005, 16)
        Kp = K // world
        S = P.shard(rank * Kp, (rank + 1) * Kp)
        T = dev_layer(S)
        lut = _C.prepack_lut(T["lut"], torch.bfloat16)
        cols, vals = _C.prepack_outliers(T["q"], T["lut"], T["off"], T["cols"], T["vals"], N, Kp, 4,
                                         torch.bfloat16, S.G, S.goff)
        A = T["A"].to(torch.bfloat16).contiguous()
        M = 8
        x = torch.empty((M, Kp), dtype=torch.bfloat16, device=dev)
        y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)

        def call():
            _C.gemv_allreduce(comm, x, T["q"], lut, y, N, Kp, 4, S.wpr, T["off"], cols, vals, None, T["B"],
                              T["gamma"], S.scale, S.G, S.goff, 1, lora_A=A)

        x.copy_(_inputs(77, K, M)[:, rank * Kp:(rank + 1) * Kp].to(dev))
        call()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                call()
        torch.cuda.current_stream().wait_stream(s)
        for i in range(3):
            x.copy_(_inputs(500 + i, K, M)[:, rank * Kp:(rank + 1) * Kp].to(dev))
            dist.barrier()
            g.replay()
            torch.cuda.synchronize()
            out[("graph", M, i)] = y.float().cpu().numpy()
        del g
        torch.cuda.synchronize()
        out["flag"] = comm.error()
        results[rank] = out
    finally:
        dist.barrier()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_allreduce_matches_unsharded_oracle(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=900)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [dict(results[r]) for r in range(world)]
    assert all(r["flag"] == 0 for r in res), [r["flag"] for r in res]
    # every rank holds the same sum, bit for bit
    keys = [k for k in res[0] if k != "flag" and not (isinstance(k, tuple) and k[1] == "split")]
    for k in keys:
        for r in range(1, world):
            assert np.array_equal(res[0][k], res[r][k]), (k, r)
    # against the oracle's float64 forward of the unsharded layer
    for ci, (name, N, K, Ms, split) in enumerate(CASES):
        P = make_np_parts(np.random.default_rng(100 + ci), N, K, 128, 0.005, 16)
        L = P.full()
        W = L.dense()
        if split:
            assert all(r[(name, "split")] == split for r in res), [r[(name, "split")] for r in res]
        for M in Ms:
            for i in range(3):
                x = _inputs(1000 * ci + 10 * M + i, K, M).float().numpy()
                h = x.astype(np.float64) @ P.A.astype(np.float64).T
                ref = O.forward_f64(W, x, h, P.B, P.gamma, P.scale)
                e = rel_err(res[0][(name, M, i)], ref)
                assert e <= TOL, (name, M, i, e)
    P = make_np_parts(np.random.default_rng(100), *CASES[0][1:3], 128, 0.005, 16)
    W = P.full().dense()
    for i in range(3):
        x = _inputs(500 + i, CASES[0][2], 8).float().numpy()
        h = x.astype(np.float64) @ P.A.astype(np.float64).T
        e = rel_err(res[0][("graph", 8, i)], O.forward_f64(W, x, h, P.B, P.gamma, P.scale))
        assert e <= TOL, ("graph", i, e)


def test_fused_allreduce_wait_runs_out():
    """A peer that never arrives: rank 0 of a 2-rank group whose second
    buffer nobody writes.  The kernel's bounded wait gives up (2 s), sets the
    error word and returns; the context stays usable."""
    import ctypes
    import time
    from qwen_wlqfastshot_helen_beta_b200 import _C, _lib, synthetic as S
    lib = _lib.lib
    N, K = 64, 512
    bufs = []
    for _ in range(2):
        ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
        _lib.check(lib.wlq_tp_buffer_alloc(int(lib.wlq_tp_buffer_bytes(2, N)), ctypes.byref(ptr), handle), "alloc")
        bufs.append(ptr.value)

    class Lonely:  # the shape TPComm has, with a silent second rank
        world, rank, max_N = 2, 0, N
        bufs_c = (ctypes.c_void_p * 2)(*bufs)
    Lonely.bufs = Lonely.bufs_c
    try:
        L = S.make_layer(N, K, group_size=128, density=0.01, r=16, seed=3).prepack(torch.bfloat16)
        x = torch.randn((2, K), device="cuda").to(torch.bfloat16)
        h = S.lora_h(L, x)
        y = torch.zeros((2, N), dtype=torch.bfloat16, device="cuda")
        t0 = time.time()
        _C.gemv_allreduce(Lonely, x, L.q_packed, L.lut_packed, y, N, K, 4, L.words_per_row, L.chunk_offsets,
                          L.cols_packed, L.delta_packed, h, L.lora_B, L.dora_gamma, L.lora_scale, L.group_size,
                          L.group_offset, 1)
        torch.cuda.synchronize()
        waited = time.time() - t0
        flags = ctypes.c_uint(0)
        _lib.check(lib.wlq_tp_error(ctypes.c_void_p(bufs[0]), ctypes.byref(flags), 1), "wlq_tp_error")
        assert flags.value & 1, "the wait should have run out"
        assert 1.0 < waited < 30.0, waited
        # the context is still usable: a plain call gives the right answer
        ref = S.forward(L, x, h=h)
        again = S.forward(L, x, h=h)
        assert torch.equal(ref, again)
    finally:
        for b in bufs:
            lib.wlq_tp_buffer_free(ctypes.c_void_p(b))
