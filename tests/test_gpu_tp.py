"""Fused row-parallel all-reduce (wlq_gemv_allreduce) on 2 GPUs: each rank's
K shard through the GEMV with the sum over ranks done in the kernel over
NVLink peer memory, against the ranks' own outputs summed after an NCCL
all-gather.  Eager calls (h given, or h = A x of the rank's columns of A
computed in the kernel) and CUDA-graph replays (the per-tile epochs advance
on the device), several token counts.  Skipped with fewer than 2 GPUs."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, port, results):
    import sys
    sys.path.insert(0, ROOT)
    from datetime import timedelta
    import torch.distributed as dist
    from qwen_wlqfastshot_helen_beta_b200 import _C, synthetic as S
    from qwen_wlqfastshot_helen_beta_b200.tp import TPComm
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            timeout=timedelta(seconds=60), device_id=dev)
    comm = None
    try:
        N, Kp = 3584, 1792  # row-parallel shard of a 3584-wide K
        L = S.make_layer(N, Kp, group_size=128, density=0.005, r=16, seed=40 + rank, device=dev)
        L.prepack(torch.bfloat16)
        comm = TPComm(max_N=N)
        lut, cols, vals, fmt = L.operands_for(torch.bfloat16)
        errs = []
        gen = torch.Generator(device=dev)
        gen.manual_seed(9 + rank)

        def fused(x, h, out, in_kernel_h=False):
            if in_kernel_h:  # this rank's columns of A, h = A x computed in the kernel
                _C.gemv_allreduce(comm, x, L.q_packed, lut, out, N, Kp, 4, L.words_per_row, L.chunk_offsets, cols,
                                  vals, None, L.lora_B, L.dora_gamma, L.lora_scale, L.group_size, L.group_offset,
                                  fmt, lora_A=L.lora_A_act)
                return
            _C.gemv_allreduce(comm, x, L.q_packed, lut, out, N, Kp, 4, L.words_per_row, L.chunk_offsets, cols,
                              vals, h, L.lora_B, L.dora_gamma, L.lora_scale, L.group_size, L.group_offset, fmt)

        def check(x, h, y):
            own = S.forward(L, x, h=h).float()
            parts = [torch.empty_like(own) for _ in range(2)]
            dist.all_gather(parts, own)
            ref = parts[0] + parts[1]
            errs.append(float((y.float() - ref).abs().max() / ref.abs().max()))

        for M in (1, 5, 16):
            for i in range(4):  # repeated calls: epochs and slot parity advance
                x = torch.randn((M, Kp), generator=gen, device=dev).to(torch.bfloat16)
                h = S.lora_h(L, x)
                y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
                fused(x, h, y, in_kernel_h=i % 2 == 1)
                check(x, h, y)
        # a down-proj shard (K = 9472 per rank): the K split takes a cluster of
        # more than 8 CTAs, whose reduction feeds the exchange
        Kd = 9472
        Ld = S.make_layer(N, Kd, group_size=128, density=0.005, r=16, seed=60 + rank, device=dev)
        Ld.prepack(torch.bfloat16)
        lutd, colsd, valsd, fmtd = Ld.operands_for(torch.bfloat16)
        for M in (1, 16):
            x = torch.randn((M, Kd), generator=gen, device=dev).to(torch.bfloat16)
            h = S.lora_h(Ld, x)
            y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            _C.gemv_allreduce(comm, x, Ld.q_packed, lutd, y, N, Kd, 4, Ld.words_per_row, Ld.chunk_offsets, colsd,
                              valsd, None, Ld.lora_B, Ld.dora_gamma, Ld.lora_scale, Ld.group_size, Ld.group_offset,
                              fmtd, lora_A=Ld.lora_A_act)
            own = S.forward(Ld, x, h=h).float()
            parts = [torch.empty_like(own) for _ in range(2)]
            dist.all_gather(parts, own)
            ref = parts[0] + parts[1]
            errs.append(float((y.float() - ref).abs().max() / ref.abs().max()))
        # the same inside a CUDA graph, replayed with new inputs
        M = 8
        x = torch.randn((M, Kp), generator=gen, device=dev).to(torch.bfloat16)
        h = S.lora_h(L, x)
        y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        fused(x, h, y)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                fused(x, h, y)
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(3):
            x.copy_(torch.randn((M, Kp), generator=gen, device=dev).to(torch.bfloat16))
            h.copy_(S.lora_h(L, x))
            dist.barrier()
            g.replay()
            torch.cuda.synchronize()
            check(x, h, y)
        del g
        torch.cuda.synchronize()
        results[rank] = {"errs": errs, "flag": comm.error()}
    finally:
        dist.barrier()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def test_fused_allreduce_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(2):
        res = dict(results[r])
        assert res["flag"] == 0, res
        assert max(res["errs"]) <= 1e-2, res


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
