"""Benchmark of the WLQ 4-bit LUT decode GEMV on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (config 1): the four Qwen2.5-7B linears -- qkv 3584->4608, o
3584->3584, gate_up 3584->37888, down 18944->3584 -- at decode batch
M in {1, 4, 8, 16}, bf16 activations, benchmark quantisation recipe (one
16-entry fp16 codebook per row and 128 columns, DoRA rank 16, 0.5% outliers),
seeded synthetic weights and activations.  One step = the 16 (linear, M)
forward calls, each through the C ABI entry point wlq_gemm, on one of several
rotating weight copies whose total exceeds the 126 MB L2 (inputs larger than
L2; no flush needed).

Metric: algorithmic bytes (indices, codebooks, outlier CSR, DoRA tensors,
activations, outputs) / time, in GB/s, whole job.  ``value`` times K steps of
a CUDA graph of the step with inputs resident in HBM; ``roofline`` divides
this GPU's bytes per step by the same graph's time per step (kernel time per
step <= ms_per_step) and by the measured HBM copy bandwidth, with per-launch
figures from a second graph that has an event pair around every launch;
``e2e`` times K steps through the public op with host (pinned) activations
copied in and outputs copied out every step.  Sub-objects: ``gemm`` (BASELINE
config 2, the prefill op), ``cpu_baseline`` and ``cpu_baseline_config0``
(the reference's CPU steps; BASELINE config 0 beside this package's op),
``reference_gpu_baseline`` (the reference's own CUDA kernels on this GPU).

With --gpus N > 1 (torchrun, one rank per GPU) the linears are sharded the way
vLLM tensor parallelism shards them (qkv/gate_up by output rows, o/down by
input columns, the latter followed by the all-reduce of [M, hidden]: fused
into the decode GEMV, NCCL after the prefill GEMM); value = bytes of the
whole layer / max-over-ranks time (strong scaling); ``tp_allreduce`` gives
per-call times of the row-parallel layers with and without the fusion.

--impl reference times the reference's CPU dequantize-then-matmul path
(oracle/cpu_baseline.py) on the host cores on the same workload and metric.
--vllm-decode ours|reference runs BASELINE config 3 inside vLLM.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "W4-LUT GEMV GB/s vs HBM peak; GEMM TFLOPS; Qwen2.5-7B decode tok/s"
SHAPES = [("qkv", 3584, 4608), ("o", 3584, 3584), ("gate_up", 3584, 37888), ("down", 18944, 3584)]
MS = [1, 4, 8, 16]
GEMM_MS = [512, 2048, 8192]  # BASELINE config 2 (prefill)
GROUP = 128
RANK = 16
DENSITY = 0.005
FALLBACK_HBM_GBS = 6650.0


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": FALLBACK_HBM_GBS}, "fallback"


# ----------------------------------------------------------------- clocks

class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.period, self.stop_evt, self.thread = period_s, threading.Event(), None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nvml = None

    def _sample(self):
        try:
            self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
            mask = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            for bit, name in self.REASONS.items():
                if mask & bit:
                    self.reasons.add(name)
        except Exception:
            pass

    def _run(self):
        while not self.stop_evt.is_set():
            self._sample()
            time.sleep(self.period)

    def __enter__(self):
        if self.nvml:
            self._sample()
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        return self

    def __exit__(self, *a):
        if self.nvml:
            self.stop_evt.set()
            self.thread.join()
            self._sample()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


# ------------------------------------------------------- graph event nodes

class GraphEvents:
    """Timing events that can be recorded inside a captured CUDA graph
    (cudaEventRecordWithFlags with cudaEventRecordExternal)."""

    def __init__(self):
        import torch
        self.torch = torch
        self.rt = None
        for name in ("libcudart.so.12", "libcudart.so"):
            try:
                self.rt = ctypes.CDLL(name)
                break
            except OSError:
                continue
        if self.rt is not None:
            self.rt.cudaEventRecordWithFlags.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint]
            self.rt.cudaEventRecordWithFlags.restype = ctypes.c_int

    def record(self, ev):
        stream = self.torch.cuda.current_stream()
        if self.rt is None:
            ev.record(stream)
            return
        rc = self.rt.cudaEventRecordWithFlags(ctypes.c_void_p(ev.cuda_event), ctypes.c_void_p(stream.cuda_stream), 1)
        if rc != 0:
            raise RuntimeError(f"cudaEventRecordWithFlags failed: {rc}")


# ------------------------------------------------------------ workloads

def build_layers(copies, rank, world, device, seed0=1000):
    """copies x 4 linears (the rank's tensor-parallel shard of each)."""
    import torch
    from qwen_wlqfastshot_helen_beta_b200 import synthetic as S
    layers = []
    for c in range(copies):
        row = {}
        for si, (name, K, N) in enumerate(SHAPES):
            seed = seed0 + 97 * c + si
            if world > 1 and name in ("qkv", "gate_up"):
                Np = N // world
                L = S.make_layer(Np, K, group_size=GROUP, density=DENSITY, r=RANK, seed=seed + 7919 * rank,
                                 device=device)
            elif world > 1:
                Kp = K // world
                L = S.make_layer(N, Kp, group_size=GROUP, group_offset=(rank * Kp) % GROUP, density=DENSITY,
                                 r=RANK, seed=seed + 7919 * rank, device=device)
            else:
                L = S.make_layer(N, K, group_size=GROUP, density=DENSITY, r=RANK, seed=seed, device=device)
            row[name] = L.prepack(torch.bfloat16)
        layers.append(row)
        torch.cuda.synchronize()
    return layers


def bench_config(world, copies=3):
    """The workload both arms report."""
    return {
        "workload": "qwen2.5-7b decode GEMV sweep (BASELINE config 1): qkv 3584->4608, o 3584->3584, "
                    "gate_up 3584->37888, down 18944->3584 at M in {1,4,8,16}",
        "group_size": GROUP, "lora_rank": RANK, "outlier_density": DENSITY, "act_dtype": "bf16",
        "parallelism": f"tp{world}" if world > 1 else "single",
        "l2": f"inputs larger than L2: {copies} rotating weight copies per rank",
        "timing": "CUDA graph of K steps without per-launch nodes, events around the replay",
        "launch": "consecutive GEMV launches overlap (wlq_gemv_set_overlap(1), programmatic dependent launch): "
                  "weights are static during the timed steps",
    }


def full_layer_bytes(M):
    """Algorithmic bytes of one unsharded (linear, M) call of the recipe."""
    tot = 0
    for name, K, N in SHAPES:
        wpr = ((K + 7) // 8 + 3) // 4 * 4
        ng = (K + GROUP - 1) // GROUP
        nnz = int(round(N * K * DENSITY))
        ncsr = (K + 511) // 512
        tot += N * wpr * 4 + N * ng * 32 + N * (ncsr + 1) * 4 + 3 * nnz
        tot += N * RANK * 2 + N * 2 + RANK * K * 2 + M * K * 2 + M * N * 2
    return tot


def run_ours(args):
    import torch
    import torch.distributed as dist
    from qwen_wlqfastshot_helen_beta_b200 import _C, _lib
    from qwen_wlqfastshot_helen_beta_b200 import synthetic as S

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    peaks, peaks_kind = measured_peaks()
    copies = args.copies
    layers = build_layers(copies, rank, world, dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)

    # resident inputs per (copy, linear, M); the GEMV computes h = A x itself
    calls = []  # (copy, name, M, layer, x, A, out)
    for c in range(copies):
        for name, K, N in SHAPES:
            L = layers[c][name]
            for M in MS:
                x = torch.randn((M, L.K), generator=gen, device=dev).to(torch.bfloat16)
                out = torch.empty((M, L.N), dtype=torch.bfloat16, device=dev)
                calls.append((c, name, M, L, x, L.lora_A_act, out))
    lib = _lib.lib
    stream = torch.cuda.current_stream()
    # the weights are written (built, prepacked) before this point and never
    # during the timed steps: consecutive GEMV launches may overlap
    # (wlq_gemv_set_overlap: a GEMV reads its weights before the previous
    # kernel in the stream has completed)
    torch.cuda.synchronize()
    _lib.check(lib.wlq_gemv_set_overlap(1), "wlq_gemv_set_overlap")

    # row-parallel layers (o, down) at N > 1: the all-reduce fused into the
    # GEMV over NVLink peer memory (wlq_gemv_allreduce)
    comm = None
    if world > 1:
        from qwen_wlqfastshot_helen_beta_b200.tp import TPComm
        comm = TPComm(max_N=max(N for _, _, N in SHAPES))

    def vp(t):
        return ctypes.c_void_p(t.data_ptr())

    def launch(L, x, a, out, name=None):
        """One decode call (M <= 16) with h = A x inside the GEMV."""
        if comm is not None and name in ("o", "down"):
            _C.gemv_allreduce(comm, x, L.q_packed, L.lut_packed, out, L.N, L.K, 4, L.words_per_row,
                              L.chunk_offsets, L.cols_packed, L.delta_packed, None, L.lora_B, L.dora_gamma,
                              L.lora_scale, L.group_size, L.group_offset, _lib.WLQ_LUT_PREPACKED, lora_A=a)
            return
        rc = lib.wlq_gemv_lora_a(vp(L.q_packed), vp(L.lut_packed), vp(x), vp(out), vp(L.chunk_offsets),
                                 vp(L.cols_packed), vp(L.delta_packed), vp(L.lora_B), vp(a), vp(L.dora_gamma),
                                 L.lora_scale, L.r, x.shape[0], L.N, L.K, 4, L.words_per_row, L.group_size,
                                 L.group_offset, _lib.WLQ_LUT_PREPACKED, _lib.WLQ_DTYPE_BF16,
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        _lib.check(rc, "wlq_gemv_lora_a")

    gemm_ws = _C.gemm_workspace(dev)  # the stream-K workspace, made before any capture

    def launch_gemm(L, x, H, out):
        """One prefill call (M > 16) as the op runs it: H = X A^T on this
        package's kernel (wlq_lora_h), then the tensor-core GEMM with its
        stream-K schedule."""
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = lib.wlq_lora_h(vp(x), vp(L.lora_A_act), vp(H), x.shape[0], L.K, L.r, _lib.WLQ_DTYPE_BF16, st)
        _lib.check(rc, "wlq_lora_h")
        rc = lib.wlq_gemm_streamk(vp(x), vp(L.q_packed), vp(L.lut_packed), vp(out), vp(L.chunk_offsets),
                                  vp(L.cols_packed), vp(L.delta_packed), vp(H), vp(L.lora_B), vp(L.dora_gamma),
                                  L.lora_scale, L.r, x.shape[0], L.N, L.K, 4, L.words_per_row, L.group_size,
                                  L.group_offset, _lib.WLQ_LUT_PREPACKED, _lib.WLQ_DTYPE_BF16, vp(gemm_ws),
                                  gemm_ws.numel(), st)
        _lib.check(rc, "wlq_gemm_streamk")

    def reduce_if_rowpar(name, out):  # NCCL only without the fused path
        if world > 1 and comm is None and name in ("o", "down"):
            dist.all_reduce(out)

    # one step per weight copy; per-kernel event nodes inside the graph
    ge = GraphEvents()
    per_copy = [[cl for cl in calls if cl[0] == c] for c in range(copies)]
    steps_total = args.warmup + args.steps
    order = [s % copies for s in range(steps_total)]
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(2 * 16 * steps_total)]
    for ev in evs:  # torch creates the CUDA event on first record; do it outside capture
        ev.record()

    # eager warm-up (also loads the kernels) before capture
    for c in range(copies):
        for (_, name, M, L, x, a, out) in per_copy[c]:
            launch(L, x, a, out, name)
            reduce_if_rowpar(name, out)
    torch.cuda.synchronize()

    def capture(step_range, ev_base, events):
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                e = ev_base
                for st in step_range:
                    for (_, name, M, L, x, a, out) in per_copy[order[st]]:
                        if events:
                            ge.record(evs[e])
                        launch(L, x, a, out, name)
                        if events:
                            ge.record(evs[e + 1])
                        e += 2
                        reduce_if_rowpar(name, out)
        torch.cuda.current_stream().wait_stream(s)
        return g

    # the headline graph has no event nodes between launches; a second graph
    # of the same steps with an event pair around every launch gives the
    # kernel-only durations for the roofline
    g_warm = capture(range(0, args.warmup), 0, False)
    g_time = capture(range(args.warmup, steps_total), 0, False)
    g_kern = capture(range(args.warmup, steps_total), 2 * 16 * args.warmup, True)
    g_warm.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    align = torch.zeros(1, device=dev)
    with ClockSampler(local) as clk:
        if world > 1:
            # start every rank's timed region together: a spin kernel keeps the
            # stream busy while the host enqueues, then a one-element all-reduce
            # completes at nearly the same moment on every rank, before t0
            torch.cuda._sleep(4_000_000)
            dist.all_reduce(align)
        t0.record()
        g_time.replay()
        t1.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    elapsed_ms = t0.elapsed_time(t1)
    g_kern.replay()
    torch.cuda.synchronize()
    kern_ms = 0.0
    kern_bytes = 0
    per_cfg = {}
    e = 2 * 16 * args.warmup
    for st in range(args.warmup, steps_total):
        for (_, name, M, L, x, _a, out) in per_copy[order[st]]:
            d = evs[e].elapsed_time(evs[e + 1])  # kernel-only time of this launch
            b = L.algorithmic_bytes(M)
            kern_ms += d
            kern_bytes += b
            acc = per_cfg.setdefault(f"{name}/M{M}", [0.0, 0])
            acc[0] += d
            acc[1] += b
            e += 2
    step_bytes_rank = sum(cl[3].algorithmic_bytes(cl[2]) for cl in per_copy[0])
    step_bytes_job = sum(full_layer_bytes(M) for M in MS) if world > 1 else step_bytes_rank
    t = torch.tensor([elapsed_ms, kern_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms, kern_ms_max = float(t[0]), float(t[1])
    value = step_bytes_job * args.steps / (elapsed_ms * 1e-3) / 1e9

    # ---- e2e: public op, host activations in, outputs out, every step
    import qwen_wlqfastshot_helen_beta_b200  # noqa: F401  (torch ops)
    # a step's activations (x and h of every launch) sit in one pinned host
    # buffer and go over in one copy; the outputs land in one device buffer
    # and come back in one copy, the way a serving stack stages a batch
    def arena(tensors):
        offs, n = [], 0
        for t in tensors:
            offs.append(n)
            n += (t.numel() * t.element_size() + 255) // 256 * 256
        return offs, n

    ins = [x for (_, _, _, _, x, _, _) in per_copy[0]]
    outs = [out for (*_r, out) in per_copy[0]]
    in_offs, in_n = arena(ins)
    out_offs, out_n = arena(outs)
    in_host = torch.empty(in_n, dtype=torch.uint8).pin_memory()
    in_dev = torch.empty(in_n, dtype=torch.uint8, device=dev)
    out_host = torch.empty(out_n, dtype=torch.uint8).pin_memory()
    out_dev = torch.empty(out_n, dtype=torch.uint8, device=dev)

    def view(buf, off, t):
        return buf[off:off + t.numel() * t.element_size()].view(t.dtype).view(t.shape)

    for t, o in zip(ins, in_offs):
        view(in_host, o, t).copy_(t.cpu())
    host = []
    for i, (c, name, M, L, x, a, out) in enumerate(per_copy[0]):
        host.append((name, L, view(in_dev, in_offs[i], x), a, view(out_dev, out_offs[i], out)))
    h2d = sum(t.numel() * t.element_size() for t in ins)
    d2h = sum(t.numel() * t.element_size() for t in outs)

    def e2e_enqueue():
        in_dev.copy_(in_host, non_blocking=True)
        for (name, L, xd, a, od) in host:
            if comm is not None and name in ("o", "down"):
                _C.gemv_allreduce(comm, xd, L.q_packed, L.lut_packed, od, L.N, L.K, 4, L.words_per_row,
                                  L.chunk_offsets, L.cols_packed, L.delta_packed, None, L.lora_B, L.dora_gamma,
                                  L.lora_scale, L.group_size, L.group_offset, 1, lora_A=a)
            else:
                torch.ops.wlq_fastShot.gemm(xd, L.q_packed, L.lut_packed, od, L.N, L.K, 4, L.words_per_row,
                                            L.chunk_offsets, L.cols_packed, L.delta_packed, None, L.lora_B,
                                            L.dora_gamma, L.lora_scale, L.group_size, L.group_offset, 1, a)
            reduce_if_rowpar(name, od)
        out_host.copy_(out_dev, non_blocking=True)

    def e2e_step():
        e2e_enqueue()
        torch.cuda.current_stream().synchronize()

    # the graphed step overlaps the read-back: the step's activations go over
    # in one copy, and every call's output comes back on a copy stream as
    # soon as it is written, while the step's later calls run (the 16 calls
    # of a step are independent; the host still waits for the whole step's
    # outputs).  Per-call input copies were measured too: their events add a
    # plain dependency to every launch, which cost the GEMV launch overlap
    # (-8 % at 2 GPUs).
    s_d2h = torch.cuda.Stream()
    out_slices = [(view(out_host, o, t), view(out_dev, o, t)) for t, o in zip(outs, out_offs)]

    def e2e_enqueue_pipelined():
        main = torch.cuda.current_stream()
        s_d2h.wait_stream(main)
        in_dev.copy_(in_host, non_blocking=True)
        for i, (name, L, xd, a, od) in enumerate(host):
            if comm is not None and name in ("o", "down"):
                _C.gemv_allreduce(comm, xd, L.q_packed, L.lut_packed, od, L.N, L.K, 4, L.words_per_row,
                                  L.chunk_offsets, L.cols_packed, L.delta_packed, None, L.lora_B, L.dora_gamma,
                                  L.lora_scale, L.group_size, L.group_offset, 1, lora_A=a)
            else:
                torch.ops.wlq_fastShot.gemm(xd, L.q_packed, L.lut_packed, od, L.N, L.K, 4, L.words_per_row,
                                            L.chunk_offsets, L.cols_packed, L.delta_packed, None, L.lora_B,
                                            L.dora_gamma, L.lora_scale, L.group_size, L.group_offset, 1, a)
            reduce_if_rowpar(name, od)
            done = torch.cuda.Event()
            done.record(main)
            s_d2h.wait_event(done)
            with torch.cuda.stream(s_d2h):
                out_slices[i][0].copy_(out_slices[i][1], non_blocking=True)
        main.wait_stream(s_d2h)

    def timed_e2e(step_fn):
        for _ in range(args.warmup):
            step_fn()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            step_fn()
        e1.record()
        torch.cuda.synchronize()
        te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        return float(te[0])

    # eager: one op call per (linear, M), the host waiting for each step's outputs
    eager_ms = timed_e2e(e2e_step)
    # graph: the same step (host->device copies, ops, device->host copies)
    # captured once and replayed, as vLLM runs decode; the host still waits
    # for every step's outputs
    g_e2e = torch.cuda.CUDAGraph()
    s_e2e = torch.cuda.Stream()
    s_e2e.wait_stream(torch.cuda.current_stream())
    enqueue = e2e_enqueue_pipelined if args.e2e_copies == "pipelined" else e2e_enqueue
    with torch.cuda.stream(s_e2e):
        enqueue()
        with torch.cuda.graph(g_e2e, stream=s_e2e):
            enqueue()
    torch.cuda.current_stream().wait_stream(s_e2e)
    torch.cuda.synchronize()

    def graph_step():
        g_e2e.replay()
        torch.cuda.current_stream().synchronize()

    e2e_ms = timed_e2e(graph_step)
    e2e_value = step_bytes_job * args.steps / (e2e_ms * 1e-3) / 1e9
    eager_value = step_bytes_job * args.steps / (eager_ms * 1e-3) / 1e9

    gemm = gemm_leg(layers, dev, launch_gemm, peaks, peaks_kind, local, world, rank)
    tp_detail = tp_allreduce_leg(per_copy[0], comm, launch, dev, world) if world > 1 else None
    config0 = ref_gpu = None
    if world == 1 and not args.no_baselines:
        config0 = cpu_baseline_config0(dev, args.cpu_budget)
        ref_gpu = reference_gpu_baseline(dev, peaks)

    result = None
    if rank == 0:
        # the dominant kernel's achieved bandwidth, from the headline graph
        # (its launches back to back, no event nodes): algorithmic bytes of
        # this rank's launches / this rank's share of the timed region
        achieved = step_bytes_rank * args.steps / (elapsed_ms * 1e-3) / 1e9
        peak = float(peaks["hbm_gbs"])
        traffic = None
        tp = os.path.join(ROOT, "profiles", "gemv_traffic.json")
        if os.path.exists(tp):
            with open(tp) as f:
                traffic = json.load(f).get("bytes_per_step")
        result = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(elapsed_ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded; BASELINE config-1 recipe)",
            "config": bench_config(world, copies),
            "roofline": {
                "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic,
                "peak_source": f"{peaks_kind} hbm_gbs (MEASURED_PEAKS.json)" if peaks_kind == "measured"
                else "fallback 6650 GB/s",
                "kernel": "gemv_kernel with h = A x in the kernel (wlq_gemv_kernel.cuh), all 16 (linear, M) "
                          "launches of a step",
                "timing": "headline graph (the step's launches back to back); achieved = this GPU's algorithmic "
                          "bytes per step / ms_per_step, so kernel time per step <= ms_per_step",
                "per_config_gbs": {k: round(v[1] / (v[0] * 1e-3) / 1e9, 1) for k, v in per_cfg.items()},
                "per_config_timing": "a second graph of the same steps with an event pair around every launch "
                                     "(event nodes serialise and add time: a lower bound per launch)",
                "event_graph_gbs": round(kern_bytes / (kern_ms * 1e-3) / 1e9, 1),
            },
            "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "path": "torch.ops.wlq_fastShot.gemm(..., lora_A) on every (linear, M) of a step (h = A x "
"inside the GEMV); every step the step's activations copied in from one pinned host buffer, "
                            "and every call's output read back into pinned host memory on a copy stream as soon as it "
                            "is written (overlapping the step's later calls; no copy crosses a step boundary); the "
                            "step replayed as one CUDA graph (as vLLM runs decode), host synchronised per step; "
                            "eager_value: one copy in, the calls, one copy out, no overlap",
                    "eager_value": round(eager_value, 1)},
            "gpu_launches": 16 * args.steps,
            "clocks": clk.summary(),
        }
        if gemm is not None:
            result["gemm"] = gemm
        if tp_detail is not None:
            result["tp_allreduce"] = tp_detail
        if config0 is not None:
            result["cpu_baseline_config0"] = config0
        if ref_gpu is not None:
            result["reference_gpu_baseline"] = ref_gpu
    if world > 1:
        del g_warm, g_time, g_kern, g_e2e
        torch.cuda.synchronize()
        dist.barrier()
        if comm is not None:
            err = comm.error()
            comm.close()
            if err and rank == 0:
                raise RuntimeError("fused all-reduce: a rank timed out waiting for another")
        dist.destroy_process_group()
    return result, layers if rank == 0 else None


def tp_allreduce_leg(calls, comm, launch, dev, world, reps=20):
    """Per-call time of the row-parallel decode layers (o, down) at M = 1 and
    16 on this rank's K shard: the GEMV alone, the GEMV followed by vLLM's
    NCCL all-reduce of [M, N], and the GEMV with the all-reduce fused
    (wlq_gemv_allreduce); graphs of `reps` calls, max over ranks."""
    import torch
    import torch.distributed as dist
    out = {}
    for (_, name, M, L, x, a, y) in calls:
        if name not in ("o", "down") or M not in (1, 16):
            continue
        variants = {"gemv_alone": lambda: launch(L, x, a, y),
                    "gemv_then_nccl": lambda: (launch(L, x, a, y), dist.all_reduce(y)),
                    "fused": lambda: launch(L, x, a, y, name)}
        row = {}
        for key, fn in variants.items():
            fn()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    for _ in range(reps):
                        fn()
            torch.cuda.current_stream().wait_stream(s)
            g.replay()
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            t = torch.tensor([e0.elapsed_time(e1) / reps * 1e3], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            row[key + "_us"] = round(float(t[0]), 2)
            del g
        out[f"{name}/M{M}"] = row
    return {"unit": "us per call, max over ranks", "shard": f"K / {world} per rank", "per_config": out}


def gemm_leg(layers, dev, launch, peaks, peaks_kind, local, world=1, rank=0, reps=10, warmup=3):
    """the prefill op (H = X A^T on wlq_lora_h, then the
    tcgen05 GEMM of wlq_gemm.cu) on the four linears at M in GEMM_MS, each
    (linear, M) a CUDA graph of `reps` calls timed with events; TFLOPS =
    2 M N K / time.  With world > 1 each rank runs its tensor-parallel shard
    (qkv / gate_up by rows, o / down by K) and the row-parallel layers end
    with an NCCL all-reduce of [M, N] inside the graph, as vLLM runs them;
    times are the max over ranks, TFLOPS count the unsharded layer."""
    import torch
    import torch.distributed as dist
    gen = torch.Generator(device=dev)
    gen.manual_seed(77)
    cfgs = []
    for name, K, N in SHAPES:
        L = layers[0][name]
        for M in GEMM_MS:
            x = torch.randn((M, L.K), generator=gen, device=dev).to(torch.bfloat16)
            H = torch.empty((M, L.r), dtype=torch.float32, device=dev)
            cfgs.append((name, M, K, N, L, x, H, torch.empty((M, L.N), dtype=torch.bfloat16, device=dev)))
    rowpar = lambda name: world > 1 and name in ("o", "down")  # noqa: E731
    for _ in range(warmup):
        for (name, M, K, N, L, x, H, out) in cfgs:
            launch(L, x, H, out)
            if rowpar(name):
                dist.all_reduce(out)
    torch.cuda.synchronize()

    def graph_of(L, x, H, out, with_ar):
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for _ in range(reps):
                    launch(L, x, H, out)
                    if with_ar:
                        dist.all_reduce(out)
        torch.cuda.current_stream().wait_stream(s)
        return g

    graphs = [graph_of(L, x, H, out, rowpar(name)) for (name, M, K, N, L, x, H, out) in cfgs]
    kgraphs = [graph_of(L, x, H, out, False) if rowpar(name) else None for (name, M, K, N, L, x, H, out) in cfgs]

    def timed(g):
        g.replay()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / reps], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0])

    per, ar_share, tot_ms, tot_flops = {}, {}, 0.0, 0.0
    with ClockSampler(local) as clk:
        for cfg, g, kg in zip(cfgs, graphs, kgraphs):
            name, M, K, N = cfg[:4]
            ms = timed(g)
            fl = 2.0 * M * N * K  # the unsharded layer
            per[f"{name}/M{M}"] = round(fl / (ms * 1e-3) / 1e12, 1)
            if kg is not None:
                ar_share[f"{name}/M{M}"] = round(max(0.0, 1.0 - timed(kg) / ms), 3)
            tot_ms += ms
            tot_flops += fl
    tflops = tot_flops / (tot_ms * 1e-3) / 1e12
    peak = float(peaks.get("bf16_tflops", 1590.0))
    del graphs, kgraphs
    out = {
        "metric": "GEMM TFLOPS (2*M*N*K / time of the prefill op: wlq_lora_h + wlq_gemm_streamk)",
        "value": round(tflops, 1), "unit": "TFLOP/s",
        "config": "BASELINE config 2: qkv/o/gate_up/down at M in {512, 2048, 8192}, bf16, group 128, "
                  "rank 16, 0.5% outliers; weights L2-resident across M tiles as in a real prefill",
        "ms_all_configs": round(tot_ms, 3),
        "per_config_tflops": per,
        "roofline": {"bound": "tensor", "achieved": round(tflops / world, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(tflops / world / peak, 4),
                     "peak_source": f"{peaks_kind} bf16_tflops (cuBLAS burst, MEASURED_PEAKS.json)"
                     if peaks_kind == "measured" else "fallback 1590 TFLOP/s",
                     "kernel": "gemm_kernel (wlq_gemm.cu), with lora_h_kernel (wlq_lora_h.cu) in the timed op"},
        "gpu_launches": 2 * reps * len(cfgs),
        "clocks": clk.summary(),
    }
    if world > 1:
        out["parallelism"] = (f"tp{world}: qkv/gate_up split by output rows, o/down by K with an NCCL all-reduce "
                              f"of [M, N] bf16 after the GEMM (in the timed graph); time = max over ranks")
        out["tflops_per_gpu"] = round(tflops / world, 1)
        out["allreduce_share"] = ar_share
    return out


def cpu_baseline_config0(dev, budget_s=15.0, reps=50):
    """BASELINE config 0 (K=4864 -> N=896, M=8, fp32 activations, group-128
    recipe): ms per call of this package's op the way WLQLinearMethod.apply
    runs it (x cast to fp16, h = A x inside the GEMV, output cast back to
    fp32), device-resident and end to end from pinned host memory, beside the
    reference's CPU dequantize-then-matmul steps (oracle/cpu_baseline.py) on
    the box's host cores, all threads and one thread; parity = normwise max
    relative error between the two outputs on the same inputs.  The layer is
    made with numpy (oracle/synthetic_np.py) so both sides read the same
    bytes."""
    import torch
    import qwen_wlqfastshot_helen_beta_b200  # noqa: F401  (torch ops)
    from qwen_wlqfastshot_helen_beta_b200 import _C
    from oracle import synthetic_np as SN
    N0, K0, M0 = 896, 4864, 8
    L = SN.make_layer(N0, K0, group_size=GROUP, density=DENSITY, r=RANK, seed=2024)
    d = dev
    q = torch.from_numpy(L.q_packed).to(d)
    lut = torch.from_numpy(L.lut_c).to(d)
    off = torch.from_numpy(L.chunk_offsets).to(d)
    cols16 = torch.from_numpy(L.chunk_cols).to(d)
    vals8 = torch.from_numpy(L.chunk_vals).to(d)
    lutp = _C.prepack_lut(lut, torch.float16)
    colsp, deltap = _C.prepack_outliers(q, lut, off, cols16, vals8, N0, K0, 4, torch.float16, GROUP, 0)
    A = torch.from_numpy(L.lora_A).to(d)
    B = torch.from_numpy(L.lora_B).to(d)
    gam = torch.from_numpy(L.dora_gamma).to(d)
    torch.cuda.synchronize()  # weights complete before any (overlapping) GEMV reads them
    rng = np.random.default_rng(4)
    x_np = rng.standard_normal((M0, K0)).astype(np.float32)
    x_host = torch.from_numpy(x_np).pin_memory()
    y_host = torch.empty((M0, N0), dtype=torch.float32).pin_memory()
    x_dev = x_host.to(d)
    out16 = torch.empty((M0, N0), dtype=torch.float16, device=d)

    def op(xd):
        x16 = xd.to(torch.float16)
        torch.ops.wlq_fastShot.gemm(x16, q, lutp, out16, N0, K0, 4, L.words_per_row, off, colsp, deltap, None, B,
                                    gam, L.lora_scale, GROUP, 0, 1, A)
        return out16.float()

    for _ in range(5):
        op(x_dev)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        op(x_dev)
    e1.record()
    torch.cuda.synchronize()
    dev_ms = e0.elapsed_time(e1) / reps

    def e2e_call():
        y_host.copy_(op(x_host.to(d, non_blocking=True)), non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for _ in range(5):
        e2e_call()
    e0.record()
    for _ in range(reps):
        e2e_call()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / reps
    y_gpu = y_host.numpy().copy()

    # the reference's CPU steps on the same layer and activations
    def cpu_ms(threads):
        torch.set_num_threads(threads)
        xt = torch.from_numpy(x_np)
        times, y = [], None
        t_start = time.perf_counter()
        for i in range(200):
            dt, _, y = _cpu_call(L, M0, None, xt)
            if i >= 3:
                times.append(dt)
            if i >= 23 and time.perf_counter() - t_start > budget_s / 2:
                break
        return statistics.median(times) * 1e3, len(times), y

    cores = os.cpu_count() or 1
    cpu_all_ms, n_all, y_cpu = cpu_ms(cores)
    cpu_one_ms, n_one, _ = cpu_ms(1)
    torch.set_num_threads(cores)
    y_cpu = y_cpu.numpy()
    err = float(np.max(np.abs(y_gpu - y_cpu)) / max(1e-30, float(np.max(np.abs(y_cpu)))))
    try:
        cpu_model = next(l.split(":", 1)[1].strip() for l in open("/proc/cpuinfo") if l.startswith("model name"))
    except Exception:
        cpu_model = "unknown"
    return {
        "workload": "BASELINE config 0: one 4864 -> 896 layer (Qwen2.5-0.5B down_proj shape), M=8 fp32 "
                    "activations ~N(0,1), group-128 codebooks, DoRA rank 16, 0.5% outliers",
        "ours_ms_per_call": round(dev_ms, 4),
        "ours_e2e_ms_per_call": round(e2e_ms, 4),
        "ours_path": "x cast to fp16, torch.ops.wlq_fastShot.gemm(..., lora_A) (h = A x inside the GEMV), output "
                     "cast to fp32, as WLQLinearMethod.apply runs it; e2e adds the pinned host->device copy of x "
                     "and the device->host copy of y, host synchronised per call",
        "reference_cpu_ms_per_call": round(cpu_all_ms, 3),
        "reference_cpu_ms_per_call_1thread": round(cpu_one_ms, 3),
        "cores": cores, "cpu_model": cpu_model,
        "reference_cpu_path": "oracle/cpu_baseline.py: unpack -> gather -> outlier overwrite -> fp32 matmul -> "
                              "DoRA epilogue (the reference's torch steps), h = F.linear(x, A) in fp32; median of "
                              f"{n_all} (all threads) / {n_one} (1 thread) calls after 3 warm-up calls",
        "speedup_e2e_vs_cpu": round(cpu_all_ms / e2e_ms, 1),
        "max_rel_err_vs_cpu": err,
        "tolerance": 5e-3,
    }


def reference_gpu_baseline(dev, peaks, reps=20):
    """The reference's own CUDA kernels (compiled from its sources for
    sm_100a into oracle/_ref by oracle/build_ref.sh) timed on this GPU beside
    this package's path, on per-row codebooks (the only layout the
    reference's kernels read), fp16 activations, config-1 and config-2 shapes.
    Reference composition per call, as vllm_wlq/linear_method.py:937-1009 and
    csrc/vllm_binding.cpp:253-419 run it: F.linear(x, A).float(), then
    launch_gemv_chunk_csr (M = 1), launch_gemm_metalog_dora (2 <= M <= 15) or
    launch_dequant_patch_metalog + torch.mm + launch_fused_dora_epilogue
    (M >= 16).  Ours: torch.ops.wlq_fastShot.gemm(..., lora_A) on the
    prepacked layer (one GEMV launch for M <= 16; wlq_lora_h + the tcgen05
    GEMM above).  Each (linear, M) is a CUDA graph of `reps` calls over two
    weight copies; a baseline leg, not part of the product path."""
    import torch
    path = os.path.join(ROOT, "oracle", "_ref", "libwlq_ref_kernels.so")
    if not os.path.exists(path):
        return {"unavailable": "oracle/_ref/libwlq_ref_kernels.so not built (needs the reference tree at build time)"}
    import qwen_wlqfastshot_helen_beta_b200  # noqa: F401  (torch ops)
    from qwen_wlqfastshot_helen_beta_b200 import synthetic as S
    ref = ctypes.CDLL(path)
    ci, cf = ctypes.c_int, ctypes.c_float
    vp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    copies = []
    for c in range(2):
        row = {}
        for si, (name, K, N) in enumerate(SHAPES):
            L = S.make_layer(N, K, group_size=0, density=DENSITY, r=RANK, seed=5000 + 31 * c + si, device=dev)
            row[name] = L.prepack(torch.float16)
        copies.append(row)
    torch.cuda.synchronize()
    gen = torch.Generator(device=dev)
    gen.manual_seed(99)
    ws = torch.zeros(32 * max(N for _, _, N in SHAPES), dtype=torch.float32, device=dev)
    Wd = torch.empty(max(N * K for _, K, N in SHAPES), dtype=torch.float16, device=dev)

    def ref_call(L, x, out):
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        M, N, K = x.shape[0], L.N, L.K
        nc = (K + 511) // 512
        h = torch.nn.functional.linear(x, L.lora_A).float()
        if M == 1:
            ref.launch_gemv_chunk_csr(vp(L.q_packed), vp(L.lut_c), vp(x), vp(out), vp(ws), vp(L.chunk_offsets),
                                      vp(L.chunk_cols), vp(L.chunk_vals), vp(L.lora_B), vp(h), vp(L.dora_gamma),
                                      cf(L.lora_scale), ci(L.r), ci(N), ci(K), ci(4), ci(nc), st)
        elif M < 16:
            ref.launch_gemm_metalog_dora(vp(x), vp(L.q_packed), vp(L.lut_c), vp(out), vp(L.chunk_offsets),
                                         vp(L.chunk_cols), vp(L.chunk_vals), vp(h), vp(L.lora_B), vp(L.dora_gamma),
                                         cf(L.lora_scale), ci(L.r), ci(M), ci(N), ci(K), ci(4), ci(L.words_per_row),
                                         ci(nc), ci(512), st)
        else:
            W = Wd[:N * K].view(N, K)
            ref.launch_dequant_patch_metalog(vp(L.q_packed), vp(L.lut_c), vp(W), vp(L.chunk_offsets),
                                             vp(L.chunk_cols), vp(L.chunk_vals), ci(N), ci(K), ci(4),
                                             ci(L.words_per_row), ci(nc), ci(512), st)
            torch.mm(x, W.t(), out=out)
            ref.launch_fused_dora_epilogue(vp(out), vp(h), vp(L.lora_B), vp(L.dora_gamma), cf(L.lora_scale),
                                           ci(L.r), ci(M), ci(N), st)

    def our_call(L, x, out):
        torch.ops.wlq_fastShot.gemm(x, L.q_packed, L.lut_packed, out, L.N, L.K, 4, L.words_per_row,
                                    L.chunk_offsets, L.cols_packed, L.delta_packed, None, L.lora_B, L.dora_gamma,
                                    L.lora_scale, 0, 0, 1, L.lora_A_act)

    def time_graph(fn, name, x, out):
        for c in range(2):
            fn(copies[c][name], x, out)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for i in range(reps):
                    fn(copies[i % 2][name], x, out)
        torch.cuda.current_stream().wait_stream(s)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) / reps

    gemv, gemm = {}, {}
    sums = {"gemv": [0.0, 0.0, 0.0], "gemm": [0.0, 0.0, 0.0]}  # ref ms, our ms, bytes or flops
    for name, K, N in SHAPES:
        for M in MS + GEMM_MS:
            x = torch.randn((M, K), generator=gen, device=dev).to(torch.float16)
            out_r = torch.empty((M, N), dtype=torch.float16, device=dev)
            out_o = torch.empty((M, N), dtype=torch.float16, device=dev)
            t_ref = time_graph(ref_call, name, x, out_r)
            t_our = time_graph(our_call, name, x, out_o)
            err = ((out_o.float() - out_r.float()).abs().max() / out_r.float().abs().max()).item()
            key = f"{name}/M{M}"
            if M <= 16:
                b = copies[0][name].algorithmic_bytes(M)
                gemv[key] = {"ref_us": round(t_ref * 1e3, 2), "ours_us": round(t_our * 1e3, 2),
                             "ref_gbs": round(b / (t_ref * 1e-3) / 1e9, 1), "ours_gbs": round(b / (t_our * 1e-3) / 1e9, 1),
                             "speedup": round(t_ref / t_our, 2), "max_rel_diff": round(err, 5)}
                acc = sums["gemv"]
                acc[2] += b
            else:
                fl = 2.0 * M * N * K
                gemm[key] = {"ref_us": round(t_ref * 1e3, 1), "ours_us": round(t_our * 1e3, 1),
                             "ref_tflops": round(fl / (t_ref * 1e-3) / 1e12, 1),
                             "ours_tflops": round(fl / (t_our * 1e-3) / 1e12, 1),
                             "speedup": round(t_ref / t_our, 2), "max_rel_diff": round(err, 5)}
                acc = sums["gemm"]
                acc[2] += fl
            acc[0] += t_ref
            acc[1] += t_our
            del x, out_r, out_o
    g_, m_ = sums["gemv"], sums["gemm"]
    return {
        "layout": "per-row fp16 codebooks (the reference's), rank 16, 0.5% outliers, fp16 activations, "
                  "2 rotating weight copies",
        "reference_kernels": "oracle/_ref/libwlq_ref_kernels.so (the reference's csrc/gemv_kernel.cu and "
                             "csrc/gemm_kernel.cu built for sm_100a) + torch.mm (cuBLAS) + F.linear for h",
        "gemv_vs_ref_gpu": round(g_[0] / g_[1], 2),
        "gemv_ref_gbs": round(g_[2] / (g_[0] * 1e-3) / 1e9, 1),
        "gemv_ours_gbs": round(g_[2] / (g_[1] * 1e-3) / 1e9, 1),
        "gemm_vs_ref_gpu": round(m_[0] / m_[1], 2),
        "gemm_ref_tflops": round(m_[2] / (m_[0] * 1e-3) / 1e12, 1),
        "gemm_ours_tflops": round(m_[2] / (m_[1] * 1e-3) / 1e12, 1),
        "per_config_gemv": gemv,
        "per_config_gemm": gemm,
    }


# ---------------------------------------------------------- CPU baseline

def _cpu_sample_layers(seed=5, rows=512):
    """Row blocks (<= ``rows`` rows, full K) of each linear, generated with
    numpy alone (oracle/synthetic_np.py): the CPU legs load no library of
    this repository."""
    from oracle import synthetic_np as SN
    out = []
    for si, (name, K, N) in enumerate(SHAPES):
        n = min(N, rows)
        out.append((name, K, N, n, SN.make_layer(n, K, group_size=GROUP, density=DENSITY, r=RANK, seed=seed + si)))
    return out


def _cpu_operands(L):
    """The layer's tensors as the reference's CPU steps take them (cached)."""
    import torch
    ops = getattr(L, "_cpu_ops", None)
    if ops is None:
        ops = (L.q_packed, torch.from_numpy(L.lut_c), L.chunk_offsets,
               None if L.chunk_cols is None else L.chunk_cols.astype(np.int64), L.chunk_vals,
               torch.from_numpy(L.lora_A).float(), torch.from_numpy(L.lora_B), torch.from_numpy(L.dora_gamma))
        L._cpu_ops = ops
    return ops


def _cpu_call(L, M, gen, x=None):
    """One forward through the reference's CPU steps: h = A x (the
    reference's F.linear, vllm_wlq/linear_method.py:962-963), then
    oracle/cpu_baseline.py.  Returns (seconds, algorithmic bytes, y)."""
    import torch
    from oracle.cpu_baseline import cpu_forward
    q, lut, off, cols, vals, A, B, gam = _cpu_operands(L)
    if x is None:
        x = torch.randn((M, L.K), generator=gen).to(torch.bfloat16)
    t = time.perf_counter()
    h = torch.nn.functional.linear(x.float(), A)
    y = cpu_forward(q, L.words_per_row, lut, L.N, L.K, L.group_size, L.group_offset, off, cols, vals, x.float(), h,
                    B, gam, L.lora_scale)
    return time.perf_counter() - t, L.algorithmic_bytes(M), y


def cpu_baseline(budget_s=15.0):
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    gen = torch.Generator()
    gen.manual_seed(7)
    layers = _cpu_sample_layers()
    tot_t = tot_b = 0.0
    n = 0
    t_start = time.perf_counter()
    _cpu_call(layers[0][4], 1, gen)  # warm-up
    while True:
        for (name, K, N, rows, L) in layers:
            for M in MS:
                dt, b, _ = _cpu_call(L, M, gen)
                tot_t += dt
                tot_b += b
                n += 1
        if time.perf_counter() - t_start > budget_s:
            break
    return {"value": round(tot_b / tot_t / 1e9, 3), "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{n} calls: 512-row blocks (full K) of each of the 4 linears at M in {{1,4,8,16}}, "
                      f"the reference's torch dequantize-then-matmul steps (oracle/cpu_baseline.py) on layers "
                      f"made with numpy (oracle/synthetic_np.py), {tot_t:.1f} s of CPU time"}


def run_reference(args):
    import torch
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    torch.set_num_threads(os.cpu_count() or 1)
    gen = torch.Generator()
    gen.manual_seed(11)
    layers = _cpu_sample_layers()
    cfgs = [(L, M) for (_, _, _, _, L) in layers for M in MS]
    for s in range(args.warmup):
        _cpu_call(*cfgs[s % len(cfgs)], gen)
    tot_t = tot_b = 0.0
    for s in range(args.steps):
        dt, b, _ = _cpu_call(*cfgs[s % len(cfgs)], gen)
        tot_t += dt
        tot_b += b
    value = tot_b / tot_t / 1e9
    cores = torch.get_num_threads()
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(tot_t * 1e3 / args.steps, 3), "higher_is_better": True,
        "scaling": "strong" if int(os.environ.get("WORLD_SIZE", "1")) > 1 else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; BASELINE config-1 recipe)",
        "config": bench_config(int(os.environ.get("WORLD_SIZE", "1")), args.copies),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": "each step: one 512-row block (full K) of one linear at one M, cycling over "
                                   "the 4 linears x M in {1,4,8,16}; the reference's torch dequantize-then-"
                                   "matmul steps (oracle/cpu_baseline.py) on layers made with numpy "
                                   "(oracle/synthetic_np.py); no library of this repository is loaded"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_case(args):
    """One (linear, M) configuration, eager launches over `copies` rotating
    weight copies: the small command the ncu captures profile."""
    import torch
    from qwen_wlqfastshot_helen_beta_b200 import synthetic as S
    parts = args.case.split(":")
    name, M = parts[-2], int(parts[-1])  # "name:M" or "gemm:name:M"
    K, N = {n: (k, nn) for n, k, nn in SHAPES}[name]
    torch.cuda.set_device(0)
    layers = [S.make_layer(N, K, group_size=GROUP, density=DENSITY, r=RANK, seed=300 + c).prepack(torch.bfloat16)
              for c in range(args.copies)]
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    x = torch.randn((M, K), generator=gen, device="cuda").to(torch.bfloat16)
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    import qwen_wlqfastshot_helen_beta_b200  # noqa: F401  (torch ops)

    def call(i):  # the op as apply() runs it: decode folds h = A x, prefill runs wlq_lora_h + the GEMM
        L = layers[i % len(layers)]
        if M <= 16:
            S.forward_fold(L, x, out)
        else:
            torch.ops.wlq_fastShot.gemm(x, L.q_packed, L.lut_packed, out, N, K, 4, L.words_per_row, L.chunk_offsets,
                                        L.cols_packed, L.delta_packed, None, L.lora_B, L.dora_gamma, L.lora_scale,
                                        GROUP, 0, 1, L.lora_A_act)

    for i in range(args.warmup):
        call(i)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.steps):
        call(i)
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / args.steps
    b = layers[0].algorithmic_bytes(M)
    print(json.dumps({"case": args.case, "ms_per_call": round(ms, 5), "bytes": b, "GB/s": round(b / ms / 1e6, 1),
                      "TFLOP/s": round(2.0 * M * N * K / ms / 1e9, 1)}))


def _load_by_path(name, rel):
    """A module of this repository loaded from its file, without importing
    its package (whose import loads libwlq_b200.so)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, rel))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def run_vllm_decode(args):
    """BASELINE config 3 inside vLLM, one plugin per process: a random-init
    Qwen2.5-7B-shaped model in the reference's on-disk format (per-row
    codebooks, the only layout the reference reads; DoRA rank 16 per
    projection, 0.5% outliers), batch 32 x (1024 prompt + 256 generated)
    tokens, decode as full CUDA graphs.  --vllm-decode ours: this package's
    quantisation method; reference: the unmodified reference plugin installed
    in baseline/_ref (its kernels JIT-compiled from compute_90 PTX), with this
    package never imported.  Prints one JSON line."""
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    ck = _load_by_path("_wlq_checkpoint", "qwen_wlqfastshot_helen_beta_b200/checkpoint.py")
    model = args.model
    if not os.path.isfile(os.path.join(model, "config.json")):
        t0 = time.time()
        ck.write_checkpoint(model, num_layers=args.layers, group_size=0, seed=0)
        print(f"checkpoint written in {time.time() - t0:.0f} s", file=sys.stderr, flush=True)
    if args.vllm_decode == "reference":
        ref = os.path.join(ROOT, "baseline", "_ref")
        if not os.path.isdir(os.path.join(ref, "vllm_wlq")):
            print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref/vllm_wlq is not installed"}))
            return
        sys.path.insert(0, ref)
        import vllm_wlq
        vllm_wlq.register()
    else:
        from qwen_wlqfastshot_helen_beta_b200 import register
        register()
    from vllm import LLM, SamplingParams
    batch, prompt, gen = 32, 1024, 256
    llm = LLM(model=model, dtype="bfloat16", skip_tokenizer_init=True, seed=0, max_model_len=prompt + gen + 16,
              max_num_seqs=batch, gpu_memory_utilization=0.80, enable_prefix_caching=False,
              compilation_config={"mode": 0, "cudagraph_mode": "FULL_DECODE_ONLY"})
    with open(os.path.join(model, "config.json")) as f:
        vocab = json.load(f)["vocab_size"]
    rng = np.random.default_rng(0)
    prompts = [{"prompt_token_ids": rng.integers(0, vocab, size=prompt).tolist()} for _ in range(batch)]

    def run(n):
        sp = SamplingParams(max_tokens=n, min_tokens=n, ignore_eos=True, temperature=0.0, detokenize=False)
        t = time.perf_counter()
        outs = llm.generate(prompts, sp, use_tqdm=False)
        return time.perf_counter() - t, sum(len(o.outputs[0].token_ids) for o in outs), outs

    run(4)  # warm-up
    t1, _, _ = run(1)
    tg, ntok, outs = run(gen)
    first = [list(o.outputs[0].token_ids[:8]) for o in outs[:2]]
    print(json.dumps({
        "impl": args.vllm_decode, "metric": "Qwen2.5-7B decode tok/s (vLLM, every linear WLQ)",
        "value": round(ntok / tg, 1), "unit": "tok/s", "decode_tok_s": round(batch * (gen - 1) / max(tg - t1, 1e-9), 1),
        "prefill_s": round(t1, 3), "generate_s": round(tg, 3), "tokens": ntok, "first_tokens": first,
        "config": {"model": "random-init Qwen2.5-7B shape, per-row codebooks, rank 16, 0.5% outliers",
                   "layers": args.layers or 28, "batch": batch, "prompt": prompt, "gen": gen, "dtype": "bf16",
                   "parallelism": "single", "cudagraph_mode": "FULL_DECODE_ONLY", "compile": "off"},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--e2e-copies", choices=("pipelined", "single"), default="pipelined",
                    help="e2e graph: one copy in, then every call's output read back on a copy stream while the "
                         "step's later calls run (default), or one copy in and one out around the calls")
    ap.add_argument("--case", default=None, help="name:M (M <= 16: GEMV; larger: GEMM), one configuration for "
                    "profiling; a gemm: prefix is accepted")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--copies", type=int, default=3)
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-baselines", action="store_true", help="skip the config-0 CPU leg and the reference's GPU "
                    "kernels leg")
    ap.add_argument("--vllm-decode", choices=["ours", "reference"], default=None,
                    help="BASELINE config 3 in vLLM with this package's or the reference's plugin")
    ap.add_argument("--model", default="/tmp/wlq_qwen7b_rowlut", help="checkpoint directory for --vllm-decode")
    ap.add_argument("--layers", type=int, default=None, help="layer count of the --vllm-decode model (28)")
    args = ap.parse_args()
    if args.vllm_decode:
        run_vllm_decode(args)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.case:
        run_case(args)
        return
    if args.impl == "reference":
        r = run_reference(args)
        if r is not None:
            print(json.dumps(r), flush=True)
        return
    result, _ = run_ours(args)
    if result is not None:
        world = result["n_gpus"]
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline(args.cpu_budget)
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
