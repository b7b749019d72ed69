"""The reference's ``vllm_wlq._C`` module surface over this package's C ABI.

Same function names, argument order and meaning as the pybind module of
csrc/vllm_binding.cpp:455-532 (``gemv_forward``, ``gemm_forward``,
``dequant_w0``, ``decode_ef_to_chunk_csr``, ``repack_q_indices_row_aligned``,
``init_workspaces``), each implemented by one call into libwlq_b200.so.  Like
the reference, optional tensors that are ``None`` or empty are absent, the
GPU functions launch on the current CUDA stream and raise ``RuntimeError`` on
bad input.  Two trailing keyword arguments select per-group codebooks
(``lut_group_size`` / ``lut_group_offset``, 0 = one codebook per row as in the
reference).  The GPU functions accept fp16 (as the reference) or bf16
activations; ``out`` must have the activation dtype.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import numpy as np
import torch

from ._lib import WLQ_DTYPE_BF16, WLQ_DTYPE_F16, WLQ_LUT_F16, WLQ_LUT_PREPACKED, check, lib

_NONE = None


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _opt(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    """None / undefined / empty -> None (csrc/vllm_binding.cpp:272-286)."""
    if t is None or t.numel() == 0:
        return None
    return t


def words_per_row(K: int, bits: int) -> int:
    return int(lib.wlq_words_per_row(int(K), int(bits)))


def _act_dtype(t: torch.Tensor) -> int:
    if t.dtype == torch.float16:
        return WLQ_DTYPE_F16
    if t.dtype == torch.bfloat16:
        return WLQ_DTYPE_BF16
    raise RuntimeError(f"wlq: activations must be float16 or bfloat16, got {t.dtype}")


def _require(cond: bool, msg) -> None:
    """Raises with `msg` (a string, or a callable that formats it: checks on
    the per-call path format their message only when they fail)."""
    if not cond:
        raise RuntimeError(f"wlq: {msg() if callable(msg) else msg}")


def _check_common(name, tensors, required):
    for nm, t in zip(required, tensors):
        _require(t is not None, lambda: f"{name}: {nm} is required")
        _require(t.is_cuda, lambda: f"{name}: {nm} must be a CUDA tensor")
        _require(t.is_contiguous(), lambda: f"{name}: {nm} must be contiguous")


def _check_opt(name, nm, t, dtype, device):
    if t is None:
        return
    _require(t.is_cuda and t.device == device, lambda: f"{name}: {nm} must be on {device}")
    _require(t.is_contiguous(), lambda: f"{name}: {nm} must be contiguous")
    _require(t.dtype == dtype, lambda: f"{name}: {nm} must be {dtype}, got {t.dtype}")


def _linear_checks(name, x, q_packed, lut_c, out, N, K, bits, wpr, offs, cols, vals, lora_B, lora_h, gamma,
                   group_size, group_offset, lut_format=WLQ_LUT_F16, lora_A=None):
    _check_common(name, (q_packed, lut_c, x, out), ("q_packed", "lut_c", "x", "out"))
    _require(bits == 4, lambda: f"{name}: the fused kernels read 4-bit indices only (bits={bits})")
    dev = x.device
    for nm, t in (("q_packed", q_packed), ("lut_c", lut_c), ("out", out)):
        _require(t.device == dev, lambda: f"{name}: {nm} must be on {dev}")
    _require(q_packed.dtype == torch.int32, lambda: f"{name}: q_packed must be int32")
    _require(lut_c.dtype == torch.float16, lambda: f"{name}: lut_c must be float16")
    _require(out.dtype == x.dtype, lambda: f"{name}: out dtype {out.dtype} must match x dtype {x.dtype}")
    _require(K > 0 and x.numel() % K == 0, lambda: f"{name}: x has {x.numel()} elements, not a multiple of K={K}")
    M = x.numel() // K
    _require(out.numel() == M * N, lambda: f"{name}: out has {out.numel()} elements, expected {M}x{N}")
    _require(q_packed.numel() >= N * wpr, lambda: f"{name}: q_packed has {q_packed.numel()} words, need {N}x{wpr}")
    ng = (K + group_offset + group_size - 1) // group_size if group_size > 0 else 1
    kcb = 1 << bits
    _require(lut_c.numel() == N * ng * kcb,
             lambda: f"{name}: lut_c has {lut_c.numel()} entries, expected {N}x{ng}x{kcb} (group_size={group_size})")
    if offs is not None and cols is not None and vals is not None:
        chunk_m = 640 if bits == 3 else 512
        nc = (K + chunk_m - 1) // chunk_m
        _check_opt(name, "chunk_offsets", offs, torch.int32, dev)
        # prepacked layers carry uint32 records (column | value << 16)
        _check_opt(name, "chunk_cols", cols, torch.int32 if lut_format == WLQ_LUT_PREPACKED else torch.uint16, dev)
        # prepacked layers carry float32 corrections in place of e5m2 bytes
        _check_opt(name, "chunk_vals", vals, torch.float32 if lut_format == WLQ_LUT_PREPACKED else torch.uint8, dev)
        _require(offs.numel() == N * (nc + 1), lambda: f"{name}: chunk_offsets must be [{N}, {nc + 1}]")
        _require(cols.numel() == vals.numel(), lambda: f"{name}: chunk_cols and chunk_vals lengths differ")
    r = 0
    _require(lora_h is None or lora_A is None, lambda: f"{name}: give lora_h or lora_A, not both")
    if lora_B is not None and (lora_h is not None or lora_A is not None) and gamma is not None:
        _check_opt(name, "lora_B", lora_B, torch.float16, dev)
        _check_opt(name, "dora_gamma", gamma, torch.float16, dev)
        r = int(lora_B.size(1)) if lora_B.dim() > 1 else 0
        _require(lora_B.numel() == N * r, lambda: f"{name}: lora_B must be [{N}, r]")
        _require(gamma.numel() == N, lambda: f"{name}: dora_gamma must have {N} values")
        if lora_h is not None:
            _check_opt(name, "lora_h", lora_h, torch.float32, dev)
            _require(lora_h.numel() == M * r, lambda: f"{name}: lora_h must hold {M}x{r} values")
        else:
            _check_opt(name, "lora_A", lora_A, x.dtype, dev)  # A in the activation type
            _require(lora_A.numel() == r * K, lambda: f"{name}: lora_A must be [{r}, {K}]")
    return M, r


def _stream(dev: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


class _DeviceGuard:
    """Makes `dev` the current CUDA device for the duration of a call (the C
    ABI launches on the current device)."""

    __slots__ = ("dev", "prev")

    def __init__(self, dev: torch.device):
        self.dev = dev.index if dev.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.dev:
            self.prev = cur
            torch.cuda.set_device(self.dev)

    def __exit__(self, *a):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


def gemv_forward(q_packed, lut_c, x, out, N, K, bits, chunk_offsets=None, chunk_cols=None, chunk_vals=None,
                 lora_B=None, lora_h=None, dora_gamma=None, lora_scale=1.0, lut_group_size=0,
                 lut_group_offset=0, lut_format=WLQ_LUT_F16):
    """Decode GEMV, M = x.numel() / K <= 16 (csrc/vllm_binding.cpp:253-315)."""
    N, K, bits = int(N), int(K), int(bits)
    offs, cols, vals = _opt(chunk_offsets), _opt(chunk_cols), _opt(chunk_vals)
    lb, lh, gm = _opt(lora_B), _opt(lora_h), _opt(dora_gamma)
    wpr = words_per_row(K, bits)
    M, r = _linear_checks("gemv_forward", x, q_packed, lut_c, out, N, K, bits, wpr, offs, cols, vals, lb, lh, gm,
                          int(lut_group_size), int(lut_group_offset), int(lut_format))
    with _DeviceGuard(x.device):
        rc = lib.wlq_gemv(_ptr(q_packed), _ptr(lut_c), _ptr(x), _ptr(out), _ptr(offs), _ptr(cols), _ptr(vals),
                          _ptr(lb), _ptr(lh), _ptr(gm), float(lora_scale), r, M, N, K, bits, wpr,
                          int(lut_group_size), int(lut_group_offset), int(lut_format), _act_dtype(x),
                          _stream(x.device))
    check(rc, "wlq_gemv")


def lora_h(x, lora_A, out=None):
    """H = x lora_A^T in fp32 ([M, r]) on this package's tensor-core kernel
    (wlq_lora_h): the DoRA low-rank input of the calls that do not compute it
    inside the decode GEMV.  Replaces F.linear(x, lora_A).float()
    (vllm_wlq/linear_method.py:962-963, 984); x [.., K] and lora_A [r, K] in
    the same activation dtype."""
    _check_common("lora_h", (x, lora_A), ("x", "lora_A"))
    _require(lora_A.dim() == 2, "lora_h: lora_A must be [r, K]")
    r, K = int(lora_A.shape[0]), int(lora_A.shape[1])
    _require(lora_A.dtype == x.dtype, lambda: f"lora_h: lora_A dtype {lora_A.dtype} must match x dtype {x.dtype}")
    _require(lora_A.device == x.device, lambda: f"lora_h: lora_A must be on {x.device}")
    _require(K > 0 and x.numel() % K == 0, lambda: f"lora_h: x has {x.numel()} elements, not a multiple of K={K}")
    M = x.numel() // K
    if out is None:
        out = torch.empty((M, r), dtype=torch.float32, device=x.device)
    _require(out.is_cuda and out.is_contiguous() and out.dtype == torch.float32 and out.numel() == M * r,
             lambda: f"lora_h: out must be a contiguous float32 CUDA tensor of {M}x{r} values")
    with _DeviceGuard(x.device):
        rc = lib.wlq_lora_h(_ptr(x), _ptr(lora_A), _ptr(out), M, K, r, _act_dtype(x), _stream(x.device))
    check(rc, "wlq_lora_h")
    return out


_SM_COUNT = {}


def folds_h(M, N, K, r, lut_format, x) -> bool:
    """Whether gemv_lora_a takes this call (the GEMV computing h = A x): up
    to 16 tokens with r <= 48, or 17..32 tokens with r <= 16 when the
    tensor-core GEMM's 128-row tiles would not fill the device (the rule
    wlq_gemm applies, csrc/wlq_abi.cu gemv_preferred); prepacked layout and
    16-byte aligned rows either way."""
    if not (0 < r <= 48 and lut_format == WLQ_LUT_PREPACKED and K % 8 == 0 and x.data_ptr() % 16 == 0):
        return False
    if M <= 16:
        return True
    if M > 32 or r > 16:
        return False
    dev = x.device.index if x.device.index is not None else torch.cuda.current_device()
    if dev not in _SM_COUNT:
        _SM_COUNT[dev] = torch.cuda.get_device_properties(dev).multi_processor_count
    return (N + 127) // 128 < _SM_COUNT[dev]


def gemv_lora_a(q_packed, lut_c, x, out, N, K, bits, chunk_offsets, chunk_cols, chunk_vals, lora_B, lora_A,
                dora_gamma, lora_scale=1.0, lut_group_size=0, lut_group_offset=0, lut_format=WLQ_LUT_PREPACKED):
    """Decode GEMV (M <= 32) that computes the DoRA input h = lora_A x itself
    (lora_A [r, K] in x's dtype, r <= 48, r <= 16 above 16 tokens; prepacked
    layout): one launch in place of F.linear + .float() + GEMV
    (vllm_wlq/linear_method.py:962-999)."""
    N, K, bits = int(N), int(K), int(bits)
    offs, cols, vals = _opt(chunk_offsets), _opt(chunk_cols), _opt(chunk_vals)
    lb, la, gm = _opt(lora_B), _opt(lora_A), _opt(dora_gamma)
    wpr = words_per_row(K, bits)
    M, r = _linear_checks("gemv_lora_a", x, q_packed, lut_c, out, N, K, bits, wpr, offs, cols, vals, lb, None, gm,
                          int(lut_group_size), int(lut_group_offset), int(lut_format), lora_A=la)
    with _DeviceGuard(x.device):
        rc = lib.wlq_gemv_lora_a(_ptr(q_packed), _ptr(lut_c), _ptr(x), _ptr(out), _ptr(offs), _ptr(cols),
                                 _ptr(vals), _ptr(lb), _ptr(la), _ptr(gm), float(lora_scale), r, M, N, K, bits, wpr,
                                 int(lut_group_size), int(lut_group_offset), int(lut_format), _act_dtype(x),
                                 _stream(x.device))
    check(rc, "wlq_gemv_lora_a")


# One stream-K workspace per device (wlq_gemm_streamk), allocated and zeroed
# on the device's first GEMM call outside CUDA-graph capture and kept for the
# process (its flags are left zero by every call).  The torch ops run on one
# stream per device, as vLLM runs a model; calls on several streams at once
# would share it and must use gemm_forward(..., workspace=False).
_GEMM_WS = {}


def gemm_workspace(dev: torch.device):
    """This device's stream-K workspace, or None while a CUDA graph is being
    captured before it exists (the call then takes the data-parallel
    schedule)."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _GEMM_WS.get(idx)
    if ws is None:
        if torch.cuda.is_current_stream_capturing():
            return None
        nbytes = int(lib.wlq_gemm_workspace_bytes(idx))
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=torch.device("cuda", idx))
        _GEMM_WS[idx] = ws
    return ws


def gemm_forward(X, q_packed, lut_c, out, N, K, bits, words_per_row, chunk_offsets=None, chunk_cols=None,
                 chunk_vals=None, lora_H=None, lora_B=None, dora_gamma=None, lora_scale=1.0, lut_group_size=0,
                 lut_group_offset=0, lut_format=WLQ_LUT_F16, workspace=True):
    """Batched forward for any M (csrc/vllm_binding.cpp:318-419).  The
    tensor-core path takes the stream-K schedule with this device's
    workspace (workspace=False: the data-parallel schedule of wlq_gemm)."""
    N, K, bits, wpr = int(N), int(K), int(bits), int(words_per_row)
    offs, cols, vals = _opt(chunk_offsets), _opt(chunk_cols), _opt(chunk_vals)
    lb, lh, gm = _opt(lora_B), _opt(lora_H), _opt(dora_gamma)
    M, r = _linear_checks("gemm_forward", X, q_packed, lut_c, out, N, K, bits, wpr, offs, cols, vals, lb, lh, gm,
                          int(lut_group_size), int(lut_group_offset), int(lut_format))
    ws = gemm_workspace(X.device) if workspace and M > 16 else None
    with _DeviceGuard(X.device):
        if ws is not None:
            rc = lib.wlq_gemm_streamk(_ptr(X), _ptr(q_packed), _ptr(lut_c), _ptr(out), _ptr(offs), _ptr(cols),
                                      _ptr(vals), _ptr(lh), _ptr(lb), _ptr(gm), float(lora_scale), r, M, N, K, bits,
                                      wpr, int(lut_group_size), int(lut_group_offset), int(lut_format),
                                      _act_dtype(X), _ptr(ws), ws.numel(), _stream(X.device))
        else:
            rc = lib.wlq_gemm(_ptr(X), _ptr(q_packed), _ptr(lut_c), _ptr(out), _ptr(offs), _ptr(cols), _ptr(vals),
                              _ptr(lh), _ptr(lb), _ptr(gm), float(lora_scale), r, M, N, K, bits, wpr,
                              int(lut_group_size), int(lut_group_offset), int(lut_format), _act_dtype(X),
                              _stream(X.device))
    check(rc, "wlq_gemm_streamk" if ws is not None else "wlq_gemm")


def gemv_allreduce(comm, X, q_packed, lut_c, out, N, K, bits, words_per_row, chunk_offsets=None, chunk_cols=None,
                   chunk_vals=None, lora_H=None, lora_B=None, dora_gamma=None, lora_scale=1.0, lut_group_size=0,
                   lut_group_offset=0, lut_format=WLQ_LUT_F16, lora_A=None):
    """Row-parallel decode forward (M <= 16) on this rank's K shard with the
    all-reduce of `out` over `comm`'s ranks fused into the kernel (see
    qwen_wlqfastshot_helen_beta_b200.tp.TPComm).  The DoRA input is lora_H,
    or lora_A (this rank's K columns of A, computed into h in the kernel as in
    gemv_lora_a).  Every rank of the group must make the same calls in the
    same order."""
    N, K, bits, wpr = int(N), int(K), int(bits), int(words_per_row)
    offs, cols, vals = _opt(chunk_offsets), _opt(chunk_cols), _opt(chunk_vals)
    lb, lh, la, gm = _opt(lora_B), _opt(lora_H), _opt(lora_A), _opt(dora_gamma)
    M, r = _linear_checks("gemv_allreduce", X, q_packed, lut_c, out, N, K, bits, wpr, offs, cols, vals, lb, lh, gm,
                          int(lut_group_size), int(lut_group_offset), int(lut_format), lora_A=la)
    with _DeviceGuard(X.device):
        rc = lib.wlq_gemv_allreduce(_ptr(q_packed), _ptr(lut_c), _ptr(X), _ptr(out), _ptr(offs), _ptr(cols),
                                    _ptr(vals), _ptr(lb), _ptr(lh), _ptr(la), _ptr(gm), float(lora_scale), r, M, N,
                                    K, bits, wpr, int(lut_group_size), int(lut_group_offset), int(lut_format),
                                    _act_dtype(X), comm.bufs, comm.rank, comm.world, comm.max_N, _stream(X.device))
    check(rc, "wlq_gemv_allreduce")


def dequant_w0(q_packed, lut_c, W_out, N, K, bits, words_per_row, chunk_offsets, chunk_cols, chunk_vals,
               lut_group_size=0, lut_group_offset=0):
    """Dense fp16 W = codebook[q] with outliers replaced, bit-exact
    (csrc/vllm_binding.cpp:421-453).  CUDA tensors run the GPU kernel; CPU
    tensors the host codec (load time without a GPU)."""
    N, K, bits, wpr = int(N), int(K), int(bits), int(words_per_row)
    offs, cols, vals = _opt(chunk_offsets), _opt(chunk_cols), _opt(chunk_vals)
    _require(W_out.dtype == torch.float16 and W_out.is_contiguous() and W_out.numel() == N * K,
             "dequant_w0: W_out must be a contiguous float16 [N, K] tensor")
    _require(q_packed.dtype == torch.int32 and lut_c.dtype == torch.float16, "dequant_w0: q int32, lut fp16")
    _require(q_packed.is_contiguous() and lut_c.is_contiguous(), "dequant_w0: inputs must be contiguous")
    if W_out.is_cuda:
        for nm, t in (("q_packed", q_packed), ("lut_c", lut_c), ("chunk_offsets", offs), ("chunk_cols", cols),
                      ("chunk_vals", vals)):
            _require(t is None or (t.is_cuda and t.device == W_out.device and t.is_contiguous()),
                     lambda: f"dequant_w0: {nm} must be a contiguous tensor on {W_out.device}")
        with _DeviceGuard(W_out.device):
            rc = lib.wlq_dequant(_ptr(q_packed), _ptr(lut_c), _ptr(W_out), _ptr(offs), _ptr(cols), _ptr(vals),
                                 N, K, bits, wpr, int(lut_group_size), int(lut_group_offset),
                                 _stream(W_out.device))
        check(rc, "wlq_dequant")
        return
    for nm, t in (("q_packed", q_packed), ("lut_c", lut_c), ("chunk_offsets", offs), ("chunk_cols", cols),
                  ("chunk_vals", vals)):
        _require(t is None or (not t.is_cuda and t.is_contiguous()), lambda: f"dequant_w0: {nm} must be a CPU tensor")
    rc = lib.wlq_dequant_host(_ptr(q_packed), _ptr(lut_c), _ptr(W_out), _ptr(offs), _ptr(cols), _ptr(vals),
                              N, K, bits, wpr, int(lut_group_size), int(lut_group_offset))
    check(rc, "wlq_dequant_host")


def prepack_lut(lut_c: torch.Tensor, act_dtype: torch.dtype) -> torch.Tensor:
    """fp16 codebooks (any shape ending in 16) -> the WLQ_LUT_PREPACKED layout
    for `act_dtype` (same shape, stored as float16 bits).  CUDA tensors use the
    GPU kernel, CPU tensors the host codec."""
    _require(lut_c.dtype == torch.float16 and lut_c.is_contiguous() and lut_c.shape[-1] == 16,
             "prepack_lut: lut_c must be a contiguous float16 tensor with 16 entries per codebook")
    dt = WLQ_DTYPE_BF16 if act_dtype == torch.bfloat16 else WLQ_DTYPE_F16
    out = torch.empty_like(lut_c)
    n = lut_c.numel() // 16
    if lut_c.is_cuda:
        with _DeviceGuard(lut_c.device):
            check(lib.wlq_prepack_lut(_ptr(lut_c), _ptr(out), n, dt, _stream(lut_c.device)), "wlq_prepack_lut")
    else:
        check(lib.wlq_prepack_lut_host(_ptr(lut_c), _ptr(out), n, dt), "wlq_prepack_lut_host")
    return out


def prepack_outliers(q_packed, lut_c, chunk_offsets, chunk_cols, chunk_vals, N, K, bits, act_dtype,
                     lut_group_size=0, lut_group_offset=0):
    """Reference-layout outliers -> (int32 records: global column | value in
    the MMA type << 16, float32 corrections) for `act_dtype`, the
    WLQ_LUT_PREPACKED outlier stream (CUDA tensors; each row's entries in
    ascending column order)."""
    offs, cols, vals = _opt(chunk_offsets), _opt(chunk_cols), _opt(chunk_vals)
    if offs is None or cols is None or vals is None:
        return None, None
    dev = q_packed.device
    for nm, t in (("q_packed", q_packed), ("lut_c", lut_c), ("chunk_offsets", offs), ("chunk_cols", cols),
                  ("chunk_vals", vals)):
        _require(t.is_cuda and t.device == dev and t.is_contiguous(),
                 lambda: f"prepack_outliers: {nm} must be on {dev}")
    _require(vals.dtype == torch.uint8 and cols.dtype == torch.uint16, "prepack_outliers: e5m2 bytes / uint16 cols")
    gcols = torch.empty(cols.numel(), dtype=torch.int32, device=dev)
    delta = torch.empty(cols.numel(), dtype=torch.float32, device=dev)
    dt = WLQ_DTYPE_BF16 if act_dtype == torch.bfloat16 else WLQ_DTYPE_F16
    with _DeviceGuard(dev):
        rc = lib.wlq_prepack_outliers(_ptr(q_packed), _ptr(lut_c), _ptr(offs), _ptr(cols), _ptr(vals), cols.numel(),
                                      int(N), int(K), int(bits), words_per_row(K, bits), int(lut_group_size),
                                      int(lut_group_offset), dt, _ptr(gcols), _ptr(delta), _stream(dev))
    check(rc, "wlq_prepack_outliers")
    return gcols, delta


def init_workspaces(max_N, max_K, device):
    """Interface parity with csrc/vllm_binding.cpp:241-251; no workspace is needed."""
    dev = torch.device(device)
    check(lib.wlq_init_workspaces(int(max_N), int(max_K), dev.index or 0), "wlq_init_workspaces")


def device_error(device=None, clear: bool = True) -> int:
    """Device error word (bit 0: a bounded pipeline wait in a GEMM kernel
    gave up, so that call's output is undefined).  Synchronous."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    flags = ctypes.c_uint(0)
    check(lib.wlq_device_error(dev.index or 0, ctypes.byref(flags), 1 if clear else 0), "wlq_device_error")
    return int(flags.value)


# ----------------------------------------------------------------- codecs ---

def _cpu_i32(t: torch.Tensor) -> torch.Tensor:
    t = t.detach().to("cpu").contiguous()
    if t.dtype != torch.int32:
        t = t.view(torch.int32) if t.element_size() == 4 else t.to(torch.int32)
    return t


def repack_q_indices_row_aligned(q_packed_raw, N, K, bits) -> Tuple[torch.Tensor, int]:
    """Continuous stream -> row-aligned int32 words (csrc/vllm_binding.cpp:198-236)."""
    src = _cpu_i32(q_packed_raw)
    wpr = words_per_row(K, bits)
    out = torch.zeros(int(N) * wpr, dtype=torch.int32)
    w = ctypes.c_int64(0)
    check(lib.wlq_repack_q_indices_row_aligned(_ptr(src), src.numel(), int(N), int(K), int(bits), _ptr(out),
                                                out.numel(), ctypes.byref(w)), "wlq_repack_q_indices_row_aligned")
    return out, int(w.value)


def repack_q_indices_slice(q_packed_raw, N_full, K_full, bits, r0, r1, c0, c1) -> Tuple[torch.Tensor, int]:
    """Rows [r0,r1) x cols [c0,c1) of a continuous stream -> row-aligned words."""
    src = _cpu_i32(q_packed_raw)
    wpr = words_per_row(int(c1) - int(c0), bits)
    out = torch.zeros((int(r1) - int(r0)) * wpr, dtype=torch.int32)
    w = ctypes.c_int64(0)
    check(lib.wlq_repack_q_indices_slice(_ptr(src), src.numel(), int(N_full), int(K_full), int(bits), int(r0),
                                          int(r1), int(c0), int(c1), _ptr(out), out.numel(), ctypes.byref(w)),
          "wlq_repack_q_indices_slice")
    return out, int(w.value)


def decode_ef_to_chunk_csr(ef_tile_meta, ef_bitstream, N, K, tile_size, chunk_m):
    """EF tiles -> (chunk_offsets int32 [N, nc+1], chunk_cols uint16) (csrc/vllm_binding.cpp:94-196)."""
    meta = ef_tile_meta.detach().to("cpu", torch.int64).contiguous()
    bs = _cpu_i32(ef_bitstream)
    N, K, tile_size, chunk_m = int(N), int(K), int(tile_size), int(chunk_m)
    nc = (K + chunk_m - 1) // chunk_m
    offs = torch.zeros((N, nc + 1), dtype=torch.int32)
    nnz = ctypes.c_int64(0)
    n_tiles = meta.numel() // 2
    check(lib.wlq_decode_ef_to_chunk_csr(_ptr(meta), n_tiles, _ptr(bs), bs.numel(), N, K, tile_size, chunk_m,
                                         _ptr(offs), None, 0, ctypes.byref(nnz)), "wlq_decode_ef_to_chunk_csr")
    cols = torch.empty(int(nnz.value), dtype=torch.uint16)
    check(lib.wlq_decode_ef_to_chunk_csr(_ptr(meta), n_tiles, _ptr(bs), bs.numel(), N, K, tile_size, chunk_m,
                                         _ptr(offs), _ptr(cols), cols.numel(), ctypes.byref(nnz)),
          "wlq_decode_ef_to_chunk_csr")
    return offs, cols


def decode_ef_positions(ef_tile_meta, ef_bitstream, N, K, tile_size) -> np.ndarray:
    """EF tiles -> sorted flat outlier positions r*K + c (int64 numpy)."""
    meta = ef_tile_meta.detach().to("cpu", torch.int64).contiguous()
    bs = _cpu_i32(ef_bitstream)
    cnt = ctypes.c_int64(0)
    n_tiles = meta.numel() // 2
    check(lib.wlq_decode_ef_positions(_ptr(meta), n_tiles, _ptr(bs), bs.numel(), int(N), int(K), int(tile_size),
                                      None, 0, ctypes.byref(cnt)), "wlq_decode_ef_positions")
    pos = torch.empty(int(cnt.value), dtype=torch.int64)
    check(lib.wlq_decode_ef_positions(_ptr(meta), n_tiles, _ptr(bs), bs.numel(), int(N), int(K), int(tile_size),
                                      _ptr(pos), pos.numel(), ctypes.byref(cnt)), "wlq_decode_ef_positions")
    return pos.numpy()


def positions_to_chunk_csr(positions, N, K, chunk_m):
    """Sorted flat positions -> (chunk_offsets, chunk_cols) (vllm_wlq/linear_method.py:284-303)."""
    pos = torch.as_tensor(np.ascontiguousarray(positions, dtype=np.int64))
    N, K, chunk_m = int(N), int(K), int(chunk_m)
    nc = (K + chunk_m - 1) // chunk_m
    offs = torch.zeros((N, nc + 1), dtype=torch.int32)
    cols = torch.empty(pos.numel(), dtype=torch.uint16)
    check(lib.wlq_positions_to_chunk_csr(_ptr(pos), pos.numel(), N, max(K, 1), chunk_m, _ptr(offs), _ptr(cols)),
          "wlq_positions_to_chunk_csr")
    return offs, cols


def build_chunk_csr_from_mask(mask, chunk_m):
    """Dense bool mask [N, K] -> (chunk_offsets, chunk_cols) (vllm_wlq/linear_method.py:284-303)."""
    m = np.ascontiguousarray(np.asarray(mask), dtype=np.uint8)
    N, K = m.shape
    nc = (K + chunk_m - 1) // chunk_m
    offs = torch.zeros((N, nc + 1), dtype=torch.int32)
    nnz = ctypes.c_int64(0)
    mp = ctypes.c_void_p(m.ctypes.data)
    check(lib.wlq_build_chunk_csr(mp, N, K, int(chunk_m), _ptr(offs), None, 0, ctypes.byref(nnz)),
          "wlq_build_chunk_csr")
    cols = torch.empty(int(nnz.value), dtype=torch.uint16)
    check(lib.wlq_build_chunk_csr(mp, N, K, int(chunk_m), _ptr(offs), _ptr(cols), cols.numel(), ctypes.byref(nnz)),
          "wlq_build_chunk_csr")
    return offs, cols


def fp16_to_fp8_bytes(vals: torch.Tensor) -> torch.Tensor:
    """fp16 outlier values -> e5m2 bytes (vllm_wlq/linear_method.py:306-308)."""
    v = vals.detach().to("cpu").contiguous()
    if v.dtype != torch.float16:
        raise RuntimeError("fp16_to_fp8_bytes: expects float16 values")
    out = torch.empty(v.numel(), dtype=torch.uint8)
    check(lib.wlq_fp16_to_fp8_bytes(_ptr(v), v.numel(), _ptr(out)), "wlq_fp16_to_fp8_bytes")
    return out
