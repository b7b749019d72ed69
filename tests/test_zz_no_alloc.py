"""wlq_gemm_streamk_noalloc: the stream-K tensor-core GEMM on the library's
static scratch, for callers that cannot allocate device memory (an FFI host
without a device allocator, or a serving loop that must not call cudaMalloc
because it synchronises the device and breaks stream capture).  Called
through the C ABI on a shape whose schedule splits every output tile over
several SMs, twice in a row (the second call reuses the scratch the first
one left), against the same op with a caller workspace (wlq_gemm_streamk)
and against the oracle.  Collected last, so a run that stops at the first
failure has run every other test; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

from _gpu import dev_layer, inputs
from _layers import make_np_layer, reference_output, rel_err

pytestmark = pytest.mark.gpu

TOL = 2e-2  # bf16 activations, normwise max relative error


def test_gemm_without_allocation_matches_workspace_path():
    from qwen_wlqfastshot_helen_beta_b200 import _C, _lib
    lib = _lib.lib
    assert torch.cuda.is_available()
    N, K, M, G = 3584, 3584, 512, 128  # 28 output tiles: stream-K over the SMs
    rng = np.random.default_rng(2026)
    L = make_np_layer(rng, N, K, G, 0, density=0.005, r=16)
    T = dev_layer(L)
    dtype = torch.bfloat16
    x, h = inputs(rng, L, M, dtype)
    lut = _C.prepack_lut(T["lut"], dtype)
    cols, vals = _C.prepack_outliers(T["q"], T["lut"], T["off"], T["cols"], T["vals"], N, K, 4, dtype, G, 0)
    y_ws = torch.empty((M, N), dtype=dtype, device="cuda")
    _C.gemm_forward(x, T["q"], lut, y_ws, N, K, 4, L.wpr, T["off"], cols, vals, h, T["B"], T["gamma"], L.scale,
                    G, 0, 1, workspace=True)
    torch.cuda.synchronize()
    oracle = reference_output(L, x.float().cpu().numpy(), h.cpu().numpy())

    def p(t):
        return ctypes.c_void_p(t.data_ptr())

    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        y = torch.full((M, N), float("nan"), dtype=dtype, device="cuda")
        rc = lib.wlq_gemm_streamk_noalloc(p(x), p(T["q"]), p(lut), p(y), p(T["off"]), p(cols), p(vals), p(h),
                                          p(T["B"]), p(T["gamma"]), L.scale, L.r, M, N, K, 4, L.wpr, G, 0,
                                          _lib.WLQ_LUT_PREPACKED, _lib.WLQ_DTYPE_BF16, stream)
        _lib.check(rc, "wlq_gemm_streamk_noalloc")
        torch.cuda.synchronize()
        assert _C.device_error() == 0, call
        assert torch.isfinite(y).all(), call
        assert rel_err(y.float().cpu().numpy(), y_ws.float().cpu().numpy()) <= TOL, call
        assert rel_err(y.float().cpu().numpy(), oracle) <= TOL, call
