"""Parity of the sm_100a CUDA path with the oracle and with the reference's own
CUDA kernels (compiled from source into oracle/_ref).  B200 only."""
import ctypes
import os

import numpy as np
import pytest
import torch

from _gpu import C, dev_layer, inputs, run_ours
from _layers import make_np_layer, reference_output, rel_err
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TOL = {torch.float16: 5e-3, torch.bfloat16: 2e-2}  # normwise max relative error


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "the gpu tests need a CUDA device"
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield


# ------------------------------------------------------------------ dequant

@pytest.mark.parametrize("N,K,G,goff,density", [
    (64, 1024, 0, 0, 0.01), (40, 203, 0, 0, 0.05), (33, 1100, 0, 0, 0.02), (7, 37, 0, 0, 0.3),
    (48, 1000, 128, 0, 0.01), (20, 448, 128, 64, 0.02), (16, 640, 32, 0, 0.0), (5, 2, 0, 0, 0.5)])
def test_dequant_bit_exact(N, K, G, goff, density):
    rng = np.random.default_rng(N * 1000 + K)
    L = make_np_layer(rng, N, K, G, goff, density=density, outliers=density > 0)
    T = dev_layer(L)
    W = torch.empty((N, K), dtype=torch.float16, device="cuda")
    C().dequant_w0(T["q"], T["lut"], W, N, K, 4, L.wpr, T["off"], T["cols"], T["vals"], G, goff)
    torch.cuda.synchronize()
    assert np.array_equal(W.cpu().numpy().view(np.uint16), L.dense().view(np.uint16))


def test_dequant_other_bit_widths():
    rng = np.random.default_rng(9)
    for bits, (N, K) in [(1, (9, 70)), (2, (5, 33)), (3, (6, 1300))]:
        idx = rng.integers(0, 1 << bits, size=(N, K), dtype=np.uint8)
        q, wpr = O.pack_row_aligned(idx, bits)
        lut = rng.standard_normal((N, 1 << bits)).astype(np.float16)
        chunk_m = 640 if bits == 3 else 512
        off, cols = O.build_chunk_csr(rng.random((N, K)) < 0.05, chunk_m)
        vals = rng.integers(0, 256, size=cols.size, dtype=np.uint8)
        ref = O.dequant(q, wpr, lut, N, K, bits, 0, 0, off, cols, vals, chunk_m)
        W = torch.empty((N, K), dtype=torch.float16, device="cuda")
        C().dequant_w0(torch.from_numpy(q.view(np.int32)).cuda(), torch.from_numpy(lut).cuda(), W, N, K, bits, wpr,
                       torch.from_numpy(off).cuda(), torch.from_numpy(cols).cuda(), torch.from_numpy(vals).cuda())
        torch.cuda.synchronize()
        assert np.array_equal(W.cpu().numpy().view(np.uint16), ref.view(np.uint16)), bits


# --------------------------------------------------------- GEMV vs oracle

LAYER_CASES = [
    # N, K, G, goff, outliers, dora
    (64, 1024, 0, 0, True, True),
    (40, 203, 0, 0, True, True),       # ragged K, N not a multiple of 16
    (100, 4096, 128, 0, True, True),   # per-group codebooks
    (48, 448, 128, 64, True, False),   # tensor-parallel shard starting mid-group
    (33, 1100, 32, 0, False, True),
    (16, 130, 0, 0, True, False),
    (64, 18944, 128, 0, True, True),  # activations too large to stage: they stream through the ring
]


@pytest.mark.parametrize("case", LAYER_CASES, ids=lambda c: f"N{c[0]}K{c[1]}G{c[2]}o{c[3]}")
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_gemv_matches_oracle(case, dtype):
    N, K, G, goff, outl, dora = case
    rng = np.random.default_rng(N + K + G)
    L = make_np_layer(rng, N, K, G, goff, density=0.02, outliers=outl, dora=dora)
    T = dev_layer(L)
    for M in (1, 2, 3, 7, 8, 9, 15, 16):
        x, h = inputs(rng, L, M, dtype)
        ref = reference_output(L, x.float().cpu().numpy(), None if h is None else h.cpu().numpy())
        ys = []
        for fmt in (0, 1):  # reference fp16 codebooks, prepacked codebooks
            y = run_ours(L, T, x, h, gemv=(M == 1), fmt=fmt)
            e = rel_err(y.float().cpu().numpy(), ref)
            assert e <= TOL[dtype], (M, fmt, e)
            assert torch.isfinite(y).all()
            ys.append(y)
        assert torch.equal(ys[0], ys[1])  # same arithmetic either way


FOLD_CASES = [
    # N, K, G, goff, r
    (64, 1024, 0, 0, 16),      # per-row codebooks, K split over a 3-CTA cluster (ranks of 3, 3, 2 chunks)
    (100, 4096, 128, 0, 16),   # per-group codebooks, 8-CTA cluster
    (48, 448, 128, 64, 8),     # shard starting mid-group, rank below one MMA tile
    (300, 1024, 32, 0, 24),    # 32-wide groups, rank in two MMA tiles
    (64, 18944, 128, 0, 32),   # activations too large to stage, read through L1
    (1200, 512, 128, 0, 16),   # many row tiles, no cluster
    (4100, 384, 128, 0, 16),   # no K split, ragged last CTA
    (18944, 1024, 128, 0, 32), # no K split, rank in two MMA tiles
    (256, 3584, 128, 0, 48),   # rank in three MMA tiles (a fused qkv of three rank-16 adapters), 2-stage ring
    (100, 1024, 0, 0, 40),     # per-row codebooks, rank 40 padded to three tiles
]


@pytest.mark.parametrize("case", FOLD_CASES, ids=lambda c: f"N{c[0]}K{c[1]}G{c[2]}o{c[3]}r{c[4]}")
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_gemv_lora_a_matches_oracle(case, dtype):
    """wlq_gemv_lora_a (h = A x computed inside the GEMV) against the oracle
    with the reference's h = fp16(A x), and against the GEMV given that h."""
    N, K, G, goff, r = case
    rng = np.random.default_rng(N + K + r)
    L = make_np_layer(rng, N, K, G, goff, density=0.02, r=r)
    T = dev_layer(L)
    lut = C().prepack_lut(T["lut"], dtype)
    cols, vals = C().prepack_outliers(T["q"], T["lut"], T["off"], T["cols"], T["vals"], L.N, L.K, 4, dtype, L.G,
                                      L.goff)
    A = T["A"].to(dtype).contiguous()
    for M in (1, 2, 5, 8, 9, 16) + ((17, 32) if r <= 16 else ()):  # r > 16 above 16 tokens: see folds_h
        x, h = inputs(rng, L, M, dtype)
        ref = reference_output(L, x.float().cpu().numpy(), h.cpu().numpy())
        y = torch.full((M, N), float("nan"), dtype=dtype, device="cuda")
        C().gemv_lora_a(T["q"], lut, x, y, N, K, 4, T["off"], cols, vals, T["B"], A, T["gamma"], L.scale, L.G,
                        L.goff)
        torch.cuda.synchronize()
        assert torch.isfinite(y).all(), M
        e = rel_err(y.float().cpu().numpy(), ref)
        assert e <= TOL[dtype], (M, e)
        if M <= 16:
            y_h = run_ours(L, T, x, h, gemv=(M == 1), fmt=1)
            assert rel_err(y.float().cpu().numpy(), y_h.float().cpu().numpy()) <= 1e-2, M


def test_gemv_lora_a_rejects():
    """The in-kernel h needs the prepacked layout, r <= 48 and 16-byte rows."""
    rng = np.random.default_rng(3)
    L = make_np_layer(rng, 32, 256, 0, 0, r=56)
    T = dev_layer(L)
    x = torch.randn((2, 256), device="cuda", dtype=torch.float16)
    y = torch.empty((2, 32), device="cuda", dtype=torch.float16)
    lut = C().prepack_lut(T["lut"], torch.float16)
    cols, vals = C().prepack_outliers(T["q"], T["lut"], T["off"], T["cols"], T["vals"], 32, 256, 4, torch.float16)
    with pytest.raises(RuntimeError, match="r <= 48"):
        C().gemv_lora_a(T["q"], lut, x, y, 32, 256, 4, T["off"], cols, vals, T["B"], T["A"], T["gamma"], 1.0)
    L = make_np_layer(rng, 32, 256, 0, 0, r=16)
    T = dev_layer(L)
    with pytest.raises(RuntimeError, match="prepacked"):
        C().gemv_lora_a(T["q"], T["lut"], x, y, 32, 256, 4, T["off"], T["cols"], T["vals"], T["B"], T["A"],
                        T["gamma"], 1.0, lut_format=0)


@pytest.mark.parametrize("split", [11, 13, 16])
def test_gemv_forced_split_matches_oracle(split):
    """K split over non-portable clusters (more than 8 CTAs, not a power of
    two) forced through wlq_gemv_set_split: the cluster reduction of 11, 13
    or 16 partial tiles against the oracle, h given and h computed in the
    kernel, and wlq_gemv_last_split reporting the split that ran."""
    from qwen_wlqfastshot_helen_beta_b200 import _lib
    lib = _lib.lib
    rng = np.random.default_rng(split)
    N, K = 160, 18944  # 148 chunks of 128 columns
    L = make_np_layer(rng, N, K, 128, 0, density=0.01, r=16)
    T = dev_layer(L)
    dtype = torch.bfloat16
    lut = C().prepack_lut(T["lut"], dtype)
    cols, vals = C().prepack_outliers(T["q"], T["lut"], T["off"], T["cols"], T["vals"], N, K, 4, dtype, 128, 0)
    A = T["A"].to(dtype).contiguous()
    _lib.check(lib.wlq_gemv_set_split(split), "wlq_gemv_set_split")
    try:
        for M in (1, 8, 16):
            x, h = inputs(rng, L, M, dtype)
            ref = reference_output(L, x.float().cpu().numpy(), h.cpu().numpy())
            y = torch.full((M, N), float("nan"), dtype=dtype, device="cuda")
            C().gemv_lora_a(T["q"], lut, x, y, N, K, 4, T["off"], cols, vals, T["B"], A, T["gamma"], L.scale, 128, 0)
            torch.cuda.synchronize()
            assert lib.wlq_gemv_last_split() == split
            assert rel_err(y.float().cpu().numpy(), ref) <= TOL[dtype], (M, "h in the kernel")
            y2 = run_ours(L, T, x, h, gemv=(M == 1), fmt=1)
            assert lib.wlq_gemv_last_split() == split
            assert rel_err(y2.float().cpu().numpy(), ref) <= TOL[dtype], (M, "h given")
    finally:
        _lib.check(lib.wlq_gemv_set_split(0), "wlq_gemv_set_split")
    with pytest.raises(RuntimeError, match="outside"):
        _lib.check(lib.wlq_gemv_set_split(17), "wlq_gemv_set_split")


@pytest.mark.parametrize("G,goff", [(0, 0), (64, 0), (128, 64)], ids=["per_row", "g64", "g128_off64"])
@pytest.mark.parametrize("r", [0, 16, 32], ids=["h_given", "h_r16", "h_r32"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_gemv_16warp_ctas_match_oracle(G, goff, r, dtype):
    """The one-CTA-per-SM shape (16 warps sharing one staged copy of the
    activations, a 2-stage ring per warp) against the oracle: K unsplit
    (forced split 1) with a ragged last 128-column chunk, 8 and 16 tokens
    (activations too large for 4-warp CTAs to stage), per-row and per-group
    codebooks, h given (r = 0 here) and h computed in the kernel (rank 16 and
    32), and wlq_gemv_last_warps reporting the shape that ran."""
    from qwen_wlqfastshot_helen_beta_b200 import _lib
    lib = _lib.lib
    rng = np.random.default_rng(100 + G + r + goff)
    N = 80
    _lib.check(lib.wlq_gemv_set_split(1), "wlq_gemv_set_split")
    try:
        for M, K in ((8, 3104), (16, 1440)):
            L = make_np_layer(rng, N, K, G, goff, density=0.01, r=max(r, 16))
            T = dev_layer(L)
            x, h = inputs(rng, L, M, dtype)
            ref = reference_output(L, x.float().cpu().numpy(), h.cpu().numpy())
            if r == 0:
                y = run_ours(L, T, x, h, gemv=True, fmt=1)
            else:
                lut = C().prepack_lut(T["lut"], dtype)
                cols, vals = C().prepack_outliers(T["q"], T["lut"], T["off"], T["cols"], T["vals"], N, K, 4, dtype, G,
                                                  goff)
                y = torch.full((M, N), float("nan"), dtype=dtype, device="cuda")
                C().gemv_lora_a(T["q"], lut, x, y, N, K, 4, T["off"], cols, vals, T["B"], T["A"].to(dtype).contiguous(),
                                T["gamma"], L.scale, G, goff)
                torch.cuda.synchronize()
            assert lib.wlq_gemv_last_warps() == 16, (M, K)
            assert lib.wlq_gemv_last_split() == 1
            assert rel_err(y.float().cpu().numpy(), ref) <= TOL[dtype], (M, K)
    finally:
        _lib.check(lib.wlq_gemv_set_split(0), "wlq_gemv_set_split")


@pytest.mark.parametrize("M,K,r", [(1, 3584, 16), (7, 1000, 48), (64, 3584, 64), (200, 4864, 48), (512, 18944, 16),
                                   (2048, 3584, 80), (8192, 3584, 48), (33, 1004, 16), (130, 3586, 24)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_lora_h_matches_fp32(M, K, r, dtype):
    """wlq_lora_h (H = X A^T on the tensor core, fp32 accumulation; K split
    over a cluster for few token tiles, ranks past 64 in a second grid plane,
    unaligned rows on the row kernel) against the same product in fp32."""
    g = torch.Generator(device="cuda")
    g.manual_seed(M * 7 + K + r)
    X = torch.randn((M, K), generator=g, device="cuda").to(dtype)
    A = (torch.randn((r, K), generator=g, device="cuda") * 0.01).to(dtype)
    H = C().lora_h(X, A)
    torch.cuda.synchronize()
    ref = X.double() @ A.double().t()
    err = ((H.double() - ref).abs().max() / ref.abs().max()).item()
    assert H.shape == (M, r) and H.dtype == torch.float32
    assert err <= 1e-5, err
    H2 = C().lora_h(X, A)  # the cluster reduction sums in rank order: the same bits every call
    assert torch.equal(H, H2)


def test_gemv_outlier_edges():
    """Outliers at the first and last column, in a ragged last chunk, a row
    made only of outliers, and rows without any."""
    rng = np.random.default_rng(77)
    N, K = 24, 1100
    L = make_np_layer(rng, N, K, 0, 0, outliers=False, dora=True)
    mask = np.zeros((N, K), bool)
    mask[0, 0] = mask[0, K - 1] = True
    mask[1, 1024:] = True
    mask[2, :] = True
    mask[5, 511:513] = True
    L.off, L.cols = O.build_chunk_csr(mask, 512)
    L.vals = O.fp16_to_fp8_bytes((rng.standard_normal(L.cols.size) * 0.1).astype(np.float16))
    T = dev_layer(L)
    for M in (1, 4, 16):
        for dtype in (torch.float16, torch.bfloat16):
            x, h = inputs(rng, L, M, dtype)
            ref = reference_output(L, x.float().cpu().numpy(), h.cpu().numpy())
            for fmt in (0, 1):
                y = run_ours(L, T, x, h, fmt=fmt)
                assert rel_err(y.float().cpu().numpy(), ref) <= TOL[dtype], (M, dtype, fmt)


# ------------------------------------------------- the reference's kernels

def _ref_lib():
    path = os.path.join(ROOT, "oracle", "_ref", "libwlq_ref_kernels.so")
    if not os.path.exists(path):
        pytest.skip("reference kernels not built (oracle/build_ref.sh needs the reference tree)")
    lib = ctypes.CDLL(path)
    return lib


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _compare_with_reference_kernels(lib, L, Ms, rng, tol=5e-3):
    """Same inputs through the reference's own CUDA kernels and ours, both
    against the oracle (fp16 activations, as the reference casts them)."""
    T = dev_layer(L)
    N, K = L.N, L.K
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    nc = (K + 511) // 512
    i, f = ctypes.c_int, ctypes.c_float
    # bit-exact dequant against launch_dequant_patch_metalog
    Wr = torch.empty((N, K), dtype=torch.float16, device="cuda")
    lib.launch_dequant_patch_metalog(_p(T["q"]), _p(T["lut"]), _p(Wr), _p(T["off"]), _p(T["cols"]), _p(T["vals"]),
                                     i(N), i(K), i(4), i(L.wpr), i(nc), i(512), stream)
    Wm = torch.empty_like(Wr)
    C().dequant_w0(T["q"], T["lut"], Wm, N, K, 4, L.wpr, T["off"], T["cols"], T["vals"])
    torch.cuda.synchronize()
    assert torch.equal(Wr.view(torch.int16), Wm.view(torch.int16))
    del Wm
    ws = torch.zeros(32 * N, dtype=torch.float32, device="cuda")
    W = L.dense()
    for M in Ms:
        x, h = inputs(rng, L, M, torch.float16)
        ref = torch.empty((M, N), dtype=torch.float16, device="cuda")
        if M == 1:
            lib.launch_gemv_chunk_csr(_p(T["q"]), _p(T["lut"]), _p(x), _p(ref), _p(ws), _p(T["off"]), _p(T["cols"]),
                                      _p(T["vals"]), _p(T["B"]), _p(h), _p(T["gamma"]), f(L.scale), i(L.r), i(N),
                                      i(K), i(4), i(nc), stream)
        elif M < 16:
            lib.launch_gemm_metalog_dora(_p(x), _p(T["q"]), _p(T["lut"]), _p(ref), _p(T["off"]), _p(T["cols"]),
                                         _p(T["vals"]), _p(h), _p(T["B"]), _p(T["gamma"]), f(L.scale), i(L.r), i(M),
                                         i(N), i(K), i(4), i(L.wpr), i(nc), i(512), stream)
        else:
            torch.mm(x, Wr.t(), out=ref)
            lib.launch_fused_dora_epilogue(_p(ref), _p(h), _p(T["B"]), _p(T["gamma"]), f(L.scale), i(L.r), i(M), i(N),
                                           stream)
        torch.cuda.synchronize()
        y = run_ours(L, T, x, h, gemv=(M == 1))
        oracle = O.forward_f64(W, x.float().cpu().numpy(), h.cpu().numpy(), L.B, L.gamma, L.scale)
        e_ours = rel_err(y.float().cpu().numpy(), oracle)
        e_ref = rel_err(ref.float().cpu().numpy(), oracle)
        e_pair = rel_err(y.float().cpu().numpy(), ref.float().cpu().numpy())
        assert e_ours <= tol and e_ref <= tol and e_pair <= tol, (M, e_ours, e_ref, e_pair)


@pytest.mark.parametrize("N,K", [(256, 1024), (96, 3584), (40, 512)])
def test_against_reference_kernels(N, K):
    """Same inputs through launch_gemv_chunk_csr (M=1), launch_gemm_metalog_dora
    (2<=M<=15) and dequant + cuBLAS + epilogue (M>=16), the reference's three
    paths (csrc/vllm_binding.cpp:253-419); fp16, per-row codebooks."""
    lib = _ref_lib()
    rng = np.random.default_rng(N * K)
    L = make_np_layer(rng, N, K, 0, 0, density=0.01, outliers=True, dora=True)
    _compare_with_reference_kernels(lib, L, (1, 4, 15, 16, 32), rng)


@pytest.mark.parametrize("name,K,N", [("qkv", 3584, 4608), ("o", 3584, 3584), ("gate_up", 3584, 37888),
                                      ("down", 18944, 3584)])
def test_against_reference_kernels_config1(name, K, N):
    """The BASELINE config-1 shapes at full size with per-row codebooks (the
    reference's layout), 0.5% outliers and rank 16: the reference's three
    kernel paths and ours against the oracle at M in {1, 4, 8, 16}."""
    lib = _ref_lib()
    rng = np.random.default_rng(K + N)
    L = make_np_layer(rng, N, K, 0, 0, density=0.005, outliers=True, dora=True)
    _compare_with_reference_kernels(lib, L, (1, 4, 8, 16), rng)


# ------------------------------------------------------------- full sizes

@pytest.mark.parametrize("name", ["qkv", "o", "gate_up", "down"])
def test_full_size_shapes(name):
    """BASELINE config-1 shapes with the benchmark recipe (128-wide codebook
    groups, rank 16, 0.5% outliers) against the oracle: dequantisation
    bit-exact on every row, and the GEMV (h given, and h = A x computed in
    the kernel at every token count 1..32) against the oracle's float64
    forward on 512 sampled rows over the full K."""
    from qwen_wlqfastshot_helen_beta_b200 import synthetic as S
    K, N = S.QWEN25_7B[name]
    L = S.make_layer(N, K, group_size=128, density=0.005, r=16, seed=11)
    W = torch.empty((N, K), dtype=torch.float16, device="cuda")
    C().dequant_w0(L.q_packed, L.lut_c, W, N, K, 4, L.words_per_row, L.chunk_offsets, L.chunk_cols, L.chunk_vals,
                   128, 0)
    W_ref = O.dequant(L.q_packed.cpu().numpy(), L.words_per_row, L.lut_c.cpu().numpy(), N, K, 4, 128, 0,
                      L.chunk_offsets.cpu().numpy(), L.chunk_cols.cpu().numpy(), L.chunk_vals.cpu().numpy())
    assert np.array_equal(W.cpu().numpy().view(np.uint16), W_ref.view(np.uint16))
    del W
    rows = np.sort(np.random.default_rng(1).choice(N, size=512, replace=False))
    W_rows = np.ascontiguousarray(W_ref[rows])
    del W_ref
    A64 = L.lora_A.float().cpu().numpy().astype(np.float64)
    B_rows = L.lora_B.cpu().numpy()[rows]
    g_rows = L.dora_gamma.cpu().numpy()[rows]
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    for M in (1, 16):  # h given (computed on the GPU, fp32)
        x = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
        h = S.lora_h(L, x)
        y = S.forward(L, x, h=h)
        ref = O.forward_f64(W_rows, x.float().cpu().numpy(), h.cpu().numpy(), B_rows, g_rows, L.lora_scale)
        e = rel_err(y.float().cpu().numpy()[:, rows], ref)
        assert e <= 2e-2, (name, M, e)
    # the GEMV computing h = A x itself (the decode path apply() takes), every token count
    L.prepack(torch.bfloat16)
    for M in range(1, 33):
        x = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
        y = S.forward_fold(L, x)
        xf = x.float().cpu().numpy()
        h64 = xf.astype(np.float64) @ A64.T
        ref = O.forward_f64(W_rows, xf, h64, B_rows, g_rows, L.lora_scale)
        e = rel_err(y.float().cpu().numpy()[:, rows], ref)
        assert e <= 2e-2, (name, M, "h in the kernel", e)


# ------------------------------------------------------ torch op surface

def test_custom_ops_opcheck_and_graph_capture():
    import qwen_wlqfastshot_helen_beta_b200  # noqa: F401  (registers the ops)
    rng = np.random.default_rng(4)
    L = make_np_layer(rng, 128, 512, 0, 0, density=0.01)
    T = dev_layer(L)
    x, h = inputs(rng, L, 1, torch.float16)
    out = torch.empty((1, L.N), dtype=torch.float16, device="cuda")
    args = (T["q"], T["lut"], x.squeeze(0), out.squeeze(0), L.N, L.K, 4, T["off"], T["cols"], T["vals"], T["B"],
            h.squeeze(0), T["gamma"], L.scale)
    torch.library.opcheck(torch.ops.wlq_fastShot.gemv.default, args)
    X, H = inputs(rng, L, 8, torch.float16)
    out8 = torch.empty((8, L.N), dtype=torch.float16, device="cuda")
    gargs = (X, T["q"], T["lut"], out8, L.N, L.K, 4, L.wpr, T["off"], T["cols"], T["vals"], H, T["B"], T["gamma"],
             L.scale)
    torch.library.opcheck(torch.ops.wlq_fastShot.gemm.default, gargs)
    # capture both ops in one CUDA graph and replay with new inputs
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            torch.ops.wlq_fastShot.gemv(*args)
            torch.ops.wlq_fastShot.gemm(*gargs)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        torch.ops.wlq_fastShot.gemv(*args)
        torch.ops.wlq_fastShot.gemm(*gargs)
    x2, h2 = inputs(rng, L, 1, torch.float16)
    X2, H2 = inputs(rng, L, 8, torch.float16)
    x.copy_(x2)
    h.copy_(h2)
    X.copy_(X2)
    H.copy_(H2)
    graph.replay()
    torch.cuda.synchronize()
    e1 = run_ours(L, T, x, h, gemv=True)
    e8 = run_ours(L, T, X, H)
    assert torch.equal(out, e1) and torch.equal(out8, e8)


def test_errors_are_raised():
    rng = np.random.default_rng(2)
    L = make_np_layer(rng, 32, 256, 0, 0)
    T = dev_layer(L)
    x, h = inputs(rng, L, 2, torch.float16)
    out = torch.empty((2, 32), dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="4-bit"):
        C().gemm_forward(x, T["q"], T["lut"], out, 32, 256, 3, 28, None, None, None)
    with pytest.raises(RuntimeError, match="dtype"):
        C().gemm_forward(x, T["q"], T["lut"], out.to(torch.bfloat16), 32, 256, 4, L.wpr, None, None, None)
    with pytest.raises(RuntimeError, match="float16 or bfloat16"):
        C().gemm_forward(x.float(), T["q"], T["lut"], out.float(), 32, 256, 4, L.wpr, None, None, None)
    with pytest.raises(RuntimeError, match="lut_c"):
        C().gemm_forward(x, T["q"], T["lut"][:16], out, 32, 256, 4, L.wpr, None, None, None)
    with pytest.raises(RuntimeError, match="multiple of 32"):
        C().gemm_forward(x, T["q"], torch.zeros(32 * 3 * 16, dtype=torch.float16, device="cuda"), out, 32, 256, 4,
                         L.wpr, None, None, None, lut_group_size=128, lut_group_offset=16)


def test_prepack_outlier_records():
    """wlq_prepack_outliers: per entry a record (global column | outlier value
    in the MMA type << 16) and the correction outlier - codebook value; rows
    reordered by ascending column, also when a chunk lists its entries in
    reverse."""
    rng = np.random.default_rng(31)
    N, K, G, goff = 24, 1500, 128, 64
    L = make_np_layer(rng, N, K, G, goff, density=0.03)
    cols_rev, vals_rev = L.cols.copy(), L.vals.copy()  # every chunk reversed: still a valid chunk-CSR
    for r in range(N):
        for c in range(L.off.shape[1] - 1):
            a, b = L.off[r, c], L.off[r, c + 1]
            cols_rev[a:b] = L.cols[a:b][::-1]
            vals_rev[a:b] = L.vals[a:b][::-1]
    Wcb = O.dequant(L.q, L.wpr, L.lut, N, K, 4, G, goff)  # codebook values, no outliers
    d = "cuda"
    q = torch.from_numpy(L.q.view(np.int32)).to(d)
    lut = torch.from_numpy(np.ascontiguousarray(L.lut)).to(d)
    off = torch.from_numpy(L.off).to(d)
    for dtype in (torch.float16, torch.bfloat16):
        for cols, vals in ((L.cols, L.vals), (cols_rev, vals_rev)):
            rec, delta = C().prepack_outliers(q, lut, off, torch.from_numpy(cols.astype(np.uint16)).to(d),
                                              torch.from_numpy(vals).to(d), N, K, 4, dtype, G, goff)
            rec = rec.cpu().numpy().view(np.uint32)
            delta = delta.cpu().numpy()
            for r in range(N):
                a, b = L.off[r, 0], L.off[r, -1]
                gcol = (rec[a:b] & 0xFFFF).astype(np.int64)
                chunk = np.repeat(np.arange(L.off.shape[1] - 1), np.diff(L.off[r]))
                ref_cols = chunk * 512 + L.cols[a:b].astype(np.int64)
                order = np.argsort(ref_cols, kind="stable")
                assert np.array_equal(gcol, ref_cols[order]), r  # ascending, same set
                ov = torch.from_numpy(O.fp8_bytes_to_fp16(L.vals[a:b][order])).to(dtype)
                vbits = ov.view(torch.int16).numpy().view(np.uint16).astype(np.uint32)
                assert np.array_equal(rec[a:b] >> 16, vbits), r
                cb = torch.from_numpy(Wcb[r, gcol]).to(dtype).float().numpy()
                assert np.array_equal(delta[a:b], ov.float().numpy() - cb), r


def test_gemv_overlap_opt_in_matches_plain_launches():
    """wlq_gemv_set_overlap: off by default; with it on, consecutive GEMV
    launches (programmatic dependent launches, weights read before the
    previous kernel completes) give bit-identical outputs to plain launches,
    for a chain where each call's input is the previous call's output, with
    4-warp CTAs (1 and 2 tokens) and 16-warp CTAs (9 and 16 tokens on an
    unsplit K of 1440, a ragged last chunk).  The weights are written and the device
    synchronised before the overlapping calls, as the contract asks."""
    from qwen_wlqfastshot_helen_beta_b200 import _lib
    lib = _lib.lib
    assert lib.wlq_gemv_get_overlap() == 0
    dtype = torch.bfloat16
    rng = np.random.default_rng(77)
    K = 1440
    layers = []
    for N in (K, K, 80):
        L = make_np_layer(rng, N, K, 128, 0, density=0.01, r=16)
        T = dev_layer(L)
        lut = C().prepack_lut(T["lut"], dtype)
        cols, vals = C().prepack_outliers(T["q"], T["lut"], T["off"], T["cols"], T["vals"], N, K, 4, dtype, 128, 0)
        layers.append((L, T, lut, cols, vals, T["A"].to(dtype).contiguous()))
    torch.cuda.synchronize()

    def chain(M):
        x = torch.from_numpy(np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)).to("cuda", dtype)
        outs, warps = [], []
        for L, T, lut, cols, vals, A in layers:
            y = torch.empty((M, L.N), dtype=dtype, device="cuda")
            C().gemv_lora_a(T["q"], lut, x, y, L.N, L.K, 4, T["off"], cols, vals, T["B"], A, T["gamma"], L.scale, 128, 0)
            warps.append(lib.wlq_gemv_last_warps())
            outs.append(y)
            if L.N == K:
                x = y  # the next call reads this call's output
        torch.cuda.synchronize()
        return [o.cpu() for o in outs], warps

    _lib.check(lib.wlq_gemv_set_split(1), "wlq_gemv_set_split")
    try:
        shapes = set()
        for M in (1, 2, 9, 16):
            plain, wp = chain(M)
            _lib.check(lib.wlq_gemv_set_overlap(1), "wlq_gemv_set_overlap")
            try:
                assert lib.wlq_gemv_get_overlap() == 1
                over, wo = chain(M)
            finally:
                _lib.check(lib.wlq_gemv_set_overlap(0), "wlq_gemv_set_overlap")
            assert wp == wo, (M, wp, wo)
            shapes.update(wp)
            for a, b in zip(plain, over):
                assert torch.isfinite(a.float()).all()
                assert torch.equal(a, b), M
        assert shapes == {4, 16}, shapes
    finally:
        _lib.check(lib.wlq_gemv_set_split(0), "wlq_gemv_set_split")
    with pytest.raises(RuntimeError, match="0 or 1"):
        _lib.check(lib.wlq_gemv_set_overlap(2), "wlq_gemv_set_overlap")
