"""Parity of the tensor-core prefill GEMM (wlq_gemm, M > 16) with the oracle:
per-row and per-group codebooks (steps spanning one or two groups), both
codebook/outlier layouts, ragged M / N / K, rows dense with outliers, the
low-rank term folded in as extra K steps, and the shapes that fall back to
16-token GEMV slices.  B200 only."""
import numpy as np
import pytest
import torch

from _gpu import C, dev_layer, inputs, run_ours
from _layers import make_np_layer, reference_output, rel_err
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 5e-3, torch.bfloat16: 2e-2}  # normwise max relative error


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "the gpu tests need a CUDA device"
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    assert C().device_error() == 0  # no bounded wait ran out in this module


GEMM_CASES = [
    # N, K, G, goff, outliers, dora
    (128, 1024, 0, 0, True, True),     # per-row codebooks, one N tile
    (300, 1536, 128, 0, True, True),   # N not a multiple of 8 (scalar stores), 128-wide groups
    (256, 1088, 128, 64, True, True),  # shard starting mid-group: steps span two groups
    (130, 1024, 32, 0, True, False),   # 32-wide groups: two groups per step
    (200, 2048, 64, 32, True, True),   # 64-wide groups offset by 32
    (96, 1096, 0, 0, True, True),      # K not a multiple of 64: ragged last step
    (64, 512, 128, 0, False, False),   # no outliers, no low-rank term
    (40, 203, 0, 0, True, True),       # K % 8 != 0: 16-token GEMV slices
]


@pytest.mark.parametrize("case", GEMM_CASES, ids=lambda c: f"N{c[0]}K{c[1]}G{c[2]}o{c[3]}")
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_gemm_matches_oracle(case, dtype):
    N, K, G, goff, outl, dora = case
    rng = np.random.default_rng(7 * N + K + G)
    L = make_np_layer(rng, N, K, G, goff, density=0.02, outliers=outl, dora=dora)
    T = dev_layer(L)
    for M in (17, 24, 32, 128, 200, 300):
        x, h = inputs(rng, L, M, dtype)
        ref = reference_output(L, x.float().cpu().numpy(), None if h is None else h.cpu().numpy())
        ys = []
        for fmt in (0, 1):  # up to 32 tokens the prepacked layout runs on the GEMV-class kernel
            y = run_ours(L, T, x, h, fmt=fmt)
            assert torch.isfinite(y).all(), (M, fmt)
            e = rel_err(y.float().cpu().numpy(), ref)
            assert e <= TOL[dtype], (M, fmt, e)
            ys.append(y.float())
        if M > 32:  # the two layouts patch the same outlier values into the tile
            assert rel_err(ys[1].cpu().numpy(), ys[0].cpu().numpy()) <= 1e-3, M


def test_gemm_outlier_edges():
    """Outliers at the first and last column, a row made only of outliers
    (more per chunk than the per-thread window), a run across a step
    boundary, and rows without any; two N tiles, M spanning two accumulators."""
    rng = np.random.default_rng(78)
    N, K = 160, 1096
    L = make_np_layer(rng, N, K, 128, 0, outliers=False, dora=True)
    mask = np.zeros((N, K), bool)
    mask[0, 0] = mask[0, K - 1] = True
    mask[1, 1024:] = True
    mask[2, :] = True
    mask[5, 60:70] = True
    mask[129, 500:530] = True
    mask[150:160, ::97] = True
    L.off, L.cols = O.build_chunk_csr(mask, 512)
    L.vals = O.fp16_to_fp8_bytes((rng.standard_normal(L.cols.size) * 0.1).astype(np.float16))
    T = dev_layer(L)
    for M in (33, 257):
        for dtype in (torch.float16, torch.bfloat16):
            x, h = inputs(rng, L, M, dtype)
            ref = reference_output(L, x.float().cpu().numpy(), h.cpu().numpy())
            for fmt in (0, 1):
                y = run_ours(L, T, x, h, fmt=fmt)
                assert rel_err(y.float().cpu().numpy(), ref) <= TOL[dtype], (M, dtype, fmt)


def test_gemm_rank_above_one_step():
    """A low-rank term of rank 80 takes two extra K steps."""
    rng = np.random.default_rng(5)
    L = make_np_layer(rng, 128, 512, 128, 0, density=0.01, r=80)
    T = dev_layer(L)
    x, h = inputs(rng, L, 150, torch.float16)
    ref = reference_output(L, x.float().cpu().numpy(), h.cpu().numpy())
    y = run_ours(L, T, x, h)
    assert rel_err(y.float().cpu().numpy(), ref) <= TOL[torch.float16]


def _oracle_rows(L, N, K, rows):
    """Oracle (bit-exact) dequantised weights of the sampled rows, their B
    rows and magnitudes, and A in float64."""
    W = O.dequant(L.q_packed.cpu().numpy(), L.words_per_row, L.lut_c.cpu().numpy(), N, K, 4, 128, 0,
                  L.chunk_offsets.cpu().numpy(), L.chunk_cols.cpu().numpy(), L.chunk_vals.cpu().numpy())
    return (np.ascontiguousarray(W[rows]), L.lora_B.cpu().numpy()[rows], L.dora_gamma.cpu().numpy()[rows],
            L.lora_A.float().cpu().numpy().astype(np.float64))


@pytest.mark.parametrize("name,M", [("qkv", 512), ("o", 2048), ("down", 512)])
def test_gemm_full_size_shapes(name, M):
    """BASELINE config-2 shapes with the benchmark recipe against the
    oracle's float64 forward on 128 sampled rows x 64 sampled tokens over the
    full K (h given, and h from wlq_lora_h as the prefill op runs it)."""
    from qwen_wlqfastshot_helen_beta_b200 import synthetic as S
    K, N = S.QWEN25_7B[name]
    L = S.make_layer(N, K, group_size=128, density=0.005, r=16, seed=12)
    rng = np.random.default_rng(5)
    rows = np.sort(rng.choice(N, size=128, replace=False))
    toks = np.sort(rng.choice(M, size=64, replace=False))
    W_rows, B_rows, g_rows, _ = _oracle_rows(L, N, K, rows)
    g = torch.Generator(device="cuda")
    g.manual_seed(4)
    x = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
    h = S.lora_h(L, x)
    y = S.forward(L, x, h=h)
    ref = O.forward_f64(W_rows, x.float().cpu().numpy()[toks], h.cpu().numpy()[toks], B_rows, g_rows, L.lora_scale)
    e = rel_err(y.float().cpu().numpy()[toks][:, rows], ref)
    assert e <= 2e-2, (name, M, e)


@pytest.mark.parametrize("name,M", [("qkv", 24), ("o", 32), ("down", 32), ("gate_up", 32)])
def test_decode_batch_17_to_32(name, M):
    """Decode batches of 17..32 tokens at BASELINE shapes through wlq_gemm:
    the GEMV-class kernel (four 8-token MMA tiles) where the tensor-core
    GEMM would not fill the device (qkv, o, down), the GEMM otherwise
    (gate_up); against the oracle's float64 forward on 512 sampled rows over
    the full K, h given and h computed in the kernel."""
    from qwen_wlqfastshot_helen_beta_b200 import synthetic as S
    K, N = S.QWEN25_7B[name]
    L = S.make_layer(N, K, group_size=128, density=0.005, r=16, seed=21).prepack(torch.bfloat16)
    rows = np.sort(np.random.default_rng(6).choice(N, size=512, replace=False))
    W_rows, B_rows, g_rows, A64 = _oracle_rows(L, N, K, rows)
    g = torch.Generator(device="cuda")
    g.manual_seed(6)
    x = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
    h = S.lora_h(L, x)
    xf = x.float().cpu().numpy()
    ref_h = O.forward_f64(W_rows, xf, h.cpu().numpy(), B_rows, g_rows, L.lora_scale)
    ref_f = O.forward_f64(W_rows, xf, xf.astype(np.float64) @ A64.T, B_rows, g_rows, L.lora_scale)
    for y, ref in ((S.forward(L, x, h=h), ref_h), (S.forward_fold(L, x), ref_f)):
        e = rel_err(y.float().cpu().numpy()[:, rows], ref)
        assert e <= 2e-2, (name, M, e)


@pytest.mark.parametrize("N,K,M", [(9472, 1024, 512), (4608, 3584, 2048), (3584, 1024, 512)])
def test_gemm_cta_shapes(N, K, M):
    """Problem sizes for which the launcher picks each CTA shape (256 or 128
    tokens x 256 or 128 rows), in bf16 and fp16, against the oracle's
    float64 forward on 128 sampled rows x 64 sampled tokens."""
    from qwen_wlqfastshot_helen_beta_b200 import synthetic as S
    L = S.make_layer(N, K, group_size=128, density=0.005, r=16, seed=N + M)
    rng = np.random.default_rng(N + M)
    rows = np.sort(rng.choice(N, size=128, replace=False))
    toks = np.sort(rng.choice(M, size=64, replace=False))
    W_rows, B_rows, g_rows, _ = _oracle_rows(L, N, K, rows)
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    x = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
    h = S.lora_h(L, x)
    for dt in (torch.bfloat16, torch.float16):
        xx = x.to(dt)
        y = S.forward(L.prepack(dt) if dt != torch.bfloat16 else L, xx, h=h)
        ref = O.forward_f64(W_rows, xx.float().cpu().numpy()[toks], h.cpu().numpy()[toks], B_rows, g_rows,
                            L.lora_scale)
        e = rel_err(y.float().cpu().numpy()[toks][:, rows], ref)
        assert e <= 2e-2, (N, K, M, dt, e)


# ------------------------------------------------------------ stream-K

SK_CASES = [
    # N, K, M, G, r: o/down-like shapes whose tiles do not fill whole waves
    (3584, 3584, 512, 128, 16),    # 28 tiles of 256 x 256: every tile split over several CTAs
    (3584, 18944, 512, 128, 16),   # long K: many steps per CTA, low-rank step in a later segment
    (3584, 3584, 8192, 128, 16),   # 448 tiles: 2 data-parallel waves, then stream-K over the rest
    (1000, 1100, 300, 0, 80),      # ragged N, M and K, per-row codebooks, two low-rank steps
    (4736, 2368, 2048, 128, 16),   # a tensor-parallel shard shape
    (256, 512, 64, 128, 16),       # one tile split over a few CTAs
]


@pytest.mark.parametrize("case", SK_CASES, ids=lambda c: f"N{c[0]}K{c[1]}M{c[2]}G{c[3]}r{c[4]}")
def test_gemm_streamk_matches_oracle(case):
    """wlq_gemm_streamk (the stream-K schedule: partial tiles summed through
    the workspace in CTA order) against the oracle and against the
    data-parallel schedule, on both codebook layouts; repeated calls give the
    same bits (the fix-up order is fixed) and leave the workspace flags zero."""
    from qwen_wlqfastshot_helen_beta_b200 import _C as CC
    N, K, M, G, r = case
    rng = np.random.default_rng(N + K + M)
    L = make_np_layer(rng, N, K, G, 0, density=0.005, r=r)
    T = dev_layer(L)
    dtype = torch.bfloat16
    x, h = inputs(rng, L, M, dtype)
    ref = reference_output(L, x.float().cpu().numpy(), h.cpu().numpy())
    lutp = CC.prepack_lut(T["lut"], dtype)
    colsp, valsp = CC.prepack_outliers(T["q"], T["lut"], T["off"], T["cols"], T["vals"], N, K, 4, dtype, G, 0)
    for lut, cols, vals, fmt in ((lutp, colsp, valsp, 1), (T["lut"], T["cols"], T["vals"], 0)):
        ys = []
        for ws in (True, True, False):
            y = torch.full((M, N), float("nan"), dtype=dtype, device="cuda")
            CC.gemm_forward(x, T["q"], lut, y, N, K, 4, L.wpr, T["off"], cols, vals, h, T["B"], T["gamma"], L.scale,
                            G, 0, fmt, workspace=ws)
            torch.cuda.synchronize()
            assert CC.device_error() == 0
            assert torch.isfinite(y).all(), (fmt, ws)
            e = rel_err(y.float().cpu().numpy(), ref)
            assert e <= 2e-2, (fmt, ws, e)
            ys.append(y)
        assert torch.equal(ys[0], ys[1]), fmt  # deterministic
        assert rel_err(ys[0].float().cpu().numpy(), ys[2].float().cpu().numpy()) <= 1e-2, fmt
    ws = CC.gemm_workspace(torch.device("cuda"))
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert int(ws[:4 * sms].view(torch.int32).abs().sum()) == 0  # flags left zero
