"""The C oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py).  CPU only."""
import numpy as np
import pytest

from oracle import oracle as O


def _cases(g, prefix):
    return sorted({k.split("_")[0] for k in g if k.startswith(prefix)})


def test_unpack_pack_repack(golden_codecs):
    g = golden_codecs
    for c in _cases(g, "pack"):
        N, K, bits, wpr = (int(v) for v in g[f"{c}_meta"])
        words = g[f"{c}_words"]
        idx = O.unpack_continuous(words, N, K, bits)
        assert np.array_equal(idx, g[f"{c}_idx"]), c
        packed, wpr2 = O.pack_row_aligned(idx, bits)
        assert wpr2 == wpr and np.array_equal(packed, g[f"{c}_aligned"]), c
        rep, wpr3 = O.repack_row_aligned(words, N, K, bits)
        assert wpr3 == wpr and np.array_equal(rep, g[f"{c}_aligned"]), c
        assert np.array_equal(O.unpack_row_aligned(packed, N, K, bits), idx), c
        assert wpr % 4 == 0


def test_build_chunk_csr(golden_codecs):
    g = golden_codecs
    for c in _cases(g, "csr"):
        N, K, chunk_m = (int(v) for v in g[f"{c}_meta"])
        off, cols = O.build_chunk_csr(g[f"{c}_mask"], chunk_m)
        assert np.array_equal(off, g[f"{c}_offsets"]), c
        assert np.array_equal(cols, g[f"{c}_cols"]), c
        assert np.array_equal(O.fp16_to_fp8_bytes(g[f"{c}_vals_f16"]), g[f"{c}_vals_u8"]), c


def test_fp16_to_fp8_edges(golden_codecs):
    g = golden_codecs
    got = O.fp16_to_fp8_bytes(g["fp8_in_u16"].view(np.float16))
    assert np.array_equal(got, g["fp8_out_u8"])


def test_elias_fano(golden_codecs):
    g = golden_codecs
    for c in _cases(g, "ef"):
        H, W, tile = (int(v) for v in g[f"{c}_meta"])
        meta, bs, ref = g[f"{c}_tile_meta"], g[f"{c}_bitstream"], g[f"{c}_mask"]
        assert np.array_equal(O.decode_ef_mask(meta, bs, H, W, tile), ref), c
        for chunk_m in (512, 640, 64):
            off, cols = O.decode_ef_to_chunk_csr(meta, bs, H, W, tile, chunk_m)
            off2, cols2 = O.build_chunk_csr(ref, chunk_m)
            assert np.array_equal(off, off2) and np.array_equal(cols, cols2), (c, chunk_m)


def test_tp_outlier_slicing(golden_codecs):
    g = golden_codecs
    mask, vals = g["tp_mask"], g["tp_vals"]
    pos = np.flatnonzero(mask.reshape(-1))
    r0, r1 = 4, 9
    keep = (pos // mask.shape[1] >= r0) & (pos // mask.shape[1] < r1)
    assert np.array_equal(mask[r0:r1], g["tp_row_mask"]) and np.array_equal(vals[keep], g["tp_row_vals"])
    c0, c1 = 10, 30
    keep = (pos % mask.shape[1] >= c0) & (pos % mask.shape[1] < c1)
    assert np.array_equal(mask[:, c0:c1], g["tp_col_mask"]) and np.array_equal(vals[keep], g["tp_col_vals"])


def _layer_names(g):
    return sorted({k.split("__")[0] for k in g if "__" in k})


def test_layer_dequant_and_forward(golden_layers):
    g = golden_layers
    for name in _layer_names(g):
        p = name + "__"
        lut = g[p + "lut"]
        N, K = g[p + "W"].shape
        wpr = int(g[p + "wpr"][0])
        W = O.dequant(g[p + "q_aligned"], wpr, lut, N, K, 4, 0, 0,
                      g[p + "offsets"], g[p + "cols"], g[p + "vals"])
        assert np.array_equal(W.view(np.uint16), g[p + "W"].view(np.uint16)), name
        x16 = g[p + "x"].astype(np.float16).astype(np.float32)
        if int(g[p + "has_dora"][0]):
            y = O.forward_f64(W, x16, g[p + "h"], g[p + "lora_B"], g[p + "gamma"], float(g[p + "scale"][0]))
        else:
            y = O.forward_f64(W, x16)
        ref = g[p + "y"]
        assert np.max(np.abs(y - ref)) <= 1e-9 * max(1.0, np.max(np.abs(ref))), name


def test_layer_gamma(golden_layers):
    """gamma = m / ||W + s B A||_row against the reference's torch computation
    (fp16 result; one ulp of slack for the fp32 norm's summation order)."""
    g = golden_layers
    checked = 0
    for name in _layer_names(g):
        p = name + "__"
        if not int(g[p + "has_dora"][0]):
            continue
        K_full, K_part, tp, rank, row_par, r, M, nsh = (int(v) for v in g[p + "meta"])
        A = g[p + "lora_A_f16"].astype(np.float32)  # gamma was computed from the fp32 A/B before the fp16 cast
        ms = [g.get(f"{p}in{i}_m") for i in range(nsh)]
        m_vec = None
        if all(m is not None for m in ms):
            if row_par or tp == 1:
                m_vec = np.concatenate(ms)
            else:
                m_vec = np.concatenate([m.reshape(-1)[rank * (m.size // tp):(rank + 1) * (m.size // tp)] for m in ms])
        As = [g[f"{p}in{i}_lora_A"] for i in range(nsh)]
        Bs = [g[f"{p}in{i}_lora_B"] for i in range(nsh)]
        if row_par and tp > 1:
            As = [a[:, rank * K_part:(rank + 1) * K_part] for a in As]
        if not row_par and tp > 1:
            Bs = [b[rank * (b.shape[0] // tp):(rank + 1) * (b.shape[0] // tp)] for b in Bs]
        A32 = np.concatenate(As, 0)
        Bf = np.zeros((sum(b.shape[0] for b in Bs), sum(b.shape[1] for b in Bs)), np.float32)
        ro = co = 0
        for b in Bs:
            Bf[ro:ro + b.shape[0], co:co + b.shape[1]] = b
            ro += b.shape[0]
            co += b.shape[1]
        gam = O.dora_gamma(g[p + "W"], A32, Bf, float(g[p + "scale"][0]), m_vec)
        ref = g[p + "gamma"]
        ulps = np.abs(gam.view(np.int16).astype(np.int32) - ref.view(np.int16).astype(np.int32))
        assert ulps.max() <= 1, (name, ulps.max())
        assert np.array_equal(A, g[p + "lora_A_f16"].astype(np.float32))
        checked += 1
    assert checked >= 4
