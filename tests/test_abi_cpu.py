"""The C ABI library on the CPU: it loads, exports exactly what
include/wlq_b200.h declares, validates arguments without touching a GPU, and
its load-time codecs match the reference's golden vectors."""
import os
import re

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_functions():
    src = open(os.path.join(ROOT, "include", "wlq_b200.h")).read()
    return sorted(set(re.findall(r"WLQ_API\s+[\w\s\*]+?\b(wlq_\w+)\s*\(", src)))


def test_library_exports_header():
    from qwen_wlqfastshot_helen_beta_b200 import _lib
    declared = _header_functions()
    assert len(declared) >= 15
    for name in declared:
        assert hasattr(_lib.lib, name), name
    assert sorted(_lib.SIGNATURES) == declared
    assert _lib.lib.wlq_abi_version() == 1


def test_library_export_table_is_exactly_the_abi():
    import subprocess
    from qwen_wlqfastshot_helen_beta_b200 import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = sorted(l.split()[-1] for l in out.splitlines() if l.strip())
    assert exported == _header_functions()


def test_argument_validation_without_gpu():
    import ctypes
    from qwen_wlqfastshot_helen_beta_b200._lib import lib
    p = ctypes.c_void_p(16)
    # argument order: ..., r, M, N, K, bits, words_per_row, group_size, group_offset, lut_format, act_dtype, stream
    # bits != 4 is rejected before any device call
    rc = lib.wlq_gemv(p, p, p, p, None, None, None, None, None, None, 1.0, 0, 1, 8, 64, 3, 4, 0, 0, 0, 0, None)
    assert rc == 2 and b"4-bit" in lib.wlq_last_error()
    # wrong words_per_row
    rc = lib.wlq_gemm(p, p, p, p, None, None, None, None, None, None, 1.0, 0, 32, 8, 64, 4, 7, 0, 0, 0, 0, None)
    assert rc == 1 and b"words_per_row" in lib.wlq_last_error()
    # unknown dtype / codebook format
    rc = lib.wlq_gemm(p, p, p, p, None, None, None, None, None, None, 1.0, 0, 32, 8, 64, 4, 8, 0, 0, 0, 7, None)
    assert rc == 2
    rc = lib.wlq_gemm(p, p, p, p, None, None, None, None, None, None, 1.0, 0, 32, 8, 64, 4, 8, 0, 0, 5, 0, None)
    assert rc == 1 and b"lut_format" in lib.wlq_last_error()
    # misaligned q
    rc = lib.wlq_gemv(ctypes.c_void_p(18), p, p, p, None, None, None, None, None, None, 1.0, 0, 1, 8, 64, 4, 8, 0, 0,
                      0, 0, None)
    assert rc == 3
    # empty problem is a no-op success
    assert lib.wlq_gemv(None, None, None, None, None, None, None, None, None, None, 1.0, 0, 0, 0, 0, 4, 0, 0, 0, 0,
                        0, None) == 0
    assert lib.wlq_init_workspaces(-1, 4, 0) == 1
    assert lib.wlq_init_workspaces(4096, 4096, 0) == 0
    assert lib.wlq_words_per_row(3584, 4) == 448 and lib.wlq_words_per_row(18944, 4) == 2368
    assert lib.wlq_words_per_row(37, 4) == 8 and lib.wlq_words_per_row(50, 3) == 8
    # prepacking: overlapping buffers and bad dtypes are refused
    buf = ctypes.create_string_buffer(64 + 16)
    base = (ctypes.addressof(buf) + 15) // 16 * 16
    assert lib.wlq_prepack_lut(ctypes.c_void_p(base), ctypes.c_void_p(base), 1, 0, None) == 1
    assert lib.wlq_prepack_lut_host(ctypes.c_void_p(base), ctypes.c_void_p(base + 32), 1, 9) == 1


def test_prepack_host_layout():
    """Prepacked codebook = entries in the MMA type, low bytes then high bytes."""
    from qwen_wlqfastshot_helen_beta_b200 import _C
    from oracle import oracle as O
    rng = np.random.default_rng(8)
    lut = (rng.standard_normal((5, 3, 16)) * 0.03).astype(np.float16)
    lut[0, 0, :4] = np.array([0.0, -0.0, 6e-5, 65504], np.float16)
    for dt in (torch.float16, torch.bfloat16):
        pk = _C.prepack_lut(torch.from_numpy(lut), dt).numpy().view(np.uint8).reshape(-1, 32)
        flat = lut.reshape(-1, 16)
        if dt == torch.float16:
            vals = flat.view(np.uint16)
        else:
            vals = np.array([[O.lib().orc_f32_to_bf16(float(v)) for v in row] for row in flat.astype(np.float32)],
                            np.uint16)
        assert np.array_equal(pk[:, :16], (vals & 0xFF).astype(np.uint8))
        assert np.array_equal(pk[:, 16:], (vals >> 8).astype(np.uint8))


def test_codecs_repack_against_golden(golden_codecs):
    from qwen_wlqfastshot_helen_beta_b200 import _C
    g = golden_codecs
    for c in sorted({k.split("_")[0] for k in g if k.startswith("pack")}):
        N, K, bits, wpr = (int(v) for v in g[f"{c}_meta"])
        q, w = _C.repack_q_indices_row_aligned(torch.from_numpy(g[f"{c}_words"].view(np.int32)), N, K, bits)
        assert w == wpr
        assert np.array_equal(q.numpy().view(np.uint32), g[f"{c}_aligned"]), c


def test_codecs_slice_matches_unpack_slice_pack(golden_codecs):
    from oracle import oracle as O
    from qwen_wlqfastshot_helen_beta_b200 import _C
    g = golden_codecs
    for c in sorted({k.split("_")[0] for k in g if k.startswith("pack")}):
        N, K, bits, wpr = (int(v) for v in g[f"{c}_meta"])
        idx = g[f"{c}_idx"]
        for (r0, r1, c0, c1) in [(0, N, 0, K), (1, N, 0, K), (0, N, K // 3, K - 1), (N // 2, N, 5, K // 2 + 5)]:
            if r1 <= r0 or c1 <= c0:
                continue
            q, w = _C.repack_q_indices_slice(torch.from_numpy(g[f"{c}_words"].view(np.int32)), N, K, bits, r0, r1,
                                             c0, c1)
            ref, wref = O.pack_row_aligned(idx[r0:r1, c0:c1], bits)
            assert w == wref and np.array_equal(q.numpy().view(np.uint32), ref), (c, r0, r1, c0, c1)


def test_codecs_csr_and_fp8_against_golden(golden_codecs):
    from qwen_wlqfastshot_helen_beta_b200 import _C
    g = golden_codecs
    for c in sorted({k.split("_")[0] for k in g if k.startswith("csr")}):
        N, K, chunk_m = (int(v) for v in g[f"{c}_meta"])
        off, cols = _C.build_chunk_csr_from_mask(g[f"{c}_mask"], chunk_m)
        assert np.array_equal(off.numpy(), g[f"{c}_offsets"]) and np.array_equal(cols.numpy(), g[f"{c}_cols"]), c
        pos = np.flatnonzero(g[f"{c}_mask"].reshape(-1))
        off2, cols2 = _C.positions_to_chunk_csr(pos, N, K, chunk_m)
        assert np.array_equal(off2.numpy(), g[f"{c}_offsets"]) and np.array_equal(cols2.numpy(), g[f"{c}_cols"])
        v8 = _C.fp16_to_fp8_bytes(torch.from_numpy(g[f"{c}_vals_f16"]))
        assert np.array_equal(v8.numpy(), g[f"{c}_vals_u8"]), c
    v8 = _C.fp16_to_fp8_bytes(torch.from_numpy(g["fp8_in_u16"].view(np.float16)))
    assert np.array_equal(v8.numpy(), g["fp8_out_u8"])


def test_codecs_elias_fano_against_golden(golden_codecs):
    from oracle import oracle as O
    from qwen_wlqfastshot_helen_beta_b200 import _C
    g = golden_codecs
    for c in sorted({k.split("_")[0] for k in g if k.startswith("ef")}):
        H, W, tile = (int(v) for v in g[f"{c}_meta"])
        meta = torch.from_numpy(g[f"{c}_tile_meta"])
        bs = torch.from_numpy(g[f"{c}_bitstream"].view(np.int32))
        ref = g[f"{c}_mask"]
        pos = _C.decode_ef_positions(meta, bs, H, W, tile)
        assert np.array_equal(pos, np.flatnonzero(ref.reshape(-1))), c
        for chunk_m in (512, 640, 64):
            off, cols = _C.decode_ef_to_chunk_csr(meta, bs, H, W, tile, chunk_m)
            off2, cols2 = O.build_chunk_csr(ref, chunk_m)
            assert np.array_equal(off.numpy(), off2) and np.array_equal(cols.numpy(), cols2), (c, chunk_m)


def test_host_dequant_against_golden(golden_layers):
    from qwen_wlqfastshot_helen_beta_b200 import _C
    g = golden_layers
    for name in sorted({k.split("__")[0] for k in g if "__" in k}):
        p = name + "__"
        N, K = g[p + "W"].shape
        W = torch.empty((N, K), dtype=torch.float16)
        _C.dequant_w0(torch.from_numpy(g[p + "q_aligned"]), torch.from_numpy(g[p + "lut"]), W, N, K, 4,
                      int(g[p + "wpr"][0]), torch.from_numpy(g[p + "offsets"]),
                      torch.from_numpy(g[p + "cols"]), torch.from_numpy(g[p + "vals"]))
        assert np.array_equal(W.numpy().view(np.uint16), g[p + "W"].view(np.uint16)), name


def test_host_dequant_grouped_against_oracle():
    from oracle import oracle as O
    from qwen_wlqfastshot_helen_beta_b200 import _C
    rng = np.random.default_rng(5)
    for (N, K, G, goff) in [(7, 300, 128, 0), (5, 448, 128, 64), (3, 1000, 64, 32), (4, 97, 32, 0)]:
        idx = rng.integers(0, 16, size=(N, K), dtype=np.uint8)
        q, wpr = O.pack_row_aligned(idx, 4)
        ng = -(-(K + goff) // G)
        lut = rng.standard_normal((N, ng, 16)).astype(np.float16)
        mask = rng.random((N, K)) < 0.03
        off, cols = O.build_chunk_csr(mask, 512)
        vals = rng.integers(0, 256, size=cols.size, dtype=np.uint8)
        ref = O.dequant(q, wpr, lut, N, K, 4, G, goff, off, cols, vals)
        W = torch.empty((N, K), dtype=torch.float16)
        _C.dequant_w0(torch.from_numpy(q.view(np.int32)), torch.from_numpy(lut), W, N, K, 4, wpr,
                      torch.from_numpy(off), torch.from_numpy(cols), torch.from_numpy(vals), G, goff)
        assert np.array_equal(W.numpy().view(np.uint16), ref.view(np.uint16)), (N, K, G, goff)


def test_tp_buffer_bytes_hold_the_packed_slots():
    """wlq_tp_buffer_bytes: an error word, one call counter per 16-row tile,
    then per parity, source rank and token a row of 8-byte words holding
    every tile's eight words (two 16-bit values and a 32-bit epoch each, two
    words per 16-byte store): the row is even and at least 8 words per tile,
    also for widths below 16 rows."""
    from qwen_wlqfastshot_helen_beta_b200 import _lib

    def up(v, a):
        return (v + a - 1) // a * a

    for world in (2, 4, 8):
        for max_N in (1, 3, 15, 16, 17, 100, 256, 3584, 18944, 37888):
            tiles = (max_N + 15) // 16
            stride = up(max(max_N, 8 * tiles), 2)
            data = up(128 + 4 * tiles, 256)
            want = up(data + 2 * world * 16 * stride * 8, 256)
            got = int(_lib.lib.wlq_tp_buffer_bytes(world, max_N))
            assert got == want, (world, max_N, got, want)
            # the last word of the last tile of the last row lies inside
            last = data + 8 * ((2 * world * 16 - 1) * stride + tiles * 8 - 1)
            assert last + 8 <= got
