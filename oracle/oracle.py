"""numpy front end of the C oracle (``oracle/wlq_oracle.c``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg, never by the product package.  Each
wrapper names the reference file:line its C function restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "wlq_oracle.c")
LIB = os.path.join(HERE, "_build", "liboracle.so")

_lib = None


def build(force: bool = False) -> str:
    """Compile the C oracle with gcc (no GPU, no CUDA)."""
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        subprocess.check_call(["gcc", "-O2", "-shared", "-fPIC", "-o", LIB, SRC, "-lm"])
    return LIB


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB)
        i64, i32, p = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
        sig = {
            "orc_f16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
            "orc_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
            "orc_f32_to_bf16": (ctypes.c_uint16, [ctypes.c_float]),
            "orc_words_per_row": (i64, [i64, i32]),
            "orc_unpack_continuous": (i32, [p, i64, i64, i64, i32, p]),
            "orc_pack_row_aligned": (None, [p, i64, i64, i32, p]),
            "orc_repack_row_aligned": (None, [p, i64, i64, i64, i32, p]),
            "orc_unpack_row_aligned": (None, [p, i64, i64, i32, i64, p]),
            "orc_fp16_to_fp8_bytes": (None, [p, i64, p]),
            "orc_build_chunk_csr": (i64, [p, i64, i64, i64, p, p]),
            "orc_decode_ef_to_chunk_csr": (i64, [p, i64, p, i64, i64, i64, i64, i64, p, p, i64]),
            "orc_decode_ef_mask": (i32, [p, p, i64, i64, i64, i64, p]),
            "orc_encode_ef": (i64, [p, i64, i64, i64, p, p, i64]),
            "orc_dequant": (None, [p, i64, p, i64, i64, i32, i64, i64, p, p, p, i64, p]),
            "orc_forward_f64": (None, [p, p, i64, i64, i64, p, p, p, i64, ctypes.c_double, p]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return None if a is None else np.ascontiguousarray(a, dtype=dtype)


def symbols_per_word(bits: int) -> int:
    return 10 if bits == 3 else 32 // bits


def words_per_row(K: int, bits: int) -> int:
    """vllm_wlq/linear_method.py:329-330."""
    return int(lib().orc_words_per_row(K, bits))


def unpack_continuous(words, N, K, bits):
    """vllm_wlq/linear_method.py:315-323 -> uint8 [N,K]."""
    w = _c(np.asarray(words).view(np.uint32), np.uint32)
    out = np.empty((N, K), np.uint8)
    rc = lib().orc_unpack_continuous(_p(w), w.size, N, K, bits, _p(out))
    if rc != 0:
        raise ValueError("index stream too short")
    return out


def pack_row_aligned(idx, bits):
    """vllm_wlq/linear_method.py:326-338 -> (uint32 [N*wpr], wpr)."""
    idx = _c(idx, np.uint8)
    N, K = idx.shape
    wpr = words_per_row(K, bits)
    out = np.empty(N * wpr, np.uint32)
    lib().orc_pack_row_aligned(_p(idx), N, K, bits, _p(out))
    return out, wpr


def repack_row_aligned(words, N, K, bits):
    """csrc/vllm_binding.cpp:198-236 -> (uint32 [N*wpr], wpr)."""
    w = _c(np.asarray(words).view(np.uint32), np.uint32)
    wpr = words_per_row(K, bits)
    out = np.empty(N * wpr, np.uint32)
    lib().orc_repack_row_aligned(_p(w), w.size, N, K, bits, _p(out))
    return out, wpr


def unpack_row_aligned(q, N, K, bits, wpr=None):
    """csrc/gemv_kernel.cu:168-189 index read -> uint8 [N,K]."""
    q = _c(np.asarray(q).view(np.uint32), np.uint32)
    wpr = words_per_row(K, bits) if wpr is None else wpr
    out = np.empty((N, K), np.uint8)
    lib().orc_unpack_row_aligned(_p(q), N, K, bits, wpr, _p(out))
    return out


def fp16_to_fp8_bytes(vals_f16):
    """vllm_wlq/linear_method.py:306-308."""
    h = _c(np.asarray(vals_f16, dtype=np.float16).view(np.uint16), np.uint16)
    out = np.empty(h.size, np.uint8)
    lib().orc_fp16_to_fp8_bytes(_p(h), h.size, _p(out))
    return out


def fp8_bytes_to_fp16(vals_u8):
    """csrc/gemv_kernel.cu:273: fp16 bits = u8 << 8."""
    return (np.asarray(vals_u8, np.uint16) << 8).view(np.float16)


def build_chunk_csr(mask, chunk_m):
    """vllm_wlq/linear_method.py:284-312 (offsets, cols) for a bool mask [N,K]."""
    m = _c(mask, np.uint8)
    N, K = m.shape
    nc = (K + chunk_m - 1) // chunk_m
    offsets = np.empty((N, nc + 1), np.int32)
    nnz = int(lib().orc_build_chunk_csr(_p(m), N, K, chunk_m, _p(offsets), None))
    cols = np.empty(nnz, np.uint16)
    lib().orc_build_chunk_csr(_p(m), N, K, chunk_m, _p(offsets), _p(cols))
    return offsets, cols


def decode_ef_to_chunk_csr(meta, bitstream, N, K, tile, chunk_m):
    """csrc/vllm_binding.cpp:94-196 -> (offsets [N,nc+1] int32, cols uint16)."""
    meta = _c(meta, np.int64).reshape(-1, 2)
    bs = _c(np.asarray(bitstream).view(np.uint32), np.uint32)
    nc = (K + chunk_m - 1) // chunk_m
    offsets = np.zeros((N, nc + 1), np.int32)
    cap = int(meta[:, 1].sum()) if meta.size else 0
    cols = np.empty(max(cap, 1), np.uint16)
    kept = int(lib().orc_decode_ef_to_chunk_csr(_p(meta), meta.shape[0], _p(bs), bs.size, N, K, tile,
                                                chunk_m, _p(offsets), _p(cols), cap))
    if kept < 0:
        raise ValueError("EF decode capacity")
    return offsets, cols[:kept].copy()


def decode_ef_mask(meta, bitstream, H, W, tile):
    """vllm_wlq/linear_method.py:243-281 -> bool [H,W]."""
    meta = _c(meta, np.int64).reshape(-1, 2)
    bs = _c(np.asarray(bitstream).view(np.uint32), np.uint32)
    out = np.empty((H, W), np.uint8)
    rc = lib().orc_decode_ef_mask(_p(meta), _p(bs), bs.size, H, W, tile, _p(out))
    if rc != 0:
        raise ValueError("truncated EF stream")
    return out.astype(bool)


def encode_ef(mask, tile):
    """Test-data encoder for the EF layout the decoders read -> (meta int64 [T,2], words uint32)."""
    m = _c(mask, np.uint8)
    H, W = m.shape
    ty = -(-H // tile)
    tx = -(-W // tile)
    meta = np.zeros((ty * tx, 2), np.int64)
    cap = int(m.sum()) * 2 + ty * tx * (tile * tile // 8 + 64) // 32 + 64
    bs = np.zeros(cap, np.uint32)
    used = int(lib().orc_encode_ef(_p(m), H, W, tile, _p(meta), _p(bs), cap))
    if used < 0:
        raise ValueError("EF encode capacity")
    return meta, bs[:max(used, 1)].copy()


def dequant(q, wpr, lut_f16, N, K, bits, group_size=0, group_offset=0,
            offsets=None, cols=None, vals=None, chunk_m=None):
    """csrc/gemm_kernel.cu:322-445 -> fp16 [N,K] (bit-exact)."""
    q = _c(np.asarray(q).view(np.uint32), np.uint32)
    lut = _c(np.asarray(lut_f16, np.float16).view(np.uint16), np.uint16)
    if chunk_m is None:
        chunk_m = 640 if bits == 3 else 512
    W = np.empty((N, K), np.uint16)
    has_outl = offsets is not None and cols is not None and vals is not None and np.asarray(cols).size > 0
    off = _c(offsets, np.int32) if has_outl else None
    cl = _c(cols, np.uint16) if has_outl else None
    vl = _c(vals, np.uint8) if has_outl else None
    lib().orc_dequant(_p(q), wpr, _p(lut), N, K, bits, group_size, group_offset,
                      _p(off), _p(cl), _p(vl), chunk_m, _p(W))
    return W.view(np.float16)


def forward_f64(W_f16, x, h=None, B_f16=None, gamma_f16=None, scale=1.0):
    """y = gamma * (W x + s * B h) in float64 (csrc/gemm_kernel.cu:271-293)."""
    W = _c(np.asarray(W_f16, np.float16).view(np.uint16), np.uint16)
    N, K = W.shape
    x = _c(np.asarray(x, np.float32).reshape(-1, K), np.float32)
    M = x.shape[0]
    dora = h is not None and B_f16 is not None and gamma_f16 is not None
    r = int(np.asarray(B_f16).shape[1]) if dora else 0
    hh = _c(np.asarray(h, np.float32).reshape(M, r), np.float32) if dora else None
    B = _c(np.asarray(B_f16, np.float16).view(np.uint16), np.uint16) if dora else None
    g = _c(np.asarray(gamma_f16, np.float16).view(np.uint16), np.uint16) if dora else None
    y = np.empty((M, N), np.float64)
    lib().orc_forward_f64(_p(W), _p(x), M, N, K, _p(hh), _p(B), _p(g), r, float(scale), _p(y))
    return y


def dora_gamma(W_f16, A, B, scale, m_vec=None):
    """gamma = m / ||W + s B A||_row, m defaulting to ||W||_row, rounded to fp16
    (vllm_wlq/linear_method.py:625-635, 890-897), evaluated in float64."""
    W = np.asarray(W_f16, np.float16).astype(np.float64)
    V = W + float(scale) * (np.asarray(B, np.float64) @ np.asarray(A, np.float64))
    nv = np.maximum(np.linalg.norm(V, axis=1), 1e-12)
    m = np.linalg.norm(W, axis=1) if m_vec is None else np.asarray(m_vec, np.float64).reshape(-1)
    return (m / nv).astype(np.float16)
