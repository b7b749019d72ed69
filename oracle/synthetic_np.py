"""Seeded synthetic WLQ layers built with numpy alone, for the CPU legs of
bench.py (``cpu_baseline``, ``--impl reference`` and the config-0 leg) and
for tests that need a layer without the CUDA library.

TEST / BASELINE INFRASTRUCTURE ONLY.  Nothing here loads a shared library,
so the reference arm of bench.py runs the reference's CPU steps on inputs
made without this repository's product code.

Recipe (applied to any [N, K]):
* W0 ~ N(0, 0.02);
* one codebook of 16 sorted fp16 levels per (row, group of ``group_size``
  columns) -- ``group_size == 0`` gives one per row, the reference's layout
  (vllm_wlq/linear_method.py:482-484) -- with level i =
  std(group) * Phi^-1((i + 0.5) / 16) * (1 + U(-0.05, 0.05));
* indices: the nearest level, packed row-aligned, 8 per int32 word, least
  significant nibble first (vllm_wlq/linear_method.py:326-338);
* outliers: a fraction ``density`` of uniform positions with fp16 values
  ~ N(0, 0.1), stored as e5m2 bytes (u16 + 0x80) >> 8
  (vllm_wlq/linear_method.py:306-308) in chunk-CSR with 512-wide chunks
  (:284-303); they replace the codebook weight;
* DoRA rank r: A ~ N(0, 0.01) [r, K], B ~ N(0, 0.01) [N, r] (fp16),
  m = ||W0||_row * (1 + U(-0.1, 0.1)), s = 1, and
  gamma = m / ||W_patched + s B A||_row rounded to fp16 (:625-635).
"""
from __future__ import annotations

from dataclasses import dataclass
from statistics import NormalDist
from typing import Optional

import numpy as np

_Q16 = np.array([NormalDist().inv_cdf((i + 0.5) / 16) for i in range(16)], np.float64)
CHUNK_M = 512


def words_per_row(K: int) -> int:
    return ((K + 7) // 8 + 3) // 4 * 4


@dataclass
class NpSyntheticLayer:
    N: int
    K: int
    group_size: int
    group_offset: int
    q_packed: np.ndarray      # int32 [N * wpr]
    words_per_row: int
    lut_c: np.ndarray         # fp16 [N, 16] or [N, ngroups, 16]
    chunk_offsets: Optional[np.ndarray]  # int32 [N, nc + 1]
    chunk_cols: Optional[np.ndarray]     # uint16 [nnz], chunk-local
    chunk_vals: Optional[np.ndarray]     # uint8 [nnz], e5m2 bytes
    lora_A: Optional[np.ndarray]         # fp16 [r, K]
    lora_B: Optional[np.ndarray]         # fp16 [N, r]
    magnitude: Optional[np.ndarray]      # float32 [N]
    dora_gamma: Optional[np.ndarray]     # fp16 [N]
    lora_scale: float
    nnz: int

    @property
    def r(self) -> int:
        return 0 if self.lora_B is None else int(self.lora_B.shape[1])

    def indices(self, r0: int = 0, r1: Optional[int] = None) -> np.ndarray:
        """uint8 [rows, K] symbols of rows [r0, r1)."""
        r1 = self.N if r1 is None else r1
        w = self.q_packed.view(np.uint32).reshape(self.N, self.words_per_row)[r0:r1]
        sh = np.arange(8, dtype=np.uint32) * 4
        return ((w[:, :, None] >> sh) & 15).astype(np.uint8).reshape(r1 - r0, -1)[:, :self.K]

    def dense(self, r0: int = 0, r1: Optional[int] = None) -> np.ndarray:
        """fp16 [rows, K]: codebook gather, then outliers replaced."""
        r1 = self.N if r1 is None else r1
        idx = self.indices(r0, r1).astype(np.int64)
        lut = self.lut_c.reshape(self.N, -1, 16)[r0:r1]
        if self.group_size > 0:
            grp = (np.arange(self.K) + self.group_offset) // self.group_size
            W = np.take_along_axis(lut.reshape(r1 - r0, -1), idx + 16 * grp[None, :], axis=1)
        else:
            W = np.take_along_axis(lut.reshape(r1 - r0, 16), idx, axis=1)
        if self.chunk_cols is not None and self.nnz > 0:
            off = self.chunk_offsets[r0:r1]
            nc = off.shape[1] - 1
            counts = np.diff(off, axis=1).reshape(-1)
            rows = np.repeat(np.repeat(np.arange(r1 - r0), nc), counts)
            chunk = np.repeat(np.tile(np.arange(nc), r1 - r0), counts)
            a, b = int(off[0, 0]), int(off[-1, -1])
            cols = chunk * CHUNK_M + self.chunk_cols[a:b].astype(np.int64)
            W[rows, cols] = (self.chunk_vals[a:b].astype(np.uint16) << 8).view(np.float16)
        return W

    def algorithmic_bytes(self, M: int) -> int:
        """HBM bytes one forward moves (the same count as the CUDA path's)."""
        ncsr = (self.K + CHUNK_M - 1) // CHUNK_M
        b = self.N * self.words_per_row * 4 + self.lut_c.size * 2
        if self.chunk_cols is not None:
            b += self.N * (ncsr + 1) * 4 + 3 * self.nnz
        if self.lora_B is not None:
            b += self.N * self.r * 2 + self.N * 2 + self.r * self.K * 2
        return b + M * self.K * 2 + M * self.N * 2


def make_layer(N: int, K: int, *, group_size: int = 128, group_offset: int = 0, density: float = 0.005,
               r: int = 16, seed: int = 0, row_block: int = 256) -> NpSyntheticLayer:
    rng = np.random.default_rng(seed)
    G = group_size
    ng = (K + group_offset + G - 1) // G if G > 0 else 1
    wpr = words_per_row(K)
    q = np.zeros((N, wpr), np.uint32)
    lut = np.empty((N, ng, 16), np.float16)
    norms = np.empty(N, np.float64)
    for n0 in range(0, N, row_block):
        n1 = min(N, n0 + row_block)
        W0 = rng.standard_normal((n1 - n0, K), dtype=np.float32) * np.float32(0.02)
        norms[n0:n1] = np.sqrt(np.einsum("ij,ij->i", W0, W0, dtype=np.float64))
        if G > 0:
            padl, padr = group_offset, ng * G - K - group_offset
            Wg = np.pad(W0, ((0, 0), (padl, padr))).reshape(n1 - n0, ng, G).astype(np.float64)
            cnt = np.full(ng, float(G))
            cnt[0] -= padl
            cnt[-1] -= padr
            mean = Wg.sum(2) / cnt
            std = np.sqrt(np.maximum((Wg * Wg).sum(2) / cnt - mean * mean, 1e-24))
            gidx = (np.arange(K) + group_offset) // G
        else:
            std = W0.astype(np.float64).std(axis=1, keepdims=True)
            gidx = np.zeros(K, np.int64)
        jit = 1.0 + rng.uniform(-0.05, 0.05, size=std.shape + (16,))
        lv = np.sort(std[..., None] * _Q16 * jit, axis=-1).astype(np.float16)
        lut[n0:n1] = lv
        lvf = lv.astype(np.float32)
        mids = (lvf[..., 1:] + lvf[..., :-1]) * 0.5            # [rows, ng, 15]
        idx = np.zeros((n1 - n0, K), np.uint8)
        for j in range(15):
            idx += (W0 > mids[:, gidx, j]).astype(np.uint8)
        pad = np.zeros((n1 - n0, wpr * 8), np.uint32)
        pad[:, :K] = idx
        pad = pad.reshape(n1 - n0, wpr, 8) << (np.arange(8, dtype=np.uint32) * 4)
        q[n0:n1] = np.bitwise_or.reduce(pad, axis=2)
    offs = cols = vals = None
    nnz = 0
    if density > 0:
        total = N * K
        nnz = int(round(total * density))
        pos = np.sort(rng.choice(total, size=nnz, replace=False))
        v16 = (rng.standard_normal(nnz) * 0.1).astype(np.float16)
        u = v16.view(np.uint16).astype(np.int32)
        vals = np.clip((u + 0x80) >> 8, 0, 255).astype(np.uint8)
        rows, cc = pos // K, pos % K
        nc = (K + CHUNK_M - 1) // CHUNK_M
        counts = np.bincount(rows * nc + cc // CHUNK_M, minlength=N * nc).reshape(N, nc)
        flat = np.cumsum(counts.reshape(-1)).reshape(N, nc)
        offs = np.zeros((N, nc + 1), np.int64)
        offs[:, 1:] = flat
        offs[1:, 0] = flat[:-1, -1]
        offs = offs.astype(np.int32)
        cols = (cc % CHUNK_M).astype(np.uint16)
    L = NpSyntheticLayer(N, K, G, group_offset, q.reshape(-1).view(np.int32), wpr,
                         lut if G > 0 else lut.reshape(N, 16), offs, cols, vals, None, None, None, None, 1.0, nnz)
    if r > 0:
        A = (rng.standard_normal((r, K)) * 0.01).astype(np.float16)
        B = (rng.standard_normal((N, r)) * 0.01).astype(np.float16)
        m = norms * (1.0 + rng.uniform(-0.1, 0.1, N))
        BA = B.astype(np.float32) @ A.astype(np.float32)
        gam = np.empty(N, np.float64)
        for n0 in range(0, N, row_block):
            n1 = min(N, n0 + row_block)
            V = L.dense(n0, n1).astype(np.float32) + np.float32(L.lora_scale) * BA[n0:n1]
            nv = np.sqrt(np.einsum("ij,ij->i", V, V, dtype=np.float64))
            gam[n0:n1] = m[n0:n1] / np.maximum(nv, 1e-12)
        L.lora_A, L.lora_B, L.magnitude = A, B, m.astype(np.float32)
        L.dora_gamma = gam.astype(np.float16)
    return L
