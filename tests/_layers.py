"""Seeded small layers in numpy for the parity tests (built with the oracle's
packers, so the CUDA path and the oracle read identical bytes)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np

from oracle import oracle as O


@dataclass
class NpLayer:
    N: int
    K: int
    G: int
    goff: int
    q: np.ndarray          # uint32 [N * wpr]
    wpr: int
    lut: np.ndarray        # fp16 [N,16] or [N,ng,16]
    off: Optional[np.ndarray]
    cols: Optional[np.ndarray]
    vals: Optional[np.ndarray]
    A: Optional[np.ndarray]  # fp16 [r, K]
    B: Optional[np.ndarray]  # fp16 [N, r]
    gamma: Optional[np.ndarray]
    scale: float

    @property
    def r(self):
        return 0 if self.B is None else self.B.shape[1]

    def dense(self):
        return O.dequant(self.q, self.wpr, self.lut, self.N, self.K, 4, self.G, self.goff, self.off, self.cols,
                         self.vals)


def make_np_layer(rng, N, K, G=0, goff=0, density=0.01, r=16, scale=2.0, outliers=True, dora=True):
    idx = rng.integers(0, 16, size=(N, K), dtype=np.uint8)
    q, wpr = O.pack_row_aligned(idx, 4)
    ng = -(-(K + goff) // G) if G > 0 else 1
    base = np.sort(rng.standard_normal((N, ng, 16)) * 0.02, axis=-1).astype(np.float16)
    lut = base if G > 0 else base.reshape(N, 16)
    off = cols = vals = None
    if outliers:
        mask = rng.random((N, K)) < density
        off, cols = O.build_chunk_csr(mask, 512)
        vals = O.fp16_to_fp8_bytes((rng.standard_normal(cols.size) * 0.1).astype(np.float16))
    A = B = gamma = None
    if dora and r > 0:
        A = (rng.standard_normal((r, K)) * 0.01).astype(np.float16)
        B = (rng.standard_normal((N, r)) * 0.01).astype(np.float16)
        gamma = (1.0 + rng.uniform(-0.2, 0.2, N)).astype(np.float16)
    return NpLayer(N, K, G, goff, q, wpr, lut, off, cols, vals, A, B, gamma, scale)


def reference_output(L: NpLayer, x_act: np.ndarray, h: Optional[np.ndarray]):
    """float64 oracle output for activations already rounded to the act dtype."""
    W = L.dense()
    if L.B is not None and h is not None:
        return O.forward_f64(W, x_act, h, L.B, L.gamma, L.scale)
    return O.forward_f64(W, x_act)


def rel_err(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(1e-30, np.max(np.abs(ref))))


@dataclass
class NpLayerParts:
    """A layer's dense pieces (indices, codebooks, outlier mask and values,
    DoRA tensors) from which any K shard is cut the way vLLM's row-parallel
    layers shard K (vllm_wlq/linear_method.py:753-761, 841-850)."""
    N: int
    K: int
    G: int
    idx: np.ndarray        # uint8 [N, K]
    lut: np.ndarray        # fp16 [N, ng, 16] (G > 0) or [N, 16]
    mask: np.ndarray       # bool [N, K]
    vals: np.ndarray       # uint8 [N, K], e5m2 byte where mask
    A: np.ndarray          # fp16 [r, K]
    B: np.ndarray          # fp16 [N, r]
    gamma: np.ndarray      # fp16 [N]
    scale: float

    def shard(self, c0: int, c1: int) -> NpLayer:
        """Columns [c0, c1): codebook groups from c0 // G, group offset c0 % G."""
        K = c1 - c0
        q, wpr = O.pack_row_aligned(self.idx[:, c0:c1], 4)
        if self.G > 0:
            g0, g1 = c0 // self.G, (c1 - 1) // self.G + 1
            lut, goff = np.ascontiguousarray(self.lut[:, g0:g1]), c0 % self.G
        else:
            lut, goff = self.lut, 0
        m = self.mask[:, c0:c1]
        off, cols = O.build_chunk_csr(m, 512)
        vals = np.ascontiguousarray(self.vals[:, c0:c1][m])
        return NpLayer(self.N, K, self.G, goff, q, wpr, lut, off, cols, vals,
                       np.ascontiguousarray(self.A[:, c0:c1]), self.B, self.gamma, self.scale)

    def full(self) -> NpLayer:
        return self.shard(0, self.K)


def make_np_parts(rng, N, K, G=128, density=0.005, r=16, scale=1.0) -> NpLayerParts:
    idx = rng.integers(0, 16, size=(N, K), dtype=np.uint8)
    ng = -(-K // G) if G > 0 else 1
    base = np.sort(rng.standard_normal((N, ng, 16)) * 0.02, axis=-1).astype(np.float16)
    lut = base if G > 0 else base.reshape(N, 16)
    mask = rng.random((N, K)) < density
    vals = np.zeros((N, K), np.uint8)
    vals[mask] = O.fp16_to_fp8_bytes((rng.standard_normal(int(mask.sum())) * 0.1).astype(np.float16))
    A = (rng.standard_normal((r, K)) * 0.01).astype(np.float16)
    B = (rng.standard_normal((N, r)) * 0.01).astype(np.float16)
    gamma = (1.0 + rng.uniform(-0.2, 0.2, N)).astype(np.float16)
    return NpLayerParts(N, K, G, idx, lut, mask, vals, A, B, gamma, scale)
