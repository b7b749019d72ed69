"""Seeded synthetic WLQ layers in the kernel layout.

No public checkpoint or dataset is involved: layers follow the benchmark
recipe of the WLQ format, generated with torch on any device.

* W0 ~ N(0, 0.02) [N, K];
* per (row, group) codebook of 16 sorted levels
  std(group) * Phi^-1((i + 0.5) / 16) * (1 + U(-0.05, 0.05)), fp16;
  ``group_size=0`` gives one codebook per row (the reference's layout);
* indices = nearest level, packed row-aligned (8 per int32 word, LSB first);
* DoRA rank r: A ~ N(0, 0.01) [r, K], B ~ N(0, 0.01) [N, r],
  m = ||W0||_row * (1 + U(-0.1, 0.1)), gamma = m / ||W + s B A||_row (fp16);
* outliers: a fraction `density` of positions, uniform, fp16 ~ N(0, 0.1)
  stored as e5m2 bytes ((u16 + 0x80) >> 8), in chunk-CSR with 512-wide chunks;
  they replace the codebook weight.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from statistics import NormalDist
from typing import Optional

import torch

from . import _C

_Q16 = torch.tensor([NormalDist().inv_cdf((i + 0.5) / 16) for i in range(16)], dtype=torch.float64)


@dataclass
class SyntheticLayer:
    N: int
    K: int
    q_packed: torch.Tensor      # int32 [N * wpr]
    words_per_row: int
    lut_c: torch.Tensor         # fp16 [N, 16] or [N, ngroups, 16]
    group_size: int
    group_offset: int
    chunk_offsets: Optional[torch.Tensor]
    chunk_cols: Optional[torch.Tensor]
    chunk_vals: Optional[torch.Tensor]
    lora_A: Optional[torch.Tensor]   # fp16 [r, K]
    lora_B: Optional[torch.Tensor]   # fp16 [N, r]
    dora_gamma: Optional[torch.Tensor]
    lora_scale: float
    nnz: int
    lut_packed: Optional[torch.Tensor] = None   # WLQ_LUT_PREPACKED layout for packed_dtype
    cols_packed: Optional[torch.Tensor] = None
    delta_packed: Optional[torch.Tensor] = None
    packed_dtype: Optional[torch.dtype] = None
    lora_A_act: Optional[torch.Tensor] = None   # A in packed_dtype, for the GEMV that computes h = A x

    def prepack(self, act_dtype: torch.dtype) -> "SyntheticLayer":
        self.lut_packed = _C.prepack_lut(self.lut_c.contiguous(), act_dtype)
        if self.lora_A is not None:
            self.lora_A_act = self.lora_A.to(act_dtype).contiguous()
        if self.chunk_cols is not None and self.q_packed.is_cuda:
            self.cols_packed, self.delta_packed = _C.prepack_outliers(
                self.q_packed, self.lut_c, self.chunk_offsets, self.chunk_cols, self.chunk_vals, self.N, self.K, 4,
                act_dtype, self.group_size, self.group_offset)
        self.packed_dtype = act_dtype
        return self

    def operands_for(self, act_dtype: torch.dtype):
        """(codebooks, outlier cols, outlier vals, lut_format) for act_dtype."""
        if self.lut_packed is not None and self.packed_dtype == act_dtype and \
                (self.chunk_cols is None or self.cols_packed is not None):
            return self.lut_packed, self.cols_packed, self.delta_packed, 1
        return self.lut_c, self.chunk_cols, self.chunk_vals, 0

    @property
    def r(self) -> int:
        return 0 if self.lora_B is None else int(self.lora_B.shape[1])

    def algorithmic_bytes(self, M: int) -> int:
        """HBM bytes one forward must move: indices, codebooks, outlier CSR,
        DoRA tensors (A and B as 2-byte [r, K] and [N, r], gamma), x and out
        (2 B); h = A x is an intermediate of the forward."""
        ncsr = (self.K + 511) // 512
        b = self.N * self.words_per_row * 4 + self.lut_c.numel() * 2
        if self.chunk_cols is not None:
            b += self.N * (ncsr + 1) * 4 + 3 * self.nnz
        if self.lora_B is not None:
            b += self.N * self.r * 2 + self.N * 2 + self.r * self.K * 2
        b += M * self.K * 2 + M * self.N * 2
        return b


def pack_rows(idx: torch.Tensor) -> torch.Tensor:
    """uint8/int [N, K] 4-bit symbols -> row-aligned int32 words [N * wpr]."""
    N, K = idx.shape
    wpr = _C.words_per_row(K, 4)
    pad = wpr * 8 - K
    q = torch.nn.functional.pad(idx.to(torch.int64), (0, pad)).view(N, wpr, 8)
    shifts = torch.arange(8, device=idx.device, dtype=torch.int64) * 4
    words = (q << shifts).sum(dim=2)
    words = torch.where(words >= 2 ** 31, words - 2 ** 32, words)
    return words.to(torch.int32).reshape(-1)


def make_layer(N: int, K: int, *, group_size: int = 128, group_offset: int = 0, density: float = 0.005,
               r: int = 16, lora_alpha: Optional[float] = None, seed: int = 0, device="cuda",
               row_block: int = 4096, with_dora: bool = True) -> SyntheticLayer:
    """One quantized layer following the recipe above, generated in row blocks."""
    device = torch.device(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    G = group_size
    ng = (K + group_offset + G - 1) // G if G > 0 else 1
    wpr = _C.words_per_row(K, 4)
    q_all = torch.empty(N * wpr, dtype=torch.int32, device=device)
    lut_all = torch.empty((N, ng, 16) if G > 0 else (N, 16), dtype=torch.float16, device=device)
    norms = torch.empty(N, dtype=torch.float32, device=device)
    q16 = _Q16.to(device=device, dtype=torch.float32)
    for n0 in range(0, N, row_block):
        n1 = min(N, n0 + row_block)
        W0 = torch.randn((n1 - n0, K), generator=gen, device=device) * 0.02
        norms[n0:n1] = W0.norm(dim=1)
        if G > 0:
            padl, padr = group_offset, ng * G - K - group_offset
            Wg = torch.nn.functional.pad(W0, (padl, padr)).view(n1 - n0, ng, G)
            cnt = torch.full((ng,), float(G), device=device)
            cnt[0] -= padl
            cnt[-1] -= padr
            mean = Wg.sum(2) / cnt
            var = (Wg * Wg).sum(2) / cnt - mean * mean
            std = var.clamp_min(1e-12).sqrt()
        else:
            std = W0.std(dim=1, keepdim=True)
        jit = 1.0 + (torch.rand(std.shape + (16,), generator=gen, device=device) * 0.1 - 0.05)
        lv = torch.sort(std.unsqueeze(-1) * q16 * jit, dim=-1).values.to(torch.float16)
        lvf = lv.float()
        mids = (lvf[..., 1:] + lvf[..., :-1]) * 0.5  # [rows, ng, 15] / [rows, 1, 15]
        if G > 0:
            gidx = (torch.arange(K, device=device) + group_offset) // G
            m_k = mids[:, gidx, :]  # [rows, K, 15]
        else:
            m_k = mids.expand(n1 - n0, K, 15) if mids.dim() == 3 else mids.unsqueeze(1).expand(n1 - n0, K, 15)
        idx = (W0.unsqueeze(-1) > m_k).sum(-1)
        q_all[n0 * wpr:n1 * wpr] = pack_rows(idx)
        lut_all[n0:n1] = lv if G > 0 else lv.reshape(n1 - n0, 16)
        del W0, m_k, idx
    offs = cols = vals = None
    nnz = 0
    if density > 0:
        total = N * K
        nnz = int(round(total * density))
        pos = torch.randperm(total, generator=gen, device=device)[:nnz].sort().values
        v16 = (torch.randn(nnz, generator=gen, device=device) * 0.1).to(torch.float16)
        u = v16.view(torch.int16).to(torch.int32) & 0xFFFF
        vals = ((u + 0x80) >> 8).clamp(0, 255).to(torch.uint8)
        rows, cc = pos // K, pos % K
        nc = (K + 511) // 512
        counts = torch.bincount(rows * nc + cc // 512, minlength=N * nc).view(N, nc)
        offs = torch.zeros((N, nc + 1), dtype=torch.int64, device=device)
        flat = torch.cumsum(counts.reshape(-1), 0).view(N, nc)
        offs[:, 1:] = flat
        offs[1:, 0] = flat[:-1, -1]
        offs = offs.to(torch.int32)
        cols = (cc % 512).to(torch.int16).view(torch.uint16)  # values < 512: same bits
    lora_A = lora_B = gamma = None
    scale = 1.0
    if with_dora and r > 0:
        A = torch.randn((r, K), generator=gen, device=device) * 0.01
        B = torch.randn((N, r), generator=gen, device=device) * 0.01
        scale = float(lora_alpha if lora_alpha is not None else r) / r
        m = norms * (1.0 + (torch.rand(N, generator=gen, device=device) * 0.2 - 0.1))
        lora_A = A.to(torch.float16).contiguous()
        lora_B = B.to(torch.float16).contiguous()
        # gamma from the dequantised weights, as at load time
        gam = torch.empty(N, dtype=torch.float32, device=device)
        for n0 in range(0, N, row_block):
            n1 = min(N, n0 + row_block)
            Wd = torch.empty((n1 - n0, K), dtype=torch.float16, device=device)
            sub_off = None if offs is None else (offs[n0:n1] - offs[n0, 0]).contiguous()
            a0 = 0 if offs is None else int(offs[n0, 0])
            a1 = 0 if offs is None else int(offs[n1 - 1, -1])
            _C.dequant_w0(q_all[n0 * wpr:n1 * wpr], lut_all[n0:n1].contiguous(), Wd, n1 - n0, K, 4, wpr, sub_off,
                          None if cols is None else cols[a0:a1], None if vals is None else vals[a0:a1],
                          G, group_offset)
            V = Wd.float() + scale * (B[n0:n1] @ A)
            gam[n0:n1] = m[n0:n1] / V.norm(dim=1).clamp_min(1e-12)
        gamma = gam.to(torch.float16)
    return SyntheticLayer(N, K, q_all, wpr, lut_all, G, group_offset, offs, cols, vals, lora_A, lora_B, gamma,
                          scale, nnz)


def lora_h(layer: SyntheticLayer, x: torch.Tensor) -> Optional[torch.Tensor]:
    """h = A x in the activation dtype, as fp32 (vllm_wlq/linear_method.py:962-963, 984)."""
    if layer.lora_A is None:
        return None
    A = layer.lora_A if x.dtype == torch.float16 else layer.lora_A.to(x.dtype)
    return torch.nn.functional.linear(x, A).float()


def forward(layer: SyntheticLayer, x: torch.Tensor, out: Optional[torch.Tensor] = None,
            h: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One call of the batched op on a synthetic layer (x [M, K])."""
    M = x.shape[0]
    if out is None:
        out = torch.empty((M, layer.N), dtype=x.dtype, device=x.device)
    if h is None:
        h = lora_h(layer, x)
    lut, cols, vals, fmt = layer.operands_for(x.dtype)
    _C.gemm_forward(x, layer.q_packed, lut, out, layer.N, layer.K, 4, layer.words_per_row,
                    layer.chunk_offsets, cols, vals, h, layer.lora_B, layer.dora_gamma,
                    layer.lora_scale, layer.group_size, layer.group_offset, fmt)
    return out


def forward_fold(layer: SyntheticLayer, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Decode forward (M <= 16) with h = A x computed inside the GEMV
    (prepacked layer, x in its packed dtype)."""
    M = x.shape[0]
    if out is None:
        out = torch.empty((M, layer.N), dtype=x.dtype, device=x.device)
    lut, cols, vals, fmt = layer.operands_for(x.dtype)
    _C.gemv_lora_a(layer.q_packed, lut, x, out, layer.N, layer.K, 4, layer.chunk_offsets, cols, vals, layer.lora_B,
                   layer.lora_A_act, layer.dora_gamma, layer.lora_scale, layer.group_size, layer.group_offset, fmt)
    return out


QWEN25_7B = {  # name: (K in, N out) of the fused vLLM linears
    "qkv": (3584, 4608),
    "o": (3584, 3584),
    "gate_up": (3584, 37888),
    "down": (18944, 3584),
}


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


__all__ = ["SyntheticLayer", "make_layer", "forward", "lora_h", "pack_rows", "QWEN25_7B", "ceil_div", "math"]
