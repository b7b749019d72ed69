"""Port of the reference's CPU dequantize-then-matmul path, the timed CPU
baseline of bench.py (``cpu_baseline`` and ``--impl reference``).

TEST / BASELINE INFRASTRUCTURE ONLY.  The steps and their order follow the
reference's own torch code: unpack the packed indices with numpy shifts
(vllm_wlq/linear_method.py:315-323), gather the codebook values with
``torch.gather`` (:881), overwrite the outlier positions with the e5m2 bytes
shifted into fp16 (:887-888), multiply in fp32 and apply the DoRA epilogue
y = gamma * (x W^T + s h B^T) (csrc/gemm_kernel.cu:280-289).  The reference
keeps one codebook per row; the per-group codebooks of the benchmark recipe
are gathered the same way with the group index folded into the gather index.
"""
from __future__ import annotations

import numpy as np
import torch


def cpu_forward(q_words: np.ndarray, wpr: int, lut: torch.Tensor, N: int, K: int, group_size: int,
                group_offset: int, offsets: np.ndarray, cols: np.ndarray, vals: np.ndarray, x: torch.Tensor,
                h: torch.Tensor = None, B: torch.Tensor = None, gamma: torch.Tensor = None,
                scale: float = 1.0) -> torch.Tensor:
    """x [M, K] float32 -> y [M, N] float32 on the CPU."""
    shifts = np.arange(8, dtype=np.uint32) * 4
    words = np.ascontiguousarray(q_words).view(np.uint32).reshape(N, wpr)
    idx = ((words[:, :, None] >> shifts[None, None, :]) & 15).reshape(N, wpr * 8)[:, :K]
    idx_t = torch.from_numpy(idx.astype(np.int64))
    if group_size > 0:
        grp = (torch.arange(K) + group_offset) // group_size
        W = torch.gather(lut.reshape(N, -1).float(), 1, idx_t + 16 * grp[None, :])
    else:
        W = torch.gather(lut.reshape(N, 16).float(), 1, idx_t)
    if cols is not None and len(cols) > 0:
        nc = offsets.shape[1] - 1
        counts = np.diff(offsets, axis=1).reshape(-1)
        rows = np.repeat(np.repeat(np.arange(N), nc), counts)
        chunk = np.repeat(np.tile(np.arange(nc), N), counts)
        start = offsets[0, 0]
        c = chunk * 512 + np.asarray(cols, np.int64)[start:start + counts.sum()]
        v = (torch.from_numpy(np.asarray(vals, np.uint8)[start:start + counts.sum()].astype(np.int32)) << 8)
        W[torch.from_numpy(rows), torch.from_numpy(c)] = v.to(torch.int16).view(torch.float16).float()
    y = x.float() @ W.t()
    if h is not None and B is not None and gamma is not None:
        y = (y + scale * (h.float() @ B.float().t())) * gamma.float()
    return y
