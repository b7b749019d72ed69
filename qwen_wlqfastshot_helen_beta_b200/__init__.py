"""B200 (sm_100a) WLQ 4-bit LUT linear method for vLLM.

Drop-in for the reference plugin's hot path (vllm_wlq/__init__.py:1-90):
the same ``torch.ops.wlq_fastShot.gemv`` / ``torch.ops.wlq_fastShot.gemm``
custom ops (the reference schema with optional trailing arguments for
per-group codebooks, the prepacked layout and ``lora_A``, the DoRA matrix A
given in place of h = A x so the decode GEMV computes h itself; ``out``
mutated, fake implementations for CUDA-graph capture and torch.compile),
``init_workspaces`` and the ``register`` vLLM plugin entry point.  ``WLQFastShotConfig`` / ``WLQLinearMethod`` import vLLM
and are loaded on first access.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _C

__all__ = ["WLQFastShotConfig", "WLQLinearMethod", "init_workspaces", "register", "_C"]


def _register_ops():
    @torch.library.custom_op("wlq_fastShot::gemv", mutates_args={"out"})
    def _gemv_op(
        q_packed: torch.Tensor,
        lut_c: torch.Tensor,
        x: torch.Tensor,
        out: torch.Tensor,
        N: int,
        K: int,
        bits: int,
        chunk_offsets: Optional[torch.Tensor] = None,
        chunk_cols: Optional[torch.Tensor] = None,
        chunk_vals: Optional[torch.Tensor] = None,
        lora_B: Optional[torch.Tensor] = None,
        lora_h: Optional[torch.Tensor] = None,
        dora_gamma: Optional[torch.Tensor] = None,
        lora_scale: float = 1.0,
        lut_group_size: int = 0,
        lut_group_offset: int = 0,
        lut_format: int = 0,
        lora_A: Optional[torch.Tensor] = None,
    ) -> None:
        if lora_A is not None and lora_h is None:
            if _C.folds_h(1, int(N), int(K), int(lora_A.shape[0]), lut_format, x):  # h = A x inside the GEMV
                _C.gemv_lora_a(q_packed, lut_c, x, out, N, K, bits, chunk_offsets, chunk_cols, chunk_vals, lora_B,
                               lora_A, dora_gamma, lora_scale, lut_group_size, lut_group_offset, lut_format)
                return
            lora_h = _C.lora_h(x.reshape(1, int(K)), lora_A)  # this package's own kernel, before the GEMV
        _C.gemv_forward(q_packed, lut_c, x, out, N, K, bits, chunk_offsets, chunk_cols, chunk_vals, lora_B,
                        lora_h, dora_gamma, lora_scale, lut_group_size, lut_group_offset, lut_format)

    @_gemv_op.register_fake
    def _gemv_fake(q_packed, lut_c, x, out, N, K, bits, chunk_offsets=None, chunk_cols=None, chunk_vals=None,
                   lora_B=None, lora_h=None, dora_gamma=None, lora_scale=1.0, lut_group_size=0,
                   lut_group_offset=0, lut_format=0, lora_A=None):
        return None

    @torch.library.custom_op("wlq_fastShot::gemm", mutates_args={"out"})
    def _gemm_op(
        X: torch.Tensor,
        q_packed: torch.Tensor,
        lut_c: torch.Tensor,
        out: torch.Tensor,
        N: int,
        K: int,
        bits: int,
        words_per_row: int,
        chunk_offsets: Optional[torch.Tensor] = None,
        chunk_cols: Optional[torch.Tensor] = None,
        chunk_vals: Optional[torch.Tensor] = None,
        lora_H: Optional[torch.Tensor] = None,
        lora_B: Optional[torch.Tensor] = None,
        dora_gamma: Optional[torch.Tensor] = None,
        lora_scale: float = 1.0,
        lut_group_size: int = 0,
        lut_group_offset: int = 0,
        lut_format: int = 0,
        lora_A: Optional[torch.Tensor] = None,
    ) -> None:
        if lora_A is not None and lora_H is None:
            M = X.numel() // int(K)
            if _C.folds_h(M, int(N), int(K), int(lora_A.shape[0]), lut_format, X):  # h = A x inside the GEMV
                _C.gemv_lora_a(q_packed, lut_c, X, out, N, K, bits, chunk_offsets, chunk_cols, chunk_vals, lora_B,
                               lora_A, dora_gamma, lora_scale, lut_group_size, lut_group_offset, lut_format)
                return
            # otherwise H = X A^T on this package's own kernel, before the GEMM
            lora_H = _C.lora_h(X.reshape(M, int(K)), lora_A)
        _C.gemm_forward(X, q_packed, lut_c, out, N, K, bits, words_per_row, chunk_offsets, chunk_cols,
                        chunk_vals, lora_H, lora_B, dora_gamma, lora_scale, lut_group_size, lut_group_offset,
                        lut_format)

    @_gemm_op.register_fake
    def _gemm_fake(X, q_packed, lut_c, out, N, K, bits, words_per_row, chunk_offsets=None, chunk_cols=None,
                   chunk_vals=None, lora_H=None, lora_B=None, dora_gamma=None, lora_scale=1.0, lut_group_size=0,
                   lut_group_offset=0, lut_format=0, lora_A=None):
        return None


def _ops_registered() -> bool:
    try:
        return torch._C._dispatch_has_kernel_for_dispatch_key("wlq_fastShot::gemv", "CompositeExplicitAutograd") or \
            hasattr(torch.ops.wlq_fastShot, "gemv")
    except (AttributeError, RuntimeError):
        return False


if not _ops_registered():
    _register_ops()


def init_workspaces(max_N: int, max_K: int, device: torch.device):
    """Interface parity with vllm_wlq/__init__.py:79-81 (no workspace needed)."""
    _C.init_workspaces(int(max_N), int(max_K), device)


def register():
    """vLLM general-plugin entry point: registers the quantization config."""
    from . import quant_config  # noqa: F401  (decorators register "wlq_fastShot" / "wlq_fastshot")


def __getattr__(name):
    if name == "WLQFastShotConfig":
        from .quant_config import WLQFastShotConfig
        return WLQFastShotConfig
    if name == "WLQLinearMethod":
        from .linear_method import WLQLinearMethod
        return WLQLinearMethod
    raise AttributeError(name)
