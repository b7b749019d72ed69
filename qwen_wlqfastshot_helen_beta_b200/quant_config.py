"""vLLM quantization config ``wlq_fastShot`` / ``wlq_fastshot``.

Same names, keys, defaults and layer routing as the reference
(vllm_wlq/quant_config.py:10-82).  Differences: ``get_min_capability`` is 100
(this build runs sm_100a only) and one optional key, ``lut_group_size``
(default 0 = one 16-entry codebook per output row, the reference's layout;
e.g. 128 = one codebook per row and 128-column group).
"""
from typing import Any, Dict, List, Optional

import torch
from vllm.model_executor.layers.linear import LinearBase, UnquantizedLinearMethod
from vllm.model_executor.layers.quantization import register_quantization_config
from vllm.model_executor.layers.quantization.base_config import QuantizationConfig

from .linear_method import WLQLinearMethod

_DEFAULT_MODEL_ID = "wichtel-labs/Qwen3.8-27B-WLQ-FastShot"


@register_quantization_config("wlq_fastshot")
@register_quantization_config("wlq_fastShot")
class WLQFastShotConfig(QuantizationConfig):
    """Config of the WLQ FastShot 4-bit LUT quantization (wlq_fastShot)."""

    def __init__(self, bits: int = 4, outlier_fraction: float = 0.05, chunk_m: int = 512, use_dora: bool = True,
                 model_id: Optional[str] = None, lut_group_size: int = 0):
        super().__init__()
        self.bits = bits
        self.outlier_fraction = outlier_fraction
        self.chunk_m = 640 if bits == 3 else chunk_m
        self.use_dora = use_dora
        self.model_id = model_id or _DEFAULT_MODEL_ID
        self.lut_group_size = int(lut_group_size)

    def get_name(self) -> str:
        return "wlq_fastShot"

    def get_supported_act_dtypes(self) -> List[torch.dtype]:
        return [torch.float16, torch.bfloat16]

    @classmethod
    def get_min_capability(cls) -> int:
        return 100

    @classmethod
    def get_config_filenames(cls) -> List[str]:
        return ["/config.json"]

    @classmethod
    def from_config(cls, config: Dict[str, Any]) -> "WLQFastShotConfig":
        q_cfg = config.get("quantization_config") or config
        bits = q_cfg.get("bits", 4)
        return cls(
            bits=bits,
            outlier_fraction=q_cfg.get("outlier_fraction", 0.05),
            chunk_m=640 if bits == 3 else q_cfg.get("chunk_m", 512),
            use_dora=q_cfg.get("use_dora", True),
            model_id=config.get("_name_or_path", _DEFAULT_MODEL_ID),
            lut_group_size=q_cfg.get("lut_group_size", 0),
        )

    def get_quant_method(self, layer: torch.nn.Module, prefix: str) -> Optional[Any]:
        if not isinstance(layer, LinearBase):
            return None
        if prefix.startswith("model.visual") or "visual" in prefix or "blocks." in prefix or "lm_head" in prefix:
            return UnquantizedLinearMethod()
        if any(s in prefix for s in ("conv1d", "router", "shared_expert_gate")):
            return UnquantizedLinearMethod()
        layer.vllm_prefix = prefix
        return WLQLinearMethod(self)

    def get_scaled_act_names(self) -> List[str]:
        return []
