"""Loads a golden layer case through WLQLinearMethod (shared by the CPU and GPU tests)."""
import json
import os
from types import SimpleNamespace

import numpy as np
import torch

PROJ = {"qkv_proj": ["q_proj", "k_proj", "v_proj"], "gate_up_proj": ["gate_proj", "up_proj"],
        "o_proj": ["o_proj"], "down_proj": ["down_proj"]}
CASES = {  # name -> (proj, shard ids)
    "qkv_tp1_ef": ("qkv_proj", ["q", "k", "v"]),
    "o_tp1_mask1b": ("o_proj", [None]),
    "gateup_tp2_r1_ef": ("gate_up_proj", [0, 1]),
    "down_tp2_r0_ef": ("down_proj", [None]),
    "down_tp2_r1_noout": ("down_proj", [None]),
    "o_tp1_nodora": ("o_proj", [None]),
}
NAMES = ["q_packed", "lut_c", "bits", "outlier_values", "ef_tile_size", "ef_tile_meta", "ef_bitstream",
         "outlier_mask_1bit"]


def write_adapter(d, proj, g, p, r, scale):
    from safetensors.torch import save_file
    os.makedirs(os.path.join(d, "lora_adapter_distilled"), exist_ok=True)
    t = {}
    for i, pn in enumerate(PROJ[proj]):
        mod = "self_attn" if pn in ("q_proj", "k_proj", "v_proj", "o_proj") else "mlp"
        base = f"base_model.model.model.layers.3.{mod}.{pn}"
        t[f"{base}.lora_A.weight"] = torch.from_numpy(g[f"{p}in{i}_lora_A"])
        t[f"{base}.lora_B.weight"] = torch.from_numpy(g[f"{p}in{i}_lora_B"])
        if f"{p}in{i}_m" in g:
            t[f"{base}.lora_magnitude_vector"] = torch.from_numpy(g[f"{p}in{i}_m"])
    save_file(t, os.path.join(d, "lora_adapter_distilled", "adapter_model.safetensors"))
    with open(os.path.join(d, "lora_adapter_distilled", "adapter_config.json"), "w") as f:
        json.dump({"lora_alpha": scale * r, "r": r}, f)


def load_case(lm_module, g, name, tmp_path, monkeypatch, device="cpu"):
    p = name + "__"
    proj, sids = CASES[name]
    K_full, K_part, tp, rank, row_par, r, M, nsh = (int(v) for v in g[p + "meta"])
    mdir = str(tmp_path / name)
    os.makedirs(mdir, exist_ok=True)
    if int(g[p + "has_dora"][0]):
        write_adapter(mdir, proj, g, p, int(g[f"{p}in0_lora_B"].shape[1]), float(g[p + "scale"][0]))
    lm_module.reset_dora_cache()
    monkeypatch.setattr(lm_module, "get_tp_info", lambda: (rank, tp))
    method = lm_module.WLQLinearMethod(SimpleNamespace(bits=4, model_id=mdir, lut_group_size=0))
    layer = torch.nn.Module()
    layer.is_row_parallel = bool(row_par)
    luts = [g[f"{p}in{i}_lut_c"] for i in range(nsh)]
    parts = [l.shape[0] for l in luts] if (row_par or tp == 1) else [l.shape[0] // tp for l in luts]
    method.create_weights(layer, K_part, parts, K_full, sum(parts) * (1 if row_par else tp), torch.float16)
    layer.vllm_prefix = ("model.layers.3.self_attn." if proj in ("qkv_proj", "o_proj") else "model.layers.3.mlp.") + proj
    for i, sid in enumerate(sids):
        for nm in NAMES:
            key = f"{p}in{i}_{nm}"
            if key in g:
                prm = getattr(layer, nm)
                args = () if sid is None else (sid,)
                prm.weight_loader(prm, torch.from_numpy(np.ascontiguousarray(g[key])), *args)
    if device == "cpu":
        monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    method.process_weights_after_loading(layer)
    return method, layer
