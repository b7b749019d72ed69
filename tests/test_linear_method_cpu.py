"""WLQLinearMethod's load path against the reference's own load path
(golden vectors from vllm_wlq/linear_method.py:413-935 run on the same
checkpoints, tests/golden/make_golden.py).  CPU only; imports vLLM."""
import json
import os

import numpy as np
import pytest
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


def write_adapter(d, proj, g, p, nsh, r, scale):
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


@pytest.fixture(scope="module")
def lm_module():
    pytest.importorskip("vllm")
    from qwen_wlqfastshot_helen_beta_b200 import linear_method
    return linear_method


def load_case(lm_module, g, name, tmp_path, monkeypatch, device="cpu"):
    from types import SimpleNamespace
    p = name + "__"
    proj, sids = CASES[name]
    K_full, K_part, tp, rank, row_par, r, M, nsh = (int(v) for v in g[p + "meta"])
    mdir = str(tmp_path / name)
    os.makedirs(mdir, exist_ok=True)
    if int(g[p + "has_dora"][0]):
        write_adapter(mdir, proj, g, p, nsh, int(g[f"{p}in0_lora_B"].shape[1]), float(g[p + "scale"][0]))
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


@pytest.mark.parametrize("name", sorted(CASES))
def test_load_path_matches_reference(lm_module, golden_layers, name, tmp_path, monkeypatch):
    g = golden_layers
    p = name + "__"
    _, layer = load_case(lm_module, g, name, tmp_path, monkeypatch)
    assert layer.words_per_row == int(g[p + "wpr"][0])
    assert np.array_equal(layer.q_packed_aligned.numpy(), g[p + "q_aligned"])
    assert np.array_equal(layer.lut_c.numpy().view(np.uint16), g[p + "lut"].view(np.uint16))
    assert np.array_equal(layer.chunk_offsets.numpy(), g[p + "offsets"])
    assert np.array_equal(layer.chunk_cols.numpy(), g[p + "cols"])
    assert np.array_equal(layer.chunk_vals.numpy(), g[p + "vals"])
    assert layer.has_dora == bool(g[p + "has_dora"][0])
    if layer.has_dora:
        assert np.array_equal(layer.lora_A_f16.numpy().view(np.uint16), g[p + "lora_A_f16"].view(np.uint16))
        assert np.array_equal(layer.lora_B.numpy().view(np.uint16), g[p + "lora_B"].view(np.uint16))
        ulps = np.abs(layer.dora_gamma.numpy().view(np.int16).astype(np.int32) -
                      g[p + "gamma"].view(np.int16).astype(np.int32))
        assert ulps.max() <= 1
        assert layer.lora_scale == pytest.approx(float(g[p + "scale"][0]))


def test_apply_refuses_cpu_tensors(lm_module, golden_layers, tmp_path, monkeypatch):
    method, layer = load_case(lm_module, golden_layers, "o_tp1_nodora", tmp_path, monkeypatch)
    with pytest.raises(RuntimeError, match="CUDA"):
        method.apply(layer, torch.zeros(2, layer.K, dtype=torch.float16))


def test_quant_config_surface(lm_module):
    from qwen_wlqfastshot_helen_beta_b200.quant_config import WLQFastShotConfig
    c = WLQFastShotConfig.from_config({"quantization_config": {"bits": 4, "lut_group_size": 128},
                                       "_name_or_path": "some/model"})
    assert c.get_name() == "wlq_fastShot" and c.bits == 4 and c.chunk_m == 512 and c.lut_group_size == 128
    assert c.model_id == "some/model" and c.get_min_capability() == 100
    assert torch.bfloat16 in c.get_supported_act_dtypes()
    assert WLQFastShotConfig.from_config({"bits": 3}).chunk_m == 640
