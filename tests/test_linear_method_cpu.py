"""WLQLinearMethod's load path against the reference's own load path
(golden vectors from vllm_wlq/linear_method.py:413-935 run on the same
checkpoints, tests/golden/make_golden.py).  CPU only; imports vLLM."""
import numpy as np
import pytest
import torch

from _golden_layer import CASES, load_case  # noqa: E402


@pytest.fixture(scope="module")
def lm_module():
    pytest.importorskip("vllm")
    from qwen_wlqfastshot_helen_beta_b200 import linear_method
    return linear_method


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
