"""WLQLinearMethod end to end on the GPU: the reference's checkpoints loaded
through this package's loader, then apply() against the reference's own
forward on the same inputs (golden vectors)."""
import numpy as np
import pytest
import torch

from _golden_layer import CASES, load_case
from _layers import rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lm_module():
    pytest.importorskip("vllm")
    from qwen_wlqfastshot_helen_beta_b200 import linear_method
    return linear_method


@pytest.mark.parametrize("name", sorted(CASES))
def test_apply_matches_reference_forward(lm_module, golden_layers, name, tmp_path, monkeypatch):
    assert torch.cuda.is_available()
    g = golden_layers
    p = name + "__"
    method, layer = load_case(lm_module, g, name, tmp_path, monkeypatch, device="cuda")
    assert layer.q_packed_aligned.is_cuda
    ulps = 0
    if layer.has_dora:
        ulps = np.abs(layer.dora_gamma.cpu().numpy().view(np.int16).astype(np.int32) -
                      g[p + "gamma"].view(np.int16).astype(np.int32)).max()
    assert ulps <= 1
    x = torch.from_numpy(g[p + "x"]).cuda()
    ref = g[p + "y"]
    for dtype, tol in ((torch.float16, 5e-3), (torch.bfloat16, 2e-2), (torch.float32, 5e-3)):
        y = method.apply(layer, x.to(dtype))
        assert y.dtype == dtype and y.shape == (x.shape[0], layer.N)
        assert rel_err(y.float().cpu().numpy(), ref) <= tol, (name, dtype)
        if x.shape[0] > 1:  # M = 1 through the gemv op as well
            y1 = method.apply(layer, x[:1].to(dtype))
            assert rel_err(y1.float().cpu().numpy(), ref[:1]) <= tol, (name, dtype, "M=1")
    bias = torch.randn(layer.N, device="cuda", dtype=torch.float16)
    yb = method.apply(layer, x.to(torch.float16), bias)
    assert rel_err(yb.float().cpu().numpy(), ref + bias.float().cpu().numpy()) <= 5e-3
