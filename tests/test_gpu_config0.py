"""BASELINE config 0 end to end on the GPU: a 4864 -> 896 layer (the
Qwen2.5-0.5B down_proj shape) written in the reference's on-disk format,
loaded through WLQLinearMethod (create_weights / weight_loader /
process_weights_after_loading) and run through apply() with M = 8 fp32
activations (apply casts them to fp16 as the reference does,
vllm_wlq/linear_method.py:947-948, and casts the output back, :1004).

The layer follows the config-0 recipe (oracle/synthetic_np.py): W0 ~ N(0,
0.02), 16 normal-quantile levels with 5% jitter per row (the reference's
layout) or per 128-column group (the benchmark recipe), nearest-level
indices, 0.5% outliers, DoRA rank 16 with m = ||W0||_row (1 + U(-0.1, 0.1))).
The output is checked against the oracle's float64 forward, against the
reference's CPU dequantize-then-matmul steps (oracle/cpu_baseline.py) and,
for per-row codebooks, against the reference's own wmma kernel
(launch_gemm_metalog_dora, csrc/gemm_kernel.cu:527-596), the kernel the
reference runs for 2 <= M <= 15.
"""
import ctypes
import json
import os
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from _layers import rel_err
from oracle import oracle as O
from oracle import synthetic_np as SN

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
N, K, M = 896, 4864, 8
TOL = 5e-3  # fp16 activations, fp32 accumulation: normwise max relative error


@pytest.fixture(scope="module")
def lm_module():
    pytest.importorskip("vllm")
    assert torch.cuda.is_available()
    from qwen_wlqfastshot_helen_beta_b200 import linear_method
    return linear_method


def checkpoint_tensors(L):
    """The layer in the reference's on-disk format: continuous 4-bit words,
    codebooks, a 1-bit outlier mask (np.packbits, big bit order) and fp16
    outlier values in mask order (vllm_wlq/linear_method.py:315-323, 500-501)."""
    idx = L.indices().reshape(-1).astype(np.uint32)
    pad = (-idx.size) % 8
    idx = np.concatenate([idx, np.zeros(pad, np.uint32)]).reshape(-1, 8)
    words = np.bitwise_or.reduce(idx << (np.arange(8, dtype=np.uint32) * 4), axis=1).view(np.int32)
    mask = np.zeros((L.N, L.K), bool)
    vals = np.zeros((L.N, L.K), np.uint8)
    nc = L.chunk_offsets.shape[1] - 1
    for n in range(L.N):
        for c in range(nc):
            a, b = L.chunk_offsets[n, c], L.chunk_offsets[n, c + 1]
            cols = c * 512 + L.chunk_cols[a:b].astype(np.int64)
            mask[n, cols] = True
            vals[n, cols] = L.chunk_vals[a:b]
    v16 = (vals[mask].astype(np.uint16) << 8).view(np.float16)  # e5m2 values, exact in fp16
    return {"q_packed": torch.from_numpy(words.copy()), "lut_c": torch.from_numpy(L.lut_c.copy()),
            "bits": torch.tensor([4], dtype=torch.int32),
            "outlier_mask_1bit": torch.from_numpy(np.packbits(mask.reshape(-1))),
            "outlier_values": torch.from_numpy(v16.copy())}


def load_layer(lm_module, L, tmp_path, monkeypatch):
    from safetensors.torch import save_file
    mdir = str(tmp_path / f"cfg0_g{L.group_size}")
    os.makedirs(os.path.join(mdir, "lora_adapter_distilled"), exist_ok=True)
    base = "base_model.model.model.layers.3.mlp.down_proj"
    save_file({f"{base}.lora_A.weight": torch.from_numpy(L.lora_A), f"{base}.lora_B.weight": torch.from_numpy(L.lora_B),
               f"{base}.lora_magnitude_vector": torch.from_numpy(L.magnitude)},
              os.path.join(mdir, "lora_adapter_distilled", "adapter_model.safetensors"))
    with open(os.path.join(mdir, "lora_adapter_distilled", "adapter_config.json"), "w") as f:
        json.dump({"lora_alpha": L.r, "r": L.r}, f)
    lm_module.reset_dora_cache()
    monkeypatch.setattr(lm_module, "get_tp_info", lambda: (0, 1))
    method = lm_module.WLQLinearMethod(SimpleNamespace(bits=4, model_id=mdir, lut_group_size=L.group_size))
    layer = torch.nn.Module()
    layer.is_row_parallel = True
    method.create_weights(layer, K, [N], K, N, torch.float16)
    layer.vllm_prefix = "model.layers.3.mlp.down_proj"
    for nm, t in checkpoint_tensors(L).items():
        prm = getattr(layer, nm)
        prm.weight_loader(prm, t)
    method.process_weights_after_loading(layer)
    return method, layer


@pytest.mark.parametrize("G", [0, 128], ids=["per_row", "group128"])
def test_config0_apply(lm_module, G, tmp_path, monkeypatch):
    L = SN.make_layer(N, K, group_size=G, density=0.005, r=16, seed=2024 + G)
    method, layer = load_layer(lm_module, L, tmp_path, monkeypatch)
    assert layer.has_dora and layer.lora_scale == 1.0
    # gamma from the load path against the recipe's float64 gamma
    ulps = np.abs(layer.dora_gamma.cpu().numpy().view(np.int16).astype(np.int32) -
                  L.dora_gamma.view(np.int16).astype(np.int32)).max()
    assert ulps <= 2, ulps
    # dequantised weights: bit-exact with the oracle's gather + outlier overwrite
    W = O.dequant(L.q_packed, L.words_per_row, L.lut_c, N, K, 4, G, 0, L.chunk_offsets, L.chunk_cols, L.chunk_vals)
    assert np.array_equal(W.view(np.uint16), L.dense().view(np.uint16))
    rng = np.random.default_rng(4)
    x = rng.standard_normal((M, K)).astype(np.float32)  # config 0: fp32 activations ~ N(0, 1)
    y = method.apply(layer, torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    assert y.dtype == torch.float32 and y.shape == (M, N)
    y = y.cpu().numpy()
    # the reference's numerics: x rounded to fp16, h = fp16(A x) (F.linear in fp16)
    x16 = x.astype(np.float16).astype(np.float32)
    h16 = (x16.astype(np.float64) @ L.lora_A.astype(np.float64).T).astype(np.float16).astype(np.float32)
    gam = layer.dora_gamma.cpu().numpy()
    ref = O.forward_f64(W, x16, h16, L.lora_B, gam, 1.0)
    e_oracle = rel_err(y, ref)
    assert e_oracle <= TOL, e_oracle
    # the reference's CPU dequantize-then-matmul steps on the same inputs
    from oracle.cpu_baseline import cpu_forward
    y_cpu = cpu_forward(L.q_packed, L.words_per_row, torch.from_numpy(L.lut_c), N, K, G, 0, L.chunk_offsets,
                        L.chunk_cols.astype(np.int64), L.chunk_vals, torch.from_numpy(x16),
                        torch.from_numpy(h16), torch.from_numpy(L.lora_B), torch.from_numpy(gam), 1.0).numpy()
    assert rel_err(y, y_cpu) <= TOL
    assert rel_err(y_cpu, ref) <= 1e-5  # the CPU steps in fp32 against float64
    # M = 1 through the gemv op
    y1 = method.apply(layer, torch.from_numpy(x[:1]).cuda()).cpu().numpy()
    assert rel_err(y1, ref[:1]) <= TOL
    if G == 0:
        # the reference's own wmma kernel (per-row codebooks only) on the same device tensors
        path = os.path.join(ROOT, "oracle", "_ref", "libwlq_ref_kernels.so")
        if not os.path.exists(path):
            pytest.skip("reference kernels not built (oracle/build_ref.sh needs the reference tree)")
        lib = ctypes.CDLL(path)
        xd = torch.from_numpy(x16).cuda().to(torch.float16)
        hd = torch.from_numpy(h16).cuda()
        yr = torch.empty((M, N), dtype=torch.float16, device="cuda")

        def p(t):
            return ctypes.c_void_p(t.data_ptr())
        i = ctypes.c_int
        lib.launch_gemm_metalog_dora(p(xd), p(layer.q_packed_aligned), p(layer.lut_c), p(yr), p(layer.chunk_offsets),
                                     p(layer.chunk_cols), p(layer.chunk_vals), p(hd), p(layer.lora_B),
                                     p(layer.dora_gamma), ctypes.c_float(1.0), i(16), i(M), i(N), i(K), i(4),
                                     i(layer.words_per_row), i((K + 511) // 512), i(512),
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        yr = yr.float().cpu().numpy()
        assert rel_err(yr, ref) <= TOL
        assert rel_err(y, yr) <= TOL
