"""The synthetic checkpoint writer (qwen_wlqfastshot_helen_beta_b200/checkpoint.py)
against WLQLinearMethod's load path: a 2-layer Qwen2-shaped checkpoint is
written, every fused vLLM linear (qkv, o, gate_up, down of layer 1) is loaded
from the safetensors files the way vLLM's Qwen2 loader feeds it (per-shard
weight_loader calls with the q/k/v and 0/1 shard ids), and the loaded layer
must reproduce exactly what was written: the dequantised weights (indices,
codebooks, outlier overwrite) and the DoRA adapter.  CPU only; imports vLLM."""
import json
import os
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import oracle as O

ARCH = {"hidden_size": 256, "intermediate_size": 640, "num_hidden_layers": 2, "num_attention_heads": 4,
        "num_key_value_heads": 2, "vocab_size": 1000, "rope_theta": 1e6, "rms_norm_eps": 1e-6,
        "max_position_embeddings": 4096}
FUSED = {"qkv_proj": ("self_attn", [("q_proj", "q"), ("k_proj", "k"), ("v_proj", "v")]),
         "o_proj": ("self_attn", [("o_proj", None)]),
         "gate_up_proj": ("mlp", [("gate_proj", 0), ("up_proj", 1)]),
         "down_proj": ("mlp", [("down_proj", None)])}
NAMES = ["q_packed", "lut_c", "bits", "outlier_mask_1bit", "outlier_values"]


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    pytest.importorskip("vllm")
    from qwen_wlqfastshot_helen_beta_b200 import checkpoint
    d = str(tmp_path_factory.mktemp("wlq_ckpt"))
    checkpoint.write_checkpoint(d, ARCH, group_size=128, density=0.01, rank=8, seed=3, shard_bytes=1 << 20)
    return d


def _tensors(d):
    from safetensors.torch import load_file
    with open(os.path.join(d, "model.safetensors.index.json")) as f:
        files = sorted(set(json.load(f)["weight_map"].values()))
    out = {}
    for fn in files:
        out.update(load_file(os.path.join(d, fn)))
    return out


def _dense_written(t, pre, K, N):
    """[N, K] fp16 weights straight from the written tensors: continuous
    4-bit words, per-(row, 128-column group) codebooks, mask-order outliers."""
    words = t[pre + ".q_packed"].numpy().view(np.uint32)
    sym = ((words[:, None] >> (np.arange(8, dtype=np.uint32) * 4)) & 15).reshape(-1)[:N * K].reshape(N, K)
    lut = t[pre + ".lut_c"].numpy()
    W = np.take_along_axis(lut[:, np.arange(K) // 128, :], sym[:, :, None].astype(np.int64), axis=2)[:, :, 0]
    mask = np.unpackbits(t[pre + ".outlier_mask_1bit"].numpy())[:N * K].astype(bool)
    vals = O.fp8_bytes_to_fp16(O.fp16_to_fp8_bytes(t[pre + ".outlier_values"].numpy()))
    W = W.reshape(-1).copy()
    W[mask] = vals
    return W.reshape(N, K)


def test_config_and_files(ckpt):
    with open(os.path.join(ckpt, "config.json")) as f:
        cfg = json.load(f)
    assert cfg["architectures"] == ["Qwen2ForCausalLM"] and cfg["num_hidden_layers"] == 2
    q = cfg["quantization_config"]
    assert q["quant_method"] == "wlq_fastShot" and q["bits"] == 4 and q["lut_group_size"] == 128
    assert q["_name_or_path"] == ckpt
    t = _tensors(ckpt)
    assert t["model.embed_tokens.weight"].dtype == torch.bfloat16
    assert t["model.layers.0.self_attn.q_proj.bias"].shape == (256,)
    assert os.path.isfile(os.path.join(ckpt, "lora_adapter_distilled", "adapter_model.safetensors"))


@pytest.mark.parametrize("fused", sorted(FUSED))
def test_loads_through_linear_method(ckpt, fused, monkeypatch):
    from qwen_wlqfastshot_helen_beta_b200 import checkpoint, linear_method as lm
    from qwen_wlqfastshot_helen_beta_b200.quant_config import WLQFastShotConfig
    with open(os.path.join(ckpt, "config.json")) as f:
        qcfg = WLQFastShotConfig.from_config(json.load(f)["quantization_config"])
    assert qcfg.model_id == ckpt and qcfg.lut_group_size == 128
    t = _tensors(ckpt)
    mod, parts = FUSED[fused]
    projs = checkpoint._projections(ARCH)
    K = projs[parts[0][0]][0]
    Ns = [projs[p][1] for p, _ in parts]
    lm.reset_dora_cache()
    monkeypatch.setattr(lm, "get_tp_info", lambda: (0, 1))
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    method = lm.WLQLinearMethod(qcfg)
    layer = torch.nn.Module()
    layer.is_row_parallel = fused in ("o_proj", "down_proj")
    method.create_weights(layer, K, Ns, K, sum(Ns), torch.bfloat16)
    layer.vllm_prefix = f"model.layers.1.{mod}.{fused}"
    for pname, sid in parts:
        for nm in NAMES:
            prm = getattr(layer, nm)
            prm.weight_loader(prm, t[f"model.layers.1.{mod}.{pname}.{nm}"], *(() if sid is None else (sid,)))
    method.process_weights_after_loading(layer)

    ref = np.concatenate([_dense_written(t, f"model.layers.1.{mod}.{p}", K, projs[p][1]) for p, _ in parts])
    got = O.dequant(layer.q_packed_aligned.numpy().view(np.uint32).reshape(-1), layer.words_per_row,
                    layer.lut_c.numpy(), layer.N, layer.K, 4, layer.lut_group_size, layer.lut_group_offset,
                    layer.chunk_offsets.numpy(), layer.chunk_cols.numpy(), layer.chunk_vals.numpy())
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
    # the DoRA adapter: A stacked over the fused projections, B block-diagonal
    assert layer.has_dora and layer.lora_A_f16.shape == (8 * len(parts), K)
    from safetensors.torch import load_file
    ad = load_file(os.path.join(ckpt, "lora_adapter_distilled", "adapter_model.safetensors"))
    A = np.concatenate([ad[f"base_model.model.model.layers.1.{mod}.{p}.lora_A.weight"].numpy() for p, _ in parts])
    assert np.array_equal(layer.lora_A_f16.numpy().view(np.uint16), A.view(np.uint16))
    assert layer.lora_scale == pytest.approx(1.0)
