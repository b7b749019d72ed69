"""Generate the golden fixtures in this directory by running the REFERENCE's own
Python code (``vllm_wlq/linear_method.py``) on seeded synthetic inputs.

Runs only where the read-only reference tree exists (default path below, or
``--ref``); the GPU box and the tests never need it, they read the committed
``*.npz`` files.  The reference's compiled ``_C`` module is replaced by an
empty stub so that ``process_weights_after_loading`` takes its pure
numpy/torch path (vllm_wlq/linear_method.py:676-935), which runs the
reference's own unpack / EF-decode / pack / chunk-CSR / gamma code.

The reference ships no EF encoder; EF streams are written by the test-data
encoder in ``oracle/wlq_oracle.c`` and then DECODED by the reference, so the
decoded masks below are the reference's output.

    python tests/golden/make_golden.py [--ref /path/to/reference]
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
import tempfile
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
from oracle import oracle as O  # noqa: E402  (test-data EF encoder only)


def load_reference(ref_root: str):
    pkg = types.ModuleType("vllm_wlq")
    pkg.__path__ = [os.path.join(ref_root, "vllm_wlq")]
    sys.modules["vllm_wlq"] = pkg
    sys.modules["vllm_wlq._C"] = types.ModuleType("vllm_wlq._C")  # no compiled codecs
    spec = importlib.util.spec_from_file_location(
        "vllm_wlq.linear_method", os.path.join(ref_root, "vllm_wlq", "linear_method.py"))
    lm = importlib.util.module_from_spec(spec)
    sys.modules["vllm_wlq.linear_method"] = lm
    spec.loader.exec_module(lm)
    return lm


def normal_quantile_lut(rng, std, n_levels=16):
    """Sorted levels std * Phi^-1((i+0.5)/16) * (1 + U(-0.05, 0.05))."""
    from statistics import NormalDist
    base = np.array([NormalDist().inv_cdf((i + 0.5) / n_levels) for i in range(n_levels)])
    lv = std[..., None] * base * (1.0 + rng.uniform(-0.05, 0.05, size=std.shape + (n_levels,)))
    return np.sort(lv, axis=-1).astype(np.float16)


# --------------------------------------------------------------------------- #
# 1. codec vectors
# --------------------------------------------------------------------------- #
def codec_vectors(lm, rng):
    out = {}
    for ci, (N, K, bits) in enumerate([(7, 13, 4), (5, 37, 4), (9, 512, 4), (3, 50, 3),
                                       (4, 33, 2), (3, 70, 1), (6, 1100, 4)]):
        spw = 10 if bits == 3 else 32 // bits
        n_words = (N * K + spw - 1) // spw
        words = rng.integers(0, 2 ** 32, size=n_words, dtype=np.uint64).astype(np.uint32)
        idx = lm.unpack_indices_continuous(torch.from_numpy(words.view(np.int32)), N, K, bits)
        packed, wpr = lm.pack_indices_row_aligned(idx, bits)
        out[f"pack{ci}_meta"] = np.array([N, K, bits, wpr], np.int64)
        out[f"pack{ci}_words"] = words
        out[f"pack{ci}_idx"] = idx.astype(np.uint8)
        out[f"pack{ci}_aligned"] = packed.astype(np.uint32)

    for ci, (N, K, chunk_m, dens) in enumerate([(5, 700, 512, 0.05), (8, 1100, 512, 0.01),
                                                (3, 1300, 640, 0.02), (4, 100, 512, 0.0)]):
        mask = rng.random((N, K)) < dens
        vals = (rng.standard_normal(int(mask.sum())) * 0.1).astype(np.float16)
        off, cols, v8 = lm.build_chunk_csr(mask, torch.from_numpy(vals), chunk_m)
        out[f"csr{ci}_meta"] = np.array([N, K, chunk_m], np.int64)
        out[f"csr{ci}_mask"] = mask
        out[f"csr{ci}_vals_f16"] = vals
        out[f"csr{ci}_offsets"] = off.numpy()
        out[f"csr{ci}_cols"] = cols.numpy()
        out[f"csr{ci}_vals_u8"] = v8.numpy()

    # edge bytes of the fp16 -> e5m2 conversion
    special = np.array([0x0000, 0x007F, 0x0080, 0x00FF, 0x3C00, 0x3C7F, 0x3C80, 0x3CFF, 0x7BFF,
                        0x7C00, 0x7F80, 0x7FFF, 0x8000, 0x807F, 0x8080, 0xBC80, 0xFBFF, 0xFF80,
                        0xFFFF], np.uint16)
    rnd = rng.integers(0, 65536, size=4000).astype(np.uint16)
    allv = np.concatenate([special, rnd])
    _, _, v8 = lm.build_chunk_csr(np.ones((1, allv.size), bool), torch.from_numpy(allv.view(np.float16)), 1 << 16)
    out["fp8_in_u16"] = allv
    out["fp8_out_u8"] = v8.numpy()

    # Elias-Fano: encoded here, decoded by both reference decoders
    for ci, (H, W, tile, dens) in enumerate([(70, 130, 64, 0.02), (64, 64, 64, 0.3), (33, 200, 32, 0.01),
                                             (130, 70, 64, 0.0), (20, 20, 64, 0.9)]):
        mask = rng.random((H, W)) < dens
        meta, bs = O.encode_ef(mask, tile)
        ref_np = lm.decode_elias_fano(meta, bs, (H, W), tile_size=tile)
        use_jit = lm._USE_JIT
        lm._USE_JIT = False
        ref_np2 = lm.decode_elias_fano(meta, bs, (H, W), tile_size=tile)
        lm._USE_JIT = use_jit
        assert np.array_equal(ref_np, ref_np2), "reference EF decoders disagree"
        out[f"ef{ci}_meta"] = np.array([H, W, tile], np.int64)
        out[f"ef{ci}_tile_meta"] = meta
        out[f"ef{ci}_bitstream"] = bs
        out[f"ef{ci}_mask"] = ref_np.astype(bool)

    # TP slicing of an outlier mask + value list
    mask = rng.random((12, 40)) < 0.1
    vals = torch.from_numpy(np.arange(int(mask.sum()), dtype=np.float32).astype(np.float16))
    m_r, v_r = lm.slice_outliers_for_tp(mask, vals, row_slice=(4, 9))
    m_c, v_c = lm.slice_outliers_for_tp(mask, vals, col_slice=(10, 30))
    out["tp_mask"] = mask
    out["tp_vals"] = vals.numpy()
    out["tp_row_mask"], out["tp_row_vals"] = m_r, v_r.numpy()
    out["tp_col_mask"], out["tp_col_vals"] = m_c, v_c.numpy()
    return out


# --------------------------------------------------------------------------- #
# 2. the load path + forward of whole layers
# --------------------------------------------------------------------------- #
PROJ = {"qkv_proj": ["q_proj", "k_proj", "v_proj"], "gate_up_proj": ["gate_proj", "up_proj"],
        "o_proj": ["o_proj"], "down_proj": ["down_proj"]}


def make_checkpoint(rng, shard_rows, K_full, bits, outlier_mode, dens, r, with_m):
    """Checkpoint tensors in the reference's on-disk format, one entry per shard."""
    shards = []
    for N_s in shard_rows:
        W0 = rng.standard_normal((N_s, K_full)) * 0.02
        lut = normal_quantile_lut(rng, W0.std(axis=1))
        lvl = lut.astype(np.float64)
        idx = np.abs(W0[:, :, None] - lvl[:, None, :]).argmin(axis=2).astype(np.uint8)
        spw = 10 if bits == 3 else 32 // bits
        flat = idx.reshape(-1).astype(np.uint32)
        pad = (-flat.size) % spw
        flat = np.concatenate([flat, np.zeros(pad, np.uint32)]).reshape(-1, spw)
        words = np.bitwise_or.reduce(flat << (np.arange(spw, dtype=np.uint32) * bits)[None, :], axis=1)
        mask = rng.random((N_s, K_full)) < dens
        vals = (rng.standard_normal(int(mask.sum())) * 0.1).astype(np.float16)
        sh = {"q_packed": words.astype(np.uint32).view(np.int32), "lut_c": lut,
              "bits": np.array([bits], np.int32), "outlier_values": vals, "mask": mask, "W0": W0}
        if outlier_mode == "ef":
            meta, bs = O.encode_ef(mask, 64)
            sh["ef_tile_size"] = np.array([64], np.int32)
            sh["ef_tile_meta"] = meta
            sh["ef_bitstream"] = bs.view(np.int32)
        elif outlier_mode == "mask1b":
            sh["outlier_mask_1bit"] = np.packbits(mask.reshape(-1))
        A = (rng.standard_normal((r, K_full)) * 0.01).astype(np.float32)
        B = (rng.standard_normal((N_s, r)) * 0.01).astype(np.float32)
        sh["lora_A"], sh["lora_B"] = A, B
        if with_m:
            sh["m"] = (np.linalg.norm(W0, axis=1) * (1 + rng.uniform(-0.1, 0.1, N_s))).astype(np.float32)
        shards.append(sh)
    return shards


def write_adapter(dirname, layer_idx, proj_names, shards, lora_alpha):
    from safetensors.torch import save_file
    os.makedirs(os.path.join(dirname, "lora_adapter_distilled"), exist_ok=True)
    tensors = {}
    for p, sh in zip(proj_names, shards):
        mod = "self_attn" if p in ("q_proj", "k_proj", "v_proj", "o_proj") else "mlp"
        base = f"base_model.model.model.layers.{layer_idx}.{mod}.{p}"
        tensors[f"{base}.lora_A.weight"] = torch.from_numpy(sh["lora_A"])
        tensors[f"{base}.lora_B.weight"] = torch.from_numpy(sh["lora_B"])
        if "m" in sh:
            tensors[f"{base}.lora_magnitude_vector"] = torch.from_numpy(sh["m"])
    save_file(tensors, os.path.join(dirname, "lora_adapter_distilled", "adapter_model.safetensors"))
    with open(os.path.join(dirname, "lora_adapter_distilled", "adapter_config.json"), "w") as f:
        json.dump({"lora_alpha": lora_alpha, "r": int(shards[0]["lora_B"].shape[1])}, f)


def run_reference_load(lm, proj, shards, K_part, tp_rank, tp_size, row_parallel, model_dir):
    from types import SimpleNamespace
    lm._DORA_INDEXED = None
    lm._DORA_CONFIG_CACHE = None
    lm._DORA_WEIGHTS_CACHE = None
    lm.get_tp_info = lambda: (tp_rank, tp_size)
    cfg = SimpleNamespace(bits=int(shards[0]["bits"][0]), model_id=model_dir)
    method = lm.WLQLinearMethod(cfg)
    layer = torch.nn.Module()
    layer.is_row_parallel = row_parallel
    if row_parallel or tp_size == 1:
        parts = [sh["lut_c"].shape[0] for sh in shards]
    else:
        parts = [sh["lut_c"].shape[0] // tp_size for sh in shards]
    method.create_weights(layer, K_part, parts, K_part * (tp_size if row_parallel else 1),
                          sum(parts) * (1 if row_parallel else tp_size), torch.float16)
    layer.vllm_prefix = f"model.layers.3.self_attn.{proj}" if proj in ("qkv_proj", "o_proj") else f"model.layers.3.mlp.{proj}"
    names = ["q_packed", "lut_c", "bits", "outlier_values", "ef_tile_size", "ef_tile_meta", "ef_bitstream",
             "outlier_mask_1bit"]
    shard_ids = {"qkv_proj": ["q", "k", "v"], "gate_up_proj": [0, 1]}.get(proj, [None])
    for sid, sh in zip(shard_ids, shards):
        for nm in names:
            if nm in sh:
                p = getattr(layer, nm)
                if sid is None:
                    p.weight_loader(p, torch.from_numpy(np.ascontiguousarray(sh[nm])))
                else:
                    p.weight_loader(p, torch.from_numpy(np.ascontiguousarray(sh[nm])), sid)
    method.process_weights_after_loading(layer)
    return layer


def reference_forward(layer, x_f32):
    """The reference's apply() with its CUDA op replaced by the reference's own
    dequantize-then-matmul composition (vllm_wlq/linear_method.py:879-897, 946-1009)."""
    import torch.nn.functional as F
    N, K = layer.N, layer.K
    bits = layer.quant_bits
    spw = 10 if bits == 3 else 32 // bits
    q = np.ascontiguousarray(layer.q_packed_aligned.numpy()).view(np.uint32).reshape(N, layer.words_per_row)
    shifts = np.arange(spw, dtype=np.uint32) * bits
    idx = ((q[:, :, None] >> shifts[None, None, :]) & ((1 << bits) - 1)).reshape(N, -1)[:, :K]
    W = torch.gather(layer.lut_c.float(), 1, torch.from_numpy(idx.astype(np.int64)))
    off, cols, vals = layer.chunk_offsets.numpy(), layer.chunk_cols.numpy().astype(np.int64), layer.chunk_vals
    chunk_m = 640 if bits == 3 else 512
    if vals.numel() > 0:
        vf = (vals.to(torch.int32) << 8).to(torch.int16).view(torch.float16).float()
        for n in range(N):
            for c in range(off.shape[1] - 1):
                s0, s1 = off[n, c], off[n, c + 1]
                if s1 > s0:
                    W[n, torch.from_numpy(cols[s0:s1] + c * chunk_m)] = vf[s0:s1]
    x16 = torch.from_numpy(x_f32).to(torch.float16)
    y = x16.double() @ W.double().t()
    h = None
    if layer.has_dora:
        h = F.linear(x16, layer.lora_A_f16).float()
        y = (y + layer.lora_scale * (h.double() @ layer.lora_B.double().t())) * layer.dora_gamma.double()
    return y.numpy(), (None if h is None else h.numpy()), W.to(torch.float16).numpy()


LAYER_CASES = [
    # name, proj, shard_rows(full), K_full, tp_size, tp_rank, outlier_mode, density, r, with_m, M
    ("qkv_tp1_ef", "qkv_proj", [48, 16, 16], 1100, 1, 0, "ef", 0.01, 8, True, 3),
    ("o_tp1_mask1b", "o_proj", [40], 203, 1, 0, "mask1b", 0.03, 4, False, 5),
    ("gateup_tp2_r1_ef", "gate_up_proj", [64, 64], 520, 2, 1, "ef", 0.02, 8, True, 2),
    ("down_tp2_r0_ef", "down_proj", [24], 1100, 2, 0, "ef", 0.01, 8, True, 4),
    ("down_tp2_r1_noout", "down_proj", [24], 1100, 2, 1, "none", 0.0, 8, True, 1),
    ("o_tp1_nodora", "o_proj", [36], 640, 1, 0, "ef", 0.01, 0, False, 6),
]


def layer_vectors(lm, rng, tmpdir):
    out = {}
    for name, proj, rows, K_full, tp, rank, mode, dens, r, with_m, M in LAYER_CASES:
        row_par = proj in ("o_proj", "down_proj")
        K_part = K_full // tp if row_par else K_full
        shards = make_checkpoint(rng, rows, K_full, 4, mode, dens, max(r, 1), with_m)
        mdir = os.path.join(tmpdir, name)
        if r > 0:
            write_adapter(mdir, 3, PROJ[proj], shards, lora_alpha=2 * r)
        else:
            os.makedirs(mdir, exist_ok=True)
        layer = run_reference_load(lm, proj, shards, K_part, rank, tp, row_par, mdir)
        x = rng.standard_normal((M, K_part)).astype(np.float32)
        y, h, Wd = reference_forward(layer, x)
        pre = f"{name}__"
        out[pre + "meta"] = np.array([K_full, K_part, tp, rank, int(row_par), r, M, len(rows)], np.int64)
        for si, sh in enumerate(shards):
            for nm in ["q_packed", "lut_c", "bits", "outlier_values", "ef_tile_size", "ef_tile_meta",
                       "ef_bitstream", "outlier_mask_1bit", "lora_A", "lora_B", "m"]:
                if nm in sh:
                    out[f"{pre}in{si}_{nm}"] = np.ascontiguousarray(sh[nm])
        out[pre + "q_aligned"] = layer.q_packed_aligned.numpy()
        out[pre + "wpr"] = np.array([layer.words_per_row], np.int64)
        out[pre + "lut"] = layer.lut_c.numpy()
        out[pre + "offsets"] = layer.chunk_offsets.numpy()
        out[pre + "cols"] = layer.chunk_cols.numpy()
        out[pre + "vals"] = layer.chunk_vals.numpy()
        out[pre + "has_dora"] = np.array([int(layer.has_dora)], np.int64)
        if layer.has_dora:
            out[pre + "lora_A_f16"] = layer.lora_A_f16.numpy()
            out[pre + "lora_B"] = layer.lora_B.numpy()
            out[pre + "gamma"] = layer.dora_gamma.numpy()
            out[pre + "scale"] = np.array([layer.lora_scale], np.float64)
            out[pre + "h"] = h
        out[pre + "x"] = x
        out[pre + "y"] = y
        out[pre + "W"] = Wd
        print(f"  {name}: N={layer.N} K={layer.K} nnz={layer.chunk_cols.numel()} dora={layer.has_dora}")
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=None, help="reference source tree (default: WLQ_REFERENCE_TREE, else a "
                    "'reference' directory beside this repository)")
    args = ap.parse_args()
    if args.ref is None:
        sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
        from oracle.reference_tree import locate
        args.ref = locate()
        if args.ref is None:
            sys.exit("reference tree not found: pass --ref or set WLQ_REFERENCE_TREE")
    lm = load_reference(args.ref)
    rng = np.random.default_rng(20261201)
    codecs = codec_vectors(lm, rng)
    np.savez_compressed(os.path.join(HERE, "codecs.npz"), **codecs)
    with tempfile.TemporaryDirectory() as td:
        layers = layer_vectors(lm, rng, td)
    np.savez_compressed(os.path.join(HERE, "layers.npz"), **layers)
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
