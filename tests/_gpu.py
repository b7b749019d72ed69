"""Device-side helpers shared by the GPU parity tests: layers from
tests/_layers.py moved to the GPU, seeded inputs, and calls through the
package's reference-compatible entry points."""
import numpy as np
import torch


def C():
    from qwen_wlqfastshot_helen_beta_b200 import _C
    return _C


def dev_layer(L):
    d = "cuda"
    t = {
        "q": torch.from_numpy(L.q.view(np.int32)).to(d),
        "lut": torch.from_numpy(np.ascontiguousarray(L.lut)).to(d),
        "off": None if L.off is None else torch.from_numpy(L.off).to(d),
        "cols": None if L.cols is None else torch.from_numpy(L.cols.astype(np.uint16)).to(d),
        "vals": None if L.vals is None else torch.from_numpy(L.vals).to(d),
        "A": None if L.A is None else torch.from_numpy(L.A).to(d),
        "B": None if L.B is None else torch.from_numpy(L.B).to(d),
        "gamma": None if L.gamma is None else torch.from_numpy(L.gamma).to(d),
    }
    return t


def run_ours(L, T, x, h, gemv=False, fmt=0):
    M = x.shape[0]
    out = torch.full((M, L.N), float("nan"), dtype=x.dtype, device="cuda")
    lut, cols, vals = T["lut"], T["cols"], T["vals"]
    if fmt == 1:
        lut = C().prepack_lut(T["lut"], x.dtype)
        if cols is not None:
            cols, vals = C().prepack_outliers(T["q"], T["lut"], T["off"], T["cols"], T["vals"], L.N, L.K, 4, x.dtype,
                                              L.G, L.goff)
    if gemv:
        C().gemv_forward(T["q"], lut, x, out, L.N, L.K, 4, T["off"], cols, vals, T["B"], h,
                         T["gamma"], L.scale, L.G, L.goff, fmt)
    else:
        C().gemm_forward(x, T["q"], lut, out, L.N, L.K, 4, L.wpr, T["off"], cols, vals, h, T["B"],
                         T["gamma"], L.scale, L.G, L.goff, fmt)
    torch.cuda.synchronize()
    return out


def inputs(rng, L, M, dtype):
    x = torch.from_numpy(rng.standard_normal((M, L.K)).astype(np.float32)).to("cuda", dtype)
    h = None
    if L.A is not None:
        h = torch.nn.functional.linear(x, torch.from_numpy(L.A).to("cuda", dtype)).float()
    return x, h
