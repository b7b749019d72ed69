"""ctypes binding of libwlq_b200.so, the package's C ABI (include/wlq_b200.h).

The shared library is built in-tree by ``qwen_wlqfastshot_helen_beta_b200/build.py``.
There is no fallback: if it is missing, importing this module raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libwlq_b200.so")

WLQ_OK = 0
WLQ_DTYPE_F16 = 0
WLQ_DTYPE_BF16 = 1
WLQ_LUT_F16 = 0
WLQ_LUT_PREPACKED = 1
ABI_VERSION = 1

_i32, _i64, _f32, _p = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p
_p64 = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); the exact set declared in include/wlq_b200.h
SIGNATURES = {
    "wlq_last_error": (ctypes.c_char_p, []),
    "wlq_abi_version": (_i32, []),
    "wlq_gemv": (_i32, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _f32, _i32, _i32, _i32, _i32, _i32, _i32,
                        _i32, _i32, _i32, _i32, _p]),
    "wlq_gemv_lora_a": (_i32, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _f32, _i32, _i32, _i32, _i32, _i32, _i32,
                               _i32, _i32, _i32, _i32, _p]),
    "wlq_gemm": (_i32, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _f32, _i32, _i32, _i32, _i32, _i32, _i32,
                        _i32, _i32, _i32, _i32, _p]),
    "wlq_lora_h": (_i32, [_p, _p, _p, _i32, _i32, _i32, _i32, _p]),
    "wlq_gemm_workspace_bytes": (ctypes.c_size_t, [_i32]),
    "wlq_gemm_streamk_noalloc": (_i32, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _f32, _i32, _i32, _i32, _i32, _i32,
                                        _i32, _i32, _i32, _i32, _i32, _p]),
    "wlq_gemm_streamk": (_i32, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _f32, _i32, _i32, _i32, _i32, _i32, _i32,
                                _i32, _i32, _i32, _i32, _p, ctypes.c_size_t, _p]),
    "wlq_prepack_lut": (_i32, [_p, _p, _i64, _i32, _p]),
    "wlq_prepack_lut_host": (_i32, [_p, _p, _i64, _i32]),
    "wlq_prepack_outliers": (_i32, [_p, _p, _p, _p, _p, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _p, _p,
                                    _p]),
    "wlq_dequant": (_i32, [_p, _p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _i32, _i32, _p]),
    "wlq_init_workspaces": (_i32, [_i64, _i64, _i32]),
    "wlq_device_error": (_i32, [_i32, ctypes.POINTER(ctypes.c_uint), _i32]),
    "wlq_gemv_set_split": (_i32, [_i32]),
    "wlq_gemv_last_split": (_i32, []),
    "wlq_gemv_last_warps": (_i32, []),
    "wlq_gemv_set_overlap": (_i32, [_i32]),
    "wlq_gemv_get_overlap": (_i32, []),
    "wlq_tp_buffer_bytes": (ctypes.c_size_t, [_i32, _i32]),
    "wlq_tp_buffer_alloc": (_i32, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]),
    "wlq_tp_buffer_open": (_i32, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "wlq_tp_buffer_close": (_i32, [_p]),
    "wlq_tp_buffer_free": (_i32, [_p]),
    "wlq_tp_error": (_i32, [_p, ctypes.POINTER(ctypes.c_uint), _i32]),
    "wlq_gemv_allreduce": (_i32, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _f32, _i32, _i32, _i32, _i32, _i32,
                                  _i32, _i32, _i32, _i32, _i32, ctypes.POINTER(ctypes.c_void_p), _i32, _i32, _i32,
                                  _p]),
    "wlq_words_per_row": (_i64, [_i64, _i32]),
    "wlq_repack_q_indices_row_aligned": (_i32, [_p, _i64, _i64, _i64, _i32, _p, _i64, _p64]),
    "wlq_repack_q_indices_slice": (_i32, [_p, _i64, _i64, _i64, _i32, _i64, _i64, _i64, _i64, _p, _i64, _p64]),
    "wlq_decode_ef_positions": (_i32, [_p, _i64, _p, _i64, _i64, _i64, _i64, _p, _i64, _p64]),
    "wlq_positions_to_chunk_csr": (_i32, [_p, _i64, _i64, _i64, _i64, _p, _p]),
    "wlq_decode_ef_to_chunk_csr": (_i32, [_p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _i64, _p64]),
    "wlq_build_chunk_csr": (_i32, [_p, _i64, _i64, _i64, _p, _p, _i64, _p64]),
    "wlq_fp16_to_fp8_bytes": (_i32, [_p, _i64, _p]),
    "wlq_dequant_host": (_i32, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i32, _i64, _i64, _i64]),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python qwen_wlqfastshot_helen_beta_b200/build.py` "
            "(nvcc for sm_100a); there is no fallback implementation")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.wlq_abi_version() != ABI_VERSION:
        raise ImportError(f"{LIB_PATH}: ABI version {lib.wlq_abi_version()} != {ABI_VERSION}; rebuild it")
    return lib


lib = _load()


class WLQError(RuntimeError):
    """A libwlq_b200 entry point returned a non-zero status."""


def check(rc: int, what: str) -> None:
    if rc != WLQ_OK:
        msg = lib.wlq_last_error().decode(errors="replace")
        raise WLQError(f"{what} failed with status {rc}: {msg}")
