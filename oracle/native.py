"""TEST INFRASTRUCTURE ONLY: ctypes access to the oracle's C restatement
(oracle/liboracle.so) and to the reference's own CUDA kernels compiled from
its sources (oracle/_ref/libsoinfer_ref.so, built by `make -C oracle ref`)."""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_P, _I, _I64, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
_oracle = None
_ref = None


def oracle_lib_path() -> str:
    return os.path.join(_HERE, "liboracle.so")


def ref_lib_path() -> str:
    return os.path.join(_HERE, "_ref", "libsoinfer_ref.so")


def oracle_lib():
    global _oracle
    if _oracle is None:
        lib = ctypes.CDLL(oracle_lib_path())
        lib.oracle_topk_ref.argtypes = [_P, _I, _I, _P, _P]
        lib.oracle_topk_ref.restype = None
        lib.oracle_gemv_w4a16.argtypes = [_P, _P, _P, _P, _I64, _I64, _I64, _I]
        lib.oracle_gemv_w4a16.restype = None
        _oracle = lib
    return _oracle


def ref_available() -> bool:
    return os.path.exists(ref_lib_path())


def ref_lib():
    """The reference kernels; every ref_* function launches on the legacy
    default stream (callers synchronize)."""
    global _ref
    if _ref is None:
        lib = ctypes.CDLL(ref_lib_path())
        sigs = {
            "ref_gemv_w4a16_group": [_P, _P, _P, _P, _I, _I, _I, _I],
            "ref_gemv_w4a16_group_lop3": [_P, _P, _P, _P, _I, _I, _I, _I],
            "ref_gemv_w8a16": [_P, _P, _P, _P, _I, _I, _I, _I, _I],
            "ref_topk_threshold_select": [_P, _I, _I, _P, _P],
            "ref_sparse_accumulate": [_P, _P, _P, _P, _I, _I, _I, _I],
            "ref_build_dip_descriptors": [_P, _I, _P, _P, _P, _P],
            "ref_gemv_dip_fused_up": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I],
            "ref_gemv_dip_fused_down": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I],
            "ref_decode_attention": [_P, _P, _P, _P, _I, _I, _I, _I, _I, _F],
            "ref_rmsnorm": [_P, _P, _P, _I, _I, _F],
            "ref_rope_apply": [_P, _P, _P, _I, _I],
        }
        for name, args in sigs.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = None
        _ref = lib
    return _ref


def topk_ref_c(v: np.ndarray, k: int):
    v = np.ascontiguousarray(v, np.float32)
    out = np.empty(k, np.int32)
    cnt = np.zeros(1, np.int32)
    oracle_lib().oracle_topk_ref(v.ctypes.data, v.size, k, out.ctypes.data, cnt.ctypes.data)
    return out, int(cnt[0])


def gemv_w4a16_c(packed: np.ndarray, scale: np.ndarray, x: np.ndarray, K: int, group_size: int, threads: int = 1):
    packed = np.ascontiguousarray(packed, np.uint8)
    scale = np.ascontiguousarray(scale, np.float32)
    x16 = np.ascontiguousarray(x, np.float16).view(np.uint16)
    y = np.empty(packed.shape[0], np.float32)
    oracle_lib().oracle_gemv_w4a16(packed.ctypes.data, scale.ctypes.data, x16.ctypes.data, y.ctypes.data,
                                   packed.shape[0], K, group_size, threads)
    return y
