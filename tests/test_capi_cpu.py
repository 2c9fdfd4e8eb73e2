"""The C ABI library on a machine without a GPU: it loads, exports every
symbol include/soinfer_b200.h declares, and reports argument errors through
status codes and soinfer_last_error() without touching CUDA (no compute call
is made here)."""
import ctypes
import os
import re

import pytest

from soinfer import _C

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "soinfer_b200.h")


def _declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(soinfer_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = ctypes.CDLL(_C.lib_path())
    declared = _declared_symbols()
    assert len(declared) >= 20
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, f"declared but not exported: {missing}"
    # and the ctypes signature table covers exactly the declared surface
    assert sorted(_C._SIGNATURES) == declared


def test_abi_version_and_status_strings():
    lib = _C.lib()
    assert lib.soinfer_abi_version() == 1
    assert lib.soinfer_status_string(0) == b"SOINFER_OK"
    assert lib.soinfer_status_string(1) == b"SOINFER_ERR_INVALID_ARGUMENT"
    assert lib.soinfer_status_string(99) == b"SOINFER_ERR_UNKNOWN"


@pytest.mark.parametrize("group_size,num_groups,msg", [(7, 1, "multiple of 8"), (32, 3, "num_groups")])
def test_invalid_gemv_arguments_rejected_without_launch(group_size, num_groups, msg):
    lib = _C.lib()
    st = lib.soinfer_gemv_w4a16_group(None, None, None, None, 4, 64, group_size, num_groups, None)
    assert st == 1
    assert msg in lib.soinfer_last_error().decode()


def test_invalid_selector_and_attention_arguments():
    lib = _C.lib()
    assert lib.soinfer_topk_threshold_select(None, 1024, 0, None, None, None) == 1
    assert "k must be in [1, I]" in lib.soinfer_last_error().decode()
    assert lib.soinfer_topk_select_exact(None, 1024, 1025, None, None, None) == 1
    assert lib.soinfer_decode_attention(None, None, None, None, 15, 8, 64, 128, 1, None, 0, None) == 1
    assert "multiple of num_kv_heads" in lib.soinfer_last_error().decode()
    assert lib.soinfer_kv_cache_append(None, None, None, None, 4, 16, 32, 16, None) == 1
    assert "pos out of range" in lib.soinfer_last_error().decode()
    assert lib.soinfer_rmsnorm(None, None, None, 1, 7, 1e-6, None) == 1


def test_sparse_workspace_query_and_empty_calls():
    lib = _C.lib()
    assert lib.soinfer_sparse_workspace_bytes(2048, 3072) > 2048 * 4
    assert lib.soinfer_sparse_workspace_bytes(0, 3072) == 0
    # zero-size requests succeed without a GPU
    assert lib.soinfer_gemv_w4a16_group(None, None, None, None, 0, 64, 32, 2, None) == 0
    assert lib.soinfer_gemv_dip_fused_up(None, None, 0, None, None, 0, None, 0, None, None, 64, 32, 2, None) == 0


def test_host_gather_validates_indices():
    lib = _C.lib()
    matrix = (ctypes.c_uint8 * 64)()
    staging = (ctypes.c_uint8 * 64)()
    idx = (ctypes.c_int64 * 2)(0, 9)
    st = lib.soinfer_gather_rows_staged(matrix, 4, 16, idx, 2, staging, 64, ctypes.c_void_p(1), 64, None)
    assert st == 1 and "out of range" in lib.soinfer_last_error().decode()
