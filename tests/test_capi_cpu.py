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


# fake device addresses: the checks below fail before any pointer is touched or any CUDA call is made
P = ctypes.c_void_p(0x10000)
P2 = ctypes.c_void_p(0x20000)


def _err():
    return _C.lib().soinfer_last_error().decode()


def test_batch_gemm_and_quantizer_arguments():
    lib = _C.lib()
    # batch-8 GEMM: M <= 8 tokens, strides cover K / N, alignment
    assert lib.soinfer_gemm_w4a16(P, P, P, 2048, P, 6144, 9, 6144, 2048, 128, 16, None) == 1
    assert "M (tokens)" in _err()
    assert lib.soinfer_gemm_w4a16(P, P, P, 2048, P, 6144, 0, 6144, 2048, 128, 16, None) == 0
    assert lib.soinfer_gemm_w4a16(P, P, P, 100, P, 6144, 2, 6144, 2048, 128, 16, None) == 1
    assert "row strides" in _err()
    assert lib.soinfer_gemm_w4a16(P, P, ctypes.c_void_p(0x10001), 2048, P, 6144, 2, 6144, 2048, 128, 16, None) == 1
    assert "misaligned" in _err()
    assert lib.soinfer_gemm_w4a16(P, P, P, 2048, P, 6144, 2, 6144, 2048, 128, 15, None) == 1
    assert "num_groups" in _err()
    # GPU quantizer: dtype, group size, shape
    assert lib.soinfer_quantize_pack_int4(P, 3, 16, 256, 256, 128, P, P, None) == 1 and "dtype" in _err()
    assert lib.soinfer_quantize_pack_int4(P, 0, 16, 256, 256, 12, P, P, None) == 1 and "power of two" in _err()
    assert lib.soinfer_quantize_pack_int4(P, 0, 16, 256, 100, 128, P, P, None) == 1 and "row stride" in _err()
    assert lib.soinfer_quantize_pack_int4(P, 0, 0, 256, 256, 128, P, P, None) == 0


def _task(N=64, K=2048, g=128, dep=-1, y=P2, residual=None, glu=None, norm_w=None, norm_out=None):
    return _C._GemvTask(P, P, P, y, N, K, g, (K + g - 1) // g, dep, residual, glu, norm_w, 1e-6, norm_out)


def _tasks(*ts):
    arr = (_C._GemvTask * len(ts))(*ts)
    return arr, len(ts)


def test_batched_gemv_arguments():
    lib = _C.lib()
    assert lib.soinfer_gemv_batch_workspace_bytes(-1) == 0
    assert lib.soinfer_gemv_batch_workspace_bytes(_C.MAX_BATCH_TASKS + 1) == 0
    assert lib.soinfer_gemv_batch_workspace_bytes(8) >= 9 * 4
    assert lib.soinfer_gemv_w4a16_batch(None, 0, None, 0, None) == 0
    assert lib.soinfer_gemv_w4a16_batch(None, _C.MAX_BATCH_TASKS + 1, None, 0, None) == 1
    assert "num_tasks" in _err()
    assert lib.soinfer_gemv_w4a16_batch(None, 1, None, 0, None) == 1 and "null task list" in _err()
    cases = [
        ((_task(dep=0),), "dep must be -1 or an earlier task"),
        ((_task(y=None),), "null pointer"),  # y == NULL only with peers
        ((_task(g=100),), "multiple of 8"),
        ((_task(N=0),), "N must be >= 1"),
        ((_task(norm_out=P),), "norm_out needs norm_weight"),
        ((_task(norm_w=ctypes.c_void_p(0x10008)),), "norm prologue"),
        # an epilogue input written by an earlier task of the batch must use its row split
        ((_task(N=64, y=P2), _task(N=128, glu=P2)), "N differs"),
        ((_task(N=64, y=P2), _task(N=128, residual=P2)), "N differs"),
    ]
    for ts, msg in cases:
        arr, n = _tasks(*ts)
        assert lib.soinfer_gemv_w4a16_batch(ctypes.addressof(arr), n, None, 0, None) == 1, msg
        assert msg in _err(), (msg, _err())


def _peers(world=2, rank=0, slot=4096, bases=None):
    ps = _C.PeerSetStruct()
    for r in range(world):
        ps.base[r] = (bases[r] if bases is not None else 0x100000 * (r + 1))
    ps.rank, ps.world, ps.slot_bytes = rank, world, slot
    return ps


def test_peer_set_and_exchange_arguments():
    lib = _C.lib()
    assert lib.soinfer_peer_buffer_bytes(8, 2) == 0
    assert lib.soinfer_peer_buffer_bytes(16, 0) == 0
    assert lib.soinfer_peer_buffer_bytes(16, _C.MAX_PEERS + 1) == 0
    assert lib.soinfer_peer_buffer_bytes(1024, 2) == 256 + 2 * 2 * 1024  # header + two parities x world slots
    ar = lib.soinfer_tp_allreduce_add_rmsnorm
    assert ar(None, P, None, None, P2, None, 64, 1e-6, None) == 1 and "null peer set" in _err()
    bad_sets = [
        (_peers(world=0), "world size"),
        (_peers(world=2, rank=2), "rank out of range"),
        (_peers(slot=24), "slot_bytes"),
        (_peers(bases=[0x100000, 0]), "peer buffer 1 null"),
        (_peers(bases=[0x100000, 0x200010]), "256-byte aligned"),
    ]
    for ps, msg in bad_sets:
        assert ar(ctypes.byref(ps), P, None, None, P2, None, 64, 1e-6, None) == 1, msg
        assert msg in _err(), (msg, _err())
    ps = _peers()
    assert ar(ctypes.byref(ps), P, None, None, P2, None, 12, 1e-6, None) == 1 and "multiple of 8" in _err()
    assert ar(ctypes.byref(ps), P, None, None, P2, None, 4096, 1e-6, None) == 1 and "slot_bytes" in _err()
    assert ar(ctypes.byref(ps), P, None, None, None, None, 64, 1e-6, None) == 1 and "null output" in _err()
    assert ar(ctypes.byref(ps), P, None, None, P2, P2, 64, 1e-6, None) == 1 and "weight with out_norm" in _err()
    assert ar(ctypes.byref(ps), ctypes.c_void_p(0x10008), None, None, P2, None, 64, 1e-6, None) == 1
    assert "16-byte aligned" in _err()
    assert lib.soinfer_tp_allgather(ctypes.byref(ps), P, 4096 + 16, P2, None) == 1 and "nbytes" in _err()
    assert lib.soinfer_tp_allgather(ctypes.byref(ps), P, 24, P2, None) == 1 and "nbytes" in _err()
    assert lib.soinfer_tp_argmax(ctypes.byref(ps), P, P, -1, P2, None) == 1 and "offset" in _err()
    assert lib.soinfer_tp_argmax(ctypes.byref(ps), None, P, 0, P2, None) == 1 and "null pointer" in _err()
    tp = lib.soinfer_gemv_w4a16_tp_partial
    assert tp(ctypes.byref(ps), P, P, P, 4096, 2048, 128, 16, None) == 1 and "2N <= slot_bytes" in _err()
    assert tp(ctypes.byref(ps), P, P, P, 64, 2000, 8, 250, None) == 1 and "multiples of 128" in _err()
    # batched tensor-parallel GEMV: one peer task, no epilogue on it
    bt = lib.soinfer_gemv_w4a16_batch_tp
    arr, n = _tasks(_task(y=None), _task(y=None))
    assert bt(ctypes.byref(ps), ctypes.addressof(arr), n, None, 0, None) == 1 and "at most one task" in _err()
    arr, n = _tasks(_task(y=None, residual=P2))
    assert bt(ctypes.byref(ps), ctypes.addressof(arr), n, None, 0, None) == 1 and "no epilogue" in _err()
    arr, n = _tasks(_task(N=4096, y=None))
    assert bt(ctypes.byref(ps), ctypes.addressof(arr), n, None, 0, None) == 1 and "exceed the exchange slot" in _err()


def test_graph_step_bookkeeping_arguments():
    lib = _C.lib()
    # embedding row: sizes and pointers are checked before anything is launched
    assert lib.soinfer_decode_step_embed(P, 0, 2048, P, 16, P, P2, None) == 1 and "invalid sizes" in _err()
    assert lib.soinfer_decode_step_embed(P, 1000, 2048, P, 0, P, P2, None) == 1 and "invalid sizes" in _err()
    assert lib.soinfer_decode_step_embed(P, 1000, 2048, None, 16, P, P2, None) == 1 and "null pointer" in _err()
    assert lib.soinfer_decode_step_embed(P, 1000, 2048, P, 16, None, P2, None) == 1 and "null pointer" in _err()
    # token / position advance
    assert lib.soinfer_decode_step_advance(P, 0, P, P, P, None) == 1 and "ids_len" in _err()
    assert lib.soinfer_decode_step_advance(P, 16, P, P, None, None) == 1 and "null pointer" in _err()
    assert lib.soinfer_decode_step_advance(None, 16, P, P, P, None) == 1 and "null pointer" in _err()


def _fused_layers(n=1, misaligned_weight=False, null_cache=False):
    arr = (_C._FusedLayer * n)()
    for layer in arr:
        for m in range(7):
            layer.Wq[m] = 0x10008 if misaligned_weight else 0x10000
            layer.scale[m] = 0x20000
        layer.input_norm = layer.post_norm = layer.q_norm = layer.k_norm = 0x30000
        layer.k_cache = 0 if null_cache else 0x40000
        layer.v_cache = 0x50000
    return arr


def test_fused_decode_arguments():
    lib = _C.lib()
    f = lib.soinfer_decode_layers_fused
    ok = dict(num_layers=1, hidden=2048, intermediate=6144, heads=16, kv=8, hd=128, g=128, max_seq=64)

    def call(layers, x=P, ws=P, **over):
        a = {**ok, **over}
        return f(ctypes.addressof(layers) if layers is not None else None, a["num_layers"], a["hidden"],
                 a["intermediate"], a["heads"], a["kv"], a["hd"], a["g"], a["max_seq"], ctypes.c_float(1e-6), P, P, P,
                 x, ws, 1 << 24, None)

    layers = _fused_layers()
    assert call(None) == 1 and "null pointer" in _err()
    assert call(layers, max_seq=0) == 1 and "sizes must be positive" in _err()
    # shapes this build does not serve: SOINFER_ERR_UNSUPPORTED, nothing launched
    assert call(layers, hd=64) == 3 and "head_dim 128" in _err()
    assert call(layers, g=64) == 3
    assert call(layers, heads=12) == 3  # not a multiple of num_kv_heads
    assert call(layers, hidden=2000) == 3
    assert call(layers, num_layers=65) == 3 and "64 layers" in _err()
    assert call(layers, x=ctypes.c_void_p(0x10002)) == 1 and "aligned" in _err()
    assert call(_fused_layers(misaligned_weight=True)) == 3 and "16-byte aligned" in _err()
    assert call(_fused_layers(null_cache=True)) == 1 and "null norm weight or cache" in _err()
