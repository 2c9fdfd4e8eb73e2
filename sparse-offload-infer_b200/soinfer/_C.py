"""Torch-tensor front end of the sm_100a C ABI (libsoinfer_b200.so).

Mirrors the reference's pybind11 module ``soinfer._C`` (csrc/bindings.cpp:26-610
of sparse-offload-infer): the same function names, argument order and
preconditions, each failed precondition raised as ``RuntimeError`` (the
reference's TORCH_CHECK), outputs freshly allocated, and every kernel launched
on torch's *current* CUDA stream of the inputs' device.  The library is bound
with ctypes over plain pointers; no torch type crosses the ABI.

There is no CPU fallback: if the shared library is missing, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_LIB_NAME = "libsoinfer_b200.so"
_lib = None
_lib_error: str | None = None
_lock = threading.Lock()

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_F32 = ctypes.c_float
_INT = ctypes.c_int

# name -> (restype, argtypes); kept in step with include/soinfer_b200.h
_SIGNATURES = {
    "soinfer_abi_version": (_INT, []),
    "soinfer_last_error": (ctypes.c_char_p, []),
    "soinfer_status_string": (ctypes.c_char_p, [_INT]),
    "soinfer_device_errors": (_INT, [_P]),
    "soinfer_gemv_w4a16_group": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _P]),
    "soinfer_gemv_w4a16_group_lop3": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _P]),
    "soinfer_gemv_w4a16_group_ex": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, ctypes.c_uint32, _P]),
    "soinfer_gemv_batch_workspace_bytes": (_I64, [_I64]),
    "soinfer_gemv_w4a16_batch": (_INT, [_P, _I64, _P, _I64, _P]),
    "soinfer_gemv_w4a16_rows": (_INT, [_P, _P, _I64, _P, _I64, _P, _P, _I64, _I64, _I64, _P, _P]),
    "soinfer_gemv_w8a16": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P]),
    "soinfer_topk_threshold_select": (_INT, [_P, _I64, _I64, _P, _P, _P]),
    "soinfer_topk_threshold_select_abs_f16": (_INT, [_P, _I64, _I64, _P, _P, _P]),
    "soinfer_topk_select_exact": (_INT, [_P, _I64, _I64, _P, _P, _P]),
    "soinfer_build_dip_descriptors": (_INT, [_P, _I64, _P, _I64, _P, _P, _P, _P]),
    "soinfer_gemv_dip_fused_up": (_INT, [_P, _P, _I64, _P, _P, _I64, _P, _I64, _P, _P, _I64, _I64, _I64, _P]),
    "soinfer_sparse_workspace_bytes": (_I64, [_I64, _I64]),
    "soinfer_gemv_w4a16_sparse_accumulate": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _I64, _P]),
    "soinfer_gemv_fp16": (_INT, [_P, _P, _P, _I64, _I64, _P]),
    "soinfer_lm_head_argmax_workspace_bytes": (_I64, []),
    "soinfer_gemv_fp16_argmax": (_INT, [_P, _P, _P, _I64, _I64, _P, _P, _I64, _P]),
    "soinfer_gemv_w4a16_sparse_accumulate_noalloc": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _P]),
    "soinfer_gemv_w4a16_sparse_rows": (_INT, [_P, _P, _I64, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _I64, _P, _P]),
    "soinfer_gemv_dip_fused_down": (_INT, [_P, _P, _I64, _P, _P, _I64, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _I64,
                                           _P]),
    "soinfer_gather_rows_staged": (_INT, [_P, _I64, _I64, _P, _I64, _P, _I64, _P, _I64, _P]),
    "soinfer_gather_rows_naive": (_INT, [_P, _I64, _I64, _P, _I64, _P, _I64, _P]),
    "soinfer_gather_rows_device": (_INT, [_P, _I64, _I64, _P, _I64, _P, _P]),
    "soinfer_rmsnorm": (_INT, [_P, _P, _P, _I64, _I64, _F32, _P]),
    "soinfer_rope_apply": (_INT, [_P, _P, _P, _I64, _I64, _P]),
    "soinfer_kv_cache_append": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _P]),
    "soinfer_decode_attention_workspace_bytes": (_I64, [_I64, _I64, _I64]),
    "soinfer_decode_attention": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _I64, _P]),
    "soinfer_add_rmsnorm": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _F32, _P]),
    "soinfer_swiglu": (_INT, [_P, _P, _P, _P, _I64, _P]),
    "soinfer_head_norm_rope": (_INT, [_P, _P, _P, _P, _P, _P, _P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64, _P,
                                      _F32, _P]),
    "soinfer_rope_apply_at": (_INT, [_P, _P, _P, _I64, _I64, _I64, _P, _P]),
    "soinfer_kv_cache_append_at": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _P, _P]),
    "soinfer_decode_step_embed": (_INT, [_P, _I64, _I64, _P, _I64, _P, _P, _P]),
    "soinfer_decode_step_advance": (_INT, [_P, _I64, _P, _P, _P, _P]),
    "soinfer_decode_attention_at": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _P, _I64, _P]),
    "soinfer_quantize_pack_int4": (_INT, [_P, ctypes.c_int32, _I64, _I64, _I64, _I64, _P, _P, _P]),
    "soinfer_gemm_w4a16": (_INT, [_P, _P, _P, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P]),
    "soinfer_peer_buffer_bytes": (_I64, [_I64, ctypes.c_int32]),
    "soinfer_peer_buffer_create": (_INT, [_I64, _P, _P]),
    "soinfer_peer_buffer_open": (_INT, [_P, _P]),
    "soinfer_peer_buffer_close": (_INT, [_P]),
    "soinfer_peer_buffer_destroy": (_INT, [_P]),
    "soinfer_peer_buffer_reset": (_INT, [_P, _P]),
    "soinfer_gather_rows_device_multi": (_INT, [_P, ctypes.c_int32, _P, _P, _I64, _P]),
    "soinfer_gemm_batch_workspace_bytes": (_I64, []),
    "soinfer_decode_fused_workspace_bytes": (_I64, [_I64, _I64, _I64, _I64, _I64]),
    "soinfer_decode_layers_fused": (_INT, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _F32, _P, _P, _P, _P,
                                           _P, _I64, _P]),
    "soinfer_gemm_w4a16_batch": (_INT, [_P, _I64, _I64, _P, _I64, _P]),
    "soinfer_tp_allreduce_add_rmsnorm": (_INT, [_P, _P, _P, _P, _P, _P, _I64, _F32, _P]),
    "soinfer_gemv_w4a16_tp_partial": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _P]),
    "soinfer_gemv_w4a16_batch_tp": (_INT, [_P, _P, _I64, _P, _I64, _P]),
    "soinfer_tp_allgather": (_INT, [_P, _P, _I64, _P, _P]),
    "soinfer_tp_argmax": (_INT, [_P, _P, _P, _I64, _P, _P]),
}


def lib_path() -> str:
    return os.path.join(os.path.dirname(os.path.abspath(__file__)), _LIB_NAME)


def lib():
    """The loaded shared library; raises RuntimeError if it is not built."""
    global _lib, _lib_error
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = lib_path()
            try:
                handle = ctypes.CDLL(path)
            except OSError as exc:
                _lib_error = f"soinfer CUDA library not available at {path}: {exc} (build it with __graft_entry__.build())"
                raise RuntimeError(_lib_error) from exc
            for name, (restype, argtypes) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = handle
    return _lib


def is_available() -> bool:
    try:
        lib()
        return True
    except RuntimeError:
        return False


def last_error() -> str:
    return lib().soinfer_last_error().decode()


def device_errors() -> int:
    """Reads and clears the device-side error bits (bit 0: a bounded copy or
    dependency wait timed out; bit 1: a peer-exchange wait timed out -- a rank
    never signalled).  When any bit is set, a kernel that gave up may have
    left its self-resetting counters dirty, so every cached workspace is
    re-zeroed before this returns (the next launch starts clean).  A peer
    timeout also needs PeerExchange.reset() on every rank."""
    flags = ctypes.c_int(0)
    _call("soinfer_device_errors", ctypes.byref(flags))
    if flags.value:
        torch.cuda.synchronize()
        reset_workspaces()
        torch.cuda.synchronize()
    return flags.value


def _call(fn_name: str, *args) -> None:
    status = getattr(lib(), fn_name)(*args)
    if status != 0:
        msg = lib().soinfer_last_error().decode()
        kind = lib().soinfer_status_string(status).decode()
        raise RuntimeError(f"{msg} [{kind}]")


def _check(cond: bool, *msg) -> None:
    if not cond:
        raise RuntimeError("".join(str(m) for m in msg))


def _check_cuda(t: torch.Tensor, name: str, dtype: torch.dtype, dtype_msg: str) -> None:
    _check(t.is_cuda, name, ": input must be a CUDA tensor")
    _check(t.dtype == dtype, name, dtype_msg)
    _check(t.is_contiguous(), name, ": input must be contiguous")


def _f16(t, name):
    _check_cuda(t, name, torch.float16, ": only float16 is supported")


def _f32(t, name):
    _check_cuda(t, name, torch.float32, ": only float32 is supported")


def _same_device(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts[1:]:
        _check(t.device == dev, "all tensors must be on the same CUDA device, got ", dev, " and ", t.device)
    return dev


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None or t.numel() == 0 else t.data_ptr()


def _cdiv(a: int, b: int) -> int:
    return -(-a // b)


# ---------------------------------------------------------------- workspaces
# One zero-initialised workspace per (kind, device, stream); the kernels leave
# the sparse workspace zeroed again on exit, so it is reused across calls.
_workspaces: dict[tuple, torch.Tensor] = {}


def _workspace(kind: str, dev: torch.device, nbytes: int) -> torch.Tensor:
    key = (kind, dev.index, _stream(dev))
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=dev)
        _workspaces[key] = ws
    return ws


# -------------------------------------------------------------------- GEMVs
FLAG_PDL = 1


def _gemv_w4a16_group_impl(fn: str, name: str, Wq_packed, scale, x, K: int, group_size: int,
                           out: torch.Tensor | None = None, pdl: bool = False) -> torch.Tensor:
    _check(Wq_packed.is_cuda, name, "(Wq_packed): must be a CUDA tensor")
    _check(Wq_packed.dtype == torch.uint8, name, "(Wq_packed): must be uint8 (AWQ-packed int4)")
    _check(Wq_packed.is_contiguous(), name, "(Wq_packed): must be contiguous")
    _check(Wq_packed.dim() == 2, name, "(Wq_packed): must be 2D [N, ceil(K/8)*4]")
    _f16(x, "x")
    _check(x.dim() == 1 and x.size(0) == K, name, ": x must be 1D [K]")
    _check(K >= 1, name, ": K must be >= 1")
    _check(group_size >= 1 and group_size % 8 == 0, name, ": group_size must be a positive multiple of 8")
    N = Wq_packed.size(0)
    _check(Wq_packed.size(1) == _cdiv(K, 8) * 4, name, ": Wq_packed.size(1) must be ceil(K/8)*4 for the given K")
    _check(scale.is_cuda, name, ": scale must be a CUDA tensor")
    _check(scale.dtype == torch.float32, name, ": scale must be float32")
    _check(scale.is_contiguous(), name, ": scale must be contiguous")
    _check(scale.dim() == 2 and scale.size(0) == N, name,
           ": scale must be 2D [N, num_groups] (grouped int4 has no per-tensor broadcast)")
    num_groups = scale.size(1)
    _check(num_groups == _cdiv(K, group_size), name, ": scale's num_groups must be ceil(K/group_size) for the given K "
           "and group_size, got ", num_groups, " but expected ", _cdiv(K, group_size))
    dev = _same_device(Wq_packed, scale, x)
    y = out if out is not None else torch.empty(N, dtype=torch.float16, device=dev)
    with torch.cuda.device(dev):
        if pdl:
            _call("soinfer_gemv_w4a16_group_ex", _ptr(Wq_packed), _ptr(scale), _ptr(x), _ptr(y), N, K, group_size,
                  num_groups, FLAG_PDL, _stream(dev))
        else:
            _call(fn, _ptr(Wq_packed), _ptr(scale), _ptr(x), _ptr(y), N, K, group_size, num_groups, _stream(dev))
    return y


def gemv_w4a16_group(Wq_packed, scale, x, K: int, group_size: int, out=None, pdl: bool = False) -> torch.Tensor:
    return _gemv_w4a16_group_impl("soinfer_gemv_w4a16_group", "gemv_w4a16_group", Wq_packed, scale, x, K, group_size,
                                  out, pdl)


def gemv_w4a16_group_lop3(Wq_packed, scale, x, K: int, group_size: int, out=None, pdl: bool = False) -> torch.Tensor:
    """pdl=True: programmatic dependent launch (only when the weights are not
    written by the kernel preceding this one on the stream)."""
    return _gemv_w4a16_group_impl("soinfer_gemv_w4a16_group_lop3", "gemv_w4a16_group_lop3", Wq_packed, scale, x, K,
                                  group_size, out, pdl)


def _check_fp16_gemv(name, W, x):
    """Reference check_gemv_shapes (csrc/bindings.cpp) + the 16-byte vector-load rule."""
    _f16(W, name + "(W)")
    _f16(x, name + "(x)")
    _check(W.dim() == 2 and W.is_contiguous(), name, ": W must be a contiguous 2D [N, K] tensor")
    _check(x.dim() == 1 and x.is_contiguous(), name, ": x must be a contiguous 1D [K] tensor")
    _check(W.size(1) == x.size(0), name, ": W.size(1) must equal x.size(0)")
    _check(W.size(1) % 8 == 0, name, ": K must be a multiple of 8 (float4-vectorized loads)")
    return _same_device(W, x)


def gemv_fp16_v3(W, x, out=None) -> torch.Tensor:
    """fp16 GEMV, fp32 accumulation (the decode LM head)."""
    dev = _check_fp16_gemv("gemv_fp16_v3", W, x)
    y = out if out is not None else torch.empty(W.size(0), dtype=torch.float16, device=dev)
    with torch.cuda.device(dev):
        _call("soinfer_gemv_fp16", _ptr(W), _ptr(x), _ptr(y), W.size(0), W.size(1), _stream(dev))
    return y


def gemv_fp16_argmax(W, x, logits: bool = False, out_idx=None):
    """Greedy next token: argmax of the fp16 logits W x (lowest index among
    equal maxima), fused into the LM head GEMV.  Returns (idx int32 [1] on the
    device, logits fp16 [N] or None)."""
    dev = _check_fp16_gemv("gemv_fp16_argmax", W, x)
    _check(W.size(0) >= 1, "gemv_fp16_argmax: W must have at least one row")
    idx = out_idx if out_idx is not None else torch.empty(1, dtype=torch.int32, device=dev)
    y = torch.empty(W.size(0), dtype=torch.float16, device=dev) if logits else None
    with torch.cuda.device(dev):
        nbytes = lib().soinfer_lm_head_argmax_workspace_bytes()
        ws = _workspace("argmax", dev, nbytes)
        _call("soinfer_gemv_fp16_argmax", _ptr(W), _ptr(x), _ptr(y), W.size(0), W.size(1), _ptr(idx), ws.data_ptr(),
              ws.numel(), _stream(dev))
    return idx, y


class _GemvTask(ctypes.Structure):
    _fields_ = [("Wq", _P), ("scale", _P), ("x", _P), ("y", _P), ("N", _I64), ("K", _I64), ("group_size", _I64),
                ("num_groups", _I64), ("dep", _I64), ("residual", _P), ("glu_gate", _P), ("norm_weight", _P),
                ("norm_eps", _F32), ("norm_out", _P)]


MAX_BATCH_TASKS = 256


class GemvBatch:
    """A prepared list of INT4 GEMVs run as one persistent kernel
    (soinfer_gemv_w4a16_batch).  tasks: sequence of
    (Wq_packed, scale, x, y, K, group_size, dep[, residual[, glu_gate[, (norm_weight, eps[, norm_out])]]])
    with dep = index of an earlier task whose output feeds this task's x, or
    -1; residual / glu_gate (fp16 [N] or None) add the epilogues
    y = residual + fp16(silu(glu_gate) * fp16(W x)) of the C ABI; a
    (norm_weight fp16 [K], eps) pair multiplies RMSNorm(x) * norm_weight
    instead of x (computed in the kernel; a third element, fp16 [K], receives
    the normalised x).  The tensors
    must stay alive and keep their storage while the batch is used.
    peers (a PeerSetStruct): tensor-parallel batch (soinfer_gemv_w4a16_batch_tp)
    in which one task may have y = None -- its rows go to every rank's
    exchange inbox."""

    def __init__(self, tasks, peers=None):
        n = len(tasks)
        _check(0 < n <= MAX_BATCH_TASKS, "gemv_w4a16_batch: 1 ..", MAX_BATCH_TASKS, " tasks")
        arr = (_GemvTask * n)()
        dev = None
        for i, task in enumerate(tasks):
            W, scale, x, y, K, group_size, dep = task[:7]
            residual = task[7] if len(task) > 7 else None
            glu = task[8] if len(task) > 8 else None
            norm = task[9] if len(task) > 9 else None
            if norm is not None:
                _f16(norm[0], f"gemv_w4a16_batch[task {i}](norm_weight)")
                _check(norm[0].numel() == K, f"gemv_w4a16_batch[task {i}]", ": norm_weight must hold K values")
                if len(norm) > 2 and norm[2] is not None:
                    _f16(norm[2], f"gemv_w4a16_batch[task {i}](norm_out)")
                    _check(norm[2].numel() == K, f"gemv_w4a16_batch[task {i}]", ": norm_out must hold K values")
            name = f"gemv_w4a16_batch[task {i}]"
            _check(W.is_cuda and W.dtype == torch.uint8 and W.is_contiguous() and W.dim() == 2, name,
                   "(Wq_packed): must be a contiguous 2D uint8 CUDA tensor")
            _check(W.size(1) == _cdiv(K, 8) * 4, name, ": Wq_packed.size(1) must be ceil(K/8)*4 for the given K")
            _f32(scale, name + "(scale)")
            _check(scale.dim() == 2 and scale.size(0) == W.size(0), name, ": scale must be 2D [N, num_groups]")
            _f16(x, name + "(x)")
            _check(x.numel() == K, name, ": x must hold K values")
            if y is None:
                _check(peers is not None, name, ": y may be None only in a tensor-parallel batch (peers)")
            else:
                _f16(y, name + "(y)")
                _check(y.numel() == W.size(0), name, ": y must hold N values")
            _check(-1 <= dep < i, name, ": dep must be -1 or an earlier task index")
            for e, en in ((residual, "residual"), (glu, "glu_gate")):
                if e is not None:
                    _f16(e, f"{name}({en})")
                    _check(e.numel() == W.size(0) and e.is_contiguous(), name, f": {en} must hold N values")
            d = _same_device(W, scale, x, *([y] if y is not None else []))
            _check(dev is None or d == dev, name, ": all tasks must be on one device")
            dev = d
            arr[i] = _GemvTask(W.data_ptr(), scale.data_ptr(), x.data_ptr(), _ptr(y), W.size(0), K, group_size,
                               scale.size(1), dep, _ptr(residual), _ptr(glu),
                               _ptr(norm[0]) if norm is not None else None,
                               float(norm[1]) if norm is not None else 0.0,
                               _ptr(norm[2]) if norm is not None and len(norm) > 2 else None)
        self._arr, self.n, self.device = arr, n, dev
        self._keep = [tuple(t) for t in tasks]
        self.peers = peers

    def run(self) -> None:
        dev = self.device
        with torch.cuda.device(dev):
            ws = _workspace("batch", dev, lib().soinfer_gemv_batch_workspace_bytes(self.n))
            if self.peers is None:
                _call("soinfer_gemv_w4a16_batch", ctypes.addressof(self._arr), self.n, ws.data_ptr(), ws.numel(),
                      _stream(dev))
            else:
                _call("soinfer_gemv_w4a16_batch_tp", ctypes.byref(self.peers), ctypes.addressof(self._arr), self.n,
                      ws.data_ptr(), ws.numel(), _stream(dev))


def gemv_w4a16_batch(tasks, peers=None) -> None:
    """Runs the tasks (see GemvBatch) as one persistent kernel on the current stream."""
    GemvBatch(tasks, peers).run()


def reset_workspaces() -> None:
    """Re-zero every cached workspace (needed after a device error left a
    kernel's self-resetting counters dirty; device_errors() calls it)."""
    for ws in _workspaces.values():
        with torch.cuda.device(ws.device):
            ws.zero_()


def gemv_w4a16_rows(Wq_packed, scale, rows, x, K: int, group_size: int, out: torch.Tensor | None = None,
                    glu_gate: torch.Tensor | None = None):
    """Row-indirect INT4 GEMV; glu_gate (fp16 [N]): the output is
    fp16(silu(glu_gate[rows]) * y) (DIP's SwiGLU in the epilogue)."""
    name = "gemv_w4a16_rows"
    _check(Wq_packed.is_cuda and Wq_packed.dtype == torch.uint8 and Wq_packed.is_contiguous() and Wq_packed.dim() == 2,
           name, "(Wq_packed): must be a contiguous 2D uint8 CUDA tensor")
    _check(Wq_packed.size(1) == _cdiv(K, 8) * 4, name, ": Wq_packed.size(1) must be ceil(K/8)*4 for the given K")
    _f32(scale, name + "(scale)")
    _check(scale.dim() == 2 and scale.size(0) == Wq_packed.size(0), name, ": scale must be 2D [N, num_groups]")
    _check_cuda(rows, name + "(rows)", torch.int32, ": must be int32")
    _check(rows.dim() == 1, name, ": rows must be 1D")
    _f16(x, name + "(x)")
    _check(x.dim() == 1 and x.size(0) == K, name, ": x must be 1D [K]")
    if glu_gate is not None:
        _f16(glu_gate, name + "(glu_gate)")
        _check(glu_gate.numel() == Wq_packed.size(0), name, ": glu_gate must hold N values")
    dev = _same_device(Wq_packed, scale, rows, x)
    y = out if out is not None else torch.empty(rows.numel(), dtype=torch.float16, device=dev)
    with torch.cuda.device(dev):
        _call("soinfer_gemv_w4a16_rows", _ptr(Wq_packed), _ptr(scale), Wq_packed.size(0), _ptr(rows), rows.numel(),
              _ptr(x), _ptr(y), K, group_size, scale.size(1), _ptr(glu_gate), _stream(dev))
    return y


def gemv_w8a16(Wq, scale, x, group_size: int) -> torch.Tensor:
    _check(Wq.is_cuda, "gemv_w8a16(Wq): must be a CUDA tensor")
    _check(Wq.dtype == torch.int8, "gemv_w8a16(Wq): must be int8")
    _check(Wq.is_contiguous(), "gemv_w8a16(Wq): must be contiguous")
    _check(Wq.dim() == 2, "gemv_w8a16(Wq): must be 2D [N, K]")
    _f16(x, "gemv_w8a16(x)")
    _check(x.dim() == 1 and x.size(0) == Wq.size(1), "gemv_w8a16: x must be 1D [K] matching Wq's K")
    _check(group_size >= 1, "gemv_w8a16: group_size must be >= 1")
    N, K = Wq.size(0), Wq.size(1)
    _check(scale.is_cuda, "gemv_w8a16: scale must be a CUDA tensor")
    _check(scale.dtype == torch.float32, "gemv_w8a16: scale must be float32")
    _check(scale.is_contiguous(), "gemv_w8a16: scale must be contiguous")
    _check(scale.dim() == 2, "gemv_w8a16: scale must be 2D [N or 1, num_groups]")
    _check(scale.size(0) == N or scale.size(0) == 1,
           "gemv_w8a16: scale.size(0) must be N (per-channel/group) or 1 (per-tensor broadcast)")
    num_groups = scale.size(1)
    row_stride = 0 if scale.size(0) == 1 else num_groups
    _check(num_groups == 1 or group_size % 4 == 0, "gemv_w8a16: group_size must be a multiple of 4 when num_groups > 1")
    _check(num_groups == 1 or num_groups == _cdiv(K, group_size), "gemv_w8a16: scale's num_groups must be 1 or "
           "ceil(K/group_size) for the given K and group_size, got ", num_groups, " but expected ",
           _cdiv(K, group_size))
    dev = _same_device(Wq, scale, x)
    y = torch.empty(N, dtype=torch.float16, device=dev)
    with torch.cuda.device(dev):
        _call("soinfer_gemv_w8a16", _ptr(Wq), _ptr(scale), _ptr(x), _ptr(y), N, K, group_size, num_groups, row_stride,
              _stream(dev))
    return y


# ------------------------------------------------------------- selection
def _topk_impl(fn: str, name: str, abs_g, k: int):
    _f32(abs_g, name + "(abs_g)")
    _check(abs_g.dim() == 1, name, ": abs_g must be 1D [I]")
    n = abs_g.size(0)
    _check(1 <= k <= n, name, ": k must be in [1, I]")
    dev = abs_g.device
    idx = torch.empty(k, dtype=torch.int32, device=dev)
    count = torch.empty(1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _call(fn, _ptr(abs_g), n, k, _ptr(idx), _ptr(count), _stream(dev))
    return idx, count


def topk_threshold_select(abs_g, k: int):
    return _topk_impl("soinfer_topk_threshold_select", "topk_threshold_select", abs_g, k)


def topk_select_exact(abs_g, k: int):
    return _topk_impl("soinfer_topk_select_exact", "topk_select_exact", abs_g, k)


def topk_threshold_select_abs_f16(gate, k: int):
    """The reference selector on |gate| of an fp16 gate vector (no fp32 copy)."""
    name = "topk_threshold_select_abs_f16"
    _f16(gate, name + "(gate)")
    _check(gate.dim() == 1 and gate.is_contiguous(), name, ": gate must be a contiguous 1D [I] tensor")
    n = gate.size(0)
    _check(1 <= k <= n, name, ": k must be in [1, I]")
    dev = gate.device
    idx = torch.empty(k, dtype=torch.int32, device=dev)
    count = torch.empty(1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _call("soinfer_topk_threshold_select_abs_f16", _ptr(gate), n, k, _ptr(idx), _ptr(count), _stream(dev))
    return idx, count


def build_dip_descriptors(selected_indices, slot_of):
    name = "build_dip_descriptors"
    _check(selected_indices.is_cuda and selected_indices.dtype == torch.int32 and selected_indices.dim() == 1
           and selected_indices.is_contiguous(), name, "(selected_indices): must be a contiguous 1D int32 CUDA tensor")
    _check(slot_of.is_cuda and slot_of.dtype == torch.int32 and slot_of.dim() == 1 and slot_of.is_contiguous(),
           name, "(slot_of): must be a contiguous 1D int32 CUDA tensor")
    dev = _same_device(selected_indices, slot_of)
    k = selected_indices.size(0)
    desc = torch.empty(k, dtype=torch.int32, device=dev)
    miss = torch.empty(k, dtype=torch.int32, device=dev)
    count = torch.empty(1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _call("soinfer_build_dip_descriptors", _ptr(selected_indices), k, _ptr(slot_of), slot_of.numel(), _ptr(desc),
              _ptr(miss), count.data_ptr(), _stream(dev))
    return desc, miss, count


# ------------------------------------------------------- DIP fused GEMVs
def _check_dip_common(cache_Wq, cache_scale, staging_Wq, staging_scale, descriptors, row_dim: int, name: str):
    expected = _cdiv(row_dim, 8) * 4
    _check(cache_Wq.is_cuda and cache_Wq.dtype == torch.uint8 and cache_Wq.dim() == 2 and cache_Wq.is_contiguous()
           and cache_Wq.size(1) == expected, name,
           "(cache_Wq): must be a contiguous 2D uint8 CUDA tensor [C, ceil(row_dim/8)*4]")
    _check(staging_Wq.is_cuda and staging_Wq.dtype == torch.uint8 and staging_Wq.dim() == 2
           and staging_Wq.is_contiguous() and staging_Wq.size(1) == expected, name,
           "(staging_Wq): must be a contiguous 2D uint8 CUDA tensor [M, ceil(row_dim/8)*4]")
    _check(cache_scale.is_cuda and cache_scale.dtype == torch.float32 and cache_scale.dim() == 2
           and cache_scale.is_contiguous(), name, "(cache_scale): must be a contiguous 2D float32 CUDA tensor")
    _check(staging_scale.is_cuda and staging_scale.dtype == torch.float32 and staging_scale.dim() == 2
           and staging_scale.is_contiguous(), name, "(staging_scale): must be a contiguous 2D float32 CUDA tensor")
    _check(cache_scale.size(1) == staging_scale.size(1), name,
           ": cache_scale and staging_scale must have the same num_groups")
    _check(cache_scale.size(0) == cache_Wq.size(0) and staging_scale.size(0) == staging_Wq.size(0), name,
           ": scale rows must match weight rows")
    _check(descriptors.is_cuda and descriptors.dtype == torch.int32 and descriptors.dim() == 1
           and descriptors.is_contiguous(), name, "(descriptors): must be a contiguous 1D int32 CUDA tensor")


def gemv_dip_fused_up(cache_Wq, cache_scale, staging_Wq, staging_scale, descriptors, x, K: int, group_size: int,
                      out: torch.Tensor | None = None):
    name = "gemv_dip_fused_up"
    _check_dip_common(cache_Wq, cache_scale, staging_Wq, staging_scale, descriptors, K, name)
    _f16(x, "gemv_dip_fused_up(x)")
    _check(x.dim() == 1 and x.size(0) == K, name, ": x must be 1D [K]")
    _check(group_size >= 1 and group_size % 8 == 0, name, ": group_size must be a positive multiple of 8")
    num_groups = cache_scale.size(1)
    _check(num_groups == _cdiv(K, group_size), name, ": cache_scale/staging_scale's num_groups must be "
           "ceil(K/group_size) for the given K and group_size, got ", num_groups, " but expected ",
           _cdiv(K, group_size))
    dev = _same_device(cache_Wq, cache_scale, staging_Wq, staging_scale, descriptors, x)
    k = descriptors.size(0)
    y = out if out is not None else torch.empty(k, dtype=torch.float16, device=dev)
    with torch.cuda.device(dev):
        _call("soinfer_gemv_dip_fused_up", _ptr(cache_Wq), _ptr(cache_scale), cache_Wq.size(0), _ptr(staging_Wq),
              _ptr(staging_scale), staging_Wq.size(0), _ptr(descriptors), k, _ptr(x), _ptr(y), K, group_size,
              num_groups, _stream(dev))
    return y


def _sparse_ws(dev, H: int, k: int):
    nbytes = lib().soinfer_sparse_workspace_bytes(H, max(k, 1))
    ws = _workspace("sparse", dev, nbytes)
    return ws.data_ptr(), ws.numel()


def _sparse_accumulate_args(name, Wq_selected, scale_selected, h_selected, H, group_size, out):
    """Reference-style argument checks of the sparse accumulate ops; returns (k, num_groups, device, y)."""
    _check(Wq_selected.is_cuda and Wq_selected.dtype == torch.uint8 and Wq_selected.is_contiguous(), name,
           "(Wq_selected): must be a contiguous CUDA uint8 tensor")
    _check(Wq_selected.dim() == 2, name, "(Wq_selected): must be 2D [k, ceil(H/8)*4]")
    _check(H >= 1, name, ": H must be >= 1")
    _check(group_size >= 1 and group_size % 8 == 0, name, ": group_size must be a positive multiple of 8")
    k = Wq_selected.size(0)
    _check(Wq_selected.size(1) == _cdiv(H, 8) * 4, name, ": Wq_selected.size(1) must be ceil(H/8)*4 for the given H")
    _check(scale_selected.is_cuda and scale_selected.dtype == torch.float32 and scale_selected.is_contiguous(), name,
           "(scale_selected): must be a contiguous CUDA float32 tensor")
    _check(scale_selected.dim() == 2 and scale_selected.size(0) == k, name,
           ": scale_selected must be 2D [k, num_groups]")
    _f16(h_selected, "gemv_w4a16_sparse_accumulate(h_selected)")
    _check(h_selected.dim() == 1 and h_selected.size(0) == k, name, ": h_selected must be 1D [k]")
    num_groups = scale_selected.size(1)
    _check(num_groups == _cdiv(H, group_size), name, ": scale_selected's num_groups must be ceil(H/group_size) for "
           "the given H and group_size, got ", num_groups, " but expected ", _cdiv(H, group_size))
    dev = _same_device(Wq_selected, scale_selected, h_selected)
    y = out if out is not None else torch.empty(H, dtype=torch.float16, device=dev)
    return k, num_groups, dev, y


def gemv_w4a16_sparse_accumulate(Wq_selected, scale_selected, h_selected, H: int, group_size: int,
                                 out: torch.Tensor | None = None):
    name = "gemv_w4a16_sparse_accumulate"
    k, num_groups, dev, y = _sparse_accumulate_args(name, Wq_selected, scale_selected, h_selected, H, group_size, out)
    with torch.cuda.device(dev):
        ws, wsb = _sparse_ws(dev, H, k)
        _call("soinfer_gemv_w4a16_sparse_accumulate", _ptr(Wq_selected), _ptr(scale_selected), _ptr(h_selected),
              _ptr(y), H, k, group_size, num_groups, ws, wsb, _stream(dev))
    return y


def gemv_w4a16_sparse_accumulate_noalloc(Wq_selected, scale_selected, h_selected, H: int, group_size: int,
                                         out: torch.Tensor | None = None):
    """gemv_w4a16_sparse_accumulate with the kernel's scratch in a per-device
    static device array instead of a workspace (no reference counterpart).
    Calls that overlap in time on one device race on that scratch; make the
    first call on a device before capturing a CUDA graph."""
    name = "gemv_w4a16_sparse_accumulate_noalloc"
    k, num_groups, dev, y = _sparse_accumulate_args(name, Wq_selected, scale_selected, h_selected, H, group_size, out)
    with torch.cuda.device(dev):
        _call("soinfer_gemv_w4a16_sparse_accumulate_noalloc", _ptr(Wq_selected), _ptr(scale_selected),
              _ptr(h_selected), _ptr(y), H, k, group_size, num_groups, _stream(dev))
    return y


def gemv_w4a16_sparse_rows(Wq_T, scale_T, rows, h_selected, H: int, group_size: int,
                           out: torch.Tensor | None = None, residual: torch.Tensor | None = None):
    """Row-indirect sparse down GEMV; residual (fp16 [H]): the output is
    fp16(residual + y) (the layer's residual add in the epilogue)."""
    name = "gemv_w4a16_sparse_rows"
    _check(Wq_T.is_cuda and Wq_T.dtype == torch.uint8 and Wq_T.is_contiguous() and Wq_T.dim() == 2, name,
           "(Wq_T): must be a contiguous 2D uint8 CUDA tensor")
    _check(Wq_T.size(1) == _cdiv(H, 8) * 4, name, ": Wq_T.size(1) must be ceil(H/8)*4 for the given H")
    _f32(scale_T, name + "(scale_T)")
    _check(scale_T.dim() == 2 and scale_T.size(0) == Wq_T.size(0), name, ": scale_T must be 2D [I, num_groups]")
    _check_cuda(rows, name + "(rows)", torch.int32, ": must be int32")
    _f16(h_selected, name + "(h_selected)")
    k = rows.numel()
    _check(h_selected.dim() == 1 and h_selected.size(0) == k, name, ": h_selected must be 1D [k]")
    if residual is not None:
        _f16(residual, name + "(residual)")
        _check(residual.numel() == H, name, ": residual must hold H values")
    dev = _same_device(Wq_T, scale_T, rows, h_selected)
    y = out if out is not None else torch.empty(H, dtype=torch.float16, device=dev)
    with torch.cuda.device(dev):
        ws, wsb = _sparse_ws(dev, H, k)
        _call("soinfer_gemv_w4a16_sparse_rows", _ptr(Wq_T), _ptr(scale_T), Wq_T.size(0), _ptr(rows), _ptr(h_selected),
              _ptr(y), H, k, group_size, scale_T.size(1), ws, wsb, _ptr(residual), _stream(dev))
    return y


def gemv_dip_fused_down(cache_Wq, cache_scale, staging_Wq, staging_scale, descriptors, h_selected, H: int,
                        group_size: int, out: torch.Tensor | None = None):
    name = "gemv_dip_fused_down"
    _check_dip_common(cache_Wq, cache_scale, staging_Wq, staging_scale, descriptors, H, name)
    _f16(h_selected, "gemv_dip_fused_down(h_selected)")
    k = descriptors.size(0)
    _check(h_selected.dim() == 1 and h_selected.size(0) == k, name, ": h_selected must be 1D [k]")
    _check(H >= 1, name, ": H must be >= 1")
    _check(group_size >= 1 and group_size % 8 == 0, name, ": group_size must be a positive multiple of 8")
    num_groups = cache_scale.size(1)
    _check(num_groups == _cdiv(H, group_size), name, ": cache_scale/staging_scale's num_groups must be "
           "ceil(H/group_size) for the given H and group_size, got ", num_groups, " but expected ",
           _cdiv(H, group_size))
    dev = _same_device(cache_Wq, cache_scale, staging_Wq, staging_scale, descriptors, h_selected)
    y = out if out is not None else torch.empty(H, dtype=torch.float16, device=dev)
    with torch.cuda.device(dev):
        ws, wsb = _sparse_ws(dev, H, k)
        _call("soinfer_gemv_dip_fused_down", _ptr(cache_Wq), _ptr(cache_scale), cache_Wq.size(0), _ptr(staging_Wq),
              _ptr(staging_scale), staging_Wq.size(0), _ptr(descriptors), _ptr(h_selected), _ptr(y), H, k, group_size,
              num_groups, ws, wsb, _stream(dev))
    return y


# ------------------------------------------------------------------ gathers
def _check_gather_common(matrix, indices, gpu_dst, name):
    _check(matrix.device.type == "cpu" and matrix.is_pinned(), name, "(matrix): must be pinned host memory")
    _check(matrix.dtype == torch.uint8 and matrix.dim() == 2 and matrix.is_contiguous(), name,
           "(matrix): must be a contiguous 2D uint8 tensor [num_rows, row_nbytes]")
    _check(indices.device.type == "cpu" and indices.dtype == torch.int64 and indices.dim() == 1, name,
           "(indices): must be a 1D int64 CPU tensor")
    _check(gpu_dst.is_cuda and gpu_dst.dtype == torch.uint8 and gpu_dst.is_contiguous(), name,
           "(gpu_dst): must be a contiguous CUDA uint8 tensor")
    k = indices.size(0)
    _check(gpu_dst.numel() >= k * matrix.size(1), name, "(gpu_dst): too small for k * row_nbytes bytes")


def gather_rows_staged(matrix, indices, staging, gpu_dst) -> None:
    name = "gather_rows_staged"
    _check_gather_common(matrix, indices, gpu_dst, name)
    _check(staging.device.type == "cpu" and staging.is_pinned() and staging.dtype == torch.uint8,
           "gather_rows_staged(staging): must be pinned host uint8 memory")
    k, rb = indices.size(0), matrix.size(1)
    _check(staging.numel() >= k * rb, "gather_rows_staged(staging): too small for k * row_nbytes bytes")
    indices = indices.contiguous()
    dev = gpu_dst.device
    with torch.cuda.device(dev):
        _call("soinfer_gather_rows_staged", _ptr(matrix), matrix.size(0), rb, _ptr(indices), k, _ptr(staging),
              staging.numel(), _ptr(gpu_dst), gpu_dst.numel(), _stream(dev))


def gather_rows_naive(matrix, indices, gpu_dst) -> None:
    name = "gather_rows_naive"
    _check_gather_common(matrix, indices, gpu_dst, name)
    indices = indices.contiguous()
    dev = gpu_dst.device
    with torch.cuda.device(dev):
        _call("soinfer_gather_rows_naive", _ptr(matrix), matrix.size(0), matrix.size(1), _ptr(indices),
              indices.size(0), _ptr(gpu_dst), gpu_dst.numel(), _stream(dev))


def gather_rows_device(matrix, rows, gpu_dst) -> None:
    """Device-driven gather of rows `rows` (int32 CUDA) of `matrix` (CUDA, or
    pinned host memory read zero-copy) into gpu_dst (CUDA uint8)."""
    name = "gather_rows_device"
    _check(matrix.dtype == torch.uint8 and matrix.dim() == 2 and matrix.is_contiguous(), name,
           "(matrix): must be a contiguous 2D uint8 tensor")
    _check(matrix.is_cuda or matrix.is_pinned(), name, "(matrix): must be CUDA or pinned host memory")
    _check_cuda(rows, name + "(rows)", torch.int32, ": must be int32")
    _check(gpu_dst.is_cuda and gpu_dst.dtype == torch.uint8 and gpu_dst.is_contiguous(), name,
           "(gpu_dst): must be a contiguous CUDA uint8 tensor")
    k, rb = rows.numel(), matrix.size(1)
    _check(gpu_dst.numel() >= k * rb, name, "(gpu_dst): too small for k * row_nbytes bytes")
    dev = gpu_dst.device
    with torch.cuda.device(dev):
        _call("soinfer_gather_rows_device", _ptr(matrix), matrix.size(0), rb, _ptr(rows), k, _ptr(gpu_dst),
              _stream(dev))


class _GatherSrc(ctypes.Structure):
    _fields_ = [("matrix", _P), ("num_rows", _I64), ("row_nbytes", _I64), ("dst", _P)]


def gather_rows_device_multi(pairs, rows, count=None, max_k: int | None = None) -> None:
    """One launch gathering rows[j] of every (matrix, dst) pair for
    j < min(count[0], max_k) (count: int32 [1] CUDA, read on the device; None:
    max_k rows).  matrix: 2D uint8 (CUDA or pinned host, read zero-copy) or any
    contiguous 2D tensor viewed as bytes per row; dst: CUDA, >= max_k rows."""
    name = "gather_rows_device_multi"
    _check(1 <= len(pairs) <= 4, name, ": 1 to 4 (matrix, dst) pairs")
    _check_cuda(rows, name + "(rows)", torch.int32, ": must be int32")
    max_k = rows.numel() if max_k is None else max_k
    _check(0 <= max_k <= rows.numel(), name, ": max_k must be in [0, rows.numel()]")
    if count is not None:
        _check_cuda(count, name + "(count)", torch.int32, ": must be int32")
    arr = (_GatherSrc * len(pairs))()
    dev = rows.device
    for i, (m, d) in enumerate(pairs):
        _check(m.dim() == 2 and m.is_contiguous() and (m.is_cuda or m.is_pinned()), name,
               f"(matrix {i}): must be a contiguous 2D CUDA or pinned host tensor")
        rb = m.size(1) * m.element_size()
        _check(d.is_cuda and d.is_contiguous() and d.device == dev, name, f"(dst {i}): must be a contiguous CUDA tensor "
               "on the rows' device")
        _check(d.numel() * d.element_size() >= max_k * rb, name, f"(dst {i}): too small for max_k rows")
        arr[i] = _GatherSrc(m.data_ptr(), m.size(0), rb, d.data_ptr())
    with torch.cuda.device(dev):
        _call("soinfer_gather_rows_device_multi", ctypes.addressof(arr), len(pairs), _ptr(rows), _ptr(count), max_k,
              _stream(dev))


# ----------------------------------------------------- attention-side glue
def rmsnorm(x, weight, eps: float = 1e-6) -> torch.Tensor:
    _f16(x, "rmsnorm(x)")
    _f16(weight, "rmsnorm(weight)")
    _check(x.dim() == 2, "rmsnorm: x must be 2D [rows, hidden]")
    _check(weight.dim() == 1 and weight.size(0) == x.size(1), "rmsnorm: weight shape must match x's hidden dim")
    _check(x.size(1) % 2 == 0, "rmsnorm: hidden dim must be even (half2 vectorization)")
    dev = _same_device(x, weight)
    out = torch.empty_like(x)
    with torch.cuda.device(dev):
        _call("soinfer_rmsnorm", _ptr(x), _ptr(weight), _ptr(out), x.size(0), x.size(1), float(eps), _stream(dev))
    return out


def rope_apply(x, cos_vals, sin_vals) -> None:
    _f16(x, "rope_apply(x)")
    _check(x.dim() == 2, "rope_apply: x must be 2D [num_heads, head_dim]")
    _check(x.size(1) % 2 == 0, "rope_apply: head_dim must be even")
    _check(cos_vals.is_cuda and cos_vals.dtype == torch.float32 and cos_vals.is_contiguous(),
           "rope_apply: cos_vals must be a contiguous float32 CUDA tensor")
    _check(sin_vals.shape == cos_vals.shape and sin_vals.is_cuda and sin_vals.dtype == torch.float32
           and sin_vals.is_contiguous(), "rope_apply: sin_vals must match cos_vals (contiguous float32 CUDA, same shape)")
    _check(cos_vals.dim() == 1 and cos_vals.size(0) == x.size(1) // 2,
           "rope_apply: cos_vals/sin_vals must be 1D [head_dim / 2]")
    dev = _same_device(x, cos_vals, sin_vals)
    with torch.cuda.device(dev):
        _call("soinfer_rope_apply", _ptr(x), _ptr(cos_vals), _ptr(sin_vals), x.size(0), x.size(1), _stream(dev))


def kv_cache_append(k_cache, v_cache, k_new, v_new, pos: int) -> None:
    for t, n in ((k_cache, "k_cache"), (v_cache, "v_cache"), (k_new, "k_new"), (v_new, "v_new")):
        _f16(t, f"kv_cache_append({n})")
    _check(k_cache.dim() == 3 and v_cache.shape == k_cache.shape,
           "kv_cache_append: k_cache/v_cache must be 3D [num_kv_heads, max_seq_len, head_dim] and same shape")
    _check(k_new.shape == v_new.shape, "kv_cache_append: k_new/v_new must have the same shape")
    _check(k_new.dim() == 2 and k_new.size(0) == k_cache.size(0) and k_new.size(1) == k_cache.size(2),
           "kv_cache_append: k_new/v_new must be 2D [num_kv_heads, head_dim] matching the cache")
    nkv, max_seq, hd = k_cache.shape
    _check(0 <= pos < max_seq, "kv_cache_append: pos out of range for max_seq_len")
    dev = _same_device(k_cache, v_cache, k_new, v_new)
    with torch.cuda.device(dev):
        _call("soinfer_kv_cache_append", _ptr(k_cache), _ptr(v_cache), _ptr(k_new), _ptr(v_new), nkv, max_seq, hd,
              pos, _stream(dev))


def _check_pos_dev(pos_dev, name):
    _check(pos_dev.is_cuda and pos_dev.dtype == torch.int32 and pos_dev.numel() == 1, name,
           "(pos_dev): must be a one-element int32 CUDA tensor")


def decode_step_embed(embed, ids, pos_dev, x) -> None:
    """x [hidden] = embed[ids[*pos_dev]] on the device (the graph decode step's
    input row); an out-of-range position or token id writes nothing."""
    name = "decode_step_embed"
    _f16(embed, f"{name}(embed)")
    _f16(x, f"{name}(x)")
    _check(embed.dim() == 2 and embed.is_contiguous(), name, "(embed): must be a contiguous 2D [vocab, hidden] tensor")
    _check(x.is_contiguous() and x.numel() == embed.size(1), name, "(x): must be contiguous with hidden elements")
    _check(ids.is_cuda and ids.dtype == torch.int32 and ids.dim() == 1 and ids.is_contiguous(), name,
           "(ids): must be a contiguous 1D int32 CUDA tensor")
    _check_pos_dev(pos_dev, name)
    dev = _same_device(embed, ids, pos_dev, x)
    with torch.cuda.device(dev):
        _call("soinfer_decode_step_embed", _ptr(embed), embed.size(0), embed.size(1), _ptr(ids), ids.numel(),
              _ptr(pos_dev), _ptr(x), _stream(dev))


def decode_step_advance(ids, pos_dev, prompt_len, next_token) -> None:
    """ids[*pos_dev + 1] = *next_token unless that position is still in the
    prompt (< *prompt_len), then *pos_dev += 1 -- on the device."""
    name = "decode_step_advance"
    _check(ids.is_cuda and ids.dtype == torch.int32 and ids.dim() == 1 and ids.is_contiguous(), name,
           "(ids): must be a contiguous 1D int32 CUDA tensor")
    for t, n in ((pos_dev, "pos_dev"), (prompt_len, "prompt_len"), (next_token, "next_token")):
        _check(t.is_cuda and t.dtype == torch.int32 and t.numel() == 1, name,
               f"({n}): must be a one-element int32 CUDA tensor")
    dev = _same_device(ids, pos_dev, prompt_len, next_token)
    with torch.cuda.device(dev):
        _call("soinfer_decode_step_advance", _ptr(ids), ids.numel(), _ptr(pos_dev), _ptr(prompt_len),
              _ptr(next_token), _stream(dev))


def add_rmsnorm(x, x2, weight, eps: float = 1e-6):
    """(rmsnorm(fp16(x + x2)), fp16(x + x2)); x, x2: fp16 [rows, hidden]."""
    name = "add_rmsnorm"
    for t, n in ((x, "x"), (x2, "x2"), (weight, "weight")):
        _f16(t, f"{name}({n})")
    _check(x.dim() == 2 and x.is_contiguous() and x2.shape == x.shape and x2.is_contiguous(), name,
           ": x and x2 must be contiguous 2D [rows, hidden] of the same shape")
    _check(weight.dim() == 1 and weight.size(0) == x.size(1), name, ": weight shape must match x's hidden dim")
    _check(x.size(1) % 2 == 0, name, ": hidden dim must be even")
    dev = _same_device(x, x2, weight)
    out, sum_out = torch.empty_like(x), torch.empty_like(x)
    with torch.cuda.device(dev):
        _call("soinfer_add_rmsnorm", _ptr(x), _ptr(x2), _ptr(weight), _ptr(out), _ptr(sum_out), x.size(0), x.size(1),
              float(eps), _stream(dev))
    return out, sum_out


def swiglu(gate, up, idx=None) -> torch.Tensor:
    """fp16(silu(float(gate[idx])) * float(up)); idx (int32) may be None (gate itself)."""
    name = "swiglu"
    _f16(gate, name + "(gate)")
    _f16(up, name + "(up)")
    _check(gate.is_contiguous() and up.is_contiguous() and up.dim() == 1 and gate.dim() == 1, name,
           ": gate and up must be contiguous 1D tensors")
    if idx is None:
        _check(gate.numel() == up.numel(), name, ": gate and up must have the same length")
    else:
        _check_cuda(idx, name + "(idx)", torch.int32, ": must be int32")
        _check(idx.numel() == up.numel(), name, ": idx and up must have the same length")
    dev = _same_device(gate, up) if idx is None else _same_device(gate, up, idx)
    out = torch.empty_like(up)
    with torch.cuda.device(dev):
        _call("soinfer_swiglu", _ptr(gate), _ptr(up), _ptr(idx), _ptr(out), up.numel(), _stream(dev))
    return out


def head_norm_rope(q, k, v, q_norm, k_norm, cos_vals, sin_vals, k_cache, v_cache, pos: int = 0, pos_dev=None,
                   eps: float = 1e-6) -> None:
    """Per-head RMSNorm + RoPE of q (in place) and k, then k / v appended to the
    caches at pos (or *pos_dev with cos / sin tables [max_pos, head_dim/2])."""
    name = "head_norm_rope"
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (q_norm, "q_norm"), (k_norm, "k_norm"), (k_cache, "k_cache"),
                 (v_cache, "v_cache")):
        _f16(t, f"{name}({n})")
        _check(t.is_contiguous(), name, f"({n}): must be contiguous")
    _check(q.dim() == 2 and k.dim() == 2 and v.shape == k.shape and k_cache.dim() == 3 and v_cache.shape == k_cache.shape,
           name, ": q [NQ, hd], k / v [NKV, hd], caches [NKV, max_seq, hd]")
    nq, hd = q.shape
    nkv, max_seq, chd = k_cache.shape
    _check(k.size(0) == nkv and k.size(1) == hd and chd == hd, name, ": head counts / head_dim disagree")
    _check(q_norm.numel() == hd and k_norm.numel() == hd, name, ": q_norm / k_norm must be [head_dim]")
    for t, n in ((cos_vals, "cos"), (sin_vals, "sin")):
        _f32(t, f"{name}({n})")
        _check(t.is_contiguous() and t.size(-1) == hd // 2, name, f"({n}): last dim must be head_dim / 2")
    if pos_dev is None:
        _check(0 <= pos < max_seq, name, ": pos out of range for max_seq_len")
        table_rows = 1
    else:
        _check_pos_dev(pos_dev, name)
        _check(cos_vals.dim() == 2, name, ": with pos_dev, cos / sin must be tables [max_pos, head_dim/2]")
        table_rows = cos_vals.size(0)
    dev = _same_device(q, k, v, k_cache)
    with torch.cuda.device(dev):
        _call("soinfer_head_norm_rope", _ptr(q), _ptr(k), _ptr(v), _ptr(q_norm), _ptr(k_norm), _ptr(cos_vals),
              _ptr(sin_vals), table_rows, _ptr(k_cache), _ptr(v_cache), nq, nkv, hd, max_seq, pos, _ptr(pos_dev),
              float(eps), _stream(dev))


def rope_apply_at(x, cos_table, sin_table, pos_dev) -> None:
    """rope_apply with the position read on the device: row *pos_dev of the
    fp32 tables [max_pos, head_dim / 2] (capturable in a CUDA graph)."""
    name = "rope_apply_at"
    _f16(x, name + "(x)")
    _check(x.dim() == 2 and x.size(1) % 2 == 0, name, ": x must be 2D [num_heads, even head_dim]")
    for t, n in ((cos_table, "cos_table"), (sin_table, "sin_table")):
        _f32(t, f"{name}({n})")
        _check(t.dim() == 2 and t.size(1) == x.size(1) // 2 and t.is_contiguous(), name,
               f"({n}): must be contiguous 2D [max_pos, head_dim / 2]")
    _check(sin_table.shape == cos_table.shape, name, ": cos_table and sin_table must have the same shape")
    _check_pos_dev(pos_dev, name)
    dev = _same_device(x, cos_table, sin_table, pos_dev)
    with torch.cuda.device(dev):
        _call("soinfer_rope_apply_at", _ptr(x), _ptr(cos_table), _ptr(sin_table), cos_table.size(0), x.size(0),
              x.size(1), _ptr(pos_dev), _stream(dev))


def kv_cache_append_at(k_cache, v_cache, k_new, v_new, pos_dev) -> None:
    """kv_cache_append at position *pos_dev (read on the device)."""
    name = "kv_cache_append_at"
    for t, n in ((k_cache, "k_cache"), (v_cache, "v_cache"), (k_new, "k_new"), (v_new, "v_new")):
        _f16(t, f"{name}({n})")
    _check(k_cache.dim() == 3 and v_cache.shape == k_cache.shape, name,
           ": k_cache/v_cache must be 3D [num_kv_heads, max_seq_len, head_dim] and same shape")
    _check(k_new.shape == v_new.shape and k_new.dim() == 2 and k_new.size(0) == k_cache.size(0)
           and k_new.size(1) == k_cache.size(2), name, ": k_new/v_new must be 2D [num_kv_heads, head_dim]")
    _check_pos_dev(pos_dev, name)
    nkv, max_seq, hd = k_cache.shape
    dev = _same_device(k_cache, v_cache, k_new, v_new, pos_dev)
    with torch.cuda.device(dev):
        _call("soinfer_kv_cache_append_at", _ptr(k_cache), _ptr(v_cache), _ptr(k_new), _ptr(v_new), nkv, max_seq, hd,
              _ptr(pos_dev), _stream(dev))


def decode_attention_at(q, k_cache, v_cache, pos_dev, out: torch.Tensor | None = None) -> torch.Tensor:
    """decode_attention over positions [0, *pos_dev + 1) (read on the device)."""
    name = "decode_attention_at"
    _f16(q, name + "(q)")
    _f16(k_cache, name + "(k_cache)")
    _f16(v_cache, name + "(v_cache)")
    _check(q.dim() == 2 and k_cache.dim() == 3 and v_cache.shape == k_cache.shape and q.size(1) == k_cache.size(2),
           name, ": q [num_q_heads, head_dim], caches [num_kv_heads, max_seq_len, head_dim]")
    _check_pos_dev(pos_dev, name)
    nq, (nkv, max_seq, hd) = q.size(0), k_cache.shape
    _check(nq % nkv == 0, name, ": num_q_heads must be a multiple of num_kv_heads")
    dev = _same_device(q, k_cache, v_cache, pos_dev)
    y = out if out is not None else torch.empty(nq, hd, dtype=torch.float16, device=dev)
    with torch.cuda.device(dev):
        nbytes = lib().soinfer_decode_attention_workspace_bytes(nq, max_seq, hd)
        ws = _workspace("attn", dev, nbytes)
        _call("soinfer_decode_attention_at", _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(y), nq, nkv, max_seq, hd,
              _ptr(pos_dev), ws.data_ptr(), ws.numel(), _stream(dev))
    return y


def decode_attention(q, k_cache, v_cache, cur_len: int, out: torch.Tensor | None = None) -> torch.Tensor:
    _f16(q, "decode_attention(q)")
    _f16(k_cache, "decode_attention(k_cache)")
    _f16(v_cache, "decode_attention(v_cache)")
    _check(q.dim() == 2, "decode_attention: q must be 2D [num_q_heads, head_dim]")
    _check(k_cache.dim() == 3 and v_cache.shape == k_cache.shape,
           "decode_attention: k_cache/v_cache must be 3D [num_kv_heads, max_seq_len, head_dim] and same shape")
    _check(q.size(1) == k_cache.size(2), "decode_attention: q's head_dim must match the cache's head_dim")
    nq, (nkv, max_seq, hd) = q.size(0), k_cache.shape
    _check(nq % nkv == 0, "decode_attention: num_q_heads must be a multiple of num_kv_heads")
    _check(1 <= cur_len <= max_seq, "decode_attention: cur_len out of range for max_seq_len")
    dev = _same_device(q, k_cache, v_cache)
    y = out if out is not None else torch.empty(nq, hd, dtype=torch.float16, device=dev)
    with torch.cuda.device(dev):
        nbytes = lib().soinfer_decode_attention_workspace_bytes(nq, max_seq, hd)
        ws = _workspace("attn", dev, nbytes)
        _call("soinfer_decode_attention", _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(y), nq, nkv, max_seq, hd,
              cur_len, ws.data_ptr(), ws.numel(), _stream(dev))
    return y


# ------------------------------------------------------------ multi-token GEMM
def gemm_w4a16(Wq_packed, scale, X, K: int, group_size: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Y [M, N] fp16 = X [M, K] (fp16, M <= 8 tokens) times the INT4 weights'
    transpose -- every token's reference GEMV, one pass over the weights."""
    name = "gemm_w4a16"
    _check(Wq_packed.is_cuda and Wq_packed.dtype == torch.uint8 and Wq_packed.is_contiguous() and Wq_packed.dim() == 2,
           name, "(Wq_packed): must be a contiguous 2D uint8 CUDA tensor")
    _check(Wq_packed.size(1) == _cdiv(K, 8) * 4, name, ": Wq_packed.size(1) must be ceil(K/8)*4 for the given K")
    _f32(scale, name + "(scale)")
    _check(scale.dim() == 2 and scale.size(0) == Wq_packed.size(0), name, ": scale must be 2D [N, num_groups]")
    _check(X.is_cuda and X.dtype == torch.float16, name, "(X): must be a float16 CUDA tensor")
    _check(X.dim() == 2 and X.size(1) == K and X.stride(1) == 1 and 1 <= X.size(0) <= 8, name,
           ": X must be [M <= 8, K] with unit K stride")
    dev = _same_device(Wq_packed, scale, X)
    M, N = X.size(0), Wq_packed.size(0)
    Y = out if out is not None else torch.empty(M, N, dtype=torch.float16, device=dev)
    _check(Y.shape == (M, N) and Y.stride(1) == 1 and Y.dtype == torch.float16, name, ": out must be fp16 [M, N]")
    with torch.cuda.device(dev):
        _call("soinfer_gemm_w4a16", _ptr(Wq_packed), _ptr(scale), _ptr(X), X.stride(0), _ptr(Y), Y.stride(0), M, N,
              K, group_size, scale.size(1), _stream(dev))
    return Y


class _GemmTask(ctypes.Structure):
    _fields_ = [("Wq", _P), ("scale", _P), ("X", _P), ("Y", _P), ("N", _I64), ("K", _I64), ("group_size", _I64),
                ("num_groups", _I64), ("ldx", _I64), ("ldy", _I64)]


class GemmBatch:
    """A prepared list of independent multi-token INT4 GEMMs run as one
    launch (soinfer_gemm_w4a16_batch): tasks = sequence of
    (Wq_packed [N, K/2] uint8, scale [N, G] f32, X [M, K] fp16, Y [M, N] fp16,
    K, group_size), every X with the same M <= 8 rows.  The tensors must stay
    alive while the batch is used."""

    def __init__(self, tasks):
        n = len(tasks)
        _check(0 < n <= MAX_BATCH_TASKS, "gemm_w4a16_batch: 1 ..", MAX_BATCH_TASKS, " tasks")
        arr = (_GemmTask * n)()
        dev, M = None, None
        for i, (W, scale, X, Y, K, group_size) in enumerate(tasks):
            name = f"gemm_w4a16_batch[task {i}]"
            _check(W.is_cuda and W.dtype == torch.uint8 and W.is_contiguous() and W.dim() == 2, name,
                   "(Wq_packed): must be a contiguous 2D uint8 CUDA tensor")
            _check(W.size(1) == _cdiv(K, 8) * 4, name, ": Wq_packed.size(1) must be ceil(K/8)*4 for the given K")
            _f32(scale, name + "(scale)")
            _check(scale.dim() == 2 and scale.size(0) == W.size(0), name, ": scale must be 2D [N, num_groups]")
            _check(X.is_cuda and X.dtype == torch.float16 and X.dim() == 2 and X.size(1) == K and X.stride(1) == 1,
                   name, ": X must be fp16 [M, K] with unit K stride")
            _check(Y.is_cuda and Y.dtype == torch.float16 and Y.dim() == 2 and Y.size(1) == W.size(0)
                   and Y.size(0) == X.size(0) and Y.stride(1) == 1, name, ": Y must be fp16 [M, N]")
            _check(M is None or X.size(0) == M, name, ": every task must have the same M")
            M = X.size(0)
            d = _same_device(W, scale, X, Y)
            _check(dev is None or d == dev, name, ": all tasks must be on one device")
            dev = d
            arr[i] = _GemmTask(W.data_ptr(), scale.data_ptr(), X.data_ptr(), Y.data_ptr(), W.size(0), K, group_size,
                               scale.size(1), X.stride(0), Y.stride(0))
        _check(1 <= M <= 8, "gemm_w4a16_batch: M must be in [1, 8]")
        self._arr, self.n, self.m, self.device = arr, n, M, dev
        self._keep = [tuple(t) for t in tasks]

    def run(self) -> None:
        dev = self.device
        with torch.cuda.device(dev):
            ws = _workspace("gemm_batch", dev, lib().soinfer_gemm_batch_workspace_bytes())
            _call("soinfer_gemm_w4a16_batch", ctypes.addressof(self._arr), self.n, self.m, ws.data_ptr(), ws.numel(),
                  _stream(dev))


class _FusedLayer(ctypes.Structure):
    _fields_ = [("Wq", _P * 7), ("scale", _P * 7), ("input_norm", _P), ("post_norm", _P), ("q_norm", _P),
                ("k_norm", _P), ("k_cache", _P), ("v_cache", _P)]


class FusedDecode:
    """Every decoder layer of a batch-1 decode step in one cooperative launch
    (soinfer_decode_layers_fused).  layers = sequence of dicts with
    "w" (7 packed INT4 weights: q, k, v, o, gate, up, down; group size 128),
    "s" (their fp32 scales), "input_norm", "post_norm", "q_norm", "k_norm"
    (fp16) and "k_cache" / "v_cache" (fp16 [num_kv_heads, max_seq, 128]).
    run(x, pos_dev) transforms the hidden state x [hidden] in place (the
    input embedding in, the last layer's output out) at the position held in
    pos_dev (int32 [1] CUDA).  The tensors must stay alive while it is used."""

    def __init__(self, layers, hidden: int, intermediate: int, num_heads: int, num_kv_heads: int, head_dim: int,
                 max_seq: int, eps: float, cos_table, sin_table, group_size: int = 128):
        name = "decode_layers_fused"
        n = len(layers)
        _check(n >= 1, name, ": at least one layer")
        arr = (_FusedLayer * n)()
        dev = None
        for i, ly in enumerate(layers):
            _check(len(ly["w"]) == 7 and len(ly["s"]) == 7, name, ": seven weights per layer")
            for w, sc in zip(ly["w"], ly["s"]):
                _check(w.is_cuda and w.dtype == torch.uint8 and w.is_contiguous(), name, ": weights: contiguous uint8 CUDA")
                _f32(sc, name + "(scale)")
                dev = dev or w.device
            for key in ("input_norm", "post_norm", "q_norm", "k_norm", "k_cache", "v_cache"):
                _f16(ly[key], f"{name}({key})")
            _check(ly["k_cache"].is_contiguous() and ly["v_cache"].is_contiguous(), name, ": caches must be contiguous")
            arr[i] = _FusedLayer((_P * 7)(*[w.data_ptr() for w in ly["w"]]), (_P * 7)(*[sc.data_ptr() for sc in ly["s"]]),
                                 ly["input_norm"].data_ptr(), ly["post_norm"].data_ptr(), ly["q_norm"].data_ptr(),
                                 ly["k_norm"].data_ptr(), ly["k_cache"].data_ptr(), ly["v_cache"].data_ptr())
        _check(cos_table.is_cuda and cos_table.dtype == torch.float32 and sin_table.dtype == torch.float32, name,
               ": cos / sin tables must be fp32 CUDA")
        self._arr, self.n, self.device = arr, n, dev
        self.shape = (hidden, intermediate, num_heads, num_kv_heads, head_dim, group_size, max_seq)
        self.eps = float(eps)
        self._keep = (list(layers), cos_table, sin_table)
        self.ws_bytes = lib().soinfer_decode_fused_workspace_bytes(hidden, intermediate, num_heads, num_kv_heads,
                                                                   head_dim)

    def run(self, x, pos_dev) -> None:
        H, I, NQ, NKV, HD, G, S = self.shape
        _f16(x, "decode_layers_fused(x)")
        _check(x.numel() == H and x.is_contiguous(), "decode_layers_fused", ": x must be contiguous [hidden]")
        _check_cuda(pos_dev, "decode_layers_fused(pos_dev)", torch.int32, ": must be int32")
        dev = self.device
        cos_table, sin_table = self._keep[1], self._keep[2]
        with torch.cuda.device(dev):
            ws = _workspace("fused_decode", dev, self.ws_bytes)
            _call("soinfer_decode_layers_fused", ctypes.addressof(self._arr), self.n, H, I, NQ, NKV, HD, G, S,
                  self.eps, cos_table.data_ptr(), sin_table.data_ptr(), pos_dev.data_ptr(), x.data_ptr(),
                  ws.data_ptr(), ws.numel(), _stream(dev))


# ------------------------------------------------------------ load-time quantization
_QUANT_DTYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def quantize_pack_int4(w, group_size: int):
    """GPU group-wise INT4 quantize + AWQ pack of w [N, K] (fp32 / fp16 / bf16
    CUDA, unit stride along K): (packed uint8 [N, ceil(Kp/8)*4], scale fp32
    [N, Kp/g], Kp), bit-exact with soinfer.quant.formats.quantize +
    pack.pack_int4 on the CPU."""
    name = "quantize_pack_int4"
    _check(w.is_cuda and w.dim() == 2 and w.stride(1) == 1, name, "(w): must be a 2D CUDA tensor with unit K stride")
    _check(w.dtype in _QUANT_DTYPES, name, "(w): dtype must be float32, float16 or bfloat16")
    _check(group_size in (8, 16, 32, 64, 128, 256), name, ": group_size must be a power of two in [8, 256]")
    N, K = w.shape
    Kp = _cdiv(K, group_size) * group_size
    packed = torch.empty(N, Kp // 2, dtype=torch.uint8, device=w.device)
    scale = torch.empty(N, Kp // group_size, dtype=torch.float32, device=w.device)
    with torch.cuda.device(w.device):
        _call("soinfer_quantize_pack_int4", _ptr(w), _QUANT_DTYPES[w.dtype], N, K, w.stride(0), group_size,
              _ptr(packed), _ptr(scale), _stream(w.device))
    return packed, scale, Kp


# ------------------------------------------------------------ tensor-parallel exchange
IPC_HANDLE_BYTES = 64
MAX_PEERS = 8


class PeerSetStruct(ctypes.Structure):
    _fields_ = [("base", _P * MAX_PEERS), ("rank", ctypes.c_int32), ("world", ctypes.c_int32),
                ("slot_bytes", _I64)]


def peer_buffer_bytes(slot_bytes: int, world: int) -> int:
    n = lib().soinfer_peer_buffer_bytes(slot_bytes, world)
    _check(n > 0, "peer_buffer_bytes: slot_bytes must be a positive multiple of 16 and world in [1, 8]")
    return n


def peer_buffer_create(nbytes: int, device) -> tuple[int, bytes]:
    """A zeroed device buffer for peer exchange on `device` and its CUDA IPC handle."""
    ptr = _P()
    handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    with torch.cuda.device(device):
        _call("soinfer_peer_buffer_create", nbytes, ctypes.byref(ptr), handle)
    return ptr.value, handle.raw


def peer_buffer_open(handle: bytes, device) -> int:
    """Maps another process's exchange buffer (its IPC handle) into this one."""
    _check(len(handle) == IPC_HANDLE_BYTES, "peer_buffer_open: handle must be 64 bytes")
    ptr = _P()
    with torch.cuda.device(device):
        _call("soinfer_peer_buffer_open", ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES), ctypes.byref(ptr))
    return ptr.value


def peer_buffer_close(ptr: int, device) -> None:
    with torch.cuda.device(device):
        _call("soinfer_peer_buffer_close", ptr)


def peer_buffer_destroy(ptr: int, device) -> None:
    with torch.cuda.device(device):
        _call("soinfer_peer_buffer_destroy", ptr)


def peer_buffer_reset(ptr: int, device) -> None:
    """Zeroes this rank's exchange header on the current stream (recovery after a peer timeout)."""
    with torch.cuda.device(device):
        _call("soinfer_peer_buffer_reset", ptr, _stream(torch.device(device)))


def tp_allreduce_add_rmsnorm(peers: PeerSetStruct, partial, residual, weight, out_sum, out_norm, eps: float,
                             device) -> None:
    """See soinfer_tp_allreduce_add_rmsnorm (partial None: pushed by gemv_w4a16_tp_partial)."""
    n = out_sum.numel()
    for t, nm in ((partial, "partial"), (residual, "residual"), (out_norm, "out_norm")):
        if t is not None:
            _f16(t, f"tp_allreduce_add_rmsnorm({nm})")
            _check(t.numel() == n and t.device == device, f"tp_allreduce_add_rmsnorm: {nm} must match out_sum")
    with torch.cuda.device(device):
        _call("soinfer_tp_allreduce_add_rmsnorm", ctypes.byref(peers), _ptr(partial), _ptr(residual), _ptr(weight),
              _ptr(out_sum), _ptr(out_norm), n, eps, _stream(device))


def gemv_w4a16_tp_partial(peers: PeerSetStruct, Wq_packed, scale, x, K: int, group_size: int) -> None:
    """Row-parallel INT4 GEMV whose rows go to every rank's exchange inbox."""
    name = "gemv_w4a16_tp_partial"
    _check(Wq_packed.is_cuda and Wq_packed.dtype == torch.uint8 and Wq_packed.is_contiguous() and Wq_packed.dim() == 2,
           name, "(Wq_packed): must be a contiguous 2D uint8 CUDA tensor")
    _f32(scale, name + "(scale)")
    _f16(x, name + "(x)")
    _check(x.dim() == 1 and x.size(0) == K, name, ": x must be 1D [K]")
    dev = _same_device(Wq_packed, scale, x)
    with torch.cuda.device(dev):
        _call("soinfer_gemv_w4a16_tp_partial", ctypes.byref(peers), _ptr(Wq_packed), _ptr(scale), _ptr(x),
              Wq_packed.size(0), K, group_size, scale.size(1), _stream(dev))


def tp_allgather(peers: PeerSetStruct, local, out) -> None:
    _check(local.is_cuda and local.is_contiguous() and out.is_contiguous(), "tp_allgather: contiguous CUDA tensors")
    nbytes = local.numel() * local.element_size()
    _check(out.numel() * out.element_size() == nbytes * peers.world, "tp_allgather: out must be world x local")
    with torch.cuda.device(local.device):
        _call("soinfer_tp_allgather", ctypes.byref(peers), _ptr(local), nbytes, _ptr(out), _stream(local.device))


def tp_argmax(peers: PeerSetStruct, logits, local_idx, offset: int, out_idx) -> None:
    _f16(logits, "tp_argmax(logits)")
    _check_cuda(local_idx, "tp_argmax(local_idx)", torch.int32, ": must be int32")
    _check_cuda(out_idx, "tp_argmax(out_idx)", torch.int32, ": must be int32")
    dev = _same_device(logits, local_idx, out_idx)
    with torch.cuda.device(dev):
        _call("soinfer_tp_argmax", ctypes.byref(peers), _ptr(logits), _ptr(local_idx), offset, _ptr(out_idx),
              _stream(dev))
