"""Typed wrappers over the sm_100a C ABI -- the drop-in op surface.

Same names, signatures and error behaviour as the reference's
python/soinfer/ops.py (sparse-offload-infer), restricted to the decode hot
path; each wrapper runs a hand-written sm_100a kernel through
libsoinfer_b200.so (see soinfer._C).  Additions beyond the reference are
marked "B200 addition".
"""
from __future__ import annotations

import torch

from . import _C


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """RMSNorm over the last dim. x: [rows, hidden] half, weight: [hidden] half, hidden even.
    Reference: ops.py:67-69, csrc/kernels/rmsnorm.cu:9-42."""
    return _C.rmsnorm(x, weight, eps)


def gemv_fp16_v3(W: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """fp16 GEMV y = W x with fp32 accumulation (the decode LM head). W: [N, K] half, x: [K] half, K % 8 == 0.
    Reference: ops.py:82-84, csrc/kernels/gemv_fp16.cu:60-95."""
    return _C.gemv_fp16_v3(W, x)


def lm_head_argmax(W: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """B200 addition: the greedy next token, argmax over the fp16 logits of W x (lowest index among equal
    maxima, like torch.argmax), fused into the LM head GEMV.  Returns an int32 [1] CUDA tensor.
    Replaces gemv_fp16_v3 + torch.argmax (reference runtime/generate.py:452-454)."""
    return _C.gemv_fp16_argmax(W, x)[0]


def gemv_w8a16(Wq: torch.Tensor, scale: torch.Tensor, x: torch.Tensor, group_size: int) -> torch.Tensor:
    """y = dequant(Wq, scale) @ x. Wq: [N,K] int8 symmetric; scale: [N,num_groups] or [1,num_groups] fp32
    (per-tensor broadcast); num_groups == 1 means one scale per row.  Reference: ops.py:92-96."""
    return _C.gemv_w8a16(Wq, scale, x, group_size)


def gemv_w4a16_group(Wq_packed: torch.Tensor, scale: torch.Tensor, x: torch.Tensor, K: int,
                     group_size: int) -> torch.Tensor:
    """y = dequant(Wq_packed, scale) @ x. Wq_packed: [N, ceil(K/8)*4] uint8 AWQ-order INT4; scale:
    [N, num_groups] fp32; group_size a positive multiple of 8.  Reference: ops.py:99-103."""
    return _C.gemv_w4a16_group(Wq_packed, scale, x, K, group_size)


def gemv_w4a16_group_lop3(Wq_packed: torch.Tensor, scale: torch.Tensor, x: torch.Tensor, K: int,
                          group_size: int) -> torch.Tensor:
    """Same contract as gemv_w4a16_group and the same sm_100a kernel (outputs identical by construction).
    Reference: ops.py:106-109."""
    return _C.gemv_w4a16_group_lop3(Wq_packed, scale, x, K, group_size)


def gemv_w4a16_rows(Wq_packed: torch.Tensor, scale: torch.Tensor, rows: torch.Tensor, x: torch.Tensor, K: int,
                    group_size: int, glu_gate: torch.Tensor | None = None) -> torch.Tensor:
    """B200 addition: y[r] = (row rows[r] of dequant(Wq_packed, scale)) . x for a device-resident matrix --
    the gather of selected up_proj rows fused into the GEMV (bit-identical to
    gemv_w4a16_group_lop3(Wq_packed[rows], scale[rows], x, K, group_size)). rows: int32 CUDA.
    glu_gate: y = swiglu(glu_gate, y, rows) computed in the epilogue (DIP's h_sel)."""
    return _C.gemv_w4a16_rows(Wq_packed, scale, rows, x, K, group_size, glu_gate=glu_gate)


def topk_threshold_select(abs_g: torch.Tensor, k: int) -> torch.Tensor:
    """The reference's DIP selector, bit-exact: fp32 threshold bisection (24 steps from [0, max+1e-3]),
    then the first k qualifying indices in ascending order. abs_g: 1D float32 CUDA, non-negative.
    Returns int32 [k].  Reference: ops.py:151-158, csrc/kernels/topk_select.cu:10-96."""
    indices, _count = _C.topk_threshold_select(abs_g, k)
    return indices


def topk_select_exact(abs_g: torch.Tensor, k: int) -> torch.Tensor:
    """B200 addition: exact top-k (ties at the k-th value broken by the lower index), ascending index order."""
    indices, _count = _C.topk_select_exact(abs_g, k)
    return indices


def gather_rows_staged(matrix: torch.Tensor, indices: torch.Tensor, staging: torch.Tensor,
                       gpu_dst: torch.Tensor) -> None:
    """Host gather of the selected rows of a pinned matrix into pinned staging (multi-threaded), then one
    H2D copy into gpu_dst on the current stream (asynchronous: synchronize before reading gpu_dst).
    indices: 1D int64 CPU.  Reference: ops.py:161-168."""
    _C.gather_rows_staged(matrix, indices, staging, gpu_dst)


def gather_rows_naive(matrix: torch.Tensor, indices: torch.Tensor, gpu_dst: torch.Tensor) -> None:
    """One cudaMemcpyAsync per selected row (baseline for gather_rows_staged). Reference: ops.py:171-176."""
    _C.gather_rows_naive(matrix, indices, gpu_dst)


def gather_rows_device(matrix: torch.Tensor, rows: torch.Tensor, gpu_dst: torch.Tensor) -> None:
    """B200 addition: SM-driven gather of rows (int32 CUDA indices) of a device-resident or pinned host
    matrix (zero-copy) into gpu_dst -- no host round trip for the indices."""
    _C.gather_rows_device(matrix, rows, gpu_dst)


def gather_rows_device_multi(pairs, rows: torch.Tensor, count: torch.Tensor | None = None,
                             max_k: int | None = None) -> None:
    """B200 addition: one device-driven gather of rows[j], j < min(count, max_k), from every (matrix, dst)
    pair; count (int32 [1] CUDA) is read on the device -- no host round trip for the miss count."""
    _C.gather_rows_device_multi(pairs, rows, count, max_k)


def gemv_w4a16_sparse_accumulate(Wq_selected: torch.Tensor, scale_selected: torch.Tensor,
                                 h_selected: torch.Tensor, H: int, group_size: int) -> torch.Tensor:
    """Sparse 'down' GEMV: y[H] = sum_i h_selected[i] * dequant(W_T[i, :]) over k gathered rows of the
    transposed down_proj.  Deterministic.  Reference: ops.py:179-188."""
    return _C.gemv_w4a16_sparse_accumulate(Wq_selected, scale_selected, h_selected, H, group_size)


def gemv_w4a16_sparse_rows(Wq_T: torch.Tensor, scale_T: torch.Tensor, rows: torch.Tensor, h_selected: torch.Tensor,
                           H: int, group_size: int, residual: torch.Tensor | None = None) -> torch.Tensor:
    """B200 addition: sparse 'down' GEMV over rows `rows` (int32 CUDA) of a resident transposed matrix,
    bit-identical to gemv_w4a16_sparse_accumulate(Wq_T[rows], scale_T[rows], h_selected, H, group_size);
    residual: residual + y computed in the epilogue."""
    return _C.gemv_w4a16_sparse_rows(Wq_T, scale_T, rows, h_selected, H, group_size, residual=residual)


def build_dip_descriptors(selected_indices: torch.Tensor, slot_of: torch.Tensor):
    """Per selected channel: cache slot (slot_of[c] >= 0) or staging miss position | 1<<31, plus the
    compacted miss list (ascending selected order) and its length.  Returns (descriptors, miss_channels,
    miss_count); only miss_channels[:miss_count.item()] is valid.  Reference: ops.py:191-199."""
    return _C.build_dip_descriptors(selected_indices, slot_of)


def gemv_dip_fused_up(cache_Wq: torch.Tensor, cache_scale: torch.Tensor, staging_Wq: torch.Tensor,
                      staging_scale: torch.Tensor, descriptors: torch.Tensor, x: torch.Tensor, K: int,
                      group_size: int) -> torch.Tensor:
    """Cache-or-stream 'up' GEMV: y[j] = W_sel[j] . x with row j read from the hot cache or the staging
    buffer per its descriptor; bit-identical to gemv_w4a16_group_lop3 on the same rows.
    Reference: ops.py:202-211."""
    return _C.gemv_dip_fused_up(cache_Wq, cache_scale, staging_Wq, staging_scale, descriptors, x, K, group_size)


def gemv_dip_fused_down(cache_Wq: torch.Tensor, cache_scale: torch.Tensor, staging_Wq: torch.Tensor,
                        staging_scale: torch.Tensor, descriptors: torch.Tensor, h_selected: torch.Tensor, H: int,
                        group_size: int) -> torch.Tensor:
    """Cache-or-stream 'down' GEMV; bit-identical to gemv_w4a16_sparse_accumulate on the same rows.
    Reference: ops.py:214-219."""
    return _C.gemv_dip_fused_down(cache_Wq, cache_scale, staging_Wq, staging_scale, descriptors, h_selected, H,
                                  group_size)


def precompute_rope_cos_sin(head_dim: int, theta: float, pos: int, device, dtype=torch.float32):
    """cos/sin [head_dim/2] for absolute position pos: angle_i = pos / theta^(2i/head_dim) (HF Qwen3
    RotaryEmbedding convention).  Reference: ops.py:222-227."""
    exponents = torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim
    angles = pos * (1.0 / (theta ** exponents))
    return angles.cos().to(dtype).contiguous(), angles.sin().to(dtype).contiguous()


def apply_rope(x: torch.Tensor, cos_vals: torch.Tensor, sin_vals: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE on x [num_heads, head_dim] half, in place; returns x.  Reference: ops.py:230-235."""
    _C.rope_apply(x, cos_vals, sin_vals)
    return x


def qk_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """Qwen3 per-head QK-norm == RMSNorm over head_dim for every head.  Reference: ops.py:238-243."""
    return rmsnorm(x, weight, eps)


def kv_cache_append(k_cache: torch.Tensor, v_cache: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                    pos: int) -> None:
    """k_cache/v_cache[:, pos, :] = k_new/v_new (each [num_kv_heads, head_dim] half), in place.
    Reference: ops.py:246-250."""
    _C.kv_cache_append(k_cache, v_cache, k_new, v_new, pos)


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, cur_len: int) -> torch.Tensor:
    """Single-query GQA attention over k_cache/v_cache[:, :cur_len]; query head qh reads kv head
    qh // (NQ // NKV).  q: [NQ, hd] half (already RoPE'd); caches [NKV, max_seq, hd] half.
    Reference: ops.py:253-260."""
    return _C.decode_attention(q, k_cache, v_cache, cur_len)


# ------------------------------------------------------------------ B200 additions: device-position forms
def precompute_rope_table(head_dim: int, theta: float, max_pos: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """B200 addition: cos / sin tables [max_pos, head_dim / 2] whose row p equals
    precompute_rope_cos_sin(head_dim, theta, p) element for element (same fp32 ops)."""
    exponents = torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim
    inv_freq = 1.0 / (theta ** exponents)
    angles = torch.arange(max_pos, dtype=torch.float32, device=device)[:, None] * inv_freq[None, :]
    return angles.cos().contiguous(), angles.sin().contiguous()


def apply_rope_at(x: torch.Tensor, cos_table: torch.Tensor, sin_table: torch.Tensor, pos_dev: torch.Tensor) -> torch.Tensor:
    """B200 addition: apply_rope (in place on x, returns x) with the position read on the device (rows of the
    tables); graph-capturable."""
    _C.rope_apply_at(x, cos_table, sin_table, pos_dev)
    return x


def kv_cache_append_at(k_cache: torch.Tensor, v_cache: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                       pos_dev: torch.Tensor) -> None:
    """B200 addition: kv_cache_append at the device position *pos_dev; graph-capturable."""
    _C.kv_cache_append_at(k_cache, v_cache, k_new.contiguous(), v_new.contiguous(), pos_dev)


def decode_attention_at(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, pos_dev: torch.Tensor) -> torch.Tensor:
    """B200 addition: decode_attention over [0, *pos_dev + 1), the length read on the device; graph-capturable."""
    return _C.decode_attention_at(q.contiguous(), k_cache, v_cache, pos_dev)


# ------------------------------------------------------------------ B200 additions: fused decode glue
def topk_threshold_select_abs(gate: torch.Tensor, k: int) -> torch.Tensor:
    """B200 addition: topk_threshold_select(gate.float().abs(), k) on an fp16 gate, without the fp32 copy."""
    return _C.topk_threshold_select_abs_f16(gate, k)[0]


def add_rmsnorm(x: torch.Tensor, x2: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6):
    """B200 addition: (rmsnorm(x + x2), x + x2) in one kernel, bit-identical to the fp16 add then rmsnorm."""
    return _C.add_rmsnorm(x, x2, weight, eps)


def swiglu(gate: torch.Tensor, up: torch.Tensor, idx: torch.Tensor | None = None) -> torch.Tensor:
    """B200 addition: (F.silu(gate[idx].float()) * up.float()).half() in one kernel."""
    return _C.swiglu(gate, up, idx)


def head_norm_rope(q, k, v, q_norm, k_norm, cos_vals, sin_vals, k_cache, v_cache, pos: int = 0, pos_dev=None,
                   eps: float = 1e-6) -> None:
    """B200 addition: qk_norm of q and k, RoPE of both, q in place, k / v appended to the caches at pos (or the
    device position pos_dev with cos / sin tables) -- one kernel for reference ops.py:238-250's sequence."""
    _C.head_norm_rope(q, k, v, q_norm, k_norm, cos_vals, sin_vals, k_cache, v_cache, pos, pos_dev, eps)


def gemm_w4a16(Wq_packed: torch.Tensor, scale: torch.Tensor, X: torch.Tensor, K: int, group_size: int) -> torch.Tensor:
    """B200 addition: batched decode -- Y [M, N] = X [M, K] W^T for M <= 8 tokens in one pass over the INT4
    weights (each row of Y is the reference's gemv_w4a16_group_lop3 of that token)."""
    return _C.gemm_w4a16(Wq_packed, scale, X, K, group_size)
