"""TEST INFRASTRUCTURE ONLY: numpy restatement of the reference algorithms.

Each function cites the sparse-offload-infer file:line it restates.  Float
semantics: quantize / pack / selection follow the reference's float32
arithmetic exactly (bit-exact); GEMV / attention references are computed in
float64 from the exactly dequantized weights (the reference tests' own oracle
is fp32 torch.mv of formats.dequantize(qt), tests/test_m4_kernels.py:157-168;
float64 is the closer-to-exact version of the same quantity).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
TINY = np.finfo(np.float32).tiny
AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)  # csrc/include/layout.h:19-51


def cdiv(a: int, b: int) -> int:
    return -(-a // b)


def qmax_for_bits(bits: int) -> int:
    return 2 ** (bits - 1) - 1


# ---------------------------------------------------------------- quantize
def quantize_group(w, group_size: int, bits: int = 4):
    """formats.quantize, granularity 'group', min_max scale
    (python/soinfer/quant/formats.py:55-65, :103-110; calibrate.py:22-27).
    Returns (q int8 [..., padded_K], scale f32 [..., num_groups])."""
    w = np.asarray(w, dtype=np.float32)
    k = w.shape[-1]
    groups = cdiv(k, group_size)
    pad = groups * group_size - k
    if pad:
        w = np.concatenate([w, np.zeros(w.shape[:-1] + (pad,), np.float32)], axis=-1)
    grouped = w.reshape(w.shape[:-1] + (groups, group_size))
    qmax = qmax_for_bits(bits)
    amax = np.abs(grouped).max(axis=-1)
    scale = np.maximum(amax / F32(qmax), TINY).astype(np.float32)
    q = np.clip(np.rint(grouped / scale[..., None]), -qmax, qmax).astype(np.int8)
    return q.reshape(w.shape), scale


def quantize_per_channel(w, bits: int = 8):
    """formats.quantize 'per_channel' (formats.py:97-101). scale [..., N, 1]."""
    w = np.asarray(w, dtype=np.float32)
    qmax = qmax_for_bits(bits)
    scale = np.maximum(np.abs(w).max(axis=-1) / F32(qmax), TINY).astype(np.float32)
    q = np.clip(np.rint(w / scale[..., None]), -qmax, qmax).astype(np.int8)
    return q, scale[..., None]


def quantize_per_tensor(w, bits: int = 8):
    """formats.quantize 'per_tensor' (formats.py:90-95). scale [1, 1]."""
    w = np.asarray(w, dtype=np.float32)
    qmax = qmax_for_bits(bits)
    scale = np.maximum(np.abs(w).max() / F32(qmax), TINY).astype(np.float32)
    q = np.clip(np.rint(w / scale), -qmax, qmax).astype(np.int8)
    return q, np.full((1, 1), scale, np.float32)


# -------------------------------------------------------------------- pack
def pack_int4(q):
    """pack.pack_int4 (python/soinfer/quant/pack.py:31-50) / layout.h:19-51:
    byte0 = v0|v2<<4, byte1 = v4|v6<<4, byte2 = v1|v3<<4, byte3 = v5|v7<<4."""
    q = np.asarray(q, dtype=np.int8)
    k = q.shape[-1]
    groups = cdiv(k, 8)
    pad = groups * 8 - k
    if pad:
        q = np.concatenate([q, np.zeros(q.shape[:-1] + (pad,), np.int8)], axis=-1)
    nib = (q.astype(np.int16) & 0xF).reshape(q.shape[:-1] + (groups, 8))
    v = [nib[..., i] for i in range(8)]
    out = np.stack([v[0] | (v[2] << 4), v[4] | (v[6] << 4), v[1] | (v[3] << 4), v[5] | (v[7] << 4)], axis=-1)
    return out.astype(np.uint8).reshape(q.shape[:-1] + (groups * 4,))


def unpack_int4(packed, orig_k: int):
    """pack.unpack_int4 (pack.py:53-69)."""
    packed = np.asarray(packed, dtype=np.uint8)
    groups = packed.shape[-1] // 4
    b = packed.astype(np.int16).reshape(packed.shape[:-1] + (groups, 4))
    lo, hi = b & 0xF, (b >> 4) & 0xF
    vals = np.stack([lo[..., 0], lo[..., 2], hi[..., 0], hi[..., 2], lo[..., 1], lo[..., 3], hi[..., 1], hi[..., 3]],
                    axis=-1)
    vals = np.where(vals >= 8, vals - 16, vals)
    return vals.reshape(packed.shape[:-1] + (groups * 8,))[..., :orig_k].astype(np.int8)


def dequant_int4(packed, scale, K: int, group_size: int):
    """fp32 dequantized INT4 weights [N, K]: scale[n, k//g] * q[n, k]
    (csrc/kernels/dequant.cuh:29-58 is exact; formats.dequantize :113-123)."""
    q = unpack_int4(packed, K).astype(np.float32)
    s = np.repeat(np.asarray(scale, np.float32), group_size, axis=-1)[..., :K]
    return q * s


def dequant_int8(Wq, scale, group_size: int):
    q = np.asarray(Wq, np.int8).astype(np.float32)
    s = np.asarray(scale, np.float32)
    if s.shape[-1] == 1:
        return q * s
    return q * np.repeat(s, group_size, axis=-1)[..., : q.shape[-1]]


# -------------------------------------------------------------------- GEMV
def gemv_w4a16(packed, scale, x, K: int, group_size: int):
    """y = dequant(Wq, scale) @ x (csrc/kernels/gemv_w4a16_group.cu:77-127;
    test oracle tests/test_m4_kernels.py:157-168). float64 accumulate."""
    W = dequant_int4(packed, scale, K, group_size).astype(np.float64)
    return W @ np.asarray(x, np.float16).astype(np.float64)[:K]


def gemv_w8a16(Wq, scale, x, group_size: int):
    """csrc/kernels/gemv_w8a16.cu:22-62 (scale row broadcast when scale has 1 row)."""
    W = dequant_int8(Wq, scale, group_size).astype(np.float64)
    return W @ np.asarray(x, np.float16).astype(np.float64)


def sparse_accumulate(Wsel_packed, scale_sel, h, H: int, group_size: int):
    """y[c] = sum_i h[i] * scale[i, c/g] * q[i, c]
    (csrc/kernels/gemv_sparse_accumulate.cu:10-38). float64."""
    W = dequant_int4(Wsel_packed, scale_sel, H, group_size).astype(np.float64)
    return np.asarray(h, np.float16).astype(np.float64) @ W


def sparse_accumulate_f32_sequential(Wsel_packed, scale_sel, h, H: int, group_size: int):
    """The reference kernel's own float32 order: one accumulator per column,
    acc += (h_i * s) * v sequentially over i (gemv_sparse_accumulate.cu:24-35)."""
    q = unpack_int4(Wsel_packed, H).astype(np.float32)
    s = np.repeat(np.asarray(scale_sel, np.float32), group_size, axis=-1)[..., :H]
    hf = np.asarray(h, np.float16).astype(np.float32)
    acc = np.zeros(H, np.float32)
    for i in range(q.shape[0]):
        acc = acc + (hf[i] * s[i]) * q[i]
    return acc


# --------------------------------------------------------------- selection
def topk_threshold_select_ref(v, k: int):
    """The reference selector, bit-exact (csrc/kernels/topk_select.cu:17-95):
    hi = max(0, max v) + 1e-3f; 24 fp32 steps mid = 0.5f*(lo+hi),
    lo = mid if count(v >= mid) >= k else hi = mid; output the first k indices
    (ascending) with v >= lo.  Returns (idx int32 [k] padded with -1, count)."""
    v = np.asarray(v, np.float32)
    m = F32(np.fmax.reduce(np.concatenate([np.zeros(1, np.float32), v])))
    lo, hi = F32(0.0), F32(m + F32(1e-3))
    for _ in range(24):
        mid = F32(F32(0.5) * F32(lo + hi))
        if np.count_nonzero(v >= mid) >= k:
            lo = mid
        else:
            hi = mid
    sel = np.nonzero(v >= lo)[0][:k]
    out = np.full(k, -1, np.int32)
    out[: sel.size] = sel
    return out, int(sel.size)


def topk_exact(v, k: int):
    """Exact top-k, ties at the k-th value broken by the lower index, NaN
    ranked lowest, output in ascending index order."""
    v = np.asarray(v, np.float32).astype(np.float64)
    nan = np.isnan(v)
    key = np.where(nan, 0.0, -v)
    order = np.lexsort((np.arange(v.size), key, nan))
    return np.sort(order[:k]).astype(np.int32)


def build_dip_descriptors(sel, slot_of):
    """csrc/kernels/gemv_dip_fused.cu:17-42 with deterministic miss order
    (ascending selected position)."""
    sel = np.asarray(sel, np.int64)
    slot_of = np.asarray(slot_of, np.int64)
    desc = np.empty(sel.size, np.int64)
    misses = []
    for j, c in enumerate(sel):
        s = slot_of[c]
        if s >= 0:
            desc[j] = s
        else:
            desc[j] = len(misses) | (1 << 31)
            misses.append(c)
    desc = desc.astype(np.uint32).view(np.int32)
    return desc, np.asarray(misses, np.int32), len(misses)


# ---------------------------------------------------------- attention side
def rmsnorm(x, w, eps: float):
    """csrc/kernels/rmsnorm.cu:9-42: out = fp16((x * rsqrt(mean(x^2)+eps)) * w)."""
    xf = np.asarray(x, np.float16).astype(np.float64)
    wf = np.asarray(w, np.float16).astype(np.float64)
    inv = 1.0 / np.sqrt((xf * xf).mean(axis=-1, keepdims=True) + eps)
    return (xf * inv * wf).astype(np.float16)


def rope(x, cos_v, sin_v):
    """csrc/kernels/rope.cu:5-19 rotate-half: (x1, x2) -> (x1 c - x2 s, x2 c + x1 s)."""
    xf = np.asarray(x, np.float16).astype(np.float64)
    half = xf.shape[-1] // 2
    x1, x2 = xf[..., :half], xf[..., half:]
    c, s = np.asarray(cos_v, np.float64), np.asarray(sin_v, np.float64)
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1).astype(np.float16)


def decode_attention(q, k_cache, v_cache, cur_len: int):
    """csrc/kernels/decode_attention.cu:17-55: qh reads kv head qh // (NQ/NKV);
    softmax(q.k / sqrt(hd)) @ v over positions [0, cur_len). float64."""
    q = np.asarray(q, np.float16).astype(np.float64)
    kc = np.asarray(k_cache, np.float16).astype(np.float64)
    vc = np.asarray(v_cache, np.float16).astype(np.float64)
    nq, hd = q.shape
    rep = nq // kc.shape[0]
    out = np.empty((nq, hd))
    for h in range(nq):
        kv = h // rep
        s = kc[kv, :cur_len] @ q[h] / np.sqrt(hd)
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ vc[kv, :cur_len]
    return out


def silu(x):
    return x / (1.0 + np.exp(-x))


def dip_mlp_block(x, gate, up, down_t, k: int, group_size: int, H: int, gate_out=None):
    """DIP MLP block (runtime/generate.py:276-310): gate GEMV (fp16 out) ->
    |gate| -> reference selector -> up GEMV on the selected rows (fp16) ->
    h = fp16(silu(gate_sel) * up_sel) -> sparse down accumulate.  gate / up /
    down_t are (packed, scale) pairs; down_t is the transposed down_proj
    [I, H].  `gate_out` (fp16) may be supplied to evaluate the selection on a
    given gate vector.  Returns dict of intermediates; y is float64."""
    gp, gs = gate
    up_p, up_s = up
    dp, ds = down_t
    g16 = (np.asarray(gate_out, np.float16) if gate_out is not None
           else gemv_w4a16(gp, gs, x, H, group_size).astype(np.float16))
    idx, _ = topk_threshold_select_ref(np.abs(g16.astype(np.float32)), k)
    u16 = gemv_w4a16(up_p[idx], up_s[idx], x, H, group_size).astype(np.float16)
    hsel = (silu(g16[idx].astype(np.float32)) * u16.astype(np.float32)).astype(np.float16)
    y = sparse_accumulate(dp[idx], ds[idx], hsel, H, group_size)
    return {"gate": g16, "idx": idx, "up_sel": u16, "h_sel": hsel, "y": y}
