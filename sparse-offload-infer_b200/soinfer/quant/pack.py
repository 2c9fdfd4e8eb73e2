"""INT4 / INT8 bit packing, byte-identical to the reference packing contract
(csrc/include/layout.h:19-51 and python/soinfer/quant/pack.py:31-69 of
sparse-offload-infer) and to what the sm_100a kernels unpack.

INT4: values are taken 8 at a time along K (K zero-padded to a multiple of 8)
and stored in 4 bytes with nibble j of the little-endian word holding value
AWQ_ORDER[j], AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7):
    byte0 = v0 | v2 << 4, byte1 = v4 | v6 << 4,
    byte2 = v1 | v3 << 4, byte3 = v5 | v7 << 4
(two's-complement nibbles).  The low half-word thus holds the even values and
the high half-word the odd ones, so one 32-bit word unpacks to the four
consecutive K pairs (v0,v1) .. (v6,v7) with one mask per half2.

INT8: no packing (one int8 per value); the functions exist so both formats
share one API.
"""
from __future__ import annotations

import torch

GROUP = 8
AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)
# byte b of a packed group holds (low nibble, high nibble) = values _BYTE_SRC[b]
_BYTE_SRC = ((0, 2), (4, 6), (1, 3), (5, 7))


def pack_int8(q: torch.Tensor) -> tuple[torch.Tensor, int]:
    if q.dtype != torch.int8:
        raise ValueError(f"pack_int8 expects int8, got {q.dtype}")
    return q.clone(), q.shape[-1]


def unpack_int8(packed: torch.Tensor, orig_k: int) -> torch.Tensor:
    if packed.dtype != torch.int8:
        raise ValueError(f"unpack_int8 expects int8, got {packed.dtype}")
    return packed[..., :orig_k].clone()


def pack_int4(q: torch.Tensor) -> tuple[torch.Tensor, int]:
    """q: int8 in [-8, 7], shape [..., K] -> (uint8 [..., ceil(K/8)*4], K)."""
    if q.dtype != torch.int8:
        raise ValueError(f"pack_int4 expects int8, got {q.dtype}")
    k = q.shape[-1]
    extra = (-k) % GROUP
    if extra:
        q = torch.nn.functional.pad(q, (0, extra))
    groups = q.shape[-1] // GROUP
    nib = (q.to(torch.int16) & 0xF).reshape(*q.shape[:-1], groups, GROUP)
    out = torch.empty(*q.shape[:-1], groups, GROUP // 2, dtype=torch.int16, device=q.device)
    for b, (lo, hi) in enumerate(_BYTE_SRC):
        out[..., b] = nib[..., lo] | (nib[..., hi] << 4)
    return out.to(torch.uint8).reshape(*q.shape[:-1], groups * (GROUP // 2)), k


def unpack_int4(packed: torch.Tensor, orig_k: int) -> torch.Tensor:
    """Inverse of pack_int4: uint8 [..., ceil(orig_k/8)*4] -> int8 [..., orig_k]."""
    if packed.dtype != torch.uint8:
        raise ValueError(f"unpack_int4 expects uint8, got {packed.dtype}")
    groups = packed.shape[-1] // (GROUP // 2)
    by = packed.to(torch.int16).reshape(*packed.shape[:-1], groups, GROUP // 2)
    vals = torch.empty(*packed.shape[:-1], groups, GROUP, dtype=torch.int16, device=packed.device)
    for b, (lo, hi) in enumerate(_BYTE_SRC):
        vals[..., lo] = by[..., b] & 0xF
        vals[..., hi] = (by[..., b] >> 4) & 0xF
    vals = torch.where(vals >= 8, vals - 16, vals)
    return vals.reshape(*packed.shape[:-1], groups * GROUP)[..., :orig_k].to(torch.int8)
