"""Symmetric weight quantization formats (per-tensor, per-channel, group,
block32, mx_e8m0) -- the load-time half of the hot path.

Contract (identical to the reference, python/soinfer/quant/formats.py:24-123
of sparse-offload-infer, so packed weights and scales are bit-identical):
  * symmetric, no zero point: W ~= scale * q with q in [-qmax, qmax],
    qmax = 2**(bits-1) - 1 (7 for INT4, 127 for INT8);
  * quantization runs along the last dim K; group formats zero-pad K up to a
    multiple of the group size before grouping;
  * scale = max(|w| over the group) / qmax, clamped below at float32 tiny;
    mx_e8m0 rounds that scale to the nearest power of two;
  * q = clamp(round_half_to_even(w / scale), -qmax, qmax), stored as int8
    (one value per byte -- see pack.py for INT4 bit packing);
  * scale is float32 [..., N, num_groups] (num_groups = 1 for per-tensor and
    per-channel; per-tensor scale has shape [1, 1]).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from . import calibrate

GRANULARITIES = ("per_tensor", "per_channel", "group", "block32", "mx_e8m0")
_FIXED_GROUP = {"block32": 32, "mx_e8m0": 32}


def qmax_for_bits(bits: int) -> int:
    return (1 << (bits - 1)) - 1


@dataclass
class QuantConfig:
    bits: int
    granularity: str
    group_size: Optional[int] = None  # required for "group"; forced to 32 for block32 / mx_e8m0

    def __post_init__(self) -> None:
        if self.granularity not in GRANULARITIES:
            raise ValueError(f"unknown granularity {self.granularity!r}, must be one of {GRANULARITIES}")
        if self.granularity in _FIXED_GROUP:
            self.group_size = _FIXED_GROUP[self.granularity]
        elif self.granularity == "group" and not self.group_size:
            raise ValueError("granularity='group' requires group_size")


@dataclass
class QuantTensor:
    qweight: torch.Tensor  # int8 [..., N, padded_K]
    scale: torch.Tensor  # float32 [..., N, num_groups]
    config: QuantConfig
    orig_k: int  # K before group padding; dequantize() truncates back to it


def _pad_last(w: torch.Tensor, multiple: int) -> torch.Tensor:
    k = w.shape[-1]
    extra = (-k) % multiple
    if extra == 0:
        return w
    return torch.nn.functional.pad(w, (0, extra))


def round_to_pow2(scale: torch.Tensor) -> torch.Tensor:
    """Nearest power of two of a non-negative scale (E8M0 style); 0 stays 0."""
    positive = scale > 0
    exps = torch.round(torch.log2(torch.where(positive, scale, torch.ones_like(scale))))
    return torch.where(positive, torch.exp2(exps), torch.zeros_like(scale))


def _round_clamp(v: torch.Tensor, qmax: int) -> torch.Tensor:
    return torch.round(v).clamp_(-qmax, qmax).to(torch.int8)


def quantize(w: torch.Tensor, config: QuantConfig, scale_fn=None) -> QuantTensor:
    """Quantize float w [..., N, K] per `config`.

    scale_fn(grouped, amax, qmax) -> scale overrides the scale rule (default
    calibrate.min_max); `grouped` holds the values sharing one scale along its
    last dim and amax == grouped.abs().amax(-1)."""
    w = w.float()
    qmax = qmax_for_bits(config.bits)
    k = w.shape[-1]
    rule = calibrate.min_max if scale_fn is None else scale_fn

    if config.granularity == "per_tensor":
        flat = w.reshape(-1)
        scale = rule(flat, flat.abs().max(), qmax).reshape(1, 1)
        return QuantTensor(_round_clamp(w / scale, qmax), scale.to(torch.float32), config, k)

    if config.granularity == "per_channel":
        scale = rule(w, w.abs().amax(dim=-1), qmax)  # [..., N]
        q = _round_clamp(w / scale.unsqueeze(-1), qmax)
        return QuantTensor(q, scale.unsqueeze(-1).to(torch.float32), config, k)

    g = config.group_size
    padded = _pad_last(w, g)
    num_groups = padded.shape[-1] // g
    grouped = padded.reshape(*padded.shape[:-1], num_groups, g)
    scale = rule(grouped, grouped.abs().amax(dim=-1), qmax)  # [..., N, num_groups]
    if config.granularity == "mx_e8m0":
        scale = round_to_pow2(scale)
    q = _round_clamp(grouped / scale.unsqueeze(-1), qmax)
    return QuantTensor(q.reshape(*padded.shape), scale.to(torch.float32), config, k)


def dequantize(qt: QuantTensor) -> torch.Tensor:
    q = qt.qweight.float()
    if qt.config.granularity in ("per_tensor", "per_channel"):
        return q * qt.scale
    g = qt.config.group_size
    grouped = q.reshape(*q.shape[:-1], q.shape[-1] // g, g)
    return (grouped * qt.scale.unsqueeze(-1)).reshape(q.shape)[..., : qt.orig_k]


def fraction_exact_zero(qt: QuantTensor) -> float:
    """Fraction of the (unpadded) quantized values that are exactly zero."""
    return (qt.qweight[..., : qt.orig_k] == 0).float().mean().item()
