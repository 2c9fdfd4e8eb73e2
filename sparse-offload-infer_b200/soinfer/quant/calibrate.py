"""Scale-selection rules for formats.quantize (reference
python/soinfer/quant/calibrate.py:22-84 of sparse-offload-infer).

Every rule has the signature rule(grouped, amax, qmax) -> scale, where the
values sharing one scale lie along grouped's last dim and
amax == grouped.abs().amax(-1).
"""
from __future__ import annotations

import torch

_TINY = torch.finfo(torch.float32).tiny


def min_max(grouped: torch.Tensor, amax: torch.Tensor, qmax: int) -> torch.Tensor:
    """scale = amax / qmax (floored at float32 tiny) -- the load-time default."""
    return (amax / qmax).clamp(min=_TINY)


def percentile(grouped: torch.Tensor, amax: torch.Tensor, qmax: int, pct: float = 99.9) -> torch.Tensor:
    """Scale from the pct-th percentile of |w| (never above amax)."""
    clip = torch.quantile(grouped.abs().float(), pct / 100.0, dim=-1)
    return (torch.minimum(clip, amax) / qmax).clamp(min=_TINY)


def mse_optimal(grouped: torch.Tensor, amax: torch.Tensor, qmax: int, num_candidates: int = 32,
                min_frac: float = 0.5) -> torch.Tensor:
    """Grid search over fractions of the min-max scale in [min_frac, 1], keeping
    per group the candidate with the smallest reconstruction MSE (ties keep the
    earlier, smaller candidate)."""
    base = (amax / qmax).clamp(min=_TINY)
    best = base.clone()
    best_err = torch.full_like(base, float("inf"))
    for frac in torch.linspace(min_frac, 1.0, num_candidates):
        cand = base * frac.item()
        q = torch.clamp(torch.round(grouped / cand.unsqueeze(-1)), -qmax, qmax)
        err = (q * cand.unsqueeze(-1) - grouped).pow(2).mean(dim=-1)
        better = err < best_err
        best = torch.where(better, cand, best)
        best_err = torch.where(better, err, best_err)
    return best


def awq_scale(w: torch.Tensor, act_abs_mean: torch.Tensor, alpha: float = 0.5) -> torch.Tensor:
    """Activation-aware per-input-channel scale s_k = mean|x_k|^alpha,
    normalised to mean 1 (Lin et al., 2023): quantize w * s, feed x / s."""
    if act_abs_mean.shape[-1] != w.shape[-1]:
        raise ValueError(f"act_abs_mean has K={act_abs_mean.shape[-1]}, w has K={w.shape[-1]}")
    s = act_abs_mean.float().clamp(min=_TINY).pow(alpha)
    return s / s.mean()


def apply_awq_scale(w: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    return w * s
