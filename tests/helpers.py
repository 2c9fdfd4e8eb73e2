"""Shared test helpers: seeded synthetic weights and the parity tolerance.

Parity bar for floating-point outputs (GEMV, sparse accumulate, attention):
max-abs error <= 1e-2 and relative L2 error <= 1e-3 against the float64
oracle, plus the reference tests' own elementwise bound
|diff| < 1e-2 + 5e-3 * |expected| (tests/test_m4_kernels.py:21-30).
Integer / index / byte outputs are compared bit-exactly.
"""
from __future__ import annotations

import numpy as np
import torch

from soinfer.quant import formats, pack

MAX_ABS = 1e-2
REL_L2 = 1e-3
ELEM_ABS, ELEM_REL = 1e-2, 5e-3


def assert_close(actual, expected, label: str, max_abs: float | None = MAX_ABS, rel_l2: float = REL_L2) -> None:
    """max_abs=None skips the absolute bound (for unit-variance test data whose
    outputs are large enough that one fp16 ulp exceeds 1e-2; the reference
    tests use only the magnitude-scaled bound there)."""
    a = (actual.detach().float().cpu().numpy() if isinstance(actual, torch.Tensor) else np.asarray(actual)).astype(
        np.float64)
    e = (expected.detach().float().cpu().numpy() if isinstance(expected, torch.Tensor) else np.asarray(expected)).astype(
        np.float64)
    assert a.shape == e.shape, f"{label}: shape {a.shape} vs {e.shape}"
    assert np.all(np.isfinite(a)), f"{label}: non-finite output"
    diff = np.abs(a - e)
    mx = float(diff.max()) if diff.size else 0.0
    rel = float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30)) if diff.size else 0.0
    assert max_abs is None or mx <= max_abs, f"{label}: max-abs {mx:.3e} > {max_abs}"
    assert rel <= rel_l2, f"{label}: rel-L2 {rel:.3e} > {rel_l2}"
    bound = ELEM_ABS + ELEM_REL * np.abs(e)
    assert np.all(diff < bound), f"{label}: elementwise bound violated (worst {float((diff - bound).max()):.3e})"


def int4_weights(n: int, k: int, g: int = 128, seed: int = 0, std: float = 0.02):
    """Seeded W ~ N(0, std) [n, k] -> (packed uint8, scale f32, packed_k) CPU tensors."""
    gen = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=gen) * std
    qt = formats.quantize(w, formats.QuantConfig(bits=4, granularity="group", group_size=g))
    packed, packed_k = pack.pack_int4(qt.qweight)
    return packed, qt.scale.contiguous(), packed_k


def fp16_randn(n: int, seed: int, std: float = 1.0) -> torch.Tensor:
    gen = torch.Generator().manual_seed(seed)
    return (torch.randn(n, generator=gen) * std).half()
