"""Selector parity on the GPU (mirrors the reference's tests/test_m7_kernels.py).

Ref mode must reproduce the reference selector bit-exactly (indices, order and
count) -- checked against the oracle restatement (pinned to the reference's
own kernel in test_ref_kernels_gpu.py) on continuous data, fp16-derived ties,
heavy ties, maximum sizes and k in {1, n}.  Exact mode is checked against an
exact top-k with lower-index tie-break."""
import numpy as np
import pytest
import torch

import soinfer.ops as ops
from soinfer import _C
from oracle import reference_port as port

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _gate_mags(n, seed):
    rng = np.random.default_rng(seed)
    return np.abs(rng.standard_normal(n).astype(np.float16)).astype(np.float32)


CASES = [(6144, 3072), (17408, 8704), (11008, 5504), (1024, 1), (1024, 1024), (4096, 1), (100, 37), (1, 1),
         (60000, 30000), (65537, 2)]


@pytest.mark.parametrize("n,k", CASES)
@pytest.mark.parametrize("dist", ["fp16_gate", "continuous", "heavy_ties"])
def test_ref_mode_bit_exact(n, k, dist):
    rng = np.random.default_rng(n + k)
    if dist == "fp16_gate":
        v = _gate_mags(n, n)
    elif dist == "continuous":
        v = (rng.random(n) * 10).astype(np.float32)
    else:
        v = rng.integers(0, 10, n).astype(np.float32)
    idx, cnt = _C.topk_threshold_select(torch.from_numpy(v).to(DEV), k)
    e_idx, e_cnt = port.topk_threshold_select_ref(v, k)
    assert int(cnt.item()) == e_cnt
    assert np.array_equal(idx.cpu().numpy(), e_idx)


@pytest.mark.parametrize("n,k", CASES)
@pytest.mark.parametrize("dist", ["fp16_gate", "heavy_ties", "with_nan_neg"])
def test_exact_mode(n, k, dist):
    rng = np.random.default_rng(2 * n + k)
    if dist == "fp16_gate":
        v = _gate_mags(n, n + 1)
    elif dist == "heavy_ties":
        v = rng.integers(0, 5, n).astype(np.float32)
    else:
        v = rng.standard_normal(n).astype(np.float32)
        v[rng.integers(0, n, max(1, n // 50))] = np.nan
        v[0] = -0.0
    idx = ops.topk_select_exact(torch.from_numpy(v).to(DEV), k)
    assert np.array_equal(idx.cpu().numpy(), port.topk_exact(v, k))


@pytest.mark.parametrize("n,k", [(11008, 5504), (17408, 8704), (1024, 1), (1024, 1024), (4096, 1)])
def test_matches_torch_topk_set_on_continuous_data(n, k):
    torch.manual_seed(0)
    abs_g = torch.rand(n, device=DEV) * 10.0
    for fn in (ops.topk_threshold_select, ops.topk_select_exact):
        idx = fn(abs_g, k)
        assert idx.dtype == torch.int32 and idx.shape == (k,)
        assert set(idx.tolist()) == set(torch.topk(abs_g, k).indices.tolist())


def test_repeat_determinism_at_config_scale():
    torch.manual_seed(4)
    abs_g = torch.rand(6144, device=DEV) * 10.0
    first = ops.topk_threshold_select(abs_g, 3072)
    for _ in range(9):
        assert torch.equal(ops.topk_threshold_select(abs_g, 3072), first)


def test_negative_values_short_count_tail():
    """Precondition v >= 0 violated: fewer than k values reach tau; the count
    says how many were written and the tail is -1 (the reference leaves it
    uninitialised)."""
    v = np.array([-1, -2, 3, -4, 5, -6], np.float32)
    idx, cnt = _C.topk_threshold_select(torch.from_numpy(v).to(DEV), 4)
    e, ec = port.topk_threshold_select_ref(v, 4)
    assert int(cnt.item()) == ec == 2
    assert np.array_equal(idx.cpu().numpy(), e)


def test_rejects_bad_arguments():
    abs_g = torch.rand(1024, device=DEV)
    with pytest.raises(RuntimeError):
        ops.topk_threshold_select(abs_g, 0)
    with pytest.raises(RuntimeError):
        ops.topk_threshold_select(abs_g, 1025)
    with pytest.raises(RuntimeError):
        ops.topk_threshold_select(torch.rand(4, 256, device=DEV), 10)
    with pytest.raises(RuntimeError):
        ops.topk_select_exact(abs_g.half(), 10)


@pytest.mark.parametrize("n,k", [(6144, 3072), (17408, 8704), (2176, 1088), (1000, 1), (77, 77), (300, 150)])
@pytest.mark.parametrize("dist", ["normal", "ties", "special"])
def test_fp16_abs_selector_bit_exact_with_reference(n, k, dist):
    """The |fp16 gate| selector (16-bit keys, two radix passes) against the
    reference semantics on gate.float().abs(): indices and count bit-exact,
    including heavy ties, zeros, +-inf and NaN (NaN never qualifies)."""
    gen = torch.Generator().manual_seed(n + k)
    if dist == "normal":
        g = torch.randn(n, generator=gen).half()
    elif dist == "ties":
        g = (torch.randint(-6, 7, (n,), generator=gen).float() * 0.25).half()
    else:
        g = torch.randn(n, generator=gen).half()
        g[:: 7] = 0.0
        g[3:: 11] = -0.0
        g[5:: 13] = float("inf")
        g[2:: 17] = float("nan")
        g[1:: 19] = -float("inf")
    idx, count = _C.topk_threshold_select_abs_f16(g.to(DEV), k)
    e_idx, e_count = port.topk_threshold_select_ref(g.float().abs().numpy(), k)
    got = idx.cpu().numpy()
    assert int(count.item()) == int(e_count), (int(count.item()), int(e_count))
    assert np.array_equal(got[: int(e_count)], e_idx[: int(e_count)])
    assert np.all(got[int(e_count):] == -1)
