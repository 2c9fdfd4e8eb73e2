"""fp16 LM-head GEMV (gemv_fp16_v3) and its fused greedy argmax on the GPU:
against a float64 reference of the same fp16 inputs, ties resolved to the
lowest index (torch.argmax's rule), the workspace left reusable, ragged and
large K, and the reference's argument checks."""
import numpy as np
import pytest
import torch

from soinfer import _C, ops
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rand(n, k, seed, std=0.05):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, k, generator=g) * std).half().to(DEV), torch.randn(k, generator=g).half().to(DEV)


@pytest.mark.parametrize("N,K", [(1, 8), (1000, 2048), (151936, 2048), (4099, 5120), (64, 32768)])
def test_gemv_fp16_matches_float64(N, K):
    W, x = _rand(N, K, seed=N + K)
    y = ops.gemv_fp16_v3(W, x)
    ref = W.double().cpu().numpy() @ x.double().cpu().numpy()
    assert_close(y, ref, f"gemv_fp16 {N}x{K}", max_abs=None)


@pytest.mark.parametrize("N,K", [(1000, 2048), (151936, 2048), (777, 5120)])
def test_argmax_is_first_max_of_fp16_logits(N, K):
    W, x = _rand(N, K, seed=7 * N + K)
    for _ in range(2):  # the second call checks the workspace was left zeroed
        idx, logits = _C.gemv_fp16_argmax(W, x, logits=True)
        assert torch.equal(logits, ops.gemv_fp16_v3(W, x))
        assert int(idx.item()) == int(torch.argmax(logits).item())
    assert int(ops.lm_head_argmax(W, x).item()) == int(torch.argmax(logits).item())


def test_argmax_ties_pick_lowest_index():
    K = 256
    W = torch.zeros(5000, K, dtype=torch.float16, device=DEV)
    x = torch.ones(K, dtype=torch.float16, device=DEV)
    for r in (4321, 17, 3999):  # equal maxima
        W[r, :4] = 1.0
    assert int(ops.lm_head_argmax(W, x).item()) == 17
    W[17, :4] = 0.0
    assert int(ops.lm_head_argmax(W, x).item()) == 3999
    W.fill_(0)  # all logits +0 (and none -0 > +0): index 0
    W[2, 0] = -0.0
    assert int(ops.lm_head_argmax(W, x).item()) == 0
    W[:, 0] = -1.0  # all negative: still the first maximum
    W[4000, 0] = -0.5
    assert int(ops.lm_head_argmax(W, x).item()) == 4000


def test_argument_checks():
    W, x = _rand(16, 64, seed=1)
    with pytest.raises(RuntimeError):
        ops.gemv_fp16_v3(W, x[:32])
    with pytest.raises(RuntimeError):
        ops.gemv_fp16_v3(W.float(), x)
    with pytest.raises(RuntimeError):
        ops.gemv_fp16_v3(W[:, :60].contiguous(), x[:60].contiguous())  # K % 8
    assert ops.gemv_fp16_v3(W[:0], x).numel() == 0
