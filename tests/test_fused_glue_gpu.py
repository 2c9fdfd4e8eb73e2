"""Fused decode-layer glue on the GPU against the unfused reference
compositions: add + rmsnorm and SwiGLU bit-identical to the separate ops /
torch expressions, the fp16-|gate| selector bit-identical to the fp32 one,
per-head norm + RoPE + KV append against the oracle (and the device-position
form bit-identical to the host-position one)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import reference_port as port
from soinfer import ops
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _h(shape, seed, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * std).half().to(DEV)


@pytest.mark.parametrize("rows,hidden", [(1, 2048), (3, 5120), (1, 6)])
def test_add_rmsnorm_bit_identical(rows, hidden):
    x, x2, w = _h((rows, hidden), 1), _h((rows, hidden), 2), _h((hidden,), 3, 0.5)
    out, s = ops.add_rmsnorm(x, x2, w, 1e-6)
    ref_s = x + x2
    assert torch.equal(s, ref_s)
    assert torch.equal(out, ops.rmsnorm(ref_s, w, 1e-6))


@pytest.mark.parametrize("n", [1, 3072, 17408])
def test_swiglu_bit_identical(n):
    gate, up = _h((n,), 4, 3.0), _h((n,), 5)
    assert torch.equal(ops.swiglu(gate, up), (F.silu(gate.float()) * up.float()).half())
    big = _h((4 * n,), 6, 3.0)
    idx = torch.randperm(4 * n, generator=torch.Generator().manual_seed(7))[:n].sort()[0].int().to(DEV)
    assert torch.equal(ops.swiglu(big, up, idx), (F.silu(big.index_select(0, idx.long()).float()) * up.float()).half())


@pytest.mark.parametrize("n,k", [(6144, 3072), (17408, 8704), (100, 1)])
def test_topk_abs_f16_matches_fp32_selector(n, k):
    gate = _h((n,), n + k)
    gate[5] = 0.0
    gate[7] = -0.0
    assert torch.equal(ops.topk_threshold_select_abs(gate, k), ops.topk_threshold_select(gate.float().abs(), k))


@pytest.mark.parametrize("nq,nkv,hd", [(16, 8, 128), (40, 8, 128), (4, 2, 64)])
def test_head_norm_rope_matches_oracle(nq, nkv, hd):
    max_seq, pos, eps = 32, 9, 1e-6
    q, k, v = _h((nq, hd), 10), _h((nkv, hd), 11), _h((nkv, hd), 12)
    qw, kw = _h((hd,), 13, 0.3), _h((hd,), 14, 0.3)
    kc, vc = (torch.zeros(nkv, max_seq, hd, dtype=torch.float16, device=DEV) for _ in range(2))
    cos_v, sin_v = ops.precompute_rope_cos_sin(hd, 1e6, pos, DEV)
    q_out = q.clone()
    ops.head_norm_rope(q_out, k, v, qw, kw, cos_v, sin_v, kc, vc, pos=pos, eps=eps)
    cn, sn = cos_v.cpu().numpy(), sin_v.cpu().numpy()
    q_ref = port.rope(port.rmsnorm(q.cpu().numpy(), qw.cpu().numpy(), eps), cn, sn)
    k_ref = port.rope(port.rmsnorm(k.cpu().numpy(), kw.cpu().numpy(), eps), cn, sn)
    assert_close(q_out, q_ref.astype(np.float64), "q")
    assert_close(kc[:, pos], k_ref.astype(np.float64), "k cache row")
    assert torch.equal(vc[:, pos], v)
    assert torch.count_nonzero(kc[:, :pos]) == 0 and torch.count_nonzero(kc[:, pos + 1:]) == 0
    # device position with the table == host position
    cos_t, sin_t = ops.precompute_rope_table(hd, 1e6, max_seq, DEV)
    kc2, vc2 = torch.zeros_like(kc), torch.zeros_like(vc)
    q2 = q.clone()
    ops.head_norm_rope(q2, k, v, qw, kw, cos_t, sin_t, kc2, vc2, pos_dev=torch.tensor([pos], dtype=torch.int32,
                                                                                       device=DEV), eps=eps)
    assert torch.equal(q2, q_out) and torch.equal(kc2, kc) and torch.equal(vc2, vc)
