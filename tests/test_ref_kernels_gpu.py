"""Direct comparison with the reference's own CUDA kernels on the same B200.

oracle/_ref/libsoinfer_ref.so is the reference's csrc/kernels/*.cu compiled
from its sources for sm_100a (oracle/Makefile `ref`).  Here it pins the
oracle restatement (selector bit-exact vs the reference kernel) and shows the
sm_100a kernels agree with the reference implementation itself: selector
bit-exact, GEMV / sparse / attention within the parity tolerance.  Skipped
when the reference library was not built (it needs the reference sources)."""
import numpy as np
import pytest
import torch

import soinfer.ops as ops
from oracle import native
from oracle import reference_port as port
from soinfer import _C
from tests.helpers import assert_close, fp16_randn, int4_weights

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not native.ref_available(), reason="oracle/_ref not built (needs reference sources)")]
DEV = "cuda"


def _p(t):
    return t.data_ptr()


def _ref_topk(v: torch.Tensor, k: int):
    idx = torch.full((k,), -7, dtype=torch.int32, device=DEV)
    cnt = torch.zeros(1, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    native.ref_lib().ref_topk_threshold_select(_p(v), v.numel(), k, _p(idx), _p(cnt))
    torch.cuda.synchronize()
    return idx, int(cnt.item())


@pytest.mark.parametrize("n,k,dist,seed", [(6144, 3072, "fp16_gate", s) for s in range(8)] + [
    (17408, 8704, "fp16_gate", 0), (17408, 8704, "fp16_gate", 1), (11008, 5504, "continuous", 0),
    (8192, 2048, "heavy_ties", 0), (1024, 1, "continuous", 1), (1024, 1024, "continuous", 2), (4096, 1, "fp16_gate", 3)])
def test_selector_bit_exact_vs_reference_kernel(n, k, dist, seed):
    rng = np.random.default_rng(1000 * seed + n)
    if dist == "fp16_gate":
        v = np.abs(rng.standard_normal(n).astype(np.float16)).astype(np.float32)
    elif dist == "continuous":
        v = (rng.random(n) * 10).astype(np.float32)
    else:
        v = rng.integers(0, 10, n).astype(np.float32)
    vd = torch.from_numpy(v).to(DEV)
    r_idx, r_cnt = _ref_topk(vd, k)
    ours, cnt = _C.topk_threshold_select(vd, k)
    assert int(cnt.item()) == r_cnt
    assert torch.equal(ours[:r_cnt], r_idx[:r_cnt])
    o_idx, o_cnt = port.topk_threshold_select_ref(v, k)  # the oracle is pinned to the reference kernel
    assert o_cnt == r_cnt and np.array_equal(o_idx[:o_cnt], r_idx[:r_cnt].cpu().numpy())


@pytest.mark.parametrize("N,K", [(6144, 2048), (2048, 6144), (512, 4096)])
def test_gemv_vs_reference_kernel(N, K):
    p, s, pk = int4_weights(N, K, 128, seed=N)
    Wd, sd = p.to(DEV), s.to(DEV)
    x = fp16_randn(pk, 1).to(DEV)
    y_ref = torch.empty(N, dtype=torch.float16, device=DEV)
    torch.cuda.synchronize()
    native.ref_lib().ref_gemv_w4a16_group_lop3(_p(Wd), _p(sd), _p(x), _p(y_ref), N, pk, 128, sd.shape[1])
    torch.cuda.synchronize()
    ours = ops.gemv_w4a16_group_lop3(Wd, sd, x, pk, 128)
    oracle = port.gemv_w4a16(p.numpy(), s.numpy(), x.cpu().numpy(), pk, 128)
    assert_close(y_ref, oracle, "reference kernel vs oracle")
    assert_close(ours, y_ref.double(), "ours vs reference kernel")


def test_sparse_and_fused_down_vs_reference_kernel():
    k, H = 3072, 2048
    p, s, pk = int4_weights(k, H, 128, seed=3)
    Wd, sd = p.to(DEV), s.to(DEV)
    h = fp16_randn(k, 2, 0.5).to(DEV)
    y_ref = torch.empty(H, dtype=torch.float16, device=DEV)
    torch.cuda.synchronize()
    native.ref_lib().ref_sparse_accumulate(_p(Wd), _p(sd), _p(h), _p(y_ref), H, k, 128, sd.shape[1])
    torch.cuda.synchronize()
    assert_close(ops.gemv_w4a16_sparse_accumulate(Wd, sd, h, H, 128), y_ref.double(), "sparse vs reference kernel")


@pytest.mark.parametrize("nq,nkv,max_seq,cur_len", [(16, 8, 2048, 2048), (40, 8, 4096, 1000), (16, 8, 512, 1)])
def test_decode_attention_vs_reference_kernel(nq, nkv, max_seq, cur_len):
    torch.manual_seed(1)
    q = torch.randn(nq, 128, device=DEV, dtype=torch.float16)
    kc = torch.randn(nkv, max_seq, 128, device=DEV, dtype=torch.float16)
    vc = torch.randn_like(kc)
    out_ref = torch.empty_like(q)
    torch.cuda.synchronize()
    native.ref_lib().ref_decode_attention(_p(q), _p(kc), _p(vc), _p(out_ref), nq, nkv, max_seq, 128, cur_len,
                                          1.0 / np.sqrt(128.0))
    torch.cuda.synchronize()
    assert_close(ops.decode_attention(q, kc, vc, cur_len), out_ref.double(), "attention vs reference kernel")


def test_rmsnorm_vs_reference_kernel():
    torch.manual_seed(2)
    x = torch.randn(4, 2048, device=DEV, dtype=torch.float16)
    w = torch.randn(2048, device=DEV, dtype=torch.float16)
    out_ref = torch.empty_like(x)
    torch.cuda.synchronize()
    native.ref_lib().ref_rmsnorm(_p(x), _p(w), _p(out_ref), 4, 2048, 1e-6)
    torch.cuda.synchronize()
    assert_close(ops.rmsnorm(x, w, 1e-6), out_ref.double(), "rmsnorm vs reference kernel")
