"""Direct comparison with the reference's own CUDA kernels on the same B200.

oracle/_ref/libsoinfer_ref.so is the reference's csrc/kernels/*.cu compiled
from its sources for sm_100a (oracle/Makefile `ref`).  Here it pins the
oracle restatement (selector bit-exact vs the reference kernel) and shows the
sm_100a kernels agree with the reference implementation itself: selector
bit-exact, DIP descriptors bit-exact on cache hits (misses: same channels;
the reference's miss order comes from atomics), GEMV (naive and LOP3), INT8
GEMV (per-channel, grouped, per-tensor), sparse and cache-or-stream up /
down GEMVs, attention, rmsnorm and RoPE within the parity tolerance.  Skipped
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


def test_naive_gemv_vs_reference_kernel():
    N, K = 2048, 6144
    p, s, pk = int4_weights(N, K, 128, seed=7)
    Wd, sd = p.to(DEV), s.to(DEV)
    x = fp16_randn(pk, 8).to(DEV)
    y_ref = torch.empty(N, dtype=torch.float16, device=DEV)
    torch.cuda.synchronize()
    native.ref_lib().ref_gemv_w4a16_group(_p(Wd), _p(sd), _p(x), _p(y_ref), N, pk, 128, sd.shape[1])
    torch.cuda.synchronize()
    assert_close(ops.gemv_w4a16_group(Wd, sd, x, pk, 128), y_ref.double(), "naive GEMV vs reference kernel")


@pytest.mark.parametrize("mode", ["per_channel", "grouped", "per_tensor"])
def test_gemv_w8a16_vs_reference_kernel(mode):
    N, K = 1024, 4096
    gen = torch.Generator().manual_seed(11)
    Wq = torch.randint(-127, 128, (N, K), generator=gen, dtype=torch.int8)
    if mode == "per_channel":
        g, G, rows, stride = K, 1, N, 1
    elif mode == "grouped":
        g, G, rows, stride = 128, K // 128, N, K // 128
    else:
        g, G, rows, stride = K, 1, 1, 0
    scale = (torch.rand(rows, G, generator=gen) * 2e-3 + 5e-4).float()
    x = fp16_randn(K, 12)
    Wd, sd, xd = Wq.to(DEV), scale.to(DEV), x.to(DEV)
    y_ref = torch.empty(N, dtype=torch.float16, device=DEV)
    torch.cuda.synchronize()
    native.ref_lib().ref_gemv_w8a16(_p(Wd), _p(sd), _p(xd), _p(y_ref), N, K, g, G, stride)
    torch.cuda.synchronize()
    assert_close(ops.gemv_w8a16(Wd, sd, xd, g), y_ref.double(), f"INT8 {mode} vs reference kernel", max_abs=None)


def _dip_case(seed, I=6144, H=2048, k=3072, C=1229):
    """Config-3 shapes: a hot cache of C channels, k selected channels, the
    misses staged in the descriptors' miss order (ours: ascending)."""
    rng = np.random.default_rng(seed)
    hot = np.sort(rng.choice(I, C, replace=False))
    slot_of = np.full(I, -1, np.int32)
    slot_of[hot] = np.arange(C, dtype=np.int32)
    sel = np.sort(rng.choice(I, k, replace=False)).astype(np.int32)
    sel_d, slot_d = torch.from_numpy(sel).to(DEV), torch.from_numpy(slot_of).to(DEV)
    desc, miss, cnt = ops.build_dip_descriptors(sel_d, slot_d)
    return hot, sel_d, slot_d, desc, miss[:int(cnt.item())].cpu().numpy()


def _cache_and_staging(p, s, hot, miss_ch):
    h, m = torch.from_numpy(np.asarray(hot, np.int64)), torch.from_numpy(np.asarray(miss_ch, np.int64))
    return (p[h].contiguous().to(DEV), s[h].contiguous().to(DEV), p[m].contiguous().to(DEV),
            s[m].contiguous().to(DEV))


def test_dip_descriptors_vs_reference_kernel():
    hot, sel, slot_of, desc, _ = _dip_case(21)
    k = sel.numel()
    r_desc = torch.empty(k, dtype=torch.int32, device=DEV)
    r_miss = torch.full((k,), -1, dtype=torch.int32, device=DEV)
    r_cnt = torch.zeros(1, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    native.ref_lib().ref_build_dip_descriptors(_p(sel), k, _p(slot_of), _p(r_desc), _p(r_miss), _p(r_cnt))
    torch.cuda.synchronize()
    _, miss, cnt = ops.build_dip_descriptors(sel, slot_of)
    assert int(cnt.item()) == int(r_cnt.item())
    hit = desc >= 0
    assert torch.equal(r_desc >= 0, hit)
    assert torch.equal(desc[hit], r_desc[hit])  # cache slots: bit-exact
    # misses: the reference's positions come from atomics (any order); each descriptor still names its channel
    pos, r_pos = (desc[~hit] & 0x7FFFFFFF).long(), (r_desc[~hit] & 0x7FFFFFFF).long()
    assert torch.equal(miss[pos], sel[~hit]) and torch.equal(r_miss[r_pos], sel[~hit])
    assert torch.equal(pos, torch.arange(pos.numel(), device=DEV))  # ours: ascending selected order


def test_dip_fused_up_and_down_vs_reference_kernels():
    I, H, g = 6144, 2048, 128
    hot, sel, _, desc, miss_ch = _dip_case(22, I=I, H=H)
    k = sel.numel()
    # up: rows are channels of W_up [I, H]
    p, s, pk = int4_weights(I, H, g, seed=23)
    cW, cS, sW, sS = _cache_and_staging(p, s, hot, miss_ch)
    x = fp16_randn(pk, 24).to(DEV)
    u_ref = torch.empty(k, dtype=torch.float16, device=DEV)
    torch.cuda.synchronize()
    native.ref_lib().ref_gemv_dip_fused_up(_p(cW), _p(cS), _p(sW), _p(sS), _p(desc), _p(x), _p(u_ref), k, pk, g,
                                           s.shape[1])
    torch.cuda.synchronize()
    assert_close(ops.gemv_dip_fused_up(cW, cS, sW, sS, desc, x, pk, g), u_ref.double(), "fused up vs reference")
    # down: rows are channels of down_T [I, H]
    p2, s2, pk2 = int4_weights(I, H, g, seed=25)
    cW2, cS2, sW2, sS2 = _cache_and_staging(p2, s2, hot, miss_ch)
    h = fp16_randn(k, 26, 0.5).to(DEV)
    y_ref = torch.empty(pk2, dtype=torch.float16, device=DEV)
    torch.cuda.synchronize()
    native.ref_lib().ref_gemv_dip_fused_down(_p(cW2), _p(cS2), _p(sW2), _p(sS2), _p(desc), _p(h), _p(y_ref), pk2, k,
                                             g, s2.shape[1])
    torch.cuda.synchronize()
    assert_close(ops.gemv_dip_fused_down(cW2, cS2, sW2, sS2, desc, h, pk2, g), y_ref.double(), "fused down vs reference",
                 max_abs=None)


def test_rope_vs_reference_kernel():
    torch.manual_seed(3)
    x = torch.randn(40, 128, device=DEV, dtype=torch.float16)
    cos, sin = ops.precompute_rope_cos_sin(128, 1e6, 777, DEV)
    x_ref = x.clone()
    torch.cuda.synchronize()
    native.ref_lib().ref_rope_apply(_p(x_ref), _p(cos), _p(sin), 40, 128)
    torch.cuda.synchronize()
    assert_close(ops.apply_rope(x.clone(), cos, sin), x_ref.double(), "rope vs reference kernel")
