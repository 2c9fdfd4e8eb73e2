"""DIP path parity on the GPU (mirrors the reference's
tests/test_m7_sparse_gemv.py, test_m8_fused_gemv.py and the block-level
claims of test_m8_cached_dip_pipeline.py): sparse 'down' accumulate vs the
oracle (one-hot probes exact), descriptor construction, cache-or-stream fused
GEMVs bit-identical to the plain kernels for every cache split, and the whole
DIP MLP block at the BASELINE config shapes."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import soinfer.ops as ops
from oracle import reference_port as port
from soinfer.quant import formats, pack
from tests.helpers import assert_close, fp16_randn, int4_weights

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _packed(W, g):
    qt = formats.quantize(W.float(), formats.QuantConfig(bits=4, granularity="group", group_size=g))
    p, _ = pack.pack_int4(qt.qweight)
    return p, qt.scale.contiguous(), qt


def test_sparse_accumulate_one_hot_exact():
    torch.manual_seed(0)
    k, H, g = 20, 256, 64
    p, s, qt = _packed(torch.randn(k, H) * 3.0, g)
    deq = formats.dequantize(qt).half().to(DEV)
    for i0 in range(0, k, 3):
        h = torch.zeros(k, device=DEV, dtype=torch.float16)
        h[i0] = 1.0
        y = ops.gemv_w4a16_sparse_accumulate(p.to(DEV), s.to(DEV), h, H, g)
        assert torch.equal(y, deq[i0]), f"one-hot row {i0}"


@pytest.mark.parametrize("k,H,g", [(64, 512, 128), (37, 256, 64), (3072, 2048, 128), (8704, 5120, 128),
                                   (5, 65, 32), (1, 2048, 128), (300, 1000, 40)])
def test_sparse_accumulate_matches_oracle(k, H, g):
    p, s, pk = int4_weights(k, H, g, seed=k + H)
    h = fp16_randn(k, seed=k, std=0.5)
    y = ops.gemv_w4a16_sparse_accumulate(p.to(DEV), s.to(DEV), h.to(DEV), pk, g)
    ref = port.sparse_accumulate(p.numpy(), s.numpy(), h.numpy(), pk, g)
    assert_close(y, ref, f"sparse[{k}x{H}]")


def test_sparse_accumulate_wide_h_after_a_narrow_call():
    """H above 65536 on the scalar path (g = 8) needs more than 1024
    column-slab tickets: the ticket area grows with H and is cleared before
    the launch, because the cached workspace still holds the partial rows of
    the narrower call that ran just before."""
    p0, s0, pk0 = int4_weights(3072, 2048, 128, seed=11)
    h0 = fp16_randn(3072, seed=12, std=0.5)
    ops.gemv_w4a16_sparse_accumulate(p0.to(DEV), s0.to(DEV), h0.to(DEV), pk0, 128)
    k, H, g = 40, 70000, 8
    p, s, pk = int4_weights(k, H, g, seed=13)
    h = fp16_randn(k, seed=14, std=0.5)
    ref = port.sparse_accumulate(p.numpy(), s.numpy(), h.numpy(), pk, g)
    for rep in range(2):
        y = ops.gemv_w4a16_sparse_accumulate(p.to(DEV), s.to(DEV), h.to(DEV), pk, g)
        assert_close(y, ref, f"sparse[{k}x{H}] g={g} rep {rep}")


def test_sparse_accumulate_zero_rows_and_determinism():
    p, s, pk = int4_weights(3072, 2048, 128, seed=1)
    h = fp16_randn(3072, 2, 0.5).to(DEV)
    Wd, sd = p.to(DEV), s.to(DEV)
    a = ops.gemv_w4a16_sparse_accumulate(Wd, sd, h, 2048, 128)
    for _ in range(5):
        assert torch.equal(ops.gemv_w4a16_sparse_accumulate(Wd, sd, h, 2048, 128), a)
    empty = ops.gemv_w4a16_sparse_accumulate(Wd[:0], sd[:0], h[:0], 2048, 128)
    assert torch.equal(empty, torch.zeros_like(empty))


def test_sparse_rows_bit_identical_to_gathered():
    I, H = 6144, 2048
    p, s, pk = int4_weights(I, H, 128, seed=5)
    Wd, sd = p.to(DEV), s.to(DEV)
    rows = torch.randperm(I, generator=torch.Generator().manual_seed(2))[:3072].sort().values.int().to(DEV)
    h = fp16_randn(3072, 7, 0.5).to(DEV)
    a = ops.gemv_w4a16_sparse_rows(Wd, sd, rows, h, H, 128)
    b = ops.gemv_w4a16_sparse_accumulate(Wd[rows.long()].contiguous(), sd[rows.long()].contiguous(), h, H, 128)
    assert torch.equal(a, b)


def test_sparse_rejects_shape_mismatches():
    k, H, g = 16, 128, 32
    p, s, _ = int4_weights(k, H, g, seed=3)
    Wd, sd = p.to(DEV), s.to(DEV)
    h = torch.randn(k, device=DEV, dtype=torch.float16)
    with pytest.raises(RuntimeError):
        ops.gemv_w4a16_sparse_accumulate(Wd, sd, h, H + 8, g)
    with pytest.raises(RuntimeError):
        ops.gemv_w4a16_sparse_accumulate(Wd, sd, h[:-1], H, g)
    with pytest.raises(RuntimeError):
        ops.gemv_w4a16_sparse_accumulate(Wd, sd[:-1], h, H, g)
    with pytest.raises(RuntimeError):
        ops.gemv_w4a16_sparse_accumulate(Wd, sd, h, H, 5)
    with pytest.raises(RuntimeError):
        ops.gemv_w4a16_sparse_accumulate(Wd, sd[:, :2].contiguous(), h, H, g)


# ----------------------------------------------------------- descriptors
def test_build_dip_descriptors_hits_and_misses():
    slot_of = torch.full((32,), -1, dtype=torch.int32, device=DEV)
    for slot, c in enumerate([3, 7, 15]):
        slot_of[c] = slot
    sel = torch.tensor([1, 3, 5, 7, 9, 15], dtype=torch.int32, device=DEV)
    desc, miss, mc = ops.build_dip_descriptors(sel, slot_of)
    e_desc, e_miss, e_mc = port.build_dip_descriptors(sel.cpu().numpy(), slot_of.cpu().numpy())
    assert int(mc.item()) == e_mc == 3
    assert np.array_equal(desc.cpu().numpy(), e_desc)
    assert np.array_equal(miss[:3].cpu().numpy(), e_miss)


@pytest.mark.parametrize("k,I,hot", [(3072, 6144, 1229), (8704, 17408, 3482), (16, 16, 16), (4, 16, 0)])
def test_build_dip_descriptors_config_scale(k, I, hot):
    g = torch.Generator().manual_seed(k)
    sel = torch.randperm(I, generator=g)[:k].sort().values.int()
    hot_idx = torch.randperm(I, generator=g)[:hot].sort().values
    slot_of = torch.full((I,), -1, dtype=torch.int32)
    slot_of[hot_idx] = torch.arange(hot, dtype=torch.int32)
    desc, miss, mc = ops.build_dip_descriptors(sel.to(DEV), slot_of.to(DEV))
    e_desc, e_miss, e_mc = port.build_dip_descriptors(sel.numpy(), slot_of.numpy())
    assert int(mc.item()) == e_mc
    assert np.array_equal(desc.cpu().numpy(), e_desc)
    assert np.array_equal(miss[:e_mc].cpu().numpy(), e_miss)


# ------------------------------------------------------ fused cache-or-stream
def _split(k, seed):
    perm = torch.randperm(k, generator=torch.Generator().manual_seed(seed)).tolist()
    return sorted(perm[: k // 2]), perm[k // 2:]


def _descs(k, cache_l, staging_l):
    d = torch.empty(k, dtype=torch.int64)
    for slot, j in enumerate(cache_l):
        d[j] = slot
    for pos, j in enumerate(staging_l):
        d[j] = (pos | (1 << 31)) - (1 << 32)
    return d.int().to(DEV)


@pytest.mark.parametrize("k,H,g", [(24, 256, 64), (3072, 2048, 128), (16, 128, 32)])
def test_fused_up_mixed_sources_bit_identical_to_plain(k, H, g):
    p, s, pk = int4_weights(k, H, g, seed=k)
    Wd, sd = p.to(DEV), s.to(DEV)
    cl, sl = _split(k, 1)
    desc = _descs(k, cl, sl)
    x = fp16_randn(pk, 3).to(DEV)
    plain = ops.gemv_w4a16_group_lop3(Wd, sd, x, pk, g)
    fused = ops.gemv_dip_fused_up(Wd[cl].contiguous(), sd[cl].contiguous(), Wd[sl].contiguous(), sd[sl].contiguous(),
                                  desc, x, pk, g)
    assert torch.equal(fused, plain)
    assert_close(fused, port.gemv_w4a16(p.numpy(), s.numpy(), x.cpu().numpy(), pk, g), "fused up")
    # degenerate splits
    empty_W, empty_s = Wd[:0], sd[:0]
    all_cache = torch.arange(k, dtype=torch.int32, device=DEV)
    assert torch.equal(ops.gemv_dip_fused_up(Wd, sd, empty_W, empty_s, all_cache, x, pk, g), plain)
    all_staging = all_cache | (1 << 31)
    assert torch.equal(ops.gemv_dip_fused_up(empty_W, empty_s, Wd, sd, all_staging, x, pk, g), plain)


@pytest.mark.parametrize("k,H,g", [(24, 256, 64), (3072, 2048, 128), (16, 128, 32)])
def test_fused_down_mixed_sources_bit_identical_to_plain(k, H, g):
    p, s, pk = int4_weights(k, H, g, seed=k + 1)
    Wd, sd = p.to(DEV), s.to(DEV)
    cl, sl = _split(k, 4)
    desc = _descs(k, cl, sl)
    h = fp16_randn(k, 5, 0.5).to(DEV)
    plain = ops.gemv_w4a16_sparse_accumulate(Wd, sd, h, pk, g)
    fused = ops.gemv_dip_fused_down(Wd[cl].contiguous(), sd[cl].contiguous(), Wd[sl].contiguous(),
                                    sd[sl].contiguous(), desc, h, pk, g)
    assert torch.equal(fused, plain)
    assert_close(fused, port.sparse_accumulate(p.numpy(), s.numpy(), h.cpu().numpy(), pk, g), "fused down")
    all_staging = torch.arange(k, dtype=torch.int32, device=DEV) | (1 << 31)
    assert torch.equal(ops.gemv_dip_fused_down(Wd[:0], sd[:0], Wd, sd, all_staging, h, pk, g), plain)


def test_fused_rejects_mismatched_groups():
    p, s, pk = int4_weights(8, 64, 32, seed=7)
    Wd, sd = p.to(DEV), s.to(DEV)
    desc = torch.arange(8, dtype=torch.int32, device=DEV)
    x = torch.randn(64, device=DEV, dtype=torch.float16)
    bad = torch.empty(0, sd.shape[1] + 1, dtype=torch.float32, device=DEV)
    with pytest.raises(RuntimeError):
        ops.gemv_dip_fused_up(Wd, sd, Wd[:0], bad, desc, x, 64, 32)
    with pytest.raises(RuntimeError):
        ops.gemv_dip_fused_up(Wd, sd[:, :1].contiguous(), Wd[:0], sd[:0, :1].contiguous(), desc, x, 64, 32)


# --------------------------------------------------------- whole DIP block
@pytest.mark.parametrize("H,I,k", [(2048, 6144, 3072), (256, 512, 256)])
def test_dip_mlp_block_matches_oracle_and_cached_is_bit_identical(H, I, k):
    g = 128 if H >= 1024 else 64
    gate = int4_weights(I, H, g, seed=1)
    up = int4_weights(I, H, g, seed=2)
    down_t = int4_weights(I, H, g, seed=3)  # transposed down_proj [I, H]
    x = fp16_randn(H, 4).to(DEV)
    gW, gS = gate[0].to(DEV), gate[1].to(DEV)
    uW, uS = up[0].to(DEV), up[1].to(DEV)
    dW, dS = down_t[0].to(DEV), down_t[1].to(DEV)

    gate_out = ops.gemv_w4a16_group_lop3(gW, gS, x, H, g)
    abs_g = gate_out.float().abs().contiguous()
    idx = ops.topk_threshold_select(abs_g, k)
    e_idx, _ = port.topk_threshold_select_ref(abs_g.cpu().numpy(), k)
    assert np.array_equal(idx.cpu().numpy(), e_idx)  # bit-exact selection on the same gate values
    u_sel = ops.gemv_w4a16_rows(uW, uS, idx, x, H, g)
    h_sel = (F.silu(gate_out[idx.long()].float()) * u_sel.float()).half()
    y = ops.gemv_w4a16_sparse_rows(dW, dS, idx, h_sel, H, g)

    ref = port.dip_mlp_block(x.cpu().numpy(), (gate[0].numpy(), gate[1].numpy()), (up[0].numpy(), up[1].numpy()),
                             (down_t[0].numpy(), down_t[1].numpy()), k, g, H, gate_out=gate_out.cpu().numpy())
    assert_close(u_sel, ref["up_sel"].astype(np.float64), "dip up_sel")
    # the down input is our own h_sel (fp16 rounding of silu may differ by an ulp from the oracle's)
    y_ref = port.sparse_accumulate(down_t[0].numpy()[e_idx], down_t[1].numpy()[e_idx], h_sel.cpu().numpy(), H, g)
    assert_close(y, y_ref, "dip y")
    assert_close(h_sel, ref["h_sel"].astype(np.float64), "dip h_sel")

    # cache-aware DIP: 20% hot set, misses staged -> bit-identical to plain DIP
    hot = torch.randperm(I, generator=torch.Generator().manual_seed(9))[: I // 5].sort().values
    slot_of = torch.full((I,), -1, dtype=torch.int32)
    slot_of[hot] = torch.arange(hot.numel(), dtype=torch.int32)
    desc, miss, mc = ops.build_dip_descriptors(idx, slot_of.to(DEV))
    m = miss[: int(mc.item())].long()
    hot_d = hot.to(DEV)
    u_c = ops.gemv_dip_fused_up(uW[hot_d], uS[hot_d], uW[m].contiguous(), uS[m].contiguous(), desc, x, H, g)
    assert torch.equal(u_c, u_sel)
    y_c = ops.gemv_dip_fused_down(dW[hot_d], dS[hot_d], dW[m].contiguous(), dS[m].contiguous(), desc, h_sel, H, g)
    assert torch.equal(y_c, y)


@pytest.mark.parametrize("n,K,k", [(6144, 2048, 3072), (17408, 5120, 8704), (300, 512, 37)])
def test_fused_epilogues_equal_unfused(n, K, k):
    """The rows GEMV with the SwiGLU epilogue equals rows GEMV then swiglu, and
    the sparse down with the residual epilogue equals sparse down then the
    fp16 add -- bit for bit (the DIP layer uses the fused forms)."""
    gen = torch.Generator().manual_seed(n + k)
    uW, uS, pk = (t.to(DEV) if torch.is_tensor(t) else t for t in int4_weights(n, K, 128, seed=n))
    dW, dS, _ = (t.to(DEV) if torch.is_tensor(t) else t for t in int4_weights(n, K, 128, seed=n + 1))
    x = fp16_randn(pk, seed=k).to(DEV)
    gate = fp16_randn(n, seed=k + 1, std=2.0).to(DEV)
    idx = torch.randperm(n, generator=gen)[:k].sort()[0].int().to(DEV)
    fused = ops.gemv_w4a16_rows(uW, uS, idx, x, pk, 128, glu_gate=gate)
    plain = ops.swiglu(gate, ops.gemv_w4a16_rows(uW, uS, idx, x, pk, 128), idx)
    assert torch.equal(fused, plain)
    res = fp16_randn(pk, seed=k + 2).to(DEV)
    a = ops.gemv_w4a16_sparse_rows(dW, dS, idx, fused, pk, 128, residual=res)
    b = res + ops.gemv_w4a16_sparse_rows(dW, dS, idx, fused, pk, 128)
    assert torch.equal(a, b)
