"""INT4 / INT8 GEMV parity on the GPU (mirrors the reference's
tests/test_m4_kernels.py): exact basis-vector probes, tolerance against the
float64 oracle at the BASELINE config shapes and ragged shapes, fast-path /
generic-path agreement, row-indirect == gathered (bit-exact), and the
reference binding's error checks."""
import numpy as np
import pytest
import torch

import soinfer.ops as ops
from oracle import reference_port as port
from soinfer.quant import formats, pack
from tests.helpers import assert_close, fp16_randn, int4_weights

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _oracle_y(packed, scale, x, K, g):
    return port.gemv_w4a16(packed.numpy(), scale.numpy(), x.cpu().numpy(), K, g)


@pytest.mark.parametrize("fn", ["gemv_w4a16_group", "gemv_w4a16_group_lop3"])
@pytest.mark.parametrize("K", [256, 4096])
def test_w4a16_dequant_exact_via_basis_vectors(fn, K):
    torch.manual_seed(2)
    N, g = 16, 128
    W = torch.randn(N, K) * 3.0
    qt = formats.quantize(W, formats.QuantConfig(bits=4, granularity="group", group_size=g))
    packed, _ = pack.pack_int4(qt.qweight)
    deq = formats.dequantize(qt).half().to(DEV)
    Wd, sd = packed.to(DEV), qt.scale.to(DEV)
    eye = torch.eye(K, device=DEV, dtype=torch.float16)
    for k in range(0, K, 41):
        y = getattr(ops, fn)(Wd, sd, eye[k], K, g)
        assert torch.equal(y, deq[:, k]), f"{fn}[K={K}] column {k}"


@pytest.mark.parametrize("N,K,g", [(6144, 2048, 128), (2048, 6144, 128), (512, 4096, 128), (3072, 2048, 128),
                                   (17408, 5120, 128), (5120, 17408, 128), (1, 128, 128), (33, 256, 128),
                                   # 14B tensor-parallel row-parallel shards: o_proj / down_proj at TP 4 and 8
                                   # (10, 5, 34, 17 scale groups per row: not 16-byte scale rows)
                                   (5120, 1280, 128), (5120, 640, 128), (5120, 4352, 128), (5120, 2176, 128)])
def test_w4a16_matches_oracle_config_shapes(N, K, g):
    packed, scale, pk = int4_weights(N, K, g, seed=N + K)
    x = fp16_randn(pk, seed=K)
    y = ops.gemv_w4a16_group_lop3(packed.to(DEV), scale.to(DEV), x.to(DEV), pk, g)
    assert_close(y, _oracle_y(packed, scale, x, pk, g), f"w4a16[{N}x{K}]")


@pytest.mark.parametrize("N,K,g", [(512, 4099, 128), (64, 65, 32), (100, 512, 64), (7, 13, 8), (40, 1000, 40)])
def test_w4a16_generic_path_ragged_and_small_groups(N, K, g):
    gen = torch.Generator().manual_seed(7)
    W = torch.randn(N, K, generator=gen)
    qt = formats.quantize(W, formats.QuantConfig(bits=4, granularity="group", group_size=g))
    packed, pk = pack.pack_int4(qt.qweight)
    x = fp16_randn(pk, seed=3)
    y = ops.gemv_w4a16_group(packed.to(DEV), qt.scale.to(DEV), x.to(DEV), pk, g)
    # reference test oracle: dequant truncated to the true K, fp32 mv
    ref = torch.mv(formats.dequantize(qt).double(), x[:K].double())
    assert_close(y, ref, f"w4a16 generic [{N}x{K} g{g}]", max_abs=None)


def test_w4a16_matches_reference_golden_oracle():
    import os

    gold = np.load(os.path.join(os.path.dirname(__file__), "golden", "quant_golden.npz"))
    for case in range(3):
        p = f"gemv_{case}_"
        n, k, g, pk = (int(v) for v in gold[p + "meta"])
        y = ops.gemv_w4a16_group_lop3(torch.from_numpy(gold[p + "packed"]).to(DEV),
                                      torch.from_numpy(gold[p + "scale"]).to(DEV),
                                      torch.from_numpy(gold[p + "x"]).to(DEV), pk, g)
        assert_close(y, gold[p + "y"], f"golden gemv {case}", max_abs=None)


def test_w4a16_naive_and_lop3_agree_and_deterministic():
    packed, scale, pk = int4_weights(256, 4096, 128, seed=4)
    Wd, sd = packed.to(DEV), scale.to(DEV)
    x = fp16_randn(pk, 4).to(DEV)
    a = ops.gemv_w4a16_group(Wd, sd, x, pk, 128)
    b = ops.gemv_w4a16_group_lop3(Wd, sd, x, pk, 128)
    assert torch.equal(a, b)
    for _ in range(5):
        assert torch.equal(ops.gemv_w4a16_group_lop3(Wd, sd, x, pk, 128), a)


@pytest.mark.parametrize("N,K,nsel", [(6144, 2048, 3072), (17408, 5120, 8704), (300, 2048, 37)])
def test_rows_indirect_bit_identical_to_gathered(N, K, nsel):
    packed, scale, pk = int4_weights(N, K, 128, seed=11)
    Wd, sd = packed.to(DEV), scale.to(DEV)
    rows = torch.randperm(N, generator=torch.Generator().manual_seed(1))[:nsel].sort().values.int().to(DEV)
    x = fp16_randn(pk, 5).to(DEV)
    a = ops.gemv_w4a16_rows(Wd, sd, rows, x, pk, 128)
    b = ops.gemv_w4a16_group_lop3(Wd[rows.long()].contiguous(), sd[rows.long()].contiguous(), x, pk, 128)
    assert torch.equal(a, b)


def test_w4a16_unaligned_view_uses_generic_path():
    packed, scale, pk = int4_weights(64, 2048, 128, seed=12)
    buf = torch.zeros(packed.numel() + 4, dtype=torch.uint8, device=DEV)
    view = buf[4:].view(64, -1)
    view.copy_(packed.to(DEV))
    x = fp16_randn(pk, 6).to(DEV)
    y = ops.gemv_w4a16_group(view, scale.to(DEV), x, pk, 128)
    assert_close(y, _oracle_y(packed, scale, x.cpu(), pk, 128), "unaligned")


def test_w4a16_rejects_bad_arguments():
    packed, scale, pk = int4_weights(4, 64, 32, seed=1)
    Wd, sd = packed.to(DEV), scale.to(DEV)
    x = torch.randn(64, device=DEV, dtype=torch.float16)
    with pytest.raises(RuntimeError):
        ops.gemv_w4a16_group(Wd, sd, x, 64, 7)
    with pytest.raises(RuntimeError):
        ops.gemv_w4a16_group_lop3(Wd, sd[:, :1].contiguous(), x, 64, 32)
    with pytest.raises(RuntimeError):
        ops.gemv_w4a16_group(Wd, sd, x.float(), 64, 32)
    with pytest.raises(RuntimeError):
        ops.gemv_w4a16_group(Wd.cpu(), sd, x, 64, 32)
    with pytest.raises(RuntimeError):
        ops.gemv_w4a16_group(Wd, sd, x[:32], 64, 32)


W8_CASES = [("per_tensor", None), ("per_channel", None), ("group", 128)]


@pytest.mark.parametrize("gran,g", W8_CASES)
def test_w8a16_dequant_exact_via_basis_vectors(gran, g):
    torch.manual_seed(0)
    N, K = 16, 256
    W = torch.randn(N, K) * 3.0
    qt = formats.quantize(W, formats.QuantConfig(bits=8, granularity=gran, group_size=g))
    Wq, sd = qt.qweight.to(DEV), qt.scale.to(DEV)
    deq = formats.dequantize(qt).half().to(DEV)
    eye = torch.eye(K, device=DEV, dtype=torch.float16)
    for k in range(0, K, 37):
        assert torch.equal(ops.gemv_w8a16(Wq, sd, eye[k], g or K), deq[:, k])


@pytest.mark.parametrize("gran,g", W8_CASES)
@pytest.mark.parametrize("N,K", [(512, 4096), (5120, 5120), (17408, 5120), (64, 300)])
def test_w8a16_matches_oracle(gran, g, N, K):
    gen = torch.Generator().manual_seed(N)
    W = torch.randn(N, K, generator=gen) * 0.02
    qt = formats.quantize(W, formats.QuantConfig(bits=8, granularity=gran, group_size=g))
    x = fp16_randn(qt.qweight.shape[1], 9)  # grouped formats pad K to a multiple of the group
    y = ops.gemv_w8a16(qt.qweight.to(DEV), qt.scale.to(DEV), x.to(DEV), g or K)
    ref = port.gemv_w8a16(qt.qweight.numpy(), qt.scale.numpy(), x.numpy(), g or K)
    assert_close(y, ref, f"w8a16[{gran} {N}x{K}]")


def test_w8a16_rejects_bad_groups():
    qt = formats.quantize(torch.randn(4, 64), formats.QuantConfig(bits=8, granularity="group", group_size=16))
    Wq, sd = qt.qweight.to(DEV), qt.scale.to(DEV)
    x = torch.randn(64, device=DEV, dtype=torch.float16)
    with pytest.raises(RuntimeError):
        ops.gemv_w8a16(Wq, sd[:, :3].contiguous(), x, 16)
    qt3 = formats.quantize(torch.randn(4, 64), formats.QuantConfig(bits=8, granularity="group", group_size=3))
    with pytest.raises(RuntimeError):
        ops.gemv_w8a16(qt3.qweight.to(DEV), qt3.scale.to(DEV), x, 3)
