"""Quantize / pack parity with the reference (bit-exact), on the CPU.

Fixtures in tests/golden/quant_golden.npz were produced by the reference's own
python/soinfer/quant (tests/golden/make_golden.py).  Both the soinfer.quant
package (the product's load-time path) and the oracle restatement are checked
against them.  Mirrors the reference's tests/test_quant_roundtrip.py.
"""
import os

import numpy as np
import pytest
import torch

from oracle import reference_port as port
from soinfer.quant import calibrate, formats, pack

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "quant_golden.npz"))


@pytest.mark.parametrize("case", range(5))
def test_int4_group_quantize_pack_bit_exact(case):
    p = f"int4_{case}_"
    n, k, g, packed_k = (int(v) for v in GOLD[p + "meta"])
    w = torch.from_numpy(GOLD[p + "w"])
    qt = formats.quantize(w, formats.QuantConfig(bits=4, granularity="group", group_size=g))
    assert np.array_equal(qt.qweight.numpy(), GOLD[p + "q"])
    assert np.array_equal(qt.scale.numpy().view(np.uint32), GOLD[p + "scale"].view(np.uint32))
    packed, pk = pack.pack_int4(qt.qweight)
    assert pk == packed_k
    assert np.array_equal(packed.numpy(), GOLD[p + "packed"])
    assert np.array_equal(formats.dequantize(qt).numpy(), GOLD[p + "dequant"])
    # the oracle restatement agrees bit for bit too
    q2, s2 = port.quantize_group(GOLD[p + "w"], g)
    assert np.array_equal(q2, GOLD[p + "q"])
    assert np.array_equal(s2.view(np.uint32), GOLD[p + "scale"].view(np.uint32))
    assert np.array_equal(port.pack_int4(q2), GOLD[p + "packed"])
    assert np.array_equal(port.unpack_int4(GOLD[p + "packed"], packed_k), GOLD[p + "q"])
    deq = port.dequant_int4(GOLD[p + "packed"], GOLD[p + "scale"], packed_k, g)[:, :k]
    assert np.array_equal(deq, GOLD[p + "dequant"])


def test_config_shape_rows_bit_exact():
    torch.manual_seed(0)
    w = torch.randn(6144, 2048) * 0.02
    rows = w[:64]
    chk = GOLD["cfg_w64_check"]
    assert np.array_equal(rows[0, :16].numpy(), GOLD["cfg_w64_prefix"])
    assert abs(rows.double().sum().item() - chk[0]) < 1e-9 and abs(rows.double().abs().sum().item() - chk[1]) < 1e-9
    qt = formats.quantize(rows, formats.QuantConfig(bits=4, granularity="group", group_size=128))
    assert np.array_equal(qt.qweight.numpy(), GOLD["cfg_q64"])
    assert np.array_equal(qt.scale.numpy(), GOLD["cfg_scale64"])
    assert np.array_equal(pack.pack_int4(qt.qweight)[0].numpy(), GOLD["cfg_packed64"])


def test_awq_byte_layout_known_answer():
    """Known answer from the reference's tests/test_quant_roundtrip.py:41-59."""
    q = torch.from_numpy(GOLD["kat_q"])
    packed, k = pack.pack_int4(q)
    assert k == 8
    assert np.array_equal(packed.numpy(), GOLD["kat_packed"])
    v = [int(t) for t in GOLD["kat_q"]]
    nib = [t & 0xF for t in v]
    expected = [nib[0] | nib[2] << 4, nib[4] | nib[6] << 4, nib[1] | nib[3] << 4, nib[5] | nib[7] << 4]
    assert packed.tolist() == expected
    assert np.array_equal(port.pack_int4(GOLD["kat_q"]), GOLD["kat_packed"])


def test_pack_roundtrip_multidim_ragged():
    q = torch.from_numpy(GOLD["rt_q"])
    packed, k = pack.pack_int4(q)
    assert np.array_equal(packed.numpy(), GOLD["rt_packed"])
    assert torch.equal(pack.unpack_int4(packed, k), q)
    assert np.array_equal(port.unpack_int4(GOLD["rt_packed"], 21), GOLD["rt_q"])


@pytest.mark.parametrize("shape", [(1,), (7,), (8,), (9,), (16,), (17,), (3, 8), (3, 13), (4, 5, 21)])
def test_int4_pack_unpack_roundtrip(shape):
    q = torch.randint(-8, 8, shape, dtype=torch.int8)
    packed, k = pack.pack_int4(q)
    assert packed.shape[-1] == -(-shape[-1] // 8) * 4
    assert torch.equal(pack.unpack_int4(packed, k), q)
    assert np.array_equal(port.pack_int4(q.numpy()), packed.numpy())


@pytest.mark.parametrize("gran", ["per_tensor", "per_channel", "group"])
def test_int8_formats_bit_exact(gran):
    w = torch.from_numpy(GOLD["int8_w"])
    qt = formats.quantize(w, formats.QuantConfig(bits=8, granularity=gran, group_size=128 if gran == "group" else None))
    assert np.array_equal(qt.qweight.numpy(), GOLD[f"int8_{gran}_q"])
    assert np.array_equal(qt.scale.numpy(), GOLD[f"int8_{gran}_scale"])
    if gran == "per_channel":
        q2, s2 = port.quantize_per_channel(GOLD["int8_w"])
    elif gran == "per_tensor":
        q2, s2 = port.quantize_per_tensor(GOLD["int8_w"])
    else:
        q2, s2 = port.quantize_group(GOLD["int8_w"], 128, bits=8)
    assert np.array_equal(q2, GOLD[f"int8_{gran}_q"])
    assert np.array_equal(s2, GOLD[f"int8_{gran}_scale"])


@pytest.mark.parametrize("gran", ["block32", "mx_e8m0"])
def test_block_formats_bit_exact(gran):
    w = torch.from_numpy(GOLD["blk_w"])
    qt = formats.quantize(w, formats.QuantConfig(bits=4, granularity=gran))
    assert np.array_equal(qt.qweight.numpy(), GOLD[f"{gran}_q"])
    assert np.array_equal(qt.scale.numpy(), GOLD[f"{gran}_scale"])


def test_pack_rejects_wrong_dtypes():
    with pytest.raises(ValueError):
        pack.pack_int4(torch.zeros(4, dtype=torch.int32))
    with pytest.raises(ValueError):
        pack.unpack_int4(torch.zeros(4, dtype=torch.int8), 8)
    with pytest.raises(ValueError):
        formats.QuantConfig(bits=4, granularity="nope")
    with pytest.raises(ValueError):
        formats.QuantConfig(bits=4, granularity="group")


def test_zero_tensor_and_qmax():
    z = torch.zeros(8, 64)
    for gran in formats.GRANULARITIES:
        qt = formats.quantize(z, formats.QuantConfig(bits=8, granularity=gran, group_size=32))
        assert torch.equal(formats.dequantize(qt), z)
    w = torch.randn(8, 300) * 10
    for bits in (4, 8):
        qt = formats.quantize(w, formats.QuantConfig(bits=bits, granularity="group", group_size=128))
        assert qt.qweight.abs().max().item() <= formats.qmax_for_bits(bits)


def test_calibration_rules():
    torch.manual_seed(5)
    w = torch.randn(8, 128) * 3.0
    w[:, 0] *= 20.0
    cfg = formats.QuantConfig(bits=4, granularity="group", group_size=128)
    mm = formats.quantize(w, cfg, scale_fn=calibrate.min_max)
    mse = formats.quantize(w, cfg, scale_fn=calibrate.mse_optimal)
    err = lambda qt: (formats.dequantize(qt) - w).pow(2).mean().item()  # noqa: E731
    assert err(mse) <= err(mm) + 1e-6
    grouped = w.reshape(8, 1, 128)
    amax = grouped.abs().amax(-1)
    assert torch.all(calibrate.percentile(grouped, amax, 7, 99.0) <= calibrate.min_max(grouped, amax, 7) + 1e-8)
    x = torch.randn(128)
    s = calibrate.awq_scale(w, x.abs())
    assert torch.allclose(calibrate.apply_awq_scale(w, s) @ (x / s), w @ x, atol=1e-3)
