"""GPU load-time quantize + pack (soinfer_quantize_pack_int4) bit-exact with
the reference quantizer: the golden vectors made by the reference's own
python/soinfer/quant, random shapes (ragged K, every supported group size,
fp32 / fp16 / bf16 input, strided rows), and the edge cases of the rule --
all-zero groups (scale = float32 tiny), ties at .5 (round half to even),
values that land exactly on +-7."""
import os

import numpy as np
import pytest
import torch

from soinfer import _C
from soinfer.quant import formats, pack

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "quant_golden.npz"))


def _cpu_ref(w: torch.Tensor, g: int):
    qt = formats.quantize(w.float().cpu(), formats.QuantConfig(bits=4, granularity="group", group_size=g))
    packed, pk = pack.pack_int4(qt.qweight)
    return packed, qt.scale, pk


def _check(w: torch.Tensor, g: int, tag: str):
    p, s, pk = _C.quantize_pack_int4(w, g)
    rp, rs, rpk = _cpu_ref(w, g)
    assert pk == rpk, tag
    assert torch.equal(p.cpu(), rp), f"{tag}: packed bytes differ"
    assert np.array_equal(s.cpu().numpy().view(np.uint32), rs.numpy().view(np.uint32)), f"{tag}: scales differ"


@pytest.mark.parametrize("case", range(5))
def test_golden_vectors(case):
    pre = f"int4_{case}_"
    n, k, g, packed_k = (int(v) for v in GOLD[pre + "meta"])
    p, s, pk = _C.quantize_pack_int4(torch.from_numpy(GOLD[pre + "w"]).to(DEV), g)
    assert pk == packed_k
    assert np.array_equal(p.cpu().numpy(), GOLD[pre + "packed"])
    assert np.array_equal(s.cpu().numpy().view(np.uint32), GOLD[pre + "scale"].view(np.uint32))


@pytest.mark.parametrize("g", [8, 16, 32, 64, 128, 256])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_random_shapes(g, dtype):
    gen = torch.Generator(device=DEV).manual_seed(g)
    for n, k in ((1, 8), (3, 13), (37, 300), (64, 2048), (5, 4099)):
        w = (torch.randn(n, k, generator=gen, device=DEV) * 0.02).to(dtype)
        _check(w, g, f"{n}x{k} g{g} {dtype}")


def test_strided_rows_and_large():
    gen = torch.Generator(device=DEV).manual_seed(9)
    big = torch.randn(40, 700, generator=gen, device=DEV)
    _check(big[:, :640], 128, "strided view")
    _check(torch.randn(6144, 2048, generator=gen, device=DEV) * 0.02, 128, "6144x2048")


def test_rule_edge_cases():
    g = 8
    rows = [
        [0.0] * 8,                                   # all zero: scale = tiny, q = 0
        [7.0, 2.5, -2.5, 3.5, -3.5, 0.5, -0.5, 1.5],  # scale 1: ties round to even
        [-7.0, 7.0, 6.5, -6.5, 0.0, -0.0, 4.5, 5.5],
        [1e-30, -1e-30, 0.0, 3e-31, 0.0, 0.0, 0.0, 0.0],
    ]
    w = torch.tensor(rows, dtype=torch.float32, device=DEV)
    _check(w, g, "edge cases")
    p, s, _ = _C.quantize_pack_int4(w, g)
    assert s[0, 0].item() == torch.finfo(torch.float32).tiny and int(p[0].abs().sum()) == 0
