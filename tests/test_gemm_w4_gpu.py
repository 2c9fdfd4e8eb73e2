"""Multi-token INT4 GEMM (soinfer_gemm_w4a16: M <= 8 tokens, one pass over
the weights) on the GPU: every token row against the float64 oracle GEMV at
the configs' shapes (1.7B and 14B matrices, 14B TP shards), group sizes 128
and 256, M = 1..8, strided X / Y rows, the per-token fallback shapes, exact
basis-vector probes, determinism across launches, and argument checks."""
import numpy as np
import pytest
import torch

from oracle import reference_port as port
from soinfer import _C, ops
from soinfer.quant import formats, pack
from tests.helpers import assert_close, int4_weights

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(n, k, g, m, seed):
    p, s, pk = int4_weights(n, k, g, seed=seed)
    gen = torch.Generator().manual_seed(seed + 1)
    X = torch.randn(m, pk, generator=gen).half()
    return p, s, pk, X


@pytest.mark.parametrize("n,k,g", [(6144, 2048, 128), (2048, 6144, 128), (3072, 2048, 128), (17408, 5120, 128),
                                   (5120, 2560, 128), (4352, 5120, 128), (1024, 4096, 256), (33, 256, 128),
                                   (5120, 17408, 128), (40, 300, 32), (1024, 20480, 256), (33, 19200, 128)])
@pytest.mark.parametrize("m", [1, 3, 8])
def test_tokens_match_oracle(n, k, g, m):
    p, s, pk, X = _case(n, k, g, m, seed=n + k + m)
    Y = ops.gemm_w4a16(p.to(DEV), s.to(DEV), X.to(DEV), pk, g)
    torch.cuda.synchronize()
    assert _C.device_errors() == 0
    for i in range(m):
        ref = port.gemv_w4a16(p.numpy(), s.numpy(), X[i].numpy(), pk, g)
        assert_close(Y[i], ref, f"gemm {n}x{k} g{g} token {i}/{m}")


def test_strided_rows_deterministic_and_out():
    p, s, pk, X = _case(6144, 2048, 128, 8, seed=3)
    big = torch.zeros(8, 2048 + 64, dtype=torch.float16, device=DEV)
    big[:, :2048] = X.to(DEV)
    Xs = big[:, :2048]                       # row stride 2112
    out = torch.empty(8, 6144 + 8, dtype=torch.float16, device=DEV)[:, :6144]
    a = _C.gemm_w4a16(p.to(DEV), s.to(DEV), Xs, pk, 128, out=out)
    b = ops.gemm_w4a16(p.to(DEV), s.to(DEV), X.to(DEV), pk, 128)
    assert torch.equal(a, b), "strided X / Y or a second launch changed the result"


def test_basis_vectors_exact():
    torch.manual_seed(2)
    N, K = 64, 1024
    W = torch.randn(N, K) * 3.0
    qt = formats.quantize(W, formats.QuantConfig(bits=4, granularity="group", group_size=128))
    packed, pk = pack.pack_int4(qt.qweight)
    deq = formats.dequantize(qt)
    cols = [0, 7, 129, 513, 1000, 1023, 640, 77]
    X = torch.zeros(8, K, dtype=torch.float16)
    for i, c in enumerate(cols):
        X[i, c] = 1.0
    Y = ops.gemm_w4a16(packed.to(DEV), qt.scale.to(DEV), X.to(DEV), pk, 128).cpu()
    for i, c in enumerate(cols):
        assert torch.equal(Y[i], deq[:, c].half()), f"column {c}"


def test_argument_checks():
    p, s, pk, X = _case(64, 256, 128, 9, seed=1)
    with pytest.raises(RuntimeError):
        ops.gemm_w4a16(p.to(DEV), s.to(DEV), X.to(DEV), pk, 128)  # 9 tokens
    lib = _C.lib()
    assert lib.soinfer_gemm_w4a16(None, None, None, 256, None, 64, 9, 64, 256, 128, 2, None) == 1


@pytest.mark.parametrize("m", [8, 3, 1])
def test_gemm_batch_streams_many_matrices_in_one_launch(m):
    """soinfer_gemm_w4a16_batch: 24 independent matrices (configs' gate /
    down shapes, a ragged N with group size 256, a 14B TP shard) times the
    same M tokens in one launch of the streaming kernel -- every token row
    equals the single-matrix GEMM within the GEMV tolerance, four tasks
    against the float64 oracle, X / Y with strides beyond K / N, and a
    second launch bit-identical (the work ticket resets itself)."""
    shapes = [(6144, 2048, 128), (2048, 6144, 128), (1000, 4096, 256), (4352, 5120, 128)]
    mats = [int4_weights(n, k, g, seed=200 + i) for i, (n, k, g) in enumerate(shapes)]
    dmats = [(p.to(DEV), s.to(DEV)) for p, s, _ in mats]
    gen = torch.Generator().manual_seed(m)
    tasks, hostX = [], []
    for i in range(24):
        n, k, g = shapes[i % 4]
        Xs = torch.randn(m, k + 64, generator=gen).half()
        hostX.append(Xs[:, :k])
        X = Xs.to(DEV)[:, :k]
        Y = torch.full((m, n + 8), 7.0, dtype=torch.float16, device=DEV)[:, :n]
        tasks.append((dmats[i % 4][0], dmats[i % 4][1], X, Y, k, g))
    batch = _C.GemmBatch(tasks)
    batch.run()
    torch.cuda.synchronize()
    assert _C.device_errors() == 0
    first = [t[3].clone() for t in tasks]
    batch.run()
    torch.cuda.synchronize()
    for i, (W, S, X, Y, k, g) in enumerate(tasks):
        assert torch.equal(Y, first[i]), f"task {i}: second launch differs"
        single = ops.gemm_w4a16(W, S, X.contiguous(), k, g)
        for r in range(m):
            assert_close(Y[r], single[r].double().cpu().numpy(), f"batch task {i} token {r} vs single GEMM")
    for i in range(4):
        p, s, pk = mats[i]
        for r in range(m):
            ref = port.gemv_w4a16(p.numpy(), s.numpy(), hostX[i][r].numpy(), pk, shapes[i][2])
            assert_close(tasks[i][3][r], ref, f"batch task {i} token {r} vs oracle")
