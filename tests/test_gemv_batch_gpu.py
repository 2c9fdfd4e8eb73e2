"""Persistent batched INT4 GEMV (soinfer_gemv_w4a16_batch) parity on the GPU:
independent and chained tasks at the BASELINE config shapes against the
float64 oracle, exact basis-vector probes through the biased-MMA path,
determinism across launches (the counters reset themselves), the per-task
fallback for shapes outside the fast path, and argument checks."""
import numpy as np
import pytest
import torch

import soinfer.ops as ops
from oracle import reference_port as port
from soinfer import _C
from soinfer.quant import formats, pack
from tests.helpers import assert_close, fp16_randn, int4_weights

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _dev(w):
    return w[0].to(DEV), w[1].to(DEV), w[2]


@pytest.mark.parametrize("shapes", [
    [(6144, 2048), (2048, 6144), (3072, 2048)],
    [(17408, 5120), (5120, 17408), (1024, 5120)],
    [(16, 128), (1, 256), (300, 1024), (6144, 2048)],
])
def test_independent_tasks_match_oracle(shapes):
    tasks, refs = [], []
    for i, (n, k) in enumerate(shapes):
        p, s, pk = int4_weights(n, k, 128, seed=10 + i)
        x = fp16_randn(pk, 20 + i)
        y = torch.empty(n, dtype=torch.float16, device=DEV)
        tasks.append((p.to(DEV), s.to(DEV), x.to(DEV), y, pk, 128, -1))
        refs.append(port.gemv_w4a16(p.numpy(), s.numpy(), x.numpy(), pk, 128))
    _C.gemv_w4a16_batch(tasks)
    torch.cuda.synchronize()
    assert _C.device_errors() == 0
    for i, t in enumerate(tasks):
        assert_close(t[3], refs[i], f"batch task {i} {shapes[i]}")


def test_large_independent_batch_takes_the_stream_kernel():
    """A batch of plain, independent GEMVs large enough for the streaming
    kernel (gemv_stream.cu: one warp per 48-row unit over the full K, units
    handed out by a ticket): 40 tasks over four matrices -- the configs[0]
    gate and down shapes, a ragged N and a group size of 256 -- every task
    against the single-GEMV op, three of them against the float64 oracle, and
    two launches bit-identical (the ticket resets itself)."""
    shapes = [(6144, 2048, 128), (2048, 6144, 128), (6000, 2048, 128), (4000, 4096, 256)]
    mats = [int4_weights(n, k, g, seed=80 + i) for i, (n, k, g) in enumerate(shapes)]
    dmats = [(p.to(DEV), s.to(DEV)) for p, s, _ in mats]
    tasks, xs = [], []
    for i in range(40):
        m = i % 4
        n, k, g = shapes[m]
        x = fp16_randn(k, 90 + i)
        xs.append(x)
        tasks.append((dmats[m][0], dmats[m][1], x.to(DEV), torch.empty(n, dtype=torch.float16, device=DEV), k, g, -1))
    batch = _C.GemvBatch(tasks)
    batch.run()
    torch.cuda.synchronize()
    assert _C.device_errors() == 0
    first = [t[3].clone() for t in tasks]
    for t in tasks:
        t[3].fill_(0)
    batch.run()
    torch.cuda.synchronize()
    for i, t in enumerate(tasks):
        assert torch.equal(t[3], first[i]), f"task {i}: second launch differs"
        single = ops.gemv_w4a16_group_lop3(t[0], t[1], t[2], t[4], t[5])
        assert_close(t[3], single.float().cpu().numpy(), f"stream task {i} vs single GEMV")
    for i in (0, 1, 2, 3):
        p, s, pk = mats[i % 4]
        ref = port.gemv_w4a16(p.numpy(), s.numpy(), xs[i].numpy(), pk, shapes[i % 4][2])
        assert_close(tasks[i][3], ref, f"stream task {i} vs oracle")


def _kernel_names(fn):
    """Names of the CUDA kernels fn launches (CUPTI through torch.profiler)."""
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return {e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA}


def test_chained_large_batch_takes_the_stream_kernel():
    """Dependent tasks on the streaming kernel: 30 gate -> down chains (each
    down reads its gate's output: the planner numbers every gate unit before
    any down unit, a waiting warp leaves bubbles instead of blocking), one
    chain extended by a third task that writes in place over the first gate's
    output after the down has read it (write after read / write after write,
    allowed because it waits for both).  Every output against the same chain
    run as ordered single-GEMV ops, the launch seen to be gemv_stream_kernel,
    two launches bit-identical and the workspace's counters zero afterwards."""
    shapes = [(6144, 2048), (2048, 6144)]
    mats = [int4_weights(n, k, 128, seed=300 + i) for i, (n, k) in enumerate(shapes)]
    (gw, gs), (dw, ds) = [(p.to(DEV), s.to(DEV)) for p, s, _ in mats]
    tasks, xs, gates, downs = [], [], [], []
    for c in range(30):
        x = fp16_randn(2048, 400 + c).to(DEV)
        a = torch.empty(6144, dtype=torch.float16, device=DEV)
        b = torch.empty(2048, dtype=torch.float16, device=DEV)
        xs.append(x)
        gates.append(len(tasks))
        tasks.append((gw, gs, x, a, 2048, 128, -1))
        downs.append(len(tasks))
        tasks.append((dw, ds, a, b, 6144, 128, len(tasks) - 1))
    a0, b0 = tasks[gates[0]][3], tasks[downs[0]][3]
    tasks.append((gw, gs, b0, a0, 2048, 128, downs[0]))  # b0 -> a0, in place over gate 0's output
    batch = _C.GemvBatch(tasks)
    names = _kernel_names(batch.run)
    assert any("gemv_stream_kernel" in n for n in names), sorted(names)
    assert _C.device_errors() == 0
    first = [t[3].clone() for t in tasks]
    for t in tasks:
        t[3].fill_(0)
    batch.run()
    torch.cuda.synchronize()
    assert _C.device_errors() == 0
    for i, t in enumerate(tasks):
        assert torch.equal(t[3], first[i]), f"task {i}: second launch differs"
    dev = torch.device("cuda", torch.cuda.current_device())
    ws = _C._workspaces[("batch", dev.index, _C._stream(dev))]
    assert int(ws.count_nonzero()) == 0, "stream counters not reset"
    for c in range(30):
        a_ref = ops.gemv_w4a16_group_lop3(gw, gs, xs[c], 2048, 128)
        b_ref = ops.gemv_w4a16_group_lop3(dw, ds, a_ref, 6144, 128)
        if c > 0:
            assert_close(tasks[gates[c]][3], a_ref.double().cpu().numpy(), f"chain {c} gate")
        assert_close(tasks[downs[c]][3], b_ref.double().cpu().numpy(), f"chain {c} down")
        if c == 0:
            a2_ref = ops.gemv_w4a16_group_lop3(gw, gs, b_ref, 2048, 128)
            assert_close(a0, a2_ref.double().cpu().numpy(), "chain 0 third task (in place)")


def test_mixed_item_sizes_share_the_ring():
    """One CTA's item stream mixes large and small items in an irregular
    order, so the ring's wrap point moves from lap to lap: every task still
    matches the oracle, launch after launch (a placement that overwrote a live
    item would corrupt whichever task was still being consumed)."""
    mats = [int4_weights(n, k, 128, seed=60 + i) for i, (n, k) in enumerate([(6144, 2048), (740, 2048), (300, 4096)])]
    dmats = [(p.to(DEV), s.to(DEV), pk) for p, s, pk in mats]
    order = [0, 1, 0, 0, 2, 1, 1, 0, 2, 0, 1, 0, 0, 0, 2, 2, 1, 0, 1, 0, 2, 0, 0, 1]
    tasks, refs = [], []
    for i, m in enumerate(order):
        p, s, pk = mats[m]
        x = fp16_randn(pk, 70 + i)
        y = torch.empty(p.size(0), dtype=torch.float16, device=DEV)
        tasks.append((dmats[m][0], dmats[m][1], x.to(DEV), y, pk, 128, -1))
        refs.append(port.gemv_w4a16(p.numpy(), s.numpy(), x.numpy(), pk, 128))
    batch = _C.GemvBatch(tasks)
    for rep in range(3):
        batch.run()
        torch.cuda.synchronize()
        assert _C.device_errors() == 0
        for i, t in enumerate(tasks):
            assert_close(t[3], refs[i], f"rep {rep} task {i} (matrix {order[i]})")


@pytest.mark.parametrize("shapes,g", [
    # tensor-parallel shards of the 14B layer: K-segmented down_proj (TP 1 / 2), scale rows of
    # 17, 10, 5 groups (not 16-byte rows: staged by plain loads)
    ([(5120, 17408), (5120, 8704), (5120, 2176), (5120, 1280), (5120, 640)], 128),
    ([(2048, 17408), (1000, 8192)], 256),   # segments of whole 256-groups
    ([(4352, 5120), (17, 8704)], 128),      # gate/up shard at TP 4 next to a ragged segmented task
])
def test_segmented_and_unaligned_scale_tasks_match_oracle(shapes, g):
    tasks, refs = [], []
    for i, (n, k) in enumerate(shapes):
        p, s, pk = int4_weights(n, k, g, seed=40 + i)
        x = fp16_randn(pk, 50 + i)
        y = torch.empty(n, dtype=torch.float16, device=DEV)
        tasks.append((p.to(DEV), s.to(DEV), x.to(DEV), y, pk, g, -1))
        refs.append(port.gemv_w4a16(p.numpy(), s.numpy(), x.numpy(), pk, g))
    batch = _C.GemvBatch(tasks)
    for rep in range(2):
        batch.run()
        torch.cuda.synchronize()
        assert _C.device_errors() == 0
        for i, t in enumerate(tasks):
            assert_close(t[3], refs[i], f"batch task {i} {shapes[i]} g{g}")
        if rep == 0:
            first = [t[3].clone() for t in tasks]
    assert all(torch.equal(a, t[3]) for a, t in zip(first, tasks)), "results differ across launches"


def test_chained_gate_down_layers():
    H, I, L = 2048, 6144, 8
    x0 = fp16_randn(H, 1).to(DEV)
    layers = [(int4_weights(I, H, 128, seed=2 * l), int4_weights(H, I, 128, seed=2 * l + 1)) for l in range(L)]
    ys = [torch.empty(I, dtype=torch.float16, device=DEV) for _ in range(L)]
    outs = [torch.empty(H, dtype=torch.float16, device=DEV) for _ in range(L)]
    tasks = []
    x = x0
    for l, (gw, dw) in enumerate(layers):
        tasks.append((gw[0].to(DEV), gw[1].to(DEV), x, ys[l], H, 128, -1 if l == 0 else 2 * l - 1))
        tasks.append((dw[0].to(DEV), dw[1].to(DEV), ys[l], outs[l], I, 128, 2 * l))
        x = outs[l]
    batch = _C.GemvBatch(tasks)
    for rep in range(3):
        batch.run()
        torch.cuda.synchronize()
        assert _C.device_errors() == 0
        # every task against the oracle evaluated on the same (fp16) input the kernel read
        for l, (gw, dw) in enumerate(layers):
            xin = x0 if l == 0 else outs[l - 1]
            # activations grow ~1.4x per layer; beyond unit scale one fp16 ulp
            # exceeds 1e-2, so the magnitude-scaled bounds apply
            assert_close(ys[l], port.gemv_w4a16(gw[0].numpy(), gw[1].numpy(), xin.cpu().numpy(), H, 128), f"gate {l}",
                         max_abs=None)
            assert_close(outs[l], port.gemv_w4a16(dw[0].numpy(), dw[1].numpy(), ys[l].cpu().numpy(), I, 128),
                         f"down {l}", max_abs=None)
        if rep == 0:
            first = [o.clone() for o in outs]
        else:
            assert all(torch.equal(a, b) for a, b in zip(first, outs)), "batch results differ across launches"


def test_basis_vectors_exact_through_batch():
    torch.manual_seed(2)
    N, K = 64, 1024
    W = torch.randn(N, K) * 3.0
    qt = formats.quantize(W, formats.QuantConfig(bits=4, granularity="group", group_size=128))
    packed, _ = pack.pack_int4(qt.qweight)
    deq = formats.dequantize(qt).half().to(DEV)
    Wd, sd = packed.to(DEV), qt.scale.to(DEV)
    eye = torch.eye(K, device=DEV, dtype=torch.float16)
    cols = list(range(0, K, 37))
    ys = [torch.empty(N, dtype=torch.float16, device=DEV) for _ in cols]
    _C.gemv_w4a16_batch([(Wd, sd, eye[k].contiguous(), ys[i], K, 128, -1) for i, k in enumerate(cols)])
    torch.cuda.synchronize()
    for i, k in enumerate(cols):
        assert torch.equal(ys[i], deq[:, k]), f"column {k}"


def test_fallback_path_matches_single_op():
    # K not a multiple of 128 -> ordered single-GEMV launches
    p, s, pk = int4_weights(100, 200, 8, seed=3)
    x = fp16_randn(pk, 4).to(DEV)
    y = torch.empty(100, dtype=torch.float16, device=DEV)
    _C.gemv_w4a16_batch([(p.to(DEV), s.to(DEV), x, y, pk, 8, -1)])
    assert torch.equal(y, ops.gemv_w4a16_group_lop3(p.to(DEV), s.to(DEV), x, pk, 8))


def test_batch_rejects_bad_tasks():
    p, s, pk = int4_weights(16, 256, 128, seed=5)
    Wd, sd = p.to(DEV), s.to(DEV)
    x = torch.randn(256, device=DEV, dtype=torch.float16)
    y = torch.empty(16, device=DEV, dtype=torch.float16)
    with pytest.raises(RuntimeError):
        _C.gemv_w4a16_batch([(Wd, sd, x, y, 256, 128, 0)])  # self dependency
    with pytest.raises(RuntimeError):
        _C.gemv_w4a16_batch([(Wd, sd, x[:128], y, 256, 128, -1)])
    with pytest.raises(RuntimeError):
        _C.gemv_w4a16_batch([(Wd, sd[:, :1].contiguous(), x, y, 256, 128, -1)])
    with pytest.raises(RuntimeError):
        _C.gemv_w4a16_batch([])


def test_glu_and_residual_epilogues_equal_unfused():
    H, I = 2048, 6144
    gw, uw, dw = int4_weights(I, H, 128, seed=41), int4_weights(I, H, 128, seed=42), int4_weights(H, I, 128, seed=43)
    h3 = fp16_randn(H, 44).to(DEV)
    h2 = fp16_randn(H, 45).to(DEV)
    gate = torch.empty(I, dtype=torch.float16, device=DEV)
    hidden = torch.empty(I, dtype=torch.float16, device=DEV)
    out = torch.empty(H, dtype=torch.float16, device=DEV)
    up_plain = torch.empty(I, dtype=torch.float16, device=DEV)
    down_plain = torch.empty(H, dtype=torch.float16, device=DEV)
    G = [(w[0].to(DEV), w[1].to(DEV)) for w in (gw, uw, dw)]
    _C.gemv_w4a16_batch([(G[0][0], G[0][1], h3, gate, H, 128, -1),
                         (G[1][0], G[1][1], h3, hidden, H, 128, -1, None, gate),
                         (G[2][0], G[2][1], hidden, out, I, 128, 1, h2)])
    _C.gemv_w4a16_batch([(G[1][0], G[1][1], h3, up_plain, H, 128, -1)])
    assert torch.equal(hidden, ops.swiglu(gate, up_plain))
    _C.gemv_w4a16_batch([(G[2][0], G[2][1], hidden, down_plain, I, 128, -1)])
    assert torch.equal(out, h2 + down_plain)
    # the per-task fallback (K not a multiple of 128) applies the same epilogues
    p, s, pk = int4_weights(100, 200, 8, seed=46)
    x = fp16_randn(pk, 47).to(DEV)
    r = fp16_randn(100, 48).to(DEV)
    gv = fp16_randn(100, 49).to(DEV)
    y = torch.empty(100, dtype=torch.float16, device=DEV)
    _C.gemv_w4a16_batch([(p.to(DEV), s.to(DEV), x, y, pk, 8, -1, r, gv)])
    plain = ops.gemv_w4a16_group_lop3(p.to(DEV), s.to(DEV), x, pk, 8)
    assert torch.equal(y, r + ops.swiglu(gv, plain))


@pytest.mark.parametrize("k", [2048, 5120, 6144])
def test_norm_prologue_matches_rmsnorm_then_gemv(k):
    """Tasks with a norm prologue multiply rmsnorm(x) * w (computed inside the
    kernel) -- against the oracle on the oracle's rmsnorm, and against the
    separate rmsnorm op followed by the plain batched GEMV (the same fp16
    vector up to the sum-of-squares order: within one fp16 ulp per element)."""
    n = 3072
    p, s, pk = int4_weights(n, k, 128, seed=k)
    gen = torch.Generator().manual_seed(k + 1)
    x = (torch.randn(k, generator=gen) * 3).half()
    w = (torch.rand(k, generator=gen) + 0.5).half()
    eps = 1e-6
    y = torch.empty(n, dtype=torch.float16, device=DEV)
    y2 = torch.empty(n, dtype=torch.float16, device=DEV)
    P, S, X, Wn = p.to(DEV), s.to(DEV), x.to(DEV), w.to(DEV)
    _C.gemv_w4a16_batch([(P, S, X, y, pk, 128, -1, None, None, (Wn, eps)),
                         (P, S, X, y2, pk, 128, -1, None, None, (Wn, eps))])
    h = ops.rmsnorm(X.unsqueeze(0), Wn, eps).squeeze(0)
    ref_sep = torch.empty(n, dtype=torch.float16, device=DEV)
    _C.gemv_w4a16_batch([(P, S, h, ref_sep, pk, 128, -1)])
    torch.cuda.synchronize()
    assert _C.device_errors() == 0
    assert torch.equal(y, y2), "two tasks with the same prologue differ"
    hn = port.rmsnorm(x.numpy()[None], w.numpy(), eps)[0]
    assert_close(y, port.gemv_w4a16(p.numpy(), s.numpy(), hn, pk, 128), f"norm prologue K={k}", max_abs=None)
    assert_close(y, ref_sep.double(), f"norm prologue vs rmsnorm op K={k}", max_abs=None)


def test_batch_after_a_timed_out_dependency_matches_oracle():
    """Failure detection without a fault: the batch workspace's completion
    counter of task 0 is set far below zero, so task 1's dependency wait can
    never be satisfied -- it gives up after its bound (1 s), sets the error
    bit and exits, leaving the counters dirty.  device_errors() reports the
    bit and re-zeroes the cached workspaces, and the same batch then matches
    the oracle."""
    p0, s0, k0 = int4_weights(6144, 2048, 128, seed=31)
    p1, s1, k1 = int4_weights(2048, 6144, 128, seed=32)
    x = fp16_randn(k0, 33)
    y0 = torch.empty(6144, dtype=torch.float16, device=DEV)
    y1 = torch.empty(2048, dtype=torch.float16, device=DEV)
    batch = _C.GemvBatch([(p0.to(DEV), s0.to(DEV), x.to(DEV), y0, k0, 128, -1),
                          (p1.to(DEV), s1.to(DEV), y0, y1, k1, 128, 0)])
    batch.run()
    torch.cuda.synchronize()
    assert _C.device_errors() == 0
    ws = _C._workspace("batch", torch.device(DEV, torch.cuda.current_device()),
                       _C.lib().soinfer_gemv_batch_workspace_bytes(2))
    ws[:4].view(torch.int32).fill_(-(1 << 30))  # a completion count nothing can raise to the grid size
    batch.run()
    torch.cuda.synchronize()
    assert _C.device_errors() & 1, "the timed-out dependency wait did not report"
    y0.zero_(), y1.zero_()
    batch.run()
    torch.cuda.synchronize()
    assert _C.device_errors() == 0
    r0 = port.gemv_w4a16(p0.numpy(), s0.numpy(), x.numpy(), k0, 128)
    assert_close(y0, r0, "task 0 after recovery")
    r1 = port.gemv_w4a16(p1.numpy(), s1.numpy(), y0.cpu().numpy(), k1, 128)
    assert_close(y1, r1, "task 1 after recovery")
