"""Tensor-parallel host logic on CPU: the shard plan, shard slicing of
quantized matrices (== quantizing the slice), and -- with two gloo ranks --
the row-parallel partial GEMVs reduced by all_reduce against the unsharded
oracle, plus the cross-rank greedy-token agreement (ties to the lowest
global index)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import reference_port as port
from soinfer.runtime.tp import ShardPlan, agree_argmax, shard_packed


def _plan(rank=0, world=2, **kw):
    args = dict(num_heads=4, num_kv_heads=2, head_dim=64, hidden=256, intermediate=512, vocab=1000)
    args.update(kw)
    return ShardPlan(rank, world, **args)


def test_shard_plan_slices_and_checks():
    p = _plan(1, 2)
    assert p.q_rows == (128, 256) and p.kv_rows == (64, 128) and p.inter_rows == (256, 512)
    assert p.vocab_rows == (500, 1000) and p.local_heads == 2 and p.local_kv_heads == 1
    assert p.weight_slice("model.layers.0.self_attn.o_proj.weight") == (1, (128, 256))
    assert p.weight_slice("mlp.down_proj.weight") == (1, (256, 512))
    assert p.weight_slice("mlp.down_proj_T.weight") == (0, (256, 512))
    for bad in (dict(num_heads=3), dict(intermediate=384), dict(head_dim=32)):
        with pytest.raises(ValueError):
            _plan(0, 2, **bad)
    with pytest.raises(ValueError):
        _plan(2, 2)
    q14 = ShardPlan(7, 8, 40, 8, 128, 5120, 17408, 151936)  # 14B at 8 GPUs
    assert q14.inter_rows == (15232, 17408) and q14.local_kv_heads == 1


def test_shard_packed_equals_quantizing_the_slice():
    rng = np.random.default_rng(0)
    w = rng.standard_normal((64, 512)).astype(np.float32)
    q, s = port.quantize_group(w, 128)
    packed = torch.from_numpy(port.pack_int4(q))
    scale = torch.from_numpy(s)
    for axis, sl in ((0, (16, 48)), (1, (128, 384))):
        pk, sc = shard_packed(packed, scale, axis, sl, 128)
        ws = w[sl[0]:sl[1]] if axis == 0 else w[:, sl[0]:sl[1]]
        q2, s2 = port.quantize_group(ws, 128)
        assert np.array_equal(pk.numpy(), port.pack_int4(q2)) and np.array_equal(sc.numpy(), s2)
    with pytest.raises(ValueError):
        shard_packed(packed, scale, 1, (64, 256), 128)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port_no, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port_no))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = _plan(rank, world)
        rng = np.random.default_rng(5)
        H, I = plan.hidden, plan.intermediate
        wd = rng.standard_normal((H, I)).astype(np.float32) * 0.05  # down_proj, row-parallel
        q, s = port.quantize_group(wd, 128)
        packed, scale = torch.from_numpy(port.pack_int4(q)), torch.from_numpy(s)
        x = rng.standard_normal(I).astype(np.float16)
        axis, sl = plan.weight_slice("mlp.down_proj.weight")
        pk, sc = shard_packed(packed, scale, axis, sl, 128)
        partial = port.gemv_w4a16(pk.numpy(), sc.numpy(), x[sl[0]:sl[1]], sl[1] - sl[0], 128)
        t = torch.from_numpy(partial.astype(np.float64))
        dist.all_reduce(t)
        full = port.gemv_w4a16(packed.numpy(), scale.numpy(), x, I, 128)
        ok_reduce = bool(np.allclose(t.numpy(), full, rtol=1e-12, atol=1e-9))
        # greedy agreement: rank 0 holds the max at local 7, rank 1 ties it at local 2 (global index higher)
        lo, hi = plan.vocab_rows
        logit = torch.tensor([3.5 if rank == 0 else 3.5], dtype=torch.float16)
        idx = torch.tensor([7 if rank == 0 else 2], dtype=torch.int32)
        tie = int(agree_argmax(logit, idx, lo).item())
        logit2 = torch.tensor([1.0 if rank == 0 else 2.0], dtype=torch.float16)
        win = int(agree_argmax(logit2, idx, lo).item())
        results[rank] = (ok_reduce, tie, win, hi)
    finally:
        dist.destroy_process_group()


def test_row_parallel_reduce_and_argmax_agreement_gloo():
    world = 2
    with mp.Manager() as mgr:
        results = mgr.dict()
        mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        res = dict(results)
    assert all(res[r][0] for r in range(world)), res
    assert res[0][1] == res[1][1] == 7          # tie: the lower global index (rank 0's 7 < 500 + 2)
    assert res[0][2] == res[1][2] == 500 + 2    # rank 1's larger logit wins


def _sweep_worker(rank, world, port_no, results):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port_no)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from soinfer.runtime.tp import allreduce_sweep

    rows = allreduce_sweep("cpu", sizes=(1024, 64 * 1024), iters=3, warmup=1)
    results[rank] = rows
    dist.destroy_process_group()


def test_allreduce_sweep_reports_every_size_on_every_rank():
    """The all-reduce sweep's host logic on two gloo ranks: one row per size,
    the same (max-over-ranks) time on both ranks, a positive bus bandwidth."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port_no = s.getsockname()[1]
    results = mp.Manager().dict()
    mp.spawn(_sweep_worker, args=(2, port_no, results), nprocs=2, join=True)
    a, b = results[0], results[1]
    assert [r["bytes"] for r in a] == [1024, 64 * 1024] and a == b
    assert all(r["world"] == 2 and r["nccl_us"] > 0 and r["nccl_busbw_gbs"] >= 0 for r in a)
