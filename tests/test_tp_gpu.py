"""Tensor-parallel decode on two GPUs (NCCL, one process per GPU), each rank
also holding the unsharded model on its own device:

* a rank's shard matrices are exactly the slices of the full quantized
  matrices (same seed -> same weights);
* decoder layers with the row-parallel all-reduces match the single-GPU
  layers within a tolerance (each shard rounds its partial to fp16, so not
  bit for bit);
* the vocabulary-parallel LM head picks exactly the single-GPU argmax for
  the same normed hidden state;
* eager TP decode gives the same tokens on every rank, and the CUDA-graph TP
  decoder (NCCL collectives inside the graph) gives the eager tokens.

Skipped with fewer than two GPUs."""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ARCH_ARGS = dict(num_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2,
                 head_dim=128, vocab_size=512)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rel_l2(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _worker(rank, world, port_no, results):
    from soinfer.runtime import generate as gen
    from soinfer.runtime.loader import Architecture, synthetic_streaming_model
    from soinfer.runtime.tp import (ShardPlan, build_tp_model, generate_tp, graph_decoder_tp, run_decoder_layer_tp,
                                    tp_next_token)

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port_no), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    out = {}
    try:
        arch = Architecture(**ARCH_ARGS)
        plan = ShardPlan(rank, world, arch.num_attention_heads, arch.num_key_value_heads, arch.head_dim,
                         arch.hidden_size, arch.intermediate_size, arch.vocab_size)
        full = synthetic_streaming_model(arch, seed=3, resident=True, offload=False, include_dip=False, device=dev)
        tp = build_tp_model(arch, plan, seed=3, device=dev)

        # shards are slices of the full matrices
        exact = True
        for name, m in tp.matrices.items():
            suffix = name.split(".", 3)[3]
            axis, (a, b) = plan.weight_slice(suffix)
            fm = full.matrices[name]
            fp, fs = full.resident[name], fm.scale
            if axis == 0:
                ref_p, ref_s = fp[a:b], fs[a:b]
            else:
                ref_p, ref_s = fp[:, a // 2:b // 2], fs[:, a // 128:b // 128]
            exact &= torch.equal(tp.resident[name], ref_p) and torch.equal(m.scale, ref_s)
        lo, hi = plan.vocab_rows
        exact &= torch.equal(tp.lm_head, full.lm_head[lo:hi])
        out["shards_exact"] = bool(exact)

        # layers: TP vs single GPU, teacher-forced through both layers for 3 positions
        kf, vf = gen._kv_caches(full, 16)
        kt, vt = gen._kv_caches(tp, 16)
        pf, pt = gen.WeightPipeline(full), gen.WeightPipeline(tp)
        x = full.embed_tokens[7]
        worst = 0.0
        for pos in range(3):
            for li in range(arch.num_layers):
                yf = gen.run_decoder_layer_streaming(pf, full, li, x, pos, kf[li], vf[li])
                yt = run_decoder_layer_tp(pt, tp, li, x, pos, kt[li], vt[li])
                worst = max(worst, _rel_l2(yt, yf))
                x = yf
        out["layer_rel_l2"] = worst

        # vocabulary-parallel argmax equals the full argmax on the same xn
        g = torch.Generator(device=dev).manual_seed(11)
        agree = True
        for _ in range(4):
            xn = torch.randn(arch.hidden_size, generator=g, device=dev).half()
            want = int((full.lm_head.float() @ xn.float()).argmax().item())
            got_full = int(gen._next_token(full, xn).item())
            got_tp = int(tp_next_token(tp, xn, plan).item())
            agree &= got_tp == got_full
            out.setdefault("argmax_pairs", []).append((got_tp, got_full, want))
        out["argmax_agree"] = bool(agree)

        prompt = [3, 141, 59, 26]
        eager = generate_tp(tp, plan, prompt, 6, max_seq_len=64)
        gd = graph_decoder_tp(tp, plan, max_seq_len=64)
        graph = gd.generate(prompt, 6)
        graph2 = gd.generate([7, 7], 5)
        eager2 = generate_tp(tp, plan, [7, 7], 5, max_seq_len=64)
        out.update(eager=eager, graph=graph, graph2=graph2, eager2=eager2,
                   full=gen.generate_streaming(full, prompt, 6, max_seq_len=64))
        del gd
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        dist.destroy_process_group()
    results[rank] = out


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tensor_parallel_two_gpus():
    world = 2
    with mp.Manager() as mgr:
        results = mgr.dict()
        mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        res = dict(results)
    for r in range(world):
        o = res[r]
        assert o["shards_exact"], f"rank {r}: shard differs from the full matrix slice"
        assert o["layer_rel_l2"] < 3e-3, f"rank {r}: TP layer rel-L2 {o['layer_rel_l2']}"
        assert o["argmax_agree"], f"rank {r}: {o['argmax_pairs']}"
        assert o["graph"] == o["eager"] and o["graph2"] == o["eager2"], f"rank {r}: graph tokens differ"
    assert res[0]["eager"] == res[1]["eager"] and res[0]["eager2"] == res[1]["eager2"]
    # not asserted equal (fp16 partial rounding), recorded for the failure message of a gross error
    same = sum(a == b for a, b in zip(res[0]["eager"], res[0]["full"]))
    assert same >= len(res[0]["full"]) - 3, (res[0]["eager"], res[0]["full"])
