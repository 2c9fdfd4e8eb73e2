"""Tensor-parallel decode on 2 / 4 / 8 GPUs (one process per GPU), each rank
also holding the unsharded model on its own device:

* a rank's shard matrices are exactly the slices of the full quantized
  matrices (same seed -> same weights);
* decoder layers with the row-parallel all-reduces match the single-GPU
  layers within a tolerance (each shard rounds its partial to fp16, so not
  bit for bit);
* the vocabulary-parallel LM head picks exactly the single-GPU argmax for
  the same normed hidden state;
* eager TP decode gives the same tokens on every rank, and the CUDA-graph TP
  decoder (NCCL collectives inside the graph) gives the eager tokens;
* the peer-memory exchange kernels: all-gather is the exact concatenation,
  the all-reduce + residual equals the NCCL fp32 all-reduce bit for bit (two
  ranks: a + b is order-free) with its RMSNorm within an fp16 ulp of the
  unfused kernel, the greedy-token agreement breaks ties to the lowest global
  index, the fused row-parallel GEMV + all-reduce equals the same GEMV + NCCL, and
  decode through the exchange (eager and graph) matches the NCCL decode;
* DIP under TP: the all-gathered gate matches the unsharded gate GEMV, the
  global selection on it equals the oracle's reference selector bit for bit
  on every rank, and the layer output matches the oracle's DIP block
  evaluated on the same gate; DIP decode gives the same tokens on every rank.

Each world size is skipped when fewer GPUs are visible."""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

# shardable 2 / 4 / 8 ways: 16 q / 8 kv heads of 64, intermediate 1024 (128 channels per rank at 8)
ARCH_ARGS = dict(num_layers=2, hidden_size=512, intermediate_size=1024, num_attention_heads=16, num_key_value_heads=8,
                 head_dim=64, vocab_size=512)


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
    from soinfer import _C, ops
    from oracle import reference_port as port
    from soinfer.runtime.tp import (PeerExchange, ShardPlan, all_reduce_sum, build_tp_model, generate_dip_tp,
                                    generate_tp, graph_decoder_tp, run_decoder_layer_dip_tp, run_decoder_layer_tp,
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
        full = synthetic_streaming_model(arch, seed=3, resident=True, offload=False, include_dip=True, device=dev)
        tp = build_tp_model(arch, plan, seed=3, include_dip=True, device=dev)

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

        # ---- peer-memory exchange kernels
        ex = PeerExchange(device=dev)
        g2 = torch.Generator(device=dev).manual_seed(100 + rank)
        loc = torch.randn(1000, generator=g2, device=dev).half()[:992]
        gathered = ex.allgather(loc)
        parts = [torch.empty_like(loc) for _ in range(world)]
        dist.all_gather(parts, loc)
        out["allgather_exact"] = bool(torch.equal(gathered, torch.stack(parts)))
        H = arch.hidden_size
        partial = torch.randn(H, generator=g2, device=dev).half()
        torch.manual_seed(0)  # identical residual / weight on every rank
        resid = torch.randn(H, device=dev).half()
        w = (torch.rand(H, device=dev) + 0.5).half()
        h3x, h2x = ex.allreduce_add_rmsnorm(partial, resid, w, 1e-6)
        o = all_reduce_sum(partial)
        h3r, h2r = ops.add_rmsnorm(resid.unsqueeze(0), o.unsqueeze(0), w, 1e-6)
        out["ar_sum_exact"] = bool(torch.equal(h2x, h2r.squeeze(0)))
        out["ar_norm_maxdiff"] = float((h3x.float() - h3r.squeeze(0).float()).abs().max())
        # argmax agreement: every rank holds the same max logit -> lowest global index wins;
        # then the last rank's larger logit wins
        lg = torch.zeros(16, dtype=torch.float16, device=dev)
        lg[5] = 3.5
        li = torch.tensor([5], dtype=torch.int32, device=dev)
        out["argmax_tie"] = int(ex.argmax(lg, li, rank * 16).item())
        lg[5] = 1.0 + rank
        out["argmax_win"] = int(ex.argmax(lg, li, rank * 16).item())
        # fused row-parallel GEMV (o_proj shard) + all-reduce vs GEMV + NCCL
        name = "model.layers.0.self_attn.o_proj.weight"
        m = tp.matrices[name]
        xa = torch.randn(m.k, generator=g2, device=dev).half()
        h3f, h2f = ex.row_parallel(tp.resident[name], m.scale, xa, H, 128, residual=resid, weight=w)
        part = torch.empty(H, dtype=torch.float16, device=dev)  # the same batched kernel, output to y
        _C.gemv_w4a16_batch([(tp.resident[name], m.scale, xa, part, m.packed_k, 128, -1)])
        h3n, h2n = ops.add_rmsnorm(resid.unsqueeze(0), all_reduce_sum(part).unsqueeze(0), w, 1e-6)
        out["fused_sum_exact"] = bool(torch.equal(h2f, h2n.squeeze(0)))
        out["fused_norm_maxdiff"] = float((h3f.float() - h3n.squeeze(0).float()).abs().max())
        # decode through the exchange
        kx, vx = gen._kv_caches(tp, 16)
        kn, vn = gen._kv_caches(tp, 16)
        px, pn = gen.WeightPipeline(tp), gen.WeightPipeline(tp)
        x = tp.embed_tokens[7]
        xe = xn_ = x
        worst = 0.0
        for pos in range(3):
            for li_ in range(arch.num_layers):
                xe = run_decoder_layer_tp(px, tp, li_, xe, pos, kx[li_], vx[li_], exchange=ex)
                xn_ = run_decoder_layer_tp(pn, tp, li_, xn_, pos, kn[li_], vn[li_])
                worst = max(worst, _rel_l2(xe, xn_))
        out["exchange_layer_rel_l2"] = worst
        out["ex_eager"] = generate_tp(tp, plan, prompt, 6, max_seq_len=64, exchange=ex)
        gdx = graph_decoder_tp(tp, plan, max_seq_len=64, exchange=ex)
        out["ex_graph"] = gdx.generate(prompt, 6)
        out["ex_graph2"] = gdx.generate([7, 7], 5)
        out["ex_eager2"] = generate_tp(tp, plan, [7, 7], 5, max_seq_len=64, exchange=ex)
        del gdx

        # ---- DIP under TP
        dip_k = arch.intermediate_size // 2
        pdp = gen.WeightPipeline(tp, gen.DIP_DENSE_SUFFIXES)
        kd, vd = gen._kv_caches(tp, 16)
        tr = {}
        y = run_decoder_layer_dip_tp(pdp, tp, 0, tp.embed_tokens[11], 0, kd[0], vd[0], dip_k, plan, ex, trace=tr)
        npf = lambda name: (full.resident[f"model.layers.0.{name}"].cpu().numpy(),
                            full.matrices[f"model.layers.0.{name}"].scale.cpu().numpy())
        h3n = tr["h3"].cpu().numpy()
        blk = port.dip_mlp_block(h3n, npf("mlp.gate_proj.weight"), npf("mlp.up_proj.weight"),
                                 npf(gen.DOWN_PROJ_T_SUFFIX), dip_k, 128, H, gate_out=tr["gate"].cpu().numpy())
        import numpy as np
        ref = (tr["h2"].cpu().numpy().astype(np.float32) + blk["y"].astype(np.float16).astype(np.float32))
        out["dip_rel_l2"] = _rel_l2(y, torch.from_numpy(ref.astype(np.float16)).to(dev))
        out["dip_idx_exact"] = bool(np.array_equal(tr["idx"].cpu().numpy(), blk["idx"]))
        gm = full.matrices["model.layers.0.mlp.gate_proj.weight"]
        gate_full = ops.gemv_w4a16_group_lop3(full.resident[gm.handle.name], gm.scale, tr["h3"], gm.packed_k, 128)
        out["dip_gate_rel_l2"] = _rel_l2(tr["gate"], gate_full)
        out["dip_tokens"] = generate_dip_tp(tp, plan, prompt, 5, dip_k, ex, max_seq_len=64)
        torch.cuda.synchronize()
        out["device_errors"] = _C.device_errors()
        ex.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()
    results[rank] = out


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
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
    assert all(res[r]["eager"] == res[0]["eager"] and res[r]["eager2"] == res[0]["eager2"] for r in range(world))
    for r in range(world):
        o = res[r]
        assert o["device_errors"] == 0, f"rank {r}: device error bits {o['device_errors']}"
        assert o["allgather_exact"] and o["ar_sum_exact"] and o["fused_sum_exact"], o
        assert o["ar_norm_maxdiff"] < 4e-3 and o["fused_norm_maxdiff"] < 4e-3, o
        assert o["argmax_tie"] == 5 and o["argmax_win"] == 16 * (world - 1) + 5, o
        assert o["exchange_layer_rel_l2"] < 2e-3, o["exchange_layer_rel_l2"]
        assert o["ex_graph"] == o["ex_eager"] and o["ex_graph2"] == o["ex_eager2"], o
    assert all(res[r]["ex_eager"] == res[0]["ex_eager"] for r in range(world))
    for r in range(world):
        o = res[r]
        assert o["dip_idx_exact"], f"rank {r}: DIP selection differs from the reference selector"
        assert o["dip_gate_rel_l2"] < 1e-3 and o["dip_rel_l2"] < 2e-3, o
    assert all(res[r]["dip_tokens"] == res[0]["dip_tokens"] for r in range(world))
    # not asserted equal (fp16 partial rounding), recorded for the failure message of a gross error
    same = sum(a == b for a, b in zip(res[0]["eager"], res[0]["full"]))
    assert same >= len(res[0]["full"]) - 3, (res[0]["eager"], res[0]["full"])


def _read_i32(ptr: int, offset: int) -> int:
    """One int32 of device memory at a raw address (test-only, through the CUDA runtime)."""
    import ctypes

    cudart = ctypes.CDLL("libcudart.so.12")
    out = ctypes.c_int32()
    assert cudart.cudaMemcpy(ctypes.byref(out), ctypes.c_void_p(ptr + offset), ctypes.c_size_t(4), 2) == 0
    return out.value


def test_exchange_wait_times_out_and_reports():
    """Failure detection without a fault: a two-rank exchange whose second
    rank never signals (its buffer is a second local allocation nobody
    drives) gives up after its bounded wait (1 s), raises the peer-timeout
    device error bit and returns -- the context stays usable."""
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from soinfer import _C

    dev = torch.device("cuda", 0)
    slot = 64 * 1024
    nbytes = _C.peer_buffer_bytes(slot, 2)
    own, _ = _C.peer_buffer_create(nbytes, dev)
    other, _ = _C.peer_buffer_create(nbytes, dev)
    try:
        peers = _C.PeerSetStruct()
        peers.base[0], peers.base[1] = own, other
        peers.rank, peers.world, peers.slot_bytes = 0, 2, slot
        _C.device_errors()  # clear
        x = torch.randn(512, device=dev).half()
        out = torch.empty_like(x)
        _C.tp_allreduce_add_rmsnorm(peers, x, None, None, out, None, 1e-6, dev)
        torch.cuda.synchronize(dev)
        assert _C.device_errors() & 2, "the timed-out wait did not report kErrPeerTimeout"
        y = torch.ones(4, device=dev) * 2  # the context is still usable
        assert float(y.sum().item()) == 8.0
        assert _read_i32(own, 64) == 0, "a timed-out exchange must not advance the exchange count"
        # recovery: reset the header, then the buffer serves exchanges again (here a one-rank set)
        _C.peer_buffer_reset(own, dev)
        solo = _C.PeerSetStruct()
        solo.base[0] = own
        solo.rank, solo.world, solo.slot_bytes = 0, 1, slot
        _C.tp_allreduce_add_rmsnorm(solo, x, None, None, out, None, 1e-6, dev)
        torch.cuda.synchronize(dev)
        assert _C.device_errors() == 0
        assert torch.equal(out, x) and _read_i32(own, 64) == 1
    finally:
        torch.cuda.synchronize(dev)
        _C.peer_buffer_destroy(own, dev)
        _C.peer_buffer_destroy(other, dev)


def test_exchange_single_rank_equals_local_ops():
    """The exchange kernels on a one-rank peer set (one GPU, no peers): the
    all-reduce + residual + RMSNorm equals add_rmsnorm (a sum over one rank is
    the partial itself), the all-gather is the identity, the argmax returns
    the local index plus the offset, and the batched peer task + finish equals
    the GEMV with the residual epilogue followed by rmsnorm."""
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from soinfer import _C, ops
    from tests.helpers import int4_weights

    dev = torch.device("cuda", 0)
    slot = 64 * 1024
    own, _ = _C.peer_buffer_create(_C.peer_buffer_bytes(slot, 1), dev)
    try:
        peers = _C.PeerSetStruct()
        peers.base[0] = own
        peers.rank, peers.world, peers.slot_bytes = 0, 1, slot
        g = torch.Generator(device=dev).manual_seed(3)
        H = 5120
        part = torch.randn(H, generator=g, device=dev).half()
        res = torch.randn(H, generator=g, device=dev).half()
        w = (torch.rand(H, generator=g, device=dev) + 0.5).half()
        out_sum, out_norm = torch.empty_like(part), torch.empty_like(part)
        _C.tp_allreduce_add_rmsnorm(peers, part, res, w, out_sum, out_norm, 1e-6, dev)
        n3, n2 = ops.add_rmsnorm(res.unsqueeze(0), part.unsqueeze(0), w, 1e-6)
        assert torch.equal(out_sum, n2.squeeze(0))
        ref_norm = n3.squeeze(0).float()
        assert bool(((out_norm.float() - ref_norm).abs() <= 1e-3 + 2e-3 * ref_norm.abs()).all())
        loc = torch.randn(2048, generator=g, device=dev).half()
        gathered = torch.empty_like(loc)
        _C.tp_allgather(peers, loc, gathered)
        assert torch.equal(gathered, loc)
        logits = torch.randn(100, generator=g, device=dev).half()
        idx = torch.tensor([17], dtype=torch.int32, device=dev)
        out_idx = torch.empty(1, dtype=torch.int32, device=dev)
        _C.tp_argmax(peers, logits, idx, 1000, out_idx)
        assert int(out_idx.item()) == 1017
        p, s, pk = int4_weights(H, 2560, 128, seed=5)
        P, S = p.to(dev), s.to(dev)
        x = torch.randn(pk, generator=g, device=dev).half()
        _C.gemv_w4a16_batch([(P, S, x, None, pk, 128, -1)], peers)
        fin_sum, fin_norm = torch.empty_like(res), torch.empty_like(res)
        _C.tp_allreduce_add_rmsnorm(peers, None, res, w, fin_sum, fin_norm, 1e-6, dev)
        ref = torch.empty(H, dtype=torch.float16, device=dev)
        _C.gemv_w4a16_batch([(P, S, x, ref, pk, 128, -1, res)])
        torch.cuda.synchronize(dev)
        assert torch.equal(fin_sum, ref)
        assert _C.device_errors() == 0
    finally:
        torch.cuda.synchronize(dev)
        _C.peer_buffer_destroy(own, dev)
