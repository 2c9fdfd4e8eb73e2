"""Tensor-parallel decode across the GPUs of one node (the 14B-shaped model
on 1/2/4/8 B200s).

Sharding (Megatron-style, one process per GPU):
* column-parallel (output rows split): q_proj / k_proj / v_proj by heads
  (rank r owns query heads [r*NQ/G, (r+1)*NQ/G) and kv heads likewise),
  gate_proj / up_proj by intermediate channels;
* row-parallel (input K split): o_proj by the query-head slice of its input,
  down_proj by the intermediate slice.  K/G is a multiple of the 128 group
  size for every supported G, so a shard's scale columns are whole groups and
  slicing the quantized matrix equals quantizing the slice;
* per layer two all-reduces (sum): after o_proj and after down_proj -- the
  partial products of the row-parallel GEMVs;
* KV cache: each rank keeps its own kv heads;
* LM head: vocabulary rows split; each rank's fused argmax gives (logit,
  index) and the ranks agree on the global argmax (largest fp16 logit, then
  lowest index) from an all-gather.

Each rank's o / down GEMV rounds its partial to fp16; the partials cross the
wire in fp32 and their sum is rounded to fp16 once, so TP differs from the
single-GPU result by those roundings and the summation order (a tolerance,
not bit identity).

The shard plan is host logic (tested on CPU with gloo); the rank model is a
StreamingModel of shard matrices and runs through the same kernels.

Collectives: with a PeerExchange (the default for GPU decode) they are this
library's own kernels over peer memory -- the row-parallel GEMV stores its
fp16 output rows straight into every rank's inbox over NVLink and signals
them, and one exchange kernel sums the ranks' rows, adds the residual and
applies the following RMSNorm; the greedy token is agreed by one exchange
kernel.  Without one, torch.distributed collectives (NCCL, or gloo on CPU)
do the same steps.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class ShardPlan:
    rank: int
    world: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    hidden: int
    intermediate: int
    vocab: int
    group_size: int = 128

    def __post_init__(self):
        G = self.world
        if not 0 <= self.rank < G:
            raise ValueError(f"rank {self.rank} out of range for world size {G}")
        if self.num_heads % G or self.num_kv_heads % G:
            raise ValueError(f"head counts ({self.num_heads}, {self.num_kv_heads}) must divide by world size {G}")
        if self.intermediate % G or (self.intermediate // G) % self.group_size:
            raise ValueError(f"intermediate {self.intermediate} / {G} must be a multiple of {self.group_size}")
        if (self.num_heads // G * self.head_dim) % self.group_size:
            raise ValueError("the o_proj input slice must be whole quantization groups")

    # -- slices (start, stop) of the full dimension owned by this rank
    def _slice(self, total: int) -> tuple[int, int]:
        per = total // self.world
        return self.rank * per, (self.rank + 1) * per

    @property
    def q_rows(self) -> tuple[int, int]:
        a, b = self._slice(self.num_heads)
        return a * self.head_dim, b * self.head_dim

    @property
    def kv_rows(self) -> tuple[int, int]:
        a, b = self._slice(self.num_kv_heads)
        return a * self.head_dim, b * self.head_dim

    @property
    def inter_rows(self) -> tuple[int, int]:
        return self._slice(self.intermediate)

    @property
    def vocab_rows(self) -> tuple[int, int]:
        per = -(-self.vocab // self.world)
        return min(self.rank * per, self.vocab), min((self.rank + 1) * per, self.vocab)

    @property
    def local_heads(self) -> int:
        return self.num_heads // self.world

    @property
    def local_kv_heads(self) -> int:
        return self.num_kv_heads // self.world

    # -- which dimension of each linear weight is split, and the slice
    def weight_slice(self, suffix: str) -> tuple[int, tuple[int, int]]:
        """(axis, (start, stop)) of the full [N, K] weight this rank holds."""
        if suffix.endswith("q_proj.weight"):
            return 0, self.q_rows
        if suffix.endswith(("k_proj.weight", "v_proj.weight")):
            return 0, self.kv_rows
        if suffix.endswith(("gate_proj.weight", "up_proj.weight")):
            return 0, self.inter_rows
        if suffix.endswith("o_proj.weight"):
            return 1, self.q_rows
        if suffix.endswith("down_proj.weight"):
            return 1, self.inter_rows
        if suffix.endswith("down_proj_T.weight"):
            return 0, self.inter_rows
        raise KeyError(suffix)


def shard_packed(packed: torch.Tensor, scale: torch.Tensor, axis: int, sl: tuple[int, int], group_size: int):
    """The rows (axis 0) or K columns (axis 1) [sl) of a quantized matrix
    (packed uint8 [N, K/2], fp32 scales [N, K/g]); K slices are whole groups."""
    a, b = sl
    if axis == 0:
        return packed[a:b].contiguous(), scale[a:b].contiguous()
    if a % group_size or b % group_size:
        raise ValueError(f"K slice {sl} must be whole {group_size}-groups")
    return packed[:, a // 2:b // 2].contiguous(), scale[:, a // group_size:b // group_size].contiguous()


def agree_argmax(local_logit: torch.Tensor, local_idx: torch.Tensor, offset: int, group=None) -> torch.Tensor:
    """Global greedy token from every rank's (fp16 logit, local index): the
    largest logit, ties to the lowest global index.  local_logit: fp16 [1],
    local_idx: int32 [1]; returns int32 [1] on the local device (same value on
    every rank).  One all-gather of an int64 key per rank."""
    import torch.distributed as dist

    key = _order_key(local_logit) * (1 << 32) + (0xFFFFFFFF - (local_idx.long() + offset))
    world = dist.get_world_size(group)
    if key.is_cuda:
        keys = torch.empty(world, dtype=key.dtype, device=key.device)
        dist.all_gather_into_tensor(keys, key, group=group)
    else:
        parts = [torch.empty_like(key) for _ in range(world)]
        dist.all_gather(parts, key, group=group)
        keys = torch.cat(parts)
    best = keys.max()
    return (0xFFFFFFFF - (best & 0xFFFFFFFF)).to(torch.int32).view(1)


def _order_key(h: torch.Tensor) -> torch.Tensor:
    """fp16 -> order-preserving non-negative int64 key (as the fused argmax kernel)."""
    b = h.view(torch.int16).long() & 0xFFFF
    b = torch.where(b == 0x8000, torch.zeros_like(b), b)  # -0 -> +0
    return torch.where(b & 0x8000 != 0, 0xFFFF - b, b | 0x8000)


def build_tp_model(arch, plan: ShardPlan, seed: int = 0, group_size: int = 128, include_dip: bool = False,
                   std: float = 0.02, embed_std: float = 1.0, device=None):
    """This rank's shard of the seeded synthetic model (the same full matrices
    as runtime.loader.synthetic_streaming_model(arch, seed), sliced per the
    plan), weights resident in HBM; embeddings and norms replicated, LM head
    rows split."""
    from ..offload.load_hf_checkpoint import LoadedMatrix
    from ..offload.weight_store import WeightHandle
    from .generate import StreamingModel
    from .loader import synthetic_small_tensors, synthetic_weights

    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    matrices, resident = {}, {}
    weights = synthetic_weights(arch, seed, group_size, include_dip, std, device)
    while True:
        try:
            layer, suffix, packed, scale, packed_k, n, k = next(weights)
        except StopIteration as done:
            gen = done.value
            break
        name = f"model.layers.{layer}.{suffix}"
        axis, sl = plan.weight_slice(suffix)
        pk, sc = shard_packed(packed, scale, axis, sl, group_size)
        del packed, scale
        if axis == 0:
            n_s, k_s, pk_k = sl[1] - sl[0], k, packed_k
        else:
            n_s, k_s, pk_k = n, sl[1] - sl[0], sl[1] - sl[0]
        matrices[name] = LoadedMatrix(WeightHandle(name, -1, pk.shape[0], pk.shape[1]), sc, pk_k, n_s, k_s)
        resident[name] = pk
    norms, embed, lm_head, ones = synthetic_small_tensors(arch, gen, std, embed_std, device)
    lo, hi = plan.vocab_rows
    lm_shard = lm_head[lo:hi].contiguous()
    del lm_head
    return StreamingModel(store=None, matrices=matrices, num_layers=arch.num_layers, embed_tokens=embed,
                          lm_head=lm_shard, final_norm=ones, layer_norms=norms, hidden_size=arch.hidden_size,
                          num_attention_heads=plan.local_heads, num_key_value_heads=plan.local_kv_heads,
                          head_dim=arch.head_dim, rms_norm_eps=arch.rms_norm_eps, rope_theta=arch.rope_theta,
                          group_size=group_size, resident=resident)


class PeerExchange:
    """Peer-memory exchange among the ranks of `group` (one process per GPU,
    every rank on its own device of one node).  Creates this rank's exchange
    buffer, trades CUDA IPC handles with an all_gather_object, and maps every
    peer's buffer; all ranks must then issue the same sequence of exchange
    calls (each call is one or two kernels on the current stream).
    slot_bytes bounds the payload of one rank (fp16 hidden vector, gate
    shard, ...)."""

    def __init__(self, group=None, slot_bytes: int = 64 * 1024, device=None):
        import torch.distributed as dist

        from .. import _C

        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if self.world > _C.MAX_PEERS:
            raise ValueError(f"at most {_C.MAX_PEERS} ranks per exchange")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.slot_bytes = slot_bytes
        self._own, handle = _C.peer_buffer_create(_C.peer_buffer_bytes(slot_bytes, self.world), self.device)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self._mapped = []
        self.peers = _C.PeerSetStruct()
        for r, h in enumerate(handles):
            if r == self.rank:
                self.peers.base[r] = self._own
            else:
                p = _C.peer_buffer_open(h, self.device)
                self._mapped.append(p)
                self.peers.base[r] = p
        self.peers.rank, self.peers.world, self.peers.slot_bytes = self.rank, self.world, slot_bytes
        self._next_normed = None  # (x, rmsnorm(x)) left by the last fused all-reduce for the next layer
        dist.barrier(group=group)

    def reset(self) -> None:
        """Recovery after a peer timeout (device error bit 2): a timed-out
        exchange leaves the ranks out of step, so every rank -- between
        steps, none of its kernels in flight -- zeroes its own buffer header
        behind a barrier, and the exchanges restart from the first.
        Collective: all ranks of the group call it."""
        import torch.distributed as dist

        from .. import _C

        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        _C.peer_buffer_reset(self._own, self.device)
        torch.cuda.synchronize(self.device)
        self._next_normed = None
        dist.barrier(group=self.group)

    def allreduce_add_rmsnorm(self, partial, residual=None, weight=None, eps: float = 1e-6):
        """(out_norm or None, out_sum): out_sum = fp16(residual + sum of the ranks' partials)."""
        from .. import _C

        out_sum = torch.empty_like(partial)
        out_norm = torch.empty_like(partial) if weight is not None else None
        _C.tp_allreduce_add_rmsnorm(self.peers, partial, residual, weight, out_sum, out_norm, eps, self.device)
        return out_norm, out_sum

    def row_parallel(self, W, scale, x, n: int, group_size: int, residual=None, weight=None, eps: float = 1e-6,
                     before=()):
        """Row-parallel INT4 GEMV + all-reduce (+ residual, + RMSNorm): one
        persistent batched launch whose last task (this GEMV) pushes its rows
        to every rank -- `before` are batch tasks (GemvBatch tuples) run ahead
        of it in the same launch, and x may be one of their outputs (the GEMV
        then depends on the task producing it) -- then one exchange kernel
        finishes.  Returns (out_norm or None, out_sum) like
        allreduce_add_rmsnorm."""
        from .. import _C

        before = list(before)
        dep = next((i for i, t in enumerate(before) if t[3] is x), -1)
        _C.gemv_w4a16_batch(before + [(W, scale, x, None, x.numel(), group_size, dep)], self.peers)
        return self.finish(n, residual, weight, eps)

    def finish(self, n: int, residual=None, weight=None, eps: float = 1e-6):
        """The exchange after a launch that pushed the partial rows (row_parallel)."""
        from .. import _C

        out_sum = torch.empty(n, dtype=torch.float16, device=self.device)
        out_norm = torch.empty_like(out_sum) if weight is not None else None
        _C.tp_allreduce_add_rmsnorm(self.peers, None, residual, weight, out_sum, out_norm, eps, self.device)
        return out_norm, out_sum

    def allgather(self, local: torch.Tensor) -> torch.Tensor:
        from .. import _C

        out = torch.empty((self.world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
        _C.tp_allgather(self.peers, local.contiguous(), out)
        return out

    def argmax(self, logits: torch.Tensor, local_idx: torch.Tensor, offset: int) -> torch.Tensor:
        from .. import _C

        out = torch.empty(1, dtype=torch.int32, device=logits.device)
        _C.tp_argmax(self.peers, logits, local_idx, offset, out)
        return out

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (collective: every rank calls it)."""
        import torch.distributed as dist

        from .. import _C

        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._mapped:
            _C.peer_buffer_close(p, self.device)
        self._mapped = []
        dist.barrier(group=self.group)
        _C.peer_buffer_destroy(self._own, self.device)
        self._own = None


def all_reduce_sum(partial: torch.Tensor, group=None) -> torch.Tensor:
    """Sum of the ranks' fp16 partial vectors, accumulated in fp32, rounded once."""
    import torch.distributed as dist

    f = partial.float()
    dist.all_reduce(f, group=group)
    return f.half()


def run_decoder_layer_tp(pipeline, model, layer_idx, x_flat, pos, k_cache, v_cache, group=None, exchange=None):
    """Dense decoder layer on this rank's shard: local q / k / v heads and
    attention, row-parallel o_proj partial + all-reduce, residual + rmsnorm,
    local gate / up (SwiGLU), row-parallel down partial + all-reduce, residual.
    With a PeerExchange each row-parallel GEMV and its all-reduce, residual
    and following RMSNorm (post-attention, or the next layer's input norm)
    are two kernels -- the MLP's gate / up / down one launch plus the
    exchange -- and the next layer picks up its normed input."""
    from .generate import _attention_block

    if exchange is None:
        h2, h3 = _attention_block(pipeline, model, layer_idx, x_flat, pos, k_cache, v_cache,
                                  reduce_o=lambda o: all_reduce_sum(o, group))
        down = pipeline.next_gemv(pipeline.next_glu(h3))
        return h2 + all_reduce_sum(down, group)

    g = model.group_size

    def o_block(attn, x, post_w, eps):
        W, m = pipeline.next_resident()
        h3, h2 = exchange.row_parallel(W, m.scale, attn, model.hidden_size, g, residual=x, weight=post_w, eps=eps)
        return h2, h3

    prev = exchange._next_normed
    h_in = prev[1] if prev is not None and prev[0] is x_flat else None
    h2, h3 = _attention_block(pipeline, model, layer_idx, x_flat, pos, k_cache, v_cache, h_in=h_in, o_block=o_block)
    # MLP: gate, up (SwiGLU epilogue) and the row-parallel down in one launch, then the exchange
    (Wg, mg), (Wu, mu), (Wd, md) = (pipeline.next_resident() for _ in range(3))
    gate = torch.empty(mg.n, dtype=torch.float16, device=h3.device)
    hidden = torch.empty(mu.n, dtype=torch.float16, device=h3.device)
    nxt = layer_idx + 1
    w_next = model.layer_norms[nxt]["input_layernorm"] if nxt < model.num_layers else None
    h_next, out = exchange.row_parallel(Wd, md.scale, hidden, model.hidden_size, g, residual=h2, weight=w_next,
                                        eps=model.rms_norm_eps,
                                        before=[(Wg, mg.scale, h3, gate, mg.packed_k, g, -1),
                                                (Wu, mu.scale, h3, hidden, mu.packed_k, g, -1, None, gate)])
    exchange._next_normed = (out, h_next) if h_next is not None else None
    return out


def run_decoder_layer_dip_tp(pipeline, model, layer_idx, x_flat, pos, k_cache, v_cache, dip_k: int, plan: ShardPlan,
                             exchange: PeerExchange, trace: dict | None = None):
    """DIP layer under tensor parallelism, reference selection semantics: the
    rank's gate shard (column-parallel rows) is all-gathered, every rank runs
    the same deterministic top-dip_k |gate| selector over all I channels, and
    each rank computes only the selected channels inside its own up / down_T
    shard (rows [lo, hi)); the down partials go through the exchange
    (all-reduce + residual + next RMSNorm).  One host read per layer (the
    number of selected channels this rank owns sizes the row kernels).
    The pipeline is the DIP one (q / k / v / o / gate).  trace (optional)
    receives h3, the gathered gate and the global selection."""
    from .. import ops
    from ..offload.load_hf_checkpoint import DOWN_PROJ_T_SUFFIX
    from .generate import _attention_block

    g = model.group_size

    def o_block(attn, x, post_w, eps):
        W, m = pipeline.next_resident()
        h3, h2 = exchange.row_parallel(W, m.scale, attn, model.hidden_size, g, residual=x, weight=post_w, eps=eps)
        return h2, h3

    prev = exchange._next_normed
    h_in = prev[1] if prev is not None and prev[0] is x_flat else None
    h2, h3 = _attention_block(pipeline, model, layer_idx, x_flat, pos, k_cache, v_cache, h_in=h_in, o_block=o_block)
    gate_loc = pipeline.next_gemv(h3)
    gate = exchange.allgather(gate_loc).view(-1)
    idx = ops.topk_threshold_select_abs(gate, dip_k)          # global channels, ascending
    lo, hi = plan.inter_rows
    bounds = torch.searchsorted(idx, torch.tensor([lo, hi], dtype=torch.int32, device=idx.device))
    a, b = (int(v) for v in bounds.tolist())                   # this rank's share of the selection
    if trace is not None:
        trace.update(h2=h2, h3=h3, gate=gate, idx=idx)
    if b > a:
        loc = (idx[a:b] - lo).contiguous()
        up = model.matrix(layer_idx, "mlp.up_proj.weight")
        down_t = model.matrix(layer_idx, DOWN_PROJ_T_SUFFIX)
        h_sel = ops.gemv_w4a16_rows(model.resident[up.handle.name], up.scale, loc, h3, up.packed_k, g,
                                    glu_gate=gate_loc)
        part = ops.gemv_w4a16_sparse_rows(model.resident[down_t.handle.name], down_t.scale, loc, h_sel,
                                          model.hidden_size, g)
    else:
        part = torch.zeros(model.hidden_size, dtype=torch.float16, device=h3.device)
    nxt = layer_idx + 1
    w_next = model.layer_norms[nxt]["input_layernorm"] if nxt < model.num_layers else None
    h_next, out = exchange.allreduce_add_rmsnorm(part, residual=h2, weight=w_next, eps=model.rms_norm_eps)
    exchange._next_normed = (out, h_next) if h_next is not None else None
    return out


def generate_dip_tp(model, plan: ShardPlan, prompt_ids: list[int], n_new: int, dip_k: int, exchange: PeerExchange,
                    max_seq_len: int = 512):
    """Eager greedy decode of the TP model with DIP MLPs (every rank returns the same ids)."""
    from .generate import DIP_DENSE_SUFFIXES, WeightPipeline, _greedy

    pipeline = WeightPipeline(model, suffixes=DIP_DENSE_SUFFIXES)
    return _greedy(model, prompt_ids, n_new,
                   lambda li, x, p, kc, vc: run_decoder_layer_dip_tp(pipeline, model, li, x, p, kc, vc, dip_k, plan,
                                                                     exchange),
                   None, max_seq_len, token_fn=lambda m, xn: tp_next_token(m, xn, plan, None, exchange))


def tp_next_token(model, xn: torch.Tensor, plan: ShardPlan, group=None, exchange=None) -> torch.Tensor:
    """Greedy token over the vocabulary-parallel LM head: each rank's fused
    argmax of its rows, then the ranks agree (exchange kernel, or
    agree_argmax's all-gather)."""
    from .. import _C

    idx, logits = _C.gemv_fp16_argmax(model.lm_head, xn, logits=True)
    if exchange is not None:
        return exchange.argmax(logits, idx, plan.vocab_rows[0])
    return agree_argmax(logits.index_select(0, idx.long()), idx, plan.vocab_rows[0], group)


def generate_tp(model, plan: ShardPlan, prompt_ids: list[int], n_new: int, group=None, max_seq_len: int = 512,
                exchange=None):
    """Eager greedy decode of the TP model (every rank returns the same ids)."""
    from .generate import WeightPipeline, _greedy

    pipeline = WeightPipeline(model)
    return _greedy(model, prompt_ids, n_new,
                   lambda li, x, p, kc, vc: run_decoder_layer_tp(pipeline, model, li, x, p, kc, vc, group, exchange),
                   None, max_seq_len, token_fn=lambda m, xn: tp_next_token(m, xn, plan, group, exchange))


def graph_decoder_tp(model, plan: ShardPlan, group=None, max_seq_len: int = 2048, exchange=None):
    """GraphDecoder whose captured step is the TP layer stack (the exchange
    kernels, or NCCL collectives, inside the graph)."""
    from .generate import GraphDecoder

    return GraphDecoder(model, max_seq_len=max_seq_len,
                        layer_fn=lambda p, m, li, x, w, kc, vc: run_decoder_layer_tp(p, m, li, x, w, kc, vc, group,
                                                                                     exchange),
                        token_fn=lambda m, xn: tp_next_token(m, xn, plan, group, exchange))


__all__ = ["ShardPlan", "shard_packed", "agree_argmax", "build_tp_model", "PeerExchange", "all_reduce_sum",
           "run_decoder_layer_tp", "run_decoder_layer_dip_tp", "generate_dip_tp", "tp_next_token", "generate_tp",
           "graph_decoder_tp"]


ALLREDUCE_SWEEP_BYTES = (10 * 1024, 20 * 1024, 40 * 1024, 80 * 1024, 1 << 20, 16 << 20, 1 << 30)


def allreduce_sweep(device, group=None, sizes=ALLREDUCE_SWEEP_BYTES, iters: int = 20, warmup: int = 5,
                    exchange: "PeerExchange | None" = None) -> list[dict]:
    """Latency / bandwidth of a sum all-reduce of fp16 buffers of each size
    in bytes over `group` (torch.distributed; NCCL on GPUs), max over ranks.
    Per size: mean microseconds per all-reduce and the bus bandwidth
    (bytes x 2 (world - 1) / world / time, the usual ring-normalised figure).
    With `exchange`, sizes that fit its slot also time the peer exchange
    (soinfer_tp_allreduce_add_rmsnorm: push to every rank's inbox over NVLink,
    flag, sum in rank order) on the same buffer.  Collective: every rank of
    the group calls it with the same arguments."""
    import time

    import torch.distributed as dist

    world = dist.get_world_size(group)
    dev = torch.device(device)
    cuda = dev.type == "cuda"
    out = []

    def timed(fn, n):
        if cuda:
            torch.cuda.synchronize(dev)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(n):
                fn()
            e.record()
            torch.cuda.synchronize(dev)
            ms = s.elapsed_time(e)
        else:
            t0 = time.perf_counter()
            for _ in range(n):
                fn()
            ms = (time.perf_counter() - t0) * 1e3
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        return float(t.item()) * 1e3 / n  # microseconds per call

    for nbytes in sizes:
        n = nbytes // 2
        buf = torch.ones(n, dtype=torch.float16, device=dev)
        reps = iters if nbytes < (64 << 20) else max(3, iters // 5)
        for _ in range(warmup):
            dist.all_reduce(buf, group=group)
        us = timed(lambda: dist.all_reduce(buf, group=group), reps)
        row = {"bytes": nbytes, "world": world, "nccl_us": round(us, 2),
               "nccl_busbw_gbs": round(nbytes * 2 * (world - 1) / world / (us * 1e-6) / 1e9, 3)}
        if exchange is not None and n % 8 == 0 and nbytes <= exchange.slot_bytes:
            part = torch.randn(n, device=dev).half()
            for _ in range(warmup):
                exchange.allreduce_add_rmsnorm(part)
            row["exchange_us"] = round(timed(lambda: exchange.allreduce_add_rmsnorm(part), iters), 2)
        out.append(row)
        del buf
    return out
