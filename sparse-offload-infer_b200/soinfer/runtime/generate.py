"""Batch-1 greedy decode over the soinfer ops (reference
python/soinfer/runtime/generate.py:58-645): dense streaming, DIP (dynamic
input pruning of the MLP) and cache-aware DIP decoder layers, the generate
loops, teacher-forced NLL and channel-frequency calibration.

Weights live either in the pinned host arena, streamed to the GPU by
`WeightPipeline` one matrix ahead of compute (the reference's offload mode),
or resident in HBM (`StreamingModel.resident`, the natural B200 mode: 180 GB
holds every config here); the layer functions are the same for both.

Where the reference syncs with the host, this path stays on the device:
DIP's selected up_proj / down_proj_T rows are read in place by row-indexed
kernels (resident) or gathered by a device-driven zero-copy gather straight
from the pinned arena (offload), so the selected indices never leave the
GPU; the next token is chosen by the LM-head GEMV's fused argmax and its
embedding row is selected on the device.  Cache-aware DIP keeps the
reference's one sync per layer (the miss count sizes the staging rows).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from .. import _C, ops
from ..offload.hot_cache import HotCache
from ..offload.load_hf_checkpoint import DOWN_PROJ_T_SUFFIX, LINEAR_SUFFIXES, LoadedMatrix
from ..offload.stream_manager import StreamManager
from ..offload.weight_store import PinnedWeightStore

# q/k/v/o/gate stay dense in DIP (selection needs every |gate| value); up_proj
# and down_proj_T are read per token as the selected rows only
# (reference generate.py:49-55).
DIP_DENSE_SUFFIXES = (
    "self_attn.q_proj.weight",
    "self_attn.k_proj.weight",
    "self_attn.v_proj.weight",
    "self_attn.o_proj.weight",
    "mlp.gate_proj.weight",
)


@dataclass
class StreamingModel:
    """The arena and its per-matrix handles, the small resident tensors
    (embeddings, LM head, norms), and the streaming machinery.  `resident`
    (name -> packed uint8 CUDA tensor) switches a matrix from streamed to
    HBM-resident."""

    store: PinnedWeightStore | None
    matrices: dict[str, LoadedMatrix]
    num_layers: int
    embed_tokens: torch.Tensor | None   # [vocab, H] half, CUDA
    lm_head: torch.Tensor | None        # [vocab, H] half, CUDA
    final_norm: torch.Tensor | None     # [H] half, CUDA
    layer_norms: list[dict[str, torch.Tensor]]
    hidden_size: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rms_norm_eps: float
    rope_theta: float
    group_size: int = 128
    resident: dict[str, torch.Tensor] | None = None
    batch_gemvs: bool = True  # resident GEMVs sharing an input run as one batched launch
    stream_manager: StreamManager = field(init=False)

    def __post_init__(self) -> None:
        self.stream_manager = StreamManager(num_buffers=2, device=self.device)

    @property
    def device(self) -> torch.device:
        for m in self.matrices.values():
            return m.scale.device
        return torch.device("cuda", torch.cuda.current_device())

    def is_resident(self, name: str) -> bool:
        return self.resident is not None and name in self.resident

    def weight_source(self, m: LoadedMatrix) -> torch.Tensor:
        """The packed rows of m: the resident CUDA tensor, else its arena view (pinned host)."""
        if self.is_resident(m.handle.name):
            return self.resident[m.handle.name]
        return self.store.matrix_view(m.handle)

    def matrix(self, layer_idx: int, suffix: str) -> LoadedMatrix:
        return self.matrices[f"model.layers.{layer_idx}.{suffix}"]


class WeightPipeline:
    """Cyclic per-token weight sequence (reference generate.py:85-138).
    Streamed matrices: two device buffers, the copy of weight i+1 issued on a
    side stream while weight i's GEMV runs (events, write-after-read guard).
    Resident matrices are used in place."""

    def __init__(self, model: StreamingModel, suffixes: tuple[str, ...] = LINEAR_SUFFIXES):
        self.model = model
        self.sm = model.stream_manager
        seq = [f"model.layers.{i}.{s}" for i in range(model.num_layers) for s in suffixes]
        streamed = [n for n in seq if not model.is_resident(n)]
        self.bufs = []
        if streamed:
            max_bytes = max(model.matrices[n].n * model.matrices[n].handle.row_nbytes for n in streamed)
            self.bufs = [torch.empty(max_bytes, dtype=torch.uint8, device=model.device) for _ in range(2)]
        self._seq = seq
        self._i = 0  # index of the weight in flight
        self.cur_buf = 0
        self.cur_name = seq[0]
        self._prefetch_into(self.cur_buf, self.cur_name)

    def _advance(self) -> str:
        self._i = (self._i + 1) % len(self._seq)
        return self._seq[self._i]

    def _view(self, buf_idx: int, m: LoadedMatrix) -> torch.Tensor:
        nbytes = m.n * m.handle.row_nbytes
        return self.bufs[buf_idx][:nbytes].view(m.n, m.handle.row_nbytes)

    def _prefetch_into(self, buf_idx: int, name: str) -> None:
        if self.model.is_resident(name):
            return
        m = self.model.matrices[name]
        self.sm.prefetch(buf_idx, self._view(buf_idx, m), self.model.store.matrix_view(m.handle))

    def next_gemv(self, x_in: torch.Tensor) -> torch.Tensor:
        """GEMV of the weight in flight (its copy awaited on the GPU), then the next prefetch."""
        name = self.cur_name
        m = self.model.matrices[name]
        if self.model.is_resident(name):
            y = self._gemv(self.model.resident[name], m, x_in)
        else:
            self.sm.wait(self.cur_buf)
            y = self._gemv(self._view(self.cur_buf, m), m, x_in)
            self.sm.mark_read_done(self.cur_buf)
        nxt = 1 - self.cur_buf
        name_next = self._advance()
        self._prefetch_into(nxt, name_next)
        self.cur_buf, self.cur_name = nxt, name_next
        return y

    def next_resident(self) -> tuple[torch.Tensor, LoadedMatrix]:
        """The HBM-resident weight in flight and its matrix record, consumed
        (the caller runs its own kernel on it)."""
        name = self.cur_name
        if not self.model.is_resident(name):
            raise ValueError(f"{name} is not resident in HBM")
        self.cur_buf, self.cur_name = 1 - self.cur_buf, self._advance()
        self._prefetch_into(self.cur_buf, self.cur_name)
        return self.model.resident[name], self.model.matrices[name]

    def _gemv(self, rows: torch.Tensor, m: LoadedMatrix, x_in: torch.Tensor) -> torch.Tensor:
        if m.bits == 8:  # INT8 rows, per-channel scales (the reference's gemv_w8a16)
            return ops.gemv_w8a16(rows.view(torch.int8), m.scale, x_in, m.k)
        return ops.gemv_w4a16_group_lop3(rows, m.scale, x_in, m.packed_k, self.model.group_size)

    def _batched(self, count: int) -> list[str] | None:
        """The next `count` names when they can run as one persistent batched
        INT4 launch (resident, INT4), else None."""
        names = [self._seq[(self._i + j) % len(self._seq)] for j in range(count)]
        ok = self.model.batch_gemvs and all(self.model.is_resident(n) and self.model.matrices[n].bits == 4
                                            for n in names)
        return names if ok else None

    def next_gemvs(self, x_in: torch.Tensor, count: int, norm: tuple | None = None) -> list[torch.Tensor]:
        """The next `count` GEMVs, all on the same input.  When they are all
        HBM-resident they run as one persistent batched launch (one kernel for
        q / k / v or gate / up); otherwise one after another.  norm =
        (weight, eps): the GEMVs take rmsnorm(x_in) * weight -- computed inside
        the batched kernel, or by the rmsnorm op before the unbatched GEMVs."""
        names = self._batched(count)
        if names is not None:
            tasks = []
            for name in names:
                m = self.model.matrices[name]
                y = torch.empty(m.n, dtype=torch.float16, device=x_in.device)
                tasks.append((self.model.resident[name], m.scale, x_in, y, m.packed_k, self.model.group_size, -1,
                              None, None, norm))
            for _ in range(count):
                self.cur_buf, self.cur_name = 1 - self.cur_buf, self._advance()
            _C.gemv_w4a16_batch(tasks)
            return [t[3] for t in tasks]
        if norm is not None:
            h = ops.rmsnorm(x_in.unsqueeze(0), norm[0], norm[1]).squeeze(0)
            if len(norm) > 2 and norm[2] is not None:
                norm[2].copy_(h)
            x_in = h
        return [self.next_gemv(x_in) for _ in range(count)]

    def next_gemv_residual(self, x_in: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
        """residual + (next weight) x_in: one batched launch with the residual
        epilogue when resident, else the GEMV and an add."""
        names = self._batched(1)
        if names is not None:
            m = self.model.matrices[names[0]]
            y = torch.empty(m.n, dtype=torch.float16, device=x_in.device)
            self.cur_buf, self.cur_name = 1 - self.cur_buf, self._advance()
            _C.gemv_w4a16_batch([(self.model.resident[names[0]], m.scale, x_in, y, m.packed_k, self.model.group_size,
                                  -1, residual)])
            return y
        return residual + self.next_gemv(x_in)

    def next_glu(self, h3: torch.Tensor) -> torch.Tensor:
        """The next gate / up weights as fp16(silu(gate(h3)) * up(h3)): one batched
        launch with the SwiGLU epilogue when resident, else two GEMVs and swiglu."""
        names = self._batched(2)
        if names is not None:
            mg, mu = (self.model.matrices[n] for n in names)
            res, g = self.model.resident, self.model.group_size
            gate = torch.empty(mg.n, dtype=torch.float16, device=h3.device)
            hidden = torch.empty(mu.n, dtype=torch.float16, device=h3.device)
            for _ in range(2):
                self.cur_buf, self.cur_name = 1 - self.cur_buf, self._advance()
            _C.gemv_w4a16_batch([(res[names[0]], mg.scale, h3, gate, mg.packed_k, g, -1),
                                 (res[names[1]], mu.scale, h3, hidden, mu.packed_k, g, -1, None, gate)])
            return hidden
        gate, up = self.next_gemvs(h3, 2)
        return ops.swiglu(gate, up)

    def next_mlp(self, h3: torch.Tensor | None, h2: torch.Tensor, norm: tuple | None = None) -> torch.Tensor:
        """The next gate / up / down weights as a dense SwiGLU MLP plus the
        residual: h2 + down(fp16(silu(gate(h3)) * up(h3))), with h3 =
        rmsnorm(h2) * norm[0] computed inside the kernel when h3 is None.
        Resident weights: one persistent launch (up's epilogue applies SwiGLU,
        down depends on up and adds the residual); otherwise three GEMVs,
        swiglu and an add."""
        if h3 is None and norm is None:
            raise ValueError("next_mlp needs h3 or the norm to compute it")
        names = self._batched(3)
        if names is not None:
            mg, mu, md = (self.model.matrices[n] for n in names)
            res, g = self.model.resident, self.model.group_size
            dev = h2.device
            xin = h3 if h3 is not None else h2
            nrm = None if h3 is not None else norm
            gate = torch.empty(mg.n, dtype=torch.float16, device=dev)
            hidden = torch.empty(mu.n, dtype=torch.float16, device=dev)
            out = torch.empty(md.n, dtype=torch.float16, device=dev)
            tasks = [(res[names[0]], mg.scale, xin, gate, mg.packed_k, g, -1, None, None, nrm),
                     (res[names[1]], mu.scale, xin, hidden, mu.packed_k, g, -1, None, gate, nrm),
                     (res[names[2]], md.scale, hidden, out, md.packed_k, g, 1, h2)]
            for _ in range(3):
                self.cur_buf, self.cur_name = 1 - self.cur_buf, self._advance()
            _C.gemv_w4a16_batch(tasks)
            return out
        if h3 is None:
            h3 = ops.rmsnorm(h2.unsqueeze(0), norm[0], norm[1]).squeeze(0)
        gate, up = self.next_gemvs(h3, 2)
        return h2 + self.next_gemv(ops.swiglu(gate, up))


# --------------------------------------------------------------- attention
@dataclass
class DevicePosition:
    """A token position held on the device (int32 [1]) with RoPE tables
    [max_seq, head_dim/2]: passed as `pos` to the layer functions it makes a
    decode step independent of host values, so it can be captured in a CUDA
    graph and replayed while the position advances on the device."""

    pos: torch.Tensor
    cos_table: torch.Tensor
    sin_table: torch.Tensor


def _attention_block(pipeline: WeightPipeline, model: StreamingModel, layer_idx: int, x_flat: torch.Tensor, pos: int,
                     k_cache: torch.Tensor, v_cache: torch.Tensor, reduce_o=None, h_in: torch.Tensor | None = None,
                     o_block=None, fuse_norms: bool = False) -> tuple[torch.Tensor, torch.Tensor | None]:
    """rmsnorm -> q/k/v GEMVs -> q/k norm + RoPE + KV append (one kernel) ->
    GQA decode attention -> o GEMV -> residual add + post-attention rmsnorm
    (one kernel).  Returns (h2 = x + o, h3 = rmsnorm(h2)).  Tensor-parallel
    hooks: reduce_o maps the o GEMV output before the residual (the cross-rank
    sum of row-parallel partials); h_in is rmsnorm(x) when already computed;
    o_block(attn, x, post_norm_weight, eps) -> (h2, h3) replaces the o GEMV,
    the residual add and the rmsnorm (it consumes the o weight from the
    pipeline itself).  fuse_norms: the input rmsnorm runs inside the q/k/v
    batched kernel, the o GEMV adds the residual in its epilogue, and h3 is
    returned as None (the MLP normalises h2 in its own kernel)."""
    NQ, NKV, HD = model.num_attention_heads, model.num_key_value_heads, model.head_dim
    eps = model.rms_norm_eps
    norms = model.layer_norms[layer_idx]
    if fuse_norms and h_in is None:
        q, k, v = pipeline.next_gemvs(x_flat, 3, norm=(norms["input_layernorm"], eps))
    else:
        h = h_in if h_in is not None else ops.rmsnorm(x_flat.unsqueeze(0), norms["input_layernorm"], eps).squeeze(0)
        q, k, v = pipeline.next_gemvs(h, 3)
    q, k, v = q.view(NQ, HD), k.view(NKV, HD), v.view(NKV, HD)
    if isinstance(pos, DevicePosition):
        ops.head_norm_rope(q, k, v, norms["q_norm"], norms["k_norm"], pos.cos_table, pos.sin_table, k_cache, v_cache,
                           pos_dev=pos.pos, eps=eps)
        attn = ops.decode_attention_at(q, k_cache, v_cache, pos.pos).reshape(NQ * HD)
    else:
        cos_vals, sin_vals = ops.precompute_rope_cos_sin(HD, model.rope_theta, pos, device=x_flat.device)
        ops.head_norm_rope(q, k, v, norms["q_norm"], norms["k_norm"], cos_vals, sin_vals, k_cache, v_cache, pos=pos,
                           eps=eps)
        attn = ops.decode_attention(q, k_cache, v_cache, pos + 1).reshape(NQ * HD)
    if o_block is not None:
        return o_block(attn, x_flat, norms["post_attention_layernorm"], eps)
    if fuse_norms and reduce_o is None:
        return pipeline.next_gemv_residual(attn, x_flat), None
    o = pipeline.next_gemv(attn)
    if reduce_o is not None:
        o = reduce_o(o)
    h3, h2 = ops.add_rmsnorm(x_flat.unsqueeze(0), o.unsqueeze(0), norms["post_attention_layernorm"], eps)
    return h2.squeeze(0), h3.squeeze(0)


def _attention_and_gate(pipeline: WeightPipeline, model: StreamingModel, layer_idx: int, x_flat: torch.Tensor, pos,
                        k_cache: torch.Tensor, v_cache: torch.Tensor):
    """Attention half + the dense gate GEMV of a DIP layer: (h2, h3, gate).
    Resident weights: the norms run inside the batched kernels (q/k/v; gate,
    which also writes h3 for the selected-row kernels) and o adds the
    residual in its epilogue."""
    names = pipeline._batched(5)  # q, k, v, o, gate
    if names is None:
        h2, h3 = _attention_block(pipeline, model, layer_idx, x_flat, pos, k_cache, v_cache)
        return h2, h3, pipeline.next_gemv(h3)
    h2, _ = _attention_block(pipeline, model, layer_idx, x_flat, pos, k_cache, v_cache, fuse_norms=True)
    h3 = torch.empty_like(h2)
    norm = (model.layer_norms[layer_idx]["post_attention_layernorm"], model.rms_norm_eps, h3)
    gate = pipeline.next_gemvs(h2, 1, norm=norm)[0]
    return h2, h3, gate


def run_decoder_layer_streaming(pipeline: WeightPipeline, model: StreamingModel, layer_idx: int,
                                x_flat: torch.Tensor, pos: int, k_cache: torch.Tensor,
                                v_cache: torch.Tensor) -> torch.Tensor:
    """Dense layer: all 7 linear weights through the pipeline (reference generate.py:141-182).
    Both rmsnorms run inside the batched GEMV kernels (q/k/v and gate/up)."""
    h2, h3 = _attention_block(pipeline, model, layer_idx, x_flat, pos, k_cache, v_cache, fuse_norms=True)
    return pipeline.next_mlp(h3, h2, norm=(model.layer_norms[layer_idx]["post_attention_layernorm"],
                                            model.rms_norm_eps))


# --------------------------------------------------------------------- DIP
@dataclass
class DipBuffers:
    """Device rows for the selected (DIP) or missed (cached DIP) up_proj /
    down_proj_T rows and their scale rows, allocated once for the largest k
    (reference generate.py:185-212; no pinned staging: the gather is
    device-driven)."""

    gpu_up: torch.Tensor     # CUDA uint8 [max_k * up_row_nbytes]
    gpu_down: torch.Tensor   # CUDA uint8 [max_k * downT_row_nbytes]
    up_row_nbytes: int
    down_row_nbytes: int
    gpu_up_scale: torch.Tensor | None = None    # CUDA fp32 [max_k, up groups]
    gpu_down_scale: torch.Tensor | None = None  # CUDA fp32 [max_k, downT groups]

    @staticmethod
    def make(model: StreamingModel, max_k: int) -> "DipBuffers":
        up = model.matrix(0, "mlp.up_proj.weight")
        down_t = model.matrix(0, DOWN_PROJ_T_SUFFIX)
        up_rb, down_rb = up.handle.row_nbytes, down_t.handle.row_nbytes
        dev = model.device
        return DipBuffers(gpu_up=torch.empty(max_k * up_rb, dtype=torch.uint8, device=dev),
                          gpu_down=torch.empty(max_k * down_rb, dtype=torch.uint8, device=dev),
                          up_row_nbytes=up_rb, down_row_nbytes=down_rb,
                          gpu_up_scale=torch.empty(max_k, up.scale.size(1), dtype=torch.float32, device=dev),
                          gpu_down_scale=torch.empty(max_k, down_t.scale.size(1), dtype=torch.float32, device=dev))

    def up_rows(self, k: int) -> torch.Tensor:
        return self.gpu_up[: k * self.up_row_nbytes].view(k, self.up_row_nbytes)

    def down_rows(self, k: int) -> torch.Tensor:
        return self.gpu_down[: k * self.down_row_nbytes].view(k, self.down_row_nbytes)


def _select(gate: torch.Tensor, dip_k: int) -> torch.Tensor:
    """The reference's DIP selector on |gate| (fp32 |float(g)|): int32 [dip_k] ascending channel indices."""
    return ops.topk_threshold_select_abs(gate, dip_k)


def run_decoder_layer_dip(pipeline: WeightPipeline, model: StreamingModel, layer_idx: int, x_flat: torch.Tensor,
                          pos: int, k_cache: torch.Tensor, v_cache: torch.Tensor, dip_k: int, bufs: DipBuffers,
                          channel_counts: list[torch.Tensor] | None = None,
                          selected_out: list[list] | None = None) -> torch.Tensor:
    """DIP layer (reference generate.py:215-310): dense gate, top-dip_k |gate|
    channels, up_proj on the selected rows, h = fp16(silu(g) * u), down_proj_T
    sparse accumulate over the same rows.  channel_counts[layer] (int64 [I]
    CUDA) accumulates selections; selected_out[layer] collects the index lists
    (this one syncs)."""
    h2, h3, gate = _attention_and_gate(pipeline, model, layer_idx, x_flat, pos, k_cache, v_cache)
    idx = _select(gate, dip_k)
    idx_long = idx.long() if (channel_counts is not None or selected_out is not None
                              or not model.is_resident(model.matrix(layer_idx, "mlp.up_proj.weight").handle.name)
                              or not model.is_resident(model.matrix(layer_idx, DOWN_PROJ_T_SUFFIX).handle.name)) else None
    if channel_counts is not None:
        channel_counts[layer_idx].scatter_add_(0, idx_long, torch.ones_like(idx_long))
    if selected_out is not None:
        selected_out[layer_idx].append(idx_long.cpu().tolist())
    return dip_mlp_tail(model, layer_idx, h3, gate, idx, dip_k, bufs, idx_long, residual=h2)


def dip_mlp_tail(model: StreamingModel, layer_idx: int, h3: torch.Tensor, gate: torch.Tensor, idx: torch.Tensor,
                 dip_k: int, bufs: DipBuffers, idx_long: torch.Tensor | None = None,
                 residual: torch.Tensor | None = None) -> torch.Tensor:
    """The DIP MLP after the selection (the DIP block minus the gate GEMV
    and selector): up_proj on the selected rows, h = fp16(silu(g) * u),
    down_proj_T sparse accumulate -- resident rows read in place (SwiGLU in
    the row GEMV's epilogue, the residual in the down GEMV's), arena rows
    gathered on the device.  Returns residual + down (or down)."""
    up = model.matrix(layer_idx, "mlp.up_proj.weight")
    down_t = model.matrix(layer_idx, DOWN_PROJ_T_SUFFIX)
    g = model.group_size
    if idx_long is None and not (model.is_resident(up.handle.name) and model.is_resident(down_t.handle.name)):
        idx_long = idx.long()
    if model.is_resident(up.handle.name):
        h_sel = ops.gemv_w4a16_rows(model.resident[up.handle.name], up.scale, idx, h3, up.packed_k, g, glu_gate=gate)
    else:
        rows = bufs.up_rows(dip_k)
        ops.gather_rows_device(model.weight_source(up), idx, rows)
        u_sel = ops.gemv_w4a16_group_lop3(rows, up.scale.index_select(0, idx_long), h3, up.packed_k, g)
        h_sel = ops.swiglu(gate, u_sel, idx)
    if model.is_resident(down_t.handle.name):
        return ops.gemv_w4a16_sparse_rows(model.resident[down_t.handle.name], down_t.scale, idx, h_sel,
                                          model.hidden_size, g, residual=residual)
    rows = bufs.down_rows(dip_k)
    ops.gather_rows_device(model.weight_source(down_t), idx, rows)
    down = ops.gemv_w4a16_sparse_accumulate(rows, down_t.scale.index_select(0, idx_long), h_sel, model.hidden_size,
                                            g)
    return down if residual is None else residual + down


def run_decoder_layer_cached_dip(pipeline: WeightPipeline, model: StreamingModel, layer_idx: int,
                                 x_flat: torch.Tensor, pos, k_cache: torch.Tensor, v_cache: torch.Tensor,
                                 dip_k: int, bufs: DipBuffers, caches: list[HotCache],
                                 miss_counts: torch.Tensor | None = None) -> torch.Tensor:
    """Cache-aware DIP layer (reference generate.py:313-404): the selected
    channels resolve to hot-cache slots or staging rows (the misses, gathered
    from the arena); one fused GEMV per direction reads both.  Bit-identical
    to run_decoder_layer_dip on the same inputs.  No host read: the miss count
    stays on the device, so the layer runs inside GraphDecoder's per-token
    graph.  miss_counts (int64 [num_layers] CUDA, optional) accumulates each
    layer's miss count on the device."""
    h2, h3, gate = _attention_and_gate(pipeline, model, layer_idx, x_flat, pos, k_cache, v_cache)
    idx = _select(gate, dip_k)
    return cached_dip_mlp_tail(model, layer_idx, h3, gate, idx, bufs, caches[layer_idx], miss_counts, residual=h2)


def cached_dip_mlp_tail(model: StreamingModel, layer_idx: int, h3: torch.Tensor, gate: torch.Tensor,
                        idx: torch.Tensor, bufs: DipBuffers, cache: HotCache,
                        miss_counts: torch.Tensor | None = None,
                        residual: torch.Tensor | None = None) -> torch.Tensor:
    """The cache-aware DIP MLP after the selection (the cached-DIP block minus the
    gate GEMV and selector): the selected channels resolve to hot-cache slots
    or misses (descriptors, ordered miss list and miss count, all on the
    device); one device-driven gather brings the misses' up / down_T rows and
    scale rows (zero-copy over PCIe from the pinned arena, or from HBM when
    the matrix is resident) into staging sized for every selected channel,
    reading the count on the device; one fused GEMV per direction reads cache
    and staging rows.  Returns residual + down (or down)."""
    up = model.matrix(layer_idx, "mlp.up_proj.weight")
    down_t = model.matrix(layer_idx, DOWN_PROJ_T_SUFFIX)
    g = model.group_size
    k = idx.numel()
    desc, miss, miss_count = ops.build_dip_descriptors(idx, cache.slot_of)
    up_rows, down_rows = bufs.up_rows(k), bufs.down_rows(k)
    up_sc, down_sc = bufs.gpu_up_scale[:k], bufs.gpu_down_scale[:k]
    ops.gather_rows_device_multi([(model.weight_source(up), up_rows), (model.weight_source(down_t), down_rows),
                                  (up.scale, up_sc), (down_t.scale, down_sc)], miss, miss_count, k)
    if miss_counts is not None:
        miss_counts[layer_idx : layer_idx + 1].add_(miss_count)
    u_sel = ops.gemv_dip_fused_up(cache.up_Wq, cache.up_scale, up_rows, up_sc, desc, h3, up.packed_k, g)
    h_sel = ops.swiglu(gate, u_sel, idx)
    down = ops.gemv_dip_fused_down(cache.down_Wq, cache.down_scale, down_rows, down_sc, desc, h_sel,
                                   model.hidden_size, g)
    return down if residual is None else residual + down


def miss_row_bytes(model: StreamingModel) -> int:
    """Streamed bytes per missed channel: one up_proj row + one down_proj_T row."""
    return (model.matrix(0, "mlp.up_proj.weight").handle.row_nbytes
            + model.matrix(0, DOWN_PROJ_T_SUFFIX).handle.row_nbytes)


def dip_bytes_per_token(model: StreamingModel, dip_k: int, dense: bool = False) -> int:
    """Per-token weight bytes of the decode path (reference generate.py:407-426):
    q/k/v/o/gate in full, up_proj / down_proj_T in full (dense) or dip_k rows."""
    total = 0
    for layer in range(model.num_layers):
        for suffix in DIP_DENSE_SUFFIXES:
            m = model.matrix(layer, suffix)
            total += m.n * m.handle.row_nbytes
        up = model.matrix(layer, "mlp.up_proj.weight")
        down_t = model.matrix(layer, DOWN_PROJ_T_SUFFIX)
        total += (up.n if dense else dip_k) * up.handle.row_nbytes
        total += (down_t.n if dense else dip_k) * down_t.handle.row_nbytes
    return total


# ------------------------------------------------------------------- loops
def _kv_caches(model: StreamingModel, max_seq_len: int):
    shape = (model.num_key_value_heads, max_seq_len, model.head_dim)
    dev = model.device
    return ([torch.zeros(shape, dtype=torch.float16, device=dev) for _ in range(model.num_layers)],
            [torch.zeros(shape, dtype=torch.float16, device=dev) for _ in range(model.num_layers)])


def _next_token(model: StreamingModel, xn: torch.Tensor) -> torch.Tensor:
    return ops.lm_head_argmax(model.lm_head, xn)


def _greedy(model: StreamingModel, prompt_ids: list[int], n_new: int, run_layer, eos_token_id: int | None,
            max_seq_len: int, token_fn=None) -> list[int]:
    """Prefill the prompt one token at a time, then greedy-decode n_new tokens.
    run_layer(layer_idx, x, pos, k_cache, v_cache) -> x.  Token ids stay on
    the device until the end (a host sync per token only with an EOS id)."""
    if len(prompt_ids) + n_new > max_seq_len:
        raise ValueError(f"prompt ({len(prompt_ids)}) + n_new ({n_new}) exceeds max_seq_len ({max_seq_len})")
    k_caches, v_caches = _kv_caches(model, max_seq_len)
    dev = model.device

    def forward(x, pos):
        for li in range(model.num_layers):
            x = run_layer(li, x, pos, k_caches[li], v_caches[li])
        return x

    x = None
    for pos, tok in enumerate(prompt_ids):
        x = forward(model.embed_tokens[tok], pos)
    new_ids = []
    pos = len(prompt_ids)
    for _ in range(n_new):
        xn = ops.rmsnorm(x.unsqueeze(0), model.final_norm, model.rms_norm_eps).squeeze(0)
        idx = (token_fn or _next_token)(model, xn)  # int32 [1] on the device
        new_ids.append(idx)
        if eos_token_id is not None and int(idx.item()) == eos_token_id:
            break
        x = forward(model.embed_tokens.index_select(0, idx.long()).view(-1), pos)
        pos += 1
    out = list(prompt_ids)
    if new_ids:
        out += torch.cat(new_ids).cpu().tolist()
    return out


def generate_streaming(model: StreamingModel, prompt_ids: list[int], n_new: int, eos_token_id: int | None = None,
                       max_seq_len: int = 512) -> list[int]:
    """Greedy decode, dense layers (reference generate.py:429-463)."""
    pipeline = WeightPipeline(model)
    return _greedy(model, prompt_ids, n_new,
                   lambda li, x, p, kc, vc: run_decoder_layer_streaming(pipeline, model, li, x, p, kc, vc),
                   eos_token_id, max_seq_len)


def generate_dip(model: StreamingModel, prompt_ids: list[int], n_new: int, dip_k: int,
                 eos_token_id: int | None = None, max_seq_len: int = 512) -> list[int]:
    """Greedy decode, DIP MLPs (reference generate.py:466-500)."""
    pipeline = WeightPipeline(model, suffixes=DIP_DENSE_SUFFIXES)
    bufs = DipBuffers.make(model, dip_k)
    return _greedy(model, prompt_ids, n_new,
                   lambda li, x, p, kc, vc: run_decoder_layer_dip(pipeline, model, li, x, p, kc, vc, dip_k, bufs),
                   eos_token_id, max_seq_len)


def generate_cached_dip(model: StreamingModel, prompt_ids: list[int], n_new: int, dip_k: int,
                        caches: list[HotCache], eos_token_id: int | None = None, max_seq_len: int = 512,
                        miss_bytes: list[int] | None = None) -> list[int]:
    """Greedy decode, cache-aware DIP MLPs (reference generate.py:503-542).
    miss_bytes[layer] (optional) is increased by the streamed bytes, read
    from the device counters once at the end."""
    pipeline = WeightPipeline(model, suffixes=DIP_DENSE_SUFFIXES)
    bufs = DipBuffers.make(model, dip_k)
    counts = torch.zeros(model.num_layers, dtype=torch.int64, device=model.device) if miss_bytes is not None else None
    out = _greedy(model, prompt_ids, n_new,
                  lambda li, x, p, kc, vc: run_decoder_layer_cached_dip(pipeline, model, li, x, p, kc, vc, dip_k,
                                                                        bufs, caches, counts),
                  eos_token_id, max_seq_len)
    if miss_bytes is not None:
        per_row = miss_row_bytes(model)
        for li, c in enumerate(counts.cpu().tolist()):
            miss_bytes[li] += int(c) * per_row
    return out


class GraphDecoder:
    """Greedy decode with one CUDA graph per step (B200 addition).

    The step -- embedding of ids[pos], every decoder layer (dense or DIP),
    final norm, the LM head with its fused argmax, then ids[pos + 1] =
    next token unless it is still a prompt token, pos += 1 -- reads and writes
    only device state, so it is captured once and replayed; generating n
    tokens after a P-token prompt is P + n - 1 replays with no host work in
    between.  Weights must be HBM-resident.  Tokens equal generate_streaming /
    generate_dip on the same model (same kernels, same order)."""

    def __init__(self, model: StreamingModel, dip_k: int | None = None, max_seq_len: int = 2048, layer_fn=None,
                 token_fn=None, caches: list[HotCache] | None = None, fused: bool = False):
        """layer_fn(pipeline, model, layer_idx, x, where, k_cache, v_cache) -> x and
        token_fn(model, xn) -> int32 [1] replace the dense / DIP layer and the
        fused LM-head argmax (tensor parallelism plugs in here).  caches (with
        dip_k): cache-aware DIP -- up_proj / down_proj_T may stay in the pinned
        arena (misses read zero-copy by the device gather); the per-layer miss
        counts accumulate in self.miss_counts.  fused (dense INT4, group size
        128): every decoder layer of the step runs in one cooperative kernel
        (soinfer_decode_layers_fused) -- same bits, same tokens."""
        if caches is not None and dip_k is None:
            raise ValueError("GraphDecoder: caches need dip_k (cache-aware DIP)")
        streamed_ok = ("mlp.up_proj.weight", "mlp.down_proj.weight") if caches is not None else ()
        names = [f"model.layers.{i}.{s}" for i in range(model.num_layers) for s in LINEAR_SUFFIXES
                 if s not in streamed_ok]
        if dip_k is not None and caches is None:
            names.append(f"model.layers.0.{DOWN_PROJ_T_SUFFIX}")
        if not all(model.is_resident(n) for n in names):
            raise ValueError("GraphDecoder needs every decoder weight resident in HBM (StreamingModel.resident)")
        self.caches = caches
        self.miss_counts = (torch.zeros(model.num_layers, dtype=torch.int64, device=model.device)
                            if caches is not None else None)
        self.model, self.dip_k, self.max_seq_len = model, dip_k, max_seq_len
        dev = model.device
        self.stream = torch.cuda.Stream(dev)
        self.ids = torch.zeros(max_seq_len + 1, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.prompt_len = torch.zeros(1, dtype=torch.int32, device=dev)
        self.x_in = torch.empty(model.hidden_size, dtype=torch.float16, device=dev)  # the step's input row
        cos_t, sin_t = ops.precompute_rope_table(model.head_dim, model.rope_theta, max_seq_len, dev)
        self.where = DevicePosition(self.pos, cos_t, sin_t)
        self.k_caches, self.v_caches = _kv_caches(model, max_seq_len)
        suffixes = LINEAR_SUFFIXES if dip_k is None else DIP_DENSE_SUFFIXES
        self.pipeline = WeightPipeline(model, suffixes=suffixes)
        self.bufs = DipBuffers.make(model, dip_k) if dip_k is not None else None
        self.graph = None
        self.layer_fn, self.token_fn = layer_fn, token_fn or _next_token
        self.fused = None
        if fused:
            if dip_k is not None or layer_fn is not None or caches is not None:
                raise ValueError("GraphDecoder: fused runs the dense layer only")
            if model.group_size != 128 or any(model.matrices[n].bits != 4 for n in names):
                raise ValueError("GraphDecoder: fused needs INT4 weights with group size 128")
            layers = []
            for li in range(model.num_layers):
                mats = [model.matrices[f"model.layers.{li}.{s}"] for s in LINEAR_SUFFIXES]
                norms = model.layer_norms[li]
                layers.append({"w": [model.resident[f"model.layers.{li}.{s}"] for s in LINEAR_SUFFIXES],
                               "s": [m.scale.contiguous() for m in mats],
                               "input_norm": norms["input_layernorm"], "post_norm": norms["post_attention_layernorm"],
                               "q_norm": norms["q_norm"], "k_norm": norms["k_norm"],
                               "k_cache": self.k_caches[li], "v_cache": self.v_caches[li]})
            inter = model.matrices["model.layers.0.mlp.gate_proj.weight"].n
            self.fused = _C.FusedDecode(layers, model.hidden_size, inter, model.num_attention_heads,
                                        model.num_key_value_heads, model.head_dim, max_seq_len, model.rms_norm_eps,
                                        cos_t, sin_t)

    def _step(self) -> None:
        m, where = self.model, self.where
        x = self.x_in
        _C.decode_step_embed(m.embed_tokens, self.ids, self.pos, x)  # x = embed[ids[pos]], on the device
        if self.fused is not None:
            self.fused.run(x, self.pos)
        for li in range(m.num_layers if self.fused is None else 0):
            if self.layer_fn is not None:
                x = self.layer_fn(self.pipeline, m, li, x, where, self.k_caches[li], self.v_caches[li])
            elif self.dip_k is None:
                x = run_decoder_layer_streaming(self.pipeline, m, li, x, where, self.k_caches[li], self.v_caches[li])
            elif self.caches is not None:
                x = run_decoder_layer_cached_dip(self.pipeline, m, li, x, where, self.k_caches[li], self.v_caches[li],
                                                 self.dip_k, self.bufs, self.caches, self.miss_counts)
            else:
                x = run_decoder_layer_dip(self.pipeline, m, li, x, where, self.k_caches[li], self.v_caches[li],
                                          self.dip_k, self.bufs)
        xn = ops.rmsnorm(x.unsqueeze(0), m.final_norm, m.rms_norm_eps).squeeze(0)
        nxt = self.token_fn(m, xn)
        if nxt.dtype != torch.int32:
            nxt = nxt.to(torch.int32)
        # ids[pos + 1] = nxt unless still inside the prompt (its token stays); pos += 1
        _C.decode_step_advance(self.ids, self.pos, self.prompt_len, nxt.reshape(1))

    def _capture(self) -> None:
        # the buffers, caches and weights were made on the caller's stream
        self.stream.wait_stream(torch.cuda.current_stream(self.model.device))
        with torch.cuda.stream(self.stream):
            self.pos.zero_()
            self._step()  # warm-up: workspaces and lazy initialisation outside the capture
            self.stream.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=self.stream):
                self._step()
        torch.cuda.synchronize(self.model.device)

    def generate(self, prompt_ids: list[int], n_new: int, timings: dict | None = None) -> list[int]:
        """timings (optional): filled with CUDA-event milliseconds of the prompt
        replays ("prefill_ms") and of the n_new - 1 generating replays ("decode_ms")."""
        P = len(prompt_ids)
        if P < 1 or P + n_new > self.max_seq_len:
            raise ValueError(f"need 1 <= prompt length and prompt + n_new <= max_seq_len ({self.max_seq_len})")
        if self.graph is None:
            self._capture()
        self.stream.wait_stream(torch.cuda.current_stream(self.model.device))
        with torch.cuda.stream(self.stream):
            self.ids.zero_()
            self.ids[:P].copy_(torch.tensor(prompt_ids, dtype=torch.int32), non_blocking=False)
            self.prompt_len.fill_(P)
            self.pos.zero_()
            for kc, vc in zip(self.k_caches, self.v_caches):
                kc.zero_()
                vc.zero_()
            if self.miss_counts is not None:
                self.miss_counts.zero_()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            ev[0].record(self.stream)
            for _ in range(P):
                self.graph.replay()
            ev[1].record(self.stream)
            for _ in range(n_new - 1):
                self.graph.replay()
            ev[2].record(self.stream)
        self.stream.synchronize()
        if timings is not None:
            timings["prefill_ms"] = ev[0].elapsed_time(ev[1])
            timings["decode_ms"] = ev[1].elapsed_time(ev[2])
        return self.ids[: P + n_new].cpu().tolist()


def teacher_forced_nll(model: StreamingModel, layer_fn, token_ids: list[int], max_seq_len: int = 512) -> float:
    """Mean NLL of each real next token with the true prefix fed
    (reference generate.py:545-582).  layer_fn(model, layer_idx, x, pos,
    k_cache, v_cache) -> x selects the decode path."""
    k_caches, v_caches = _kv_caches(model, max_seq_len)
    total, count = 0.0, 0
    for pos, tok in enumerate(token_ids[:-1]):
        x = model.embed_tokens[tok]
        for li in range(model.num_layers):
            x = layer_fn(model, li, x, pos, k_caches[li], v_caches[li])
        xn = ops.rmsnorm(x.unsqueeze(0), model.final_norm, model.rms_norm_eps).squeeze(0)
        logp = F.log_softmax(ops.gemv_fp16_v3(model.lm_head, xn).float(), dim=-1)
        total += -float(logp[token_ids[pos + 1]].item())
        count += 1
    return total / count


def _calibrate(model: StreamingModel, token_ids: list[int], dip_k: int, max_seq_len: int, trace: bool):
    I = model.matrix(0, "mlp.up_proj.weight").n
    counts = [torch.zeros(I, dtype=torch.int64, device=model.device) for _ in range(model.num_layers)]
    selected = [[] for _ in range(model.num_layers)] if trace else None
    k_caches, v_caches = _kv_caches(model, max_seq_len)
    pipeline = WeightPipeline(model, suffixes=DIP_DENSE_SUFFIXES)
    bufs = DipBuffers.make(model, dip_k)
    for pos, tok in enumerate(token_ids):
        x = model.embed_tokens[tok]
        for li in range(model.num_layers):
            x = run_decoder_layer_dip(pipeline, model, li, x, pos, k_caches[li], v_caches[li], dip_k, bufs,
                                      channel_counts=counts, selected_out=selected)
    return counts, selected


def calibrate_channel_frequencies(model: StreamingModel, token_ids: list[int], dip_k: int,
                                  max_seq_len: int = 512) -> list[torch.Tensor]:
    """Per layer, how many of the tokens selected each channel, teacher-forced
    through the DIP path (reference generate.py:585-614)."""
    return _calibrate(model, token_ids, dip_k, max_seq_len, trace=False)[0]


def calibrate_with_trace(model: StreamingModel, token_ids: list[int], dip_k: int, max_seq_len: int = 512):
    """As calibrate_channel_frequencies, plus the per-token, per-layer selected
    index lists the adaptive cache policies replay (reference generate.py:617-645)."""
    return _calibrate(model, token_ids, dip_k, max_seq_len, trace=True)


__all__ = [
    "StreamingModel", "WeightPipeline", "DipBuffers", "DIP_DENSE_SUFFIXES", "DOWN_PROJ_T_SUFFIX", "LINEAR_SUFFIXES",
    "run_decoder_layer_streaming", "run_decoder_layer_dip", "run_decoder_layer_cached_dip", "dip_bytes_per_token",
    "generate_streaming", "generate_dip", "generate_cached_dip", "teacher_forced_nll",
    "calibrate_channel_frequencies", "calibrate_with_trace", "DevicePosition", "GraphDecoder",
]
