"""Decode loop over weights streamed from the pinned arena (reference
python/soinfer/runtime/generate.py:58-645).

`WeightPipeline` walks the fixed, cyclic per-token sequence of weight names
one step ahead of compute: while the INT4 GEMV of weight i runs on the
compute stream, the copy engine already streams weight i+1 into the other of
two device buffers (side stream + events, write-after-read guarded).
"""
from __future__ import annotations

import itertools
from dataclasses import dataclass, field

import torch

from .. import ops
from ..offload.load_hf_checkpoint import DOWN_PROJ_T_SUFFIX, LINEAR_SUFFIXES, LoadedMatrix
from ..offload.stream_manager import StreamManager
from ..offload.weight_store import PinnedWeightStore

# q/k/v/o/gate stay dense-streamed in DIP; up_proj and down_proj_T are fetched
# per token as the selected rows only (reference generate.py:49-55).
DIP_DENSE_SUFFIXES = (
    "self_attn.q_proj.weight",
    "self_attn.k_proj.weight",
    "self_attn.v_proj.weight",
    "self_attn.o_proj.weight",
    "mlp.gate_proj.weight",
)


@dataclass
class StreamingModel:
    """Arena + handles, the small resident tensors, and the streaming machinery."""

    store: PinnedWeightStore
    matrices: dict[str, LoadedMatrix]
    num_layers: int
    embed_tokens: torch.Tensor | None
    lm_head: torch.Tensor | None
    final_norm: torch.Tensor | None
    layer_norms: list[dict[str, torch.Tensor]]
    hidden_size: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rms_norm_eps: float
    rope_theta: float
    group_size: int = 128
    stream_manager: StreamManager = field(init=False)

    def __post_init__(self) -> None:
        self.stream_manager = StreamManager(num_buffers=2)


class WeightPipeline:
    """Double-buffered, cyclic prefetch of per-token weights (reference generate.py:85-138)."""

    def __init__(self, model: StreamingModel, suffixes: tuple[str, ...] = LINEAR_SUFFIXES):
        self.model = model
        self.sm = model.stream_manager
        seq = [f"model.layers.{i}.{s}" for i in range(model.num_layers) for s in suffixes]
        max_bytes = max(model.matrices[n].n * model.matrices[n].handle.row_nbytes for n in seq)
        dev = self.sm.device
        self.bufs = [torch.empty(max_bytes, dtype=torch.uint8, device=dev) for _ in range(2)]
        self._names = itertools.cycle(seq)
        self.cur_buf = 0
        self.cur_name = next(self._names)
        self._prefetch_into(self.cur_buf, self.cur_name)

    def _view(self, buf_idx: int, m: LoadedMatrix) -> torch.Tensor:
        nbytes = m.n * m.handle.row_nbytes
        return self.bufs[buf_idx][:nbytes].view(m.n, m.handle.row_nbytes)

    def _prefetch_into(self, buf_idx: int, name: str) -> None:
        m = self.model.matrices[name]
        self.sm.prefetch(buf_idx, self._view(buf_idx, m), self.model.store.matrix_view(m.handle))

    def next_gemv(self, x_in: torch.Tensor) -> torch.Tensor:
        """GEMV of the weight in flight (waits on its copy event), then start the next prefetch."""
        m = self.model.matrices[self.cur_name]
        self.sm.wait(self.cur_buf)
        y = ops.gemv_w4a16_group_lop3(self._view(self.cur_buf, m), m.scale, x_in, m.packed_k, self.model.group_size)
        self.sm.mark_read_done(self.cur_buf)
        nxt = 1 - self.cur_buf
        name = next(self._names)
        self._prefetch_into(nxt, name)
        self.cur_buf, self.cur_name = nxt, name
        return y


__all__ = ["StreamingModel", "WeightPipeline", "DIP_DENSE_SUFFIXES", "DOWN_PROJ_T_SUFFIX", "LINEAR_SUFFIXES"]
