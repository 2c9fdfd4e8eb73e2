"""Hot-channel cache for cache-aware DIP (reference
python/soinfer/offload/hot_cache.py:55-315).

Two independent halves:

* Policy simulation on the CPU.  Given a trace of per-token selected channel
  sets, each policy reports the hit rate it would reach.  Channels of one
  token are always visited in ascending index order (the selector's output
  order must not matter), and every tie is broken toward keeping the lower
  channel index.
    - StaticFrequencyPolicy: a fixed hot set, the top-C channels by
      (-frequency, index), chosen once from calibration counts.
    - LRUPolicy: a token's channels are looked up against the cache state at
      the end of the previous token; hits are touched in index order, then
      the token's misses are inserted in index order, each evicting the
      least recently used entry when full.
    - LFUDecayPolicy: per channel, frequency += 1 on every selection; a miss
      inserts into free space or evicts the resident channel with the lowest
      frequency (ties: the higher index goes); every `decay_every` tokens all
      frequencies are multiplied by `decay`.
* HotCache: the device-resident cache the fused DIP kernels read -- up_proj
  rows and down_proj_T rows of the hot channels plus their scales, and
  slot_of[I] (slot of channel c, -1 if not cached).  Built once per layer;
  the rows come straight from the pinned arena through the device-driven
  zero-copy gather (no staging copy, no host round trip).
"""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass
from typing import TYPE_CHECKING, Iterable, Sequence

import numpy as np
import torch

if TYPE_CHECKING:  # the simulation half imports without the CUDA library
    from ..runtime.generate import StreamingModel


def _sorted_channels(selected) -> list[int]:
    if isinstance(selected, torch.Tensor):
        selected = selected.tolist()
    return sorted(int(c) for c in selected)


@dataclass
class SimulationResult:
    policy: str
    cache_size: int
    hits: int
    total: int

    @property
    def hit_rate(self) -> float:
        return self.hits / self.total if self.total else 0.0


class StaticFrequencyPolicy:
    name = "static"

    def __init__(self, frequencies: torch.Tensor | Sequence[int], cache_size: int):
        freq = np.asarray(frequencies.tolist() if isinstance(frequencies, torch.Tensor) else list(frequencies))
        n = len(freq)
        self.cache_size = min(int(cache_size), n)
        # stable sort on -freq keeps ascending index order among equal frequencies
        order = np.argsort(-freq, kind="stable") if n else np.zeros(0, dtype=np.int64)
        self.hot_list: list[int] = [int(c) for c in order[: self.cache_size]]
        self.hot_set: frozenset[int] = frozenset(self.hot_list)

    def simulate(self, trace: Iterable) -> SimulationResult:
        hits = total = 0
        for selected in trace:
            chans = _sorted_channels(selected)
            total += len(chans)
            hits += sum(1 for c in chans if c in self.hot_set)
        return SimulationResult(self.name, self.cache_size, hits, total)


class LRUPolicy:
    name = "lru"

    def __init__(self, cache_size: int):
        self.cache_size = int(cache_size)

    def simulate(self, trace: Iterable) -> SimulationResult:
        resident: "OrderedDict[int, None]" = OrderedDict()  # least recent first
        hits = total = 0
        for selected in trace:
            chans = _sorted_channels(selected)
            total += len(chans)
            missed = []
            for c in chans:  # lookups see the state left by the previous token
                if c in resident:
                    hits += 1
                    resident.move_to_end(c)
                else:
                    missed.append(c)
            if self.cache_size <= 0:
                continue
            for c in missed:
                if len(resident) >= self.cache_size:
                    resident.popitem(last=False)
                resident[c] = None
        return SimulationResult(self.name, self.cache_size, hits, total)


class LFUDecayPolicy:
    name = "lfu_decay"

    def __init__(self, cache_size: int, decay: float = 0.98, decay_every: int = 50):
        if not 0.0 < decay <= 1.0:
            raise ValueError("decay must be in (0, 1]")
        self.cache_size = int(cache_size)
        self.decay = float(decay)
        self.decay_every = int(decay_every)

    def simulate(self, trace: Iterable) -> SimulationResult:
        freq: dict[int, float] = {}
        resident: set[int] = set()
        hits = total = 0
        for step, selected in enumerate(trace):
            for c in _sorted_channels(selected):
                total += 1
                freq[c] = freq.get(c, 0.0) + 1.0
                if c in resident:
                    hits += 1
                elif self.cache_size <= 0:
                    continue
                elif len(resident) < self.cache_size:
                    resident.add(c)
                else:
                    # evict the lowest frequency; among equals the higher index
                    victim = min(resident, key=lambda r: (freq.get(r, 0.0), -r))
                    resident.remove(victim)
                    resident.add(c)
            if self.decay_every > 0 and (step + 1) % self.decay_every == 0:
                for c in freq:
                    freq[c] *= self.decay
        return SimulationResult(self.name, self.cache_size, hits, total)


def compare_policies(trace: Sequence, cache_sizes: Sequence[int], frequencies=None, **lfu_kwargs) -> list[SimulationResult]:
    """All three policies over the same trace at every cache size.  Without
    `frequencies` the static policy uses the trace's own per-channel counts."""
    trace = list(trace)
    if frequencies is None:
        counts: dict[int, int] = {}
        for selected in trace:
            for c in _sorted_channels(selected):
                counts[c] = counts.get(c, 0) + 1
        n = max(counts) + 1 if counts else 0
        frequencies = [counts.get(c, 0) for c in range(n)]
    out = []
    for size in cache_sizes:
        out.append(StaticFrequencyPolicy(frequencies, size).simulate(trace))
        out.append(LRUPolicy(size).simulate(trace))
        out.append(LFUDecayPolicy(size, **lfu_kwargs).simulate(trace))
    return out


@dataclass
class HotCache:
    slot_of: torch.Tensor      # [I] int32 CUDA, -1 if the channel is not cached
    hot_indices: torch.Tensor  # [C] int64 CUDA, ascending
    up_Wq: torch.Tensor        # [C, up_row_nbytes] uint8 CUDA
    up_scale: torch.Tensor     # [C, up_num_groups] float32 CUDA
    down_Wq: torch.Tensor      # [C, down_row_nbytes] uint8 CUDA
    down_scale: torch.Tensor   # [C, down_num_groups] float32 CUDA

    @property
    def cache_size(self) -> int:
        return int(self.hot_indices.shape[0])

    @staticmethod
    def build(model: "StreamingModel", layer_idx: int, hot_indices) -> "HotCache":
        """Gather the hot channels' up_proj / down_proj_T rows (arena or
        device-resident matrices) and scales into device cache tensors."""
        from .. import ops
        from .load_hf_checkpoint import DOWN_PROJ_T_SUFFIX

        dev = model.device
        hot = torch.tensor(_sorted_channels(hot_indices), dtype=torch.int64)
        C = int(hot.numel())
        up = model.matrices[f"model.layers.{layer_idx}.mlp.up_proj.weight"]
        down_t = model.matrices[f"model.layers.{layer_idx}.{DOWN_PROJ_T_SUFFIX}"]
        I = up.n
        hot_dev = hot.to(dev)
        slot_of = torch.full((I,), -1, dtype=torch.int32, device=dev)
        slot_of[hot_dev] = torch.arange(C, dtype=torch.int32, device=dev)
        up_rows = torch.empty(C, up.handle.row_nbytes, dtype=torch.uint8, device=dev)
        down_rows = torch.empty(C, down_t.handle.row_nbytes, dtype=torch.uint8, device=dev)
        if C > 0:
            rows32 = hot_dev.to(torch.int32)
            ops.gather_rows_device(model.weight_source(up), rows32, up_rows)
            ops.gather_rows_device(model.weight_source(down_t), rows32, down_rows)
        return HotCache(slot_of=slot_of, hot_indices=hot_dev, up_Wq=up_rows,
                        up_scale=up.scale.index_select(0, hot_dev).contiguous(), down_Wq=down_rows,
                        down_scale=down_t.scale.index_select(0, hot_dev).contiguous())


__all__ = ["SimulationResult", "StaticFrequencyPolicy", "LRUPolicy", "LFUDecayPolicy", "compare_policies", "HotCache"]
