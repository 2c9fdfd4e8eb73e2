"""Pinned host arena of quantized weight matrices with rows as the
addressable unit (reference python/soinfer/offload/weight_store.py:26-117).

One cudaHostAlloc-backed allocation sized up front; each registered matrix
occupies a contiguous [num_rows, row_nbytes] span, so any subset of rows can
be gathered (DIP) and whole matrices streamed (dense offload) straight from
it.  Because torch pins with cudaHostAlloc, the arena is also mapped into the
device address space, which the device-driven zero-copy gather uses.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class WeightHandle:
    """One matrix's span of the arena (offset is private to the store)."""

    name: str
    offset: int
    num_rows: int
    row_nbytes: int

    @property
    def nbytes(self) -> int:
        return self.num_rows * self.row_nbytes


class PinnedWeightStore:
    def __init__(self, total_bytes: int, pin: bool = True):
        """pin=False: pageable memory (host-only use, e.g. preparing or
        inspecting an arena on a machine without a GPU)."""
        if total_bytes <= 0:
            raise ValueError("total_bytes must be positive")
        self.arena = torch.empty(total_bytes, dtype=torch.uint8, pin_memory=pin)
        self._next = 0
        self._handles: dict[str, WeightHandle] = {}

    def register(self, name: str, data: torch.Tensor) -> WeightHandle:
        """Copy data ([num_rows, row_nbytes] uint8, any device) into the next
        free span; registration order fixes the layout."""
        if name in self._handles:
            raise ValueError(f"weight {name!r} already registered")
        if data.dtype != torch.uint8 or data.dim() != 2:
            raise ValueError(f"register({name!r}): data must be 2D uint8 [num_rows, row_nbytes], got "
                             f"{tuple(data.shape)} {data.dtype}")
        rows, rb = data.shape
        end = self._next + rows * rb
        if end > self.arena.numel():
            raise ValueError(f"register({name!r}): arena overflow -- {rows * rb} bytes requested, "
                             f"{self.arena.numel() - self._next} remain")
        self.arena[self._next:end].view(rows, rb).copy_(data)
        h = WeightHandle(name, self._next, rows, rb)
        self._handles[name] = h
        self._next = end
        return h

    def adopt(self, name: str, offset: int, num_rows: int, row_nbytes: int) -> WeightHandle:
        """Registers a span whose bytes are already in the arena (a loaded
        serialized arena); spans must come in increasing offset order."""
        if name in self._handles:
            raise ValueError(f"weight {name!r} already registered")
        end = offset + num_rows * row_nbytes
        if offset < self._next or end > self.arena.numel():
            raise ValueError(f"adopt({name!r}): span [{offset}, {end}) overlaps or leaves the arena")
        h = WeightHandle(name, offset, num_rows, row_nbytes)
        self._handles[name] = h
        self._next = end
        return h

    def handle(self, name: str) -> WeightHandle:
        return self._handles[name]

    def matrix_view(self, handle: WeightHandle) -> torch.Tensor:
        return self.arena[handle.offset:handle.offset + handle.nbytes].view(handle.num_rows, handle.row_nbytes)

    def row_view(self, handle: WeightHandle, row: int) -> torch.Tensor:
        if not 0 <= row < handle.num_rows:
            raise IndexError(f"row {row} out of range for {handle.name!r} (num_rows={handle.num_rows})")
        start = handle.offset + row * handle.row_nbytes
        return self.arena[start:start + handle.row_nbytes]

    def rows_view(self, handle: WeightHandle, rows: torch.Tensor) -> torch.Tensor:
        """Selected rows copied into a new contiguous tensor (host index_select)."""
        return self.matrix_view(handle).index_select(0, rows).contiguous()

    @property
    def bytes_used(self) -> int:
        return self._next

    @property
    def bytes_total(self) -> int:
        return self.arena.numel()
