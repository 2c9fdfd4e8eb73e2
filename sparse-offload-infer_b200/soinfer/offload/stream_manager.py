"""Copy-engine prefetch streams with events (reference
python/soinfer/offload/stream_manager.py:10-86).

Buffer i has its own side stream and two events: `events[i]` marks "the H2D
copy into buffer i has landed" (the compute stream waits on it before a kernel
reads the buffer) and `read_done_events[i]` marks "the last reader of buffer i
has been issued" (the next copy into buffer i waits on it -- the
write-after-read guard the reference added, stream_manager.py:40-51).  All
waits are GPU-side (cudaStreamWaitEvent); the host never blocks.
"""
from __future__ import annotations

import torch


class StreamManager:
    def __init__(self, num_buffers: int = 2, device=None):
        if num_buffers < 1:
            raise ValueError("num_buffers must be >= 1")
        self.num_buffers = num_buffers
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.streams = [torch.cuda.Stream(device=self.device) for _ in range(num_buffers)]
        self.events = [torch.cuda.Event() for _ in range(num_buffers)]
        # never recorded until the first mark_read_done: waiting on an
        # unrecorded event is a no-op, right for a buffer's first fill
        self.read_done_events = [torch.cuda.Event() for _ in range(num_buffers)]

    def prefetch(self, buf_idx: int, gpu_buffer: torch.Tensor, host_data: torch.Tensor) -> None:
        """Async H2D copy host_data (pinned) -> gpu_buffer on buffer buf_idx's
        side stream, after the buffer's previous reader; records events[buf_idx]."""
        if not host_data.is_pinned():
            raise ValueError("prefetch: host_data must be pinned (see weight_store.PinnedWeightStore) for a real "
                             "async copy")
        if gpu_buffer.shape != host_data.shape:
            raise ValueError(f"prefetch: gpu_buffer shape {tuple(gpu_buffer.shape)} != host_data shape "
                             f"{tuple(host_data.shape)}")
        stream = self.streams[buf_idx]
        stream.wait_event(self.read_done_events[buf_idx])
        with torch.cuda.stream(stream):
            gpu_buffer.copy_(host_data, non_blocking=True)
        self.events[buf_idx].record(stream)

    def wait(self, buf_idx: int) -> None:
        """Current (compute) stream waits for buffer buf_idx's copy."""
        torch.cuda.current_stream(self.device).wait_event(self.events[buf_idx])

    def mark_read_done(self, buf_idx: int) -> None:
        """Record, on the current stream, that buffer buf_idx's reader has been issued."""
        self.read_done_events[buf_idx].record(torch.cuda.current_stream(self.device))

    def synchronize(self, buf_idx: int) -> None:
        """Host-blocking wait for buffer buf_idx's copy (timing / tests only)."""
        self.events[buf_idx].synchronize()
