"""Write-after-read ordering of the double-buffered weight stream (reference
python/soinfer/offload/stream_manager.py:40-51, the race its read_done
events fix; transfer test tests/test_offload.py:94).

A deliberately slow reader -- a bounded spin kernel of ~20 ms on the compute
stream (torch.cuda._sleep, which returns after a fixed cycle count) followed
by a copy of the buffer -- holds buffer 0 while the next prefetch into the
same buffer is issued at once on its side stream.  With the read_done guard
the copy engine waits for the reader, and the reader sees the first matrix;
with the guard disabled (a StreamManager whose prefetch skips that wait) the
second matrix lands under the sleeping reader and it sees that one instead --
so the test would catch a missing or misplaced guard."""
import pytest
import torch

from soinfer.offload.stream_manager import StreamManager

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
NBYTES = 32 << 20
SPIN_CYCLES = 40_000_000  # ~20 ms at ~2 GHz; the copy of 32 MB takes < 2 ms


class _NoGuard(StreamManager):
    """The stream manager without the write-after-read wait (the reference's
    pre-fix behaviour)."""

    def prefetch(self, buf_idx, gpu_buffer, host_data):
        stream = self.streams[buf_idx]
        with torch.cuda.stream(stream):
            gpu_buffer.copy_(host_data, non_blocking=True)
        self.events[buf_idx].record(stream)


def _run(manager_cls):
    first = torch.full((NBYTES,), 1, dtype=torch.uint8).pin_memory()
    second = torch.full((NBYTES,), 2, dtype=torch.uint8).pin_memory()
    buf = torch.empty(NBYTES, dtype=torch.uint8, device=DEV)
    sm = manager_cls(num_buffers=2, device=DEV)
    sm.prefetch(0, buf, first)
    sm.wait(0)
    torch.cuda._sleep(SPIN_CYCLES)  # the slow reader of buffer 0 ...
    seen = buf.clone()               # ... reads it after the spin
    sm.mark_read_done(0)
    sm.prefetch(0, buf, second)      # the next weight into the same buffer, issued right away
    sm.wait(0)
    after = buf.clone()
    torch.cuda.synchronize(DEV)
    return int(seen[0]), int(seen[-1]), int(after[0])


def test_next_prefetch_waits_for_the_slow_reader():
    s0, s1, after = _run(StreamManager)
    assert (s0, s1) == (1, 1), "the reader saw the next weight: the write-after-read guard did not hold"
    assert after == 2


def test_without_the_guard_the_race_shows():
    s0, s1, after = _run(_NoGuard)
    assert (s0, s1) == (2, 2), "expected the unguarded copy to land under the sleeping reader"
    assert after == 2
