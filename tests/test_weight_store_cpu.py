"""The pinned weight arena's host behaviour (reference
python/soinfer/offload/weight_store.py:26-117 and its tests/test_offload.py),
on pageable memory so it runs without a GPU: registration order fixes the
layout, views return the registered bytes, selected rows gather exactly, and
misuse raises the reference's error types (ValueError / IndexError)."""
import pytest
import torch

from soinfer.offload.weight_store import PinnedWeightStore


def _mat(rows, rb, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 256, (rows, rb), generator=g, dtype=torch.uint8)


def test_register_and_views_round_trip():
    store = PinnedWeightStore(4096, pin=False)
    a, b = _mat(8, 64, 1), _mat(5, 128, 2)
    ha, hb = store.register("a", a), store.register("b", b)
    assert torch.equal(store.matrix_view(ha), a) and torch.equal(store.matrix_view(hb), b)
    assert (ha.offset, hb.offset) == (0, 8 * 64) and store.bytes_used == 8 * 64 + 5 * 128
    for r in range(8):
        assert torch.equal(store.row_view(ha, r), a[r])
    rows = torch.tensor([4, 0, 4, 2])
    assert torch.equal(store.rows_view(hb, rows), b[rows])
    assert store.handle("b") == hb and hb.nbytes == 5 * 128
    # writing one matrix's span leaves the other untouched
    store.matrix_view(ha).zero_()
    assert torch.equal(store.matrix_view(hb), b)


def test_misuse_raises_reference_errors():
    store = PinnedWeightStore(1024, pin=False)
    h = store.register("w", _mat(4, 64, 3))
    with pytest.raises(ValueError, match="already registered"):
        store.register("w", _mat(1, 64, 4))
    with pytest.raises(ValueError, match="overflow"):
        store.register("big", _mat(16, 64, 5))
    with pytest.raises(ValueError, match="2D uint8"):
        store.register("f", torch.zeros(4, 4))
    with pytest.raises(IndexError, match="out of range"):
        store.row_view(h, 4)
    with pytest.raises(IndexError):
        store.row_view(h, -1)
    with pytest.raises(ValueError):
        PinnedWeightStore(0, pin=False)


def test_adopt_spans_in_order_only():
    store = PinnedWeightStore(1024, pin=False)
    store.arena[:256] = 7
    h = store.adopt("x", 0, 4, 64)
    assert torch.equal(store.matrix_view(h), torch.full((4, 64), 7, dtype=torch.uint8))
    with pytest.raises(ValueError, match="overlaps"):
        store.adopt("y", 128, 1, 64)  # before the end of the previous span
    with pytest.raises(ValueError, match="overlaps or leaves"):
        store.adopt("z", 1000, 1, 64)  # past the arena
