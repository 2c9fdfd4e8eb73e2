"""Row gathers are byte-exact (mirrors the reference's tests/test_gather_rows.py):
staged (host memcpy + one H2D), naive (one copy per row) and device-driven
(SM gather from device memory or zero-copy from pinned host memory)."""
import pytest
import torch

import soinfer.ops as ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _matrix(rows, rb, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 256, (rows, rb), dtype=torch.uint8, generator=g).pin_memory()


@pytest.mark.parametrize("rows,rb,k", [(6144, 1024, 3072), (17408, 2560, 8704), (64, 13, 10), (16, 1024, 0)])
def test_staged_and_naive_match_index_select(rows, rb, k):
    m = _matrix(rows, rb, rows)
    idx = torch.randperm(rows, generator=torch.Generator().manual_seed(1))[:k].to(torch.int64)
    expected = m.index_select(0, idx)
    staging = torch.empty(max(k * rb, 1), dtype=torch.uint8).pin_memory()
    dst = torch.zeros(max(k * rb, 1), dtype=torch.uint8, device=DEV)
    ops.gather_rows_staged(m, idx, staging, dst)
    torch.cuda.synchronize()
    assert torch.equal(dst[: k * rb].view(k, rb).cpu(), expected)
    dst2 = torch.zeros_like(dst)
    ops.gather_rows_naive(m, idx, dst2)
    torch.cuda.synchronize()
    assert torch.equal(dst2, dst)


@pytest.mark.parametrize("pinned_source", [False, True])
def test_device_gather(pinned_source):
    rows, rb, k = 6144, 1024, 3072
    m = _matrix(rows, rb, 7)
    src = m if pinned_source else m.to(DEV)
    idx = torch.randperm(rows, generator=torch.Generator().manual_seed(2))[:k]
    dst = torch.zeros(k * rb, dtype=torch.uint8, device=DEV)
    ops.gather_rows_device(src, idx.int().to(DEV), dst)
    torch.cuda.synchronize()
    assert torch.equal(dst.view(k, rb).cpu(), m.index_select(0, idx))


def test_gather_rejects_bad_inputs():
    m = _matrix(8, 16)
    dst = torch.zeros(64, dtype=torch.uint8, device=DEV)
    with pytest.raises(RuntimeError):  # pageable (not pinned) source
        ops.gather_rows_naive(torch.zeros(8, 16, dtype=torch.uint8), torch.tensor([0, 1]), dst)
    with pytest.raises(RuntimeError):
        ops.gather_rows_naive(m, torch.tensor([0, 99]), dst)
    with pytest.raises(RuntimeError):
        ops.gather_rows_naive(m, torch.tensor([0, 1], dtype=torch.int32), dst)
    with pytest.raises(RuntimeError):
        ops.gather_rows_staged(m, torch.arange(8), torch.empty(8, dtype=torch.uint8).pin_memory(), dst)
