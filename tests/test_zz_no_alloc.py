"""soinfer_gemv_w4a16_sparse_accumulate_noalloc: the sparse 'down' GEMV with
its scratch in a static per-device array.  Two calls in a row must match the
workspace entry point (soinfer_gemv_w4a16_sparse_accumulate) bit for bit --
the second call checks that the first left the static tickets at zero.
Collected last on purpose (the static scratch persists across tests), and
self-contained so it also passes alone."""
import pytest
import torch

from soinfer import _C
from tests.helpers import fp16_randn, int4_weights

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(k, H, g, seed):
    packed, scale, _ = int4_weights(k, H, g, seed=seed)  # k selected rows of the transposed down_proj
    h = fp16_randn(k, seed + 1)
    return packed.to(DEV), scale.to(DEV), h.to(DEV)


@pytest.mark.parametrize("H,k,g", [(2048, 3072, 128), (5120, 1088, 128), (1000, 37, 8), (70000, 16, 8)])
def test_noalloc_matches_workspace_entry_twice(H, k, g):
    for call in range(2):
        Wq, s, h = _case(k, H, g, seed=100 * call + k)
        ref = _C.gemv_w4a16_sparse_accumulate(Wq, s, h, H, g)
        got = _C.gemv_w4a16_sparse_accumulate_noalloc(Wq, s, h, H, g)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"call {call}: noalloc result differs from the workspace entry point"


def test_noalloc_into_out_and_empty():
    Wq, s, h = _case(64, 2048, 128, seed=7)
    out = torch.full((2048,), 3.0, dtype=torch.float16, device=DEV)
    _C.gemv_w4a16_sparse_accumulate_noalloc(Wq, s, h, 2048, 128, out=out)
    assert torch.equal(out, _C.gemv_w4a16_sparse_accumulate(Wq, s, h, 2048, 128))
    empty = _C.gemv_w4a16_sparse_accumulate_noalloc(Wq[:0], s[:0], h[:0], 2048, 128)
    torch.cuda.synchronize()
    assert torch.count_nonzero(empty) == 0


def test_noalloc_rejects_shapes_beyond_the_static_scratch():
    H = 196_608  # 1536 x 128; one partial row alone is 786 KB > the 512 KiB scratch
    Wq, s, h = _case(1, H, 128, seed=3)
    assert Wq.size(1) == H // 2
    with pytest.raises(RuntimeError, match="scratch"):
        _C.gemv_w4a16_sparse_accumulate_noalloc(Wq, s, h, H, 128)
