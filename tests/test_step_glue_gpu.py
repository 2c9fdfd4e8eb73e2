"""The graph decode step's device-side token bookkeeping
(soinfer_decode_step_embed / soinfer_decode_step_advance) against the torch
statements it replaces: x = embed[ids[pos]]; ids[pos + 1] = next unless pos + 1
is a prompt position; pos += 1.  Out-of-range positions and token ids write
nothing."""
import pytest
import torch

from soinfer import _C

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("hidden", [2048, 5120, 100])  # 16-byte pieces, and the scalar path
def test_step_embed_reads_the_row_of_the_token_at_pos(hidden):
    g = torch.Generator().manual_seed(hidden)
    vocab = 300
    embed = torch.randn(vocab, hidden, generator=g).half().cuda()
    ids = torch.randint(0, vocab, (40,), generator=g, dtype=torch.int32).cuda()
    x = torch.empty(hidden, dtype=torch.float16, device="cuda")
    for p in (0, 7, 39):
        pos = torch.tensor([p], dtype=torch.int32, device="cuda")
        _C.decode_step_embed(embed, ids, pos, x)
        assert torch.equal(x, embed[ids[p].long()])


def test_step_embed_out_of_range_writes_nothing():
    embed = torch.randn(10, 256).half().cuda()
    ids = torch.tensor([3, 12, -1, 4], dtype=torch.int32, device="cuda")  # ids 12 and -1 are outside the vocab
    x = torch.full((256,), 7.0, dtype=torch.float16, device="cuda")
    for p in (1, 2, 4, -1):  # bad token ids, then positions outside ids
        _C.decode_step_embed(embed, ids, torch.tensor([p], dtype=torch.int32, device="cuda"), x)
    torch.cuda.synchronize()
    assert bool((x == 7.0).all())


def _reference_advance(ids, pos, prompt_len, nxt):
    at = (pos + 1).long()
    keep = (pos + 1) < prompt_len
    ids.index_copy_(0, at, torch.where(keep, ids.index_select(0, at), nxt))
    pos.add_(1)


def test_step_advance_matches_the_torch_statements():
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, 1000, (33,), generator=g, dtype=torch.int32).cuda()
    ref_ids = ids.clone()
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    ref_pos = pos.clone()
    prompt_len = torch.tensor([9], dtype=torch.int32, device="cuda")
    for step in range(32):  # through the prompt, then generated tokens, up to the last slot
        nxt = torch.tensor([1000 + step], dtype=torch.int32, device="cuda")
        _C.decode_step_advance(ids, pos, prompt_len, nxt)
        _reference_advance(ref_ids, ref_pos, prompt_len, nxt)
        assert torch.equal(ids, ref_ids) and torch.equal(pos, ref_pos)
    assert int(pos) == 32
    nxt = torch.tensor([5], dtype=torch.int32, device="cuda")
    _C.decode_step_advance(ids, pos, prompt_len, nxt)  # pos + 1 == len(ids): nothing
    assert int(pos) == 32 and torch.equal(ids, ref_ids)


def test_step_ops_check_their_arguments():
    embed = torch.randn(10, 64).half().cuda()
    ids = torch.zeros(4, dtype=torch.int32, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError):
        _C.decode_step_embed(embed, ids.long(), pos, torch.empty(64, dtype=torch.float16, device="cuda"))
    with pytest.raises(RuntimeError):
        _C.decode_step_embed(embed, ids, pos, torch.empty(32, dtype=torch.float16, device="cuda"))
    with pytest.raises(RuntimeError):
        _C.decode_step_advance(ids, pos, pos, torch.zeros(2, dtype=torch.int32, device="cuda"))
