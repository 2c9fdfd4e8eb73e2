"""Batched greedy decode (soinfer.runtime.batch.BatchDecoder, configs[4]'s
batch-8 decode) on the GPU: B sequences decoded together in one CUDA graph
per step give, sequence by sequence, the same greedy tokens as the batch-1
eager loop (generate_streaming) on each prompt -- with B = 8 and B = 3,
distinct prompts (so every sequence attends only to its own stacked KV cache),
and replayed twice."""
import pytest
import torch

from soinfer.runtime import generate as gen
from soinfer.runtime.batch import BatchDecoder
from soinfer.runtime.loader import Architecture, synthetic_streaming_model

pytestmark = pytest.mark.gpu

ARCH = Architecture(num_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                    num_key_value_heads=2, head_dim=128, vocab_size=512)


@pytest.fixture(scope="module")
def model():
    return synthetic_streaming_model(ARCH, seed=7, resident=True, offload=False, include_dip=False)


@pytest.mark.parametrize("batch", [8, 3])
def test_batch_tokens_equal_batch1_decode(model, batch):
    g = torch.Generator().manual_seed(batch)
    prompts = torch.randint(0, ARCH.vocab_size, (batch, 5), generator=g).tolist()
    n_new = 8
    ref = [gen.generate_streaming(model, p, n_new, max_seq_len=32) for p in prompts]
    bd = BatchDecoder(model, batch, max_seq_len=32)
    assert bd.generate(prompts, n_new) == ref
    tm = {}
    assert bd.generate(prompts, n_new, timings=tm) == ref  # the captured graph again
    assert tm["decode_ms"] > 0


def test_batch_decoder_checks():
    streamed = synthetic_streaming_model(ARCH, seed=7, resident=False, offload=True, include_dip=False)
    with pytest.raises(ValueError):
        BatchDecoder(streamed, 2)
    res = synthetic_streaming_model(ARCH, seed=7, resident=True, offload=False, include_dip=False)
    with pytest.raises(ValueError):
        BatchDecoder(res, 9)
    bd = BatchDecoder(res, 2, max_seq_len=16)
    with pytest.raises(ValueError):
        bd.generate([[1, 2], [3]], 2)
