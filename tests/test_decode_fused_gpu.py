"""The fused decode step (soinfer_decode_layers_fused: every decoder layer in
one cooperative launch, phases separated by grid barriers) on the GPU.

It must reproduce the per-kernel CUDA-graph decode step bit for bit: the
same greedy tokens, and -- a stronger check, since every layer's K / V rows
depend on all earlier layers' outputs -- identical KV caches after the run.
Cases: the Qwen3-1.7B layer shape (16 q / 8 kv heads) and two other GQA
ratios (1 and 4), a down_proj long enough for the per-kernel batch to cut its
tiles into K-segments, prompts short enough for a single attention split and
long enough for many (the combine phase), and two generate calls in a row
(the barrier counters reset themselves)."""
import pytest
import torch

from soinfer import _C
from soinfer.runtime import generate as gen
from soinfer.runtime.loader import Architecture, synthetic_streaming_model

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("arch,prompt_len,n_new", [
    (Architecture(3, 2048, 6144, 16, 8, 128, 1024), 9, 12),     # 1.7B layer shape, one split
    (Architecture(2, 2048, 6144, 16, 8, 128, 1024), 300, 8),    # many splits: the combine phase
    (Architecture(2, 1024, 3072, 8, 8, 128, 512), 40, 8),       # one query head per kv head
    (Architecture(2, 2048, 5120, 16, 4, 128, 512), 70, 8),      # four query heads per kv head
    # down_proj K = 7168: the per-kernel batch cuts its 16-row tiles into K-segments,
    # the fused step does not -- the sums must not depend on the segmentation
    (Architecture(2, 1024, 7168, 8, 8, 128, 512), 40, 8),
])
def test_fused_step_equals_per_kernel_step(arch, prompt_len, n_new):
    model = synthetic_streaming_model(arch, seed=3, resident=True, offload=False, include_dip=False)
    g = torch.Generator().manual_seed(prompt_len)
    prompt = torch.randint(0, arch.vocab_size, (prompt_len,), generator=g).tolist()
    max_seq = 512
    ref = gen.GraphDecoder(model, max_seq_len=max_seq)
    fused = gen.GraphDecoder(model, max_seq_len=max_seq, fused=True)
    want = ref.generate(prompt, n_new)
    got = fused.generate(prompt, n_new)
    assert _C.device_errors() == 0
    assert got == want
    for li in range(arch.num_layers):
        assert torch.equal(fused.k_caches[li], ref.k_caches[li]), f"layer {li}: K cache differs"
        assert torch.equal(fused.v_caches[li], ref.v_caches[li]), f"layer {li}: V cache differs"
    assert fused.generate(prompt, n_new) == want  # again: the barrier counters were left at zero
    assert _C.device_errors() == 0
    torch.cuda.synchronize()
    spaces = [ws for key, ws in _C._workspaces.items() if key[0] == "fused_decode"]
    assert spaces and all(int(ws[:256].count_nonzero()) == 0 for ws in spaces), "barrier counters not reset"


def test_fused_step_rejects_unsupported_models():
    arch = Architecture(1, 256, 512, 4, 2, 64, 128)  # head_dim 64
    model = synthetic_streaming_model(arch, seed=0, resident=True, offload=False, include_dip=False)
    with pytest.raises(RuntimeError, match="UNSUPPORTED"):
        gen.GraphDecoder(model, max_seq_len=32, fused=True).generate([1, 2], 2)
    arch = Architecture(1, 256, 512, 4, 2, 128, 128)
    model = synthetic_streaming_model(arch, seed=0, resident=True, offload=False, include_dip=True)
    with pytest.raises(ValueError):
        gen.GraphDecoder(model, dip_k=128, max_seq_len=32, fused=True)
