"""Device-position ops and the CUDA-graph decode step on the GPU: the RoPE
table rows equal precompute_rope_cos_sin bit for bit; rope / KV append at a
device position equal the host-position ops exactly; attention at a device
length (its split plan fixed for max_seq) matches the oracle and the host
form; GraphDecoder produces the same tokens as the eager generate loops."""
import numpy as np
import pytest
import torch

from oracle import reference_port as port
from soinfer import ops
from soinfer.runtime import generate as gen
from soinfer.runtime.loader import Architecture, synthetic_streaming_model
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("hd,theta", [(128, 1e6), (64, 1e4)])
def test_rope_table_rows_equal_per_position(hd, theta):
    cos_t, sin_t = ops.precompute_rope_table(hd, theta, 300, DEV)
    for p in (0, 1, 7, 150, 299):
        c, s = ops.precompute_rope_cos_sin(hd, theta, p, DEV)
        assert torch.equal(cos_t[p], c) and torch.equal(sin_t[p], s), f"position {p}"


def test_rope_and_kv_append_at_device_position():
    g = torch.Generator().manual_seed(0)
    nkv, max_seq, hd = 4, 64, 128
    cos_t, sin_t = ops.precompute_rope_table(hd, 1e6, max_seq, DEV)
    kc_a, vc_a = (torch.zeros(nkv, max_seq, hd, dtype=torch.float16, device=DEV) for _ in range(2))
    kc_b, vc_b = (torch.zeros(nkv, max_seq, hd, dtype=torch.float16, device=DEV) for _ in range(2))
    pos_dev = torch.zeros(1, dtype=torch.int32, device=DEV)
    for p in (0, 5, 63):
        x = torch.randn(8, hd, generator=g).half().to(DEV)
        k = torch.randn(nkv, hd, generator=g).half().to(DEV)
        v = torch.randn(nkv, hd, generator=g).half().to(DEV)
        pos_dev.fill_(p)
        a = ops.apply_rope(x.clone(), *ops.precompute_rope_cos_sin(hd, 1e6, p, DEV))
        b = ops.apply_rope_at(x.clone(), cos_t, sin_t, pos_dev)
        assert torch.equal(a, b)
        ops.kv_cache_append(kc_a, vc_a, k, v, p)
        ops.kv_cache_append_at(kc_b, vc_b, k, v, pos_dev)
        assert torch.equal(kc_a, kc_b) and torch.equal(vc_a, vc_b)
    pos_dev.fill_(max_seq)  # out of range: no write, no change
    before = kc_b.clone()
    ops.kv_cache_append_at(kc_b, vc_b, k, v, pos_dev)
    x = torch.randn(8, hd, generator=g).half().to(DEV)
    assert torch.equal(ops.apply_rope_at(x.clone(), cos_t, sin_t, pos_dev), x)
    torch.cuda.synchronize()
    assert torch.equal(before, kc_b)


@pytest.mark.parametrize("nq,nkv,hd,max_seq", [(16, 8, 128, 2048), (40, 8, 128, 4096), (4, 2, 64, 40)])
def test_decode_attention_at_device_length(nq, nkv, hd, max_seq):
    g = torch.Generator().manual_seed(nq + max_seq)
    kc = torch.randn(nkv, max_seq, hd, generator=g).half().to(DEV)
    vc = torch.randn(nkv, max_seq, hd, generator=g).half().to(DEV)
    q = torch.randn(nq, hd, generator=g).half().to(DEV)
    pos_dev = torch.zeros(1, dtype=torch.int32, device=DEV)
    for cur_len in sorted({1, 2, 17, max_seq // 3, max_seq - 1, max_seq}):
        pos_dev.fill_(cur_len - 1)
        got = ops.decode_attention_at(q, kc, vc, pos_dev)
        ref = port.decode_attention(q.cpu().numpy(), kc.cpu().numpy(), vc.cpu().numpy(), cur_len)
        assert_close(got, ref, f"attention_at len {cur_len}")
        assert_close(got, ops.decode_attention(q, kc, vc, cur_len).double(), f"attention_at vs host len {cur_len}")


ARCH = Architecture(num_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                    num_key_value_heads=2, head_dim=128, vocab_size=512)


@pytest.fixture(scope="module")
def model():
    return synthetic_streaming_model(ARCH, seed=5, resident=True, offload=False)


def test_graph_decoder_tokens_equal_eager(model):
    prompt = [3, 141, 59, 26]
    dense = gen.generate_streaming(model, prompt, 6, max_seq_len=64)
    dip = gen.generate_dip(model, prompt, 6, 256, max_seq_len=64)
    gd = gen.GraphDecoder(model, max_seq_len=64)
    assert gd.generate(prompt, 6) == dense
    assert gd.generate([7, 7], 5) == gen.generate_streaming(model, [7, 7], 5, max_seq_len=64)  # replay again
    gdip = gen.GraphDecoder(model, dip_k=256, max_seq_len=64)
    assert gdip.generate(prompt, 6) == dip


def test_graph_cached_dip_tokens_equal_graph_dip():
    """Cache-aware DIP inside the per-token CUDA graph: no host read of the
    miss count (the descriptors, the miss gather -- zero-copy from the pinned
    arena -- and the fused GEMVs all take it on the device), and the tokens
    equal graph DIP's bit for bit over 16 new tokens for an empty cache, a 20%
    Zipf(1.1) hot set and a full cache; the device miss counters match."""
    import copy

    from soinfer.offload.hot_cache import HotCache, StaticFrequencyPolicy

    I, dip_k = ARCH.intermediate_size, ARCH.intermediate_size // 2
    full = synthetic_streaming_model(ARCH, seed=6, resident=True, offload=True, include_dip=True)
    host = copy.copy(full)  # up_proj / down_proj_T read from the pinned arena
    host.resident = {n: t for n, t in full.resident.items()
                     if not (n.endswith("mlp.up_proj.weight") or n.endswith(gen.DOWN_PROJ_T_SUFFIX))}
    prompt, n_new = [3, 141, 59, 26], 16
    ref = gen.GraphDecoder(full, dip_k=dip_k, max_seq_len=64).generate(prompt, n_new)
    assert ref == gen.generate_dip(full, prompt, n_new, dip_k, max_seq_len=64)
    rng = np.random.default_rng(0)
    freq = np.empty(I, dtype=np.int64)
    freq[rng.permutation(I)] = (1e9 / np.arange(1, I + 1) ** 1.1).astype(np.int64)
    steps = len(prompt) + n_new - 1
    for frac in (0.0, 0.2, 1.0):
        hot = StaticFrequencyPolicy(freq.tolist(), round(frac * I)).hot_list
        caches = [HotCache.build(full, li, hot) for li in range(ARCH.num_layers)]
        gd = gen.GraphDecoder(host, dip_k=dip_k, max_seq_len=64, caches=caches)
        assert gd.generate(prompt, n_new) == ref, f"cached DIP tokens differ (cache fraction {frac})"
        counts = gd.miss_counts.cpu().tolist()
        if frac == 0.0:
            assert counts == [steps * dip_k] * ARCH.num_layers
        elif frac == 1.0:
            assert counts == [0] * ARCH.num_layers
        else:
            assert all(0 < c < steps * dip_k for c in counts)


def test_graph_decoder_needs_resident_weights():
    streamed = synthetic_streaming_model(ARCH, seed=5, resident=False, offload=True)
    with pytest.raises(ValueError):
        gen.GraphDecoder(streamed)
