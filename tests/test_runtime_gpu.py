"""Decoder layers and decode loops (soinfer.runtime.generate) on the GPU:

* a dense layer against a float64 restatement composed from the oracle
  (rmsnorm, GEMVs, q/k norm, RoPE, GQA attention, SwiGLU), with fp16 rounding
  at the same op boundaries as the reference path;
* the DIP MLP block inside a layer against the oracle's dip_mlp_block,
  evaluated on the layer's own gate vector (so selection is compared on
  identical inputs);
* cache-aware DIP bit-identical to DIP (reference
  tests/test_m8_cached_dip_pipeline.py:103-138), for empty, partial and full
  caches;
* HBM-resident weights bit-identical to pinned-arena streaming;
* the generate loops, calibration and miss-byte accounting."""
import numpy as np
import pytest
import torch

from oracle import reference_port as port
from soinfer import ops
from soinfer.offload.hot_cache import HotCache, StaticFrequencyPolicy
from soinfer.runtime import generate as gen
from soinfer.runtime.loader import Architecture, synthetic_streaming_model
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu

ARCH = Architecture(num_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                    num_key_value_heads=2, head_dim=128, vocab_size=512)
DIP_K = 256


@pytest.fixture(scope="module")
def models():
    resident = synthetic_streaming_model(ARCH, seed=3, resident=True, offload=True)
    streamed = synthetic_streaming_model(ARCH, seed=3, resident=False, offload=True)
    return resident, streamed


def _np(t):
    return t.detach().cpu().numpy()


def _packed(model, layer, suffix):
    m = model.matrix(layer, suffix)
    return _np(model.weight_source(m)), _np(m.scale), m


def _layer_oracle_attention(model, layer, x, pos, kc, vc):
    """float64 restatement of the attention half; returns (h2, h3) fp16 numpy and updates kc / vc."""
    g, eps = model.group_size, model.rms_norm_eps
    NQ, NKV, HD, H = model.num_attention_heads, model.num_key_value_heads, model.head_dim, model.hidden_size
    norms = {k: _np(v) for k, v in model.layer_norms[layer].items()}

    def gemv(suffix, v, K):
        p, s, _ = _packed(model, layer, suffix)
        return port.gemv_w4a16(p, s, v, K, g).astype(np.float16)

    h = port.rmsnorm(x[None], norms["input_layernorm"], eps)[0]
    q = port.rmsnorm(gemv("self_attn.q_proj.weight", h, H).reshape(NQ, HD), norms["q_norm"], eps)
    k = port.rmsnorm(gemv("self_attn.k_proj.weight", h, H).reshape(NKV, HD), norms["k_norm"], eps)
    v = gemv("self_attn.v_proj.weight", h, H).reshape(NKV, HD)
    cos_v, sin_v = (_np(t) for t in ops.precompute_rope_cos_sin(HD, model.rope_theta, pos, device="cuda"))
    q, k = port.rope(q, cos_v, sin_v), port.rope(k, cos_v, sin_v)
    kc[:, pos], vc[:, pos] = k, v
    attn = port.decode_attention(q, kc, vc, pos + 1).astype(np.float16).reshape(-1)
    o = gemv("self_attn.o_proj.weight", attn, NQ * HD)
    h2 = (x.astype(np.float32) + o.astype(np.float32)).astype(np.float16)
    return h2, port.rmsnorm(h2[None], norms["post_attention_layernorm"], eps)[0]


def test_dense_layer_matches_oracle(models):
    model = models[0]
    H, I, g = model.hidden_size, ARCH.intermediate_size, model.group_size
    kcs, vcs = gen._kv_caches(model, 16)
    kcn = [np.zeros(tuple(kcs[0].shape), np.float16) for _ in range(2)]
    vcn = [np.zeros(tuple(vcs[0].shape), np.float16) for _ in range(2)]
    pipe = gen.WeightPipeline(model)
    x = model.embed_tokens[7]
    xn = _np(x)
    for pos in range(3):
        for layer in range(model.num_layers):
            y = gen.run_decoder_layer_streaming(pipe, model, layer, x, pos, kcs[layer], vcs[layer])
            h2, h3 = _layer_oracle_attention(model, layer, xn, pos, kcn[layer], vcn[layer])
            gp, gs, _ = _packed(model, layer, "mlp.gate_proj.weight")
            up, us, _ = _packed(model, layer, "mlp.up_proj.weight")
            dp, ds, _ = _packed(model, layer, "mlp.down_proj.weight")
            gate = port.gemv_w4a16(gp, gs, h3, H, g).astype(np.float16)
            upv = port.gemv_w4a16(up, us, h3, H, g).astype(np.float16)
            mh = (port.silu(gate.astype(np.float32)) * upv.astype(np.float32)).astype(np.float16)
            ref = (h2.astype(np.float32) + port.gemv_w4a16(dp, ds, mh, I, g).astype(np.float16)).astype(np.float16)
            # one token through a whole layer: a few fp16 roundings may land differently
            assert_close(y, ref.astype(np.float64), f"dense layer {layer} pos {pos}", max_abs=None, rel_l2=3e-3)
            x, xn = y, _np(y)


def test_dip_mlp_block_matches_oracle(models):
    model = models[0]
    H, g = model.hidden_size, model.group_size
    x = model.embed_tokens[11]
    kc1, vc1 = gen._kv_caches(model, 8)
    kc2, vc2 = gen._kv_caches(model, 8)
    bufs = gen.DipBuffers.make(model, DIP_K)
    y = gen.run_decoder_layer_dip(gen.WeightPipeline(model, gen.DIP_DENSE_SUFFIXES), model, 0, x, 0, kc1[0], vc1[0],
                                  DIP_K, bufs)
    p2 = gen.WeightPipeline(model, gen.DIP_DENSE_SUFFIXES)
    h2, h3 = gen._attention_block(p2, model, 0, x, 0, kc2[0], vc2[0])
    gate = p2.next_gemv(h3)
    gp, gs, _ = _packed(model, 0, "mlp.gate_proj.weight")
    up, us, _ = _packed(model, 0, "mlp.up_proj.weight")
    dt, dts, _ = _packed(model, 0, gen.DOWN_PROJ_T_SUFFIX)
    blk = port.dip_mlp_block(_np(h3), (gp, gs), (up, us), (dt, dts), DIP_K, g, H, gate_out=_np(gate))
    ref = (_np(h2).astype(np.float32) + blk["y"].astype(np.float16)).astype(np.float16)
    assert_close(y, ref.astype(np.float64), "dip layer", max_abs=None)
    sel = ops.topk_threshold_select(gate.float().abs(), DIP_K)
    assert np.array_equal(_np(sel), blk["idx"])


def _caches(model, hot):
    return [HotCache.build(model, layer, hot) for layer in range(model.num_layers)]


@pytest.mark.parametrize("cache_size", [0, 100, ARCH.intermediate_size])
def test_cached_dip_bit_identical_to_dip(models, cache_size):
    model = models[0]
    freq = torch.arange(ARCH.intermediate_size).flip(0).tolist()  # any ranking
    caches = _caches(model, StaticFrequencyPolicy(freq, cache_size).hot_list)
    bufs = gen.DipBuffers.make(model, DIP_K)
    pa, pb = (gen.WeightPipeline(model, gen.DIP_DENSE_SUFFIXES) for _ in range(2))
    kca, vca = gen._kv_caches(model, 8)
    kcb, vcb = gen._kv_caches(model, 8)
    miss = torch.zeros(model.num_layers, dtype=torch.int64, device="cuda")
    xa = xb = model.embed_tokens[5]
    for pos in range(3):
        for layer in range(model.num_layers):
            xa = gen.run_decoder_layer_dip(pa, model, layer, xa, pos, kca[layer], vca[layer], DIP_K, bufs)
            xb = gen.run_decoder_layer_cached_dip(pb, model, layer, xb, pos, kcb[layer], vcb[layer], DIP_K, bufs,
                                                  caches, miss)
            assert torch.equal(xa, xb), f"cached DIP differs at pos {pos} layer {layer}"
    miss = miss.cpu().tolist()
    if cache_size == ARCH.intermediate_size:
        assert miss == [0, 0]
    elif cache_size == 0:
        assert miss == [3 * DIP_K] * 2
    else:
        assert all(0 < m < 3 * DIP_K for m in miss)


def test_resident_equals_streamed(models):
    res, st = models
    res.batch_gemvs = False  # same GEMV kernel on both sides: only where the weights live differs
    prompt = [1, 2, 3, 4]
    assert gen.generate_streaming(res, prompt, 4, max_seq_len=16) == gen.generate_streaming(st, prompt, 4,
                                                                                              max_seq_len=16)
    assert gen.generate_dip(res, prompt, 4, DIP_K, max_seq_len=16) == gen.generate_dip(st, prompt, 4, DIP_K,
                                                                                         max_seq_len=16)
    res.batch_gemvs = True


def test_generate_loops_and_calibration(models):
    model = models[0]
    prompt = [9, 8, 7]
    dense = gen.generate_streaming(model, prompt, 5, max_seq_len=16)
    dip = gen.generate_dip(model, prompt, 5, DIP_K, max_seq_len=16)
    assert len(dense) == len(dip) == 8 and dense[:3] == dip[:3] == prompt
    assert all(0 <= t < ARCH.vocab_size for t in dense + dip)
    counts, trace = gen.calibrate_with_trace(model, [3, 1, 4, 1, 5, 9], DIP_K, max_seq_len=16)
    assert all(int(c.sum()) == 6 * DIP_K for c in counts)
    assert all(len(t) == 6 and all(len(s) == DIP_K for s in t) for t in trace)
    for layer in range(model.num_layers):  # the histogram is the trace's own counts
        hist = np.bincount(np.concatenate(trace[layer]), minlength=ARCH.intermediate_size)
        assert np.array_equal(hist, _np(counts[layer]))
    caches = _caches(model, StaticFrequencyPolicy(_np(counts[0]).tolist(), 128).hot_list)
    miss = [0] * model.num_layers
    cached = gen.generate_cached_dip(model, prompt, 5, DIP_K, caches, max_seq_len=16, miss_bytes=miss)
    assert cached == dip
    assert gen.dip_bytes_per_token(model, DIP_K) < gen.dip_bytes_per_token(model, DIP_K, dense=True)
    eos = dense[3]
    assert gen.generate_streaming(model, prompt, 5, eos_token_id=eos, max_seq_len=16) == prompt + [eos]
    with pytest.raises(ValueError):
        gen.generate_streaming(model, prompt, 20, max_seq_len=16)


def test_teacher_forced_nll_is_finite(models):
    model = models[0]
    pipe = gen.WeightPipeline(model)
    nll = gen.teacher_forced_nll(
        model, lambda m, li, x, p, kc, vc: gen.run_decoder_layer_streaming(pipe, m, li, x, p, kc, vc), [1, 2, 3, 4],
        max_seq_len=8)
    assert np.isfinite(nll) and nll > 0


def test_int8_per_channel_variant():
    """The INT8 per-channel weight format (the 14B benchmark's variant): a dense layer
    vs the float64 composition with the oracle's INT8 GEMV, and the graph
    decoder's tokens equal the eager loop's."""
    model = synthetic_streaming_model(ARCH, seed=8, include_dip=False, resident=True, offload=False, bits=8)
    assert all(m.bits == 8 and m.scale.shape[1] == 1 for m in model.matrices.values())
    H, I = model.hidden_size, ARCH.intermediate_size
    NQ, NKV, HD, eps = model.num_attention_heads, model.num_key_value_heads, model.head_dim, model.rms_norm_eps
    kcs, vcs = gen._kv_caches(model, 8)
    x = model.embed_tokens[3]
    y = gen.run_decoder_layer_streaming(gen.WeightPipeline(model), model, 0, x, 0, kcs[0], vcs[0])
    norms = {k: _np(v) for k, v in model.layer_norms[0].items()}

    def gemv(suffix, v):
        m = model.matrix(0, suffix)
        return port.gemv_w8a16(_np(model.resident[m.handle.name].view(torch.int8)), _np(m.scale), v,
                               m.k).astype(np.float16)

    xn = _np(x)
    h = port.rmsnorm(xn[None], norms["input_layernorm"], eps)[0]
    q = port.rmsnorm(gemv("self_attn.q_proj.weight", h).reshape(NQ, HD), norms["q_norm"], eps)
    k = port.rmsnorm(gemv("self_attn.k_proj.weight", h).reshape(NKV, HD), norms["k_norm"], eps)
    v = gemv("self_attn.v_proj.weight", h).reshape(NKV, HD)
    cos_v, sin_v = (_np(t) for t in ops.precompute_rope_cos_sin(HD, model.rope_theta, 0, device="cuda"))
    q, k = port.rope(q, cos_v, sin_v), port.rope(k, cos_v, sin_v)
    kc = np.zeros((NKV, 8, HD), np.float16)
    vc = np.zeros((NKV, 8, HD), np.float16)
    kc[:, 0], vc[:, 0] = k, v
    attn = port.decode_attention(q, kc, vc, 1).astype(np.float16).reshape(-1)
    h2 = (xn.astype(np.float32) + gemv("self_attn.o_proj.weight", attn).astype(np.float32)).astype(np.float16)
    h3 = port.rmsnorm(h2[None], norms["post_attention_layernorm"], eps)[0]
    g_, u_ = gemv("mlp.gate_proj.weight", h3), gemv("mlp.up_proj.weight", h3)
    mh = (port.silu(g_.astype(np.float32)) * u_.astype(np.float32)).astype(np.float16)
    ref = (h2.astype(np.float32) + gemv("mlp.down_proj.weight", mh).astype(np.float32)).astype(np.float16)
    assert_close(y, ref.astype(np.float64), "int8 dense layer", max_abs=None, rel_l2=3e-3)
    prompt = [5, 6, 7]
    assert gen.GraphDecoder(model, max_seq_len=32).generate(prompt, 4) == gen.generate_streaming(model, prompt, 4,
                                                                                                 max_seq_len=32)
