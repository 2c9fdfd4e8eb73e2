"""Parity with Hugging Face Qwen3 (random init, no download), the reference's
own backbone tests ported onto this build's ops:

* one decoder layer assembled from soinfer.ops (rmsnorm, fp16 GEMVs, q/k
  head norm, RoPE, KV append, decode attention, SwiGLU) against
  transformers' Qwen3DecoderLayer at positions 0 / 5 / 100 -- relative error
  < 2e-2 on elements with |hf| > 0.05 (reference tests/test_layer_parity.py:
  91-118, same bound and threshold);
* greedy decode of a 4-layer Qwen3-1.7B-shaped model, token for token equal
  to HF's model.generate(do_sample=False) (reference
  tests/test_end_to_end.py:121-132, same seeds, start tokens and lengths).

fp16 weights throughout, as in the reference tests (the INT4 paths are pinned
by the oracle and by the reference runtime test)."""
import pytest
import torch

from soinfer import ops

pytestmark = pytest.mark.gpu
transformers = pytest.importorskip("transformers")
from transformers import Qwen3Config, Qwen3ForCausalLM  # noqa: E402
from transformers.models.qwen3 import modeling_qwen3 as qwen3_mod  # noqa: E402

DEV = "cuda"
MAX_REL_ERR = 2e-2
NEAR_ZERO_THRESHOLD = 0.05


def _config(num_hidden_layers: int) -> Qwen3Config:
    return Qwen3Config(hidden_size=2048, intermediate_size=6144, num_attention_heads=16, num_key_value_heads=8,
                       head_dim=128, num_hidden_layers=num_hidden_layers, rms_norm_eps=1e-6, rope_theta=1_000_000,
                       vocab_size=100, tie_word_embeddings=False)


def _theta(config) -> float:
    rp = getattr(config, "rope_parameters", None)
    return float(rp["rope_theta"]) if rp and "rope_theta" in rp else float(config.rope_theta)


def _layer(layer, config, x, pos, k_cache, v_cache):
    """One Qwen3 decoder layer for one token from this build's ops."""
    NQ, NKV, HD = config.num_attention_heads, config.num_key_value_heads, config.head_dim
    eps = config.rms_norm_eps
    attn, mlp = layer.self_attn, layer.mlp
    h = ops.rmsnorm(x.unsqueeze(0), layer.input_layernorm.weight, eps).squeeze(0)
    q = ops.gemv_fp16_v3(attn.q_proj.weight, h).view(NQ, HD)
    k = ops.gemv_fp16_v3(attn.k_proj.weight, h).view(NKV, HD)
    v = ops.gemv_fp16_v3(attn.v_proj.weight, h).view(NKV, HD)
    q = ops.qk_norm(q.contiguous(), attn.q_norm.weight, eps)
    k = ops.qk_norm(k.contiguous(), attn.k_norm.weight, eps)
    cos_v, sin_v = ops.precompute_rope_cos_sin(HD, _theta(config), pos, DEV)
    q = ops.apply_rope(q, cos_v, sin_v)
    k = ops.apply_rope(k, cos_v, sin_v)
    ops.kv_cache_append(k_cache, v_cache, k, v.contiguous(), pos)
    a = ops.decode_attention(q, k_cache, v_cache, pos + 1).reshape(NQ * HD).contiguous()
    h2 = x + ops.gemv_fp16_v3(attn.o_proj.weight, a)
    h3 = ops.rmsnorm(h2.unsqueeze(0), layer.post_attention_layernorm.weight, eps).squeeze(0)
    g = ops.gemv_fp16_v3(mlp.gate_proj.weight, h3)
    u = ops.gemv_fp16_v3(mlp.up_proj.weight, h3)
    return h2 + ops.gemv_fp16_v3(mlp.down_proj.weight, ops.swiglu(g, u))


@pytest.mark.parametrize("pos", [0, 5, 100])
def test_decoder_layer_matches_huggingface(pos):
    torch.manual_seed(0)
    config = _config(1)
    layer = qwen3_mod.Qwen3DecoderLayer(config, layer_idx=0).to(DEV).half().eval()
    rotary = qwen3_mod.Qwen3RotaryEmbedding(config).to(DEV)
    x = torch.randn(1, 1, config.hidden_size, device=DEV, dtype=torch.float16)
    position_ids = torch.tensor([[pos]], device=DEV)
    cos, sin = rotary(x, position_ids)
    with torch.no_grad():
        hf = layer(x, attention_mask=None, position_ids=position_ids, past_key_values=None, use_cache=False,
                   position_embeddings=(cos, sin))
    hf = (hf[0] if isinstance(hf, tuple) else hf)[0, 0]
    # HF's layer sees this token alone: a one-entry cache, RoPE at pos (as the reference test builds it)
    kc = torch.zeros(config.num_key_value_heads, 1, config.head_dim, device=DEV, dtype=torch.float16)
    vc = torch.zeros_like(kc)
    mine = _layer_single(layer, config, x[0, 0].contiguous(), pos, kc, vc)
    diff = (mine.float() - hf.float()).abs()
    signal = hf.float().abs() > NEAR_ZERO_THRESHOLD
    rel = diff[signal] / hf.float().abs()[signal]
    assert rel.numel() > 0
    assert torch.all(rel < MAX_REL_ERR), f"pos={pos}: max relative error {rel.max().item():.4f}"


def _layer_single(layer, config, x, pos, k_cache, v_cache):
    """_layer with RoPE at `pos` but the token stored at cache slot 0 of a
    one-entry cache (HF's layer called without a cache sees no earlier
    tokens)."""
    NQ, NKV, HD = config.num_attention_heads, config.num_key_value_heads, config.head_dim
    eps = config.rms_norm_eps
    attn, mlp = layer.self_attn, layer.mlp
    h = ops.rmsnorm(x.unsqueeze(0), layer.input_layernorm.weight, eps).squeeze(0)
    q = ops.qk_norm(ops.gemv_fp16_v3(attn.q_proj.weight, h).view(NQ, HD).contiguous(), attn.q_norm.weight, eps)
    k = ops.qk_norm(ops.gemv_fp16_v3(attn.k_proj.weight, h).view(NKV, HD).contiguous(), attn.k_norm.weight, eps)
    v = ops.gemv_fp16_v3(attn.v_proj.weight, h).view(NKV, HD).contiguous()
    cos_v, sin_v = ops.precompute_rope_cos_sin(HD, _theta(config), pos, DEV)
    q = ops.apply_rope(q, cos_v, sin_v)
    k = ops.apply_rope(k, cos_v, sin_v)
    ops.kv_cache_append(k_cache, v_cache, k, v, 0)
    a = ops.decode_attention(q, k_cache, v_cache, 1).reshape(NQ * HD).contiguous()
    h2 = x + ops.gemv_fp16_v3(attn.o_proj.weight, a)
    h3 = ops.rmsnorm(h2.unsqueeze(0), layer.post_attention_layernorm.weight, eps).squeeze(0)
    g = ops.gemv_fp16_v3(mlp.gate_proj.weight, h3)
    u = ops.gemv_fp16_v3(mlp.up_proj.weight, h3)
    return h2 + ops.gemv_fp16_v3(mlp.down_proj.weight, ops.swiglu(g, u))


def _generate(model, config, start_token: int, n_new: int):
    L, NKV, HD = config.num_hidden_layers, config.num_key_value_heads, config.head_dim
    kcs = [torch.zeros(NKV, n_new + 1, HD, device=DEV, dtype=torch.float16) for _ in range(L)]
    vcs = [torch.zeros_like(k) for k in kcs]
    tokens, cur = [start_token], start_token
    for pos in range(n_new):
        x = model.model.embed_tokens.weight[cur].contiguous()
        for li in range(L):
            x = _layer(model.model.layers[li], config, x, pos, kcs[li], vcs[li])
        xn = ops.rmsnorm(x.unsqueeze(0), model.model.norm.weight, config.rms_norm_eps).squeeze(0)
        cur = int(ops.lm_head_argmax(model.lm_head.weight, xn).item())
        tokens.append(cur)
    return tokens


@pytest.mark.parametrize("seed,start_token,n_new", [(0, 7, 6), (1, 49, 8), (2, 17, 8)])
def test_greedy_decode_matches_huggingface_token_for_token(seed, start_token, n_new):
    torch.manual_seed(seed)
    config = _config(4)
    model = Qwen3ForCausalLM(config).to(DEV).half().eval()
    with torch.no_grad():
        hf = model.generate(torch.tensor([[start_token]], device=DEV), max_new_tokens=n_new, do_sample=False,
                            min_new_tokens=n_new)[0].tolist()
    mine = _generate(model, config, start_token, n_new)
    assert mine == hf, f"token sequence diverged: hf={hf} mine={mine}"
