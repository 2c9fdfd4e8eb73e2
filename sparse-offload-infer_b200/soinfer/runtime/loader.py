"""Model assembly (reference python/soinfer/runtime/loader.py:33-82).

* load_streaming_model: a HF checkpoint directory (config.json +
  safetensors) -> StreamingModel, decoder-layer linear weights quantized into
  the pinned arena (optionally also kept resident in HBM), embeddings / LM
  head / norms on the GPU.
* synthetic_streaming_model: the same structure with seeded random-init
  weights of a given architecture (no checkpoint needed) -- weights
  N(0, std) quantized to group-wise INT4 on the GPU, norms 1, embeddings
  N(0, embed_std).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass

import torch

from ..offload.load_hf_checkpoint import (DOWN_PROJ_T_SUFFIX, LINEAR_SUFFIXES, LoadedMatrix, load_quantized,
                                          packed_int4_bytes, quantize_and_pack, save_quantized, stream_load_layers)
from ..offload.weight_store import PinnedWeightStore, WeightHandle
from ..quant import formats, pack
from .generate import StreamingModel


def _load_small(model_dir: str, weight_map: dict[str, str], name: str, device) -> torch.Tensor:
    from safetensors import safe_open

    with safe_open(os.path.join(model_dir, weight_map[name]), framework="pt") as f:
        t = f.get_tensor(name)
    return t.to(dtype=torch.float16, device=device).contiguous()


def _rope_theta(cfg: dict) -> float:
    """RoPE base from config.json: the top-level rope_theta of older files, or
    rope_parameters.rope_theta as recent transformers write it."""
    if "rope_theta" in cfg:
        return float(cfg["rope_theta"])
    return float((cfg.get("rope_parameters") or {}).get("rope_theta", 10000.0))


def load_streaming_model(model_dir: str, group_size: int = 128, include_dip: bool = False,
                         resident: bool = False, device=None, arena_dir: str | None = None) -> StreamingModel:
    """Quantize every decoder layer's linear weights into a pinned INT4 arena
    (plus each down_proj transposed with include_dip), load embeddings, LM
    head and norms to the GPU as fp16.  resident=True also keeps every packed
    matrix in HBM (no streaming).  arena_dir: a serialized arena
    (save_quantized) -- loaded when it exists, written after quantizing when
    it does not."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with open(os.path.join(model_dir, "config.json")) as f:
        cfg = json.load(f)
    n_layers = cfg["num_hidden_layers"]
    if arena_dir is not None and os.path.exists(os.path.join(arena_dir, "index.json")):
        store, matrices, saved_g = load_quantized(arena_dir, device=device)
        if saved_g != group_size or (include_dip and not any(k.endswith(DOWN_PROJ_T_SUFFIX) for k in matrices)):
            raise ValueError(f"{arena_dir}: saved with group size {saved_g} / without the DIP transposes")
    else:
        store, matrices = stream_load_layers(model_dir, n_layers, group_size=group_size,
                                             include_down_proj_t=include_dip, quant_device=device)
        if arena_dir is not None:
            save_quantized(arena_dir, store, matrices, group_size)
    with open(os.path.join(model_dir, "model.safetensors.index.json")) as f:
        wm = json.load(f)["weight_map"]
    lm_name = "lm_head.weight" if "lm_head.weight" in wm else "model.embed_tokens.weight"  # tied embeddings
    norms = [{key: _load_small(model_dir, wm, f"model.layers.{i}.{path}.weight", device)
              for key, path in (("input_layernorm", "input_layernorm"),
                                ("post_attention_layernorm", "post_attention_layernorm"),
                                ("q_norm", "self_attn.q_norm"), ("k_norm", "self_attn.k_norm"))}
             for i in range(n_layers)]
    res = None
    if resident:
        res = {name: store.matrix_view(m.handle).to(device) for name, m in matrices.items()}
    return StreamingModel(
        store=store, matrices=matrices, num_layers=n_layers,
        embed_tokens=_load_small(model_dir, wm, "model.embed_tokens.weight", device),
        lm_head=_load_small(model_dir, wm, lm_name, device),
        final_norm=_load_small(model_dir, wm, "model.norm.weight", device),
        layer_norms=norms, hidden_size=cfg["hidden_size"], num_attention_heads=cfg["num_attention_heads"],
        num_key_value_heads=cfg["num_key_value_heads"],
        head_dim=cfg.get("head_dim", cfg["hidden_size"] // cfg["num_attention_heads"]),
        rms_norm_eps=cfg["rms_norm_eps"], rope_theta=_rope_theta(cfg), group_size=group_size, resident=res)


@dataclass(frozen=True)
class Architecture:
    num_layers: int
    hidden_size: int
    intermediate_size: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    vocab_size: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6


# the decode benchmark architectures (Qwen3-1.7B- and Qwen3-14B-shaped)
QWEN3_1_7B = Architecture(28, 2048, 6144, 16, 8, 128, 151936)
QWEN3_14B = Architecture(40, 5120, 17408, 40, 8, 128, 151936)


def _linear_shapes(arch: Architecture) -> dict[str, tuple[int, int]]:
    H, I, HD = arch.hidden_size, arch.intermediate_size, arch.head_dim
    return {
        "self_attn.q_proj.weight": (arch.num_attention_heads * HD, H),
        "self_attn.k_proj.weight": (arch.num_key_value_heads * HD, H),
        "self_attn.v_proj.weight": (arch.num_key_value_heads * HD, H),
        "self_attn.o_proj.weight": (H, arch.num_attention_heads * HD),
        "mlp.gate_proj.weight": (I, H),
        "mlp.up_proj.weight": (I, H),
        "mlp.down_proj.weight": (H, I),
    }


def synthetic_weights(arch: Architecture, seed: int, group_size: int, include_dip: bool, std: float, device,
                      bits: int = 4):
    """Yields (layer, suffix, packed uint8 CUDA, scale fp32 CUDA, packed_k, n, k) for every decoder
    linear weight in load order -- the seeded random-init matrices quantized to group-wise INT4 (the
    transposed down_proj right after its down_proj), or with bits=8 to per-channel INT8 (rows of int8
    values viewed as uint8, scale [N, 1]) -- then returns the generator for the embeddings."""
    gen = torch.Generator(device=device).manual_seed(seed)
    shapes = _linear_shapes(arch)
    for layer in range(arch.num_layers):
        for suffix in LINEAR_SUFFIXES:
            n, k = shapes[suffix]
            w = torch.randn(n, k, generator=gen, device=device) * std
            if bits == 8:
                qt = formats.quantize(w, formats.QuantConfig(bits=8, granularity="per_channel"))
                yield layer, suffix, qt.qweight.contiguous().view(torch.uint8), qt.scale.contiguous(), k, n, k
                del w
                continue
            yield _quantized(layer, suffix, w, group_size)
            if include_dip and suffix == "mlp.down_proj.weight":
                yield _quantized(layer, DOWN_PROJ_T_SUFFIX, w.t().contiguous(), group_size)
            del w
    return gen


def _quantized(layer, suffix, w, group_size):
    if w.is_cuda and group_size in (8, 16, 32, 64, 128, 256):
        from .. import _C

        packed, scale, packed_k = _C.quantize_pack_int4(w, group_size)  # one fused pass on the GPU
        return layer, suffix, packed, scale, packed_k, w.shape[0], w.shape[1]
    qt = formats.quantize(w, formats.QuantConfig(bits=4, granularity="group", group_size=group_size))
    packed, packed_k = pack.pack_int4(qt.qweight)
    return layer, suffix, packed.contiguous(), qt.scale.contiguous(), packed_k, w.shape[0], w.shape[1]


def synthetic_small_tensors(arch: Architecture, gen: torch.Generator, std: float, embed_std: float, device):
    """Norm weights (ones), embeddings N(0, embed_std), LM head N(0, std) -- drawn after the linear weights."""
    H = arch.hidden_size
    ones = torch.ones(H, dtype=torch.float16, device=device)
    norms = [{"input_layernorm": ones, "post_attention_layernorm": ones,
              "q_norm": torch.ones(arch.head_dim, dtype=torch.float16, device=device),
              "k_norm": torch.ones(arch.head_dim, dtype=torch.float16, device=device)}
             for _ in range(arch.num_layers)]
    embed = (torch.randn(arch.vocab_size, H, generator=gen, device=device) * embed_std).half()
    lm_head = (torch.randn(arch.vocab_size, H, generator=gen, device=device) * std).half()
    return norms, embed, lm_head, ones


def synthetic_streaming_model(arch: Architecture, seed: int = 0, group_size: int = 128, include_dip: bool = True,
                              resident: bool = True, offload: bool = True, std: float = 0.02,
                              embed_std: float = 1.0, device=None, bits: int = 4) -> StreamingModel:
    """Seeded random-init model of `arch`.  resident: packed matrices kept in
    HBM; offload: packed matrices also registered in the pinned arena (needed
    for streaming and for building hot caches from host memory).  bits=8: the
    INT8 per-channel variant (dense layers only: DIP reads INT4 rows)."""
    if not (resident or offload):
        raise ValueError("a model needs its weights resident, in the arena, or both")
    if bits not in (4, 8) or (bits == 8 and include_dip):
        raise ValueError("bits must be 4, or 8 without the DIP transposes")
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    shapes = _linear_shapes(arch)
    store = None
    if offload:
        total = 0
        for _layer in range(arch.num_layers):
            for suffix in LINEAR_SUFFIXES:
                total += packed_int4_bytes(*shapes[suffix], group_size) if bits == 4 else shapes[suffix][0] * shapes[
                    suffix][1]
                if include_dip and suffix == "mlp.down_proj.weight":
                    total += packed_int4_bytes(*shapes[suffix][::-1], group_size)
        store = PinnedWeightStore(total)
    matrices: dict[str, LoadedMatrix] = {}
    res: dict[str, torch.Tensor] | None = {} if resident else None
    weights = synthetic_weights(arch, seed, group_size, include_dip, std, device, bits=bits)
    while True:
        try:
            layer, suffix, packed, scale, packed_k, n, k = next(weights)
        except StopIteration as done:
            gen = done.value
            break
        name = f"model.layers.{layer}.{suffix}"
        if store is not None:
            handle = store.register(name, packed.cpu())
        else:
            handle = WeightHandle(name, -1, packed.shape[0], packed.shape[1])
        if res is not None:
            res[name] = packed
        matrices[name] = LoadedMatrix(handle, scale, packed_k, n, k, bits)
    norms, embed, lm_head, ones = synthetic_small_tensors(arch, gen, std, embed_std, device)
    return StreamingModel(store=store, matrices=matrices, num_layers=arch.num_layers, embed_tokens=embed,
                          lm_head=lm_head, final_norm=ones, layer_norms=norms, hidden_size=arch.hidden_size,
                          num_attention_heads=arch.num_attention_heads, num_key_value_heads=arch.num_key_value_heads,
                          head_dim=arch.head_dim, rms_norm_eps=arch.rms_norm_eps, rope_theta=arch.rope_theta,
                          group_size=group_size, resident=res)


__all__ = ["load_streaming_model", "synthetic_streaming_model", "synthetic_weights", "synthetic_small_tensors",
           "Architecture", "QWEN3_1_7B", "QWEN3_14B", "quantize_and_pack"]
