"""Quantize-on-load of HF safetensors checkpoints into the pinned arena
(reference python/soinfer/offload/load_hf_checkpoint.py:32-148).

Each decoder-layer linear weight is read one tensor at a time, quantized to
group-wise INT4 (min-max scales) and AWQ-packed, registered in the arena, and
its fp32 scales kept resident on the GPU.  With include_down_proj_t the
down_proj is also stored transposed ([intermediate, hidden]) so DIP can
select its rows.  Quantization can run on the GPU (torch ops, bit-identical
to the CPU result) to cut load time.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass

import torch

from ..quant import formats, pack
from .weight_store import PinnedWeightStore, WeightHandle

LINEAR_SUFFIXES = (
    "self_attn.q_proj.weight",
    "self_attn.k_proj.weight",
    "self_attn.v_proj.weight",
    "self_attn.o_proj.weight",
    "mlp.gate_proj.weight",
    "mlp.up_proj.weight",
    "mlp.down_proj.weight",
)
DOWN_PROJ_T_SUFFIX = "mlp.down_proj_T.weight"  # synthetic name: down_proj transposed for DIP row selection


@dataclass
class LoadedMatrix:
    handle: WeightHandle
    scale: torch.Tensor  # [N, num_groups] fp32, resident on the GPU
    packed_k: int
    n: int
    k: int


def quantize_and_pack(w: torch.Tensor, group_size: int, device=None) -> tuple[torch.Tensor, torch.Tensor, int]:
    """w [N, K] -> (packed uint8 [N, ceil(Kp/8)*4] on CPU, scale fp32 [N, G], packed_k)."""
    src = w.to(device) if device is not None else w
    qt = formats.quantize(src.float(), formats.QuantConfig(bits=4, granularity="group", group_size=group_size))
    packed, packed_k = pack.pack_int4(qt.qweight)
    return packed.cpu(), qt.scale.contiguous(), packed_k


def packed_int4_bytes(n: int, k: int, group_size: int = 8) -> int:
    kp = -(-k // group_size) * group_size
    return n * (-(-kp // 8) * 4)


def _weight_map(model_dir: str) -> dict[str, str]:
    with open(os.path.join(model_dir, "model.safetensors.index.json")) as f:
        return json.load(f)["weight_map"]


def plan_arena_bytes(model_dir: str, num_layers: int, suffixes: tuple[str, ...] = LINEAR_SUFFIXES,
                     transpose: bool = False, group_size: int = 8) -> int:
    """Arena size from the safetensors headers only (no tensor data read)."""
    from safetensors import safe_open

    wm = _weight_map(model_dir)
    shards: dict[str, object] = {}
    total = 0
    for layer in range(num_layers):
        for suffix in suffixes:
            name = f"model.layers.{layer}.{suffix}"
            if wm[name] not in shards:
                shards[wm[name]] = safe_open(os.path.join(model_dir, wm[name]), framework="pt")
            n, k = shards[wm[name]].get_slice(name).get_shape()
            if transpose:
                n, k = k, n
            total += packed_int4_bytes(n, k, group_size)
    return total


def stream_load_layers(model_dir: str, num_layers: int, group_size: int = 128, log_every: int = 8,
                       include_down_proj_t: bool = False, quant_device=None):
    """Quantize + register every layer's linear weights one tensor at a time.
    Returns (store, {"model.layers.{i}.{suffix}": LoadedMatrix})."""
    from safetensors import safe_open

    wm = _weight_map(model_dir)
    total = plan_arena_bytes(model_dir, num_layers, group_size=group_size)
    if include_down_proj_t:
        total += plan_arena_bytes(model_dir, num_layers, ("mlp.down_proj.weight",), transpose=True,
                                  group_size=group_size)
    store = PinnedWeightStore(total)
    matrices: dict[str, LoadedMatrix] = {}
    shards: dict[str, object] = {}
    for layer in range(num_layers):
        for suffix in LINEAR_SUFFIXES:
            name = f"model.layers.{layer}.{suffix}"
            if wm[name] not in shards:
                shards[wm[name]] = safe_open(os.path.join(model_dir, wm[name]), framework="pt")
            w = shards[wm[name]].get_tensor(name)
            n, k = w.shape
            packed, scale, pk = quantize_and_pack(w, group_size, quant_device)
            matrices[name] = LoadedMatrix(store.register(name, packed), scale.cuda(), pk, n, k)
            if include_down_proj_t and suffix == "mlp.down_proj.weight":
                wt = w.t().contiguous()
                packed_t, scale_t, pk_t = quantize_and_pack(wt, group_size, quant_device)
                name_t = f"model.layers.{layer}.{DOWN_PROJ_T_SUFFIX}"
                matrices[name_t] = LoadedMatrix(store.register(name_t, packed_t), scale_t.cuda(), pk_t, k, n)
            del w
        if log_every and ((layer + 1) % log_every == 0 or layer == num_layers - 1):
            print(f"  loaded layer {layer + 1}/{num_layers} ({store.bytes_used / 1e9:.2f} GB in arena)")
    return store, matrices
