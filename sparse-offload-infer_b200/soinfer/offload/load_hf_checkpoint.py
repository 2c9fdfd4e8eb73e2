"""Quantize-on-load of HF safetensors checkpoints into the pinned arena
(reference python/soinfer/offload/load_hf_checkpoint.py:32-148).

Each decoder-layer linear weight is read one tensor at a time, quantized to
group-wise INT4 (min-max scales) and AWQ-packed, registered in the arena, and
its fp32 scales kept resident on the GPU.  With include_down_proj_t the
down_proj is also stored transposed ([intermediate, hidden]) so DIP can
select its rows.  Quantization can run on the GPU: one fused quantize + pack
kernel (soinfer_quantize_pack_int4), bit-exact with the CPU quantizer --
unlike torch's GPU path, whose division by a scalar multiplies by the
reciprocal and can move a scale by one ulp.

save_quantized / load_quantized serialize the quantized arena (raw packed
bytes + fp32 scales + a JSON index), so a model is quantized once and later
loads are one sequential read into the pinned arena.
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
    bits: int = 4        # 4: group-wise INT4 (AWQ-packed rows); 8: INT8 rows (one int8 per value), per-channel scales


def quantize_and_pack(w: torch.Tensor, group_size: int, device=None) -> tuple[torch.Tensor, torch.Tensor, int]:
    """w [N, K] -> (packed uint8 [N, ceil(Kp/8)*4] on CPU, scale fp32 [N, G], packed_k).
    On a CUDA device (and a power-of-two group size <= 256) the fused kernel
    does it in one pass; otherwise the reference's torch path on the CPU."""
    src = w.to(device) if device is not None else w
    if src.is_cuda and group_size in (8, 16, 32, 64, 128, 256):
        from .. import _C

        if src.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            src = src.float()
        packed, scale, packed_k = _C.quantize_pack_int4(src.contiguous(), group_size)
        return packed.cpu(), scale, packed_k
    qt = formats.quantize(src.cpu().float(), formats.QuantConfig(bits=4, granularity="group", group_size=group_size))
    packed, packed_k = pack.pack_int4(qt.qweight)
    scale = qt.scale.contiguous()
    return packed, scale.to(device) if device is not None else scale, packed_k


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


# --------------------------------------------------------------- serialized arena
ARENA_FORMAT = "soinfer-b200-int4-arena-v1"


def save_quantized(path: str, store: PinnedWeightStore, matrices: dict[str, LoadedMatrix], group_size: int) -> None:
    """Writes path/arena.bin (the used arena bytes, registration order),
    path/scales.bin (every matrix's fp32 scales, same order) and
    path/index.json (format, group size, per matrix: name, arena offset,
    rows, row bytes, n, k, packed_k, scale columns, scale offset)."""
    os.makedirs(path, exist_ok=True)
    entries, soff = [], 0
    with open(os.path.join(path, "scales.bin"), "wb") as fs:
        for name, m in sorted(matrices.items(), key=lambda kv: kv[1].handle.offset):
            sc = m.scale.detach().to("cpu", torch.float32).contiguous()
            fs.write(sc.numpy().tobytes())
            entries.append({"name": name, "offset": m.handle.offset, "num_rows": m.handle.num_rows,
                            "row_nbytes": m.handle.row_nbytes, "n": m.n, "k": m.k, "packed_k": m.packed_k,
                            "scale_cols": int(sc.shape[1]), "scale_offset": soff})
            soff += sc.numel() * 4
    with open(os.path.join(path, "arena.bin"), "wb") as fa:
        fa.write(store.arena[:store.bytes_used].numpy().tobytes())
    with open(os.path.join(path, "index.json"), "w") as fi:
        json.dump({"format": ARENA_FORMAT, "group_size": group_size, "arena_bytes": store.bytes_used,
                   "matrices": entries}, fi)


def load_quantized(path: str, device=None, pin: bool = True):
    """Inverse of save_quantized: (store, {name: LoadedMatrix}, group_size);
    the arena is read straight into the (pinned) host allocation, the scales
    go to `device`."""
    import numpy as np

    with open(os.path.join(path, "index.json")) as fi:
        idx = json.load(fi)
    if idx.get("format") != ARENA_FORMAT:
        raise ValueError(f"{path}: not a {ARENA_FORMAT} directory")
    store = PinnedWeightStore(idx["arena_bytes"], pin=pin)
    with open(os.path.join(path, "arena.bin"), "rb") as fa:
        if fa.readinto(memoryview(store.arena.numpy())) != idx["arena_bytes"]:
            raise ValueError(f"{path}/arena.bin is shorter than its index says")
    scales = np.fromfile(os.path.join(path, "scales.bin"), dtype=np.float32)
    matrices = {}
    for e in idx["matrices"]:
        h = store.adopt(e["name"], e["offset"], e["num_rows"], e["row_nbytes"])
        n_sc = e["num_rows"] * e["scale_cols"]
        sc = torch.from_numpy(scales[e["scale_offset"] // 4:e["scale_offset"] // 4 + n_sc].copy())
        sc = sc.view(e["num_rows"], e["scale_cols"])
        matrices[e["name"]] = LoadedMatrix(h, sc.to(device) if device is not None else sc, e["packed_k"], e["n"],
                                           e["k"])
    return store, matrices, idx["group_size"]
