"""Serialized quantized arena (soinfer.offload.load_hf_checkpoint
save_quantized / load_quantized) on the CPU: a round trip restores the arena
bytes, every matrix's span and its scales exactly, and a load refuses a
directory of another format."""
import json
import os

import numpy as np
import pytest
import torch

from soinfer.offload.load_hf_checkpoint import LoadedMatrix, load_quantized, quantize_and_pack, save_quantized
from soinfer.offload.weight_store import PinnedWeightStore
from soinfer.quant import formats, pack


def _store(shapes, g=128):
    gen = torch.Generator().manual_seed(4)
    mats = []
    total = 0
    for n, k in shapes:
        w = torch.randn(n, k, generator=gen) * 0.02
        p, s, pk = quantize_and_pack(w, g)  # CPU: the reference's torch path
        mats.append((p, s, pk, n, k))
        total += p.numel()
    store = PinnedWeightStore(total, pin=False)
    matrices = {}
    for i, (p, s, pk, n, k) in enumerate(mats):
        name = f"model.layers.{i // 2}.m{i}"
        matrices[name] = LoadedMatrix(store.register(name, p), s, pk, n, k)
    return store, matrices


def test_round_trip_is_exact(tmp_path):
    store, matrices = _store([(64, 256), (32, 300), (17, 128)])
    save_quantized(str(tmp_path), store, matrices, 128)
    st2, m2, g = load_quantized(str(tmp_path), pin=False)
    assert g == 128 and st2.bytes_used == store.bytes_used
    assert torch.equal(st2.arena[:st2.bytes_used], store.arena[:store.bytes_used])
    assert set(m2) == set(matrices)
    for name, m in matrices.items():
        n2 = m2[name]
        assert (n2.handle.offset, n2.handle.num_rows, n2.handle.row_nbytes) == (m.handle.offset, m.handle.num_rows,
                                                                                  m.handle.row_nbytes)
        assert (n2.n, n2.k, n2.packed_k) == (m.n, m.k, m.packed_k)
        assert torch.equal(n2.scale, m.scale)
        assert torch.equal(st2.matrix_view(n2.handle), store.matrix_view(m.handle))


def test_quantize_and_pack_cpu_is_the_reference_path():
    w = torch.randn(8, 300, generator=torch.Generator().manual_seed(1))
    p, s, pk = quantize_and_pack(w, 128)
    qt = formats.quantize(w, formats.QuantConfig(bits=4, granularity="group", group_size=128))
    assert torch.equal(p, pack.pack_int4(qt.qweight)[0]) and torch.equal(s, qt.scale) and pk == 384


def test_load_rejects_other_formats(tmp_path):
    with open(os.path.join(tmp_path, "index.json"), "w") as f:
        json.dump({"format": "something-else"}, f)
    with pytest.raises(ValueError):
        load_quantized(str(tmp_path), pin=False)
    store, matrices = _store([(16, 128)])
    save_quantized(str(tmp_path / "a"), store, matrices, 128)
    with open(tmp_path / "a" / "arena.bin", "r+b") as f:
        f.truncate(10)
    with pytest.raises(ValueError):
        load_quantized(str(tmp_path / "a"), pin=False)
