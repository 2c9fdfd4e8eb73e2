"""Attention-side parity on the GPU (mirrors the reference's
tests/test_m5_kernels.py and test_m2_kernels.py): split-KV GQA decode
attention vs the float64 oracle across context lengths and head layouts,
KV-cache append, RoPE and RMSNorm / QK-norm, including HF Qwen3 when
transformers is importable."""
import math

import numpy as np
import pytest
import torch

import soinfer.ops as ops
from oracle import reference_port as port
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("nq,nkv,hd,max_seq,cur_len", [
    (16, 8, 128, 512, 1), (16, 8, 128, 512, 17), (16, 8, 128, 512, 300), (16, 8, 128, 2048, 2048),
    (40, 8, 128, 4096, 4096), (40, 8, 128, 4096, 77), (8, 8, 64, 128, 100), (12, 4, 96, 64, 63), (6, 2, 256, 40, 33),
    (32, 4, 128, 1024, 999)])
def test_decode_attention_matches_oracle(nq, nkv, hd, max_seq, cur_len):
    torch.manual_seed(4)
    q = torch.randn(nq, hd, dtype=torch.float16)
    kc = torch.randn(nkv, max_seq, hd, dtype=torch.float16)
    vc = torch.randn(nkv, max_seq, hd, dtype=torch.float16)
    out = ops.decode_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), cur_len)
    ref = port.decode_attention(q.numpy(), kc.numpy(), vc.numpy(), cur_len)
    assert_close(out, ref, f"attn[{nq}/{nkv} hd{hd} len{cur_len}]")


def test_decode_attention_after_kv_append():
    torch.manual_seed(5)
    nq, nkv, hd, max_seq = 16, 8, 128, 32
    kc = torch.zeros(nkv, max_seq, hd, device=DEV, dtype=torch.float16)
    vc = torch.zeros_like(kc)
    for pos in range(5):
        ops.kv_cache_append(kc, vc, torch.randn(nkv, hd, device=DEV, dtype=torch.float16),
                            torch.randn(nkv, hd, device=DEV, dtype=torch.float16), pos)
    q = torch.randn(nq, hd, device=DEV, dtype=torch.float16)
    out = ops.decode_attention(q, kc, vc, 5)
    assert_close(out, port.decode_attention(q.cpu().numpy(), kc.cpu().numpy(), vc.cpu().numpy(), 5), "attn+append")


def test_decode_attention_rejects_bad_arguments():
    q = torch.randn(15, 128, device=DEV, dtype=torch.float16)
    kc = torch.randn(8, 64, 128, device=DEV, dtype=torch.float16)
    with pytest.raises(RuntimeError):
        ops.decode_attention(q, kc, kc, 1)
    q = torch.randn(16, 128, device=DEV, dtype=torch.float16)
    with pytest.raises(RuntimeError):
        ops.decode_attention(q, kc, kc, 65)
    with pytest.raises(RuntimeError):
        ops.decode_attention(q, kc, kc, 0)


def test_kv_cache_append_writes_only_target_position():
    kc = torch.full((8, 64, 128), -1.0, device=DEV, dtype=torch.float16)
    vc = torch.full_like(kc, -1.0)
    torch.manual_seed(3)
    for pos in [0, 5, 63]:
        kn = torch.randn(8, 128, device=DEV, dtype=torch.float16)
        vn = torch.randn(8, 128, device=DEV, dtype=torch.float16)
        ops.kv_cache_append(kc, vc, kn, vn, pos)
        assert torch.equal(kc[:, pos], kn) and torch.equal(vc[:, pos], vn)
    assert torch.all(kc[:, 1] == -1.0) and torch.all(vc[:, 1] == -1.0)
    with pytest.raises(RuntimeError):
        ops.kv_cache_append(kc, vc, kn, vn, 64)


def test_rope_matches_math_reference():
    torch.manual_seed(6)
    x = torch.randn(16, 128, device=DEV, dtype=torch.float16)
    c, s = ops.precompute_rope_cos_sin(128, 1_000_000.0, 37, device=DEV)
    expected = port.rope(x.cpu().numpy(), c.cpu().numpy(), s.cpu().numpy())
    out = ops.apply_rope(x.clone(), c, s)
    assert_close(out, expected.astype(np.float64), "rope")


@pytest.mark.parametrize("rows,hidden", [(1, 2048), (16, 128), (3, 5120), (40, 128), (2, 6)])
def test_rmsnorm_matches_oracle(rows, hidden):
    torch.manual_seed(7)
    x = torch.randn(rows, hidden, device=DEV, dtype=torch.float16)
    w = torch.randn(hidden, device=DEV, dtype=torch.float16)
    out = ops.rmsnorm(x, w, 1e-6)
    assert_close(out, port.rmsnorm(x.cpu().numpy(), w.cpu().numpy(), 1e-6).astype(np.float64), "rmsnorm")
    odd = torch.randn(2, 7, device=DEV, dtype=torch.float16)
    with pytest.raises(RuntimeError):
        ops.rmsnorm(odd, torch.ones(7, device=DEV, dtype=torch.float16), 1e-6)


def test_qk_norm_and_rope_match_huggingface_qwen3():
    transformers = pytest.importorskip("transformers")  # noqa: F841
    from transformers.models.qwen3 import modeling_qwen3 as q3

    torch.manual_seed(8)
    x = torch.randn(16, 128, device=DEV, dtype=torch.float16)
    w = torch.randn(128, device=DEV, dtype=torch.float16)
    norm = q3.Qwen3RMSNorm(128, eps=1e-6).to(DEV).half()
    norm.weight.data.copy_(w)
    assert_close(ops.qk_norm(x, w, 1e-6), norm(x), "qk_norm vs HF")

    theta, pos = 1_000_000.0, 37
    inv = 1.0 / (theta ** (torch.arange(0, 128, 2, dtype=torch.float32, device=DEV) / 128))
    emb = torch.cat([pos * inv, pos * inv])
    cos, sin = emb.cos().half()[None, None], emb.sin().half()[None, None]
    qh = x.unsqueeze(0).unsqueeze(2)
    expected, _ = q3.apply_rotary_pos_emb(qh, qh, cos, sin, unsqueeze_dim=1)
    c, s = ops.precompute_rope_cos_sin(128, theta, pos, device=DEV)
    assert_close(ops.apply_rope(x.clone(), c, s), expected.squeeze(0).squeeze(1), "rope vs HF")
