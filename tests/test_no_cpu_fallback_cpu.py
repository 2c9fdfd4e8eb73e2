"""The product path has no CPU fallback: every hot-path op given CPU tensors
raises RuntimeError (naming the CUDA requirement, as the reference's
TORCH_CHECKs do) instead of computing on the host."""
import pytest
import torch

import soinfer.ops as ops
from soinfer import _C
from tests.helpers import int4_weights

P, S, PK = int4_weights(64, 256, 128, seed=1)
X = torch.randn(PK).half()
H16 = torch.zeros(64).half()
IDX = torch.arange(8, dtype=torch.int32)

CASES = {
    "gemv_w4a16_group": lambda: ops.gemv_w4a16_group(P, S, X, PK, 128),
    "gemv_w4a16_group_lop3": lambda: ops.gemv_w4a16_group_lop3(P, S, X, PK, 128),
    "gemv_w8a16": lambda: ops.gemv_w8a16(torch.zeros(4, 8, dtype=torch.int8), torch.ones(4, 1), torch.zeros(8).half(), 8),
    "gemv_w4a16_batch": lambda: _C.gemv_w4a16_batch([(P, S, X, torch.empty(64).half(), PK, 128, -1)]),
    "gemm_w4a16": lambda: ops.gemm_w4a16(P, S, torch.zeros(2, PK).half(), PK, 128),
    "gemv_w4a16_rows": lambda: ops.gemv_w4a16_rows(P, S, IDX, X, PK, 128),
    "topk_threshold_select": lambda: ops.topk_threshold_select(torch.rand(64), 8),
    "topk_threshold_select_abs": lambda: ops.topk_threshold_select_abs(H16, 8),
    "build_dip_descriptors": lambda: ops.build_dip_descriptors(IDX, torch.zeros(64, dtype=torch.int32)),
    "gemv_w4a16_sparse_accumulate": lambda: ops.gemv_w4a16_sparse_accumulate(P, S, H16, PK, 128),
    "gemv_w4a16_sparse_rows": lambda: ops.gemv_w4a16_sparse_rows(P, S, IDX, torch.zeros(8).half(), PK, 128),
    "gemv_dip_fused_up": lambda: ops.gemv_dip_fused_up(P, S, P, S, IDX, X, PK, 128),
    "gemv_dip_fused_down": lambda: ops.gemv_dip_fused_down(P, S, P, S, IDX, torch.zeros(8).half(), PK, 128),
    "gemv_fp16_v3": lambda: ops.gemv_fp16_v3(torch.zeros(4, 8).half(), torch.zeros(8).half()),
    "decode_attention": lambda: ops.decode_attention(torch.zeros(2, 64).half(), torch.zeros(1, 16, 64).half(),
                                                     torch.zeros(1, 16, 64).half(), 4),
    "rmsnorm": lambda: ops.rmsnorm(torch.zeros(1, 64).half(), torch.ones(64).half()),
    "add_rmsnorm": lambda: ops.add_rmsnorm(torch.zeros(1, 64).half(), torch.zeros(1, 64).half(), torch.ones(64).half()),
    "swiglu": lambda: ops.swiglu(H16, H16),
    "apply_rope": lambda: ops.apply_rope(torch.zeros(2, 64).half(), torch.ones(32), torch.zeros(32)),
    "kv_cache_append": lambda: ops.kv_cache_append(torch.zeros(1, 16, 64).half(), torch.zeros(1, 16, 64).half(),
                                                   torch.zeros(1, 64).half(), torch.zeros(1, 64).half(), 0),
    "quantize_pack_int4": lambda: _C.quantize_pack_int4(torch.randn(16, 256), 128),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_cpu_tensors_raise_instead_of_computing(name):
    with pytest.raises(RuntimeError, match="CUDA"):
        CASES[name]()
