"""Per-token weight bytes of the decode path (reference generate.py:407-426)
against the hand-computed configs[3] figures: Qwen3-1.7B shapes (28 layers,
hidden 2048, intermediate 6144, 16 q / 8 kv heads of 128), INT4 packed rows
of K/2 bytes -- 704,643,072 B dense and 528,482,304 B at DIP k = 3072."""
from dataclasses import dataclass

from soinfer.offload.load_hf_checkpoint import DOWN_PROJ_T_SUFFIX
from soinfer.runtime import generate as gen


@dataclass
class _Handle:
    row_nbytes: int


@dataclass
class _Matrix:
    n: int
    handle: _Handle


class _Shapes:
    """Just the matrix shapes the byte count reads (rows n, packed row bytes)."""

    num_layers = 28

    def matrix(self, layer, suffix):
        H, I = 2048, 6144
        rows_k = {
            "self_attn.q_proj.weight": (16 * 128, H),
            "self_attn.k_proj.weight": (8 * 128, H),
            "self_attn.v_proj.weight": (8 * 128, H),
            "self_attn.o_proj.weight": (H, 16 * 128),
            "mlp.gate_proj.weight": (I, H),
            "mlp.up_proj.weight": (I, H),
            DOWN_PROJ_T_SUFFIX: (I, H),
        }[suffix]
        return _Matrix(rows_k[0], _Handle(rows_k[1] // 2))


def test_dip_bytes_per_token_match_hand_computed():
    model = _Shapes()
    assert gen.dip_bytes_per_token(model, 3072, dense=True) == 704_643_072
    assert gen.dip_bytes_per_token(model, 3072) == 528_482_304
    # k = I selects every channel: the dense count
    assert gen.dip_bytes_per_token(model, 6144) == 704_643_072
