"""soinfer -- B200-native (sm_100a) decode hot path of sparse-offload-infer.

Drop-in for the reference's python/soinfer package: soinfer.ops (the kernel
op surface, backed by the C ABI in libsoinfer_b200.so), soinfer.quant
(quantize / pack), soinfer.offload (pinned arena, streaming, hot cache) and
soinfer.runtime (decode loops).  Importing never touches the GPU; an op call
without the built library raises RuntimeError (there is no CPU fallback).
"""
from . import quant  # noqa: F401
from . import ops  # noqa: F401
from . import offload  # noqa: F401
from . import runtime  # noqa: F401

__all__ = ["ops", "quant", "offload", "runtime"]
