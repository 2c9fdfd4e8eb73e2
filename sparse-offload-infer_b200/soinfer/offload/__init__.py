"""Host-memory side of the decode path: pinned weight arena, copy-engine
streaming, hot-channel cache, quantize-on-load (reference
python/soinfer/offload/)."""
from . import load_hf_checkpoint, stream_manager, weight_store  # noqa: F401

__all__ = ["weight_store", "stream_manager", "load_hf_checkpoint"]
