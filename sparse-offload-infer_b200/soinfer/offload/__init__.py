"""Host-memory side of the decode path: pinned weight arena, copy-engine
streaming, hot-channel cache, quantize-on-load (reference
python/soinfer/offload/)."""
from . import hot_cache, load_hf_checkpoint, stream_manager, weight_store  # noqa: F401

__all__ = ["weight_store", "stream_manager", "load_hf_checkpoint", "hot_cache"]
