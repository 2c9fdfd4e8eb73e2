"""Decode loops over the soinfer ops (reference python/soinfer/runtime/)."""
from . import generate, loader  # noqa: F401

__all__ = ["generate", "loader"]
