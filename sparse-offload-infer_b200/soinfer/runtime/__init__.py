"""Decode loops over the soinfer ops (reference python/soinfer/runtime/)."""
from . import generate  # noqa: F401

__all__ = ["generate"]
