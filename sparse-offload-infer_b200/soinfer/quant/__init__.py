from . import calibrate, formats, pack

__all__ = ["formats", "pack", "calibrate"]
