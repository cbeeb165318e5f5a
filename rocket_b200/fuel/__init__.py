from . import nvfp4

__all__ = ["nvfp4"]
