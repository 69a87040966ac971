"""B200 big-lama inpainting engine: Python host over the C ABI (include/lama_b200.h)."""

from .engine import Engine, LamaError, lib  # noqa: F401

__all__ = ["Engine", "LamaError", "lib"]
