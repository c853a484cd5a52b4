"""B200-native batch-one Qwen3-0.6B decode engine.

Drop-in for the reference's decode path (tejeshbhalla/mega-kernel):

* ``libmkb200.so`` -- the persistent sm_100a decode kernel and its C ABI
  (``include/mkb200.h``), including the reference launcher signature
  ``launch_decode_kernel`` (megakernel.cu:898-927);
* :func:`extension` -- the PyTorch extension ``megakernel_extension`` with the
  reference's ``decode(...)`` call (pytorch_binding.cu:36-48);
* :class:`DecodeEngine` -- the resident engine (weights table, transposed down
  weights, workspace and CUDA graph kept across tokens).

There is no CPU or PyTorch fallback: without the built library every entry
point raises.
"""
from __future__ import annotations

from . import _lib
from .engine import DecodeEngine, check_model, decode_call
from .rope import rope_tables

_ext = None


def extension():
    """The ``megakernel_extension`` module (built in-tree on first use)."""
    global _ext
    if _ext is None:
        from .build import build_extension
        _ext = build_extension()
    return _ext


def decode(*args, **kwargs):
    """``megakernel_extension.decode`` -- the reference's call signature."""
    return extension().decode(*args, **kwargs)


__all__ = ["DecodeEngine", "decode", "decode_call", "extension", "rope_tables", "check_model", "_lib"]
