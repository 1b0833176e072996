"""B200-native (sm_100a) int4 / int8 weight-only linear path for ComfyUI DiTs.

A drop-in for the hot path of luna-niemitalo/comfy_ui_gfx906_tools'
``nodes/ComfyUI-Gfx906Int4``: the same operator names (``ops``), packed
weight layout, scale format and node classes (``nodes``), with the compute in
hand-written CUDA for sm_100a behind a C ABI (``include/gfx906_b200.h``).
"""
from . import _lib  # noqa: F401

__version__ = "0.1.0"
