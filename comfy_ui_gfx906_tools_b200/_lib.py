"""ctypes binding of the C-ABI library ``lib/libgfx906_b200.so``.

The library is the product's only compute path. Loading fails loudly when it
is missing (build it with ``python -m comfy_ui_gfx906_tools_b200.build``);
nothing here falls back to another implementation.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
# GFX906_B200_LIB selects another build of the same library (e.g. a tuning variant).
LIB_PATH = os.environ.get("GFX906_B200_LIB") or os.path.join(_PKG_DIR, "lib", "libgfx906_b200.so")

GFX_OK = 0
GFX_ERR_INVALID = 1
GFX_ERR_UNSUPPORTED = 2
GFX_ERR_WORKSPACE = 3
GFX_ERR_CUDA = 4
GFX_ERR_DEVICE = 5

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
SCALE_F32, SCALE_F16 = 0, 1

_c_void_p = ctypes.c_void_p
_c_int = ctypes.c_int
_c_size_t = ctypes.c_size_t
_c_int64 = ctypes.c_int64

# name -> (restype, argtypes); mirrors include/gfx906_b200.h
SIGNATURES = {
    "gfx_last_error": (ctypes.c_char_p, []),
    "gfx_version": (_c_int, []),
    "gfx_device_status": (_c_int, [_c_int]),
    "gfx_selftest_wait_timeout": (_c_int, [_c_int, _c_void_p]),
    "w4a16_gemm_allgather": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_int, _c_void_p, _c_void_p, _c_int,
                                      _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_size_t,
                                      _c_void_p]),
    "w4a16_gemm_rows_allgather": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_int, _c_void_p, _c_void_p,
                                           _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_void_p,
                                           _c_size_t, _c_void_p]),
    "gfx_peer_barrier": (_c_int, [_c_void_p, _c_int, _c_int, _c_void_p]),
    "repack_q8_0": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_void_p]),
    "hadamard_rotate": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_int, _c_int64, _c_int, _c_int, _c_void_p]),
    "w4a16_gemm": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_int, _c_void_p, _c_void_p, _c_int, _c_int,
                            _c_int, _c_int, _c_int, _c_void_p, _c_size_t, _c_void_p]),
    "w4a16_gemm_noalloc": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_int, _c_void_p, _c_void_p, _c_int,
                                    _c_int, _c_int, _c_int, _c_int, _c_void_p]),
    "w4a16_workspace_bytes": (_c_size_t, [_c_int, _c_int, _c_int, _c_int]),
    "w4a16_auto_splits": (_c_int, [_c_int, _c_int, _c_int]),
    "w8a16_gemm": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_int, _c_void_p, _c_void_p, _c_int, _c_int,
                            _c_int, _c_int, _c_int, _c_void_p, _c_size_t, _c_void_p]),
    "w8a16_workspace_bytes": (_c_size_t, [_c_int, _c_int, _c_int, _c_int]),
    "quantize_pack_int4": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_void_p]),
    "quantize_int8": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_int64, _c_int, _c_void_p]),
    "repack_q4_0": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_void_p]),
    "int4_dequant": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_void_p]),
    "int4_dequant_qblock": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_void_p, _c_int, _c_int, _c_int,
                                     _c_void_p]),
    "w4a16_gemm_qblock": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_void_p, _c_int, _c_int, _c_void_p, _c_void_p,
                                   _c_int, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_size_t, _c_void_p]),
    "scales_to_f16": (_c_int, [_c_void_p, _c_void_p, _c_int64, _c_void_p, _c_void_p]),
    "quantize_int4_rows": (_c_int, [_c_void_p, _c_int64, _c_int, _c_int, _c_int, ctypes.c_uint32, _c_void_p,
                                    _c_void_p, _c_void_p]),
    "quantize_int4_cols": (_c_int, [_c_void_p, _c_int64, _c_int, _c_int, _c_void_p, _c_int, ctypes.c_uint32,
                                    _c_void_p, _c_void_p, _c_void_p]),
    "attention": (_c_int, [_c_int, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                           _c_void_p, _c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int, ctypes.c_float, _c_void_p]),
    "attention_block_rows": (_c_int, [_c_int]),
    "attention_max_tiles": (_c_int, []),
    "w4a4_gemm_exact_workspace_bytes": (_c_size_t, [_c_int, _c_int, _c_int, _c_int]),
    "w4a4_gemm_exact_splits": (_c_int, [_c_int, _c_int, _c_int, _c_int]),
    "w4a4_gemm_exact": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_void_p, _c_void_p, _c_int,
                                 _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_size_t, _c_void_p]),
}

_lock = threading.Lock()
_lib = None


class GfxError(RuntimeError):
    """A C-ABI call returned an error code; the message is the library's."""

    def __init__(self, fn: str, code: int, message: str):
        super().__init__(f"{fn} failed (code {code}): {message}")
        self.code = code


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: the sm_100a library is not built. "
                    "Run `python -m comfy_ui_gfx906_tools_b200.build` (nvcc 12.9+).")
            lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_LOCAL)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    return load().gfx_last_error().decode(errors="replace")


def call(name: str, *args) -> int:
    """Call a status-returning entry point; raise GfxError on failure."""
    rc = getattr(load(), name)(*args)
    if rc != GFX_OK:
        raise GfxError(name, rc, last_error())
    return rc
