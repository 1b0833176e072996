"""C-ABI library on the CPU: it loads, exports every symbol the public header
declares, and its host-side argument checks return the documented error codes
with messages (no GPU work is issued by any call here)."""
import ctypes
import os
import re

import pytest

from comfy_ui_gfx906_tools_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "gfx906_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", src, flags=re.M)
    return sorted(set(n for n in names if n not in ("if", "defined")))


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ("w4a16_gemm", "w4a16_workspace_bytes", "w4a16_auto_splits", "w8a16_gemm", "quantize_pack_int4",
                     "quantize_int8", "repack_q4_0", "int4_dequant", "scales_to_f16", "gfx_last_error",
                     "gfx_version", "gfx_device_status"):
        assert required in names


def test_library_exports_every_declared_symbol(built_lib):
    for name in declared_functions():
        assert hasattr(built_lib, name), f"{name} declared in include/gfx906_b200.h but not exported"
    assert set(_lib.SIGNATURES) >= set(declared_functions())


def test_version(built_lib):
    assert built_lib.gfx_version() >= 100


def _gemm(built_lib, **kw):
    args = dict(x=16, x_dtype=2, w=16, ws=16, sd=0, bias=None, y=16, out=2, M=4, N=8, K=64, splits=0)
    args.update(kw)
    return built_lib.w4a16_gemm(args["x"], args["x_dtype"], args["w"], args["ws"], args["sd"], args["bias"], args["y"],
                                args["out"], args["M"], args["N"], args["K"], args["splits"], None, 0, None)


@pytest.mark.parametrize("kw,code,needle", [
    (dict(K=48), _lib.GFX_ERR_INVALID, "K % 32 == 0"),
    (dict(N=0), _lib.GFX_ERR_INVALID, "N > 0"),
    (dict(M=-1), _lib.GFX_ERR_INVALID, "M >= 0"),
    (dict(out=7), _lib.GFX_ERR_INVALID, "out dtype"),
    (dict(x_dtype=1), _lib.GFX_ERR_UNSUPPORTED, "bfloat16"),
    (dict(sd=3), _lib.GFX_ERR_INVALID, "scale dtype"),
    (dict(splits=99), _lib.GFX_ERR_INVALID, "splits"),
    (dict(x=None), _lib.GFX_ERR_INVALID, "null pointer"),
    (dict(x=17), _lib.GFX_ERR_INVALID, "16-byte aligned"),
    (dict(sd=1, K=96), _lib.GFX_ERR_UNSUPPORTED, "K % 64"),
])
def test_gemm_argument_checks(built_lib, kw, code, needle):
    assert _gemm(built_lib, **kw) == code
    assert needle in _lib.last_error()


def test_gemm_m_zero_is_noop(built_lib):
    # binding.cpp:93: M == 0 returns an empty output without launching
    assert _gemm(built_lib, M=0) == _lib.GFX_OK


def test_loader_argument_checks(built_lib):
    assert built_lib.quantize_pack_int4(16, 0, 16, 16, 4, 40, 0, None) == _lib.GFX_ERR_INVALID
    assert "K % 32" in _lib.last_error()
    assert built_lib.quantize_pack_int4(16, 0, 16, 16, 4, 64, 5, None) == _lib.GFX_ERR_INVALID
    assert "div_mode" in _lib.last_error()
    assert built_lib.repack_q4_0(16, 16, 16, None, 4, 33, None) == _lib.GFX_ERR_INVALID
    assert built_lib.int4_dequant(16, 16, 0, 16, 9, 4, 64, None) == _lib.GFX_ERR_INVALID
    assert built_lib.quantize_pack_int4(16, 0, 16, 16, 0, 64, 0, None) == _lib.GFX_OK  # zero rows: no-op


def test_error_message_is_thread_local(built_lib):
    import threading
    _gemm(built_lib, K=48)
    msgs = {}

    def other():
        msgs["t"] = _lib.last_error()
    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert msgs["t"] == ""
    assert "K % 32" in _lib.last_error()


def test_selftest_rejects_bad_budget(built_lib):
    # argument check only: nothing is launched
    assert built_lib.gfx_selftest_wait_timeout(0, None) == 1
    assert built_lib.gfx_selftest_wait_timeout(2_000_000, None) == 1
    assert b"timeout_us" in built_lib.gfx_last_error()


def test_hadamard_rotate_argument_checks(built_lib):
    # argument checks only: nothing is launched
    assert built_lib.hadamard_rotate(None, 0, None, None, 0, 4, 96, 48, None) == 1
    assert b"group" in built_lib.gfx_last_error()
    assert built_lib.hadamard_rotate(None, 0, None, None, 0, 4, 96, 64, None) == 1
    assert built_lib.hadamard_rotate(None, 0, None, None, 0, 0, 128, 64, None) == 0  # rows == 0: no-op


def test_allgather_and_peer_barrier_argument_checks(built_lib):
    # argument checks only: nothing is launched
    ptrs = (ctypes.c_void_p * 2)(16, 32)
    nulls = (ctypes.c_void_p * 2)(16, None)
    def ag(targets, n_ranks, rank, M=4):
        return built_lib.w4a16_gemm_allgather(16, 2, 16, 16, 0, None, ctypes.cast(targets, ctypes.c_void_p), n_ranks,
                                              rank, 2, M, 8, 64, 0, None, 0, None)
    assert ag(ptrs, 9, 0) == _lib.GFX_ERR_INVALID and "n_ranks" in _lib.last_error()
    assert ag(ptrs, 2, 2) == _lib.GFX_ERR_INVALID
    assert ag(nulls, 2, 0) == _lib.GFX_ERR_INVALID and "rank 1 is null" in _lib.last_error()
    assert ag(ptrs, 2, 1, M=65) == _lib.GFX_ERR_UNSUPPORTED and "M <= 64" in _lib.last_error()
    assert ag(ptrs, 2, 1, M=0) == _lib.GFX_OK  # M == 0: no launch
    assert built_lib.gfx_peer_barrier(ctypes.cast(ptrs, ctypes.c_void_p), 2, -1, None) == _lib.GFX_ERR_INVALID
    assert built_lib.gfx_peer_barrier(ctypes.cast(nulls, ctypes.c_void_p), 2, 0, None) == _lib.GFX_ERR_INVALID
    assert "rank 1 is null" in _lib.last_error()


def test_attention_argument_checks(built_lib):
    # argument checks only: nothing is launched (the addresses are 16-byte aligned stand-ins, never read)
    P = 4096

    def att(qk=1, pv=1, q=P, qs=P, k=P, ks=P, vt=P, vs=P, keep=None, out=P, B=1, H=4, KVH=2, Lq=64, Lk=64):
        return built_lib.attention(qk, pv, q, qs, k, ks, vt, vs, keep, out, B, H, KVH, Lq, Lk, 0.0, None)

    assert att(qk=3) == _lib.GFX_ERR_INVALID and "qk_mode" in _lib.last_error()
    assert att(pv=2) == _lib.GFX_ERR_INVALID and "pv_mode" in _lib.last_error()
    assert att(H=3) == _lib.GFX_ERR_INVALID and "multiple of KVH" in _lib.last_error()
    assert att(Lk=0) == _lib.GFX_ERR_INVALID
    assert att(qs=None) == _lib.GFX_ERR_INVALID and "q_scale" in _lib.last_error()
    assert att(qk=0, qs=None, ks=None, vs=None) == _lib.GFX_ERR_INVALID and "v_scale" in _lib.last_error()
    assert att(q=P + 8) == _lib.GFX_ERR_INVALID and "16-byte" in _lib.last_error()
    assert att(keep=P, Lk=64 * 1025) == _lib.GFX_ERR_INVALID and "key tiles" in _lib.last_error()
    assert att(qk=0, qs=None, ks=None, pv=0, vs=None, B=0) == _lib.GFX_OK  # nothing to compute
    assert built_lib.attention_block_rows(0) == 64 and built_lib.attention_block_rows(2) == 128
    assert built_lib.attention_block_rows(5) == -1
    assert built_lib.attention_max_tiles() == 1024
