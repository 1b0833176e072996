"""Operator layer: the reference's Python-facing int4 surface, on sm_100a.

Mirrors ``nodes/ComfyUI-Gfx906Int4/ops.py`` of luna-niemitalo/comfy_ui_gfx906_tools
(same names, argument order, buffers, packed layout and scale format) with the
compute routed through this package's C-ABI library (``_lib``):

  * ``int4_linear`` (ops.py:167-183) -> ``gemm_w4a16``: bf16 activations
    against the packed int4 weights, fp32 accumulation (weight-only; the
    reference's ``gemm_int4`` also quantizes the activations to int4 per
    32-block, binding.cpp:53-68, which this drop-in does not do: the
    weight-only product is the one the reference's fp32 dequant-then-matmul
    oracle defines);
  * ``quantize_pack_int4`` (ops.py:108-126) and ``repack_q4_0_native``
    (ops.py:129-164) run as GPU kernels with results identical to the
    reference's torch code on the tensor's own device (CPU tensors: the
    IEEE-division semantics of torch on CPU; CUDA tensors: the reciprocal
    multiply torch uses for ``tensor / 7.0`` on CUDA);
  * ``Gfx906Int4Ops.Linear`` (ops.py:199-260) with the same buffers
    ``weight_q4`` int8 [N, K/2] / ``weight_scale`` fp32 [N, K/32], the same
    ``quantized`` rule and quantize-on-load.

There is no CPU fallback: a CUDA build of the library is required for every
compute entry point.
"""
from __future__ import annotations

import threading

import torch

from . import _lib

BLOCK = 32
ROTATION_SEED = 0

_DTYPE_CODE = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16}


def _dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise RuntimeError(f"unsupported dtype {dt}, expected float32/float16/bfloat16") from None


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(t: torch.Tensor, name: str):
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be on a CUDA device, got {t.device}")


# ---------------------------------------------------------------------------
# per-(device, stream) split-K workspace; zero-filled once, the kernel leaves
# its counters at zero after every call
# ---------------------------------------------------------------------------
_ws_lock = threading.Lock()
_workspaces: dict = {}


def _workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    key = (device.index, stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _workspaces[key] = ws
        return ws


def _rearm_workspaces(device: torch.device):
    """Zero every cached split-K workspace of `device`: after a kernel gave up
    in a bounded wait, its row blocks' arrival counters may be left non-zero,
    and a later call sharing the workspace would sum the wrong segments."""
    with _ws_lock:
        for (idx, _), ws in _workspaces.items():
            if idx == device.index:
                ws.zero_()


def device_status(device: torch.device | None = None, clear: bool = False) -> int:
    """The device's status word (synchronises it): 0 when healthy, else the
    code of the first bounded device-side wait that gave up (1-7, see
    include/gfx906_b200.h). ``clear`` resets it and re-zeroes the cached
    split-K workspaces, after which the GEMMs run again."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(device):
        v = int(_lib.load().gfx_device_status(1 if clear else 0))
        if clear:
            _rearm_workspaces(device)
            torch.cuda.synchronize(device)
    return v


def _call_gemm(name: str, device: torch.device, *args):
    """A GEMM entry point; a GFX_ERR_DEVICE (an earlier kernel gave up in a
    bounded wait) also re-zeroes this device's cached workspaces before the
    error propagates. The status stays set until ``device_status(clear=True)``."""
    try:
        _lib.call(name, *args)
    except _lib.GfxError as e:
        if e.code == _lib.GFX_ERR_DEVICE:
            _rearm_workspaces(device)
        raise


# ---------------------------------------------------------------------------
# Hadamard rotation helpers (reference ops.py:43-105), torch on the tensor's device
# ---------------------------------------------------------------------------
_HADAMARD_CACHE = {}
_ROTATION_CACHE = {}


def _hadamard(n: int, device, dtype=torch.float32):
    """Orthonormal Sylvester Hadamard matrix of order n (a power of two)."""
    key = (n, str(device), dtype)
    if key not in _HADAMARD_CACHE:
        if n & (n - 1) != 0:
            raise AssertionError(f"Hadamard order {n} must be a power of two")
        h = torch.ones(1, 1, device=device, dtype=dtype)
        while h.shape[0] < n:
            h = torch.cat([torch.cat([h, h], dim=1), torch.cat([h, -h], dim=1)], dim=0)
        _HADAMARD_CACHE[key] = h / (n ** 0.5)
    return _HADAMARD_CACHE[key]


def choose_rotation_group(in_features: int, max_group: int = 128, min_group: int = 32) -> int | None:
    """Largest power-of-two group <= max_group dividing in_features, or None
    below min_group (ops.py:54-65)."""
    g = max_group
    while g >= min_group:
        if in_features % g == 0:
            return g
        g //= 2
    return None


def rotation_signs(group: int, device) -> torch.Tensor:
    """The +-1 float vector of get_group_rotation: a CPU generator seeded
    ROTATION_SEED ^ group (ops.py:68-82)."""
    key = ("signs", group, str(device))
    if key not in _ROTATION_CACHE:
        g = torch.Generator(device="cpu").manual_seed(ROTATION_SEED ^ group)
        _ROTATION_CACHE[key] = (torch.randint(0, 2, (group,), generator=g).float() * 2 - 1).to(device)
    return _ROTATION_CACHE[key]


def get_group_rotation(in_features: int, group: int, device) -> torch.Tensor:
    """R = H_group * diag(random signs), signs from a CPU generator seeded
    ROTATION_SEED ^ group (ops.py:68-82), so folding time and forward time agree."""
    key = (in_features, group, str(device))
    if key not in _ROTATION_CACHE:
        _ROTATION_CACHE[key] = _hadamard(group, device) * rotation_signs(group, device)
    return _ROTATION_CACHE[key]


def hadamard_rotate(x: torch.Tensor, group: int, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Forward-time activation rotation on the GPU: every group-sized chunk of
    the last dim of x (CUDA) is multiplied by R = H / sqrt(group) * diag(signs)
    as a fast Walsh-Hadamard transform (one kernel, fp32 math, written
    straight in out_dtype); equal to ``apply_group_rotation`` up to fp32
    rounding."""
    _require_cuda(x, "x")
    shape = x.shape
    K = shape[-1]
    src = x.reshape(-1, K)
    if src.dtype not in _DTYPE_CODE:
        src = src.float()
    src = src.contiguous()
    out = torch.empty(src.shape, dtype=out_dtype, device=x.device)
    sign = rotation_signs(group, x.device)
    with torch.cuda.device(x.device):
        _lib.call("hadamard_rotate", src.data_ptr(), _dtype_code(src.dtype), sign.data_ptr(), out.data_ptr(),
                  _dtype_code(out_dtype), src.shape[0], K, group, _stream(x.device))
    return out.reshape(shape)


def apply_group_rotation(t: torch.Tensor, R: torch.Tensor, group: int) -> torch.Tensor:
    """Rotate every group-sized chunk of the last dim: flat @ R^T (ops.py:85-105),
    on t's own device."""
    shape = t.shape
    return (t.reshape(-1, group) @ R.t().to(t.device, t.dtype)).reshape(shape)


# ---------------------------------------------------------------------------
# packing / loader kernels
# ---------------------------------------------------------------------------
def quantize_pack_int4(t: torch.Tensor, block: int = BLOCK):
    """t [..., K] float -> (packed int8 [..., K/2], scale float32 [..., K/block]).

    Same result as the reference (ops.py:108-126) evaluated on t's device:
    a CPU tensor is quantized with torch-CPU semantics (IEEE ``amax / 7``),
    a CUDA tensor with torch-CUDA semantics (``amax * (1/7)``). The work runs
    on the GPU either way; CPU tensors are staged through the current device.
    """
    if block != BLOCK:
        raise RuntimeError(f"block must be {BLOCK}, got {block}")
    shape = t.shape
    K = shape[-1]
    if K % block != 0:
        raise AssertionError(f"last dim {K} not divisible by block {block}")
    on_cpu = not t.is_cuda
    if on_cpu and not torch.cuda.is_available():
        raise RuntimeError("quantize_pack_int4 needs a CUDA device (the packing runs as a GPU kernel)")
    dev = torch.device("cuda", torch.cuda.current_device()) if on_cpu else t.device
    src = t.reshape(-1, K)
    if src.dtype not in _DTYPE_CODE:
        src = src.float()
    src = src.to(dev).contiguous()
    rows = src.shape[0]
    packed = torch.empty(rows, K // 2, dtype=torch.int8, device=dev)
    scale = torch.empty(rows, K // block, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.call("quantize_pack_int4", src.data_ptr(), _dtype_code(src.dtype), packed.data_ptr(), scale.data_ptr(),
                  rows, K, 0 if on_cpu else 1, _stream(dev))
    packed = packed.reshape(*shape[:-1], K // 2)
    scale = scale.reshape(*shape[:-1], K // block)
    if on_cpu:
        packed, scale = packed.cpu(), scale.cpu()
    return packed, scale


def repack_q4_0_native(raw_bytes: torch.Tensor, out_features: int, in_features: int, block: int = BLOCK):
    """Lossless ggml Q4_0 -> native repack (ops.py:129-164), as a GPU kernel.
    Returns tensors on raw_bytes' device."""
    if block != BLOCK:
        raise RuntimeError(f"block must be {BLOCK}, got {block}")
    nbytes = out_features * (in_features // block) * 18
    raw = raw_bytes.reshape(-1).view(torch.uint8)
    if raw.numel() != nbytes:
        raise RuntimeError(f"expected {nbytes} Q4_0 bytes for [{out_features}, {in_features}], got {raw.numel()}")
    on_cpu = not raw.is_cuda
    dev = torch.device("cuda", torch.cuda.current_device()) if on_cpu else raw.device
    raw = raw.to(dev).contiguous()
    packed = torch.empty(out_features, in_features // 2, dtype=torch.int8, device=dev)
    scale = torch.empty(out_features, in_features // block, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.call("repack_q4_0", raw.data_ptr(), packed.data_ptr(), scale.data_ptr(), None, out_features,
                  in_features, _stream(dev))
    if on_cpu:
        packed, scale = packed.cpu(), scale.cpu()
    return packed, scale


def repack_q8_0(raw_bytes: torch.Tensor, out_features: int, in_features: int, block: int = BLOCK):
    """Lossless ggml Q8_0 -> (int8 [N, K], float32 block scales [N, K/32]), the
    format ``gemm_w8a16`` takes, as a GPU kernel (value = q * d). Returns
    tensors on raw_bytes' device. The reference instead dequantizes Q8_0 and
    re-quantizes it to int4 (nodes.py:294-301), which is lossy."""
    if block != BLOCK:
        raise RuntimeError(f"block must be {BLOCK}, got {block}")
    if in_features % block != 0:
        raise RuntimeError(f"in_features {in_features} must be a multiple of {block}")
    nbytes = out_features * (in_features // block) * 34
    raw = raw_bytes.reshape(-1).view(torch.uint8)
    if raw.numel() != nbytes:
        raise RuntimeError(f"expected {nbytes} Q8_0 bytes for [{out_features}, {in_features}], got {raw.numel()}")
    on_cpu = not raw.is_cuda
    dev = torch.device("cuda", torch.cuda.current_device()) if on_cpu else raw.device
    raw = raw.to(dev).contiguous()
    q = torch.empty(out_features, in_features, dtype=torch.int8, device=dev)
    scale = torch.empty(out_features, in_features // block, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.call("repack_q8_0", raw.data_ptr(), q.data_ptr(), scale.data_ptr(), out_features, in_features,
                  _stream(dev))
    if on_cpu:
        q, scale = q.cpu(), scale.cpu()
    return q, scale


def dequantize_int4(w_packed: torch.Tensor, w_scale: torch.Tensor, out_dtype: torch.dtype = torch.float32,
                    block: int = BLOCK):
    """Dequantize native int4 weights on the GPU: code * scale as one fp32
    multiply, rounded once to out_dtype (int4_train_test.py:46-52; bf16 out
    = nodes.py:51-52 for a bf16 model). ``block`` is the scale block: 32
    (scales [N, K/32]) or 16 (scales [N, K/16], the reference's qblock=16)."""
    _require_cuda(w_packed, "w_packed")
    N, half_k = w_packed.shape
    K = half_k * 2
    scale_code = _lib.SCALE_F16 if w_scale.dtype == torch.float16 else _lib.SCALE_F32
    if w_scale.dtype not in (torch.float16, torch.float32):
        raise RuntimeError(f"scales must be float32 or float16, got {w_scale.dtype}")
    if block not in (32, 16):
        raise RuntimeError(f"block must be 32 or 16, got {block}")
    if w_scale.numel() != N * (K // block):
        raise RuntimeError(f"scales must be [N, K/{block}] = {N * (K // block)} elements, got {w_scale.numel()}")
    wp, ws = w_packed.contiguous(), w_scale.contiguous()
    out = torch.empty(N, K, dtype=out_dtype, device=w_packed.device)
    with torch.cuda.device(w_packed.device):
        _lib.call("int4_dequant_qblock", wp.data_ptr(), ws.data_ptr(), scale_code, block, out.data_ptr(),
                  _dtype_code(out_dtype), N, K, _stream(w_packed.device))
    return out


def scales_to_f16_if_exact(w_scale: torch.Tensor):
    """fp16 copy of fp32 scales when every value survives the round trip
    exactly (true for Q4_0-sourced weights), else None."""
    _require_cuda(w_scale, "w_scale")
    s = w_scale.contiguous().float()
    out = torch.empty(s.shape, dtype=torch.float16, device=s.device)
    bad = torch.empty(1, dtype=torch.int32, device=s.device)
    with torch.cuda.device(s.device):
        _lib.call("scales_to_f16", s.data_ptr(), out.data_ptr(), s.numel(), bad.data_ptr(), _stream(s.device))
    return out if int(bad.item()) == 0 else None


# ---------------------------------------------------------------------------
# GEMM entry points
# ---------------------------------------------------------------------------
def gemm_int4_auto_splits(M: int, N: int, K: int) -> int:
    """Split-K count ``gemm_int4(..., splits=0)`` uses for [M, K] x [N, K]^T on
    the current device: the reference's auto_splits (binding.cpp:36-43,
    exported as gemm_int4_auto_splits, binding.cpp:358-361), evaluated with
    this device's SM count. The count is part of gemm_int4's numerics."""
    return int(_lib.load().w4a4_gemm_exact_splits(int(M), int(N), int(K), 0))


def gemm_w4a16_auto_splits(M: int, N: int, K: int) -> int:
    """Split-K count the W4A16 GEMM (``gemm_w4a16``) picks on the current device."""
    return int(_lib.load().w4a16_auto_splits(int(M), int(N), int(K)))


def gemm_w4a16(x: torch.Tensor, B_packed: torch.Tensor, B_scale: torch.Tensor, bias: torch.Tensor | None,
               out_dtype: torch.dtype, splits: int = 0, qblock: int = 32) -> torch.Tensor:
    """C[M, N] = x[M, K] @ dequant(B_packed, B_scale)^T (+ bias), fp32 accumulate.

    x: bf16 [M, K] (other float dtypes are converted to bf16 first).
    B_packed int8 [N, K/2]; B_scale float32 (reference format) or float16
    [N, K/32]; with ``qblock=16`` float32 [N, K/16] (one scale per 16
    elements, gemm_int4's qblock, int4_gemm_scaled.hip:153-160); bias [N] in
    out_dtype or None. Argument checks and messages follow gemm_int4
    (binding.cpp:76-101).
    """
    if not (x.is_cuda and B_packed.is_cuda):
        raise RuntimeError("inputs must be on device")
    if x.device != B_packed.device:
        raise RuntimeError("x and B must be on the same device")
    if B_packed.dtype != torch.int8:
        raise RuntimeError(f"packed weights must be int8, got {B_packed.dtype}")
    if x.dim() != 2 or B_packed.dim() != 2 or x.shape[1] != B_packed.shape[1] * 2:
        raise RuntimeError(f"expected x [M, K], B [N, K/2]; got x {tuple(x.shape)} B {tuple(B_packed.shape)}")
    M, K = x.shape
    N = B_packed.shape[0]
    if K % 32 != 0:
        raise RuntimeError(f"expected K % 32 == 0, got K={K}")
    if B_scale.dtype not in (torch.float32, torch.float16):
        raise RuntimeError(f"scales must be float32 (or float16), got {B_scale.dtype}")
    if qblock not in (32, 16):
        raise RuntimeError(f"qblock must be 32 or 16, got {qblock}")
    if qblock == 16 and B_scale.dtype != torch.float32:
        raise RuntimeError(f"qblock=16 takes float32 scales, got {B_scale.dtype}")
    if B_scale.numel() != N * (K // qblock):
        raise RuntimeError(f"scales must be [N, K/{qblock}] = {N * (K // qblock)} elements, got {B_scale.numel()}")
    if not (0 <= splits <= 16):
        raise RuntimeError(f"splits must be in [0, 16], got {splits}")
    out = torch.empty(M, N, dtype=out_dtype, device=x.device)
    if M == 0:
        return out
    bias_ptr = None
    if bias is not None:
        if bias.dtype != out_dtype:
            raise RuntimeError(f"bias dtype {bias.dtype} != out dtype {out_dtype}")
        if bias.numel() != N:
            raise RuntimeError(f"bias must have {N} elements, got {bias.numel()}")
        bias = bias.contiguous()
        bias_ptr = bias.data_ptr()
    xb = x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
    xb = xb.contiguous()
    Bp, Bs = B_packed.contiguous(), B_scale.contiguous()
    dev = x.device
    with torch.cuda.device(dev):
        stream = _stream(dev)
        if qblock == 16:  # the tensor-core kernel for every M; no workspace
            _call_gemm("w4a16_gemm_qblock", dev, xb.data_ptr(), _lib.DTYPE_BF16, Bp.data_ptr(), Bs.data_ptr(),
                       _lib.SCALE_F32, 16, bias_ptr, out.data_ptr(), _dtype_code(out_dtype), M, N, K, splits, None, 0,
                       stream)
            return out
        L = _lib.load()
        nbytes = int(L.w4a16_workspace_bytes(M, N, K, splits))
        ws = _workspace(dev, stream, nbytes)
        _call_gemm("w4a16_gemm", dev, xb.data_ptr(), _lib.DTYPE_BF16, Bp.data_ptr(), Bs.data_ptr(),
                  _lib.SCALE_F16 if Bs.dtype == torch.float16 else _lib.SCALE_F32, bias_ptr, out.data_ptr(),
                  _dtype_code(out_dtype), M, N, K, splits, ws.data_ptr() if ws is not None else None,
                  ws.numel() if ws is not None else 0, stream)
    return out


def gemm_w8a16(x: torch.Tensor, B: torch.Tensor, B_scale: torch.Tensor, bias: torch.Tensor | None,
               out_dtype: torch.dtype) -> torch.Tensor:
    """C[M, N] = x[M, K] @ dequant_int8(B, B_scale)^T (+ bias), fp32 accumulate.

    B int8 [N, K]; B_scale float32 [N, K/32] (the reference's block scales,
    from quantize_int8) or float16 [N] (one scale per output channel, applied
    to the fp32 accumulator). Checks follow gemm_int8 (binding.cpp:192-213).
    """
    if not (x.is_cuda and B.is_cuda):
        raise RuntimeError("inputs must be on device")
    if x.device != B.device:
        raise RuntimeError("x and B must be on the same device")
    if B.dtype != torch.int8:
        raise RuntimeError(f"B must be int8, got {B.dtype}")
    if x.dim() != 2 or B.dim() != 2 or x.shape[1] != B.shape[1] or x.shape[1] % 32 != 0:
        raise RuntimeError(f"expected x [M, K], B [N, K], K % 32 == 0; got x {tuple(x.shape)} B {tuple(B.shape)}")
    M, K = x.shape
    N = B.shape[0]
    if B_scale.dtype == torch.float16 and B_scale.numel() == N:
        per_channel = 1
    elif B_scale.dtype == torch.float32 and B_scale.numel() == N * (K // 32):
        per_channel = 0
    else:
        raise RuntimeError(f"scales must be float32 [N, K/32] = {N * (K // 32)} or float16 [N] = {N} elements, got "
                           f"{B_scale.dtype} {tuple(B_scale.shape)}")
    out = torch.empty(M, N, dtype=out_dtype, device=x.device)
    if M == 0:
        return out
    bias_ptr = None
    if bias is not None:
        if bias.dtype != out_dtype or bias.numel() != N:
            raise RuntimeError(f"bias must be {out_dtype} [{N}], got {bias.dtype} {tuple(bias.shape)}")
        bias = bias.contiguous()
        bias_ptr = bias.data_ptr()
    xb = (x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)).contiguous()
    Bc, Bs = B.contiguous(), B_scale.contiguous()
    with torch.cuda.device(x.device):
        _call_gemm("w8a16_gemm", x.device, xb.data_ptr(), _lib.DTYPE_BF16, Bc.data_ptr(), Bs.data_ptr(), per_channel,
                   bias_ptr, out.data_ptr(), _dtype_code(out_dtype), M, N, K, 0, None, 0, _stream(x.device))
    return out


def quantize_int8(x: torch.Tensor):
    """x [M, K] float -> (int8 [M, K], scale float32 [M, K/32]): block-32,
    scale = amax * (1/127), round-half-even, clamp +-127 (binding.cpp:174-186,
    int8_gemm.hip:217-246)."""
    _require_cuda(x, "x")
    if x.dim() != 2 or x.shape[1] % 32 != 0:
        raise RuntimeError(f"x must be [M, K] with K % 32 == 0, got {tuple(x.shape)}")
    xc = x.contiguous()
    M, K = xc.shape
    q = torch.empty(M, K, dtype=torch.int8, device=x.device)
    s = torch.empty(M, K // 32, dtype=torch.float32, device=x.device)
    if M:
        with torch.cuda.device(x.device):
            _lib.call("quantize_int8", xc.data_ptr(), _dtype_code(xc.dtype), q.data_ptr(), s.data_ptr(), M, K,
                      _stream(x.device))
    return q, s


def quantize_int4(x: torch.Tensor):
    """x [M, K] float (CUDA) -> (packed int8 [M, K/2], scale float32 [M, K/32]):
    the reference's activation quantizer (binding.cpp:53-68,
    int4_gemm_scaled.hip:197-220; scale = amax * (1/7))."""
    _require_cuda(x, "x")
    if x.dim() != 2 or x.shape[1] % 32 != 0:
        raise RuntimeError(f"x must be [M, K] with K % 32 == 0, got {tuple(x.shape)}")
    return quantize_pack_int4(x)


def _check_train_quant_input(x: torch.Tensor, mult_r: int, mult_c: int):
    """binding.cpp:317-327's checks, same substance."""
    if not (x.is_cuda and x.dtype == torch.float16 and x.dim() == 2 and x.stride(1) == 1):
        raise RuntimeError(f"x must be a device fp16 [R, C] tensor with contiguous rows, got {x.dtype} "
                           f"{tuple(x.shape)} strides {tuple(x.stride())}")
    if x.shape[0] % mult_r != 0 or x.shape[1] % mult_c != 0:
        raise RuntimeError(f"x must be [R % {mult_r} == 0, C % {mult_c} == 0], got {tuple(x.shape)}")
    if x.stride(0) % 8 != 0 or x.data_ptr() % 16 != 0:
        raise RuntimeError(f"x rows must be 16-byte aligned, got row stride {x.stride(0)}")


def quantize_int4_rows(x: torch.Tensor, sr: bool, seed: int):
    """Block-16 int4 quantize along rows for the int4 training GEMMs
    (``ext.quantize_int4_rows``, binding.cpp:329-339, int4_train_quant.hip:59-85):
    x fp16 [R, C] (C % 32 == 0) -> (packed int8 [R, C/2], scale float32 [R, C/16]),
    round to nearest even, or stochastic rounding keyed by ``seed``."""
    _check_train_quant_input(x, 1, 32)
    R, C = x.shape
    packed = torch.empty(R, C // 2, dtype=torch.int8, device=x.device)
    scale = torch.empty(R, C // 16, dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        _lib.call("quantize_int4_rows", x.data_ptr(), x.stride(0), R, C, 1 if sr else 0, int(seed) & 0xFFFFFFFF,
                  packed.data_ptr(), scale.data_ptr(), _stream(x.device))
    return packed, scale


def quantize_int4_cols(x: torch.Tensor, signs: torch.Tensor | None, sr: bool, seed: int):
    """Block-16 int4 quantize along columns, transposed (``ext.quantize_int4_cols``,
    binding.cpp:341-356, int4_train_quant.hip:87-123): x fp16 [R, C] (R % 32 == 0)
    -> (packed int8 [C, R/2], scale float32 [C, R/16]); with ``signs`` (16 fp32
    on the device) every 16-row group is first rotated by (H16 / 4) diag(signs)."""
    _check_train_quant_input(x, 32, 1)
    if signs is not None and not (signs.is_cuda and signs.dtype == torch.float32 and signs.numel() == 16
                                  and signs.is_contiguous()):
        raise RuntimeError(f"signs must be a contiguous device fp32 tensor of 16, got {signs.dtype} "
                           f"{tuple(signs.shape)}")
    R, C = x.shape
    packed = torch.empty(C, R // 2, dtype=torch.int8, device=x.device)
    scale = torch.empty(C, R // 16, dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        _lib.call("quantize_int4_cols", x.data_ptr(), x.stride(0), R, C,
                  signs.data_ptr() if signs is not None else None, 1 if sr else 0, int(seed) & 0xFFFFFFFF,
                  packed.data_ptr(), scale.data_ptr(), _stream(x.device))
    return packed, scale


def int4_linear(x: torch.Tensor, w_packed: torch.Tensor, w_scale: torch.Tensor, bias: torch.Tensor | None = None,
                rotation_group: int = 0) -> torch.Tensor:
    """x [..., K] float, packed weights from quantize_pack_int4 (folded through
    the same rotation when rotation_group != 0), bias in x.dtype or None ->
    [..., N] in x.dtype (signature of ops.py:167)."""
    shape = x.shape
    K = shape[-1]
    x2d = x.reshape(-1, K)
    if rotation_group:
        x2d = hadamard_rotate(x2d, rotation_group, torch.bfloat16)  # the GEMM's bf16 operand, one pass
    out = gemm_w4a16(x2d, w_packed, w_scale, bias, x.dtype)
    return out.reshape(*shape[:-1], w_packed.shape[0])


_exact_ws_lock = threading.Lock()
_exact_workspaces: dict = {}


def _exact_workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    """Scratch of the integer-exact GEMM per (device, stream): the e5m2 copy of
    A and its transposed scales, rewritten by every call (no state kept)."""
    key = (device.index, stream)
    with _exact_ws_lock:
        ws = _exact_workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _exact_workspaces[key] = ws
        return ws


def gemm_int4(A_packed: torch.Tensor, A_scale: torch.Tensor, B_packed: torch.Tensor, B_scale: torch.Tensor,
              bias: torch.Tensor | None, out_dtype: torch.dtype, splits: int = 0, qblock: int = 32) -> torch.Tensor:
    """The reference's block-scaled int4 GEMM op (``ext.gemm_int4``,
    binding.cpp:73-112): same arguments, checks and messages, and the same
    result bit for bit. A_packed / A_scale come from ``quantize_int4`` (int4
    activations), B is the packed weight; per output the fp32 chain
    acc = fmaf(dot, a_scale * b_scale, acc) runs over 32-element blocks (two
    16-element halves for qblock=16, int4_gemm_scaled.hip:147-160), each of
    the ``splits`` K slices from zero, slices summed in order, then the bias
    (splits=0: the reference's auto_splits, see ``gemm_int4_auto_splits``).
    The block dot products run on the tensor cores (C ABI ``w4a4_gemm_exact``)."""
    if not (A_packed.is_cuda and B_packed.is_cuda):
        raise RuntimeError("inputs must be on device")
    if A_packed.device != B_packed.device:
        raise RuntimeError("A and B must be on the same device")
    if A_packed.dtype != torch.int8 or B_packed.dtype != torch.int8:
        raise RuntimeError("packed tensors must be int8")
    if not (A_packed.dim() == 2 and B_packed.dim() == 2 and A_packed.shape[1] == B_packed.shape[1]
            and A_packed.shape[1] % 16 == 0):
        raise RuntimeError(f"expected A [M, K/2], B [N, K/2], K % 32 == 0; got A {tuple(A_packed.shape)} "
                           f"B {tuple(B_packed.shape)}")
    if A_scale.dtype != torch.float32 or B_scale.dtype != torch.float32:
        raise RuntimeError("scales must be float32")
    if qblock not in (32, 16):
        raise RuntimeError(f"qblock must be 32 or 16, got {qblock}")
    M, N, K = A_packed.shape[0], B_packed.shape[0], A_packed.shape[1] * 2
    if A_scale.numel() != M * K // qblock or B_scale.numel() != N * K // qblock:
        raise RuntimeError(f"scales must be [M, K/{qblock}] / [N, K/{qblock}] = {M * K // qblock} / "
                           f"{N * K // qblock} elements, got {A_scale.numel()} / {B_scale.numel()}")
    dev = A_packed.device
    C = torch.empty(M, N, dtype=out_dtype, device=dev)
    if M == 0:
        return C
    if bias is not None:
        if bias.dtype != out_dtype:
            raise RuntimeError(f"bias dtype {bias.dtype} != out dtype {out_dtype}")
        bias = bias.to(dev).contiguous()
    if splits < 0 or splits > 8:
        raise RuntimeError(f"splits must be in [0, 8], got {splits}")
    A, B = A_packed.contiguous(), B_packed.contiguous()
    As, Bs = A_scale.contiguous(), B_scale.contiguous()
    with torch.cuda.device(dev):
        st = _stream(dev)
        nbytes = int(_lib.load().w4a4_gemm_exact_workspace_bytes(M, N, K, qblock))
        ws = _exact_workspace(dev, st, nbytes)
        _call_gemm("w4a4_gemm_exact", dev, A.data_ptr(), As.data_ptr(), B.data_ptr(), Bs.data_ptr(), qblock,
                   bias.data_ptr() if bias is not None else None, C.data_ptr(), _dtype_code(out_dtype), M, N, K,
                   int(splits), ws.data_ptr(), ws.numel(), st)
    return C


def gemm_int8(A: torch.Tensor, A_scale: torch.Tensor, B: torch.Tensor, B_scale: torch.Tensor,
              bias: torch.Tensor | None, out_dtype: torch.dtype, config: int = 0) -> torch.Tensor:
    """The reference's block-scaled int8 GEMM op (``ext.gemm_int8``,
    binding.cpp:190-217), same arguments and checks: A / A_scale from
    ``quantize_int8`` (int8 activations), B int8 [N, K] with float32 block
    scales [N, K/32]. The A codes times their block scales are rounded once to
    bf16 and multiplied on the W8A16 tensor-core kernel, matching the
    reference's integer-block GEMM within bf16 rounding. ``config`` (the
    reference's gfx906 tile choice) is checked and otherwise unused."""
    if not (A.is_cuda and B.is_cuda):
        raise RuntimeError("inputs must be on device")
    if config < 0 or config > 3:
        raise RuntimeError(f"config must be in [0, 3], got {config}")
    if A.device != B.device:
        raise RuntimeError("A and B must be on the same device")
    if A.dtype != torch.int8 or B.dtype != torch.int8:
        raise RuntimeError("A and B must be int8")
    if not (A.dim() == 2 and B.dim() == 2 and A.shape[1] == B.shape[1] and A.shape[1] % 32 == 0):
        raise RuntimeError(f"expected A [M, K], B [N, K], K % 32 == 0; got A {tuple(A.shape)} B {tuple(B.shape)}")
    M, N, K = A.shape[0], B.shape[0], A.shape[1]
    if A_scale.dtype != torch.float32 or B_scale.dtype != torch.float32:
        raise RuntimeError("scales must be float32")
    if A_scale.numel() != M * (K // 32) or B_scale.numel() != N * (K // 32):
        raise RuntimeError(f"scales must be [M, K/32] / [N, K/32], got {tuple(A_scale.shape)} / {tuple(B_scale.shape)}")
    if M == 0:
        return torch.empty(0, N, dtype=out_dtype, device=A.device)
    xa = (A.float().reshape(M, K // 32, 32) * A_scale.reshape(M, K // 32, 1)).reshape(M, K).to(torch.bfloat16)
    return gemm_w8a16(xa, B, B_scale.reshape(N, K // 32), bias, out_dtype)


def int4_linear_w4a4(x: torch.Tensor, w_packed: torch.Tensor, w_scale: torch.Tensor, bias: torch.Tensor | None = None,
                     rotation_group: int = 0) -> torch.Tensor:
    """The reference's own ``int4_linear`` (ops.py:167-183), bit for bit: the
    activation is quantized to int4 per 32-block with ``quantize_int4``
    (int4_gemm_scaled.hip:197-220) and multiplied with the packed weights by
    the integer-exact ``gemm_int4`` (default split plan), bias in x.dtype."""
    shape = x.shape
    K = shape[-1]
    x2d = x.reshape(-1, K)
    if rotation_group:
        x2d = hadamard_rotate(x2d, rotation_group, torch.float32)  # fp32, as the reference quantizes
    pa, sa = quantize_int4(x2d.contiguous())
    out = gemm_int4(pa, sa, w_packed, w_scale.float(), bias, x.dtype)
    return out.reshape(*shape[:-1], w_packed.shape[0])


# ---------------------------------------------------------------------------
# custom_operations integration (reference ops.py:186-276)
# ---------------------------------------------------------------------------
try:  # ComfyUI present: subclass its op set exactly like the reference
    import comfy.ops as _comfy_ops  # type: ignore

    _OpsBase = _comfy_ops.disable_weight_init
except Exception:  # standalone use (tests, benches): a plain container class
    class _OpsBase:  # noqa: D401 - stand-in for comfy.ops.disable_weight_init
        """Stand-in base when ComfyUI is not importable."""


class Gfx906Int4Ops(_OpsBase):
    class Linear(torch.nn.Module):
        def __init__(self, in_features, out_features, bias=True, device=None, dtype=None, rotation_group=0):
            super().__init__()
            self.in_features = in_features
            self.out_features = out_features
            self.rotation_group = rotation_group
            # Layers narrower than one quant block stay float (ops.py:206-212).
            self.quantized = in_features % BLOCK == 0 and in_features >= BLOCK
            if self.quantized:
                self.register_buffer("weight_q4", torch.empty(out_features, in_features // 2, dtype=torch.int8,
                                                              device=device))
                self.register_buffer("weight_scale", torch.empty(out_features, in_features // BLOCK,
                                                                 dtype=torch.float32, device=device))
            else:
                self.weight = torch.nn.Parameter(torch.empty(out_features, in_features, device=device, dtype=dtype))
            if bias:
                self.bias = torch.nn.Parameter(torch.empty(out_features, device=device, dtype=dtype))
            else:
                self.register_parameter("bias", None)
            self._scale_cache = None  # (device, version, ptr, fp16 copy or False)

        quantize_device = None
        quantized_on_load = 0
        # True: the reference's W4A4 numerics (int4_linear_w4a4) instead of
        # the weight-only W4A16 product
        activation_quant = False

        def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                                  error_msgs):
            key = prefix + "weight"
            if self.quantized and self.quantize_device is not None and key in state_dict:
                w = state_dict.pop(key)
                if w.dtype not in (torch.float32, torch.float16, torch.bfloat16) or \
                        tuple(w.shape) != (self.out_features, self.in_features):
                    raise RuntimeError(f"{key}: expected a float [{self.out_features}, {self.in_features}] weight, "
                                       f"got {w.dtype} {tuple(w.shape)}")
                w_float = w.to(self.quantize_device).float()
                if self.rotation_group:
                    R = get_group_rotation(self.in_features, self.rotation_group, w_float.device)
                    w_float = apply_group_rotation(w_float, R, self.rotation_group)
                packed, scale = quantize_pack_int4(w_float, BLOCK)
                state_dict[prefix + "weight_q4"] = packed.to(w.device)
                state_dict[prefix + "weight_scale"] = scale.to(w.device)
                type(self).quantized_on_load += 1
            self._scale_cache = None
            super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                                          error_msgs)

        def _device_scale(self, weight_scale: torch.Tensor) -> torch.Tensor:
            """The scale buffer the kernel reads: an fp16 copy when every fp32
            scale is exactly an fp16 value (halves scale traffic; identical
            results), else the fp32 buffer itself. Cached per buffer version."""
            key = (weight_scale.device, weight_scale._version, weight_scale.data_ptr())
            c = self._scale_cache
            if c is not None and c[0] == key:
                return c[1] if c[1] is not None else weight_scale
            s16 = scales_to_f16_if_exact(weight_scale) if self.in_features % 64 == 0 else None
            self._scale_cache = (key, s16)
            return s16 if s16 is not None else weight_scale

        def forward(self, x):
            if not self.quantized:
                bias = self.bias.to(x.device, x.dtype) if self.bias is not None else None
                return torch.nn.functional.linear(x, self.weight.to(x.device, x.dtype), bias)
            weight_q4 = self.weight_q4.to(x.device)
            weight_scale = self.weight_scale.to(x.device)
            bias = self.bias.to(x.device, x.dtype) if self.bias is not None else None
            if self.activation_quant:  # the integer-exact GEMM takes the fp32 scales
                return int4_linear_w4a4(x, weight_q4, weight_scale, bias, self.rotation_group)
            if weight_scale is self.weight_scale:
                weight_scale = self._device_scale(weight_scale)
            return int4_linear(x, weight_q4, weight_scale, bias, self.rotation_group)


def make_load_quantizing_ops(base_ops, quantize_device, rotate):
    """custom_operations that quantize plain float Linear weights while the
    state dict loads (ops.py:263-276)."""
    class Linear(Gfx906Int4Ops.Linear):
        quantized_on_load = 0

        def __init__(self, in_features, out_features, bias=True, device=None, dtype=None):
            group = (choose_rotation_group(in_features) or 0) if rotate else 0
            super().__init__(in_features, out_features, bias, device, dtype, rotation_group=group)

    Linear.quantize_device = torch.device(quantize_device)
    return type("Gfx906Int4LoadOps", (base_ops,), {"Linear": Linear})
