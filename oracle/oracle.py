"""CPU restatement (numpy) of the reference's int4 / int8 weight path.

TEST INFRASTRUCTURE ONLY: this module is the checker the GPU kernels are
compared against and the CPU stand-in timed as the reference's CPU path. The
product package never imports it.

Pinning: every function below is checked against golden vectors that
``tests/golden/make_golden.py`` produced by importing and running the
reference's own Python (``nodes/ComfyUI-Gfx906Int4/ops.py`` with a one-class
``comfy.ops`` stub, ``nodes.py`` with module stubs, and the harness helpers
``develop/experiments/2026-10-11/int4_train_test.py:46-52`` /
``develop/harness/bench_int8.py:32-33`` extracted verbatim). The reference's
HIP quantizers and block-scaled integer GEMMs (``int4_gemm_scaled.hip``,
``int8_gemm.hip``) are gfx906 code; ``oracle/build_ref.py`` compiles those
sources unmodified for the B200 against a HIP stand-in header
(``oracle/hip_shim``), and ``tests/test_reference_kernels_gpu.py`` pins
``quantize_pack_int4`` (div_mode "recip"), ``quantize_int8`` and
``block_int_matmul`` bit for bit against the reference's own kernels run
there.

Layouts (reference ``ops.py:108-126``, ``csrc/int4_gemm_scaled.hip:6-10``):
  * native int4: int8 ``[N, K/2]``, two's-complement nibbles, interleaved:
    byte j low nibble = element 2j, high nibble = element 2j+1, i.e. element
    e of every 32-chunk is nibble e%8 of little-endian 32-bit word e/8;
    scales fp32 ``[N, K/32]``.
  * ggml Q4_0 (ingest, ``ops.py:129-164``): 18-byte blocks, fp16 ``d`` then
    16 bytes of offset-8 nibbles in split-half order (byte i low = element i,
    high = element i+16); value = (u - 8) * d.
"""
from __future__ import annotations

import numpy as np

BLOCK = 32
Q4_0_BLOCK_BYTES = 18

__all__ = [
    "BLOCK", "f32_to_bf16_bits", "bf16_bits_to_f32", "round_to_bf16", "f32_to_f16_bits",
    "quantize_pack_int4", "repack_q4_0_native", "dequant_int4", "dequant_int4_bf16_bits",
    "quantize_dequantize_int4", "build_q4_0_bytes", "w4a16_matmul", "quantize_int8",
    "dequant_int8", "w8a16_matmul", "parity_metrics", "unpack_int4_codes", "pack_int4_codes",
    "torch_cpu_dequant", "torch_cpu_w4a16", "w4a16_matmul_bf16w", "w4a4_matmul", "block_int_matmul",
    "build_q8_0_bytes", "repack_q8_0", "lowbias32", "hash_uniform", "quant_block16", "quantize_int4_rows",
    "quantize_int4_cols", "hadamard16",
]


# ---------------------------------------------------------------------------
# float helpers
# ---------------------------------------------------------------------------
def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16, returned as uint16 bit patterns
    (torch's ``Tensor.to(torch.bfloat16)`` rule for finite values)."""
    b = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_to_bf16(a: np.ndarray) -> np.ndarray:
    """fp32 values rounded to the nearest bf16 (RNE), returned as fp32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(a))


def f32_to_f16_bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).astype(np.float16).view(np.uint16)


# ---------------------------------------------------------------------------
# int4 packing (reference ops.py:108-164)
# ---------------------------------------------------------------------------
def pack_int4_codes(codes: np.ndarray) -> np.ndarray:
    """codes int [..., K] in [-8, 7] -> int8 [..., K/2], interleaved
    two's-complement nibbles (ops.py:119-121)."""
    c = np.asarray(codes).astype(np.int32)
    lo = c[..., 0::2] & 0xF
    hi = c[..., 1::2] & 0xF
    return (lo | (hi << 4)).astype(np.uint8).view(np.int8)


def unpack_int4_codes(packed: np.ndarray) -> np.ndarray:
    """int8 [..., K/2] -> int32 codes [..., K] in [-8, 7]; the exact inverse of
    ``pack_int4_codes`` (int4_train_test.py:46-51 reads the same layout as
    nibble e%8 of word e/8)."""
    p = np.ascontiguousarray(packed).view(np.uint8).astype(np.int32)
    nib = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.int32)
    nib[..., 0::2] = p & 0xF
    nib[..., 1::2] = (p >> 4) & 0xF
    return np.where(nib > 7, nib - 16, nib)


def quantize_pack_int4(t: np.ndarray, block: int = BLOCK, div_mode: str = "true"):
    """Reference ``ops.quantize_pack_int4`` (ops.py:108-126).

    t: float array [..., K] (already float32-representable: fp32, or fp16 /
    bf16 values widened exactly, as ``.float()`` does at ops.py:114).
    Returns (packed int8 [..., K/2], scale float32 [..., K/block]).

    div_mode selects how ``amax / 7.0`` is evaluated:
      "true"  -- an IEEE fp32 division: torch's CPU kernel (checked against
                 the reference run on CPU in the golden fixtures);
      "recip" -- ``amax * (1/7)``: torch's CUDA kernel for a tensor divided by
                 a Python scalar, and the reference's own HIP quantizer
                 (int4_gemm_scaled.hip:210-211).
    ``t / scale`` is a true division in both (a tensor divisor), and
    ``torch.round`` is round-half-even (numpy ``rint``).
    """
    t = np.asarray(t, dtype=np.float32)
    K = t.shape[-1]
    assert K % block == 0, f"last dim {K} not divisible by block {block}"
    tb = t.reshape(-1, K // block, block)
    amax = np.maximum(np.abs(tb).max(axis=-1, keepdims=True), np.float32(1e-8))
    if div_mode == "true":
        scale = (amax / np.float32(7.0)).astype(np.float32)
    elif div_mode == "recip":
        scale = (amax * (np.float32(1.0) / np.float32(7.0))).astype(np.float32)
    else:
        raise ValueError(f"div_mode must be 'true' or 'recip', got {div_mode!r}")
    codes = np.clip(np.rint(tb / scale), -8, 7).astype(np.int32).reshape(-1, K)
    packed = pack_int4_codes(codes)
    rows = t.shape[:-1]
    return (np.ascontiguousarray(packed.reshape(*rows, K // 2)),
            np.ascontiguousarray(scale.reshape(*rows, K // block)))


def repack_q4_0_native(raw: np.ndarray, out_features: int, in_features: int, block: int = BLOCK):
    """Reference ``ops.repack_q4_0_native`` (ops.py:129-164): a lossless bit
    shuffle of ggml Q4_0 blocks into the native layout. native nibble =
    (u - 8) & 0xF, fp32 scale = float(fp16 d)."""
    nb = in_features // block
    total = out_features * nb
    blocks = np.ascontiguousarray(raw).view(np.uint8).reshape(total, Q4_0_BLOCK_BYTES)
    scale = blocks[:, :2].copy().view(np.float16).reshape(total).astype(np.float32)
    qs = blocks[:, 2:].astype(np.int32)
    lo = ((qs & 0xF) - 8) & 0xF
    hi = (((qs >> 4) & 0xF) - 8) & 0xF
    elems = np.empty((total, block), dtype=np.int32)
    elems[:, : block // 2] = lo
    elems[:, block // 2:] = hi
    packed = (elems[:, 0::2] | (elems[:, 1::2] << 4)).astype(np.uint8).view(np.int8)
    return (np.ascontiguousarray(packed.reshape(out_features, in_features // 2)),
            np.ascontiguousarray(scale.reshape(out_features, nb)))


def build_q4_0_bytes(u: np.ndarray, d_f16: np.ndarray, block: int = BLOCK) -> np.ndarray:
    """Serialise offset-8 codes u uint8 [N, K] (0..15) and fp16 scales
    [N, K/32] into raw ggml Q4_0 bytes (the format ops.py:138-140 reads)."""
    N, K = u.shape
    nb = K // block
    ub = np.asarray(u, dtype=np.uint8).reshape(N * nb, block)
    out = np.empty((N * nb, Q4_0_BLOCK_BYTES), dtype=np.uint8)
    out[:, :2] = np.asarray(d_f16, dtype=np.float16).reshape(N * nb, 1).view(np.uint8).reshape(N * nb, 2)
    out[:, 2:] = (ub[:, : block // 2] & 0xF) | ((ub[:, block // 2:] & 0xF) << 4)
    return out.reshape(-1)


def build_q8_0_bytes(q: np.ndarray, d_f16: np.ndarray, block: int = BLOCK) -> np.ndarray:
    """ggml Q8_0 blocks (third-party format, ggml's ``block_q8_0``: fp16 d then
    32 int8 codes, value = q * d) from int8 codes q [N, K] and fp16 d [N, K/32]."""
    N, K = q.shape
    nb = K // block
    out = np.empty((N, nb, 2 + block), dtype=np.uint8)
    out[:, :, :2] = np.asarray(d_f16, np.float16).reshape(N, nb, 1).view(np.uint8).reshape(N, nb, 2)
    out[:, :, 2:] = np.asarray(q, np.int8).reshape(N, nb, block).view(np.uint8)
    return out.reshape(-1)


def repack_q8_0(raw: np.ndarray, out_features: int, in_features: int, block: int = BLOCK):
    """Q8_0 bytes -> (int8 [N, K], float32 [N, K/32] = d), lossless."""
    nb = in_features // block
    b = np.asarray(raw, np.uint8).reshape(out_features, nb, 2 + block)
    d = b[:, :, :2].copy().view(np.float16).reshape(out_features, nb).astype(np.float32)
    q = b[:, :, 2:].copy().view(np.int8).reshape(out_features, in_features)
    return q, d


def dequant_int4(packed: np.ndarray, scale: np.ndarray, block: int = BLOCK) -> np.ndarray:
    """Reference dequant (int4_train_test.py:46-52, nodes.py:51): fp32
    ``code * scale``, one IEEE multiply per element."""
    codes = unpack_int4_codes(packed).astype(np.float32)
    s = np.asarray(scale, dtype=np.float32)
    return (codes.reshape(s.shape + (block,)) * s[..., None]).reshape(codes.shape)


def dequant_int4_bf16_bits(packed: np.ndarray, scale: np.ndarray, block: int = BLOCK) -> np.ndarray:
    """The bf16 weight the W4A16 emulation feeds its matmul: the fp32 product
    rounded to bf16 (nodes.py:51-52 ``(q * scale).to(bfloat16)``)."""
    return f32_to_bf16_bits(dequant_int4(packed, scale, block))


def quantize_dequantize_int4(t: np.ndarray, block: int = BLOCK) -> np.ndarray:
    """Reference ``nodes.quantize_dequantize_int4`` (nodes.py:43-52), fp32
    result before its final ``.to(t.dtype)``."""
    t = np.asarray(t, dtype=np.float32)
    K = t.shape[-1]
    if K % block != 0:
        return t
    tb = t.reshape(-1, K // block, block)
    amax = np.maximum(np.abs(tb).max(axis=-1, keepdims=True), np.float32(1e-8))
    scale = (amax / np.float32(7.0)).astype(np.float32)
    # q stays a float here (no packing), so a negative input that rounds to
    # zero keeps its sign: -0.0 * scale = -0.0, exactly as nodes.py:50-52.
    q = np.clip(np.rint(tb / scale), np.float32(-8), np.float32(7)).astype(np.float32)
    return (q * scale).reshape(t.shape)


# ---------------------------------------------------------------------------
# int8 (reference csrc/int8_gemm.hip:217-246, develop/harness/bench_int8.py:32-43)
# ---------------------------------------------------------------------------
def quantize_int8(x: np.ndarray, block: int = BLOCK):
    """Restatement of ``quantize_int8_kernel`` (int8_gemm.hip:217-246): per
    32-block s = max(amax, 1e-8) * (1/127) (reciprocal multiply, as the
    kernel writes it), q = clamp(rint(v / s), -127, 127). Parity unpinned
    against the HIP kernel itself (it cannot run here)."""
    x = np.asarray(x, dtype=np.float32)
    K = x.shape[-1]
    xb = x.reshape(-1, K // block, block)
    amax = np.maximum(np.abs(xb).max(axis=-1, keepdims=True), np.float32(1e-8))
    s = (amax * (np.float32(1.0) / np.float32(127.0))).astype(np.float32)
    q = np.clip(np.rint(xb / s), -127, 127).astype(np.int8).reshape(x.shape)
    return q, np.ascontiguousarray(s.reshape(x.shape[:-1] + (K // block,)))


def dequant_int8(q: np.ndarray, s: np.ndarray, block: int = BLOCK) -> np.ndarray:
    """bench_int8.py:32-33: ``q.float().reshape(rows, -1, 32) * s[..., None]``."""
    qf = np.asarray(q).astype(np.float32)
    return (qf.reshape(qf.shape[0], -1, block) * np.asarray(s, np.float32)[..., None]).reshape(qf.shape)


# ---------------------------------------------------------------------------
# GEMM oracles (fp32 dequant then fp32 matmul: bench_int8.py:43)
# ---------------------------------------------------------------------------
def w4a16_matmul(x: np.ndarray, packed: np.ndarray, scale: np.ndarray, bias=None, block: int = BLOCK) -> np.ndarray:
    """``Y = X.float() @ dequant(W).T (+ bias)`` in fp32 (``block`` = the scale
    block, 32 or the reference's qblock=16)."""
    w = dequant_int4(packed, scale, block)
    y = np.asarray(x, dtype=np.float32) @ w.T
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float32)
    return y


def w4a16_matmul_bf16w(x: np.ndarray, packed: np.ndarray, scale: np.ndarray, bias=None,
                       block: int = BLOCK) -> np.ndarray:
    """``Y = X.float() @ bf16(dequant(W)).T`` in fp32: the W4A16 emulation with
    the weight rounded to bf16 (nodes.py:51-52 for a bf16 model). The
    tensor-core kernel multiplies exactly these operands, so it matches this
    oracle up to fp32 accumulation order."""
    w = round_to_bf16(dequant_int4(packed, scale, block))
    y = np.asarray(x, dtype=np.float32) @ w.T
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float32)
    return y


def _fmaf(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    """C's fmaf on float32 arrays: a * b + c with one rounding to float32. The
    product of an integer dot (<= 43 bits with the fp32 factor) is exact in
    x86 extended precision (64-bit mantissa); the sum is rounded there and
    then to float32, which equals a single rounding except when the extended
    sum lands exactly on a float32 tie after being rounded itself."""
    ld = np.longdouble
    return (np.asarray(a).astype(ld) * np.asarray(b).astype(ld) + np.asarray(c).astype(ld)).astype(np.float32)


def block_int_matmul(ca: np.ndarray, sa: np.ndarray, cb: np.ndarray, sb: np.ndarray, bias=None,
                     block: int = BLOCK, splits: int = 1) -> np.ndarray:
    """The reference's block-scaled integer GEMM (gemm_int4 and gemm_int8:
    int4_gemm_scaled.hip:53-191, int8_gemm.hip:176-194): integer codes
    ca [M, K], cb [N, K], fp32 block scales sa [M, K/block], sb [N, K/block]
    (block 32, or 16 for gemm_int4's qblock=16, where each 32-element load
    splits into two rescaled 16-element dots, int4_gemm_scaled.hip:153-160);
    per block the exact integer dot product, ``acc = fmaf(dot, sa * sb, acc)``
    in block order from acc = 0, bias added last in fp32. With ``splits`` > 1
    (gemm_int4's split-K, int4_gemm_scaled.hip:228-246) the K stages of 128
    elements are cut into ceil(stages / splits)-stage slices, each slice's
    partial is such a chain, and the partials are summed in slice order from
    0.0 before the bias (splitk_reduce_kernel, :182-191)."""
    ca = np.asarray(ca).astype(np.int64)
    cb = np.asarray(cb).astype(np.int64)
    M, K = ca.shape
    N = cb.shape[0]
    nb = K // block
    dots = np.einsum("mbk,nbk->mnb", ca.reshape(M, nb, block), cb.reshape(N, nb, block))  # exact integers
    sab = (np.asarray(sa, np.float32).reshape(M, nb)[:, None, :] *
           np.asarray(sb, np.float32).reshape(N, nb)[None, :, :]).astype(np.float32)
    k_stages = -(-K // 128)
    per = -(-k_stages // splits)
    bounds = [(s * per * 128 // block, min(nb, (s + 1) * per * 128 // block)) for s in range(splits)]
    parts = []
    for b0, b1 in bounds:
        acc = np.zeros((M, N), dtype=np.float32)
        for b in range(b0, b1):
            acc = _fmaf(dots[:, :, b].astype(np.float32), sab[:, :, b], acc)
        parts.append(acc)
    if splits == 1:
        out = parts[0]
    else:
        out = np.zeros((M, N), dtype=np.float32)
        for p_ in parts:
            out = (out + p_).astype(np.float32)
    if bias is not None:
        out = (out + np.asarray(bias, dtype=np.float32)).astype(np.float32)
    return out


def w4a4_matmul(x: np.ndarray, packed: np.ndarray, scale: np.ndarray, bias=None, block: int = BLOCK) -> np.ndarray:
    """The reference's production ``Linear.forward`` numerics (W4A4): the
    activation is quantized per 32-block like ``quantize_int4``
    (int4_gemm_scaled.hip:197-220: scale = amax * (1/7), codes = RNE(x / s)
    clamped to [-8, 7]); each 32-block contributes its exact integer dot
    product times ``sa * sb`` (an fp32 product), accumulated in block order
    with one rounding per block (``acc = fmaf(dot, sa * sb, acc)``,
    int4_gemm_scaled.hip:147-152, one split); bias added last
    (int4_gemm_scaled.hip:170-178). The HIP kernel itself cannot run here, so
    this restatement is unpinned beyond its quantizer."""
    x = np.asarray(x, dtype=np.float32)
    pa, sa = quantize_pack_int4(x, block, div_mode="recip")
    return block_int_matmul(unpack_int4_codes(pa), sa, unpack_int4_codes(np.asarray(packed)), scale, bias, block)


def w8a16_matmul(x: np.ndarray, q: np.ndarray, s: np.ndarray, bias=None) -> np.ndarray:
    w = dequant_int8(q, s)
    y = np.asarray(x, dtype=np.float32) @ w.T
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float32)
    return y


def torch_cpu_dequant(packed, scale, block: int = BLOCK):
    """The reference's dequant as torch CPU ops (int4_train_test.py:46-52):
    words >> shifts & 0xF, sign fix, ``codes * scale.repeat_interleave``.
    Used as the timed CPU path (multi-threaded like the reference's)."""
    import torch
    words = packed.contiguous().view(torch.int32)
    shifts = torch.arange(0, 32, 4, dtype=torch.int32)
    nib = (words[..., None] >> shifts) & 0xF
    codes = torch.where(nib > 7, nib - 16, nib).reshape(packed.shape[0], -1).float()
    return codes * scale.repeat_interleave(block, dim=1)


def torch_cpu_w4a16(x, packed, scale, bias=None):
    """The reference's CPU torch path: dequant then fp32 ``torch.matmul``
    (bench_int8.py:43 pattern)."""
    import torch
    y = torch.matmul(x.float(), torch_cpu_dequant(packed, scale).t())
    return y + bias.float() if bias is not None else y


def parity_metrics(got: np.ndarray, ref: np.ndarray) -> dict:
    """The north-star parity measures: max|d| / max|ref| and the mean
    relative error defined as mean|d| / mean|ref|."""
    g = np.asarray(got, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    d = np.abs(g - r)
    max_ref = float(np.abs(r).max()) if r.size else 0.0
    mean_ref = float(np.abs(r).mean()) if r.size else 0.0
    return {
        "max_abs_over_max_ref": float(d.max()) / max_ref if max_ref > 0 else float(d.max() if d.size else 0.0),
        "mean_rel": float(d.mean()) / mean_ref if mean_ref > 0 else float(d.mean() if d.size else 0.0),
        "nonfinite": int((~np.isfinite(g)).sum()),
    }


# ---------------------------------------------------------------------------
# block-16 training quantizers (int4_train_quant.hip:16-123)
# ---------------------------------------------------------------------------
def lowbias32(x: np.ndarray) -> np.ndarray:
    """Chris Wellons' lowbias32 integer hash (the counter-based hash of
    int4_train_quant.hip:18-25), elementwise on uint32."""
    x = np.asarray(x, dtype=np.uint32).copy()
    x ^= x >> np.uint32(16)
    x = (x.astype(np.uint64) * 0x7FEB352D).astype(np.uint32)
    x ^= x >> np.uint32(15)
    x = (x.astype(np.uint64) * 0x846CA68B).astype(np.uint32)
    x ^= x >> np.uint32(16)
    return x


def hash_uniform(seed: int, element: np.ndarray) -> np.ndarray:
    """u in [0, 1) with 24 bits per (seed, 64-bit element index)
    (int4_train_quant.hip:27-31)."""
    e = np.asarray(element, dtype=np.uint64)
    inner = lowbias32((e & np.uint64(0xFFFFFFFF)).astype(np.uint32) ^ lowbias32((e >> np.uint64(32)).astype(np.uint32)))
    h = lowbias32(np.uint32(seed & 0xFFFFFFFF) ^ inner)
    return ((h >> np.uint32(8)).astype(np.float32) * np.float32(1.0 / 16777216.0)).astype(np.float32)


def quant_block16(v: np.ndarray, sr: bool, seed: int, first: np.ndarray):
    """16 values per row of v [B, 16] -> (codes int [B, 16], scale float32 [B])
    (int4_train_quant.hip:33-55): scale = max(amax, 1e-8) * (1/7) in fp32,
    t = v / scale, round half even or floor(t + u), clamp to [-8, 7]."""
    v = np.asarray(v, dtype=np.float32)
    amax = np.max(np.abs(v), axis=1)
    s = (np.maximum(amax, np.float32(1e-8)) * np.float32(1.0 / 7.0)).astype(np.float32)
    t = (v / s[:, None]).astype(np.float32)
    if sr:
        u = hash_uniform(seed, np.asarray(first, dtype=np.uint64)[:, None] + np.arange(16, dtype=np.uint64)[None, :])
        r = np.floor((t + u).astype(np.float32))
    else:
        r = np.rint(t)
    return np.clip(r, -8, 7).astype(np.int64), s


def hadamard16(v: np.ndarray, signs: np.ndarray) -> np.ndarray:
    """(H16 / 4) diag(signs) v for every row of v [B, 16]: four stages of
    fp32 pair sums / differences in the reference's order
    (int4_train_quant.hip:103-116)."""
    v = (np.asarray(v, dtype=np.float32) * np.asarray(signs, dtype=np.float32)[None, :]).astype(np.float32)
    h = 1
    while h < 16:
        v = v.copy()
        for i in range(16):
            if i & h == 0:
                a, b = v[:, i].copy(), v[:, i + h].copy()
                v[:, i] = (a + b).astype(np.float32)
                v[:, i + h] = (a - b).astype(np.float32)
        h <<= 1
    return (v * np.float32(0.25)).astype(np.float32)


def quantize_int4_rows(x: np.ndarray, sr: bool = False, seed: int = 0):
    """x [R, C] (fp16 values, C % 32 == 0) -> (packed int8 [R, C/2], scale
    float32 [R, C/16]), blocks of 16 along each row (quant_rows_b16,
    int4_train_quant.hip:57-85; element index r * C + column)."""
    x = np.asarray(x, dtype=np.float32)
    R, C = x.shape
    v = x.reshape(R * C // 16, 16)
    first = (np.arange(R, dtype=np.uint64)[:, None] * np.uint64(C) +
             np.arange(0, C, 16, dtype=np.uint64)[None, :]).reshape(-1)
    codes, s = quant_block16(v, sr, seed, first)
    return pack_int4_codes(codes.reshape(R, C)), s.reshape(R, C // 16)


def quantize_int4_cols(x: np.ndarray, signs=None, sr: bool = False, seed: int = 0):
    """x [R, C] (fp16 values, R % 32 == 0) -> (packed int8 [C, R/2], scale
    float32 [C, R/16]), blocks of 16 along each column of x, i.e. rows of x^T,
    optionally rotated by hadamard16 first (quant_cols_b16,
    int4_train_quant.hip:87-123; element index c * R + row)."""
    xt = np.ascontiguousarray(np.asarray(x, dtype=np.float32).T)  # [C, R]
    C, R = xt.shape
    v = xt.reshape(C * R // 16, 16)
    if signs is not None:
        v = hadamard16(v, signs)
    first = (np.arange(C, dtype=np.uint64)[:, None] * np.uint64(R) +
             np.arange(0, R, 16, dtype=np.uint64)[None, :]).reshape(-1)
    codes, s = quant_block16(v, sr, seed, first)
    return pack_int4_codes(codes.reshape(C, R)), s.reshape(C, R // 16)
