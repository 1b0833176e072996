"""Parity against the reference's OWN kernels, run on the B200.

``oracle/build_ref.py`` compiles the reference's gfx906 sources
(nodes/ComfyUI-Gfx906Int4/csrc/int4_gemm_scaled.hip and int8_gemm.hip)
unmodified with nvcc for sm_100a against a HIP stand-in header, into
``oracle/_ref/libgfx906_ref.so`` (built where the reference checkout exists;
it travels to the GPU box prebuilt). These tests use it to pin:

  * the numpy oracle, bit for bit: ``quantize_pack_int4`` (reciprocal-divide
    mode) against ``quantize_int4_kernel`` (int4_gemm_scaled.hip:197-220),
    ``quantize_int8`` against ``quantize_int8_kernel`` (int8_gemm.hip:217-246),
    ``block_int_matmul`` against ``int4_gemm_kernel`` with 32- and 16-element
    scale blocks and split-K (int4_gemm_scaled.hip:53-191) and
    ``int8_gemm_kernel`` (int8_gemm.hip:66-213) in all four tile configs;
  * this repository's kernels: the quantizers bit for bit, ``gemm_int4`` /
    ``gemm_int8`` (integer activations dequantized to bf16, tensor-core GEMM)
    within the north-star tolerance of the reference's integer-exact GEMMs.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle as O
from comfy_ui_gfx906_tools_b200 import ops

pytestmark = pytest.mark.gpu

REF_LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                       "libgfx906_ref.so")
DT = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


@pytest.fixture(scope="module")
def ref(cuda):
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libgfx906_ref.so not built (needs the reference checkout at build time)")
    lib = ctypes.CDLL(REF_LIB)
    vp, i, lg = ctypes.c_void_p, ctypes.c_int, ctypes.c_long
    lib.ref_quantize_int4.argtypes = [i, vp, vp, vp, lg, vp]
    lib.ref_quantize_int8.argtypes = [i, vp, vp, vp, lg, vp]
    lib.ref_gemm_int4.argtypes = [i, i, vp, vp, vp, vp, vp, vp, i, i, i, i, vp, vp]
    lib.ref_gemm_int8.argtypes = [i, i, vp, vp, vp, vp, vp, vp, i, i, i, vp]
    return lib


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _ptr(t):
    return t.data_ptr() if t is not None else None


def _x(rows, K, dtype, seed, dev):
    """Activations with the edge cases of a block quantizer: an all-zero block,
    exact .5 ties of x / scale, large magnitudes, tiny values."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, K, generator=g) * 2.0
    x[0, :32] = 0.0
    x[1, :32] = torch.arange(32).float() * 0.5 - 7.5       # ties against amax/7 multiples
    x[2, 32:64] = torch.randn(32, generator=g) * 1e4
    x[3, 64:96] = torch.randn(32, generator=g) * 1e-6
    return x.to(dtype).to(dev)


def ref_quantize_int4(lib, x):
    rows, K = x.shape
    p = torch.empty(rows, K // 2, dtype=torch.int8, device=x.device)
    s = torch.empty(rows, K // 32, dtype=torch.float32, device=x.device)
    assert lib.ref_quantize_int4(DT[x.dtype], x.data_ptr(), p.data_ptr(), s.data_ptr(), rows * K // 32, _stream()) == 0
    torch.cuda.synchronize()
    return p, s


def ref_quantize_int8(lib, x):
    rows, K = x.shape
    q = torch.empty(rows, K, dtype=torch.int8, device=x.device)
    s = torch.empty(rows, K // 32, dtype=torch.float32, device=x.device)
    assert lib.ref_quantize_int8(DT[x.dtype], x.data_ptr(), q.data_ptr(), s.data_ptr(), rows * K // 32, _stream()) == 0
    torch.cuda.synchronize()
    return q, s


def ref_gemm_int4(lib, A, As, B, Bs, bias, out_dtype, qblock, splits):
    M, N, K = A.shape[0], B.shape[0], A.shape[1] * 2
    C = torch.empty(M, N, dtype=out_dtype, device=A.device)
    ws = torch.empty(splits, M, N, dtype=torch.float32, device=A.device) if splits > 1 else None
    rc = lib.ref_gemm_int4(DT[out_dtype], qblock, A.data_ptr(), As.data_ptr(), B.data_ptr(), Bs.data_ptr(), _ptr(bias),
                           C.data_ptr(), M, N, K // 32, splits, _ptr(ws), _stream())
    assert rc == 0
    torch.cuda.synchronize()
    return C


def ref_gemm_int8(lib, A, As, B, Bs, bias, out_dtype, config):
    M, N, K = A.shape[0], B.shape[0], A.shape[1]
    C = torch.empty(M, N, dtype=out_dtype, device=A.device)
    rc = lib.ref_gemm_int8(DT[out_dtype], config, A.data_ptr(), As.data_ptr(), B.data_ptr(), Bs.data_ptr(), _ptr(bias),
                           C.data_ptr(), M, N, K // 32, _stream())
    assert rc == 0
    torch.cuda.synchronize()
    return C


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_quantize_int4_pins_oracle_and_ours(cuda, ref, dtype):
    x = _x(70, 512, dtype, 1, cuda)
    rp, rs = ref_quantize_int4(ref, x)
    op, os_ = O.quantize_pack_int4(x.float().cpu().numpy(), div_mode="recip")
    assert np.array_equal(rp.cpu().numpy(), op) and np.array_equal(rs.cpu().numpy(), os_)
    p, s = ops.quantize_int4(x)
    assert torch.equal(p, rp) and torch.equal(s, rs)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_quantize_int8_pins_oracle_and_ours(cuda, ref, dtype):
    x = _x(70, 512, dtype, 2, cuda)
    rq, rs = ref_quantize_int8(ref, x)
    oq, os_ = O.quantize_int8(x.float().cpu().numpy())
    assert np.array_equal(rq.cpu().numpy(), oq) and np.array_equal(rs.cpu().numpy(), os_)
    q, s = ops.quantize_int8(x)
    assert torch.equal(q, rq) and torch.equal(s, rs)


def _int4_operands(M, N, K, qblock, seed, dev):
    rng = np.random.default_rng(seed)
    ca, cb = rng.integers(-8, 8, (M, K)), rng.integers(-8, 8, (N, K))
    sa = ((np.abs(rng.normal(0, 1, (M, K // qblock))) + 0.05) * 0.2).astype(np.float32)
    sb = (np.abs(rng.normal(0, 0.01, (N, K // qblock))) + 1e-4).astype(np.float32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    return ca, cb, sa, sb, t(O.pack_int4_codes(ca)), t(sa), t(O.pack_int4_codes(cb)), t(sb)


@pytest.mark.parametrize("qblock", [32, 16])
@pytest.mark.parametrize("splits", [1, 3])
@pytest.mark.parametrize("M,N,K", [(70, 200, 768), (1, 64, 256), (129, 33, 1024)])
def test_gemm_int4_pins_oracle(cuda, ref, qblock, splits, M, N, K):
    """fp32 output: the oracle's fmaf chain equals the reference kernel bit for
    bit, with and without split-K, for both scale blocks, with a bias."""
    ca, cb, sa, sb, A, As, B, Bs = _int4_operands(M, N, K, qblock, 10 + M + qblock + splits, cuda)
    bias = torch.linspace(-1, 1, N, device=cuda)
    got = ref_gemm_int4(ref, A, As, B, Bs, bias, torch.float32, qblock, splits).cpu().numpy()
    want = O.block_int_matmul(ca, sa, cb, sb, bias.cpu().numpy(), block=qblock, splits=splits)
    assert np.array_equal(got, want), np.abs(got - want).max()


@pytest.mark.parametrize("qblock", [32, 16])
@pytest.mark.parametrize("M", [3, 300])
def test_our_gemm_int4_matches_reference_kernel(cuda, ref, qblock, M):
    """ops.gemm_int4 (exact bf16 dequant of the int4 activations, tensor-core
    GEMM) against the reference's integer-exact kernel: north-star bar."""
    N, K = 320, 1536
    ca, cb, sa, sb, A, As, B, Bs = _int4_operands(M, N, K, qblock, 20 + M + qblock, cuda)
    bias = torch.linspace(-1, 1, N, device=cuda).to(torch.bfloat16)
    want = ref_gemm_int4(ref, A, As, B, Bs, bias, torch.bfloat16, qblock, 1).float().cpu().numpy()
    got = ops.gemm_int4(A, As, B, Bs, bias, torch.bfloat16, qblock=qblock).float().cpu().numpy()
    m = O.parity_metrics(got, want)
    assert m["nonfinite"] == 0 and m["max_abs_over_max_ref"] <= 2e-2 and m["mean_rel"] <= 5e-3, m


@pytest.mark.parametrize("config", [0, 1, 2, 3])
@pytest.mark.parametrize("M,N,K", [(77, 96, 864), (3, 130, 96)])
def test_gemm_int8_pins_oracle_and_ours(cuda, ref, config, M, N, K):
    g = torch.Generator().manual_seed(config + M)
    x = torch.randn(M, K, generator=g).to(cuda)
    w = (torch.randn(N, K, generator=g) * 0.05).to(cuda)
    A, As = ops.quantize_int8(x)
    B, Bs = ops.quantize_int8(w)
    bias = torch.linspace(-1, 1, N, device=cuda)
    got = ref_gemm_int8(ref, A, As, B, Bs, bias, torch.float32, config).cpu().numpy()
    want = O.block_int_matmul(A.cpu().numpy(), As.cpu().numpy(), B.cpu().numpy(), Bs.cpu().numpy(), bias.cpu().numpy())
    assert np.array_equal(got, want), np.abs(got - want).max()
    ours = ops.gemm_int8(A, As, B, Bs, bias, torch.float32, config=config).cpu().numpy()
    m = O.parity_metrics(ours, got)
    assert m["nonfinite"] == 0 and m["max_abs_over_max_ref"] <= 2e-2 and m["mean_rel"] <= 5e-3, m
