"""The integer-exact W4A4 GEMM (C ABI ``w4a4_gemm_exact``, ``ops.gemm_int4``)
against the reference's integer-block GEMM, bit for bit.

The reference (int4_gemm_kernel, nodes/ComfyUI-Gfx906Int4/csrc/
int4_gemm_scaled.hip:53-191) computes per output the fp32 chain
acc = fmaf((float)dot, sa * sb, acc) over 32-element blocks (two 16-element
halves for qblock 16), each split-K slice from zero, slices summed in order,
then the bias. ``oracle.block_int_matmul`` restates it (and is itself pinned
bit for bit to the reference's compiled kernels in
test_reference_kernels_gpu.py); here our kernel must equal both exactly: fp32
outputs with np.array_equal, bf16 / fp16 outputs against the reference kernel
with torch.equal. Edge cases: ragged M / N / K (K not a multiple of 128),
M = 1, empty splits, explicit and automatic split counts, no bias.
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


def _operands(M, N, K, qblock, seed, dev):
    rng = np.random.default_rng(seed)
    ca, cb = rng.integers(-8, 8, (M, K)), rng.integers(-8, 8, (N, K))
    sa = ((np.abs(rng.normal(0, 1, (M, K // qblock))) + 0.05) * 0.2).astype(np.float32)
    sb = (np.abs(rng.normal(0, 0.01, (N, K // qblock))) + 1e-4).astype(np.float32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    return ca, cb, sa, sb, t(O.pack_int4_codes(ca)), t(sa), t(O.pack_int4_codes(cb)), t(sb)


@pytest.mark.parametrize("qblock", [32, 16])
@pytest.mark.parametrize("splits", [1, 3])
@pytest.mark.parametrize("M,N,K", [(70, 200, 768), (1, 64, 256), (129, 33, 1024), (300, 130, 864), (64, 128, 96)])
def test_exact_equals_oracle(cuda, qblock, splits, M, N, K):
    ca, cb, sa, sb, A, As, B, Bs = _operands(M, N, K, qblock, 100 + M + N + qblock + splits, cuda)
    bias = torch.linspace(-1, 1, N, device=cuda)
    got = ops.gemm_int4(A, As, B, Bs, bias, torch.float32, splits=splits, qblock=qblock).cpu().numpy()
    want = O.block_int_matmul(ca, sa, cb, sb, bias.cpu().numpy(), block=qblock, splits=splits)
    assert np.array_equal(got, want), (np.abs(got - want).max(), np.argwhere(got != want)[:5])


@pytest.mark.parametrize("qblock", [32, 16])
def test_exact_large_split_runs_in_cta(cuda, qblock):
    """A split problem too large for the parallel-slice partial buffer (8 x M x N
    x 4 bytes > 64 MB): the slices run one after another inside each CTA."""
    M, N, K = 1000, 2100, 512
    ca, cb, sa, sb, A, As, B, Bs = _operands(M, N, K, qblock, 55 + qblock, cuda)
    got = ops.gemm_int4(A, As, B, Bs, None, torch.float32, splits=3, qblock=qblock).cpu().numpy()
    want = O.block_int_matmul(ca, sa, cb, sb, None, block=qblock, splits=3)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("qblock", [32, 16])
def test_exact_no_bias_and_auto_splits(cuda, qblock):
    M, N, K = 5, 96, 2048
    ca, cb, sa, sb, A, As, B, Bs = _operands(M, N, K, qblock, 7 + qblock, cuda)
    s = ops.gemm_int4_auto_splits(M, N, K)
    assert s > 1  # a small problem: the reference's plan splits K
    got = ops.gemm_int4(A, As, B, Bs, None, torch.float32, qblock=qblock).cpu().numpy()
    want = O.block_int_matmul(ca, sa, cb, sb, None, block=qblock, splits=s)
    assert np.array_equal(got, want)


def test_exact_auto_splits_follow_reference_formula(cuda):
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count

    def ref(M, N, K):  # binding.cpp:36-43
        tiles = -(-M // 64) * -(-N // 64)
        slots = sms * 2
        if tiles >= slots:
            return 1
        max_splits = min(8, max(1, (-(-(K // 32) // 4)) // 8))
        return min((12 * slots + 5 * tiles - 1) // (5 * tiles), max_splits)

    for M, N, K in [(1, 3072, 3072), (16, 9216, 3072), (256, 3072, 3072), (4608, 3072, 15360), (64, 128, 96)]:
        assert ops.gemm_int4_auto_splits(M, N, K) == ref(M, N, K)


def test_exact_rejects_bad_arguments(cuda):
    _, _, _, _, A, As, B, Bs = _operands(4, 64, 256, 32, 1, cuda)
    with pytest.raises(RuntimeError, match="qblock must be 32 or 16"):
        ops.gemm_int4(A, As, B, Bs, None, torch.float32, qblock=64)
    with pytest.raises(RuntimeError, match="splits must be in"):
        ops.gemm_int4(A, As, B, Bs, None, torch.float32, splits=9)
    with pytest.raises(RuntimeError, match="bias dtype"):
        ops.gemm_int4(A, As, B, Bs, torch.zeros(64, device=cuda), torch.bfloat16)
    assert ops.gemm_int4(A[:0], As[:0], B, Bs, None, torch.float32).shape == (0, 64)


def test_int4_linear_w4a4_is_the_reference_forward(cuda):
    """int4_linear_w4a4 = quantize_int4 + the exact GEMM with the default plan
    (ops.py:167-183 of the reference), bit for bit against the oracle."""
    M, N, K = 37, 192, 1536
    g = torch.Generator().manual_seed(5)
    x = torch.randn(M, K, generator=g)
    w = torch.randn(N, K, generator=g) * 0.05
    p, s = O.quantize_pack_int4(w.numpy(), div_mode="recip")
    bias = torch.randn(N, generator=g)
    y = ops.int4_linear_w4a4(x.to(cuda), torch.from_numpy(p).to(cuda), torch.from_numpy(s).to(cuda),
                             bias.to(cuda)).cpu().numpy()
    pa, sa = O.quantize_pack_int4(x.numpy(), div_mode="recip")
    want = O.block_int_matmul(O.unpack_int4_codes(pa), sa, O.unpack_int4_codes(p), s, bias.numpy(),
                              splits=ops.gemm_int4_auto_splits(M, N, K))
    assert np.array_equal(y, want)


@pytest.fixture(scope="module")
def ref(cuda):
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libgfx906_ref.so not built (needs the reference checkout at build time)")
    lib = ctypes.CDLL(REF_LIB)
    vp, i = ctypes.c_void_p, ctypes.c_int
    lib.ref_gemm_int4.argtypes = [i, i, vp, vp, vp, vp, vp, vp, i, i, i, i, vp, vp]
    return lib


def _ref_gemm(lib, A, As, B, Bs, bias, out_dtype, qblock, splits):
    M, N, K = A.shape[0], B.shape[0], A.shape[1] * 2
    C = torch.empty(M, N, dtype=out_dtype, device=A.device)
    ws = torch.empty(splits, M, N, dtype=torch.float32, device=A.device) if splits > 1 else None
    rc = lib.ref_gemm_int4(DT[out_dtype], qblock, A.data_ptr(), As.data_ptr(), B.data_ptr(), Bs.data_ptr(),
                           bias.data_ptr() if bias is not None else None, C.data_ptr(), M, N, K // 32, splits,
                           ws.data_ptr() if ws is not None else None, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    return C


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("qblock", [32, 16])
@pytest.mark.parametrize("M,N,K", [(3, 320, 1536), (300, 320, 1536), (1000, 640, 3072)])
def test_exact_equals_reference_kernel(cuda, ref, out_dtype, qblock, M, N, K):
    """Against the reference's own int4_gemm_kernel (+ splitk_reduce_kernel),
    compiled unmodified for this GPU, with the split count the default call uses."""
    _, _, _, _, A, As, B, Bs = _operands(M, N, K, qblock, 300 + M + qblock, cuda)
    bias = torch.linspace(-1, 1, N, device=cuda).to(out_dtype)
    splits = ops.gemm_int4_auto_splits(M, N, K)
    want = _ref_gemm(ref, A, As, B, Bs, bias, out_dtype, qblock, splits)
    got = ops.gemm_int4(A, As, B, Bs, bias, out_dtype, qblock=qblock)
    assert torch.equal(got, want), (got.float() - want.float()).abs().max().item()


@pytest.mark.parametrize("M", [4608, 16, 1])
@pytest.mark.parametrize("name,K,N", [("qkv", 3072, 9216), ("mlp_down", 12288, 3072)])
def test_exact_flux_full_size_equals_reference_kernel(cuda, ref, name, K, N, M):
    """Full-size Flux shapes, every output element, bf16 output, the default
    split plan (M = 4608: one slice; M = 16 / 1: the reference splits K 3-8 ways
    and the slices run as parallel work items): the quantize_int4 activations
    of a seeded N(0,1) x and RTN weights against the reference's kernel."""
    g = torch.Generator().manual_seed(K + N + M)
    x = torch.randn(M, K, generator=g).to(cuda)
    w = (torch.randn(N, K, generator=g) * 0.02).to(cuda)
    A, As = ops.quantize_int4(x)
    B, Bs = ops.quantize_int4(w)
    splits = ops.gemm_int4_auto_splits(M, N, K)
    want = _ref_gemm(ref, A, As, B, Bs, None, torch.bfloat16, 32, splits)
    got = ops.gemm_int4(A, As, B, Bs, None, torch.bfloat16)
    assert torch.equal(got, want)
