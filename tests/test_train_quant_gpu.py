"""The int4 training backward: block-16 quantizers (ops.quantize_int4_rows /
quantize_int4_cols, C ABI quantize_int4_rows / quantize_int4_cols) and
train_linear (linear with the int4 backward, FrozenInt4Linear), against the
numpy oracle and the reference's own quantizer kernels
(nodes/ComfyUI-Gfx906Int4/csrc/int4_train_quant.hip compiled for this GPU by
oracle/build_ref.py), bit for bit."""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle as O
from comfy_ui_gfx906_tools_b200 import ops, train_linear

pytestmark = pytest.mark.gpu

REF_LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                       "libgfx906_ref.so")


def _x(R, C, seed, dev, pad=0):
    """fp16 [R, C] (rows C + pad apart) with block edge cases: an all-zero block,
    exact ties against amax/7 multiples, huge and tiny values."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(R, C + pad, generator=g) * 1.5
    x[0, :16] = 0.0
    if R >= 4 and C >= 48:
        x[1, :16] = torch.arange(16).float() * 0.5 - 3.5
        x[2, 16:32] = torch.randn(16, generator=g).clamp(-5, 5) * 1e4  # large, finite in fp16
        x[3, 32:48] = torch.randn(16, generator=g) * 1e-4
    return x.to(torch.float16).to(dev)[:, :C]


@pytest.fixture(scope="module")
def ref(cuda):
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libgfx906_ref.so not built (needs the reference checkout at build time)")
    lib = ctypes.CDLL(REF_LIB)
    vp, i, ll, u = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_uint
    lib.ref_quant_rows_b16.argtypes = [vp, ll, i, i, i, u, vp, vp, vp]
    lib.ref_quant_cols_b16.argtypes = [vp, ll, i, i, vp, i, u, vp, vp, vp]
    return lib


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("sr", [False, True])
@pytest.mark.parametrize("R,C,pad", [(64, 96, 0), (37, 256, 32), (1, 32, 0)])
def test_quantize_rows(cuda, ref, sr, R, C, pad):
    x = _x(R, C, 3 + R + pad, cuda, pad)
    p, s = ops.quantize_int4_rows(x, sr, 12345)
    op, os_ = O.quantize_int4_rows(x.float().cpu().numpy(), sr, 12345)
    assert np.array_equal(p.cpu().numpy(), op) and np.array_equal(s.cpu().numpy(), os_)
    rp = torch.empty_like(p)
    rs = torch.empty_like(s)
    assert ref.ref_quant_rows_b16(x.data_ptr(), x.stride(0), R, C, int(sr), 12345, rp.data_ptr(), rs.data_ptr(),
                                  _stream()) == 0
    torch.cuda.synchronize()
    assert torch.equal(p, rp) and torch.equal(s, rs)


@pytest.mark.parametrize("rht", [False, True])
@pytest.mark.parametrize("sr", [False, True])
@pytest.mark.parametrize("R,C,pad", [(64, 96, 0), (96, 40, 8), (32, 1, 7)])
def test_quantize_cols(cuda, ref, rht, sr, R, C, pad):
    x = _x(R, C, 7 + C + pad, cuda, pad)
    signs = train_linear._signs(cuda) if rht else None
    p, s = ops.quantize_int4_cols(x, signs, sr, 777)
    op, os_ = O.quantize_int4_cols(x.float().cpu().numpy(), signs.cpu().numpy() if rht else None, sr, 777)
    assert np.array_equal(p.cpu().numpy(), op) and np.array_equal(s.cpu().numpy(), os_)
    rp = torch.empty_like(p)
    rs = torch.empty_like(s)
    assert ref.ref_quant_cols_b16(x.data_ptr(), x.stride(0), R, C, signs.data_ptr() if rht else None, int(sr), 777,
                                  rp.data_ptr(), rs.data_ptr(), _stream()) == 0
    torch.cuda.synchronize()
    assert torch.equal(p, rp) and torch.equal(s, rs)


def test_quantize_rejects_bad_inputs(cuda):
    with pytest.raises(RuntimeError, match="fp16"):
        ops.quantize_int4_rows(torch.zeros(4, 32, device=cuda), False, 0)
    with pytest.raises(RuntimeError, match="C % 32"):
        ops.quantize_int4_rows(torch.zeros(4, 48, device=cuda, dtype=torch.float16), False, 0)
    with pytest.raises(RuntimeError, match="R % 32"):
        ops.quantize_int4_cols(torch.zeros(16, 32, device=cuda, dtype=torch.float16), None, False, 0)
    with pytest.raises(RuntimeError, match="signs"):
        ops.quantize_int4_cols(torch.zeros(32, 32, device=cuda, dtype=torch.float16), torch.ones(8, device=cuda),
                               False, 0)


@pytest.mark.parametrize("int4_fprop", [False, True])
def test_linear_int4_backward_matches_emulation(cuda, int4_fprop):
    """train_linear.linear: forward and both gradients against the same
    quantize + block-16 integer GEMM steps emulated by the oracle, bit for bit
    (seeds 1 and 2 for dgrad's and wgrad's stochastic rounding)."""
    T, K, N = 64, 96, 160
    g = torch.Generator().manual_seed(11)
    x = (torch.randn(T, K, generator=g)).to(torch.float16).to(cuda).requires_grad_(True)
    w = (torch.randn(N, K, generator=g) * 0.1).to(torch.float16).to(cuda).requires_grad_(True)
    dy = (torch.randn(T, N, generator=g)).to(torch.float16).to(cuda)
    train_linear._seed[0] = 0
    y = train_linear.linear(x, w, int4_fprop)
    y.backward(dy)
    xn, wn, gn = x.detach().float().cpu().numpy(), w.detach().float().cpu().numpy(), dy.float().cpu().numpy()
    signs = train_linear._signs(cuda).cpu().numpy()
    if int4_fprop:
        xq, xs = O.quantize_int4_rows(xn)
        wq, ws = O.quantize_int4_rows(wn)
        want_y = O.block_int_matmul(O.unpack_int4_codes(xq), xs, O.unpack_int4_codes(wq), ws, None, block=16,
                                    splits=ops.gemm_int4_auto_splits(T, N, K)).astype(np.float16)
        assert np.array_equal(y.detach().cpu().numpy(), want_y)
    gq, gs = O.quantize_int4_rows(gn, True, 1)
    wtq, wts = O.quantize_int4_cols(wn)
    want_dx = O.block_int_matmul(O.unpack_int4_codes(gq), gs, O.unpack_int4_codes(wtq), wts, None, block=16,
                                 splits=ops.gemm_int4_auto_splits(T, K, N)).astype(np.float16)
    assert np.array_equal(x.grad.cpu().numpy(), want_dx)
    gtq, gts = O.quantize_int4_cols(gn, signs, True, 2)
    xtq, xts = O.quantize_int4_cols(xn, signs)
    want_dw = O.block_int_matmul(O.unpack_int4_codes(gtq), gts, O.unpack_int4_codes(xtq), xts, None, block=16,
                                 splits=ops.gemm_int4_auto_splits(N, K, T)).astype(np.float16)
    assert np.array_equal(w.grad.cpu().numpy(), want_dw)


def test_frozen_int4_linear_equals_linear_int4_fprop(cuda):
    T, K, N = 96, 128, 64
    g = torch.Generator().manual_seed(5)
    lin = torch.nn.Linear(K, N, bias=False).to(torch.float16).to(cuda)
    x = torch.randn(T, K, generator=g).to(torch.float16).to(cuda)
    dy = torch.randn(T, N, generator=g).to(torch.float16).to(cuda)
    frozen = train_linear.FrozenInt4Linear(lin)
    x1 = x.clone().requires_grad_(True)
    train_linear._seed[0] = 0
    y1 = frozen(x1)
    y1.backward(dy)
    x2 = x.clone().requires_grad_(True)
    w2 = lin.weight.detach().clone()  # frozen: no wgrad
    train_linear._seed[0] = 0
    y2 = train_linear.linear(x2, w2, True)
    y2.backward(dy)
    assert torch.equal(y1, y2) and torch.equal(x1.grad, x2.grad)
    with pytest.raises(ValueError, match="bias-free fp16"):
        train_linear.FrozenInt4Linear(torch.nn.Linear(K, N).to(torch.float16))
