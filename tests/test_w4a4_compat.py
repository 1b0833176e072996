"""W4A4-compatible mode: the reference's own Linear numerics (activations
quantized to int4 per 32-block before the GEMM, ops.py:167-183).

CPU: the oracle's integer-block restatement (int4_gemm_scaled.hip:147-152)
equals a direct float64 evaluation of the same formula, and differs from the
weight-only product by the size of int4 activation noise (the reference
reports ~12% relative error of its W4A4 GEMM against the float product).
GPU: ``int4_linear_w4a4`` / ``Linear.activation_quant`` match the oracle
within the north-star tolerance."""
import numpy as np
import pytest
import torch

import oracle as O


def _case(M, N, K, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    p, s = O.quantize_pack_int4(w)
    return x, p, s


def test_w4a4_oracle_is_the_integer_block_formula():
    x, p, s = _case(6, 48, 192, 1)
    got = O.w4a4_matmul(x, p, s)
    pa, sa = O.quantize_pack_int4(x, div_mode="recip")
    ca, cb = O.unpack_int4_codes(pa).astype(np.int64), O.unpack_int4_codes(p).astype(np.int64)
    ref = np.zeros((6, 48))
    for b in range(192 // 32):
        dot = (ca[:, None, b * 32:(b + 1) * 32] * cb[None, :, b * 32:(b + 1) * 32]).sum(-1)
        ref += dot * (sa[:, None, b].astype(np.float32) * s[None, :, b].astype(np.float32)).astype(np.float64)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()


def test_w4a4_differs_from_w4a16_by_activation_noise():
    x, p, s = _case(16, 128, 512, 2)
    a, b = O.w4a4_matmul(x, p, s), O.w4a16_matmul(x, p, s)
    rel = np.linalg.norm(a - b) / np.linalg.norm(b)
    assert 0.03 < rel < 0.2, rel


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 16, 300])
def test_int4_linear_w4a4_matches_reference_numerics(cuda, M):
    from comfy_ui_gfx906_tools_b200 import ops
    N, K = 256, 1024
    x, p, s = _case(M, N, K, 3 + M)
    bias = np.linspace(-0.5, 0.5, N).astype(np.float32)
    xt = torch.from_numpy(x).to(cuda)
    y = ops.int4_linear_w4a4(xt, torch.from_numpy(p).to(cuda), torch.from_numpy(s).to(cuda),
                             torch.from_numpy(bias).to(cuda))
    ref = O.w4a4_matmul(x, p, s, bias)
    m = O.parity_metrics(y.cpu().numpy(), ref)
    assert m["nonfinite"] == 0
    assert m["max_abs_over_max_ref"] <= 2e-2 and m["mean_rel"] <= 5e-3, m
    # and it is the W4A4 product, not the weight-only one
    far = O.parity_metrics(y.cpu().numpy(), O.w4a16_matmul(x, p, s, bias))
    assert far["mean_rel"] > 4 * m["mean_rel"], (m, far)


@pytest.mark.gpu
def test_linear_activation_quant_flag(cuda):
    from comfy_ui_gfx906_tools_b200 import ops
    N, K, M = 128, 512, 8
    x, p, s = _case(M, N, K, 9)
    lin = ops.Gfx906Int4Ops.Linear(K, N, bias=False, device=cuda, dtype=torch.float32)
    lin.weight_q4.copy_(torch.from_numpy(p))
    lin.weight_scale.copy_(torch.from_numpy(s))
    lin.activation_quant = True
    y = lin(torch.from_numpy(x).to(cuda)).cpu().numpy()
    m = O.parity_metrics(y, O.w4a4_matmul(x, p, s))
    assert m["max_abs_over_max_ref"] <= 2e-2 and m["mean_rel"] <= 5e-3, m


@pytest.mark.gpu
@pytest.mark.parametrize("M", [2, 200])
def test_gemm_int4_reference_op(cuda, M):
    """ops.gemm_int4 with the reference's arguments (A from quantize_int4)."""
    from comfy_ui_gfx906_tools_b200 import ops
    N, K = 320, 768
    x, p, s = _case(M, N, K, 20 + M)
    A, As = ops.quantize_int4(torch.from_numpy(x).to(cuda))
    bias = torch.linspace(-1, 1, N, device=cuda)
    y = ops.gemm_int4(A, As, torch.from_numpy(p).to(cuda), torch.from_numpy(s).to(cuda), bias, torch.float32)
    ref = O.block_int_matmul(O.unpack_int4_codes(A.cpu().numpy()), As.cpu().numpy(), O.unpack_int4_codes(p), s,
                             bias.cpu().numpy())
    m = O.parity_metrics(y.cpu().numpy(), ref)
    assert m["max_abs_over_max_ref"] <= 2e-2 and m["mean_rel"] <= 5e-3, m
    with pytest.raises(RuntimeError, match="scales must be"):
        ops.gemm_int4(A, As[:, :1], torch.from_numpy(p).to(cuda), torch.from_numpy(s).to(cuda), None, torch.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("M", [2, 64, 200])
def test_gemm_int4_qblock16_reference_op(cuda, M):
    """ops.gemm_int4(..., qblock=16): A and B with one scale per 16 elements
    (int4_gemm_scaled.hip:153-160, SUB = 2: each 32-element load splits into
    two 16-element dot products, each rescaled), against the integer-block
    formula over 16-element blocks."""
    from comfy_ui_gfx906_tools_b200 import ops
    N, K = 320, 768
    rng = np.random.default_rng(40 + M)
    ca, cb = rng.integers(-8, 8, (M, K)), rng.integers(-8, 8, (N, K))
    sa = ((np.abs(rng.normal(0, 1, (M, K // 16))) + 0.05) * 0.2).astype(np.float32)
    sb = (np.abs(rng.normal(0, 0.01, (N, K // 16))) + 1e-4).astype(np.float32)
    bias = torch.linspace(-1, 1, N, device=cuda)
    A, B = torch.from_numpy(O.pack_int4_codes(ca)).to(cuda), torch.from_numpy(O.pack_int4_codes(cb)).to(cuda)
    y = ops.gemm_int4(A, torch.from_numpy(sa).to(cuda), B, torch.from_numpy(sb).to(cuda), bias, torch.float32,
                      qblock=16)
    ref = O.block_int_matmul(ca, sa, cb, sb, bias.cpu().numpy(), block=16)
    m = O.parity_metrics(y.cpu().numpy(), ref)
    assert m["max_abs_over_max_ref"] <= 2e-2 and m["mean_rel"] <= 5e-3, m
    with pytest.raises(RuntimeError, match="scales must be"):
        ops.gemm_int4(A, torch.from_numpy(sa).to(cuda), B, torch.from_numpy(sb).to(cuda), None, torch.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("M", [3, 300])
def test_gemm_int8_reference_op(cuda, M):
    """ops.gemm_int8 with the reference's arguments (A, B from quantize_int8)."""
    from comfy_ui_gfx906_tools_b200 import ops
    N, K = 256, 1024
    rng = np.random.default_rng(30 + M)
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(cuda)
    w = torch.from_numpy((rng.standard_normal((N, K)) * 0.05).astype(np.float32)).to(cuda)
    A, As = ops.quantize_int8(x)
    B, Bs = ops.quantize_int8(w)
    y = ops.gemm_int8(A, As, B, Bs, None, torch.float32, config=1)
    ref = O.block_int_matmul(A.cpu().numpy(), As.cpu().numpy(), B.cpu().numpy(), Bs.cpu().numpy())
    m = O.parity_metrics(y.cpu().numpy(), ref)
    assert m["max_abs_over_max_ref"] <= 2e-2 and m["mean_rel"] <= 5e-3, m
    with pytest.raises(RuntimeError, match="config must be"):
        ops.gemm_int8(A, As, B, Bs, None, torch.float32, config=4)
