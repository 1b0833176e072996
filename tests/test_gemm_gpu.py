"""W4A16 GEMM parity on the GPU, called through the C ABI (ops.gemm_w4a16 ->
ctypes -> w4a16_gemm), against the oracle's fp32 dequant-then-matmul.

Tolerances are the north-star bar, with the mean relative error defined as
mean|got - ref| / mean|ref|:  max|d| <= 2e-2 * max|ref|  and  mean_rel <= 5e-3.
fp32-output cases also check a much tighter bound where the kernel's math is
exact up to fp32 rounding (the split-K kernel scales exact integer-code MMA
partials in fp32)."""
import numpy as np
import pytest
import torch

import oracle as O
from comfy_ui_gfx906_tools_b200 import ops, synthetic

pytestmark = pytest.mark.gpu

MAX_TOL = 2e-2
MEAN_TOL = 5e-3


def _weights(N, K, seed, dev):
    raw, _, _ = synthetic.q4_0_weight(N, K, seed)
    p, s = O.repack_q4_0_native(raw.numpy(), N, K)
    return p, s, torch.from_numpy(p).to(dev), torch.from_numpy(s).to(dev)


def _x(M, K, seed, dev):
    x = synthetic.activations(M, K, seed)
    return x.float().numpy(), x.to(dev)


def _check(got, ref, max_tol=MAX_TOL, mean_tol=MEAN_TOL):
    m = O.parity_metrics(got, ref)
    assert m["nonfinite"] == 0, m
    assert m["max_abs_over_max_ref"] <= max_tol, m
    assert m["mean_rel"] <= mean_tol, m
    return m


def test_gemm_golden_vector(cuda, golden):
    x = torch.from_numpy(golden["gemm_x_bits"].view(np.int16)).view(torch.bfloat16).to(cuda)
    b = torch.from_numpy(golden["gemm_bias_bits"].view(np.int16)).view(torch.bfloat16).to(cuda)
    p = torch.from_numpy(golden["q40_packed"]).to(cuda)
    s = torch.from_numpy(golden["q40_scale"]).to(cuda)
    y = ops.gemm_w4a16(x, p, s, b.float(), torch.float32)
    _check(y.cpu().numpy(), golden["gemm_y_f32"], 1e-5, 1e-5)


@pytest.mark.parametrize("M", [1, 3, 8, 16, 17, 40, 64])
@pytest.mark.parametrize("N,K", [(384, 512), (200, 96), (1000, 3072)])
def test_gemm_small_m(cuda, M, N, K):
    p, s, pd, sd = _weights(N, K, seed=N + K, dev=cuda)
    xn, xd = _x(M, K, seed=M, dev=cuda)
    ref = O.w4a16_matmul(xn, p, s)
    y32 = ops.gemm_w4a16(xd, pd, sd, None, torch.float32)
    _check(y32.cpu().numpy(), ref, 1e-5, 1e-5)
    ybf = ops.gemm_w4a16(xd, pd, sd, None, torch.bfloat16)
    _check(ybf.float().cpu().numpy(), ref)


@pytest.mark.parametrize("splits", [1, 2, 3, 7, 12])
def test_gemm_splits_agree(cuda, splits):
    N, K, M = 640, 3072, 16
    p, s, pd, sd = _weights(N, K, 1, cuda)
    xn, xd = _x(M, K, 2, cuda)
    ref = O.w4a16_matmul(xn, p, s)
    y = ops.gemm_w4a16(xd, pd, sd, None, torch.float32, splits=splits)
    _check(y.cpu().numpy(), ref, 1e-5, 1e-5)


@pytest.mark.parametrize("M,N,K,splits", [(1, 3072, 3072, 0), (16, 3072, 3072, 0), (5, 1024, 4096, 4),
                                           (9, 640, 3072, 3), (40, 384, 2048, 2), (3, 3072, 15360, 0)])
def test_gemm_cluster_splitk_matches_global_fixup(cuda, monkeypatch, M, N, K, splits):
    """Classic split-K plans reduce through distributed shared memory inside a
    cluster (opt-in, GFX906_B200_SMALLM_CLUSTER=1) or through global partials;
    both sum the K segments in the same order, so the outputs are identical
    (zero signs aside), and both match the oracle."""
    p, s, pd, sd = _weights(N, K, 91 + M, cuda)
    sd16 = ops.scales_to_f16_if_exact(sd)
    xn, xd = _x(M, K, 92 + M, cuda)
    bias = torch.linspace(-1, 1, N, device=cuda)
    out = {}
    for mode in ("1", "0"):
        monkeypatch.setenv("GFX906_B200_SMALLM_CLUSTER", mode)
        out[mode] = (ops.gemm_w4a16(xd, pd, sd16, bias, torch.float32, splits=splits) + 0.0,
                     ops.gemm_w4a16(xd, pd, sd, None, torch.bfloat16, splits=splits).float() + 0.0)
    monkeypatch.delenv("GFX906_B200_SMALLM_CLUSTER")
    assert torch.equal(out["1"][0], out["0"][0]) and torch.equal(out["1"][1], out["0"][1])
    _check(out["1"][0].cpu().numpy(), O.w4a16_matmul(xn, p, s, bias.cpu().numpy()), 1e-5, 1e-5)


def test_gemm_deterministic_and_workspace_rearmed(cuda):
    N, K, M = 512, 6144, 5
    p, s, pd, sd = _weights(N, K, 3, cuda)
    _, xd = _x(M, K, 4, cuda)
    y1 = ops.gemm_w4a16(xd, pd, sd, None, torch.float32, splits=6)
    y2 = ops.gemm_w4a16(xd, pd, sd, None, torch.float32, splits=6)
    y3 = ops.gemm_w4a16(xd, pd, sd, None, torch.float32, splits=6)
    assert torch.equal(y1, y2) and torch.equal(y2, y3)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_gemm_bias_and_out_dtypes(cuda, out_dtype):
    N, K, M = 264, 1024, 9
    p, s, pd, sd = _weights(N, K, 5, cuda)
    xn, xd = _x(M, K, 6, cuda)
    bias = (torch.randn(N, generator=torch.Generator().manual_seed(1)) * 0.1).to(out_dtype)
    ref = O.w4a16_matmul(xn, p, s, bias.float().numpy())
    for splits in (0, 1, 4):
        y = ops.gemm_w4a16(xd, pd, sd, bias.to(cuda), out_dtype, splits=splits)
        assert y.dtype == out_dtype
        _check(y.float().cpu().numpy(), ref)


def test_gemm_f16_scales_identical(cuda):
    # Q4_0-sourced fp32 scales are exact fp16 values: the fp16 scale path gives bit-identical output
    N, K, M = 768, 3072, 16
    p, s, pd, sd = _weights(N, K, 8, cuda)
    _, xd = _x(M, K, 9, cuda)
    s16 = ops.scales_to_f16_if_exact(sd)
    assert s16 is not None
    for splits in (0, 1):
        a = ops.gemm_w4a16(xd, pd, sd, None, torch.float32, splits=splits)
        b = ops.gemm_w4a16(xd, pd, s16, None, torch.float32, splits=splits)
        assert torch.equal(a, b)


def test_gemm_general_rtn_weights(cuda):
    # quantize_pack_int4 (RTN) weights carry general fp32 scales
    N, K, M = 333, 640, 12
    w = synthetic.float_weight(N, K, 12)
    p, s = O.quantize_pack_int4(w.numpy())
    xn, xd = _x(M, K, 13, cuda)
    ref = O.w4a16_matmul(xn, p, s)
    y = ops.gemm_w4a16(xd, torch.from_numpy(p).to(cuda), torch.from_numpy(s).to(cuda), None, torch.float32)
    _check(y.cpu().numpy(), ref, 1e-5, 1e-5)


def test_gemm_m_zero(cuda):
    p, s, pd, sd = _weights(64, 64, 1, cuda)
    y = ops.gemm_w4a16(torch.empty(0, 64, dtype=torch.bfloat16, device=cuda), pd, sd, None, torch.bfloat16)
    assert y.shape == (0, 64)


def test_gemm_rejects_bad_inputs(cuda):
    p, s, pd, sd = _weights(64, 64, 1, cuda)
    x = torch.zeros(2, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(RuntimeError, match="inputs must be on device"):
        ops.gemm_w4a16(x.cpu(), pd, sd, None, torch.bfloat16)
    with pytest.raises(RuntimeError, match="bias dtype"):
        ops.gemm_w4a16(x, pd, sd, torch.zeros(64, device=cuda), torch.bfloat16)
    with pytest.raises(RuntimeError, match=r"scales must be \[N, K/32\]"):
        ops.gemm_w4a16(x, pd, sd[:, :1], None, torch.bfloat16)


@pytest.mark.parametrize("name,K,N", synthetic.FLUX_SHAPES)
@pytest.mark.parametrize("M", [1, 16])
def test_gemm_flux_shapes_small_m_full_size(cuda, name, K, N, M):
    p, s, pd, sd = _weights(N, K, seed=K * 7 + N, dev=cuda)
    xn, xd = _x(M, K, seed=M + 100, dev=cuda)
    ref = O.w4a16_matmul(xn, p, s)
    y = ops.gemm_w4a16(xd, pd, sd, None, torch.bfloat16)
    _check(y.float().cpu().numpy(), ref)


def test_int4_linear_module(cuda):
    # Gfx906Int4Ops.Linear with Q4_0-sourced buffers, leading batch dims, bias in x.dtype
    N, K = 256, 512
    p, s, pd, sd = _weights(N, K, 21, cuda)
    lin = ops.Gfx906Int4Ops.Linear(K, N, bias=True, device=cuda, dtype=torch.bfloat16)
    lin.weight_q4.copy_(pd)
    lin.weight_scale.copy_(sd)
    with torch.no_grad():
        lin.bias.copy_(torch.linspace(-1, 1, N))
    x = synthetic.activations(2 * 7, K, 22).reshape(2, 7, K)
    y = lin(x.to(cuda))
    assert y.shape == (2, 7, N) and y.dtype == torch.bfloat16
    ref = O.w4a16_matmul(x.float().reshape(-1, K).numpy(), p, s, lin.bias.detach().float().cpu().numpy())
    _check(y.float().reshape(-1, N).cpu().numpy(), ref)


# ---------------------------------------------------------------------------
# large M: the tcgen05 kernel (automatic path for M > 64)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("M", [65, 256, 300, 777])
@pytest.mark.parametrize("N,K", [(384, 512), (200, 96), (1000, 3072), (129, 64)])
@pytest.mark.parametrize("f16_scales", [False, True])
def test_gemm_large_m_tcgen05(cuda, M, N, K, f16_scales):
    if f16_scales and K % 64:
        pytest.skip("fp16 scales need K % 64 == 0")
    p, s, pd, sd = _weights(N, K, seed=N + K + 1, dev=cuda)
    if f16_scales:
        sd = ops.scales_to_f16_if_exact(sd)
    xn, xd = _x(M, K, seed=M + 7, dev=cuda)
    y32 = ops.gemm_w4a16(xd, pd, sd, None, torch.float32).cpu().numpy()
    # the kernel multiplies exactly bf16(code*scale): tight against that oracle
    _check(y32, O.w4a16_matmul_bf16w(xn, p, s), 1e-5, 1e-5)
    # and within the north-star bar against the fp32 dequant-then-matmul
    _check(y32, O.w4a16_matmul(xn, p, s))
    ybf = ops.gemm_w4a16(xd, pd, sd, None, torch.bfloat16)
    _check(ybf.float().cpu().numpy(), O.w4a16_matmul(xn, p, s))


@pytest.mark.parametrize("M", [1, 9, 64, 65, 300])
def test_gemm_single_group_k32(cuda, M):
    """K = 32: one scale group per row, narrower than every tile's K extent
    (TMA fills the rest of the box with zeros) and a scale row of 4 bytes
    (not TMA-aligned, so the scales come through cp.async); both kernels, on
    either side of the M = 64 switch, with a ragged N. Each kernel is held
    tight against the oracle of its own arithmetic: the small-M kernel scales
    exact integer-code partials in fp32 (fp32 dequant oracle), the tensor-core
    kernel multiplies bf16(code * scale) (bf16-weight oracle)."""
    N, K = 130, 32
    p, s, pd, sd = _weights(N, K, seed=33, dev=cuda)
    xn, xd = _x(M, K, seed=34 + M, dev=cuda)
    bias = torch.linspace(-1, 1, N, device=cuda)
    y32 = ops.gemm_w4a16(xd, pd, sd, bias, torch.float32).cpu().numpy()
    exact = O.w4a16_matmul(xn, p, s) if M <= 64 else O.w4a16_matmul_bf16w(xn, p, s)
    _check(y32, exact + bias.cpu().numpy(), 1e-5, 1e-5)
    _check(y32, O.w4a16_matmul(xn, p, s) + bias.cpu().numpy())


@pytest.mark.parametrize("M", [1, 64, 65, 300])
@pytest.mark.parametrize("N,K", [(384, 512), (200, 96), (129, 64), (1000, 3072)])
def test_gemm_qblock16(cuda, M, N, K):
    """16-element scale blocks (gemm_int4's qblock=16, int4_gemm_scaled.hip:
    153-160): RTN weights quantized per 16 elements, fp32 scales [N, K/16], on
    the tensor-core kernel for every M. Tight against the oracle of its exact
    operands (bf16(code * scale of the element's 16-group))
    against the fp32 dequant-then-matmul; the 16-block dequant is bit-exact."""
    w = synthetic.float_weight(N, K, 90 + N)
    p, s = O.quantize_pack_int4(w.numpy(), block=16)
    assert s.shape == (N, K // 16)
    pd, sd = torch.from_numpy(p).to(cuda), torch.from_numpy(s).to(cuda)
    xn, xd = _x(M, K, 91 + M, cuda)
    bias = torch.linspace(-1, 1, N, device=cuda)
    y32 = ops.gemm_w4a16(xd, pd, sd, bias, torch.float32, qblock=16).cpu().numpy()
    _check(y32, O.w4a16_matmul_bf16w(xn, p, s, bias.cpu().numpy(), block=16), 1e-5, 1e-5)
    _check(y32, O.w4a16_matmul(xn, p, s, bias.cpu().numpy(), block=16))
    ybf = ops.gemm_w4a16(xd, pd, sd, None, torch.bfloat16, qblock=16)
    _check(ybf.float().cpu().numpy(), O.w4a16_matmul(xn, p, s, block=16))
    dq = ops.dequantize_int4(pd, sd, torch.bfloat16, block=16)
    assert np.array_equal(dq.view(torch.int16).cpu().numpy().view(np.uint16), O.dequant_int4_bf16_bits(p, s, 16))
    with pytest.raises(RuntimeError, match="float32 scales"):
        ops.gemm_w4a16(xd, pd, sd.half(), None, torch.float32, qblock=16)


def test_gemm_large_m_general_fp32_scales(cuda):
    N, K, M = 520, 1024, 400
    w = synthetic.float_weight(N, K, 31)
    p, s = O.quantize_pack_int4(w.numpy())
    xn, xd = _x(M, K, 32, cuda)
    y = ops.gemm_w4a16(xd, torch.from_numpy(p).to(cuda), torch.from_numpy(s).to(cuda), None, torch.float32)
    _check(y.cpu().numpy(), O.w4a16_matmul_bf16w(xn, p, s), 1e-5, 1e-5)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_gemm_large_m_bias(cuda, out_dtype):
    N, K, M = 300, 768, 333
    p, s, pd, sd = _weights(N, K, 41, cuda)
    xn, xd = _x(M, K, 42, cuda)
    bias = (torch.randn(N, generator=torch.Generator().manual_seed(3)) * 0.1).to(out_dtype)
    y = ops.gemm_w4a16(xd, pd, sd, bias.to(cuda), out_dtype)
    assert y.dtype == out_dtype
    _check(y.float().cpu().numpy(), O.w4a16_matmul(xn, p, s, bias.float().numpy()))


def test_gemm_large_m_matches_small_m_path(cuda):
    # the tcgen05 kernel (M=512) and the small-M kernel (the same first 64 rows)
    # agree within the bf16 rounding of the tensor-core weight operand
    N, K, M = 640, 2048, 512
    p, s, pd, sd = _weights(N, K, 51, cuda)
    _, xd = _x(M, K, 52, cuda)
    a = ops.gemm_w4a16(xd, pd, sd, None, torch.float32).cpu().numpy()
    b = ops.gemm_w4a16(xd[:64].contiguous(), pd, sd, None, torch.float32, splits=1).cpu().numpy()
    _check(a[:64], b)
    assert ops.gemm_w4a16(xd, pd, sd, None, torch.float32, splits=3).equal(
        ops.gemm_w4a16(xd, pd, sd, None, torch.float32))  # splits does not change the M > 64 result


def test_gemm_large_m_deterministic(cuda):
    N, K, M = 768, 3072, 1024
    p, s, pd, sd = _weights(N, K, 61, cuda)
    _, xd = _x(M, K, 62, cuda)
    y1 = ops.gemm_w4a16(xd, pd, sd, None, torch.bfloat16)
    y2 = ops.gemm_w4a16(xd, pd, sd, None, torch.bfloat16)
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("M,N,K", [(100, 384, 512), (300, 1000, 3072), (777, 129, 64), (1024, 640, 2048)])
@pytest.mark.parametrize("f16_scales", [False, True])
def test_gemm_large_m_cta_pair_matches_single_cta(cuda, monkeypatch, M, N, K, f16_scales):
    """The opt-in CTA-pair kernel (cta_group::2) and the default one-CTA
    kernel, selected through GFX906_B200_TC_CTA, compute the same products
    with the same K order; both are checked against the oracle too."""
    p, s, pd, sd = _weights(N, K, 71 + M, cuda)
    if f16_scales:
        sd = ops.scales_to_f16_if_exact(sd)
    xn, xd = _x(M, K, 72 + M, cuda)
    out = {}
    for c in ("1", "2"):
        monkeypatch.setenv("GFX906_B200_TC_CTA", c)
        out[c] = ops.gemm_w4a16(xd, pd, sd, None, torch.float32)
    monkeypatch.delenv("GFX906_B200_TC_CTA")
    torch.testing.assert_close(out["1"], out["2"], rtol=1e-5, atol=1e-5 * out["1"].abs().max().item())
    for c in ("1", "2"):
        _check(out[c].cpu().numpy(), O.w4a16_matmul_bf16w(xn, p, s), 1e-5, 1e-5)


@pytest.mark.parametrize("per_channel", [False, True])
def test_gemm_int8_cta_pair_matches_single_cta(cuda, monkeypatch, per_channel):
    M, N, K = 640, 384, 1024
    rng = np.random.default_rng(81)
    w = np.clip(np.round(rng.normal(0, 40, (N, K))), -127, 127).astype(np.int8)
    xn, xd = _x(M, K, 82, cuda)
    if per_channel:
        sc = (np.abs(rng.normal(0, 0.01, N)) + 1e-4).astype(np.float16)
    else:
        sc = (np.abs(rng.normal(0, 0.01, (N, K // 32))) + 1e-4).astype(np.float32)
    wd, sdd = torch.from_numpy(w).to(cuda), torch.from_numpy(sc).to(cuda)
    out = {}
    for c in ("1", "2"):
        monkeypatch.setenv("GFX906_B200_TC_CTA", c)
        out[c] = ops.gemm_w8a16(xd, wd, sdd, None, torch.float32)
    monkeypatch.delenv("GFX906_B200_TC_CTA")
    torch.testing.assert_close(out["1"], out["2"], rtol=1e-5, atol=1e-5 * out["1"].abs().max().item())


def test_gemm_config1_single_linear_full(cuda):
    """Config 1 exactly: X [256, 3072] bf16 ~ N(0, 1), W [3072, 3072] from
    synthetic Q4_0 blocks (u ~ U{0..15}, d = fp16(|N(0, 0.02)|/7 + 1e-4)),
    no bias, bf16 output; every element checked against the fp32
    dequant-then-matmul, and the fp32 output against the exact-operand oracle."""
    M, N, K = 256, 3072, 3072
    p, s, pd, sd = _weights(N, K, seed=101, dev=cuda)
    xn, xd = _x(M, K, seed=102, dev=cuda)
    y = ops.gemm_w4a16(xd, pd, sd, None, torch.bfloat16)
    assert y.dtype == torch.bfloat16 and y.shape == (M, N)
    _check(y.float().cpu().numpy(), O.w4a16_matmul(xn, p, s))
    y32 = ops.gemm_w4a16(xd, pd, sd, None, torch.float32).cpu().numpy()
    _check(y32, O.w4a16_matmul_bf16w(xn, p, s), 1e-5, 1e-5)


@pytest.mark.parametrize("name,K,N", synthetic.FLUX_SHAPES)
def test_gemm_flux_shapes_m4608_full_size(cuda, name, K, N):
    """The Flux linear sweep (config 2) at full size, every row: the fp32
    output against the oracle of the kernel's exact operands (bf16(code *
    scale), fp32 accumulation) at 1e-5, the bf16 output against the fp32
    dequant-then-matmul at the north-star bar, and every row through a
    size-independent checksum: sum_n Y[m, n] == X[m] . sum_n W[n] (linearity),
    in fp64."""
    M = 4608
    p, s, pd, sd = _weights(N, K, seed=K * 3 + N, dev=cuda)
    sd16 = ops.scales_to_f16_if_exact(sd)
    x = synthetic.activations(M, K, seed=77)
    xn = x.float().numpy()
    y32 = ops.gemm_w4a16(x.to(cuda), pd, sd16, None, torch.float32).cpu().numpy()
    # fp32 summation order over K differs from numpy's (a K-dependent bound,
    # still ~500x tighter than the north-star bar)
    acc_tol = max(1e-5, 3e-7 * np.sqrt(K))
    _check(y32, O.w4a16_matmul_bf16w(xn, p, s), acc_tol, acc_tol)
    y = ops.gemm_w4a16(x.to(cuda), pd, sd16, None, torch.bfloat16).float()
    _check(y.cpu().numpy(), O.w4a16_matmul(xn, p, s))
    wsum = O.round_to_bf16(O.dequant_int4(p, s)).astype(np.float64).sum(axis=0)   # [K]
    want = xn.astype(np.float64) @ wsum                                            # [M]
    gotsum = y.double().sum(dim=1).cpu().numpy()
    scale = np.abs(xn).astype(np.float64) @ np.abs(wsum)
    assert np.max(np.abs(gotsum - want) / (scale + 1e-30)) < 2e-3


# ---------------------------------------------------------------------------
# int8 weights (W8A16): the config-3 layout (per-channel fp16 scale) and
# the reference's block-32 layout (quantize_int8 output)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("M", [1, 77, 300, 1000])
@pytest.mark.parametrize("N,K", [(96, 864), (3, 96), (384, 3456)])
def test_gemm_int8_block_scales(cuda, M, N, K):
    # bench_int8.py:37-48 shapes: ragged M / N, bias; B from quantize_int8 (block-32 fp32 scales)
    g = torch.Generator().manual_seed(M + N)
    w = torch.randn(N, K, generator=g).to(cuda)
    bq, bs = ops.quantize_int8(w)
    qw, sw = O.quantize_int8(w.cpu().numpy())
    assert np.array_equal(bq.cpu().numpy(), qw) and np.array_equal(bs.cpu().numpy(), sw)
    x = synthetic.activations(M, K, seed=M)
    bias = torch.randn(N, generator=g)
    y = ops.gemm_w8a16(x.to(cuda), bq, bs, bias.to(cuda), torch.float32).cpu().numpy()
    ref = O.w8a16_matmul(x.float().numpy(), qw, sw, bias.numpy())
    _check(y, ref)


@pytest.mark.parametrize("name,K,N", synthetic.FLUX_SHAPES)
@pytest.mark.parametrize("M", [1, 16, 4608])
def test_gemm_int8_channel_scales_flux(cuda, name, K, N, M):
    """Config 3 at every Flux shape: int8 ~round(N(0,40)) clipped, one fp16
    scale per output channel, against the reference's int8 dequant + fp32
    matmul (bench_int8.py:32-43 restated by oracle.w8a16_matmul, with the
    channel scale replicated to the [N, K/32] block layout). M=4608 checks 96
    sampled rows exactly and every row through the linearity checksum."""
    q, s = synthetic.int8_weight(N, K, seed=5 + K + N)
    x = synthetic.activations(M, K, seed=6 + M)
    xd, qd, sdd = x.to(cuda), q.to(cuda), s.to(cuda)
    y = ops.gemm_w8a16(xd, qd, sdd, None, torch.bfloat16).float()
    y32 = ops.gemm_w8a16(xd, qd, sdd, None, torch.float32)
    s_blk = np.repeat(s.float().numpy()[:, None], K // 32, axis=1)
    rows = np.arange(M) if M <= 64 else np.random.default_rng(1).choice(M, 96, replace=False)
    rows_d = torch.from_numpy(rows).to(cuda)
    ref = O.w8a16_matmul(x[rows].float().numpy(), q.numpy(), s_blk)
    _check(y[rows_d].cpu().numpy(), ref)
    acc_tol = max(1e-5, 3e-7 * np.sqrt(K))  # fp32 summation order over K
    _check(y32[rows_d].cpu().numpy(), ref, acc_tol, acc_tol)  # exact codes, fp32 channel scale
    if M > 64:
        wsum = (q.double() * s.double()[:, None]).sum(dim=0).numpy()                # [K]
        xn = x.double().numpy()
        want = xn @ wsum
        scale = np.abs(xn) @ np.abs(wsum)
        gotsum = y32.double().sum(dim=1).cpu().numpy()
        assert np.max(np.abs(gotsum - want) / (scale + 1e-30)) < 1e-4


def test_quantize_int4_activation_semantics(cuda):
    x = (torch.randn(64, 256, generator=torch.Generator().manual_seed(9))).to(cuda, torch.float16)
    p, s = ops.quantize_int4(x)
    pw, sw = O.quantize_pack_int4(x.float().cpu().numpy(), div_mode="recip")
    assert np.array_equal(p.cpu().numpy(), pw) and np.array_equal(s.cpu().numpy(), sw)
