"""The allocation-free W4A16 entry point (w4a16_gemm_noalloc), called through
the C ABI. It exists for callers that cannot allocate device memory (a plugin
host that passes only input/output pointers, or code that must not issue a
synchronising cudaMalloc) but need the small-M path, whose regular entry point
takes a caller-provided scratch workspace. On two calls in a row (the fixed
scratch array keeps the last call's contents, and the counters must come back
re-armed) its output must equal the regular entry point's and match the CPU
oracle's fp32 dequant-then-matmul (1e-5: both kernels scale exact integer-code
partials in fp32). This file sorts last so that a run stopping at the first
failure has run everything else."""
import pytest
import torch

import oracle as O
from comfy_ui_gfx906_tools_b200 import _lib, ops, synthetic

pytestmark = pytest.mark.gpu


def _call_noalloc(x, p, s, out_dtype, bias=None):
    M, K = x.shape
    N = p.shape[0]
    y = torch.empty(M, N, dtype=out_dtype, device=x.device)
    code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[out_dtype]
    sd = 1 if s.dtype == torch.float16 else 0
    rc = _lib.load().w4a16_gemm_noalloc(x.data_ptr(), 2, p.data_ptr(), s.data_ptr(), sd,
                                        bias.data_ptr() if bias is not None else None, y.data_ptr(), code, M, N, K, 0,
                                        torch.cuda.current_stream().cuda_stream)
    return rc, y


@pytest.mark.parametrize("M,N,K,f16", [(1, 3072, 3072, True), (16, 9216, 3072, True), (5, 1000, 640, False),
                                       (40, 700, 1024, False)])
def test_noalloc_matches_regular_entry_point(cuda, M, N, K, f16):
    raw, _, _ = synthetic.q4_0_weight(N, K, seed=M + N)
    pn, sn = O.repack_q4_0_native(raw.numpy(), N, K)
    p, s = torch.from_numpy(pn).to(cuda), torch.from_numpy(sn).to(cuda)
    if f16:
        s = ops.scales_to_f16_if_exact(s)
    xc = synthetic.activations(M, K, seed=K)
    x = xc.to(cuda)
    bias = torch.linspace(-1, 1, N, device=cuda)
    oracle = O.w4a16_matmul(xc.float().numpy(), pn, sn, bias.cpu().numpy())
    ref = ops.gemm_w4a16(x, p, s, bias, torch.float32)
    for _ in range(2):  # two calls in a row share the fixed scratch
        rc, y = _call_noalloc(x, p, s, torch.float32, bias)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        for want in (ref.cpu().numpy(), oracle):
            m = O.parity_metrics(got, want)
            assert m["nonfinite"] == 0 and m["max_abs_over_max_ref"] <= 1e-5 and m["mean_rel"] <= 1e-5, m
    rc, ybf = _call_noalloc(x, p, s, torch.bfloat16, bias.bfloat16())
    assert rc == 0
    assert torch.equal(ybf, ops.gemm_w4a16(x, p, s, bias.bfloat16(), torch.bfloat16))


def test_noalloc_rejects_what_it_cannot_cover(cuda):
    raw, _, _ = synthetic.q4_0_weight(256, 256, seed=1)
    p, s = ops.repack_q4_0_native(raw.to(cuda), 256, 256)
    x = synthetic.activations(65, 256, seed=2).to(cuda)
    rc, _ = _call_noalloc(x, p, s, torch.float32)
    assert rc == _lib.GFX_ERR_UNSUPPORTED and "M > 64" in _lib.last_error()
    big_n = 1 << 20  # 64 tokens x 1M rows: far more partials than the fixed scratch holds
    rc = _lib.load().w4a16_gemm_noalloc(x.data_ptr(), 2, p.data_ptr(), s.data_ptr(), 0, None, x.data_ptr(), 2, 64,
                                        big_n, 256 * 64, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.GFX_ERR_UNSUPPORTED and "scratch" in _lib.last_error()
