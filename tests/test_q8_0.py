"""Lossless ggml Q8_0 ingest onto the int8 (W8A16) path: the GPU repack is
bit-exact against the oracle's restatement of the block format, and the
repacked weights through ``gemm_w8a16`` match the fp32 dequant-then-matmul."""
import numpy as np
import pytest
import torch

import oracle as O


def _q8_0(N, K, seed):
    rng = np.random.default_rng(seed)
    q = np.clip(np.round(rng.normal(0, 40, (N, K))), -127, 127).astype(np.int8)
    d = (np.abs(rng.normal(0, 0.02, (N, K // 32))) / 40 + 1e-5).astype(np.float16)
    return q, d, O.build_q8_0_bytes(q, d)


def test_q8_0_oracle_round_trip():
    q, d, raw = _q8_0(5, 96, 1)
    assert raw.size == 5 * 3 * 34
    q2, s2 = O.repack_q8_0(raw, 5, 96)
    assert np.array_equal(q2, q) and np.array_equal(s2, d.astype(np.float32))


def test_q8_0_argument_checks(built_lib):
    assert built_lib.repack_q8_0(None, None, None, 4, 48, None) == 1  # K % 32
    assert built_lib.repack_q8_0(None, None, None, 0, 64, None) == 0  # N == 0: no-op


@pytest.mark.gpu
@pytest.mark.parametrize("N,K", [(1, 32), (7, 96), (300, 3072)])
def test_q8_0_repack_bit_exact(cuda, N, K):
    from comfy_ui_gfx906_tools_b200 import ops
    q, d, raw = _q8_0(N, K, N + K)
    gq, gs = ops.repack_q8_0(torch.from_numpy(raw).to(cuda), N, K)
    assert np.array_equal(gq.cpu().numpy(), q)
    assert np.array_equal(gs.cpu().numpy(), d.astype(np.float32))


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 300])
def test_q8_0_through_w8a16_gemm(cuda, M):
    from comfy_ui_gfx906_tools_b200 import ops, synthetic
    N, K = 384, 1024
    q, d, raw = _q8_0(N, K, 7)
    gq, gs = ops.repack_q8_0(torch.from_numpy(raw).to(cuda), N, K)
    x = synthetic.activations(M, K, seed=M)
    y = ops.gemm_w8a16(x.to(cuda), gq, gs, None, torch.float32).cpu().numpy()
    ref = O.w8a16_matmul(x.float().numpy(), q, d.astype(np.float32))
    m = O.parity_metrics(y, ref)
    assert m["max_abs_over_max_ref"] <= 2e-2 and m["mean_rel"] <= 5e-3, m
