"""Failure detection on the GPU without a fault: every bounded device-side wait
gives up after its budget, records a status code and returns. The self-test
kernel waits on an mbarrier nothing arrives on (a flag nothing sets) with a
20 ms budget; the status word must report it, clear on request, and the CUDA
context must stay usable for the GEMM kernels afterwards."""
import numpy as np
import pytest
import torch

import oracle as O
from comfy_ui_gfx906_tools_b200 import _lib, ops, synthetic

pytestmark = pytest.mark.gpu

SELFTEST_CODE = 6  # kDevErrSelfTestTimeout


def test_bounded_wait_timeout_is_reported_and_context_survives(cuda):
    lib = _lib.load()
    lib.gfx_device_status(1)  # start from a clean status word
    assert lib.gfx_device_status(0) == 0
    stream = torch.cuda.current_stream(cuda).cuda_stream
    assert lib.gfx_selftest_wait_timeout(20000, stream) == 0
    assert lib.gfx_device_status(0) == SELFTEST_CODE
    assert lib.gfx_device_status(1) == SELFTEST_CODE  # read and clear
    assert lib.gfx_device_status(0) == 0
    # the context is intact: both GEMM kernels still run and match the oracle
    N, K = 384, 1024
    raw, _, _ = synthetic.q4_0_weight(N, K, seed=7)
    p, s = O.repack_q4_0_native(raw.numpy(), N, K)
    pd, sd = torch.from_numpy(p).to(cuda), torch.from_numpy(s).to(cuda)
    for M in (4, 300):
        x = synthetic.activations(M, K, seed=M)
        y = ops.gemm_w4a16(x.to(cuda), pd, sd, None, torch.float32).cpu().numpy()
        ref = O.w4a16_matmul(x.float().numpy(), p, s)
        m = O.parity_metrics(y, ref)
        assert m["max_abs_over_max_ref"] <= 2e-2 and m["mean_rel"] <= 5e-3, m
    assert lib.gfx_device_status(0) == 0

