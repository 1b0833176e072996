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



def test_timeout_is_reported_by_the_next_gemm_call_and_workspace_rearmed(cuda):
    """A wait that gave up is mirrored into the host-visible status word, so the
    next GEMM call reports it (GFX_ERR_DEVICE) before launching anything, with no
    device synchronisation of its own; the Python layer then re-zeroes its cached
    split-K workspaces (whose arrival counters a timed-out kernel may have left
    non-zero), and after the status is cleared the GEMMs run and match the oracle."""
    lib = _lib.load()
    ops.device_status(cuda, clear=True)
    N, K, M = 640, 3072, 16
    raw, _, _ = synthetic.q4_0_weight(N, K, seed=17)
    p, s = O.repack_q4_0_native(raw.numpy(), N, K)
    pd, sd = torch.from_numpy(p).to(cuda), torch.from_numpy(s).to(cuda)
    x = synthetic.activations(M, K, seed=18)
    ops.gemm_w4a16(x.to(cuda), pd, sd, None, torch.float32, splits=4)  # creates this stream's workspace
    stream = torch.cuda.current_stream(cuda).cuda_stream
    assert lib.gfx_selftest_wait_timeout(20000, stream) == 0
    torch.cuda.synchronize(cuda)  # the self-test kernel has given up and mirrored its code
    with pytest.raises(_lib.GfxError) as ei:
        ops.gemm_w4a16(x.to(cuda), pd, sd, None, torch.float32, splits=4)
    assert ei.value.code == _lib.GFX_ERR_DEVICE and "status 6" in str(ei.value)
    # the allocation-free entry point refuses too
    y = torch.empty(M, N, dtype=torch.float32, device=cuda)
    xd = x.to(cuda)
    rc = lib.w4a16_gemm_noalloc(xd.data_ptr(), 2, pd.data_ptr(), sd.data_ptr(), 0, None, y.data_ptr(), 0, M, N, K,
                                0, stream)
    assert rc == _lib.GFX_ERR_DEVICE
    torch.cuda.synchronize(cuda)
    for (idx, _), ws in ops._workspaces.items():
        if idx == cuda.index:
            assert int(ws[:256 * 1024].view(torch.int32).abs().sum()) == 0  # counters re-armed
    assert ops.device_status(cuda, clear=True) == SELFTEST_CODE
    assert ops.device_status(cuda) == 0
    ref = O.w4a16_matmul(x.float().numpy(), p, s)
    for _ in range(2):
        got = ops.gemm_w4a16(xd, pd, sd, None, torch.float32, splits=4).cpu().numpy()
        m = O.parity_metrics(got, ref)
        assert m["max_abs_over_max_ref"] <= 1e-5 and m["mean_rel"] <= 1e-5, m
        rc = lib.w4a16_gemm_noalloc(xd.data_ptr(), 2, pd.data_ptr(), sd.data_ptr(), 0, None, y.data_ptr(), 0, M, N,
                                    K, 0, stream)
        assert rc == 0, _lib.last_error()
        m = O.parity_metrics(y.cpu().numpy(), ref)
        assert m["max_abs_over_max_ref"] <= 1e-5 and m["mean_rel"] <= 1e-5, m
