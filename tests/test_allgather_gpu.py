"""The all-gather epilogue of the small-M kernel and the flag barrier on one GPU
(the two-rank NVLink path itself runs in test_multi_gpu.py): two local buffers
stand in for two ranks' copies of y. Each "rank" computes its half of the output
channels and stores it into both buffers; both must then hold exactly the
column-wise concatenation of the two shard GEMMs (same kernel plan, so
bit-exact), and the shard results must match the oracle. The barrier with one
rank passes at once and advances its device-side epoch counter."""
import ctypes

import pytest
import torch

import oracle as O
from comfy_ui_gfx906_tools_b200 import _lib, ops, synthetic

pytestmark = pytest.mark.gpu


def _ptrs(tensors):
    arr = (ctypes.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])
    return arr, ctypes.cast(arr, ctypes.c_void_p)


@pytest.mark.parametrize("M", [1, 5, 16, 64])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_allgather_two_local_targets(cuda, M, out_dtype):
    N, K, world = 1536, 3072, 2
    raw, _, _ = synthetic.q4_0_weight(N, K, seed=21)
    p, s = ops.repack_q4_0_native(raw.to(cuda), N, K)
    bias = torch.linspace(-1, 1, N, device=cuda).to(out_dtype)
    x = synthetic.activations(M, K, seed=22 + M).to(cuda).to(torch.bfloat16).contiguous()
    n_local = N // world
    shards = [(p[r * n_local:(r + 1) * n_local].contiguous(), s[r * n_local:(r + 1) * n_local].contiguous(),
               bias[r * n_local:(r + 1) * n_local].contiguous()) for r in range(world)]
    want = torch.cat([ops.gemm_w4a16(x, ps, ss, bs, out_dtype) for (ps, ss, bs) in shards], dim=1)
    bufs = [torch.full((M, N), float("nan"), dtype=out_dtype, device=cuda) for _ in range(world)]
    arr, targets = _ptrs(bufs)
    L = _lib.load()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    nbytes = int(L.w4a16_workspace_bytes(M, n_local, K, 0))
    ws = ops._workspace(cuda, stream, nbytes)
    for r, (ps, ss, bs) in enumerate(shards):
        _lib.call("w4a16_gemm_allgather", x.data_ptr(), _lib.DTYPE_BF16, ps.data_ptr(), ss.data_ptr(),
                  _lib.SCALE_F32, bs.data_ptr(), targets, world, r, ops._dtype_code(out_dtype), M, n_local, K, 0,
                  ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0, stream)
    torch.cuda.synchronize(cuda)
    for b in bufs:
        assert torch.equal(b, want)
    ref = O.w4a16_matmul(x.float().cpu().numpy(), p.cpu().numpy(), s.cpu().numpy()) + bias.float().cpu().numpy()
    m = O.parity_metrics(want.float().cpu().numpy(), ref)
    assert m["max_abs_over_max_ref"] <= 2e-2 and m["mean_rel"] <= 5e-3, m


def test_peer_barrier_single_rank_advances_epoch(cuda):
    L = _lib.load()
    L.gfx_device_status(1)
    flags = torch.zeros(2, dtype=torch.int32, device=cuda)  # [flag of rank 0, barrier count]
    arr, fp = _ptrs([flags])
    stream = torch.cuda.current_stream(cuda).cuda_stream
    for _ in range(3):
        _lib.call("gfx_peer_barrier", fp, 1, 0, stream)
    torch.cuda.synchronize(cuda)
    assert flags.tolist() == [3, 3]
    assert L.gfx_device_status(1) == 0
