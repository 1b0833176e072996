"""Forward-time activation rotation on the GPU (rotation_group != 0,
ops.py:85-105,176-179): the fast Walsh-Hadamard kernel equals the
reference's ``flat @ R^T`` (R = H / sqrt(g) * diag(signs), seed
ROTATION_SEED ^ g) to fp32 rounding, and int4_linear with a rotation folded
into the weights matches the oracle on the rotated activations."""
import numpy as np
import pytest
import torch

import oracle as O
from comfy_ui_gfx906_tools_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("in_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_hadamard_kernel_matches_rotation_matmul(cuda, group, in_dtype):
    rows, K = 37, 4 * group
    x = torch.randn(rows, K, generator=torch.Generator().manual_seed(group)).to(in_dtype)
    R = ops.get_group_rotation(K, group, "cpu").double()
    ref = (x.double().reshape(-1, group) @ R.t()).reshape(rows, K)
    got32 = ops.hadamard_rotate(x.to(cuda), group, torch.float32).cpu().double()
    assert (got32 - ref).abs().max() <= 1e-6 * ref.abs().max()
    got16 = ops.hadamard_rotate(x.to(cuda), group, torch.bfloat16).cpu().double()
    # one bf16 rounding of a value that is within fp32 rounding of ref
    assert ((got16 - ref).abs() <= ref.abs() * 2.0 ** -8 + 1e-6 * ref.abs().max()).all()


def test_hadamard_is_orthonormal_roundtrip(cuda):
    # R is orthonormal: rotating twice with R and then R^T-consistent data preserves the norm
    x = torch.randn(8, 512, device=cuda)
    y = ops.hadamard_rotate(x, 128, torch.float32)
    torch.testing.assert_close(y.norm(dim=1), x.norm(dim=1), rtol=1e-5, atol=0)


@pytest.mark.parametrize("M", [3, 200])
def test_int4_linear_with_rotation(cuda, M):
    N, K, g = 192, 512, 64
    rng = np.random.default_rng(M)
    w = rng.standard_normal((N, K)).astype(np.float32) * 0.05
    x = rng.standard_normal((M, K)).astype(np.float32)
    R = ops.get_group_rotation(K, g, "cpu").numpy().astype(np.float64)
    w_rot = (w.reshape(-1, g).astype(np.float64) @ R.T).reshape(N, K).astype(np.float32)  # fold (load time)
    p, s = O.quantize_pack_int4(w_rot)
    x_rot = (x.reshape(-1, g).astype(np.float64) @ R.T).reshape(M, K).astype(np.float32)  # forward time
    xt = torch.from_numpy(x).to(cuda)
    y = ops.int4_linear(xt, torch.from_numpy(p).to(cuda), torch.from_numpy(s).to(cuda), None, rotation_group=g)
    ref = O.w4a16_matmul(O.round_to_bf16(x_rot), p, s)
    m = O.parity_metrics(y.cpu().numpy(), ref)
    assert m["max_abs_over_max_ref"] <= 2e-2 and m["mean_rel"] <= 5e-3, m
    # and the rotation undoes itself: close to the unrotated float product
    far = O.parity_metrics(y.cpu().numpy(), x @ w.T)
    assert far["mean_rel"] < 0.2, far
