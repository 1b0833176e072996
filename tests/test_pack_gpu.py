"""GPU parity of the weight-format kernels against the CPU oracle and the
reference-generated golden vectors: bit-exact (integer / byte work, and the
fp32 / bf16 dequant which is one IEEE multiply plus one rounding)."""
import numpy as np
import pytest
import torch

import oracle as O
from comfy_ui_gfx906_tools_b200 import ops, synthetic

pytestmark = pytest.mark.gpu


def _bits16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def test_dequant_golden_bf16_bitexact(cuda, golden):
    p = torch.from_numpy(golden["q40_packed"]).to(cuda)
    s = torch.from_numpy(golden["q40_scale"]).to(cuda)
    got = ops.dequantize_int4(p, s, torch.bfloat16)
    assert np.array_equal(_bits16(got), golden["q40_dequant_bf16_bits"])
    got32 = ops.dequantize_int4(p, s, torch.float32).cpu().numpy()
    assert np.array_equal(got32.view(np.uint32), golden["q40_dequant_f32"].view(np.uint32))


@pytest.mark.parametrize("src", ["f32", "f16", "bf16"])
def test_dequant_general_fp32_scales_bitexact(cuda, golden, src):
    # RTN scales (amax / 7) are arbitrary fp32 values: the product rounds in fp32
    p = torch.from_numpy(golden[f"qp_{src}_packed"]).to(cuda)
    s = torch.from_numpy(golden[f"qp_{src}_scale"]).to(cuda)
    got32 = ops.dequantize_int4(p, s, torch.float32).cpu().numpy()
    assert np.array_equal(got32.view(np.uint32), golden[f"qp_{src}_dequant_f32"].view(np.uint32))
    gotbf = ops.dequantize_int4(p, s, torch.bfloat16)
    assert np.array_equal(_bits16(gotbf), O.dequant_int4_bf16_bits(golden[f"qp_{src}_packed"], golden[f"qp_{src}_scale"]))


def test_dequant_random_large_bitexact(cuda):
    g = torch.Generator().manual_seed(7)
    N, K = 768, 3072
    packed = torch.randint(-128, 128, (N, K // 2), generator=g, dtype=torch.int8)
    scale = torch.rand(N, K // 32, generator=g) * 0.01 + 1e-6
    got = ops.dequantize_int4(packed.to(cuda), scale.to(cuda), torch.bfloat16)
    assert np.array_equal(_bits16(got), O.dequant_int4_bf16_bits(packed.numpy(), scale.numpy()))
    got16 = ops.dequantize_int4(packed.to(cuda), scale.to(cuda), torch.float16).cpu().numpy()
    want16 = O.dequant_int4(packed.numpy(), scale.numpy()).astype(np.float16)
    assert np.array_equal(got16.view(np.uint16), want16.view(np.uint16))


def test_repack_q4_0_golden(cuda, golden):
    raw = torch.from_numpy(golden["q40_raw"]).to(cuda)
    p, s = ops.repack_q4_0_native(raw, 40, 192)
    assert np.array_equal(p.cpu().numpy(), golden["q40_packed"])
    assert np.array_equal(s.cpu().numpy(), golden["q40_scale"])


def test_repack_q4_0_cpu_tensor_roundtrip(cuda, golden):
    # CPU input: staged through the GPU, result returned on the CPU like the reference
    p, s = ops.repack_q4_0_native(torch.from_numpy(golden["q40_raw"]), 40, 192)
    assert p.device.type == "cpu" and np.array_equal(p.numpy(), golden["q40_packed"])


def test_repack_q4_0_full_size(cuda):
    N, K = 3072, 3072
    raw, u, d = synthetic.q4_0_weight(N, K, seed=11)
    p, s = ops.repack_q4_0_native(raw.to(cuda), N, K)
    pw, sw = O.repack_q4_0_native(raw.numpy(), N, K)
    assert np.array_equal(p.cpu().numpy(), pw)
    assert np.array_equal(s.cpu().numpy(), sw)


@pytest.mark.parametrize("src", ["f32", "f16", "bf16"])
def test_quantize_pack_cpu_semantics_golden(cuda, golden, src):
    # a CPU tensor is quantized with torch-CPU semantics (IEEE amax / 7): the
    # golden vectors are the reference run on the CPU
    x = torch.from_numpy(golden[f"qp_{src}_in"])
    x = {"f32": x, "f16": x.half(), "bf16": x.bfloat16()}[src]
    p, s = ops.quantize_pack_int4(x)
    assert p.device.type == "cpu"
    assert np.array_equal(p.numpy(), golden[f"qp_{src}_packed"])
    assert np.array_equal(s.numpy().view(np.uint32), golden[f"qp_{src}_scale"].view(np.uint32))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_quantize_pack_cuda_semantics(cuda, dtype):
    # a CUDA tensor: torch-CUDA semantics (amax * (1/7)), the oracle's "recip" mode
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(300, 512, generator=g) * 0.05)
    x[0, :32] = 0
    x[1, :32] = torch.arange(32) - 15.5
    x = x.to(dtype)
    p, s = ops.quantize_pack_int4(x.to(cuda))
    pw, sw = O.quantize_pack_int4(x.float().numpy(), div_mode="recip")
    assert np.array_equal(p.cpu().numpy(), pw)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), sw.view(np.uint32))


def test_quantize_pack_matches_torch_on_cuda(cuda):
    # the reference's own torch expression evaluated on the GPU (ops.py:114-121)
    g = torch.Generator().manual_seed(5)
    t = (torch.randn(64, 256, generator=g) * 0.1).to(cuda)
    tb = t.reshape(-1, 8, 32).float()
    amax = tb.abs().amax(dim=-1, keepdim=True).clamp_min(1e-8)
    scale = amax / 7.0
    codes = torch.round(tb / scale).clamp(-8, 7).to(torch.int32).reshape(-1, 256)
    packed = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).to(torch.uint8).view(torch.int8)
    p, s = ops.quantize_pack_int4(t)
    assert torch.equal(p, packed)
    assert torch.equal(s, scale.reshape(64, 8))


def test_scales_to_f16(cuda):
    _, _, d = synthetic.q4_0_weight(64, 256, seed=2)
    s32 = d.float().to(cuda)
    s16 = ops.scales_to_f16_if_exact(s32)
    assert s16 is not None and torch.equal(s16.float(), s32)
    assert ops.scales_to_f16_if_exact(s32 * 1.0000001) is None
