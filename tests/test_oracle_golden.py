"""The CPU oracle against golden vectors produced by running the reference's
own Python (tests/golden/make_golden.py). Pins the oracle before it is used
to judge the GPU kernels."""
import numpy as np
import pytest

import oracle as O


@pytest.mark.parametrize("src", ["f32", "f16", "bf16"])
def test_quantize_pack_int4_matches_reference(golden, src):
    p, s = O.quantize_pack_int4(golden[f"qp_{src}_in"])
    assert np.array_equal(p, golden[f"qp_{src}_packed"])
    assert np.array_equal(s.view(np.uint32), golden[f"qp_{src}_scale"].view(np.uint32))


@pytest.mark.parametrize("src", ["f32", "f16", "bf16"])
def test_dequant_matches_reference(golden, src):
    d = O.dequant_int4(golden[f"qp_{src}_packed"], golden[f"qp_{src}_scale"])
    assert np.array_equal(d.view(np.uint32), golden[f"qp_{src}_dequant_f32"].view(np.uint32))


def test_repack_q4_0_matches_reference(golden):
    p, s = O.repack_q4_0_native(golden["q40_raw"], 40, 192)
    assert np.array_equal(p, golden["q40_packed"])
    assert np.array_equal(s, golden["q40_scale"])
    assert np.array_equal(O.dequant_int4(p, s), golden["q40_dequant_f32"])
    assert np.array_equal(O.dequant_int4_bf16_bits(p, s), golden["q40_dequant_bf16_bits"])


def test_q4_0_builder_roundtrip(golden):
    assert np.array_equal(O.build_q4_0_bytes(golden["q40_u"], golden["q40_d"]), golden["q40_raw"])
    # the repack is lossless: dequant == (u - 8) * d exactly
    p, s = O.repack_q4_0_native(golden["q40_raw"], 40, 192)
    want = (golden["q40_u"].astype(np.float32) - 8) * np.repeat(golden["q40_d"].astype(np.float32), 32, axis=1)
    assert np.array_equal(O.dequant_int4(p, s), want)


def test_quantize_dequantize_matches_reference(golden):
    out = O.quantize_dequantize_int4(golden["qdq_in"])
    assert np.array_equal(out.view(np.uint32), golden["qdq_f32"].view(np.uint32))
    bf = O.bf16_bits_to_f32(golden["qdq_bf16_in_bits"])
    assert np.array_equal(O.f32_to_bf16_bits(O.quantize_dequantize_int4(bf)), golden["qdq_bf16_bits"])


def test_int8_dequant_matches_reference(golden):
    assert np.array_equal(O.dequant_int8(golden["i8_q"], golden["i8_s"]), golden["i8_dequant"])


def test_gemm_oracle_matches_reference(golden):
    x = O.bf16_bits_to_f32(golden["gemm_x_bits"])
    b = O.bf16_bits_to_f32(golden["gemm_bias_bits"])
    y = O.w4a16_matmul(x, golden["q40_packed"], golden["q40_scale"], b)
    m = O.parity_metrics(y, golden["gemm_y_f32"])
    assert m["max_abs_over_max_ref"] < 1e-6 and m["mean_rel"] < 1e-6


def test_loader_quantize_on_load_matches_reference(golden):
    # Gfx906Int4Ops.Linear quantize-on-load with rotation (ops.py:228-246)
    grp = int(golden["load_rotation_group"])
    assert grp == 128
    R = golden["rot_R_256_128"]
    w = golden["load_w"]
    rotated = (w.reshape(-1, grp) @ R.T).reshape(w.shape).astype(np.float32)
    p, s = O.quantize_pack_int4(rotated)
    # the rotation matmul is a float reduction; allow rare last-bit code flips
    codes_ref = O.unpack_int4_codes(golden["load_q4"])
    codes = O.unpack_int4_codes(p)
    assert (codes != codes_ref).mean() < 1e-3
    assert np.allclose(s, golden["load_scale"], rtol=1e-6, atol=0)


def test_parity_metrics_definition():
    ref = np.array([[1.0, -2.0], [3.0, -4.0]])
    got = ref + np.array([[0.1, 0.0], [0.0, -0.2]])
    m = O.parity_metrics(got, ref)
    assert m["max_abs_over_max_ref"] == pytest.approx(0.2 / 4.0)
    assert m["mean_rel"] == pytest.approx((0.3 / 4) / (10 / 4))


def test_bf16_rounding_helper():
    vals = np.array([1.0, 1.00390625, 1.005859375, -3.14159, 65504.0, 1e-30], dtype=np.float32)
    import torch
    want = torch.from_numpy(vals).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(O.f32_to_bf16_bits(vals), want)
