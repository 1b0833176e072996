"""Node layer (reference nodes/ComfyUI-Gfx906Int4/nodes.py): node surface and
host logic on the CPU; the loader's format dispatch and Linear swap on the GPU
against the reference-generated golden vectors and the CPU oracle."""
import numpy as np
import pytest
import torch

import oracle as O
from comfy_ui_gfx906_tools_b200 import nodes, ops, synthetic


# ----------------------------------------------------------------- CPU ----
def test_node_names_and_titles_match_reference():
    # nodes.py:602-622 for the nodes on the int4 DiT path
    assert set(nodes.NODE_CLASS_MAPPINGS) == {"Gfx906Int4Patch", "Gfx906Int4UnetLoader", "Gfx906Int4Transcode",
                                              "Gfx906RowSplitKrea2", "Gfx906FusedAttention"}
    assert nodes.NODE_DISPLAY_NAME_MAPPINGS["Gfx906RowSplitKrea2"] == "Gfx906 Split Krea2 (2 GPUs)"
    assert nodes.NODE_DISPLAY_NAME_MAPPINGS["Gfx906FusedAttention"] == "Gfx906 Fused Attention"
    assert nodes.NODE_DISPLAY_NAME_MAPPINGS["Gfx906Int4Transcode"] == "Gfx906 Int4 Transcode (native kernel, any source)"
    assert nodes.NODE_DISPLAY_NAME_MAPPINGS["Gfx906Int4Patch"] == "Gfx906 Int4 Quantize (test)"
    assert nodes.NODE_DISPLAY_NAME_MAPPINGS["Gfx906Int4UnetLoader"] == "Gfx906 Int4 UNet Loader (native kernel)"
    for name, cls in nodes.NODE_CLASS_MAPPINGS.items():
        assert cls.CATEGORY == "gfx906" and cls.RETURN_TYPES == ("MODEL",)
        assert cls.TITLE == nodes.NODE_DISPLAY_NAME_MAPPINGS[name]


def test_node_inputs():
    t = nodes.Gfx906Int4Transcode.INPUT_TYPES()["required"]
    assert t["model"] == ("MODEL",) and t["activation_rotation"][0] == "BOOLEAN"
    p = nodes.Gfx906Int4Patch.INPUT_TYPES()["required"]
    assert p["mode"][0] == ["w4a16", "w4a4_naive"] and p["block_size"][1]["default"] == 32
    assert nodes.Gfx906Int4Transcode.FUNCTION == "transcode" and nodes.Gfx906Int4UnetLoader.FUNCTION == "load_unet"


def test_find_max_layer_index():
    # module names must continue past the index ("layers.2.0"), as in a real DiT block
    m = torch.nn.Module()
    m.layers = torch.nn.ModuleList([torch.nn.Sequential(torch.nn.Linear(4, 4)) for _ in range(3)])
    assert nodes.find_max_layer_index(m) == 2
    flat = torch.nn.Module()
    flat.layers = torch.nn.ModuleList([torch.nn.Linear(4, 4) for _ in range(3)])
    assert nodes.find_max_layer_index(flat) == -1


def test_quantize_module_weight_rejects_unknown_format():
    fake = nodes._RawTensorModule(torch.zeros(4, 64, dtype=torch.int8), 4, 64)
    with pytest.raises(RuntimeError, match="already quantized"):
        nodes._quantize_module_weight(fake, 32)


def test_gguf_non_q4_0_needs_comfyui_gguf():
    import gguf
    w = torch.zeros(4, 64)
    w.tensor_type = gguf.GGMLQuantizationType.Q8_0
    with pytest.raises(RuntimeError, match="ComfyUI-GGUF is not loaded"):
        nodes._quantize_module_weight(nodes._RawTensorModule(w, 4, 64), 32)


def test_linear_quantized_rule_and_buffers():
    lin = ops.Gfx906Int4Ops.Linear(96, 40, bias=True)
    assert lin.quantized and lin.weight_q4.shape == (40, 48) and lin.weight_q4.dtype == torch.int8
    assert lin.weight_scale.shape == (40, 3) and lin.weight_scale.dtype == torch.float32
    assert set(lin.state_dict()) == {"weight_q4", "weight_scale", "bias"}
    narrow = ops.Gfx906Int4Ops.Linear(12, 8, bias=False)  # ops.py:206-212: too narrow for a block
    assert not narrow.quantized and narrow.weight.shape == (8, 12)
    with torch.no_grad():
        narrow.weight.copy_(torch.randn(8, 12))
    x = torch.randn(3, 12)
    assert torch.allclose(narrow(x), x @ narrow.weight.t())


def test_rotation_helpers_match_reference(golden):
    for kin in (96, 256, 40):
        want = int(golden[f"rot_group_{kin}"])
        assert (ops.choose_rotation_group(kin) or -1) == want
    R = ops.get_group_rotation(256, 128, "cpu")
    assert np.array_equal(R.numpy(), golden["rot_R_256_128"])


def test_load_quantizing_ops_rejects_bad_weight():
    LoadOps = ops.make_load_quantizing_ops(object, "cpu", False)
    lin = LoadOps.Linear(64, 8, bias=False)
    with pytest.raises(RuntimeError, match=r"expected a float \[8, 64\] weight"):
        lin.load_state_dict({"weight": torch.zeros(8, 32)})


# ----------------------------------------------------------------- GPU ----
@pytest.mark.gpu
def test_quantize_module_weight_plain_matches_reference(cuda, golden):
    w = torch.from_numpy(golden["qmw_in_bits"].view(np.int16)).view(torch.bfloat16)
    pk, sc, tag = nodes._quantize_module_weight(nodes._RawTensorModule(w, 16, 64), 32)
    assert tag == str(golden["qmw_tag"]) == "plain"
    assert np.array_equal(pk.numpy(), golden["qmw_packed"]) and np.array_equal(sc.numpy(), golden["qmw_scale"])


@pytest.mark.gpu
def test_quantize_module_weight_q4_0_repack(cuda, golden):
    import gguf
    raw = torch.from_numpy(golden["q40_raw"])
    raw.tensor_type = gguf.GGMLQuantizationType.Q4_0
    pk, sc, tag = nodes._quantize_module_weight(nodes._RawTensorModule(raw, 40, 192), 32)
    assert tag == "gguf_q4_0_repack"
    assert np.array_equal(pk.cpu().numpy(), golden["q40_packed"]) and np.array_equal(sc.cpu().numpy(), golden["q40_scale"])


@pytest.mark.gpu
def test_quantize_dequantize_matches_reference(cuda, golden):
    out = nodes.quantize_dequantize_int4(torch.from_numpy(golden["qdq_in"]))
    assert np.array_equal(out.numpy(), golden["qdq_f32"])  # values equal (+0.0 == -0.0)
    bf = torch.from_numpy(golden["qdq_bf16_in_bits"].view(np.int16)).view(torch.bfloat16)
    got = nodes.quantize_dequantize_int4(bf)
    want = torch.from_numpy(golden["qdq_bf16_bits"].view(np.int16)).view(torch.bfloat16)
    assert torch.equal(got.float(), want.float())


@pytest.mark.gpu
def test_load_quantizing_ops_matches_reference(cuda, golden):
    LoadOps = ops.make_load_quantizing_ops(object, "cpu", True)
    lin = LoadOps.Linear(256, 24, bias=True)
    lin.load_state_dict({"weight": torch.from_numpy(golden["load_w"]), "bias": torch.zeros(24)})
    assert lin.rotation_group == int(golden["load_rotation_group"])
    codes = O.unpack_int4_codes(lin.weight_q4.numpy())
    assert (codes != O.unpack_int4_codes(golden["load_q4"])).mean() < 1e-3
    assert np.allclose(lin.weight_scale.numpy(), golden["load_scale"], rtol=1e-6, atol=0)
    assert LoadOps.Linear.quantized_on_load == 1


@pytest.mark.gpu
def test_transcode_linears_swaps_and_matches_w4a16(cuda):
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(128, 96), torch.nn.GELU(), torch.nn.Linear(96, 64),
                                torch.nn.Linear(64, 12), torch.nn.Linear(12, 8)).to(cuda, torch.bfloat16)
    ref_w = [m.weight.detach().float().cpu().numpy() for m in model if isinstance(m, torch.nn.Linear)]
    x = torch.randn(5, 128, device=cuda, dtype=torch.bfloat16)
    converted, skipped, sources = nodes._transcode_linears(model, 32, False)
    assert converted == 3 and skipped == 1 and sources == {"plain": 3}
    assert isinstance(model[0], ops.Gfx906Int4Ops.Linear) and isinstance(model[4], torch.nn.Linear)
    # layer 0 alone: kernel output vs the oracle W4A16 emulation of the same weights (CUDA quantizer semantics)
    p, s = O.quantize_pack_int4(ref_w[0], div_mode="recip")
    y = model[0](x).float().cpu().numpy()
    ref = O.w4a16_matmul(x.float().cpu().numpy(), p, s, model[0].bias.detach().float().cpu().numpy())
    m = O.parity_metrics(y, ref)
    assert m["max_abs_over_max_ref"] <= 2e-2 and m["mean_rel"] <= 5e-3
    assert model(x).shape == (5, 8)


@pytest.mark.gpu
def test_quantize_state_dict(cuda):
    sd = {"a.weight": synthetic.float_weight(64, 96, 1).to(torch.bfloat16), "a.bias": torch.zeros(64),
          "narrow.weight": torch.zeros(8, 12), "norm.scale": torch.ones(96)}
    q, nq, npass = nodes.quantize_state_dict(sd, "cuda:0")
    assert nq == 1 and npass == 3
    assert q["a.weight_q4"].shape == (64, 48) and q["a.weight_scale"].shape == (64, 3)
    assert q["a.weight_q4"].device.type == "cpu" and "narrow.weight" in q
    p, s = O.quantize_pack_int4(sd["a.weight"].float().numpy(), div_mode="recip")
    assert np.array_equal(q["a.weight_q4"].numpy(), p) and np.array_equal(q["a.weight_scale"].numpy(), s)


@pytest.mark.gpu
def test_patch_model_w4a16(cuda):
    m = torch.nn.Module()
    m.layers = torch.nn.ModuleList([torch.nn.Sequential(torch.nn.Linear(64, 64)) for _ in range(3)]).to(cuda)
    before = m.layers[1][0].weight.detach().clone()
    q, s, h = nodes.patch_model_w4a16(m, "w4a16", True, 32)
    assert (q, s, h) == (1, 2, 0)  # layers.0. and layers.2. are spared (nodes.py:96-101)
    p, sc = O.quantize_pack_int4(before.cpu().numpy(), div_mode="recip")
    assert np.array_equal(m.layers[1][0].weight.detach().cpu().numpy(), O.dequant_int4(p, sc))
