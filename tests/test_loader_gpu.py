"""Gfx906Int4UnetLoader.load_unet end to end (reference nodes.py:483-599), with
stand-ins for the ComfyUI modules it calls (folder_paths, comfy.utils,
comfy.model_detection, comfy.model_management, comfy.model_patcher): a
synthetic bf16 checkpoint with the "model.diffusion_model." prefix is read,
stripped, quantized on the GPU into weight_q4 / weight_scale buffers, the model
is built with custom_operations = Gfx906Int4Ops and loaded, and its forward
matches the oracle's quantize-then-W4A16 of the same weights."""
import sys
import types

import numpy as np
import pytest
import torch

import oracle as O
from comfy_ui_gfx906_tools_b200 import nodes, ops

pytestmark = pytest.mark.gpu

PREFIX = "model.diffusion_model."


class TinyNet(torch.nn.Module):
    def __init__(self, operations, dtype):
        super().__init__()
        self.a = operations.Linear(64, 96, bias=True, dtype=dtype)
        self.b = operations.Linear(96, 32, bias=False, dtype=dtype)
        self.small = operations.Linear(16, 8, bias=True, dtype=dtype)  # in_features < 32: stays float

    def forward(self, x):
        return self.b(torch.nn.functional.gelu(self.a(x)))


def _checkpoint(seed=3):
    g = torch.Generator().manual_seed(seed)
    sd = {
        "a.weight": torch.randn(96, 64, generator=g) * 0.05,
        "a.bias": torch.randn(96, generator=g) * 0.01,
        "b.weight": torch.randn(32, 96, generator=g) * 0.05,
        "small.weight": torch.randn(8, 16, generator=g) * 0.05,
        "small.bias": torch.randn(8, generator=g) * 0.01,
    }
    return {PREFIX + k: v.to(torch.bfloat16) for k, v in sd.items()}


@pytest.fixture
def comfy_loader_stubs(monkeypatch):
    ckpt = _checkpoint()
    calls = {}

    fp = types.ModuleType("folder_paths")
    fp.get_full_path_or_raise = lambda kind, name: f"/models/{kind}/{name}"

    cu = types.ModuleType("comfy.utils")
    cu.load_torch_file = lambda path, return_metadata=False: (dict(ckpt), {"source": path})
    cu.state_dict_prefix_replace = lambda sd, rep, filter_keys=False: {
        k.replace(p, r, 1): v for k, v in sd.items() for p, r in rep.items() if k.startswith(p) or not filter_keys}
    cu.calculate_parameters = lambda sd: sum(v.numel() for v in sd.values())
    cu.weight_dtype = lambda sd: torch.bfloat16

    class Config:
        supported_inference_dtypes = [torch.bfloat16, torch.float32]
        custom_operations = None

        def set_inference_dtype(self, dtype, manual_cast, device=None):
            calls["inference_dtype"] = (dtype, manual_cast, device)
            self.dtype = dtype

        def get_model(self, sd, prefix):
            model = torch.nn.Module()
            model.diffusion_model = TinyNet(self.custom_operations, self.dtype)
            model.load_model_weights = lambda sd, p: model.diffusion_model.load_state_dict(sd)
            calls["get_model_keys"] = sorted(sd)
            return model

    md = types.ModuleType("comfy.model_detection")
    md.unet_prefix_from_state_dict = lambda sd: PREFIX
    md.model_config_from_unet = lambda sd, prefix, metadata=None: Config()

    mm = types.ModuleType("comfy.model_management")
    mm.unet_offload_device = lambda: torch.device("cpu")
    mm.unet_dtype = lambda model_params=0, supported_dtypes=(), weight_dtype=None: torch.bfloat16
    mm.unet_manual_cast = lambda dtype, device, supported: None
    mm.is_device_cpu = lambda d: torch.device(d).type == "cpu"

    mp = types.ModuleType("comfy.model_patcher")

    class ModelPatcher:
        def __init__(self, model, load_device=None, offload_device=None):
            self.model, self.load_device, self.offload_device = model, load_device, offload_device
    mp.ModelPatcher = ModelPatcher

    comfy = types.ModuleType("comfy")
    comfy.utils, comfy.model_detection, comfy.model_management, comfy.model_patcher = cu, md, mm, mp
    for name, mod in (("folder_paths", fp), ("comfy", comfy), ("comfy.utils", cu), ("comfy.model_detection", md),
                      ("comfy.model_management", mm), ("comfy.model_patcher", mp)):
        monkeypatch.setitem(sys.modules, name, mod)
    return ckpt, calls


def test_load_unet_quantizes_and_runs(cuda, comfy_loader_stubs):
    ckpt, calls = comfy_loader_stubs
    (patcher,) = nodes.Gfx906Int4UnetLoader().load_unet("tiny.safetensors", "cuda:0")
    net = patcher.model.diffusion_model
    assert patcher.load_device == torch.device("cuda:0")
    assert isinstance(net.a, ops.Gfx906Int4Ops.Linear) and net.a.quantized and net.b.quantized
    assert not net.small.quantized  # in_features 16 < 32 stays a float Linear
    assert "a.weight_q4" in calls["get_model_keys"] and "small.weight" in calls["get_model_keys"]
    # buffers = the reference quantizer's output for CUDA tensors (reciprocal divide)
    for name in ("a", "b"):
        w = ckpt[PREFIX + name + ".weight"].float().numpy()
        pw, sw = O.quantize_pack_int4(w, div_mode="recip")
        assert np.array_equal(getattr(net, name).weight_q4.numpy(), pw)
        assert np.array_equal(getattr(net, name).weight_scale.numpy(), sw)
    net = net.to(cuda)
    x = torch.randn(5, 64, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    with torch.no_grad():
        y = net(x.to(cuda)).float().cpu().numpy()
    pa, sa = O.quantize_pack_int4(ckpt[PREFIX + "a.weight"].float().numpy(), div_mode="recip")
    pb, sb = O.quantize_pack_int4(ckpt[PREFIX + "b.weight"].float().numpy(), div_mode="recip")
    h = O.w4a16_matmul(x.float().numpy(), pa, sa, ckpt[PREFIX + "a.bias"].float().numpy())
    h = torch.nn.functional.gelu(torch.from_numpy(h).to(torch.bfloat16)).float().numpy()
    ref = O.w4a16_matmul(h, pb, sb)
    m = O.parity_metrics(y, ref)
    assert m["nonfinite"] == 0 and m["max_abs_over_max_ref"] <= 2e-2 and m["mean_rel"] <= 5e-3, m
