"""ComfyUI node layer for the int4 weight path (reference: nodes/ComfyUI-Gfx906Int4/nodes.py).

Same node class names, inputs, return types and titles as the reference for the
nodes on the int4 DiT path:

  * ``Gfx906Int4UnetLoader`` (nodes.py:450-599): load a diffusion model straight
    into packed int4 Linears (plain float safetensors, GGUF with lossless Q4_0
    repack, other GGUF types via ComfyUI-GGUF's dequantizer);
  * ``Gfx906Int4Transcode`` (nodes.py:290-327): MODEL -> MODEL swap of every
    eligible Linear for ``Gfx906Int4Ops.Linear``;
  * ``Gfx906Int4Patch`` (nodes.py:71-124): the W4A16 emulation (quantize then
    dequantize weights in place) -- the accuracy reference of this path.

The format dispatch (``_quantize_module_weight``, nodes.py:157-223), the Linear
walk (``_transcode_linears``, nodes.py:226-287) and the state-dict quantizer of
the loader are plain functions here so they run without ComfyUI; the node
methods import ComfyUI lazily. Packing and dequantization run as this
package's GPU kernels (``ops``); results equal the reference's torch code.

The multi-GPU split node (Gfx906RowSplitKrea2) lives in row_split.py.
Out of scope (not the int4 DiT linear path): the CLIP transcode / loader
nodes, the fused-attention node and the int8 VAE node of the reference.
"""
from __future__ import annotations

import re

import torch

from . import ops
from .ops import (BLOCK, Gfx906Int4Ops, apply_group_rotation, choose_rotation_group, get_group_rotation,
                  quantize_pack_int4, repack_q4_0_native)

DEFAULT_SPARED_SUFFIXES = ("x_embedder", "final_layer", "cap_embedder", "t_embedder")


# ---------------------------------------------------------------------------
# W4A16 emulation (nodes.py:43-52)
# ---------------------------------------------------------------------------
def quantize_dequantize_int4(t: torch.Tensor, block: int = BLOCK) -> torch.Tensor:
    """Round-to-nearest int4 (block 32, amax / 7) then dequantize back to
    t.dtype: the weight the W4A16 emulation multiplies with. Runs as two GPU
    kernels (pack, dequant); a CPU tensor is staged through the current GPU
    with torch-CPU quantizer semantics. Values equal the reference's; the one
    representational difference is that a negative input rounding to code 0
    comes back as +0.0 (the reference keeps -0.0)."""
    shape = t.shape
    K = shape[-1]
    if K % block != 0:
        return t
    packed, scale = quantize_pack_int4(t.float() if t.dtype not in (torch.float32, torch.float16, torch.bfloat16)
                                       else t, block)
    dev_packed = packed if packed.is_cuda else packed.to("cuda")
    dev_scale = scale if scale.is_cuda else scale.to("cuda")
    out = ops.dequantize_int4(dev_packed.reshape(-1, K // 2), dev_scale.reshape(-1, K // block), t.dtype)
    return out.reshape(shape).to(t.device)


def find_max_layer_index(diffusion_model, prefix="layers."):
    max_idx = -1
    for name, _ in diffusion_model.named_modules():
        m = re.match(re.escape(prefix) + r"(\d+)\.", name)
        if m:
            max_idx = max(max_idx, int(m.group(1)))
    return max_idx


def make_activation_quant_hook():
    def hook(module, inputs):
        return (quantize_dequantize_int4(inputs[0]),) + inputs[1:]
    return hook


def patch_model_w4a16(diffusion_model: torch.nn.Module, mode: str = "w4a16", spare_first_last_layers: bool = True,
                      block_size: int = BLOCK):
    """In-place body of Gfx906Int4Patch.patch (nodes.py:93-124); returns the
    (quantized, spared, hooked) counts."""
    spared_prefixes = tuple()
    if spare_first_last_layers:
        max_idx = find_max_layer_index(diffusion_model)
        spared_prefixes = DEFAULT_SPARED_SUFFIXES
        if max_idx >= 0:
            spared_prefixes = spared_prefixes + ("layers.0.", f"layers.{max_idx}.")
    quantized = spared = hooked = 0
    named = dict(diffusion_model.named_modules())
    with torch.no_grad():
        for name, param in diffusion_model.named_parameters():
            if not name.endswith(".weight") or param.ndim != 2:
                continue
            if param.shape[1] % block_size != 0 or param.shape[1] < block_size:
                continue
            mod_name = name[: -len(".weight")]
            if mod_name.startswith(spared_prefixes):
                spared += 1
                continue
            param.data.copy_(quantize_dequantize_int4(param.data.float(), block_size).to(param.dtype))
            quantized += 1
            if mode == "w4a4_naive" and mod_name in named:
                named[mod_name].register_forward_pre_hook(make_activation_quant_hook())
                hooked += 1
    return quantized, spared, hooked


# ---------------------------------------------------------------------------
# format dispatch (nodes.py:157-223) and Linear walk (nodes.py:226-287)
# ---------------------------------------------------------------------------
class _RawTensorModule:
    """A raw state-dict tensor shaped like a Linear, so the loader and the
    transcode node share one format dispatch (nodes.py:145-155)."""

    def __init__(self, weight, out_features, in_features):
        self.weight = weight
        self.out_features = out_features
        self.in_features = in_features


def _get_gguf_dequant_module():
    import sys
    return sys.modules.get("ComfyUI-GGUF.dequant")


def _get_gguf_loader_module():
    import sys
    return sys.modules.get("ComfyUI-GGUF.loader")


def _is_q4_0(tensor_type) -> bool:
    try:
        import gguf  # the ggml type enum ComfyUI-GGUF tags its tensors with
        return tensor_type == gguf.GGMLQuantizationType.Q4_0
    except ImportError:
        return getattr(tensor_type, "name", str(tensor_type)) in ("Q4_0", "GGMLQuantizationType.Q4_0")


def _quantize_module_weight(module, block_size, rotation_group=0):
    """(packed int8, scale fp32, source tag) for any Linear-like module:
    Q4_0 -> lossless repack; other GGUF types -> ComfyUI-GGUF dequant then RTN;
    comfy QuantizedTensor -> dequantize() then RTN; plain float -> RTN."""
    w = module.weight
    tensor_type = getattr(w, "tensor_type", None)
    if tensor_type is not None and not rotation_group and block_size == BLOCK and _is_q4_0(tensor_type):
        data = w.data if hasattr(w, "data") else w
        packed, scale = repack_q4_0_native(torch.as_tensor(data), module.out_features, module.in_features, block_size)
        return packed, scale, "gguf_q4_0_repack"
    if tensor_type is not None:
        dequant_mod = _get_gguf_dequant_module()
        if dequant_mod is None:
            raise RuntimeError("This model has GGUF-quantized weights but ComfyUI-GGUF is not loaded "
                               "(needed to dequantize them before re-quantizing to int4).")
        w_float, source_tag = dequant_mod.dequantize_tensor(w, dtype=torch.float32), "gguf_dequant_requant"
    else:
        try:
            from comfy_kitchen.tensor import QuantizedTensor  # type: ignore
        except ImportError:
            QuantizedTensor = None
        if QuantizedTensor is not None and isinstance(w, QuantizedTensor):
            w_for_dequant = w.cuda() if w.device.type == "cpu" and torch.cuda.is_available() else w
            w_float, source_tag = w_for_dequant.dequantize().float(), "comfy_quantized_dequant_requant"
        else:
            if w.dtype not in (torch.float32, torch.float16, torch.bfloat16):
                raise RuntimeError(
                    f"weight is already quantized ({w.dtype}), not a plain float weight, GGUF tensor, or recognized "
                    f"QuantizedTensor -- this looks like a third-party quantization format this transcoder doesn't "
                    f"know how to decode.")
            w_float, source_tag = w.detach().float(), "plain"
    if rotation_group:
        R = get_group_rotation(module.in_features, rotation_group, w_float.device)
        w_float = apply_group_rotation(w_float, R, rotation_group)
        source_tag += "_rotated"
    packed, scale = quantize_pack_int4(w_float, block_size)
    return packed, scale, source_tag


def _is_mixed_precision_op(module) -> bool:
    try:
        import comfy.ops  # type: ignore
        return isinstance(module, comfy.ops.MixedPrecisionOp) and getattr(module, "weight", None) is not None
    except Exception:
        return False


def _transcode_linears(root_module, block_size, rotate):
    """Replace every eligible Linear under root_module with Gfx906Int4Ops.Linear
    in place; returns (converted, skipped, source_counts)."""
    named = dict(root_module.named_modules())
    converted, skipped = 0, 0
    source_counts = {}
    with torch.no_grad():
        for name, module in list(named.items()):
            if not (isinstance(module, torch.nn.Linear) or _is_mixed_precision_op(module)):
                continue
            if getattr(module.weight, "ndim", 2) != 2:
                skipped += 1
                continue
            in_f, out_f = module.in_features, module.out_features
            if in_f % block_size != 0 or in_f < block_size:
                skipped += 1
                continue
            rotation_group = (choose_rotation_group(in_f) or 0) if rotate else 0
            device = module.weight.device
            out_dtype = module.weight.dtype
            packed, scale, source_tag = _quantize_module_weight(module, block_size, rotation_group)
            packed, scale = packed.to(device), scale.to(device)
            source_counts[source_tag] = source_counts.get(source_tag, 0) + 1
            new_linear = Gfx906Int4Ops.Linear(in_f, out_f, bias=module.bias is not None, device=device,
                                              dtype=out_dtype, rotation_group=rotation_group)
            new_linear.weight_q4.copy_(packed)
            new_linear.weight_scale.copy_(scale)
            if module.bias is not None:
                new_linear.bias.data.copy_(module.bias.detach().float().to(out_dtype))
            parent_name, _, attr = name.rpartition(".")
            parent = named[parent_name] if parent_name else root_module
            setattr(parent, attr, new_linear)
            converted += 1
    del named
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    return converted, skipped, source_counts


def quantize_state_dict(sd: dict, device, block_size: int = BLOCK):
    """The loader's state-dict pass (nodes.py:540-576, without the ConvRot
    branch): every 2-D ``*.weight`` with in_features % 32 == 0 becomes
    ``*.weight_q4`` / ``*.weight_scale`` (quantized or repacked on `device`,
    stored on the CPU like the reference); everything else passes through.
    Returns (quantized_sd, quantized, passthrough)."""
    torch_device = torch.device(device)
    quantized_sd = {}
    quantized = passthrough = 0
    for key in list(sd.keys()):
        t = sd[key]
        base = key[: -len(".weight")] if key.endswith(".weight") else None
        if base is not None and t.ndim == 2 and t.shape[1] % block_size == 0 and t.shape[1] >= block_size:
            fake = _RawTensorModule(t, t.shape[0], t.shape[1])
            if torch_device.type == "cuda" and getattr(t, "tensor_type", None) is None:
                fake.weight = t.to(torch_device)
            packed, scale, _tag = _quantize_module_weight(fake, block_size)
            quantized_sd[base + ".weight_q4"] = packed.cpu()
            quantized_sd[base + ".weight_scale"] = scale.cpu()
            quantized += 1
        else:
            quantized_sd[key] = t
            passthrough += 1
    return quantized_sd, quantized, passthrough


def _device_list():
    return ["cpu"] + [f"cuda:{i}" for i in range(torch.cuda.device_count())]


def _default_device(devices):
    non_cpu = [d for d in devices if d != "cpu"]
    return non_cpu[1] if len(non_cpu) > 1 else (non_cpu[0] if non_cpu else "cpu")


# ---------------------------------------------------------------------------
# node classes
# ---------------------------------------------------------------------------
class Gfx906Int4Patch:
    """MODEL -> MODEL: W4A16 (or naive W4A4) quantize-dequantize of a loaded
    model's Linear weights, for accuracy tests on real prompts."""

    @classmethod
    def INPUT_TYPES(s):
        return {"required": {
            "model": ("MODEL",),
            "mode": (["w4a16", "w4a4_naive"], {"default": "w4a16"}),
            "spare_first_last_layers": ("BOOLEAN", {"default": True}),
            "block_size": ("INT", {"default": 32, "min": 16, "max": 256, "step": 16}),
        }}

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "patch"
    CATEGORY = "gfx906"
    TITLE = "Gfx906 Int4 Quantize (test)"

    def patch(self, model, mode, spare_first_last_layers, block_size):
        if block_size != BLOCK:
            raise ValueError(f"block_size must be {BLOCK} on this build (the GPU quantizer is block-32), "
                             f"got {block_size}")
        model = model.clone()
        q, s, h = patch_model_w4a16(model.model.diffusion_model, mode, spare_first_last_layers, block_size)
        print(f"[Gfx906Int4Patch] mode={mode} quantized={q} spared={s} activation_hooks={h}")
        return (model,)


class Gfx906Int4Transcode:
    """MODEL -> MODEL: every eligible Linear becomes a packed int4 Linear
    (Q4_0: lossless repack; other formats: dequantize then RTN)."""

    @classmethod
    def INPUT_TYPES(s):
        return {"required": {
            "model": ("MODEL",),
            "activation_rotation": ("BOOLEAN", {"default": False, "tooltip": "Randomized Hadamard rotation of "
                                    "weight+activation before quantizing; costs the lossless Q4_0 repack path."}),
        }}

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "transcode"
    CATEGORY = "gfx906"
    TITLE = "Gfx906 Int4 Transcode (native kernel, any source)"

    def transcode(self, model, activation_rotation):
        model = model.clone()
        converted, skipped, source_counts = _transcode_linears(model.model.diffusion_model, BLOCK,
                                                               activation_rotation)
        print(f"[Gfx906Int4Transcode] converted={converted} skipped={skipped} sources={source_counts}")
        return (model,)


class Gfx906Int4UnetLoader:
    """Load a diffusion model directly into packed int4 Linears (weights are
    quantized or repacked at load time and never materialised in full
    precision on the GPU)."""

    @classmethod
    def INPUT_TYPES(s):
        import folder_paths  # type: ignore  # noqa: F401
        devices = _device_list()
        names = list(folder_paths.get_filename_list("diffusion_models"))
        if "unet_gguf" in folder_paths.folder_names_and_paths:
            names += [n for n in folder_paths.get_filename_list("unet_gguf") if n not in names]
        return {"required": {"unet_name": (names,), "device": (devices, {"default": _default_device(devices)})}}

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "load_unet"
    CATEGORY = "gfx906"
    TITLE = "Gfx906 Int4 UNet Loader (native kernel)"

    def load_unet(self, unet_name, device):
        import comfy.model_detection  # type: ignore
        import comfy.model_management  # type: ignore
        import comfy.model_patcher  # type: ignore
        import comfy.utils  # type: ignore
        import folder_paths  # type: ignore

        unet_path = folder_paths.get_full_path_or_raise("diffusion_models", unet_name)
        torch_device = torch.device(device)
        if unet_path.endswith(".gguf"):
            gguf_loader = _get_gguf_loader_module()
            if gguf_loader is None:
                raise RuntimeError("Loading a .gguf model requires ComfyUI-GGUF to be loaded (for gguf_sd_loader).")
            sd, _extra = gguf_loader.gguf_sd_loader(unet_path)
            metadata = None
        else:
            sd, metadata = comfy.utils.load_torch_file(unet_path, return_metadata=True)
            prefix = comfy.model_detection.unet_prefix_from_state_dict(sd)
            temp_sd = comfy.utils.state_dict_prefix_replace(sd, {prefix: ""}, filter_keys=True)
            if len(temp_sd) > 0:
                sd = temp_sd
        quantized_sd, quantized, passthrough = quantize_state_dict(sd, torch_device)
        print(f"[Gfx906Int4UnetLoader] quantized={quantized} passthrough_tensors={passthrough} device={device}")
        model_config = comfy.model_detection.model_config_from_unet(sd, "", metadata=metadata)
        if model_config is None:
            raise RuntimeError(f"Could not detect model type of: {unet_path}")
        parameters = comfy.utils.calculate_parameters(sd)
        weight_dtype = comfy.utils.weight_dtype(sd)
        offload_device = comfy.model_management.unet_offload_device()
        unet_weight_dtype = list(model_config.supported_inference_dtypes)
        unet_dtype = comfy.model_management.unet_dtype(model_params=parameters, supported_dtypes=unet_weight_dtype,
                                                       weight_dtype=weight_dtype)
        manual_cast_dtype = comfy.model_management.unet_manual_cast(unet_dtype, torch_device,
                                                                    model_config.supported_inference_dtypes)
        model_config.set_inference_dtype(unet_dtype, manual_cast_dtype, device=torch_device)
        model_config.custom_operations = Gfx906Int4Ops
        model = model_config.get_model(quantized_sd, "")
        model_patcher = comfy.model_patcher.ModelPatcher(model, load_device=torch_device,
                                                         offload_device=offload_device)
        if not comfy.model_management.is_device_cpu(offload_device):
            model.to(offload_device)
        model.load_model_weights(quantized_sd, "")
        return (model_patcher,)


from .row_split import Gfx906RowSplitKrea2  # noqa: E402  (the multi-GPU split node, row_split.py)
from .attention import Gfx906FusedAttention  # noqa: E402  (the fused attention node, attention.py)

NODE_CLASS_MAPPINGS = {
    "Gfx906Int4Patch": Gfx906Int4Patch,
    "Gfx906Int4UnetLoader": Gfx906Int4UnetLoader,
    "Gfx906Int4Transcode": Gfx906Int4Transcode,
    "Gfx906RowSplitKrea2": Gfx906RowSplitKrea2,
    "Gfx906FusedAttention": Gfx906FusedAttention,
}

NODE_DISPLAY_NAME_MAPPINGS = {
    "Gfx906Int4Transcode": "Gfx906 Int4 Transcode (native kernel, any source)",
    "Gfx906Int4Patch": "Gfx906 Int4 Quantize (test)",
    "Gfx906Int4UnetLoader": "Gfx906 Int4 UNet Loader (native kernel)",
    "Gfx906RowSplitKrea2": "Gfx906 Split Krea2 (2 GPUs)",
    "Gfx906FusedAttention": "Gfx906 Fused Attention",
}
