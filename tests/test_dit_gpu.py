"""The int4 Flux-architecture DiT on the GPU: every linear runs through the
int4 kernels; the forward matches a float twin built from the bit-exact bf16
dequantization of the same packed weights (the W4A16 emulation, nodes.py:43-52)
within the bf16 noise of a multi-block network, and stays finite at the full
benchmark dims."""
import pytest
import torch

from comfy_ui_gfx906_tools_b200 import flux_dit, ops

pytestmark = pytest.mark.gpu


def _float_twin(model, cfg, dev):
    """Same architecture with torch.nn.Linear layers holding dequant(W) in bf16."""
    twin = flux_dit.FluxDiT(cfg, flux_dit.float_linear_factory(dev, torch.bfloat16, seed=9), dev, torch.bfloat16)
    src = dict(model.named_modules())
    with torch.no_grad():
        for name, m in twin.named_modules():
            s = src[name]
            if isinstance(m, torch.nn.Linear):
                assert isinstance(s, ops.Gfx906Int4Ops.Linear)
                if s.quantized:
                    m.weight.copy_(ops.dequantize_int4(s.weight_q4, s.weight_scale, torch.bfloat16))
                else:
                    m.weight.copy_(s.weight)
                if m.bias is not None:
                    m.bias.copy_(s.bias)
            elif isinstance(m, flux_dit.RMSNorm):
                m.scale.copy_(s.scale)
    return twin


def test_dit_int4_matches_dequantized_twin(cuda):
    cfg = flux_dit.tiny_config(hidden=512, heads=4, depth_double=2, depth_single=2, context_dim=256, vec_dim=128)
    model = flux_dit.FluxDiT(cfg, flux_dit.int4_linear_factory(cuda, seed=1), cuda, torch.bfloat16)
    twin = _float_twin(model, cfg, cuda)
    for L_side in (4, 12):  # 16 tokens (small-M kernel) and 144 tokens (tcgen05 kernel)
        inputs = flux_dit.make_inputs(cfg, 2, L_side, L_side, 8, cuda, seed=2)
        with torch.no_grad():
            a = model(*inputs).float()
            b = twin(*inputs).float()
        assert torch.isfinite(a).all()
        rel = ((a - b).norm() / b.norm()).item()
        assert rel < 2e-2, rel


def test_dit_full_dims_forward_finite(cuda):
    # config-4 dims (19 + 38 blocks, hidden 3072), 1024^2 latent: 64 x 64 patches + 512 text tokens
    cfg = flux_dit.DiTConfig()
    model = flux_dit.FluxDiT(cfg, flux_dit.int4_linear_factory(cuda, seed=3), cuda, torch.bfloat16)
    n_int4 = sum(1 for m in model.modules() if isinstance(m, ops.Gfx906Int4Ops.Linear) and m.quantized)
    assert n_int4 == 19 * 10 + 38 * 3 + 10  # per double block 10, per single block 3, embedders + final 10
    inputs = flux_dit.make_inputs(cfg, 1, 64, 64, 512, cuda, seed=4)
    with torch.no_grad():
        out = model(*inputs)
    assert out.shape == (1, 4096, 64) and torch.isfinite(out).all()
    assert out.float().std() > 0
