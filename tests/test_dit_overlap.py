"""The DiT blocks' overlap path on one device: an exchange that reports
``overlaps = True`` makes a single block compute its fused linear in two row
parts (q/k/v rows, then the MLP rows while the K/V exchange would run) and a
double block compute the text stream's q/k/v between start and finish. With a
local exchange the result must match the plain forward. ``linear_rows`` on an
int4 layer must equal the matching columns of the full layer (the tensor-core
kernel computes every output element the same way whatever the row range)."""
import pytest
import torch

from comfy_ui_gfx906_tools_b200 import flux_dit


class LocalOverlap(flux_dit.AttentionExchange):
    overlaps = True


def _forward_both(model, inputs):
    with torch.no_grad():
        ref = model(*inputs).float()
        saved = model.exchange
        model.exchange = LocalOverlap()
        try:
            got = model(*inputs).float()
        finally:
            model.exchange = saved
    return got, ref


def test_overlap_path_matches_plain_forward_cpu():
    cfg = flux_dit.tiny_config(depth_double=2, depth_single=2)
    model = flux_dit.FluxDiT(cfg, flux_dit.float_linear_factory("cpu", torch.float32, seed=5), "cpu", torch.float32)
    inputs = flux_dit.make_inputs(cfg, 2, 4, 6, 5, "cpu", torch.float32, seed=6)
    got, ref = _forward_both(model, inputs)
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.gpu
def test_overlap_path_matches_plain_forward_int4(cuda):
    cfg = flux_dit.tiny_config(depth_double=2, depth_single=2)
    model = flux_dit.FluxDiT(cfg, flux_dit.int4_linear_factory(cuda, seed=7), cuda)
    inputs = flux_dit.make_inputs(cfg, 2, 4, 6, 5, cuda, seed=8)
    got, ref = _forward_both(model, inputs)
    assert float((got - ref).abs().max() / ref.abs().max()) < 2e-2


@pytest.mark.gpu
@pytest.mark.parametrize("M", [5, 300])
def test_linear_rows_int4_equals_full_columns(cuda, M):
    make = flux_dit.int4_linear_factory(cuda, seed=9)
    lin = make(256, 640 + 384)
    x = torch.randn(M, 256, generator=torch.Generator().manual_seed(M)).to(cuda, torch.bfloat16)
    with torch.no_grad():
        full = lin(x)
        a = flux_dit.linear_rows(lin, x, 0, 640)
        b = flux_dit.linear_rows(lin, x, 640, 1024)
    if M > 64:  # tensor-core kernel: each element computed identically
        assert torch.equal(torch.cat([a, b], dim=-1), full)
    else:  # small-M kernel: the split-K plan follows N, so only the summation order differs
        torch.testing.assert_close(torch.cat([a, b], dim=-1).float(), full.float(), rtol=1e-2, atol=1e-2)
