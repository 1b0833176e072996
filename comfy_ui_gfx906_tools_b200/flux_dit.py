"""A Flux-architecture DiT whose linears are packed int4 (random init), for the
full-forward benchmarks and the multi-GPU split.

Architecture (the published MMDiT layout at the benchmark's dims): hidden 3072,
24 heads x 128, MLP ratio 4, 19 double-stream blocks (separate image / text
weights, joint attention over [text, image]) and 38 single-stream blocks (one
fused qkv+mlp projection, one fused output projection), adaLN modulation from a
timestep / pooled-text vector, RMS-normalised q/k, axial RoPE over (index, row,
column) position ids. Every ``Linear`` is ``Gfx906Int4Ops.Linear`` (int4
group-32 weights, this package's GEMM kernels); attention is PyTorch's SDPA.
Weights are random (no checkpoint): codes uniform over the 16 nibble values
and fp16-exact group scales, the same distribution as the GEMM benchmark.

The module is written for this package (ComfyUI's model code is not a
dependency). ``linear_factory`` lets tests build the same network from plain
``torch.nn.Linear`` layers.
"""
from __future__ import annotations

import dataclasses
import math

import torch
import torch.nn.functional as F

from .ops import Gfx906Int4Ops, int4_linear, int4_linear_w4a4


@dataclasses.dataclass
class DiTConfig:
    hidden: int = 3072
    heads: int = 24
    mlp_ratio: int = 4
    depth_double: int = 19
    depth_single: int = 38
    in_channels: int = 64        # 2x2 patches of a 16-channel latent
    context_dim: int = 4096      # text encoder features
    vec_dim: int = 768           # pooled text vector
    axes_dims: tuple = (16, 56, 56)
    theta: float = 10000.0
    guidance_embed: bool = True

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


def tiny_config(**kw) -> DiTConfig:
    """A small configuration with the same structure (for tests)."""
    base = dict(hidden=256, heads=2, mlp_ratio=4, depth_double=2, depth_single=2, in_channels=64, context_dim=128,
                vec_dim=64, axes_dims=(16, 56, 56), guidance_embed=True)
    base.update(kw)
    return DiTConfig(**base)


# ---------------------------------------------------------------------------
# linear factories
# ---------------------------------------------------------------------------
def int4_linear_factory(device, dtype=torch.bfloat16, seed: int = 0):
    """Builds Gfx906Int4Ops.Linear layers with random packed weights."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)

    def make(in_f: int, out_f: int, bias: bool = True) -> torch.nn.Module:
        lin = Gfx906Int4Ops.Linear(in_f, out_f, bias=bias, device=device, dtype=dtype)
        with torch.no_grad():
            if lin.quantized:
                lin.weight_q4.copy_(torch.randint(-128, 128, lin.weight_q4.shape, generator=gen, device=device,
                                                  dtype=torch.int32).to(torch.int8))
                s = torch.randn(lin.weight_scale.shape, generator=gen, device=device).abs() * 0.02 / 7 + 1e-4
                # fp16-exact scales, 1/sqrt(K)-normalised so activations stay O(1) through 57 blocks
                s = s * (math.sqrt(3072.0 / in_f) / 1.5)
                lin.weight_scale.copy_(s.half().float())
            else:
                lin.weight.normal_(0, 1.0 / math.sqrt(in_f), generator=gen)
            if bias:
                lin.bias.normal_(0, 0.01, generator=gen)
        return lin

    return make


def float_linear_factory(device, dtype=torch.float32, seed: int = 0):
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)

    def make(in_f: int, out_f: int, bias: bool = True) -> torch.nn.Module:
        lin = torch.nn.Linear(in_f, out_f, bias=bias, device=device, dtype=dtype)
        with torch.no_grad():
            lin.weight.normal_(0, 1.0 / math.sqrt(in_f), generator=gen)
            if bias:
                lin.bias.normal_(0, 0.01, generator=gen)
        return lin

    return make


# ---------------------------------------------------------------------------
# building blocks
# ---------------------------------------------------------------------------
def timestep_embedding(t: torch.Tensor, dim: int = 256, max_period: float = 10000.0) -> torch.Tensor:
    """Sinusoidal embedding of (scaled) timesteps: [B] -> [B, dim] (cos | sin)."""
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
    args = t.float()[:, None] * 1000.0 * freqs[None]
    return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)


def rope_tables(ids: torch.Tensor, axes_dims, theta: float) -> torch.Tensor:
    """Axial rotary tables: ids [B, L, n_axes] -> [B, 1, L, head_dim/2, 2] (cos, sin)."""
    parts = []
    for i, d in enumerate(axes_dims):
        freqs = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float64, device=ids.device) / d))
        ang = ids[..., i].double()[..., None] * freqs  # [B, L, d/2]
        parts.append(ang)
    ang = torch.cat(parts, dim=-1).float()
    return torch.stack([torch.cos(ang), torch.sin(ang)], dim=-1).unsqueeze(1)


def apply_rope(x: torch.Tensor, pe: torch.Tensor) -> torch.Tensor:
    """x [B, H, L, D] rotated pairwise (x0, x1) by the angles in pe."""
    xf = x.float().reshape(*x.shape[:-1], -1, 2)
    cos, sin = pe[..., 0], pe[..., 1]
    x0, x1 = xf[..., 0], xf[..., 1]
    out = torch.stack([x0 * cos - x1 * sin, x0 * sin + x1 * cos], dim=-1)
    return out.reshape(x.shape).to(x.dtype)


class RMSNorm(torch.nn.Module):
    def __init__(self, dim: int, device=None, dtype=None):
        super().__init__()
        self.scale = torch.nn.Parameter(torch.ones(dim, device=device, dtype=dtype))

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(x.dtype) * self.scale


def layer_norm(x):
    return F.layer_norm(x.float(), (x.shape[-1],), eps=1e-6).to(x.dtype)


class MLPEmbedder(torch.nn.Module):
    def __init__(self, make, in_dim: int, hidden: int):
        super().__init__()
        self.fc1 = make(in_dim, hidden)
        self.fc2 = make(hidden, hidden)

    def forward(self, x):
        return self.fc2(F.silu(self.fc1(x)))


class Modulation(torch.nn.Module):
    """adaLN: SiLU(vec) -> n chunks of [B, 1, hidden]."""

    def __init__(self, make, hidden: int, n: int):
        super().__init__()
        self.n = n
        self.lin = make(hidden, n * hidden)

    def forward(self, vec):
        return self.lin(F.silu(vec))[:, None, :].chunk(self.n, dim=-1)


class AttentionExchange:
    """How a block's attention sees keys/values. The default is local (all
    tokens on this device). ``parallel.TokenShard`` replaces it to gather the
    image keys/values of every rank.

    ``start(img_k, img_v)`` begins the exchange and ``finish(pending, txt_k,
    txt_v)`` returns the joint keys and values; a block computes independent
    work (the next linear) between the two, so a remote exchange overlaps it.
    ``overlaps`` tells a block whether restructuring its work for that pays."""

    overlaps = False

    def start(self, img_k, img_v):
        return img_k, img_v

    def finish(self, pending, txt_k, txt_v):
        img_k, img_v = pending
        return torch.cat([txt_k, img_k], dim=2), torch.cat([txt_v, img_v], dim=2)

    def joint_kv(self, txt_k, txt_v, img_k, img_v):
        return self.finish(self.start(img_k, img_v), txt_k, txt_v)


def linear_rows(lin, x, r0: int, r1: int):
    """Output features [r0, r1) of ``lin(x)``: the same layer restricted to
    those weight rows (row slices of the packed weight, no copy), so a fused
    linear can be computed in parts."""
    b = lin.bias[r0:r1].to(x.dtype) if lin.bias is not None else None
    if isinstance(lin, Gfx906Int4Ops.Linear) and lin.quantized:
        scale = lin._device_scale(lin.weight_scale)[r0:r1]
        fn = int4_linear_w4a4 if lin.activation_quant else int4_linear
        return fn(x, lin.weight_q4[r0:r1], scale, b, lin.rotation_group)
    return F.linear(x, lin.weight[r0:r1].to(x.dtype), b)


def attention(q, k, v):
    return F.scaled_dot_product_attention(q, k, v)


def _heads(x, heads):
    B, L, _ = x.shape
    return x.view(B, L, heads, -1).transpose(1, 2)


def _merge(x):
    B, H, L, D = x.shape
    return x.transpose(1, 2).reshape(B, L, H * D)


class DoubleBlock(torch.nn.Module):
    def __init__(self, make, cfg: DiTConfig, device=None, dtype=None):
        super().__init__()
        h, mlp = cfg.hidden, cfg.hidden * cfg.mlp_ratio
        self.heads = cfg.heads
        self.img_mod, self.txt_mod = Modulation(make, h, 6), Modulation(make, h, 6)
        self.img_qkv, self.txt_qkv = make(h, 3 * h), make(h, 3 * h)
        self.img_qn, self.img_kn = RMSNorm(cfg.head_dim, device, dtype), RMSNorm(cfg.head_dim, device, dtype)
        self.txt_qn, self.txt_kn = RMSNorm(cfg.head_dim, device, dtype), RMSNorm(cfg.head_dim, device, dtype)
        self.img_proj, self.txt_proj = make(h, h), make(h, h)
        self.img_fc1, self.img_fc2 = make(h, mlp), make(mlp, h)
        self.txt_fc1, self.txt_fc2 = make(h, mlp), make(mlp, h)

    def _qkv(self, x, mod, qkv, qn, kn):
        shift, scale = mod
        y = qkv((1 + scale) * layer_norm(x) + shift)
        q, k, v = y.chunk(3, dim=-1)
        q, k, v = _heads(q, self.heads), _heads(k, self.heads), _heads(v, self.heads)
        return qn(q), kn(k), v

    def forward(self, img, txt, vec, pe_txt, pe_img, ex: AttentionExchange):
        im = self.img_mod(vec)
        tm = self.txt_mod(vec)
        iq, ik, iv = self._qkv(img, im[0:2], self.img_qkv, self.img_qn, self.img_kn)
        iq, ik = apply_rope(iq, pe_img), apply_rope(ik, pe_img)
        pending = ex.start(ik, iv)  # the image K/V exchange runs while the text stream's linear computes
        tq, tk, tv = self._qkv(txt, tm[0:2], self.txt_qkv, self.txt_qn, self.txt_kn)
        tq, tk = apply_rope(tq, pe_txt), apply_rope(tk, pe_txt)
        k, v = ex.finish(pending, tk, tv)
        o = attention(torch.cat([tq, iq], dim=2), k, v)
        Lt = txt.shape[1]
        t_o, i_o = _merge(o[:, :, :Lt]), _merge(o[:, :, Lt:])
        img = img + im[2] * self.img_proj(i_o)
        img = img + im[5] * self.img_fc2(F.gelu(self.img_fc1((1 + im[4]) * layer_norm(img) + im[3]),
                                                approximate="tanh"))
        txt = txt + tm[2] * self.txt_proj(t_o)
        txt = txt + tm[5] * self.txt_fc2(F.gelu(self.txt_fc1((1 + tm[4]) * layer_norm(txt) + tm[3]),
                                                approximate="tanh"))
        return img, txt


class SingleBlock(torch.nn.Module):
    def __init__(self, make, cfg: DiTConfig, device=None, dtype=None):
        super().__init__()
        h = cfg.hidden
        self.mlp = h * cfg.mlp_ratio
        self.heads = cfg.heads
        self.mod = Modulation(make, h, 3)
        self.lin1 = make(h, 3 * h + self.mlp)
        self.lin2 = make(h + self.mlp, h)
        self.qn, self.kn = RMSNorm(cfg.head_dim, device, dtype), RMSNorm(cfg.head_dim, device, dtype)

    def forward(self, x, vec, Lt, pe_txt, pe_img, ex: AttentionExchange):
        shift, scale, gate = self.mod(vec)
        xin = (1 + scale) * layer_norm(x) + shift
        h = x.shape[-1]
        if ex.overlaps:
            # the fused linear in two parts: the q/k/v rows, then (while the
            # image K/V exchange runs) the MLP rows
            qkv, mlp = linear_rows(self.lin1, xin, 0, 3 * h), None
        else:
            y = self.lin1(xin)
            qkv, mlp = y[..., : 3 * h], y[..., 3 * h:]
        q, k, v = qkv.chunk(3, dim=-1)
        q, k, v = _heads(q, self.heads), _heads(k, self.heads), _heads(v, self.heads)
        q, k = self.qn(q), self.kn(k)
        pe = torch.cat([pe_txt, pe_img], dim=2)
        q, k = apply_rope(q, pe), apply_rope(k, pe)
        pending = ex.start(k[:, :, Lt:], v[:, :, Lt:])
        if mlp is None:
            mlp = linear_rows(self.lin1, xin, 3 * h, 3 * h + self.mlp)
        kk, vv = ex.finish(pending, k[:, :, :Lt], v[:, :, :Lt])
        o = _merge(attention(q, kk, vv))
        return x + gate * self.lin2(torch.cat([o, F.gelu(mlp, approximate="tanh")], dim=-1))


class FluxDiT(torch.nn.Module):
    def __init__(self, cfg: DiTConfig, make, device=None, dtype=torch.bfloat16):
        super().__init__()
        self.cfg = cfg
        h = cfg.hidden
        self.img_in = make(cfg.in_channels, h)
        self.txt_in = make(cfg.context_dim, h)
        self.time_in = MLPEmbedder(make, 256, h)
        self.vector_in = MLPEmbedder(make, cfg.vec_dim, h)
        self.guidance_in = MLPEmbedder(make, 256, h) if cfg.guidance_embed else None
        self.double_blocks = torch.nn.ModuleList([DoubleBlock(make, cfg, device, dtype)
                                                  for _ in range(cfg.depth_double)])
        self.single_blocks = torch.nn.ModuleList([SingleBlock(make, cfg, device, dtype)
                                                  for _ in range(cfg.depth_single)])
        self.final_mod = Modulation(make, h, 2)
        self.final_out = make(h, cfg.in_channels)
        self.exchange = AttentionExchange()

    def forward(self, img, img_ids, txt, txt_ids, timesteps, y, guidance=None):
        """img [B, L_img, in_channels], img_ids [B, L_img, 3], txt [B, L_txt, context_dim],
        txt_ids [B, L_txt, 3], timesteps [B], y [B, vec_dim] -> [B, L_img, in_channels]."""
        dtype = img.dtype
        x = self.img_in(img)
        t = self.txt_in(txt)
        vec = self.time_in(timestep_embedding(timesteps).to(dtype))
        if self.guidance_in is not None:
            g = guidance if guidance is not None else torch.full_like(timesteps, 3.5)
            vec = vec + self.guidance_in(timestep_embedding(g).to(dtype))
        vec = vec + self.vector_in(y.to(dtype))
        pe_img = rope_tables(img_ids, self.cfg.axes_dims, self.cfg.theta)
        pe_txt = rope_tables(txt_ids, self.cfg.axes_dims, self.cfg.theta)
        for blk in self.double_blocks:
            x, t = blk(x, t, vec, pe_txt, pe_img, self.exchange)
        Lt = t.shape[1]
        xt = torch.cat([t, x], dim=1)
        for blk in self.single_blocks:
            xt = blk(xt, vec, Lt, pe_txt, pe_img, self.exchange)
        x = xt[:, Lt:]
        shift, scale = self.final_mod(vec)
        return self.final_out((1 + scale) * layer_norm(x) + shift)


def make_inputs(cfg: DiTConfig, batch: int, h_tokens: int, w_tokens: int, txt_len: int, device, dtype=torch.bfloat16,
                seed: int = 0):
    """Synthetic inputs: a [batch, h*w, in_channels] patch sequence with its
    (0, row, col) ids, text features with zero ids, timesteps and pooled vector."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    L = h_tokens * w_tokens
    img = torch.randn(batch, L, cfg.in_channels, generator=g).to(device, dtype)
    rows = torch.arange(h_tokens).repeat_interleave(w_tokens)
    cols = torch.arange(w_tokens).repeat(h_tokens)
    img_ids = torch.stack([torch.zeros(L), rows.float(), cols.float()], dim=-1)[None].repeat(batch, 1, 1).to(device)
    txt = torch.randn(batch, txt_len, cfg.context_dim, generator=g).to(device, dtype)
    txt_ids = torch.zeros(batch, txt_len, 3, device=device)
    t = torch.rand(batch, generator=g).to(device)
    y = torch.randn(batch, cfg.vec_dim, generator=g).to(device, dtype)
    return img, img_ids, txt, txt_ids, t, y
