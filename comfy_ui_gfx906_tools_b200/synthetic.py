"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no dataset is involved anywhere in this path).

int4 weights (configs 1-2): offset-8 codes u ~ U{0..15} and one fp16 scale per
32-group along K, d = fp16(|N(0, 0.02)| / 7 + 1e-4), serialised as ggml Q4_0
blocks -- the ingest format ``repack_q4_0_native`` reads (ops.py:129-164).
int8 weights (config 3): q = clamp(round(N(0, 40)), -127, 127) with one fp16
scale per output channel, d = fp16(|N(0, 0.02)| / 40 + 1e-5).
Activations: bf16 ~ N(0, 1).
Everything is generated on the CPU from ``torch.Generator().manual_seed(seed)``.
"""
from __future__ import annotations

import torch

BLOCK = 32

# Flux DiT linear shapes at hidden 3072: (name, K, N)
FLUX_SHAPES = [
    ("qkv", 3072, 9216),
    ("proj", 3072, 3072),
    ("mlp_up", 3072, 12288),
    ("mlp_down", 12288, 3072),
    ("single_fused", 3072, 21504),
    ("single_out", 15360, 3072),
]


def q4_0_weight(N: int, K: int, seed: int):
    """Returns (raw Q4_0 bytes uint8 [N*K/32*18], u uint8 [N, K], d fp16 [N, K/32]) on CPU."""
    g = torch.Generator().manual_seed(seed)
    u = torch.randint(0, 16, (N, K), generator=g, dtype=torch.uint8)
    d = (torch.randn(N, K // BLOCK, generator=g).abs() * 0.02 / 7 + 1e-4).to(torch.float16)
    nb = N * K // BLOCK
    ub = u.reshape(nb, BLOCK)
    blocks = torch.empty(nb, 18, dtype=torch.uint8)
    blocks[:, :2] = d.reshape(nb, 1).view(torch.uint8).reshape(nb, 2)
    blocks[:, 2:] = (ub[:, :16] & 0xF) | ((ub[:, 16:] & 0xF) << 4)
    return blocks.reshape(-1), u, d


def activations(M: int, K: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(M, K, generator=g).to(torch.bfloat16)


def int8_weight(N: int, K: int, seed: int):
    """Returns (q int8 [N, K], per-channel scale fp16 [N]) on CPU."""
    g = torch.Generator().manual_seed(seed)
    q = torch.clamp(torch.round(torch.randn(N, K, generator=g) * 40), -127, 127).to(torch.int8)
    s = (torch.randn(N, generator=g).abs() * 0.02 / 40 + 1e-5).to(torch.float16)
    return q, s


def float_weight(N: int, K: int, seed: int, std: float = 0.02) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(N, K, generator=g) * std
