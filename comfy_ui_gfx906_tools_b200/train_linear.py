"""Linear layer with an int4 backward (the reference's train_linear.py, on B200).

Reference: nodes/ComfyUI-Gfx906Int4/train_linear.py:1-113. Same API and the
same numerics, bit for bit, because every step runs the reference's
arithmetic: the block-16 quantizers (``ops.quantize_int4_rows`` /
``ops.quantize_int4_cols``, int4_train_quant.hip) and the integer-exact
block-16 GEMM (``ops.gemm_int4(..., qblock=16)``, int4_gemm_scaled.hip with
SUB = 2; here on the tensor cores, csrc/w4a4_exact.cu).

  forward  y = x W^T in the input dtype (F.linear), or with ``int4_fprop`` x
           and W quantized to int4 along K (round to nearest) and multiplied
           by the int4 GEMM (train_linear.py:37-45).
  dgrad    dX = dY W: dY quantized along N with stochastic rounding, W^T
           quantized along N (train_linear.py:58-61).
  wgrad    dW = dY^T X: both quantized along the tokens after a 16-point
           random Hadamard rotation with one fixed sign vector, dY with
           stochastic rounding; fp32 GEMM output cast to W's dtype
           (train_linear.py:62-66).

Stochastic-rounding seeds come from a process-wide counter that every
stochastic quantize call advances by one (train_linear.py:26-28), so a
sequence of calls reproduces the reference's sequence of seeds.
"""
from __future__ import annotations

import threading

import torch
import torch.nn.functional as F

from . import ops

_SIGNS: dict = {}
_seed_lock = threading.Lock()
_seed = [0]


def _signs(device) -> torch.Tensor:
    """The fixed +-1 vector of the wgrad rotation: a CPU generator seeded 1234,
    sign -1 where a uniform draw is < 0.5 (train_linear.py:19-23)."""
    key = str(device)
    if key not in _SIGNS:
        g = torch.Generator().manual_seed(1234)
        _SIGNS[key] = torch.where(torch.rand(16, generator=g) < 0.5, -1.0, 1.0).to(device)
    return _SIGNS[key]


def _next_seed() -> int:
    with _seed_lock:
        _seed[0] = (_seed[0] + 1) & 0x7FFFFFFF
        return _seed[0]


def _fprop_packed(x: torch.Tensor, wq: torch.Tensor, wsc: torch.Tensor) -> torch.Tensor:
    """y = x W^T with x quantized here (block 16 along K, round to nearest) and W packed."""
    xq, xsc = ops.quantize_int4_rows(x.reshape(-1, x.shape[-1]).contiguous(), False, 0)
    return ops.gemm_int4(xq, xsc, wq, wsc, None, x.dtype, 0, 16).view(*x.shape[:-1], -1)


def _int4_fprop(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return _fprop_packed(x, *ops.quantize_int4_rows(w.contiguous(), False, 0))


class _Int4BwdLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, int4_fprop):
        ctx.save_for_backward(x, w)
        return _int4_fprop(x, w) if int4_fprop else F.linear(x, w)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        g = dy.reshape(-1, dy.shape[-1]).contiguous()
        dx = dw = None
        if ctx.needs_input_grad[0]:
            gq, gs = ops.quantize_int4_rows(g, True, _next_seed())
            wq, ws = ops.quantize_int4_cols(w, None, False, 0)  # W [N, K] -> W^T blocked along N
            dx = ops.gemm_int4(gq, gs, wq, ws, None, dy.dtype, 0, 16).view(*dy.shape[:-1], -1)
        if ctx.needs_input_grad[1]:
            signs = _signs(dy.device)
            xs = x.reshape(-1, x.shape[-1])
            gtq, gts = ops.quantize_int4_cols(g, signs, True, _next_seed())
            xtq, xts = ops.quantize_int4_cols(xs if xs.stride(-1) == 1 else xs.contiguous(), signs, False, 0)
            dw = ops.gemm_int4(gtq, gts, xtq, xts, None, torch.float32, 0, 16).to(w.dtype)
        return dx, dw, None


def linear(x: torch.Tensor, w: torch.Tensor, int4_fprop: bool = False) -> torch.Tensor:
    """F.linear(x, w) with the int4 backward; ``int4_fprop`` also quantizes the
    forward. fp16 operands; the token count (x's leading dims) must be a
    multiple of 32 (train_linear.py:69-74)."""
    return _Int4BwdLinear.apply(x, w, int4_fprop)


class _FrozenInt4(torch.autograd.Function):
    """Keeps nothing per call: no wgrad, and the dgrad uses the stored W^T."""

    @staticmethod
    def forward(ctx, x, wq, wsc, wtq, wtsc):
        ctx.wt = (wtq, wtsc)
        return _fprop_packed(x, wq, wsc)

    @staticmethod
    def backward(ctx, dy):
        gq, gs = ops.quantize_int4_rows(dy.reshape(-1, dy.shape[-1]).contiguous(), True, _next_seed())
        dx = ops.gemm_int4(gq, gs, *ctx.wt, None, dy.dtype, 0, 16).view(*dy.shape[:-1], -1)
        return dx, None, None, None, None


class FrozenInt4Linear(torch.nn.Module):
    """A frozen bias-free linear stored only as int4 (train_linear.py:89-113): W
    blocked along K for the forward and W^T blocked along N for the dgrad, both
    quantized once; equal to ``linear(x, w, int4_fprop=True)`` with w frozen."""

    def __init__(self, linear):
        super().__init__()
        w = linear.weight
        if linear.bias is not None or w.dtype != torch.float16 or w.shape[0] % 32 or w.shape[1] % 32:
            raise ValueError(f"FrozenInt4Linear: expected a bias-free fp16 weight with both dims % 32 == 0, got "
                             f"bias={linear.bias is not None} dtype={w.dtype} shape={tuple(w.shape)}")
        w = w.detach().contiguous()
        for name, t in zip(("wq", "wsc", "wtq", "wtsc"),
                           (*ops.quantize_int4_rows(w, False, 0), *ops.quantize_int4_cols(w, None, False, 0))):
            self.register_buffer(name, t)
        self.in_features, self.out_features = w.shape[1], w.shape[0]

    def forward(self, x):
        return _FrozenInt4.apply(x, self.wq, self.wsc, self.wtq, self.wtsc)
