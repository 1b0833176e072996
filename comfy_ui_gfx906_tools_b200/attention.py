"""Fused quantized attention on B200 (the reference's attention.py, csrc/attention.hip).

Reference: nodes/ComfyUI-Gfx906Int4/attention.py:1-160 (prepare step, entry
point, ComfyUI node) and csrc/attention.hip (the kernel; here
csrc/attention.cu behind the C ABI ``attention``).

The prepare step is O(L * D) tensor work around the O(L^2) kernel and keeps
the reference's arithmetic operation for operation (attention.py:31-81), so
its outputs are bit-identical to the reference's on the same device:
  * the softmax scale times log2(e) goes into Q (fp16 mode) or Q's scale (int
    modes), so the kernel's softmax runs on exp2;
  * int modes: K minus its mean over the tokens of each KV head (every score
    of a query row moves by one constant, so softmax is unchanged), then
    per-token symmetric quantization to int8 or int4 (amax / qmax);
  * int4: the head dimension is first rotated by the orthonormal 128-point
    Hadamard matrix (q . k unchanged, outliers spread);
  * V cut into 64-key tiles, transposed to [tile, channel, key]; u8 mode
    quantizes per (tile, channel) to [-127, 127] and stores value + 128.
"""
from __future__ import annotations

import logging

import torch

from . import _lib, ops

HEAD_DIM = 128
TILE = 64
QK_MODES = {"fp16": 0, "int8": 1, "int4": 2}
PV_MODES = {"fp16": 0, "u8": 1}
_LOG2E = 1.4426950408889634
# Shorter key sequences go to the host framework's own attention: the prepare
# step then costs more than the kernel saves (attention.py:23-27).
MIN_FUSED_TOKENS = 768


def _quant_per_token(x: torch.Tensor, bits: int):
    """Symmetric per-token (last dim) quantization -> (int8 codes, fp32 scale);
    attention.py:31-35."""
    qmax = 2 ** (bits - 1) - 1
    scale = x.abs().amax(-1).clamp_min(1e-8) / qmax
    codes = (x / scale[..., None]).round().clamp(-qmax - 1, qmax).to(torch.int8)
    return codes, scale


def _pack_nibbles(x: torch.Tensor) -> torch.Tensor:
    """int8 codes in [-8, 7], even last dim -> uint8, element 2i in the low
    nibble of byte i; attention.py:38-41."""
    pairs = x.reshape(*x.shape[:-1], x.shape[-1] // 2, 2).to(torch.int16)
    return ((pairs[..., 0] & 0xF) | ((pairs[..., 1] & 0xF) << 4)).to(torch.uint8)


def prepare_qk(q: torch.Tensor, k: torch.Tensor, mode: str):
    """(Q bytes, q_scale, K bytes, k_scale) for the kernel; attention.py:44-61."""
    sm_scale = HEAD_DIM ** -0.5 * _LOG2E
    none = torch.empty(0, device=q.device)
    if mode == "fp16":
        qh = (q.float() * sm_scale).half().contiguous()
        return qh.view(torch.uint8), none, k.half().contiguous().view(torch.uint8), none
    qf = q.float()
    kf = k.float()
    kf = kf - kf.mean(dim=2, keepdim=True)
    if mode == "int4":
        h = ops._hadamard(HEAD_DIM, q.device)
        qf = qf @ h
        kf = kf @ h
    bits = 8 if mode == "int8" else 4
    qc, qs = _quant_per_token(qf, bits)
    kc, ks = _quant_per_token(kf, bits)
    if mode == "int4":
        return _pack_nibbles(qc), qs * sm_scale, _pack_nibbles(kc), ks
    return qc.view(torch.uint8), qs * sm_scale, kc.view(torch.uint8), ks


def prepare_v(v: torch.Tensor, mode: str):
    """(Vt bytes [B, KVH, tiles, 128, 64 * vbytes], v_scale); attention.py:64-75."""
    B, KVH, L, D = v.shape
    tiles = -(-L // TILE)
    vt = torch.nn.functional.pad(v, (0, 0, 0, tiles * TILE - L)).reshape(B, KVH, tiles, TILE, D).transpose(-1, -2)
    if mode == "fp16":
        return vt.half().contiguous().view(torch.uint8), torch.empty(0, device=v.device)
    vf = vt.float()
    scale = vf.abs().amax(-1).clamp_min(1e-8) / 127
    codes = (vf / scale[..., None]).round().clamp(-127, 127) + 128
    return codes.to(torch.uint8).contiguous(), scale.contiguous()


def block_rows(qk: str) -> int:
    """Query rows per kernel block = rows per keep-mask block (attention.py:87-89)."""
    return _lib.load().attention_block_rows(QK_MODES[qk])


def max_tiles() -> int:
    return _lib.load().attention_max_tiles()


def attention_prepared(qb, qs, kb, ks, vt, vs, qk: str, pv: str, skip_below: float = 0.0,
                       keep=None) -> torch.Tensor:
    """The kernel on prepared inputs (the binding's ``attention``,
    binding.cpp:114-170): Q [B, H, Lq, qrow] / K [B, KVH, Lk, qrow] uint8,
    scales fp32, Vt [B, KVH, tiles, 128, 64 * vbytes] uint8 -> fp16 [B, Lq, H * 128]."""
    if qk not in QK_MODES or pv not in PV_MODES:
        raise ValueError(f"qk in {list(QK_MODES)}, pv in {list(PV_MODES)}; got qk={qk!r} pv={pv!r}")
    qrow = {"fp16": 256, "int8": 128, "int4": 64}[qk]
    vbytes = 2 if pv == "fp16" else 1
    for t, name in ((qb, "Q"), (kb, "K"), (vt, "Vt")):
        ops._require_cuda(t, name)
        if t.dtype != torch.uint8:
            raise RuntimeError(f"{name} must be uint8, got {t.dtype}")
    if qb.dim() != 4 or qb.shape[3] != qrow:
        raise RuntimeError(f"Q must be uint8 [B, H, L, {qrow}], got {tuple(qb.shape)}")
    B, H, Lq, _ = qb.shape
    if kb.dim() != 4 or kb.shape[0] != B or kb.shape[3] != qrow:
        raise RuntimeError(f"K must be uint8 [{B}, KVH, Lk, {qrow}], got {tuple(kb.shape)}")
    KVH, Lk = kb.shape[1], kb.shape[2]
    if KVH <= 0 or H % KVH:
        raise RuntimeError(f"H ({H}) must be a multiple of KVH ({KVH})")
    n_tiles = -(-Lk // TILE)
    if tuple(vt.shape) != (B, KVH, n_tiles, HEAD_DIM, TILE * vbytes):
        raise RuntimeError(f"Vt must be uint8 [{B}, {KVH}, {n_tiles}, 128, {TILE * vbytes}], got {tuple(vt.shape)}")
    if qk != "fp16" and (qs.numel() != B * H * Lq or ks.numel() != B * KVH * Lk):
        raise RuntimeError(f"q_scale/k_scale must have {B * H * Lq}/{B * KVH * Lk} elements, got "
                           f"{qs.numel()}/{ks.numel()}")
    if pv == "u8" and vs.numel() != B * KVH * n_tiles * HEAD_DIM:
        raise RuntimeError(f"v_scale must have {B * KVH * n_tiles * HEAD_DIM} elements, got {vs.numel()}")
    keep_c = None
    if keep is not None:
        rows = block_rows(qk)
        n_qb = -(-Lq // rows)
        if keep.dtype != torch.uint8 or tuple(keep.shape) != (B, H, n_qb, n_tiles):
            raise RuntimeError(f"keep must be uint8 [{B}, {H}, {n_qb}, {n_tiles}], got {keep.dtype} "
                               f"{tuple(keep.shape)}")
        if n_tiles > max_tiles():
            raise RuntimeError(f"keep supports at most {max_tiles()} key tiles, got {n_tiles}")
        keep_c = keep.contiguous()
    qb, kb, vt = qb.contiguous(), kb.contiguous(), vt.contiguous()
    qs = qs.to(torch.float32).contiguous()
    ks = ks.to(torch.float32).contiguous()
    vs = vs.to(torch.float32).contiguous()
    out = torch.empty(B, Lq, H * HEAD_DIM, dtype=torch.float16, device=qb.device)
    with torch.cuda.device(qb.device):
        _lib.call("attention", QK_MODES[qk], PV_MODES[pv], qb.data_ptr(), qs.data_ptr() if qs.numel() else None,
                  kb.data_ptr(), ks.data_ptr() if ks.numel() else None, vt.data_ptr(),
                  vs.data_ptr() if vs.numel() else None, keep_c.data_ptr() if keep_c is not None else None,
                  out.data_ptr(), B, H, KVH, Lq, Lk, float(skip_below), ops._stream(qb.device))
    return out


def fused_attention(q, k, v, qk: str = "int8", pv: str = "u8", skip_below: float = 0.0, keep=None) -> torch.Tensor:
    """softmax(q k^T / sqrt(128)) v; q [B, H, Lq, 128] post-RoPE, k / v
    [B, KVH, Lk, 128] (not GQA-expanded; Lq != Lk for the row split). keep:
    optional block-sparse mask, uint8 [B, H, ceil(Lq / block_rows(qk)),
    ceil(Lk / 64)]. Returns [B, Lq, H * 128] fp16 (attention.py:78-84)."""
    if q.shape[-1] != HEAD_DIM:
        raise ValueError(f"head dim must be {HEAD_DIM}, got {q.shape[-1]}")
    if qk not in QK_MODES or pv not in PV_MODES:
        raise ValueError(f"qk in {list(QK_MODES)}, pv in {list(PV_MODES)}; got qk={qk!r} pv={pv!r}")
    qb, qs, kb, ks = prepare_qk(q, k, qk)
    vt, vs = prepare_v(v, pv)
    return attention_prepared(qb, qs, kb, ks, vt, vs, qk, pv, skip_below, keep)


def _gqa_repeat(diffusion_model) -> int:
    """Query heads per KV head of the model's attention modules (1 when it has
    none): the override reads each KV head once instead of the expanded copy
    (attention.py:92-98)."""
    mod = next((m for m in diffusion_model.modules() if hasattr(m, "kvheads") and hasattr(m, "heads")), None)
    return mod.heads // mod.kvheads if mod is not None else 1


def make_override(qk: str, pv: str, skip_below: float, gqa_repeat: int = 1, sparsity=None):
    """ComfyUI ``optimized_attention_override``: unmasked head-dim-128 calls
    with at least MIN_FUSED_TOKENS keys run the fused kernel, everything else
    goes to ComfyUI's own backend (attention.py:101-132). ``sparsity`` (a
    block_sparse.SparsityState) supplies keep masks while the key tiles fit the
    kernel's mask limit."""

    def override(func, q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False,
                 skip_output_reshape=False, **kwargs):
        handled = (mask is None and skip_reshape and not skip_output_reshape and "scale" not in kwargs
                   and q.dim() == 4 and q.shape[1] == heads and q.shape[-1] == HEAD_DIM
                   and k.shape[2] >= MIN_FUSED_TOKENS)
        if not handled:
            return func(q, k, v, heads, mask=mask, attn_precision=attn_precision, skip_reshape=skip_reshape,
                        skip_output_reshape=skip_output_reshape, **kwargs)
        if gqa_repeat > 1 and k.shape[1] == q.shape[1]:
            k, v = k[:, ::gqa_repeat], v[:, ::gqa_repeat]
        keep = None
        if sparsity is not None and -(-k.shape[2] // TILE) <= max_tiles():
            keep = sparsity.keep(q, k, kwargs.get("transformer_options") or {})
        return fused_attention(q, k, v, qk, pv, skip_below, keep).to(q.dtype)

    return override


class Gfx906FusedAttention:
    """MODEL -> MODEL: routes the model's attention through the fused kernel
    (head dim 128, unmasked); other attention calls fall through to ComfyUI's
    backend (attention.py:135-160). sparse_tau > 0 runs block-sparse with
    masks predicted per call and heads calibrated on the first call of each
    sampling run (block_sparse.SparsityState); the reference's persistent
    calibration cache is not built, so calibration="persistent" also
    calibrates per run."""

    @classmethod
    def INPUT_TYPES(cls):
        return {
            "required": {
                "model": ("MODEL",),
                "qk": (list(QK_MODES), {"default": "int4"}),
                "pv": (list(PV_MODES), {"default": "u8"}),
                "skip_below": ("FLOAT", {"default": 1e-4, "min": 0.0, "max": 0.1, "step": 1e-5}),
                "sparse_tau": ("FLOAT", {"default": 0.0, "min": 0.0, "max": 0.999, "step": 0.001}),
                "max_missed": ("FLOAT", {"default": 0.02, "min": 0.0, "max": 0.2, "step": 0.005}),
                "calibration": (["persistent", "per_run"], {"default": "persistent"}),
            }
        }

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "patch"
    CATEGORY = "gfx906"
    TITLE = "Gfx906 Fused Attention"

    def patch(self, model, qk, pv, skip_below, sparse_tau=0.0, max_missed=0.02, calibration="persistent"):
        from . import block_sparse
        diffusion_model = model.model.diffusion_model
        sparsity = None
        if sparse_tau > 0:
            if calibration == "persistent":
                logging.warning("[Gfx906 Attention] the persistent calibration cache is not built here; "
                                "calibrating on the first step of every run")
            sparsity = block_sparse.SparsityState(sparse_tau, max_missed, block_rows(qk))
        model = model.clone()
        model.model_options.setdefault("transformer_options", {})["optimized_attention_override"] = make_override(
            qk, pv, skip_below, _gqa_repeat(diffusion_model), sparsity)
        return (model,)
