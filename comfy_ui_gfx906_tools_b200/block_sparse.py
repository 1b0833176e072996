"""Block-sparse keep masks for the fused attention kernel: predicted per call,
calibrated per (layer, head) on the first call of a sampling run.

Reference: nodes/ComfyUI-Gfx906Int4/block_sparse.py:1-235 (``predict_keep``,
``missed_mass``, ``SparsityState``). The prediction pools q over each kernel
query block and k over each 64-key tile, takes softmax(pooled q . pooled k /
sqrt(128) + log(keys in the tile)) and keeps the largest tiles of each block
until tau of that pooled mass (the tile crossing tau included, so every block
keeps one); blocks or tiles whose tokens are dissimilar (mean cosine to their
mean below SIMILARITY) keep everything. Calibration: the first call per
(layer, device, shape) of a run is dense and measures, on sampled query
blocks, the exact attention mass the prediction would drop per head; heads
above max_missed stay dense for the rest of the run; a rising sigma starts a
new run. The arithmetic is the reference's torch sequence (the masks must
agree bit for bit with the reference's on the same inputs: tests/golden).

Not built: the persistent calibration cache (CalibrationCache,
CachedSparsityState, block_sparse.py:93-318), a JSON file in ComfyUI's user
directory; ``calibration="persistent"`` calibrates per run instead.
"""
from __future__ import annotations

import logging
import threading

import torch

TILE = 64
SIMILARITY = 0.5
CALIBRATION_BLOCKS = 8          # query blocks sampled per calibration call (block_sparse.py:27-30)
CALIBRATION_CHUNK = 2 ** 26     # fp32 score elements per chunk of heads (block_sparse.py:31-34)


def block_means(x: torch.Tensor, block: int):
    """x [B, H, L, D] -> (fp32 means over each block's valid rows [B, H, n, D],
    mean cosine of each row to its block mean [B, H, n] (padding rows count as
    0), valid rows per block [n]); block_sparse.py:37-49."""
    B, H, L, D = x.shape
    n = -(-L // block)
    blocks = torch.nn.functional.pad(x, (0, 0, 0, n * block - L)).reshape(B, H, n, block, D)
    counts = torch.full((n,), block, device=x.device, dtype=torch.float32)
    counts[-1] = L - (n - 1) * block
    means = blocks.sum(3, dtype=torch.float32) / counts[:, None]
    dots = torch.einsum("bhnrd,bhnd->bhnr", blocks, means.to(x.dtype)).float()
    norms = (torch.linalg.vector_norm(blocks, dim=-1, dtype=torch.float32)
             * torch.linalg.vector_norm(means, dim=-1)[..., None])
    cosine = (dots / norms.clamp_min(1e-30)).sum(-1) / block
    return means, cosine, counts


def top_cdf(mass: torch.Tensor, tau: float) -> torch.Tensor:
    """bool keep [..., n]: the largest entries of each row until tau of its mass,
    the entry that crosses tau included; block_sparse.py:52-57."""
    ordered, order = mass.sort(-1, descending=True)
    mass_before = (ordered.cumsum(-1) - ordered) / ordered.sum(-1, keepdim=True)
    return torch.zeros_like(mass_before, dtype=torch.bool).scatter(-1, order, mass_before < tau)


def predict_keep(q: torch.Tensor, k: torch.Tensor, tau: float, rows: int) -> torch.Tensor:
    """q [B, H, Lq, 128], k [B, KVH, Lk, 128] -> bool keep [B, H, ceil(Lq / rows),
    ceil(Lk / 64)]; block_sparse.py:60-69."""
    rep = q.shape[1] // k.shape[1]
    q_mean, q_cos, _ = block_means(q, rows)
    k_mean, k_cos, k_counts = block_means(k, TILE)
    k_mean = k_mean.repeat_interleave(rep, 1)
    k_cos = k_cos.repeat_interleave(rep, 1)
    pooled = q_mean @ k_mean.transpose(-1, -2) * q.shape[-1] ** -0.5 + k_counts.log()
    keep = top_cdf(torch.softmax(pooled, -1), tau)
    return keep | (q_cos < SIMILARITY)[..., None] | (k_cos < SIMILARITY)[:, :, None, :]


def missed_mass(q: torch.Tensor, k: torch.Tensor, keep: torch.Tensor, rows: int) -> torch.Tensor:
    """Per head, the exact attention mass `keep` drops, averaged over up to
    CALIBRATION_BLOCKS evenly spaced query blocks of batch 0 -> [H] fp32;
    block_sparse.py:72-90."""
    H, Lq, D = q.shape[1:]
    Lk = k.shape[2]
    rep = H // k.shape[1]
    n_qb, n_kt = keep.shape[2], keep.shape[3]
    sampled = torch.linspace(0, n_qb - 1, min(CALIBRATION_BLOCKS, n_qb), device=q.device).round().long().unique()
    row_ids = (sampled[:, None] * rows + torch.arange(rows, device=q.device)).clamp_max(Lq - 1).flatten()
    q_rows = q[0, :, row_ids]
    dropped = ~keep[0][:, sampled]  # [H, sampled blocks, n_kt]
    out = torch.empty(H, device=q.device)
    heads_per_chunk = max(1, CALIBRATION_CHUNK // (row_ids.numel() * Lk))
    for h0 in range(0, H, heads_per_chunk):
        heads = torch.arange(h0, min(h0 + heads_per_chunk, H), device=q.device)
        p = torch.softmax(q_rows[heads].float() @ k[0, heads // rep].float().transpose(-1, -2) * D ** -0.5, -1)
        p = torch.nn.functional.pad(p, (0, n_kt * TILE - Lk)).reshape(len(heads), len(sampled), rows, n_kt, TILE)
        tile_mass = p.sum(4).mean(2)
        out[heads] = (tile_mass * dropped[heads]).sum(-1).mean(-1)
    return out


class SparsityState:
    """Which heads of each (layer, device, shape) may run sparse in the current
    sampling run (block_sparse.py:193-235); one per patched model."""

    def __init__(self, tau: float, max_missed: float, rows: int):
        self.tau, self.max_missed, self.rows = tau, max_missed, rows
        self.lock = threading.Lock()  # split nodes call from one thread per device
        self.last_sigma = {}
        self.sparse_heads = {}

    def _note_sigma(self, device, transformer_options):
        """A sigma above the device's previous one starts a new run: forget its verdicts."""
        sigmas = transformer_options.get("sigmas")
        if sigmas is None:
            return
        sigma = float(sigmas.flatten()[0])
        with self.lock:
            last = self.last_sigma.get(device)
            self.last_sigma[device] = sigma
            if last is not None and sigma > last:
                self.sparse_heads = {key: v for key, v in self.sparse_heads.items() if key[1] != device}

    def keep(self, q, k, transformer_options):
        """uint8 keep mask for the kernel, or None to run dense (the calibration
        call of a layer, or a model that does not report block_index)."""
        block = transformer_options.get("block_index")
        if block is None:
            return None
        if transformer_options.get("block_type") is not None:
            block = (transformer_options["block_type"], block)
        self._note_sigma(q.device, transformer_options)
        key = (block, q.device, q.shape[2], k.shape[2])
        keep = predict_keep(q, k, self.tau, self.rows)
        with self.lock:
            sparse = self.sparse_heads.get(key)
        if sparse is None:
            missed = missed_mass(q, k, keep, self.rows)
            sparse = missed <= self.max_missed
            with self.lock:
                self.sparse_heads[key] = sparse
            logging.info(f"[Gfx906 Attention] block {block}: {int(sparse.sum())}/{len(sparse)} heads sparse, "
                         f"missed mass median {missed.median().item():.2%}")
            return None
        return (keep | ~sparse[None, :, None, None]).to(torch.uint8)
