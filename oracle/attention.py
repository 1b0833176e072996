"""CPU restatement (numpy) of the reference's fused attention.

TEST INFRASTRUCTURE ONLY: the checker the CUDA attention kernel is compared
against. The product package never imports it.

Follows nodes/ComfyUI-Gfx906Int4/csrc/attention.hip:83-357 (attention_kernel)
step for step on inputs prepared as attention.py:31-75 prepares them (the
prepare step itself is pinned bit for bit to the reference's own Python by
tests/golden/attention_prep.npz):

  * a block of BQ query rows (64 for fp16 Q.K, 128 for the int modes,
    attention.hip:76-79, 373) visits the 64-key tiles its keep byte marks
    (all of them without a mask, :126-138);
  * per tile: s = fp16: q . k (fp32); int: ((float)(q . k) * q_scale) *
    k_scale; keys past Lk get -1e30 (:226-231); row max, alpha = exp2(m -
    m_new), l and o scaled by alpha, rel = exp2(tile max - m_new) (:232-240);
  * skip: the tile's P.V is dropped for every row of a 64-lane wave when the
    largest rel over the wave's 16 rows (rows ty + TY i, ty in [4w, 4w + 4),
    TY = BQ / 4, i < 4) is below skip_below (:241-242, thread layout :17-22);
  * p = exp2(s - m) is added to l for every key (:252-255); P.V: fp16 ->
    o += (half)p . v; u8 -> pq = rint(p * (255 / rel)), o = fmaf(rel / 255 *
    v_scale, (float)(pq . vq) - 128 * sum(pq), o) (:244-263, :291-323);
  * out = (half)(o / l) (:331-340).

Exact in the oracle where the kernel is exact (integer dot products, the
per-element float32 products and the fold); the float32 sums of l and of
the fp16 P.V products, and exp2, differ from any GPU's only in rounding.
"""
from __future__ import annotations

import numpy as np

from .oracle import _fmaf

HEAD_DIM = 128
TILE = 64
NO_SCORE = np.float32(-1e30)

__all__ = ["attention_block_rows", "attention_reference", "unpack_attention_int4", "exact_attention"]


def attention_block_rows(qk_mode: int) -> int:
    return 64 if qk_mode == 0 else 128


def unpack_attention_int4(packed: np.ndarray) -> np.ndarray:
    """uint8 [..., 64] (element 2i low nibble of byte i) -> int32 codes [..., 128]."""
    lo = (packed & 0xF).astype(np.int32)
    hi = (packed >> 4).astype(np.int32)
    codes = np.stack([lo, hi], axis=-1).reshape(*packed.shape[:-1], packed.shape[-1] * 2)
    return np.where(codes >= 8, codes - 16, codes)


def _decode_rows(x: np.ndarray, qk_mode: int) -> np.ndarray:
    if qk_mode == 0:
        return np.ascontiguousarray(x).view(np.float16).astype(np.float64)
    if qk_mode == 1:
        return np.ascontiguousarray(x).view(np.int8).astype(np.int64)
    return unpack_attention_int4(x).astype(np.int64)


def attention_reference(Q, q_scale, K, k_scale, Vt, v_scale, qk_mode: int, pv_mode: int, skip_below: float = 0.0,
                        keep=None) -> np.ndarray:
    """Prepared inputs (uint8 Q [B, H, Lq, RB], K [B, KVH, Lk, RB], Vt [B, KVH,
    tiles, 128, 64 * vbytes], fp32 scales) -> fp16 [B, Lq, H * 128]."""
    B, H, Lq = Q.shape[:3]
    KVH, Lk = K.shape[1], K.shape[2]
    rows = attention_block_rows(qk_mode)
    ty_count = rows // 4
    n_tiles = -(-Lk // TILE)
    n_qb = -(-Lq // rows)
    q_all = _decode_rows(Q, qk_mode)
    k_all = _decode_rows(K, qk_mode)
    if pv_mode == 0:
        v_all = np.ascontiguousarray(Vt).view(np.float16).astype(np.float64)  # [B, KVH, tiles, 128, 64]
    else:
        v_all = Vt.astype(np.int64)
    out = np.zeros((B, Lq, H, HEAD_DIM), dtype=np.float16)
    local = np.arange(rows)
    wave = (local % ty_count) // 4  # the 64-lane wave that owns each row
    inv255 = np.float32(1.0 / 255.0)
    with np.errstate(over="ignore", under="ignore", invalid="ignore", divide="ignore"):
        for b in range(B):
            for h in range(H):
                kvh = h // (H // KVH)
                for qb in range(n_qb):
                    r = qb * rows + local
                    valid = r < Lq
                    q = np.zeros((rows, HEAD_DIM), dtype=q_all.dtype)
                    q[valid] = q_all[b, h, r[valid]]
                    qs = np.ones(rows, dtype=np.float32)
                    if qk_mode != 0:
                        qs[valid] = q_scale.reshape(B, H, Lq)[b, h, r[valid]]
                    m = np.full(rows, NO_SCORE, dtype=np.float32)
                    l = np.zeros(rows, dtype=np.float32)
                    o = np.zeros((rows, HEAD_DIM), dtype=np.float32)
                    tiles = range(n_tiles) if keep is None else [t for t in range(n_tiles) if keep[b, h, qb, t]]
                    for t in tiles:
                        k0 = t * TILE
                        keys = k0 + np.arange(TILE)
                        kv = keys < Lk
                        kt = np.zeros((TILE, HEAD_DIM), dtype=k_all.dtype)
                        kt[kv] = k_all[b, kvh, keys[kv]]
                        if qk_mode == 0:
                            s = (q @ kt.T).astype(np.float32)
                        else:
                            ks = np.zeros(TILE, dtype=np.float32)
                            ks[kv] = k_scale.reshape(B, KVH, Lk)[b, kvh, keys[kv]]
                            s = ((q @ kt.T).astype(np.float32) * qs[:, None]) * ks[None, :]
                        s[:, ~kv] = NO_SCORE
                        tmax = s.max(axis=1)
                        m_new = np.maximum(m, tmax)
                        alpha = np.exp2(m - m_new)
                        m = m_new
                        l = l * alpha
                        o = o * alpha[:, None]
                        rel = np.exp2(tmax - m_new)
                        wave_rel = np.zeros(rows // 16, dtype=np.float32)
                        np.maximum.at(wave_rel, wave, rel)
                        run = wave_rel[wave] >= np.float32(skip_below)  # rows whose wave does the P.V
                        p = np.exp2(s - m[:, None])
                        l = (l + p.sum(axis=1, dtype=np.float32)).astype(np.float32)
                        if not run.any():
                            continue
                        vt = v_all[b, kvh, t]  # [128, 64]
                        if pv_mode == 0:
                            ph = p.astype(np.float16).astype(np.float64)
                            o[run] = (o[run] + (ph[run] @ vt.T).astype(np.float32)).astype(np.float32)
                        else:
                            pscale = rel * inv255
                            inv = np.where(rel > np.float32(1e-30), np.float32(255.0) / rel, np.float32(0.0))
                            pq = np.rint(p * inv[:, None])
                            pqsum = pq.sum(axis=1, dtype=np.float32)
                            acc = pq.astype(np.int64) @ vt.T  # [rows, 128], exact
                            vs = v_scale.reshape(B, KVH, n_tiles, HEAD_DIM)[b, kvh, t]
                            fold = _fmaf(pscale[:, None] * vs[None, :],
                                         acc.astype(np.float32) - np.float32(128.0) * pqsum[:, None], o)
                            o[run] = fold[run]
                    res = (o / l[:, None]).astype(np.float16)
                    out[b, r[valid], h] = res[valid]
    return out.reshape(B, Lq, H * HEAD_DIM)


def exact_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """softmax(q k^T / sqrt(128)) v in float64; q [B, H, Lq, 128], k / v
    [B, KVH, Lk, 128] -> [B, Lq, H * 128] (the accuracy reference of
    develop/experiments/2026-09-29/test_fused_attention.py:19-26)."""
    B, H, Lq, D = q.shape
    rep = H // k.shape[1]
    kf = np.repeat(k.astype(np.float64), rep, axis=1)
    vf = np.repeat(v.astype(np.float64), rep, axis=1)
    s = q.astype(np.float64) @ kf.transpose(0, 1, 3, 2) * D ** -0.5
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return (p @ vf).transpose(0, 2, 1, 3).reshape(B, Lq, H * D)
