"""Fused attention kernels (C ABI ``attention``: csrc/attention_tc.cu, csrc/attention.cu) against the
oracle's restatement of the reference kernel (oracle/attention.py, after
nodes/ComfyUI-Gfx906Int4/csrc/attention.hip:83-357) on the same prepared
inputs, and end to end (``fused_attention``) against exact attention.

Tolerance (floating point): the integer Q.K dots, the score products and the
u8 P.V fold are the same operations as the oracle's; exp2 and the fp32 sum
orders differ in the last bits, which can move a quantized P level by one,
so outputs (fp16) must agree to max |d| <= 4e-3 * max(1, max |ref|) and a
relative Frobenius error below 2e-3. Edge cases as the reference's tests:
ragged L (partial key tile, partial query block), GQA, Lq != Lk (the row
split), batch > 1, keep masks, skip_below.
"""
import numpy as np
import pytest
import torch

import oracle as O
from comfy_ui_gfx906_tools_b200 import attention as A

pytestmark = pytest.mark.gpu
MODES = [(qk, pv) for qk in ("fp16", "int8", "int4") for pv in ("fp16", "u8")]


def _inputs(B, H, KVH, Lq, Lk, seed, dev):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, H, Lq, 128, generator=g) * 2).half().to(dev)
    k = (torch.randn(B, KVH, Lk, 128, generator=g) * 2).half().to(dev)
    v = torch.randn(B, KVH, Lk, 128, generator=g).half().to(dev)
    return q, k, v


def _both(q, k, v, qk, pv, skip=0.0, keep=None):
    qb, qs, kb, ks = A.prepare_qk(q, k, qk)
    vt, vs = A.prepare_v(v, pv)
    got = A.attention_prepared(qb, qs, kb, ks, vt, vs, qk, pv, skip, keep).cpu().numpy()
    want = O.attention_reference(qb.cpu().numpy(), qs.cpu().numpy(), kb.cpu().numpy(), ks.cpu().numpy(),
                                 vt.cpu().numpy(), vs.cpu().numpy(), A.QK_MODES[qk], A.PV_MODES[pv], skip,
                                 keep.cpu().numpy() if keep is not None else None)
    return got, want


def _close(got, want):
    g, w = got.astype(np.float64), want.astype(np.float64)
    assert np.isfinite(g).all()
    d = np.abs(g - w).max()
    rel = np.linalg.norm(g - w) / np.linalg.norm(w)
    assert d <= 4e-3 * max(1.0, np.abs(w).max()) and rel < 2e-3, (d, rel)


@pytest.mark.parametrize("qk,pv", MODES)
@pytest.mark.parametrize("B,H,KVH,Lq,Lk", [(1, 8, 2, 300, 300), (2, 4, 4, 130, 333), (1, 2, 1, 64, 64),
                                           (1, 3, 1, 1, 97)])
def test_kernel_equals_oracle(cuda, qk, pv, B, H, KVH, Lq, Lk):
    q, k, v = _inputs(B, H, KVH, Lq, Lk, 11 + Lq + Lk + H, cuda)
    _close(*_both(q, k, v, qk, pv))


@pytest.mark.parametrize("qk,pv", MODES)
@pytest.mark.parametrize("B,H,KVH,Lq,Lk", [(1, 8, 2, 300, 300), (2, 4, 4, 130, 333)])
def test_mma_sync_kernel_equals_oracle(cuda, monkeypatch, qk, pv, B, H, KVH, Lq, Lk):
    """Every mode runs on the tcgen05 kernel (csrc/attention_tc.cu) by default
    (fp16 Q.K with a keep mask on the mma.sync kernel); GFX906_B200_ATTN_MMA_SYNC=1
    selects the mma.sync kernel (csrc/attention.cu) for all, which must agree
    with the oracle as well."""
    monkeypatch.setenv("GFX906_B200_ATTN_MMA_SYNC", "1")
    q, k, v = _inputs(B, H, KVH, Lq, Lk, 31 + Lq + Lk + H, cuda)
    _close(*_both(q, k, v, qk, pv))


@pytest.mark.parametrize("impl", ["tcgen05", "mma.sync"])
@pytest.mark.parametrize("qk,pv", [("int8", "u8"), ("int4", "u8"), ("fp16", "fp16"), ("fp16", "u8")])
def test_kernel_keep_mask_equals_oracle(cuda, monkeypatch, impl, qk, pv):
    """Keep masks per (query block, key tile): the fp16 modes' blocks are 64 rows,
    so one tcgen05 CTA of 128 rows visits the union of two blocks' tiles and each
    warp only its own block's."""
    monkeypatch.setenv("GFX906_B200_ATTN_MMA_SYNC", "1" if impl == "mma.sync" else "0")
    B, H, KVH, L = 1, 4, 2, 700
    q, k, v = _inputs(B, H, KVH, L, L, 5, cuda)
    rows, tiles = A.block_rows(qk), -(-L // 64)
    g = torch.Generator().manual_seed(3)
    keep = (torch.rand(B, H, -(-L // rows), tiles, generator=g) < 0.5).to(torch.uint8)
    keep[..., 0] = 1  # every block keeps at least one tile
    keep[0, 1, 0, :] = 0
    keep[0, 1, 0, tiles - 1] = 1  # only the partial last tile
    _close(*_both(q, k, v, qk, pv, keep=keep.to(cuda)))


@pytest.mark.parametrize("qk,pv", [("int8", "u8"), ("int4", "fp16"), ("fp16", "u8"), ("fp16", "fp16")])
def test_kernel_skip_below_equals_oracle(cuda, qk, pv):
    """skip_below drops a key tile's P.V per warp of 16 rows, the rows of one
    wave of the reference kernel; with peaked scores many tiles skip."""
    B, H, KVH, L = 1, 4, 4, 900
    q, k, v = _inputs(B, H, KVH, L, L, 8, cuda)
    q = q * 3
    got, want = _both(q, k, v, qk, pv, skip=1e-2)
    _close(got, want)
    dense, _ = _both(q, k, v, qk, pv, skip=0.0)
    assert not np.array_equal(got, dense)  # the threshold did skip work


@pytest.mark.parametrize("qk,pv,bound", [("fp16", "fp16", 2e-3), ("fp16", "u8", 1.5e-2), ("int8", "fp16", 5e-2),
                                         ("int8", "u8", 5e-2), ("int4", "fp16", 0.4), ("int4", "u8", 0.4)])
def test_fused_attention_tracks_exact_attention(cuda, qk, pv, bound):
    """End to end through fused_attention (prepare on the GPU + kernel) against
    float64 attention, the accuracy check of the reference's
    test_fused_attention.py:19-36; the bounds are the oracle's own errors on
    this input with margin (int4 Q.K on random Gaussian q, k is coarse)."""
    q, k, v = _inputs(1, 8, 2, 300, 300, 0, cuda)
    out = A.fused_attention(q, k, v, qk, pv).cpu().numpy().astype(np.float64)
    ex = O.exact_attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy())
    assert np.linalg.norm(out - ex) / np.linalg.norm(ex) < bound


def test_fused_attention_repeatable_and_stream_ordered(cuda):
    q, k, v = _inputs(1, 4, 2, 500, 500, 2, cuda)
    a = A.fused_attention(q, k, v, "int4", "u8", 1e-4)
    b = A.fused_attention(q, k, v, "int4", "u8", 1e-4)
    assert torch.equal(a, b)


def test_attention_rejects_bad_arguments(cuda):
    q, k, v = _inputs(1, 4, 2, 64, 64, 1, cuda)
    qb, qs, kb, ks = A.prepare_qk(q, k, "int8")
    vt, vs = A.prepare_v(v, "u8")
    with pytest.raises(RuntimeError, match="Vt must be uint8"):
        A.attention_prepared(qb, qs, kb, ks, vt[:, :, :, :64], vs, "int8", "u8")
    with pytest.raises(RuntimeError, match="multiple of KVH"):
        A.attention_prepared(qb[:, :3], qs[:, :3], kb, ks, vt, vs, "int8", "u8")
    with pytest.raises(RuntimeError, match="keep must be"):
        A.attention_prepared(qb, qs, kb, ks, vt, vs, "int8", "u8", 0.0, torch.ones(1, 4, 2, 1, dtype=torch.uint8,
                                                                                  device=cuda))
    assert A.block_rows("fp16") == 64 and A.block_rows("int4") == 128 and A.max_tiles() == 1024


def test_override_block_sparse_end_to_end(cuda):
    """The node's override with block-sparse masks (block_sparse.SparsityState):
    the first call of a layer in a run is dense and calibrates, later calls
    run the kernel with keep = prediction | dense heads; each equals
    fused_attention with that mask, and the sparse output stays close to dense
    (structured tokens: runs of 64 around a few centres)."""
    from comfy_ui_gfx906_tools_b200 import block_sparse as BS
    g = torch.Generator().manual_seed(9)
    centers = torch.randn(6, 128, generator=g) * 3
    L, H = 1024, 4
    ids = torch.randint(0, 6, (1, H, L // 64), generator=g).repeat_interleave(64, -1)
    q = (centers[ids] + torch.randn(1, H, L, 128, generator=g) * 0.3).half().to(cuda)
    k = (centers[ids[:, :2]] + torch.randn(1, 2, L, 128, generator=g) * 0.3).half().to(cuda)
    v = torch.randn(1, 2, L, 128, generator=g).half().to(cuda)
    state = BS.SparsityState(0.995, 0.05, A.block_rows("int4"))
    ov = A.make_override("int4", "u8", 0.0, 1, state)

    def fallthrough(*a, **kw):
        raise AssertionError("the override fell through to the host backend")

    dense = ov(fallthrough, q, k, v, H, skip_reshape=True,
               transformer_options={"block_index": 0, "sigmas": torch.tensor([1.0])})
    assert torch.equal(dense, A.fused_attention(q, k, v, "int4", "u8"))
    sparse = ov(fallthrough, q, k, v, H, skip_reshape=True,
                transformer_options={"block_index": 0, "sigmas": torch.tensor([0.9])})
    heads_ok = state.sparse_heads[(0, q.device, L, L)]
    keep = (BS.predict_keep(q, k, 0.995, A.block_rows("int4")) | ~heads_ok[None, :, None, None]).to(torch.uint8)
    assert torch.equal(sparse, A.fused_attention(q, k, v, "int4", "u8", 0.0, keep))
    rel = ((sparse.float() - dense.float()).norm() / dense.float().norm()).item()
    assert rel < 0.1, rel
