"""Fused attention, host side (no GPU): the prepare step against the
reference's own prepare step (tests/golden/attention_prep.npz, written by
make_golden_attention.py from nodes/ComfyUI-Gfx906Int4/attention.py:31-75),
the oracle's kernel restatement against exact attention and the keep-mask
emulation of develop/experiments/2026-09-29/test_keep_mask.py:51-61, and the
ComfyUI node / override wiring."""
import os

import numpy as np
import pytest
import torch

import oracle as O
from comfy_ui_gfx906_tools_b200 import attention as A

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "attention_prep.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


@pytest.mark.parametrize("mode", ["fp16", "int8", "int4"])
def test_prepare_qk_is_the_reference_prepare(gold, mode):
    qb, qs, kb, ks = A.prepare_qk(torch.from_numpy(gold["q"]), torch.from_numpy(gold["k"]), mode)
    assert np.array_equal(qb.numpy(), gold[f"qk_{mode}_qb"])
    assert np.array_equal(kb.numpy(), gold[f"qk_{mode}_kb"])
    assert np.array_equal(qs.numpy(), gold[f"qk_{mode}_qs"])
    assert np.array_equal(ks.numpy(), gold[f"qk_{mode}_ks"])


@pytest.mark.parametrize("mode", ["fp16", "u8"])
def test_prepare_v_is_the_reference_prepare(gold, mode):
    vt, vs = A.prepare_v(torch.from_numpy(gold["v"]), mode)
    assert np.array_equal(vt.numpy(), gold[f"v_{mode}_vt"])
    assert np.array_equal(vs.numpy(), gold[f"v_{mode}_vs"])


def _oracle(gold, qk, pv, skip=0.0, keep=None):
    qm, pm = A.QK_MODES[qk], A.PV_MODES[pv]
    return O.attention_reference(gold[f"qk_{qk}_qb"], gold[f"qk_{qk}_qs"], gold[f"qk_{qk}_kb"], gold[f"qk_{qk}_ks"],
                                 gold[f"v_{pv}_vt"], gold[f"v_{pv}_vs"], qm, pm, skip, keep)


def _rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b))


def test_oracle_fp16_modes_track_exact_attention(gold):
    """fp16 Q.K and P.V is exact attention up to fp16 storage of q, p and out;
    the u8 P.V adds the 8-bit P and V levels."""
    ex = O.exact_attention(gold["q"].astype(np.float32), gold["k"].astype(np.float32), gold["v"].astype(np.float32))
    assert _rel(_oracle(gold, "fp16", "fp16"), ex) < 1e-3
    assert _rel(_oracle(gold, "fp16", "u8"), ex) < 1.5e-2
    assert _rel(_oracle(gold, "int8", "u8"), ex) < 5e-2


def test_oracle_keep_mask_is_the_masked_softmax(gold):
    """A keep mask drops whole (query block, key tile) pairs from the softmax
    (test_keep_mask.py:51-61): fp16 modes against the float64 emulation."""
    q, k, v = gold["q"].astype(np.float64), gold["k"].astype(np.float64), gold["v"].astype(np.float64)
    B, H, L, D = q.shape
    n_tiles, rows = -(-L // 64), O.attention_block_rows(0)
    keep = np.ones((B, H, -(-L // rows), n_tiles), dtype=np.uint8)
    keep[0, 0, 0, 1] = 0
    keep[0, 1, 1, 0] = 0
    got = _oracle(gold, "fp16", "fp16", keep=keep).reshape(B, L, H, D)
    rep = H // k.shape[1]
    for h in range(H):
        s = q[0, h] @ k[0, h // rep].T * D ** -0.5
        mask = np.repeat(keep[0, h], 64, axis=1)[np.arange(L) // rows, :L].astype(bool)
        s = np.where(mask, s, -np.inf)
        p = np.exp(s - s.max(-1, keepdims=True))
        want = (p @ v[0, h // rep]) / p.sum(-1, keepdims=True)
        assert _rel(got[0, :, h], want) < 1e-3


def test_oracle_skip_below_zero_is_dense(gold):
    a = _oracle(gold, "int8", "u8", 0.0)
    b = _oracle(gold, "int8", "u8", 0.0, np.ones((1, 2, 1, 2), dtype=np.uint8))
    assert np.array_equal(a, b)


def test_prepared_argument_checks_on_cpu_tensors():
    x = torch.zeros(1, 1, 4, 128, dtype=torch.uint8)
    with pytest.raises(ValueError, match="qk in"):
        A.attention_prepared(x, x, x, x, x, x, "int16", "u8")
    with pytest.raises(RuntimeError, match="CUDA device"):
        A.attention_prepared(x, x, x, x, x, x, "int8", "u8")
    with pytest.raises(ValueError, match="head dim"):
        A.fused_attention(torch.zeros(1, 1, 4, 64), torch.zeros(1, 1, 4, 64), torch.zeros(1, 1, 4, 64))


def test_override_falls_through_for_unhandled_calls():
    calls = []

    def func(q, k, v, heads, **kw):
        calls.append(kw)
        return "comfy"

    ov = A.make_override("int8", "u8", 1e-4)
    q = torch.zeros(1, 2, 10, 128)
    # too few keys, a mask, a custom scale, a 3-d call: all go to ComfyUI's backend
    assert ov(func, q, q, q, 2, skip_reshape=True) == "comfy"
    big = torch.zeros(1, 2, A.MIN_FUSED_TOKENS, 128)
    assert ov(func, big, big, big, 2, mask=torch.zeros(1), skip_reshape=True) == "comfy"
    assert ov(func, big, big, big, 2, skip_reshape=True, scale=0.1) == "comfy"
    assert ov(func, big, big, big, 2, skip_reshape=False) == "comfy"
    assert len(calls) == 4


def test_node_patch_installs_override():
    class Attn(torch.nn.Module):
        heads, kvheads = 24, 8

    class DM(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.attn = Attn()

    class Model:
        def __init__(self):
            self.model = type("M", (), {"diffusion_model": DM()})()
            self.model_options = {"transformer_options": {}}

        def clone(self):
            c = Model()
            c.model = self.model
            return c

    assert A._gqa_repeat(DM()) == 3
    (patched,) = A.Gfx906FusedAttention().patch(Model(), "int4", "u8", 1e-4, 0.0)
    assert callable(patched.model_options["transformer_options"]["optimized_attention_override"])
    (sparse,) = A.Gfx906FusedAttention().patch(Model(), "int4", "u8", 1e-4, 0.5, 0.02, "per_run")
    assert callable(sparse.model_options["transformer_options"]["optimized_attention_override"])


# ---- block-sparse keep masks (block_sparse.py:60-90, 193-235 of the reference) ----
from comfy_ui_gfx906_tools_b200 import block_sparse as BS  # noqa: E402


@pytest.mark.parametrize("tau,rows", [(0.9, 128), (0.995, 64)])
def test_predict_keep_and_missed_mass_are_the_references(gold, tau, rows):
    q, k = torch.from_numpy(gold["bs_q"]), torch.from_numpy(gold["bs_k"])
    keep = BS.predict_keep(q, k, tau, rows)
    assert np.array_equal(keep.numpy(), gold[f"bs_keep_{rows}"])
    assert 0 < keep.float().mean() < 1  # a strict subset: the fixture exercises the prediction
    missed = BS.missed_mass(q, k, keep, rows)
    assert np.allclose(missed.numpy(), gold[f"bs_missed_{rows}"], rtol=1e-5, atol=1e-7)


def test_sparsity_state_calibrates_once_per_run():
    g = torch.Generator().manual_seed(4)
    q = torch.randn(1, 2, 300, 128, generator=g).half()
    k = torch.randn(1, 1, 450, 128, generator=g).half()
    st = BS.SparsityState(0.9, 1.0, 128)  # max_missed 1.0: every head may run sparse
    opts = {"block_index": 3, "sigmas": torch.tensor([1.0])}
    assert st.keep(q, k, {}) is None  # no block_index: dense
    assert st.keep(q, k, opts) is None  # first call of the layer in this run: dense, calibrates
    m = st.keep(q, k, {"block_index": 3, "sigmas": torch.tensor([0.5])})
    assert m is not None and m.dtype == torch.uint8 and tuple(m.shape) == (1, 2, 3, 8)
    assert torch.equal(m.bool(), BS.predict_keep(q, k, 0.9, 128))
    assert st.keep(q, k, {"block_index": 3, "sigmas": torch.tensor([2.0])}) is None  # sigma rose: a new run
    strict = BS.SparsityState(0.9, -1.0, 128)  # no head passes: dense masks everywhere
    strict.keep(q, k, opts)
    assert bool(strict.keep(q, k, opts).bool().all())
