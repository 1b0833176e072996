"""The in-process multi-GPU split node (Gfx906RowSplitKrea2, reference
nodes/ComfyUI-Gfx906Int4/row_split.py) on the CPU: stand-ins for the three
ComfyUI modules it imports, a small DiT that follows ComfyUI's transformer
patch protocol (post_input, attn1_patch), and CPU "devices" cpu:1..cpu:7 for
the peers. The split outputs must equal the unsplit forward (token rows: up to
fp32 summation order in attention; batch: exactly), for 2 to 4 GPUs; a GPU
whose forward raises must surface its own error; the plan falls back to one
GPU when it has to. A GPU case runs the same on two CUDA devices when present."""
import math
import sys
import threading
import types

import pytest
import torch

from comfy_ui_gfx906_tools_b200 import row_split


def _rope(q, k, pe):
    """Stand-in for comfy.ldm.flux.math.apply_rope: rotate channel pairs by
    per-token angles pe [B, 1, L, D/2]."""
    def rot(x):
        x2 = x.float().reshape(*x.shape[:-1], -1, 2)
        c, s = pe.cos(), pe.sin()
        y = torch.stack([x2[..., 0] * c - x2[..., 1] * s, x2[..., 0] * s + x2[..., 1] * c], dim=-1)
        return y.reshape(x.shape).to(x.dtype)
    return rot(q), rot(k)


@pytest.fixture
def comfy_stubs(monkeypatch):
    comfy = types.ModuleType("comfy")
    mm = types.ModuleType("comfy.model_management")
    mm.get_free_memory = lambda d: 1 << 40
    mm.free_memory = lambda need, d: None
    pe = types.ModuleType("comfy.patcher_extension")
    pe.WrappersMP = type("WrappersMP", (), {"DIFFUSION_MODEL": "diffusion_model"})
    ldm = types.ModuleType("comfy.ldm")
    flux = types.ModuleType("comfy.ldm.flux")
    fmath = types.ModuleType("comfy.ldm.flux.math")
    fmath.apply_rope = _rope
    for name, mod in (("comfy", comfy), ("comfy.model_management", mm), ("comfy.patcher_extension", pe),
                      ("comfy.ldm", ldm), ("comfy.ldm.flux", flux), ("comfy.ldm.flux.math", fmath)):
        monkeypatch.setitem(sys.modules, name, mod)
    return types.SimpleNamespace(mm=mm, pe=pe)


class TinyDiT(torch.nn.Module):
    """A small Flux-style DiT following ComfyUI's patch protocol: patchify,
    ``post_input`` patches, joint text+image blocks whose attention calls the
    ``attn1_patch`` patches (RoPE is applied by the model unless a patch
    returns pe=None), image tokens out, unpatchify, crop."""
    patch = 2

    def __init__(self, C=4, D=32, heads=2, blocks=2, ctx=8):
        super().__init__()
        g = torch.Generator().manual_seed(0)
        p = self.patch
        self.C, self.D, self.heads = C, D, heads
        self.img_in = torch.nn.Linear(C * p * p, D)
        self.txt_in = torch.nn.Linear(ctx, D)
        self.qkv = torch.nn.ModuleList([torch.nn.Linear(D, 3 * D) for _ in range(blocks)])
        self.proj = torch.nn.ModuleList([torch.nn.Linear(D, D) for _ in range(blocks)])
        self.out = torch.nn.Linear(D, C * p * p)
        with torch.no_grad():
            for prm in self.parameters():
                prm.copy_(torch.randn(prm.shape, generator=g) * 0.2)
        self.fail = False  # _forward raises (set on one replica by the error propagation test)

    def _forward(self, x, timesteps, context, attention_mask, ref_latents=None, transformer_options=None, **kw):
        if self.fail:
            raise RuntimeError("peer out of memory (planted)")
        transformer_options = transformer_options or {}
        patches = transformer_options.get("patches", {})
        B, C, H, W = x.shape
        p = self.patch
        hp, wp = -(-H // p), -(-W // p)
        xp = torch.nn.functional.pad(x, (0, wp * p - W, 0, hp * p - H))
        img = xp.reshape(B, C, hp, p, wp, p).permute(0, 2, 4, 1, 3, 5).reshape(B, hp * wp, C * p * p)
        rows = torch.arange(hp).repeat_interleave(wp).float()
        cols = torch.arange(wp).repeat(hp).float()
        img_ids = torch.stack([torch.zeros_like(rows), rows, cols], -1)[None].repeat(B, 1, 1).to(x.device)
        txt = context
        txt_ids = torch.zeros(B, txt.shape[1], 3, device=x.device)
        for fn in patches.get("post_input", []):
            o = fn({"img": img, "txt": txt, "img_ids": img_ids, "txt_ids": txt_ids})
            img, txt, img_ids, txt_ids = o["img"], o["txt"], o["img_ids"], o["txt_ids"]
        Lt = txt.shape[1]
        h = torch.cat([self.txt_in(txt), self.img_in(img)], 1) + timesteps[:, None, None]
        ids = torch.cat([txt_ids, img_ids], 1)
        hd = self.D // self.heads
        freqs = torch.arange(hd // 2, device=x.device).float() + 1.0
        pe0 = ((ids[..., 1:2] * 0.37 + ids[..., 2:3] * 0.11) * freqs)[:, None]  # [B, 1, L, hd/2]
        for qkv, proj in zip(self.qkv, self.proj):
            q, k, v = qkv(h).reshape(B, -1, 3, self.heads, hd).permute(2, 0, 3, 1, 4)
            pe = pe0
            for fn in patches.get("attn1_patch", []):
                o = fn(q, k, v, pe=pe, attn_mask=None, extra_options={})
                q, k, v, pe = o["q"], o["k"], o["v"], o["pe"]
            if pe is not None:
                q, k = _rope(q, k, pe)
            a = torch.nn.functional.scaled_dot_product_attention(q, k, v)
            h = h + proj(a.transpose(1, 2).reshape(B, -1, self.D))
        out = self.out(h[:, Lt:])
        out = out.reshape(B, hp, wp, C, p, p).permute(0, 3, 1, 4, 2, 5).reshape(B, C, hp * p, wp * p)
        return out[..., :H, :W]


class Exec:
    """Stand-in for ComfyUI's wrapper executor: calls the model's _forward."""

    def __init__(self, model):
        self.class_obj = model

    def __call__(self, *a, **k):
        return self.class_obj._forward(*a, **k)


def _split(gpus, min_tokens=0, free=1 << 40):
    rs = row_split.RowSplit(row_split.AUTO, min_tokens, gpus)
    rs.list_devices = lambda: [torch.device("cpu", i) for i in range(1, 8)]
    rs.free_memory = lambda d: free
    rs.make_room = lambda need, d: None
    return rs


def _inputs(B=1, H=13, W=10, seed=1):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(B, 4, H, W, generator=g), torch.rand(B, generator=g), torch.randn(B, 5, 8, generator=g))


@pytest.mark.parametrize("gpus", [2, 3, 4])
def test_row_split_matches_unsplit(comfy_stubs, gpus):
    m = TinyDiT()
    x, t, ctx = _inputs()
    want = m._forward(x, t, ctx, None, None, {})
    rs = _split(gpus)
    got = rs(Exec(m), x, t, ctx, None, None, {})
    assert got.shape == want.shape
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)
    assert rs.last_plan.startswith("row split") and len(rs.replicas) == gpus - 1


@pytest.mark.parametrize("gpus,B", [(2, 2), (4, 3), (3, 5)])
def test_batch_split_matches_unsplit(comfy_stubs, gpus, B):
    m = TinyDiT()
    x, t, ctx = _inputs(B=B, H=8, W=8, seed=B)
    want = m._forward(x, t, ctx, None, None, {})
    rs = _split(gpus)
    got = rs(Exec(m), x, t, ctx, None, None, {})
    torch.testing.assert_close(got, want, rtol=0, atol=0)
    assert rs.last_plan.startswith("batch split")


def test_one_gpu_fallbacks(comfy_stubs):
    m = TinyDiT()
    x, t, ctx = _inputs(H=8, W=8)
    want = m._forward(x, t, ctx, None, None, {})
    rs = _split(2, min_tokens=10_000)
    assert torch.equal(rs(Exec(m), x, t, ctx, None, None, {}), want)
    assert "min_image_tokens" in rs.last_plan
    rs = _split(2, free=1 << 20)  # no peer has room for a replica + working memory
    assert torch.equal(rs(Exec(m), x, t, ctx, None, None, {}), want)
    assert rs.last_plan.startswith("one GPU") and not rs.replicas
    rs = _split(2)
    rs.list_devices = lambda: []
    assert torch.equal(rs(Exec(m), x, t, ctx, None, None, {}), want)
    assert "no second GPU" in rs.last_plan
    assert torch.equal(rs(Exec(m), x, t, ctx, None, [x], {}), want)  # reference latents stay on one GPU
    with pytest.raises(ValueError, match="must differ"):
        row_split.RowSplit("cpu", 0, 2).pick_peers(torch.device("cpu"))


def test_peer_error_is_raised_not_a_broken_barrier(comfy_stubs):
    m = TinyDiT()
    x, t, ctx = _inputs()
    rs = _split(3)
    # the replica on cpu:2 raises before its first exchange; the other ranks must not hang
    rs.ensure_replicas(m, [torch.device("cpu", 1), torch.device("cpu", 2)])
    rs.replicas[torch.device("cpu", 2)].fail = True
    done = {}

    def call():
        try:
            rs(Exec(m), x, t, ctx, None, None, {})
        except BaseException as e:  # noqa: BLE001
            done["e"] = e
    th = threading.Thread(target=call)
    th.start()
    th.join(timeout=60)
    assert not th.is_alive(), "a rank is still waiting at the exchange barrier"
    assert isinstance(done.get("e"), RuntimeError) and "planted" in str(done["e"])


def test_node_surface(comfy_stubs):
    node = row_split.Gfx906RowSplitKrea2
    req = node.INPUT_TYPES()["required"]
    assert req["model"] == ("MODEL",) and req["device"][0][0] == "auto"
    assert req["min_image_tokens"][1]["default"] == 2048
    assert node.INPUT_TYPES()["optional"]["gpus"][1]["default"] == 2

    class Patcher:
        def __init__(self):
            self.wrappers = {}

        def clone(self):
            c = Patcher()
            c.wrappers = dict(self.wrappers)
            return c

        def remove_wrappers_with_key(self, kind, key):
            self.wrappers.pop((kind, key), None)

        def add_wrapper_with_key(self, kind, key, fn):
            self.wrappers[(kind, key)] = fn
    base = Patcher()
    (out,) = node().patch(base, "auto", 4096, gpus=4)
    w = out.wrappers[("diffusion_model", row_split.WRAPPER_KEY)]
    assert isinstance(w, row_split.RowSplit) and w.gpus == 4 and w.min_image_tokens == 4096 and not base.wrappers
    (out2,) = node().patch(out, "auto", 2048)
    assert len(out2.wrappers) == 1 and out2.wrappers[("diffusion_model", row_split.WRAPPER_KEY)].gpus == 2
    with pytest.raises(ValueError, match="gpus=2"):
        node().patch(base, "cuda:1", 2048, gpus=3)


def test_even_parts():
    assert row_split.even_parts(10, 3) == [(0, 4), (4, 7), (7, 10)]
    assert row_split.even_parts(4, 4) == [(0, 1), (1, 2), (2, 3), (3, 4)]
    assert sum(b - a for a, b in row_split.even_parts(math.prod((7, 3)), 8)) == 21


@pytest.mark.gpu
def test_row_split_on_cuda_devices(comfy_stubs):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    dev = torch.device("cuda", 0)
    m = TinyDiT().to(dev)
    x, t, ctx = (v.to(dev) for v in _inputs(H=16, W=12))
    want = m._forward(x, t, ctx, None, None, {})
    rs = row_split.RowSplit(row_split.AUTO, 0, min(4, torch.cuda.device_count()))
    rs.free_memory = lambda d: 1 << 40
    rs.make_room = lambda need, d: None
    got = rs(Exec(m), x, t, ctx, None, None, {})
    torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-4)
    assert all(d.type == "cuda" and d != dev for d in rs.replicas)
