"""In-process split of one DiT sampling step across 2-8 GPUs: the ComfyUI node
``Gfx906RowSplitKrea2`` (reference nodes/ComfyUI-Gfx906Int4/row_split.py:244-271).

ComfyUI is one process, so this split runs there: one host thread per GPU,
the diffusion model replicated onto every extra GPU on first use, and
device-to-device copies (NVLink / NVSwitch peer copies between B200s) for
the only exchange. It generalises the reference's two-GPU split to G GPUs:

  * batch >= 2 (several images, or cond + uncond under cfg): the batch is cut
    into G contiguous parts, one per GPU, no exchange at all
    (row_split.py:179-189);
  * one image with at least ``min_image_tokens`` image tokens: the latent
    rows are cut into G contiguous blocks of token rows on patch boundaries
    (row_split.py:191-206). Each GPU runs the model's own ``_forward`` on its
    block; a ``post_input`` patch offsets its RoPE row ids by its first token
    row (row_split.py:81-85), and an ``attn1`` patch applies RoPE locally and
    all-gathers every GPU's keys and values once per block (the reference
    swaps them with its one peer, row_split.py:47-64,87-96). Every GPU keeps
    the text tokens as queries; only GPU 0 contributes them as keys, so they
    count once;
  * otherwise (no second GPU, not enough free memory for a replica plus
    ``PEER_HEADROOM_BYTES`` of working memory, reference latents, a small
    image) the step runs on one GPU, with one "[Gfx906 Split]" log line per
    change of plan (row_split.py:130-164).

A GPU whose forward raises aborts the exchange barrier, so no thread waits
forever, and its error is the one re-raised (row_split.py:208-241).
``BARRIER_TIMEOUT_S`` bounds every barrier wait as the last resort.

The module imports ComfyUI lazily (``comfy.model_management``,
``comfy.patcher_extension``, ``comfy.ldm.flux.math.apply_rope``); tests
install stand-ins for them. The device list and the free-memory query are
attributes of ``RowSplit`` so that CPU tests can run the same code on CPU
"devices".
"""
from __future__ import annotations

import contextlib
import copy
import logging
import threading

import torch

WRAPPER_KEY = "gfx906_row_split"
BARRIER_TIMEOUT_S = 300
PEER_HEADROOM_BYTES = int(2.5 * 2**30)
AUTO = "auto"
MAX_GPUS = 8

_log = logging.getLogger(__name__)


def _apply_rope(q, k, pe):
    from comfy.ldm.flux.math import apply_rope  # the model's own RoPE
    return apply_rope(q, k, pe)


class KVExchange:
    """All-gather of one block's keys and values among G threads, one per
    device. Thread r publishes (k, v) in slot r and waits at the barrier;
    then it copies every other slot onto its own device -- a cross-device
    ``.to`` runs on the source device's current stream and orders itself
    after both devices' current streams, so the peer's pending kernels
    precede the copy without a host synchronisation -- and waits again, so no
    slot is overwritten by the next block before every thread has taken it.
    The result is the rank-ordered concatenation along the token dim (dim 2)."""

    def __init__(self, world: int, timeout: float = BARRIER_TIMEOUT_S):
        self.world = world
        self.barrier = threading.Barrier(world, timeout=timeout)
        self.slots = [None] * world

    def gather(self, rank: int, k: torch.Tensor, v: torch.Tensor):
        self.slots[rank] = (k, v)
        self.barrier.wait()
        ks, vs = [], []
        for q in range(self.world):
            kq, vq = self.slots[q]
            if q != rank:
                kq = kq.to(k.device, non_blocking=True)
                vq = vq.to(v.device, non_blocking=True)
            ks.append(kq)
            vs.append(vq)
        self.barrier.wait()
        return torch.cat(ks, dim=2), torch.cat(vs, dim=2)


def replicate(module: torch.nn.Module, device: torch.device) -> torch.nn.Module:
    """deepcopy with every parameter and buffer pre-mapped to a copy on
    `device`, so the source device never holds a second copy of the weights
    (int4 ``weight_q4`` / ``weight_scale`` buffers included)."""
    memo = {}
    for p in module.parameters():
        memo[id(p)] = torch.nn.Parameter(p.detach().to(device), requires_grad=False)
    for b in module.buffers():
        memo[id(b)] = b.to(device)
    return copy.deepcopy(module, memo)


def rank_patches(rank: int, row_offset: int, exchange: KVExchange):
    """The transformer patches of one GPU of a row split: ``post_input``
    offsets the image row ids, ``attn1_patch`` applies RoPE and gathers K/V."""
    txt_len = {}

    def post_input(args):
        img_ids = args["img_ids"].clone()
        img_ids[..., 1] += row_offset
        txt_len["n"] = args["txt"].shape[1]
        return {"img": args["img"], "txt": args["txt"], "img_ids": img_ids, "txt_ids": args["txt_ids"]}

    def attn1(q, k, v, pe=None, attn_mask=None, extra_options=None):
        if pe is not None:
            q, k = _apply_rope(q, k, pe)
        if rank != 0:  # only GPU 0's text tokens are keys
            k, v = k[:, :, txt_len["n"]:], v[:, :, txt_len["n"]:]
        k, v = exchange.gather(rank, k, v)
        return {"q": q, "k": k, "v": v, "pe": None}

    return {"post_input": [post_input], "attn1_patch": [attn1]}


def with_patches(transformer_options: dict, patches: dict) -> dict:
    opts = transformer_options.copy()
    merged = {k: list(v) for k, v in opts.get("patches", {}).items()}
    for name, fns in patches.items():
        merged[name] = merged.get(name, []) + fns
    opts["patches"] = merged
    return opts


def _to(value, device):
    return value.to(device) if torch.is_tensor(value) else value


def _batch_slice(value, batch: int, part: slice):
    return value[part] if torch.is_tensor(value) and value.ndim > 0 and value.shape[0] == batch else value


def module_bytes(module: torch.nn.Module) -> int:
    return sum(t.numel() * t.element_size() for t in (*module.parameters(), *module.buffers()))


def even_parts(n: int, g: int):
    """[start, stop) of g contiguous, near-equal parts of n (the first n % g
    parts one longer); parts may be empty only when n < g."""
    base, extra = divmod(n, g)
    out, s = [], 0
    for i in range(g):
        e = s + base + (1 if i < extra else 0)
        out.append((s, e))
        s = e
    return out


def _device_ctx(device: torch.device):
    return torch.cuda.device(device) if device.type == "cuda" else contextlib.nullcontext()


def _cuda_devices():
    return [torch.device("cuda", i) for i in range(torch.cuda.device_count())]


def _comfy_free_memory(device):
    import comfy.model_management as mm
    return mm.get_free_memory(device)


def _comfy_make_room(need, device):
    import comfy.model_management as mm
    mm.free_memory(need, device)


class RowSplit:
    """The DIFFUSION_MODEL wrapper: called as
    ``wrapper(executor, x, timesteps, context, attention_mask, ref_latents,
    transformer_options, **kwargs)`` (the executor's ``class_obj`` is the
    diffusion model, with ``patch`` and ``_forward``)."""

    def __init__(self, device: str = AUTO, min_image_tokens: int = 2048, gpus: int = 2):
        if not 2 <= gpus <= MAX_GPUS:
            raise ValueError(f"Gfx906 Split: gpus must be in [2, {MAX_GPUS}], got {gpus}")
        self.requested = device
        self.min_image_tokens = min_image_tokens
        self.gpus = gpus
        self.replicas = {}  # device -> replica of the diffusion model
        self.last_plan = None
        # injectable for tests: the visible devices and the memory queries
        self.list_devices = _cuda_devices
        self.free_memory = _comfy_free_memory
        self.make_room = _comfy_make_room

    def _log_plan(self, plan: str):
        if plan != self.last_plan:
            _log.info(f"[Gfx906 Split] {plan}")
            self.last_plan = plan

    def pick_peers(self, main: torch.device):
        """The extra devices: the requested one (with gpus == 2), or under
        "auto" the gpus - 1 other devices with the most free memory, checked
        every step. The main device is the latent's (row_split.py:135-148)."""
        if self.requested != AUTO:
            peer = torch.device(self.requested)
            if peer == main:
                raise ValueError(f"Gfx906 Split: second GPU must differ from the model's GPU; expected a device "
                                 f"other than {main}, got {peer} (use \"auto\")")
            return [peer]
        others = [d for d in self.list_devices() if d != main]
        others.sort(key=self.free_memory, reverse=True)
        return others[:self.gpus - 1]

    def ensure_replicas(self, dm: torch.nn.Module, peers):
        """A replica on every peer that has room for it and the working memory
        (freeing ComfyUI-managed models there first if needed); the peers that
        do not are dropped (row_split.py:150-164)."""
        for d in [d for d in self.replicas if d not in peers]:
            del self.replicas[d]
        ok = []
        for peer in peers:
            need = PEER_HEADROOM_BYTES + (0 if peer in self.replicas else module_bytes(dm))
            if self.free_memory(peer) < need:
                self.make_room(need, peer)
            free = self.free_memory(peer)
            if free < need:
                self._log_plan(f"without {peer}: {free / 2**30:.1f} GB free, a split needs {need / 2**30:.1f} GB")
                self.replicas.pop(peer, None)
                continue
            if peer not in self.replicas:
                self.replicas[peer] = replicate(dm, peer)
            ok.append(peer)
        return ok

    def __call__(self, executor, x, timesteps, context, attention_mask, ref_latents, transformer_options, **kwargs):
        dm = executor.class_obj

        def one_gpu(why):
            self._log_plan(f"one GPU: {why}")
            return executor(x, timesteps, context, attention_mask, ref_latents, transformer_options, **kwargs)

        if ref_latents:  # reference latents would be appended whole on every GPU (duplicated keys)
            return one_gpu("reference latents are not split")
        peers = self.pick_peers(x.device)
        if not peers:
            return one_gpu("no second GPU")
        peers = self.ensure_replicas(dm, peers)
        if not peers:
            return one_gpu("no peer has room for a replica")
        devices = [x.device] + peers
        batch = x.shape[0]
        if batch >= 2:
            parts = [(a, b) for a, b in even_parts(batch, min(len(devices), batch))]
            devices = devices[:len(parts)]
            args, kws = [], []
            for a, b in parts:
                sl = slice(a, b)
                args.append([_batch_slice(v, batch, sl) for v in (x, timesteps, context, attention_mask)])
                kws.append({k: _batch_slice(v, batch, sl) for k, v in kwargs.items()})
            self._log_plan("batch split: " + " + ".join(f"{d} x{b - a}" for d, (a, b) in zip(devices, parts)))
            return self.run_group(executor, devices, args, kws, [transformer_options] * len(devices), 0, None)
        patch = dm.patch
        h, w = x.shape[-2], x.shape[-1]
        h_tok = -(-h // patch)
        if h_tok * (-(-w // patch)) < self.min_image_tokens:
            return one_gpu(f"{h_tok * (-(-w // patch))} image tokens < min_image_tokens {self.min_image_tokens}")
        if h_tok < len(devices):
            devices = devices[:h_tok]
            if len(devices) < 2:
                return one_gpu(f"{h_tok} token row(s)")
        rows = even_parts(h_tok, len(devices))
        self._log_plan("row split: " + " + ".join(f"{d} rows {a}-{b}" for d, (a, b) in zip(devices, rows))
                       + " (token rows)")
        exchange = KVExchange(len(devices))
        args, opts = [], []
        for r, (a, b) in enumerate(rows):
            xs = x[..., a * patch:min(b * patch, h), :]
            args.append([xs, timesteps, context, attention_mask])
            opts.append(with_patches(transformer_options, rank_patches(r, a, exchange)))
        return self.run_group(executor, devices, args, [kwargs] * len(devices), opts, -2, exchange)

    def run_group(self, executor, devices, args, kwargs, opts, cat_dim, exchange):
        """GPU 0 through the wrapper chain on the calling thread, every other
        GPU on its replica in a worker thread; outputs concatenated along
        cat_dim on GPU 0. A failing GPU aborts the exchange barrier."""
        results = [None] * len(devices)
        errors = {}

        def run_peer(i):
            dev = devices[i]
            try:
                with _device_ctx(dev), torch.inference_mode():
                    results[i] = self.replicas[dev]._forward(
                        *[_to(v, dev) for v in args[i]], None, opts[i], **{k: _to(v, dev) for k, v in kwargs[i].items()})
            except BaseException as e:  # noqa: BLE001 - re-raised on the calling thread
                errors[i] = e
                if exchange is not None:
                    exchange.barrier.abort()

        threads = [threading.Thread(target=run_peer, args=(i,), name=f"gfx906-split-{i}")
                   for i in range(1, len(devices))]
        for t in threads:
            t.start()
        def root_cause():
            # a broken barrier only means another GPU died first: its error is the one worth showing
            real = [errors[i] for i in sorted(errors) if not isinstance(errors[i], threading.BrokenBarrierError)]
            return real[0] if real else errors[min(errors)]

        try:
            results[0] = executor(*args[0], None, opts[0], **kwargs[0])
        except BaseException as e:
            if exchange is not None:
                exchange.barrier.abort()
            for t in threads:
                t.join()
            if isinstance(e, threading.BrokenBarrierError) and errors:
                raise root_cause() from e
            raise
        for t in threads:
            t.join()
        if errors:
            raise root_cause()
        out0 = results[0]
        return torch.cat([out0] + [r.to(out0.device) for r in results[1:]], dim=cat_dim)


class Gfx906RowSplitKrea2:
    """MODEL -> MODEL. Runs each sampling step on several GPUs: the batch
    split across them when batch >= 2, otherwise the image's token rows.
    Replicates the diffusion model onto every extra GPU on first use; a step
    runs on fewer GPUs (or one) when a GPU lacks room. ``device`` and
    ``min_image_tokens`` are the reference node's inputs; the optional
    ``gpus`` (default 2, the reference's count) sets how many GPUs share a
    step."""

    @classmethod
    def INPUT_TYPES(cls):
        n = torch.cuda.device_count() if torch.cuda.is_available() else 0
        devices = [AUTO] + [f"cuda:{i}" for i in range(n)]
        return {
            "required": {
                "model": ("MODEL",),
                "device": (devices, {"default": AUTO, "tooltip": "Second GPU. auto: whichever GPUs the model is "
                                     "not on with the most free VRAM, checked every step."}),
                "min_image_tokens": ("INT", {"default": 2048, "min": 0, "max": 1 << 20, "tooltip":
                                     "Single-image steps below this many image tokens run on one GPU. Batches of "
                                     "2+ always split by batch."}),
            },
            "optional": {
                "gpus": ("INT", {"default": 2, "min": 2, "max": MAX_GPUS, "tooltip":
                         "How many GPUs share a step (device must be auto for more than 2)."}),
            },
        }

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "patch"
    CATEGORY = "gfx906"
    TITLE = "Gfx906 Split Krea2 (2 GPUs)"

    def patch(self, model, device, min_image_tokens, gpus: int = 2):
        import comfy.patcher_extension as pe
        if device != AUTO and gpus != 2:
            raise ValueError(f"Gfx906 Split: a named device takes gpus=2, got gpus={gpus} (use \"auto\")")
        model = model.clone()
        model.remove_wrappers_with_key(pe.WrappersMP.DIFFUSION_MODEL, WRAPPER_KEY)
        model.add_wrapper_with_key(pe.WrappersMP.DIFFUSION_MODEL, WRAPPER_KEY, RowSplit(device, min_image_tokens, gpus))
        return (model,)
