"""Multi-GPU split of one DiT forward: batch split and token-row split.

B200 re-design of the reference's two-GPU split
(nodes/ComfyUI-Gfx906Int4/row_split.py): one process per GPU over
``torch.distributed`` (NCCL over NVLink / NVSwitch) instead of a worker thread
and PCIe copies, for any world size that divides the work.

  * Batch split (row_split.py:179-189): rank r runs samples
    [r*B/G, (r+1)*B/G) of the batch through its own replica of the model; no
    exchange until the optional all-gather of the outputs.
  * Token-row split (row_split.py:191-206): the image tokens of one sample are
    split into G contiguous blocks of latent rows; every rank keeps all text
    tokens. Each block's attention gathers the image keys and values of all
    ranks with one asynchronous ``all_gather_into_tensor`` per tensor,
    overlapped with the block's next linear (the reference swaps K/V with its
    peer, row_split.py:47-64,87-96); queries stay local, so the
    int4 linears only ever see the rank's own tokens. Text keys come from the
    rank's own (replicated) text stream, so they count once (the reference
    drops rank 1's copy, row_split.py:90-94). RoPE uses each token's true row
    id, as the reference's post_input offset does (row_split.py:81-85).

A rank that fails raises; its peers' next collective ends with the process
group's timeout error instead of waiting forever (the reference aborts its
thread barrier, row_split.py:220-240).
"""
from __future__ import annotations

import logging

import torch
import torch.distributed as dist

from .flux_dit import AttentionExchange

_log = logging.getLogger(__name__)
_last_plan = {}


def _log_plan(kind: str, **plan):
    """One "[Gfx906 Split]" line whenever a split's plan changes (row_split.py:130-133)."""
    key = tuple(sorted(plan.items()))
    if _last_plan.get(kind) != key:
        _last_plan[kind] = key
        _log.info("[Gfx906 Split] %s %s", kind, ", ".join(f"{k}={v}" for k, v in key))


class TokenShard(AttentionExchange):
    """Gathers the image keys/values of every rank (rank order = token order).

    ``start`` issues both all-gathers asynchronously (NCCL runs them on its own
    stream) and ``finish`` waits for them, so the linear a block computes in
    between overlaps the exchange."""

    overlaps = True

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)

    def start(self, img_k, img_v):
        pending = []
        for t in (img_k, img_v):
            t = t.contiguous()
            out = torch.empty(self.world * t.shape[0], *t.shape[1:], dtype=t.dtype, device=t.device)
            work = dist.all_gather_into_tensor(out, t, group=self.group, async_op=True)  # dim-0 concatenation
            pending.append((out, work, t.shape))
        return pending

    def finish(self, pending, txt_k, txt_v):
        full = []
        for out, work, (B, H, L, D) in pending:
            work.wait()
            # [world * B, H, L, D] -> [B, H, world * L, D], rank-major along L
            full.append(out.view(self.world, B, H, L, D).permute(1, 2, 0, 3, 4).reshape(B, H, self.world * L, D))
        return torch.cat([txt_k, full[0]], dim=2), torch.cat([txt_v, full[1]], dim=2)


def row_block(h_tokens: int, rank: int, world: int):
    """Latent token rows [start, stop) owned by `rank` (contiguous, equal-sized)."""
    if h_tokens % world != 0:
        raise ValueError(f"token rows ({h_tokens}) must divide evenly over {world} ranks for the row split")
    per = h_tokens // world
    return rank * per, (rank + 1) * per


def split_forward_rows(model, img, img_ids, txt, txt_ids, timesteps, y, h_tokens: int, w_tokens: int,
                       group=None, gather_output: bool = True):
    """Token-row split forward of one batch on every rank of `group`; returns
    the full [B, L_img, C] output on every rank (or the local rows)."""
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    r0, r1 = row_block(h_tokens, rank, world)
    _log_plan("rows", world=world, rank=rank, latent_rows=f"{r0}:{r1}", h_tokens=h_tokens, w_tokens=w_tokens)
    sl = slice(r0 * w_tokens, r1 * w_tokens)
    saved = model.exchange
    model.exchange = TokenShard(group)
    try:
        out = model(img[:, sl].contiguous(), img_ids[:, sl].contiguous(), txt, txt_ids, timesteps, y)
    finally:
        model.exchange = saved
    if not gather_output:
        return out
    full = torch.empty(world * out.shape[0], *out.shape[1:], dtype=out.dtype, device=out.device)
    dist.all_gather_into_tensor(full, out.contiguous(), group=group)
    full = full.view(world, *out.shape)
    return full.permute(1, 0, 2, 3).reshape(out.shape[0], world * out.shape[1], out.shape[2])


def batch_slice(batch: int, rank: int, world: int):
    if batch % world != 0:
        raise ValueError(f"batch ({batch}) must divide evenly over {world} ranks for the batch split")
    per = batch // world
    return slice(rank * per, (rank + 1) * per)


def split_forward_batch(model, img, img_ids, txt, txt_ids, timesteps, y, group=None, gather_output: bool = True):
    """Batch split forward: each rank runs its slice of the batch; returns the
    full output on every rank (or the local slice)."""
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    sl = batch_slice(img.shape[0], rank, world)
    _log_plan("batch", world=world, rank=rank, samples=f"{sl.start}:{sl.stop}", batch=img.shape[0])
    out = model(img[sl], img_ids[sl], txt[sl], txt_ids[sl], timesteps[sl], y[sl])
    if not gather_output:
        return out
    full = torch.empty(world * out.shape[0], *out.shape[1:], dtype=out.dtype, device=out.device)
    dist.all_gather_into_tensor(full, out.contiguous(), group=group)
    return full


def channel_block(n: int, rank: int, world: int):
    """Output channels [start, stop) owned by `rank` in the output-channel split."""
    if n % world != 0:
        raise ValueError(f"output channels ({n}) must divide evenly over {world} ranks for the channel split")
    per = n // world
    return rank * per, (rank + 1) * per


class SymmetricAllGather:
    """y buffers and barrier flags in symmetric memory for the fused small-M
    GEMM + all-gather (``w4a16_gemm_allgather`` then ``gfx_peer_barrier``).

    Every rank maps every other rank's buffers (``torch.distributed``'s
    symmetric memory over NVLink). One call's kernel stores the rank's
    [M, N_local] block straight into columns [rank*N_local, (rank+1)*N_local)
    of every rank's y; the flag barrier then makes the whole [M, N] visible.
    Two y buffers alternate between calls: a rank writes buffer p again only
    after the barrier of the call in between, which every peer reaches only
    after it finished reading buffer p (its reads precede its next launch in
    stream order), so no buffer is overwritten while a peer still reads it.
    The barrier keeps its epoch on the device, so a sequence of calls can be
    captured in a CUDA graph; capture an even number of calls, so that the
    buffers keep alternating from one replay to the next.

    A peer that never reaches the barrier makes it give up after 2 s and
    record status 7: the next GEMM call on this device then raises GfxError
    (code GFX_ERR_DEVICE) before it launches anything; ``strict=True`` also
    synchronises after every barrier and raises at once.
    """

    ROWS = 64  # the small-M kernel's limit

    def __init__(self, n_max: int, dtype: torch.dtype, device: torch.device, group=None, strict: bool = False):
        self.strict = strict
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.n_max, self.dtype, self.device = n_max, dtype, device
        group_name = (group or dist.group.WORLD).group_name
        self.ybuf = symm_mem.empty((2, self.ROWS * n_max), dtype=dtype, device=device)
        self.y_ptrs = list(symm_mem.rendezvous(self.ybuf, group_name).buffer_ptrs)
        self.flags = symm_mem.empty((self.world + 1,), dtype=torch.int32, device=device)
        self.flags.zero_()
        self.f_ptrs = list(symm_mem.rendezvous(self.flags, group_name).buffer_ptrs)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)  # every rank's flags are zero before the first barrier
        import ctypes
        row = self.ROWS * n_max * self.ybuf.element_size()
        # pointer arrays built once (they outlive every call that passes them)
        self._target_arrs = [(ctypes.c_void_p * self.world)(*[p + k * row for p in self.y_ptrs]) for k in (0, 1)]
        self._targets = [ctypes.cast(a, ctypes.c_void_p) for a in self._target_arrs]
        self._flag_arr = (ctypes.c_void_p * self.world)(*self.f_ptrs)
        self._flag_ptr = ctypes.cast(self._flag_arr, ctypes.c_void_p)
        self.calls = 0

    def gemm(self, xb: torch.Tensor, w_q4: torch.Tensor, scale: torch.Tensor, bias, n_local: int) -> torch.Tensor:
        """y[M, world*n_local] (a view of the current buffer, valid until two
        calls later) = the all-gather of every rank's xb @ dequant(w)^T (+ bias).
        ``xb`` bf16 [M, K] contiguous, M <= 64; ``scale`` fp32 or fp16."""
        from . import _lib, ops
        M, K = xb.shape
        n_total = n_local * self.world
        if M > self.ROWS or n_total > self.n_max:
            raise ValueError(f"fused all-gather takes M <= {self.ROWS}, N <= {self.n_max}; got M={M}, N={n_total}")
        parity = self.calls & 1
        self.calls += 1
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device).cuda_stream
            L = _lib.load()
            ws = ops._workspace(self.device, stream, int(L.w4a16_workspace_bytes(M, n_local, K, 0)))
            ops._call_gemm("w4a16_gemm_allgather", self.device, xb.data_ptr(), _lib.DTYPE_BF16, w_q4.data_ptr(), scale.data_ptr(),
                      _lib.SCALE_F16 if scale.dtype == torch.float16 else _lib.SCALE_F32,
                      bias.data_ptr() if bias is not None else None, self._targets[parity], self.world,
                      self.rank, ops._dtype_code(self.dtype), M, n_local, K, 0,
                      ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0, stream)
            _lib.call("gfx_peer_barrier", self._flag_ptr, self.world, self.rank, stream)
            status = ops.device_status(self.device) if self.strict else 0
            if status != 0:
                raise _lib.GfxError("gfx_peer_barrier", _lib.GFX_ERR_DEVICE,
                                    f"device status {status} after the fused all-gather (a peer did not reach "
                                    "the barrier within its 2 s budget)")
        return self.ybuf[parity, :M * n_total].view(M, n_total)


class SymmetricRowGather:
    """The token-row split of a linear with its all-gather fused into the GEMM
    (``w4a16_gemm_rows_allgather`` then ``gfx_peer_barrier``).

    y buffers [m_max, n_max] live in symmetric memory (every rank maps every
    rank's buffers over NVLink). Rank r computes its rows [row0, row0 + M) and
    the GEMM's epilogue stores them into the same rows of EVERY rank's y, tile
    by tile as they are computed, so the transfer overlaps the math and no
    collective kernel competes for SMs; the flag barrier then makes the whole
    y visible. Two buffers alternate between calls (as in SymmetricAllGather:
    a buffer is rewritten only after the barrier of the call in between).
    ``strict`` synchronises after every barrier and raises on a peer timeout.
    """

    def __init__(self, m_max: int, n_max: int, dtype: torch.dtype, device: torch.device, group=None,
                 strict: bool = False):
        import ctypes
        import torch.distributed._symmetric_memory as symm_mem
        self.strict = strict
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.m_max, self.n_max, self.dtype, self.device = m_max, n_max, dtype, device
        group_name = (group or dist.group.WORLD).group_name
        self.ybuf = symm_mem.empty((2, m_max * n_max), dtype=dtype, device=device)
        y_ptrs = list(symm_mem.rendezvous(self.ybuf, group_name).buffer_ptrs)
        self.flags = symm_mem.empty((self.world + 1,), dtype=torch.int32, device=device)
        self.flags.zero_()
        f_ptrs = list(symm_mem.rendezvous(self.flags, group_name).buffer_ptrs)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)  # every rank's flags are zero before the first barrier
        row = m_max * n_max * self.ybuf.element_size()
        self._target_arrs = [(ctypes.c_void_p * self.world)(*[p + k * row for p in y_ptrs]) for k in (0, 1)]
        self._targets = [ctypes.cast(a, ctypes.c_void_p) for a in self._target_arrs]
        self._flag_arr = (ctypes.c_void_p * self.world)(*f_ptrs)
        self._flag_ptr = ctypes.cast(self._flag_arr, ctypes.c_void_p)
        self.calls = 0

    def gemm(self, x_local: torch.Tensor, w_q4: torch.Tensor, scale: torch.Tensor, bias, row0: int,
             m_total: int) -> torch.Tensor:
        """y[m_total, N] (a view of the current buffer, valid until two calls
        later): every rank's rows of x @ dequant(w)^T (+ bias), this rank's
        x_local (bf16 [M, K] contiguous) being rows [row0, row0 + M)."""
        from . import _lib, ops
        M, K = x_local.shape
        N = w_q4.shape[0]
        if m_total > self.m_max or N > self.n_max or row0 + M > m_total:
            raise ValueError(f"row gather takes m_total <= {self.m_max}, N <= {self.n_max}, row0 + M <= m_total; "
                             f"got m_total={m_total}, N={N}, row0={row0}, M={M}")
        parity = self.calls & 1
        self.calls += 1
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device).cuda_stream
            L = _lib.load()
            ws = ops._workspace(self.device, stream, int(L.w4a16_workspace_bytes(M, N, K, 0))) if M <= 64 else None
            ops._call_gemm("w4a16_gemm_rows_allgather", self.device, x_local.data_ptr(), _lib.DTYPE_BF16,
                           w_q4.data_ptr(), scale.data_ptr(),
                           _lib.SCALE_F16 if scale.dtype == torch.float16 else _lib.SCALE_F32,
                           bias.data_ptr() if bias is not None else None, self._targets[parity], self.world, row0,
                           ops._dtype_code(self.dtype), M, N, K, 0, ws.data_ptr() if ws is not None else None,
                           ws.numel() if ws is not None else 0, stream)
            _lib.call("gfx_peer_barrier", self._flag_ptr, self.world, self.rank, stream)
            status = ops.device_status(self.device) if self.strict else 0
            if status != 0:
                raise _lib.GfxError("gfx_peer_barrier", _lib.GFX_ERR_DEVICE,
                                    f"device status {status} after the fused row all-gather (a peer did not reach "
                                    "the barrier within its 2 s budget)")
        return self.ybuf[parity, :m_total * N].view(m_total, N)


class ChannelShardLinear(torch.nn.Module):
    """Output-channel split of one int4 linear for the M <= 16 (HBM-bound) case.

    Rank r keeps rows [r*N/G, (r+1)*N/G) of ``weight_q4`` / ``weight_scale`` /
    ``bias`` of a ``Gfx906Int4Ops.Linear`` and streams only those, so the
    ranks together read the weight at G times one GPU's HBM bandwidth; one
    ``all_gather_into_tensor`` of the [M, N/G] outputs (KB-scale at small M)
    rebuilds y [M, N] on every rank, or y stays sharded (``gather=False``) for
    a following layer that consumes channel shards. The reference has no such
    split (its row_split.py splits tokens or the batch); this is the B200
    re-design for the small-M (HBM-bound) multi-GPU case.

    ``local_forward(shard, x)`` computes the local slice; it defaults to the
    shard module's own forward (the CUDA kernels).

    ``fused=True`` (CUDA, M <= 64, weight-only mode) replaces the GEMM + NCCL
    all-gather by ONE kernel whose epilogue stores the rank's columns straight
    into every rank's copy of a symmetric-memory y buffer over NVLink
    (``w4a16_gemm_allgather``), followed by a bounded flag barrier over the
    same memory (``gfx_peer_barrier``); see ``SymmetricAllGather``.
    """

    def __init__(self, linear, group=None, local_forward=None, fused: bool = False):
        super().__init__()
        from .ops import Gfx906Int4Ops
        if not getattr(linear, "quantized", False):
            raise ValueError("the channel split takes a quantized Gfx906Int4Ops.Linear")
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.out_features = linear.out_features
        n0, n1 = channel_block(linear.out_features, self.rank, self.world)
        _log_plan("channels", world=self.world, rank=self.rank, channels=f"{n0}:{n1}", out_features=linear.out_features)
        dev = linear.weight_q4.device
        dtype = linear.bias.dtype if linear.bias is not None else None
        shard = Gfx906Int4Ops.Linear(linear.in_features, n1 - n0, bias=linear.bias is not None, device=dev,
                                     dtype=dtype, rotation_group=linear.rotation_group)
        with torch.no_grad():
            shard.weight_q4.copy_(linear.weight_q4[n0:n1])
            shard.weight_scale.copy_(linear.weight_scale[n0:n1])
            if linear.bias is not None:
                shard.bias.copy_(linear.bias[n0:n1])
        self.shard = shard
        self.local_forward = local_forward
        self.fused = fused
        self._sym = None

    def _forward_fused(self, x: torch.Tensor) -> torch.Tensor:
        from . import ops
        sh = self.shard
        lead, K = x.shape[:-1], x.shape[-1]
        x2 = x.reshape(-1, K)
        if sh.rotation_group:
            x2 = ops.hadamard_rotate(x2, sh.rotation_group, torch.bfloat16)
        xb = x2.to(torch.bfloat16).contiguous()
        if self._sym is None or self._sym.dtype != x.dtype or self._sym.device != x.device:
            self._sym = SymmetricAllGather(self.out_features, x.dtype, x.device, self.group)
        bias = sh.bias.to(x.dtype).contiguous() if sh.bias is not None else None
        y = self._sym.gemm(xb, sh.weight_q4, sh._device_scale(sh.weight_scale), bias, sh.out_features)
        return y.clone().reshape(*lead, self.out_features)

    def forward(self, x: torch.Tensor, gather: bool = True) -> torch.Tensor:
        rows = x.numel() // x.shape[-1]
        if (self.fused and gather and self.local_forward is None and x.is_cuda and rows <= SymmetricAllGather.ROWS
                and not getattr(self.shard, "activation_quant", False)):
            return self._forward_fused(x)
        y = self.local_forward(self.shard, x) if self.local_forward is not None else self.shard(x)
        if not gather:
            return y
        lead, n_local = y.shape[:-1], y.shape[-1]
        y2 = y.reshape(-1, n_local).contiguous()
        full = torch.empty(self.world * y2.shape[0], n_local, dtype=y2.dtype, device=y2.device)
        dist.all_gather_into_tensor(full, y2, group=self.group)  # rank-major blocks of rows
        full = full.view(self.world, y2.shape[0], n_local).permute(1, 0, 2).reshape(y2.shape[0], -1)
        return full.reshape(*lead, self.world * n_local)


def token_shard_linear(linear, x: torch.Tensor, group=None, gather: bool = True, local_forward=None) -> torch.Tensor:
    """Token-row split of one large-M linear (weights replicated on every
    rank): rank r computes rows [r*M/G, (r+1)*M/G) of x [..., M, K] -> y, and
    one ``all_gather_into_tensor`` rebuilds y [..., M, N] on every rank when
    ``gather`` (else the rank's rows are returned). No exchange is needed for
    the GEMM itself. ``local_forward(linear, x)`` computes the local rows; it
    defaults to ``linear(x)`` (the CUDA kernels)."""
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    lead, K = x.shape[:-1], x.shape[-1]
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    if M % world != 0:
        raise ValueError(f"token rows ({M}) must divide evenly over {world} ranks for the token split")
    per = M // world
    _log_plan("tokens", world=world, rank=rank, rows=f"{rank * per}:{(rank + 1) * per}", M=M)
    xs = x2[rank * per:(rank + 1) * per]
    y = local_forward(linear, xs) if local_forward is not None else linear(xs)
    if not gather:
        return y
    full = torch.empty(world * per, y.shape[-1], dtype=y.dtype, device=y.device)
    dist.all_gather_into_tensor(full, y.contiguous(), group=group)  # rank-major = row order
    return full.reshape(*lead, y.shape[-1])
