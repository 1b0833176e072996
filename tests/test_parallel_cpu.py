"""Multi-process split logic on the CPU (gloo, world size 2): the token-row and
batch splits reproduce the single-process forward of the same DiT, the
output-channel split of one int4 linear gathers the same y as the unsplit
layer (local slices computed by the oracle), and a rank that fails makes its
peer's collective end with an error (bounded timeout) instead of waiting
forever (reference: row_split.py:208-241)."""
import datetime
import multiprocessing as mp
import os
import socket
import traceback

import pytest
import torch

H_TOK, W_TOK, TXT, BATCH = 4, 6, 5, 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model_and_inputs():
    from comfy_ui_gfx906_tools_b200 import flux_dit
    torch.manual_seed(0)
    cfg = flux_dit.tiny_config(depth_double=2, depth_single=2)
    model = flux_dit.FluxDiT(cfg, flux_dit.float_linear_factory("cpu", torch.float32, seed=3), "cpu", torch.float32)
    with torch.no_grad():
        for m in model.modules():
            if isinstance(m, flux_dit.RMSNorm):
                m.scale.uniform_(0.5, 1.5)
    inputs = flux_dit.make_inputs(cfg, BATCH, H_TOK, W_TOK, TXT, "cpu", torch.float32, seed=4)
    return model, inputs


def _worker(rank, world, port, mode, q):
    try:
        import torch.distributed as dist
        from comfy_ui_gfx906_tools_b200 import parallel
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
        torch.set_num_threads(2)
        model, inputs = _model_and_inputs()
        with torch.no_grad():
            if mode == "fail_after":
                parallel.split_forward_rows(model, *inputs, H_TOK, W_TOK)  # one full exchange succeeds
                if rank == 1:
                    raise RuntimeError("rank 1 failed after an exchange")
                try:
                    parallel.split_forward_rows(model, *inputs, H_TOK, W_TOK)
                    q.put((rank, "no-error", None))
                except Exception as e:
                    q.put((rank, "error", type(e).__name__))
                return
            if mode == "fail":
                if rank == 1:
                    raise RuntimeError("rank 1 failed before the exchange")
                try:
                    parallel.split_forward_rows(model, *inputs, H_TOK, W_TOK)
                    q.put((rank, "no-error", None))
                except Exception as e:  # the peer's collective must end with an error
                    q.put((rank, "error", type(e).__name__))
                return
            if mode == "channel":
                q.put((rank, "ok", _channel_split_error(parallel)))
                dist.destroy_process_group()
                return
            ref = model(*inputs)
            if mode == "rows":
                got = parallel.split_forward_rows(model, *inputs, H_TOK, W_TOK)
            else:
                got = parallel.split_forward_batch(model, *inputs)
        q.put((rank, "ok", float((got - ref).abs().max() / ref.abs().max())))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "exception", traceback.format_exc()))


def _channel_split_error(parallel):
    """Max relative error of the gathered channel-split output against the
    unsplit layer, both through the oracle's W4A16 matmul (bit-identical
    slices: the split must only move rows around)."""
    import numpy as np
    import oracle as O
    from comfy_ui_gfx906_tools_b200 import ops
    N, K, M = 96, 128, 3
    g = torch.Generator().manual_seed(5)
    w = torch.randn(N, K, generator=g)
    p, s = O.quantize_pack_int4(w.numpy())
    lin = ops.Gfx906Int4Ops.Linear(K, N, bias=True, dtype=torch.float32)
    with torch.no_grad():
        lin.weight_q4.copy_(torch.from_numpy(p))
        lin.weight_scale.copy_(torch.from_numpy(s))
        lin.bias.copy_(torch.randn(N, generator=g))
    x = torch.randn(1, M, K, generator=g)

    def oracle_forward(mod, xx):
        y = O.w4a16_matmul(xx.reshape(-1, K).numpy(), mod.weight_q4.numpy(), mod.weight_scale.numpy(),
                           mod.bias.detach().numpy())
        return torch.from_numpy(np.asarray(y, dtype=np.float32)).reshape(*xx.shape[:-1], -1)

    split = parallel.ChannelShardLinear(lin, local_forward=oracle_forward)
    got = split(x)
    ref = oracle_forward(lin, x)
    assert got.shape == ref.shape == (1, M, N)
    local = split(x, gather=False)
    assert local.shape == (1, M, N // 2)
    # token-row split of the same layer (large-M case): rows [r*M/G, (r+1)*M/G) per rank
    xt = torch.randn(2, 4, K, generator=g)
    got_t = parallel.token_shard_linear(lin, xt, local_forward=oracle_forward)
    ref_t = oracle_forward(lin, xt)
    assert got_t.shape == ref_t.shape == (2, 4, N)
    err_t = float((got_t - ref_t).abs().max() / ref_t.abs().max())
    return max(float((got - ref).abs().max() / ref.abs().max()), err_t)


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = []
    for _ in range(2):
        results.append(q.get(timeout=120))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(results)


@pytest.mark.parametrize("mode", ["rows", "batch", "channel"])
def test_split_matches_single_process(mode):
    res = _run(mode)
    for rank, status, val in res:
        assert status == "ok", val
        assert val < 1e-5, (rank, val)


@pytest.mark.parametrize("mode", ["fail", "fail_after"])
def test_failed_rank_surfaces_as_error(mode):
    res = dict((r, (s, v)) for r, s, v in _run(mode))
    assert res[1][0] == "exception" and "rank 1 failed" in res[1][1]
    assert res[0][0] == "error", res[0]


def test_row_block_partition():
    from comfy_ui_gfx906_tools_b200 import parallel
    assert [parallel.row_block(128, r, 4) for r in range(4)] == [(0, 32), (32, 64), (64, 96), (96, 128)]
    with pytest.raises(ValueError):
        parallel.row_block(10, 0, 4)
    assert parallel.batch_slice(8, 3, 4) == slice(6, 8)
    assert [parallel.channel_block(96, r, 3) for r in range(3)] == [(0, 32), (32, 64), (64, 96)]
    with pytest.raises(ValueError):
        parallel.channel_block(10, 0, 4)
