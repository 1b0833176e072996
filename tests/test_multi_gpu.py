"""Splits across two GPUs over NCCL (skipped with fewer than two GPUs): the
output-channel split (NCCL all-gather, and the fused kernel that stores into every rank's
symmetric-memory buffer), the token-row split of an int4 linear (torch all-gather, and the GEMM whose
epilogue stores its rows into every rank's buffer) and the batch / token-row splits of an
int4 DiT match the same computation on one GPU. Every rank runs as its own
spawned process with a short process-group timeout."""
import datetime
import multiprocessing as mp
import os
import socket
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        import torch.distributed as dist
        from comfy_ui_gfx906_tools_b200 import flux_dit, ops, parallel, synthetic
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        out = {}
        # output-channel split of one int4 linear, M = 1 and 16
        N, K = 1536, 3072
        raw, _, _ = synthetic.q4_0_weight(N, K, seed=3)
        p, s = ops.repack_q4_0_native(raw.to(dev), N, K)
        lin = ops.Gfx906Int4Ops.Linear(K, N, bias=True, device=dev, dtype=torch.bfloat16)
        with torch.no_grad():
            lin.weight_q4.copy_(p)
            lin.weight_scale.copy_(s)
            lin.bias.copy_(torch.linspace(-1, 1, N, device=dev))
        split = parallel.ChannelShardLinear(lin)
        for m in (1, 16):
            x = synthetic.activations(m, K, seed=4).to(dev)
            ref = lin(x).float()
            got = split(x).float()
            out[f"channel_m{m}"] = float((got - ref).abs().max() / ref.abs().max())
        # fused GEMV + all-gather over symmetric memory: six back-to-back calls (both y buffers used
        # three times) must equal the NCCL split bit for bit, and no peer barrier may time out
        from comfy_ui_gfx906_tools_b200 import _lib
        _lib.load().gfx_device_status(1)
        fused = parallel.ChannelShardLinear(lin, fused=True)
        xs = [synthetic.activations(m, K, seed=20 + i).to(dev) for i, m in enumerate((1, 16, 64, 3, 1, 40))]
        got = [fused(x) for x in xs]
        torch.cuda.synchronize()
        want = [split(x) for x in xs]
        out["fused_exact"] = all(torch.equal(a, b) for a, b in zip(got, want))
        out["fused_status"] = int(_lib.load().gfx_device_status(1))
        # the same calls captured in a CUDA graph (two calls: the buffers keep alternating) and replayed
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            fused(xs[0])
            fused(xs[1])
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            g0, g1 = fused(xs[0]), fused(xs[1])
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        out["fused_graph_exact"] = bool(torch.equal(g0, want[0]) and torch.equal(g1, want[1]))
        out["fused_graph_status"] = int(_lib.load().gfx_device_status(1))
        del graph
        out["fused_vs_one"] = max(float((g.float() - lin(x).float()).abs().max() / lin(x).float().abs().max())
                                  for g, x in zip(got, xs))
        # token-row split of the same linear at large M (weights replicated)
        xt = synthetic.activations(512, K, seed=5).to(dev)
        ref = lin(xt).float()
        got = parallel.token_shard_linear(lin, xt).float()
        out["tokens"] = float((got - ref).abs().max() / ref.abs().max())
        # token-row split with the all-gather fused into the GEMM: each rank's epilogue stores its rows into
        # every rank's symmetric-memory y; M = 600 (tcgen05 kernel, 300 rows per rank) and M = 40 (small-M
        # kernel); several calls so both buffers are reused. Each rank's rows must equal the plain kernel
        # run on the same rows (same M, same plan), bit for bit.
        rg = parallel.SymmetricRowGather(600, N, torch.bfloat16, dev)
        bad = []
        for call, mt in enumerate((600, 40, 600, 40)):
            xa = synthetic.activations(mt, K, seed=30 + mt).to(dev)
            per = mt // world
            yg = rg.gemm(xa[rank * per:(rank + 1) * per].contiguous(), p, s, None, rank * per, mt).clone()
            torch.cuda.synchronize()
            for src in range(world):
                want = ops.gemm_w4a16(xa[src * per:(src + 1) * per].contiguous(), p, s, None, torch.bfloat16)
                got = yg[src * per:(src + 1) * per]
                if not torch.equal(got, want):
                    bad.append((call, mt, src, float((got.float() - want.float()).abs().max())))
        out["rowgather_bad"] = bad
        out["rowgather_status"] = int(_lib.load().gfx_device_status(1))
        # int4 DiT (tiny): batch split and token-row split against the one-GPU forward
        cfg = flux_dit.tiny_config(depth_double=2, depth_single=2)
        model = flux_dit.FluxDiT(cfg, flux_dit.int4_linear_factory(dev, seed=11), dev)
        inputs = flux_dit.make_inputs(cfg, 2, 4, 6, 5, dev, seed=12)
        with torch.no_grad():
            ref = model(*inputs).float()
            gb = parallel.split_forward_batch(model, *inputs).float()
            gr = parallel.split_forward_rows(model, *inputs, 4, 6).float()
        out["batch"] = float((gb - ref).abs().max() / ref.abs().max())
        out["rows"] = float((gr - ref).abs().max() / ref.abs().max())
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", out))
    except Exception:
        q.put((rank, "exception", traceback.format_exc()))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_splits_match_one_gpu():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for rank, status, val in res:
        assert status == "ok", val
        # the channel split reorders nothing inside a dot product: fp32 rounding only
        assert val["channel_m1"] < 1e-2 and val["channel_m16"] < 1e-2, val
        assert val["fused_exact"] and val["fused_status"] == 0 and val["fused_vs_one"] < 1e-2, val
        assert val["fused_graph_exact"] and val["fused_graph_status"] == 0, val
        assert val["tokens"] < 1e-6, val  # the same rows through the same kernel
        assert not val["rowgather_bad"] and val["rowgather_status"] == 0, (val["rowgather_bad"],
                                                                            val["rowgather_status"])
        # bf16 activations through 4 blocks; the split changes only which GPU computes what
        assert val["batch"] < 2e-2 and val["rows"] < 2e-2, val
