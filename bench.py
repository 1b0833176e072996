"""Benchmark of the int4 W4A16 linear path on B200 (driver contract: one JSON line).

Workload (config 2, "flux_linear_sweep"): one step = the six Flux DiT
linear shapes at hidden 3072 ((K, N) in qkv 3072x9216, proj 3072x3072, mlp-up
3072x12288, mlp-down 12288x3072, single-fused 3072x21504, single-out
15360x3072), M = 4608 tokens each, bf16 activations, int4 group-32 weights
from synthetic ggml Q4_0 blocks, bf16 output. metric = whole-job TFLOP/s
(2*M*N*K per GEMM). Each step reads > 126 MB (L2) of distinct inputs, so the
timed loop does not run out of L2. The M in {1, 16} variants of the same
weights are reported as GB/s of algorithmic bytes in "small_m".

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun: every rank runs the same per-GPU workload (its own
4608 tokens; weak scaling, no data-path collective), timing is the max over
ranks of CUDA-event time. --impl reference times the reference's CPU torch
path (dequant + fp32 matmul; the oracle's torch port) on this host's cores.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

SHAPES = [("qkv", 3072, 9216), ("proj", 3072, 3072), ("mlp_up", 3072, 12288), ("mlp_down", 12288, 3072),
          ("single_fused", 3072, 21504), ("single_out", 15360, 3072)]
METRIC = "int4 W4A16 GEMM TFLOP/s at M=4608 over the six Flux linear shapes"
UNIT = "TFLOP/s"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(r[0] for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[2]) if v.lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows)}


def setup_dist(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v, world, dev):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
def cpu_reference_sample(shape_idx, rows, seed=0):
    """Reference CPU torch path on one shape: full dequant + fp32 matmul of `rows`
    tokens; returns (t_dequant, t_matmul, flops_extrapolated_to_4608, seconds_extrapolated)."""
    import oracle as O
    from comfy_ui_gfx906_tools_b200 import synthetic
    name, K, N = SHAPES[shape_idx]
    raw, _, _ = synthetic.q4_0_weight(N, K, seed=seed + shape_idx)
    p, s = O.repack_q4_0_native(raw.numpy(), N, K)
    pt, st = torch.from_numpy(p), torch.from_numpy(s)
    x = synthetic.activations(rows, K, seed=seed + 50)
    t0 = time.perf_counter()
    w = O.torch_cpu_dequant(pt, st)
    t1 = time.perf_counter()
    y = torch.matmul(x.float(), w.t())
    t2 = time.perf_counter()
    del y
    t_dq, t_mm = t1 - t0, t2 - t1
    M = 4608
    return t_dq, t_mm, 2.0 * M * N * K, t_dq + t_mm * (M / rows)


def run_reference(args, world, rank):
    if rank != 0:
        return
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    rows = 256
    for i in range(args.warmup):
        cpu_reference_sample(i % len(SHAPES), rows)
    flops = secs = 0.0
    t_start = time.perf_counter()
    for i in range(args.steps):
        _, _, f, s = cpu_reference_sample(i % len(SHAPES), rows)
        flops += f
        secs += s
    wall = time.perf_counter() - t_start
    value = flops / secs / 1e12
    sample = (f"per step one Flux shape (round-robin): full torch-CPU dequant of W + fp32 matmul of {rows} of the "
              f"4608 rows, extrapolated to M=4608 as t_dequant + t_matmul*4608/{rows}")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * secs / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "flux_linear_sweep", "M": 4608, "shapes": [s[0] for s in SHAPES]},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": wall,
    }))


# ---------------------------------------------------------------------------
def make_weights(dev, seed):
    from comfy_ui_gfx906_tools_b200 import ops, synthetic
    ws = []
    for i, (name, K, N) in enumerate(SHAPES):
        raw, _, _ = synthetic.q4_0_weight(N, K, seed=seed + i)
        p, s = ops.repack_q4_0_native(raw.to(dev), N, K)
        s16 = ops.scales_to_f16_if_exact(s)
        ws.append((name, K, N, p, s16 if s16 is not None else s))
    return ws


def time_steps(fn, steps, warmup, world, dev, stream, soak_s=0.0):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    # clock soak: keep the GPU busy (untimed) long enough for the nvidia-smi
    # sampler to see the clocks under this load before the timed region
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < soak_s:
        fn()
        torch.cuda.synchronize(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        fn()
    b.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    return a.elapsed_time(b)


def run_ours(args, world, rank, local):
    from comfy_ui_gfx906_tools_b200 import ops, synthetic
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    pk = peaks()
    M = args.m
    weights = make_weights(dev, seed=1000)
    xs = [synthetic.activations(M, K, seed=2000 + i).to(dev) for i, (_, K, _, _, _) in enumerate(weights)]
    flops_step = sum(2.0 * M * N * K for (_, K, N, _, _) in weights)

    # --- device-resident timed loop, with per-launch events for the roofline ---
    launch_ms = [0.0] * len(weights)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in weights]
    record = {"on": False}

    def step():
        for i, ((_, K, N, p, s), x) in enumerate(zip(weights, xs)):
            if record["on"]:
                ev[i][0].record(stream)
            ops.gemm_w4a16(x, p, s, None, torch.bfloat16)
            if record["on"]:
                ev[i][1].record(stream)

    def timed_step():
        step()
        torch.cuda.synchronize(dev)
        for i in range(len(weights)):
            launch_ms[i] += ev[i][0].elapsed_time(ev[i][1])

    clocks = ClockSampler(dev.index)
    with clocks:
        ms_total = time_steps(step, args.steps, args.warmup, world, dev, stream, soak_s=1.0)
    ms_total = max_over_ranks(ms_total, world, dev)
    ms_step = ms_total / args.steps
    value = world * flops_step / (ms_step * 1e-3) / 1e12
    # per-launch durations, measured on the launching stream in a second pass
    record["on"] = True
    for _ in range(args.steps):
        timed_step()
    record["on"] = False
    avg_launch_ms = sum(launch_ms) / (args.steps * len(weights))
    achieved = (flops_step / len(weights)) / (avg_launch_ms * 1e-3) / 1e12
    peak = pk["bf16_tflops_sustained"]
    traffic = None
    tf = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tf):
        traffic = json.load(open(tf)).get("w4a16_large_m")

    # --- small M (HBM bound): GB/s of algorithmic bytes, CUDA-graph replay, rotated weight copies ---
    small = {}
    if not args.no_small:
        copies = [weights] + [make_weights(dev, seed=3000 + 100 * c) for c in range(2)]
        for Ms in (1, 16):
            xsm = [synthetic.activations(Ms, K, seed=4000 + i).to(dev) for i, (_, K, _, _, _) in enumerate(weights)]
            outs = []

            def small_pass():
                for cp in copies:
                    for (_, K, N, p, s), x in zip(cp, xsm):
                        ops.gemm_w4a16(x, p, s, None, torch.bfloat16)
            # warm up on the capture stream so its split-K workspace exists before capture
            cs = torch.cuda.Stream(dev)
            cs.wait_stream(stream)
            with torch.cuda.stream(cs):
                small_pass()
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cs):
                small_pass()
            nbytes = 0
            for cp in copies:
                for (_, K, N, p, s) in cp:
                    nbytes += N * K // 2 + N * (K // 32) * s.element_size() + Ms * K * 2 + Ms * N * 2
            reps = 20
            ms = time_steps(g.replay, reps, 3, world, dev, stream) / reps
            ms = max_over_ranks(ms, world, dev)
            small[f"M{Ms}"] = {"GB_s": world * nbytes / (ms * 1e-3) / 1e9, "us_per_gemm": 1e3 * ms / (3 * len(weights)),
                               "frac_hbm": (nbytes / (ms * 1e-3) / 1e9) / pk["hbm_gbs"], "bytes_per_pass": nbytes,
                               "launches_per_pass": 3 * len(weights)}
            del g
        del copies

    # --- M <= 16 on N > 1 GPUs: output-channel split of each GEMM (one all-gather of y) ---
    tp = None
    if world > 1 and not args.no_small:
        import math
        import torch.distributed as dist
        from comfy_ui_gfx906_tools_b200 import parallel
        full_bytes = sum(N * K // 2 + N * (K // 32) * 2 for (_, K, N) in SHAPES)
        ncopy = max(3, math.ceil(3 * 126e6 * world / full_bytes))  # per-rank shards of all copies > 2x L2
        shard_sets = []
        for c in range(ncopy):
            cp = weights if c == 0 else make_weights(dev, seed=5000 + 100 * c)
            sh = []
            for (_, K, N, p, s) in cp:
                n0, n1 = parallel.channel_block(N, rank, world)
                sh.append((K, N, p[n0:n1].contiguous(), s[n0:n1].contiguous()))
            shard_sets.append(sh)
            del cp
        tp = {"copies": ncopy, "split": f"output channels / {world}, all_gather_into_tensor of y",
              "fused": "w4a16_gemm_allgather (epilogue stores into every rank's symmetric-memory y) + peer barrier"}
        sag = parallel.SymmetricAllGather(max(N for (_, _, N) in SHAPES), torch.bfloat16, dev)
        for Ms in (1, 16):
            xsm = [synthetic.activations(Ms, K, seed=4000 + i).to(dev).to(torch.bfloat16).contiguous()
                   for i, (_, K, _) in enumerate(SHAPES)]
            outs = [torch.empty(world * Ms, N // world, dtype=torch.bfloat16, device=dev) for (_, _, N) in SHAPES]

            def tp_pass():
                for sh in shard_sets:
                    for (K, N, p, s), x, o in zip(sh, xsm, outs):
                        y = ops.gemm_w4a16(x, p, s, None, torch.bfloat16)
                        dist.all_gather_into_tensor(o, y)

            def fused_pass():
                for sh in shard_sets:
                    for (K, N, p, s), x in zip(sh, xsm):
                        sag.gemm(x, p, s, None, N // world)
            reps = 5
            nbytes = ncopy * sum(N * K // 2 + N * (K // 32) * 2 + Ms * K * 2 + Ms * N * 2 for (_, K, N) in SHAPES)
            # the fused pass captured once in a CUDA graph (an even number of calls, so the
            # y buffers keep alternating between replays): the host launches one graph
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                fused_pass()
            torch.cuda.current_stream(dev).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                fused_pass()
            for key, fn in ((f"M{Ms}", tp_pass), (f"M{Ms}_fused", fused_pass), (f"M{Ms}_fused_graph", graph.replay)):
                ms = max_over_ranks(time_steps(fn, reps, 2, world, dev, stream) / reps, world, dev)
                tp[key] = {"GB_s": nbytes / (ms * 1e-3) / 1e9, "us_per_gemm": 1e3 * ms / (ncopy * len(SHAPES)),
                           "frac_hbm_aggregate": (nbytes / (ms * 1e-3) / 1e9) / (world * pk["hbm_gbs"])}
            del graph
        del shard_sets, sag

    # --- int8 weights (config 3): the six shapes at M=4608, per-channel fp16 scales ---
    int8 = None
    if not args.no_int8:
        w8 = []
        for i, (name, K, N, _, _) in enumerate(weights):
            q, sc = synthetic.int8_weight(N, K, seed=5000 + i)
            w8.append((q.to(dev), sc.to(dev)))

        def step8():
            for (q, sc), x in zip(w8, xs):
                ops.gemm_w8a16(x, q, sc, None, torch.bfloat16)
        ms8 = max_over_ranks(time_steps(step8, args.steps, args.warmup, world, dev, stream), world, dev)
        ms8 /= args.steps
        int8 = {"value": world * flops_step / (ms8 * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": ms8,
                "weights": "int8 ~round(N(0,40)) clipped to +-127, one fp16 scale per output channel",
                "frac_of_sustained_peak": (flops_step / (ms8 * 1e-3) / 1e12) / pk["bf16_tflops_sustained"]}
        del w8

    # --- e2e: public API with host buffers, H2D of x and D2H of y inside the timed region ---
    # (pinned host buffers; the copies of one step overlap its GEMMs and each other)
    e2e = None
    if not args.no_e2e:
        xh = [x.cpu().pin_memory() for x in xs]
        yh = [torch.empty(M, N, dtype=torch.bfloat16).pin_memory() for (_, K, N, _, _) in weights]
        xd = [torch.empty_like(x) for x in xs]

        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

        def e2e_step():
            # host->device copies on s_in, GEMMs on the launching stream, device->host on
            # s_out: copies of shape i+1 / i-1 overlap GEMM i and run in both PCIe directions
            s_in.wait_stream(stream)
            s_out.wait_stream(stream)
            landed = []
            with torch.cuda.stream(s_in):
                for i in range(len(weights)):
                    xd[i].copy_(xh[i], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(s_in)
                    landed.append(ev)
            for i, (_, K, N, p, s) in enumerate(weights):
                stream.wait_event(landed[i])
                y = ops.gemm_w4a16(xd[i], p, s, None, torch.bfloat16)
                done = torch.cuda.Event()
                done.record(stream)
                s_out.wait_event(done)
                y.record_stream(s_out)
                with torch.cuda.stream(s_out):
                    yh[i].copy_(y, non_blocking=True)
            stream.wait_stream(s_out)  # the step ends when the last result is on the host
        ms_e2e = max_over_ranks(time_steps(e2e_step, max(2, args.steps // 2), 2, world, dev, stream), world, dev)
        ms_e2e /= max(2, args.steps // 2)
        e2e = {"value": world * flops_step / (ms_e2e * 1e-3) / 1e12, "unit": UNIT,
               "h2d_bytes_per_step": sum(x.numel() * 2 for x in xs),
               "d2h_bytes_per_step": sum(M * N * 2 for (_, K, N, _, _) in weights), "ms_per_step": ms_e2e}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = len(os.sched_getaffinity(0))
        torch.set_num_threads(cores)
        best = None
        for _ in range(2):
            t_dq, t_mm, f, s = cpu_reference_sample(0, 256)
            best = s if best is None else min(best, s)
        cpu = {"value": f / best / 1e12, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": "qkv 3072x9216: torch-CPU dequant of the full weight + fp32 matmul of 256 of 4608 rows, "
                         "extrapolated to M=4608 (t_dequant + 18*t_matmul), best of 2"}

    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "flux_linear_sweep", "M": M, "shapes": [s[0] for s in SHAPES],
                       "weights": "int4 group-32, ggml Q4_0 synthetic (fp16-exact scales)",
                       "l2": "each step reads > 126 MB of distinct inputs (no flush needed)",
                       "clock_soak_s": 1.0,
                       "parallelism": f"replicas x{world} (per-GPU token block, no collective)"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "peak_kind": f"bf16 dense sustained ({pk['source']})",
                         "frac_of_burst": achieved / pk["bf16_tflops"], "traffic": traffic},
            "cpu_baseline": cpu, "e2e": e2e, "small_m": small, "int8": int8,
            **({"small_m_channel_split": tp} if tp is not None else {}),
            "gpu_launches": args.steps * len(weights), "clocks": clocks.summary(),
        }
        print(json.dumps(out))


def run_dit(args, world, rank, local):
    """Configs 4-5: the full Flux-architecture DiT forward (random int4
    weights), batch split or token-row split across the ranks."""
    from comfy_ui_gfx906_tools_b200 import flux_dit, ops, parallel
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    cfg = flux_dit.DiTConfig()
    model = flux_dit.FluxDiT(cfg, flux_dit.int4_linear_factory(dev, seed=11), dev)  # same seed: identical replicas
    side = args.res // 16
    split = args.split if world > 1 else "none"
    batch = args.batch if args.batch else (8 if split == "batch" else 1)
    inputs = flux_dit.make_inputs(cfg, batch, side, side, 512, dev, seed=12)
    macs = {"n": 0}

    def count(mod, inp, out):
        macs["n"] += inp[0].numel() // inp[0].shape[-1] * mod.in_features * mod.out_features
    hooks = [m.register_forward_hook(count) for m in model.modules() if isinstance(m, ops.Gfx906Int4Ops.Linear)]

    def fwd():
        with torch.no_grad():
            if split == "batch":
                return parallel.split_forward_batch(model, *inputs, gather_output=False)
            if split == "rows":
                return parallel.split_forward_rows(model, *inputs, side, side, gather_output=False)
            return model(*inputs)
    fwd()
    torch.cuda.synchronize(dev)
    linear_flop = 2.0 * macs["n"]  # this rank's int4-linear work per forward
    for h in hooks:
        h.remove()
    ms = max_over_ranks(time_steps(fwd, args.steps, args.warmup, world, dev, stream), world, dev) / args.steps
    tokens = batch * (side * side + 512)
    if rank == 0:
        print(json.dumps({
            "metric": "Flux DiT forward tokens/s (int4 linears)", "value": tokens / (ms * 1e-3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random int4 weights)",
            "config": {"workload": f"flux_dit_{args.res}", "batch": batch, "image_tokens": side * side,
                       "text_tokens": 512, "split": split, "blocks": "19 double + 38 single, hidden 3072"},
            "linear_tflops_per_gpu": linear_flop / (ms * 1e-3) / 1e12,
        }))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--m", type=int, default=4608)
    ap.add_argument("--no-small", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-int8", action="store_true")
    ap.add_argument("--workload", choices=["gemm", "dit"], default="gemm")
    ap.add_argument("--res", type=int, default=1024, help="dit: latent resolution in pixels (1024 or 2048)")
    ap.add_argument("--split", choices=["batch", "rows"], default="batch", help="dit: how N > 1 ranks split")
    ap.add_argument("--batch", type=int, default=0, help="dit: batch (default 8 for the batch split, else 1)")
    args = ap.parse_args()
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = setup_dist(args.gpus)
    try:
        if args.workload == "dit":
            run_dit(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
