"""Benchmark of the int4 W4A16 linear path on B200 (driver contract: one JSON line).

Workload (config 2, "flux_linear_sweep"): one step = the six Flux DiT linear
shapes at hidden 3072 ((K, N) in qkv 3072x9216, proj 3072x3072, mlp-up
3072x12288, mlp-down 12288x3072, single-fused 3072x21504, single-out
15360x3072), M = 4608 tokens each, bf16 activations, int4 group-32 weights
from synthetic ggml Q4_0 blocks, bf16 output. metric = whole-job TFLOP/s
(2*M*N*K per GEMM). Each step reads > 126 MB (L2) of distinct inputs, so the
timed loop does not run out of L2.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python bench.py --case qkv --m 1 [--reps 20] [--graph] [--copies 3]   (one GEMM shape, for ncu / quick timing)
  python bench.py --attention-case int4/u8 [--tokens 4608] [--heads 24]  (one fused-attention shape)

N = 1: the whole 4608-token sweep on one GPU. N > 1 (torchrun, one rank per
GPU, NCCL): the same fixed workload split by token rows (rank r computes rows
[r*M/N, (r+1)*M/N) of every GEMM, weights replicated) with one
all_gather_into_tensor of each GEMM's output inside the timed region,
overlapped with the next GEMM (strong scaling); timing is the max over ranks
of CUDA-event time, and a "parity" key compares the gathered output with the
same GEMMs run whole on one GPU and with a torch fp32 dequant-then-matmul.
The M in {1, 16} variants of the same weights are reported as GB/s of
algorithmic bytes in "small_m" (output-channel split at N > 1), the int8
config-3 sweep in "int8", the row-split DiT forward (config 5) in "dit_rows".
--impl reference times the reference's CPU torch path (dequant + fp32 matmul,
the oracle's torch port) on this host's cores, full size.
"""
from __future__ import annotations

import argparse
import json
import os
import platform
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
M_FULL = 4608


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def workload_config(world: int) -> dict:
    """The `config` of both arms' JSON lines (identical for a given N)."""
    return {"workload": "flux_linear_sweep", "M": M_FULL, "shapes": [s[0] for s in SHAPES],
            "weights": "int4 group-32, ggml Q4_0 synthetic (fp16-exact scales)",
            "l2": "each step reads > 126 MB of distinct inputs (no flush needed)",
            "parallelism": ("single GPU" if world == 1 else
                            f"token rows / {world} (weights replicated), y all-gathered to every rank inside the "
                            "timed region")}


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


def setup_dist():
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


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


# ---------------------------------------------------------------------------
# the reference's CPU torch path (the oracle's torch port), full size
# ---------------------------------------------------------------------------
def cpu_reference_inputs(seed=0):
    """Native int4 weights of the six shapes (the reference's own repack of the
    same synthetic Q4_0 blocks) and the M=4608 activations, on the CPU."""
    import oracle as O
    from comfy_ui_gfx906_tools_b200 import synthetic
    out = []
    for i, (name, K, N) in enumerate(SHAPES):
        raw, _, _ = synthetic.q4_0_weight(N, K, seed=seed + i)
        p, s = O.repack_q4_0_native(raw.numpy(), N, K)
        x = synthetic.activations(M_FULL, K, seed=seed + 50 + i)
        out.append((name, K, N, torch.from_numpy(p), torch.from_numpy(s), x))
    return out


def cpu_reference_step(inputs, M=M_FULL):
    """One full sweep of the reference CPU path: per shape the torch dequant
    (int4_train_test.py:46-52) then the fp32 matmul of M rows (bench_int8.py:43),
    timed separately. Returns {shape: (t_dequant, t_matmul)}."""
    import oracle as O
    times = {}
    for name, K, N, p, s, x in inputs:
        xf = x[:M].float()
        t0 = time.perf_counter()
        w = O.torch_cpu_dequant(p, s)
        t1 = time.perf_counter()
        y = torch.matmul(xf, w.t())
        t2 = time.perf_counter()
        del y, w
        times[name] = (t1 - t0, t2 - t1)
    return times


def cpu_baseline_best_of(reps=3):
    """cpu_baseline: the six shapes at M=4608, dequant and matmul timed
    separately, best of `reps` per shape and phase; plus M in {1, 16} as GB/s."""
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    inputs = cpu_reference_inputs()
    best = {}
    for _ in range(reps):
        for name, (tdq, tmm) in cpu_reference_step(inputs).items():
            b = best.get(name, (float("inf"), float("inf")))
            best[name] = (min(b[0], tdq), min(b[1], tmm))
    flops = sum(2.0 * M_FULL * N * K for (_, K, N) in SHAPES)
    t_total = sum(a + b for a, b in best.values())
    small = {}
    for Ms in (1, 16):
        bs = {}
        for _ in range(reps):
            for name, (tdq, tmm) in cpu_reference_step(inputs, Ms).items():
                bs[name] = min(bs.get(name, float("inf")), tdq + tmm)
        nbytes = sum(N * K // 2 + N * (K // 32) * 4 + Ms * K * 2 + Ms * N * 2 for (_, K, N) in SHAPES)
        small[f"M{Ms}"] = {"GB_s": nbytes / sum(bs.values()) / 1e9, "s_per_sweep": sum(bs.values())}
    return {"value": flops / t_total / 1e12, "unit": UNIT, "cores": cores, "kind": "port",
            "cpu_model": cpu_model(),
            "sample": "the full workload: six Flux shapes at M=4608, torch-CPU dequant of each weight and fp32 "
                      f"matmul timed separately, best of {reps} per shape and phase (no extrapolation)",
            "per_shape_s": {k: {"dequant": v[0], "matmul": v[1]} for k, v in best.items()},
            "dequant_s": sum(v[0] for v in best.values()), "matmul_s": sum(v[1] for v in best.values()),
            "small_m": small}


def run_reference(args, world, rank):
    """--impl reference: the reference CPU path on the whole workload, one full
    six-shape sweep at M=4608 per step, on rank 0 only."""
    if rank != 0:
        return
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    inputs = cpu_reference_inputs()
    flops = sum(2.0 * M_FULL * N * K for (_, K, N) in SHAPES)
    for _ in range(args.warmup):
        cpu_reference_step(inputs)
    secs = 0.0
    dq = mm = 0.0
    for _ in range(args.steps):
        t = cpu_reference_step(inputs)
        secs += sum(a + b for a, b in t.values())
        dq += sum(a for a, _ in t.values())
        mm += sum(b for _, b in t.values())
    value = args.steps * flops / secs / 1e12
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * secs / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "cpu_model": cpu_model(),
                         "sample": "each step the full workload: six Flux shapes at M=4608, torch-CPU dequant + "
                                   "fp32 matmul (the reference's CPU torch path), no extrapolation",
                         "dequant_s_per_step": dq / args.steps, "matmul_s_per_step": mm / args.steps},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
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


def time_steps(fn, steps, warmup, world, dev, stream, soak_s=0.0, on_step=None):
    """Device time of `steps` back-to-back calls of fn (CUDA events on the
    launching stream, barrier + synchronize on both sides). on_step(k), when
    given, is called before timed step k (k = -1 for warm-up and soak)."""
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
    for k in range(steps):
        if on_step is not None:
            on_step(k)
        fn()
    b.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    if on_step is not None:
        on_step(-1)
    return a.elapsed_time(b)


def parity_of(got: torch.Tensor, ref: torch.Tensor) -> dict:
    d = (got.double() - ref.double()).abs()
    r = ref.double().abs()
    return {"max_abs_over_max_ref": float(d.max() / r.max()), "mean_rel": float(d.mean() / r.mean()),
            "nonfinite": int((~torch.isfinite(got)).sum())}


def torch_reference_rows(x, p, s, rows):
    """fp32 dequant-then-matmul of the sampled rows in torch on the GPU (the
    bit-exact dequant kernel, then a plain fp32 matmul)."""
    from comfy_ui_gfx906_tools_b200 import ops
    w = ops.dequantize_int4(p, s, torch.float32)
    return x[rows].float() @ w.t()


def run_ours(args, world, rank, local):
    from comfy_ui_gfx906_tools_b200 import ops, synthetic
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    pk = peaks()
    M = M_FULL
    per = M // world
    r0 = rank * per
    weights = make_weights(dev, seed=1000)
    xs = [synthetic.activations(M, K, seed=2000 + i).to(dev) for i, (_, K, _, _, _) in enumerate(weights)]
    xloc = [x[r0:r0 + per].contiguous() for x in xs]
    flops_step = sum(2.0 * M * N * K for (_, K, N, _, _) in weights)
    dist = None
    if world > 1:
        import torch.distributed as dist
    yfull = [torch.empty(M, N, dtype=torch.bfloat16, device=dev) for (_, _, N, _, _) in weights] if world > 1 else None
    # N > 1: all_gather_into_tensor of each GEMM's rows on NCCL's stream, overlapped with the next GEMM;
    # --fused-gather: each GEMM's epilogue stores its rows into every rank's y (symmetric memory over NVLink),
    # then a flag barrier (measured slower at N = 2: 1.95 vs 1.57 ms per step)
    gather = None
    if world > 1 and args.fused_gather:
        from comfy_ui_gfx906_tools_b200.parallel import SymmetricRowGather
        gather = SymmetricRowGather(M, max(N for (_, _, N, _, _) in weights), torch.bfloat16, dev)

    # --- device-resident timed loop ---
    # per-launch CUDA events inside the timed region itself (same clocks and
    # back-to-back regime as the step time; one event pair per launch)
    ev = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in weights] for _ in range(args.steps)]
    record = {"k": -1}

    def on_step(k):
        record["k"] = k

    def step():
        works = []
        k = record["k"]
        for i, ((_, K, N, p, s), x) in enumerate(zip(weights, xloc)):
            if k >= 0:
                ev[k][i][0].record(stream)
            if gather is not None:  # GEMM + all-gather in one kernel, then the flag barrier
                gather.gemm(x, p, s, None, r0, M)
            else:
                y = ops.gemm_w4a16(x, p, s, None, torch.bfloat16)
            if k >= 0:
                ev[k][i][1].record(stream)
            if world > 1 and gather is None:  # this GEMM's rows to every rank, overlapped with the next GEMM
                works.append(dist.all_gather_into_tensor(yfull[i], y, async_op=True))
        for w in works:
            w.wait()

    clocks = ClockSampler(dev.index)
    with clocks:
        ms_total = time_steps(step, args.steps, args.warmup, world, dev, stream, soak_s=1.0, on_step=on_step)
    ms_total = max_over_ranks(ms_total, world, dev)
    ms_step = ms_total / args.steps
    value = flops_step / (ms_step * 1e-3) / 1e12
    launch_ms = [sum(ev[k][i][0].elapsed_time(ev[k][i][1]) for k in range(args.steps)) for i in range(len(weights))]
    avg_launch_ms = sum(launch_ms) / (args.steps * len(weights))
    achieved = (flops_step / world / len(weights)) / (avg_launch_ms * 1e-3) / 1e12
    traffic = None
    tf = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tf):
        traffic = json.load(open(tf)).get("w4a16_large_m")

    # --- parity of the timed step's output: sampled rows against a torch fp32
    # dequant-then-matmul, and (N > 1) the gathered rows against the whole
    # GEMM on one GPU ---
    parity = {}
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(5))[:64].sort().values.to(dev)
    for i, ((name, K, N, p, s), x) in enumerate(zip(weights, xs)):
        if gather is not None:
            y = gather.gemm(xloc[i], p, s, None, r0, M).clone()
        else:
            y = yfull[i] if world > 1 else ops.gemm_w4a16(x, p, s, None, torch.bfloat16)
        ent = parity_of(y[rows].float(), torch_reference_rows(x, p, s, rows))
        if world > 1:
            whole = ops.gemm_w4a16(x, p, s, None, torch.bfloat16)
            ent["vs_one_gpu"] = parity_of(y.float(), whole.float())
            ent["bit_identical_to_one_gpu"] = bool(torch.equal(y, whole))
            del whole
        parity[name] = ent
    parity_ok = all(e["max_abs_over_max_ref"] <= 2e-2 and e["mean_rel"] <= 5e-3 and e["nonfinite"] == 0
                    for e in parity.values())

    # --- small M (HBM bound): GB/s of algorithmic bytes, CUDA-graph replay, rotated weight copies ---
    small = {}
    if not args.no_small and world == 1:
        copies = [weights] + [make_weights(dev, seed=3000 + 100 * c) for c in range(2)]
        for Ms in (1, 16):
            xsm = [synthetic.activations(Ms, K, seed=4000 + i).to(dev) for i, (_, K, _, _, _) in enumerate(weights)]

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
            small[f"M{Ms}"] = {"GB_s": nbytes / (ms * 1e-3) / 1e9, "us_per_gemm": 1e3 * ms / (3 * len(weights)),
                               "frac_hbm": (nbytes / (ms * 1e-3) / 1e9) / pk["hbm_gbs"], "bytes_per_pass": nbytes,
                               "launches_per_pass": 3 * len(weights)}
            del g
        del copies

    # --- M <= 16 on N > 1 GPUs: output-channel split of each GEMM (one all-gather of y) ---
    tp = None
    if world > 1 and not args.no_small:
        tp = run_channel_split(args, world, rank, dev, stream, weights, pk)

    # --- int8 weights (config 3): the six shapes at M=4608, per-channel fp16 scales ---
    int8 = None
    if not args.no_int8 and world == 1:
        w8 = []
        for i, (name, K, N, _, _) in enumerate(weights):
            q, sc = synthetic.int8_weight(N, K, seed=5000 + i)
            w8.append((q.to(dev), sc.to(dev)))

        def step8():
            for (q, sc), x in zip(w8, xs):
                ops.gemm_w8a16(x, q, sc, None, torch.bfloat16)
        ms8 = time_steps(step8, args.steps, args.warmup, world, dev, stream) / args.steps
        int8 = {"value": flops_step / (ms8 * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": ms8,
                "weights": "int8 ~round(N(0,40)) clipped to +-127, one fp16 scale per output channel",
                "frac_of_burst_peak": (flops_step / (ms8 * 1e-3) / 1e12) / pk["bf16_tflops"]}
        del w8

    # --- the reference's own W4A4 numerics (gemm_int4, integer-exact, bit-identical to the
    # reference's kernel; tests/test_w4a4_exact_gpu.py): the six shapes at M=4608 on int4
    # activations from quantize_int4 and the same packed weights with fp32 scales ---
    w4a4 = None
    if not args.no_int8 and world == 1:
        xq = [ops.quantize_int4(x) for x in xs]
        w32 = [(p, s.float()) for (_, _, _, p, s) in weights]

        def step4():
            for (a, sa), (p, s) in zip(xq, w32):
                ops.gemm_int4(a, sa, p, s, None, torch.bfloat16)
        ms4 = time_steps(step4, args.steps, args.warmup, world, dev, stream) / args.steps
        w4a4 = {"value": flops_step / (ms4 * 1e-3) / 1e12, "unit": "TOPS (int4 x int4, 2*M*N*K)", "ms_per_step": ms4,
                "numerics": "bit-identical to the reference's int4_gemm_kernel (integer block dots on tcgen05 "
                            "kind::f8f6f4, the reference's fp32 chain and split plan)",
                "includes": "per call: e5m2 pre-pass of A, scale transpose, the GEMM"}
        del xq, w32

    # --- the fused quantized attention (the reference's attention.hip; tests/test_attention_gpu.py):
    # Flux 1024^2 attention, batch 1, 24 heads, 4096 image + 512 text tokens, head dim 128, on inputs
    # prepared once (the kernel alone), with torch's SDPA on the same fp16 q / k / v for context ---
    attn = None
    if not args.no_attention and world == 1:
        from comfy_ui_gfx906_tools_b200 import attention as fa
        La, Ha = 4608, 24
        ga = torch.Generator(device=dev).manual_seed(77)
        qa, ka, va = (torch.randn(1, Ha, La, 128, device=dev, dtype=torch.float16, generator=ga) for _ in range(3))
        flop_a = 4.0 * La * La * 128 * Ha
        attn = {"unit": "TFLOP/s (4 * L^2 * 128 * heads)", "shape": {"batch": 1, "heads": Ha, "tokens": La},
                "inputs": "prepared once, L2-resident (a compute-bound kernel)", "modes": {}}
        for qk, pv in (("int4", "u8"), ("int8", "u8"), ("int8", "fp16"), ("fp16", "fp16")):
            prep = (*fa.prepare_qk(qa, ka, qk), *fa.prepare_v(va, pv))
            msa = time_steps(lambda: fa.attention_prepared(*prep, qk, pv, 1e-4), args.steps, args.warmup, world, dev,
                             stream) / args.steps
            attn["modes"][f"{qk}/{pv}"] = {"ms": msa, "value": flop_a / (msa * 1e-3) / 1e12,
                                          "kernel": "attention_tc_kernel (tcgen05)"}
            del prep
        mss = time_steps(lambda: torch.nn.functional.scaled_dot_product_attention(qa, ka, va), args.steps,
                         args.warmup, world, dev, stream) / args.steps
        attn["torch_sdpa_fp16"] = {"ms": mss, "value": flop_a / (mss * 1e-3) / 1e12}
        del qa, ka, va

    # --- e2e: public API with host buffers, H2D of x and D2H of y inside the timed region ---
    # (pinned host buffers; the copies of one step overlap its GEMMs and each other)
    e2e = None
    if not args.no_e2e:
        xh = [x.cpu().pin_memory() for x in xloc]
        yh = [torch.empty(M if world > 1 else per, N, dtype=torch.bfloat16).pin_memory()
              for (_, K, N, _, _) in weights]
        xd = [torch.empty_like(x) for x in xloc]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

        def e2e_step():
            # host->device copies on s_in, GEMMs (and the all-gathers) on the launching
            # stream, device->host on s_out: the copies of shape i+1 / i-1 overlap GEMM i
            s_in.wait_stream(stream)
            s_out.wait_stream(stream)
            landed = []
            with torch.cuda.stream(s_in):
                for i in range(len(weights)):
                    xd[i].copy_(xh[i], non_blocking=True)
                    ev_ = torch.cuda.Event()
                    ev_.record(s_in)
                    landed.append(ev_)
            for i, (_, K, N, p, s) in enumerate(weights):
                stream.wait_event(landed[i])
                y = ops.gemm_w4a16(xd[i], p, s, None, torch.bfloat16)
                if world > 1:
                    dist.all_gather_into_tensor(yfull[i], y)
                    y = yfull[i]
                done = torch.cuda.Event()
                done.record(stream)
                s_out.wait_event(done)
                y.record_stream(s_out)
                with torch.cuda.stream(s_out):
                    yh[i].copy_(y, non_blocking=True)
            stream.wait_stream(s_out)  # the step ends when the last result is on the host
        n_e2e = max(2, args.steps // 2)
        ms_e2e = max_over_ranks(time_steps(e2e_step, n_e2e, 2, world, dev, stream), world, dev) / n_e2e
        e2e = {"value": flops_step / (ms_e2e * 1e-3) / 1e12, "unit": UNIT,
               "h2d_bytes_per_step": sum(x.numel() * 2 for x in xloc),
               "d2h_bytes_per_step": sum(y.numel() * 2 for y in yh), "ms_per_step": ms_e2e}

    # --- config 5 at N GPUs: the 2048^2 DiT forward, token rows split across the ranks ---
    dit = None
    if not args.no_dit:
        dit = run_dit_rows(world, rank, dev, stream, steps=2, warmup=1)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline_best_of(3)

    if rank == 0:
        peak = pk["bf16_tflops"]
        out = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload_config(world),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak,
                         "peak_kind": f"bf16 dense burst ({pk['source']}): the 20-step timed loop is ~45 ms",
                         "frac_of_sustained": achieved / pk["bf16_tflops_sustained"],
                         "step_frac": (value / world) / peak, "traffic": traffic,
                         "kernel": ("wq_tc_kernel<1, bf16, 1, false> (tcgen05), mean over the six shapes' launches" +
                                    ("; with the fused all-gather, each launch's time includes its peer stores "
                                     "and the flag barrier" if gather is not None else "")),
                         "launch_ms": {weights[i][0]: launch_ms[i] / args.steps for i in range(len(weights))}},
            "parity": {"ok": parity_ok, "rows_sampled": 64, "per_shape": parity,
                       "reference": "torch fp32 dequant-then-matmul of the sampled rows (north-star tolerance "
                                    "2e-2 max-abs ratio, 5e-3 mean relative error)"},
            "cpu_baseline": cpu, "e2e": e2e, "small_m": small, "int8": int8, "w4a4_exact": w4a4,
            **({"attention": attn} if attn is not None else {}),
            **({"small_m_channel_split": tp} if tp is not None else {}),
            **({"dit_rows": dit} if dit is not None else {}),
            **({"allgather": ("fused: each GEMM's epilogue stores its rows into every rank's y (symmetric memory, "
                              "NVLink peer stores), then a flag barrier kernel" if gather is not None else
                              "NCCL all_gather_into_tensor per GEMM, async on NCCL's stream")} if world > 1 else {}),
            "gpu_launches": args.steps * len(weights), "clocks": clocks.summary(),
        }
        print(json.dumps(out))


def run_channel_split(args, world, rank, dev, stream, weights, pk):
    """M in {1, 16} at N > 1: each rank streams N/G of every weight's rows;
    GEMM + NCCL all-gather, and the fused kernel (peer stores + flag barrier)."""
    import math
    import torch.distributed as dist
    from comfy_ui_gfx906_tools_b200 import ops, parallel, synthetic
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
    return tp


def run_dit_rows(world, rank, dev, stream, steps, warmup, res=2048):
    """Config 5: the full Flux-architecture DiT forward at res^2 (random int4
    weights), token rows split across the ranks (one image-K/V all-gather per
    attention); tokens/s over the ranks, max-over-ranks CUDA-event time."""
    from comfy_ui_gfx906_tools_b200 import flux_dit, parallel
    cfg = flux_dit.DiTConfig()
    model = flux_dit.FluxDiT(cfg, flux_dit.int4_linear_factory(dev, seed=11), dev)  # same seed: identical replicas
    side = res // 16
    inputs = flux_dit.make_inputs(cfg, 1, side, side, 512, dev, seed=12)

    def fwd():
        with torch.no_grad():
            if world > 1:
                return parallel.split_forward_rows(model, *inputs, side, side, gather_output=False)
            return model(*inputs)
    ms = max_over_ranks(time_steps(fwd, steps, warmup, world, dev, stream), world, dev) / steps
    tokens = side * side + 512
    del model
    torch.cuda.empty_cache()
    return {"metric": "Flux DiT forward tokens/s (int4 linears)", "value": tokens / (ms * 1e-3), "unit": "tokens/s",
            "ms_per_forward": ms, "steps": steps, "warmup": warmup,
            "config": {"workload": f"flux_dit_{res}", "batch": 1, "image_tokens": side * side, "text_tokens": 512,
                       "split": "token rows" if world > 1 else "none",
                       "blocks": "19 double + 38 single, hidden 3072"}}


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


def run_attention_case(args):
    """One fused-attention shape on cuda:0 (the command the attention ncu
    summary under profiles/ profiles): batch 1, --heads heads, --tokens keys
    and queries, seeded N(0, 1) fp16 q / k / v prepared once; prints the time
    per call and TFLOP/s (4 * L^2 * 128 * heads)."""
    from comfy_ui_gfx906_tools_b200 import attention as fa
    qk, pv = args.attention_case.split("/")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L, Hh = args.tokens, args.heads
    g = torch.Generator(device=dev).manual_seed(77)
    q, k, v = (torch.randn(1, Hh, L, 128, device=dev, dtype=torch.float16, generator=g) for _ in range(3))
    prep = (*fa.prepare_qk(q, k, qk), *fa.prepare_v(v, pv))
    for _ in range(2):
        fa.attention_prepared(*prep, qk, pv, args.skip_below)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.reps):
        fa.attention_prepared(*prep, qk, pv, args.skip_below)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.reps
    print(json.dumps({"attention": f"{qk}/{pv}", "tokens": L, "heads": Hh, "ms": ms,
                      "tflops": 4.0 * L * L * 128 * Hh / (ms * 1e-3) / 1e12, "skip_below": args.skip_below}))


def run_case(args):
    """One GEMM shape on cuda:0, timed with CUDA events (the command the ncu
    summaries under profiles/ profile): synthetic Q4_0 weights used through
    their fp16 scale copy as Gfx906Int4Ops.Linear does, activations bf16
    N(0, 1); prints the time per GEMM, TFLOP/s and GB/s of algorithmic bytes
    (N*K/2 + N*K/32*scale_bytes + 2*M*K + 2*M*N)."""
    from comfy_ui_gfx906_tools_b200 import ops, synthetic
    shapes = {name: (K, N) for name, K, N in SHAPES}
    K, N = (args.k, args.n) if args.n and args.k else shapes[args.case]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ws = []
    for c in range(args.copies):
        raw, _, _ = synthetic.q4_0_weight(N, K, seed=10 + c)
        p, s = ops.repack_q4_0_native(raw.to(dev), N, K)
        if not args.fp32_scales:
            s = ops.scales_to_f16_if_exact(s)
        ws.append((p, s))
    x = synthetic.activations(args.m, K, seed=1).to(dev)
    stream = torch.cuda.Stream(dev)
    if args.w4a4:  # the integer-exact W4A4 GEMM: int4 activations from quantize_int4, fp32 weight scales
        xa, xs = ops.quantize_int4(x)
        ws = [(p, s.float()) for p, s in ws]

    def run():
        for i in range(args.reps):
            p, s = ws[i % args.copies]
            if args.w4a4:
                ops.gemm_int4(xa, xs, p, s, None, torch.bfloat16, splits=args.splits)
            elif args.int8:
                ops.gemm_w8a16(x, p8[i % args.copies][0], p8[i % args.copies][1], None, torch.bfloat16)
            else:
                ops.gemm_w4a16(x, p, s, None, torch.bfloat16, splits=args.splits)

    p8 = [tuple(t.to(dev) for t in synthetic.int8_weight(N, K, seed=20 + c)) for c in range(args.copies)] \
        if args.int8 else None
    with torch.cuda.stream(stream):
        run()  # warm-up (also creates this stream's split-K workspace)
        torch.cuda.synchronize(dev)
        fn = run
        if args.graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                run()
            fn = g.replay
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
    us = 1e3 * e0.elapsed_time(e1) / args.reps
    sb = 2 if args.int8 else ws[0][1].element_size()
    if args.w4a4:  # packed A + its fp32 scales instead of bf16 x
        nbytes = N * K // 2 + N * (K // 32) * 4 + args.m * K // 2 + args.m * (K // 32) * 4 + 2 * args.m * N
        print(json.dumps({"case": args.case if not (args.n and args.k) else f"{N}x{K}", "M": args.m, "N": N, "K": K,
                          "us": 1e3 * e0.elapsed_time(e1) / args.reps, "w4a4_exact": True,
                          "tops": 2 * args.m * N * K / (1e3 * e0.elapsed_time(e1) / args.reps) / 1e6,
                          "GB_s": nbytes / (1e3 * e0.elapsed_time(e1) / args.reps) / 1e3, "graph": args.graph,
                          "copies": args.copies, "splits": args.splits}))
        return
    wbytes = N * K if args.int8 else N * K // 2 + N * (K // 32) * sb
    nbytes = wbytes + 2 * args.m * K + 2 * args.m * N
    print(json.dumps({"case": args.case if not (args.n and args.k) else f"{N}x{K}", "M": args.m, "N": N, "K": K,
                      "us": us, "tflops": 2 * args.m * N * K / us / 1e6, "GB_s": nbytes / us / 1e3,
                      "graph": args.graph, "copies": args.copies, "splits": args.splits, "int8": args.int8}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-small", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-int8", action="store_true")
    ap.add_argument("--no-dit", action="store_true")
    ap.add_argument("--no-attention", action="store_true")
    ap.add_argument("--fused-gather", action="store_true",
                    help="N > 1: all-gather y from the GEMM's own epilogue (peer stores + flag barrier) instead of "
                         "NCCL after each GEMM")
    ap.add_argument("--workload", choices=["gemm", "dit"], default="gemm")
    ap.add_argument("--res", type=int, default=1024, help="dit: latent resolution in pixels (1024 or 2048)")
    ap.add_argument("--split", choices=["batch", "rows"], default="batch", help="dit: how N > 1 ranks split")
    ap.add_argument("--batch", type=int, default=0, help="dit: batch (default 8 for the batch split, else 1)")
    ap.add_argument("--case", default=None, choices=[s[0] for s in SHAPES] + ["custom"],
                    help="time one GEMM shape instead of the bench (with --m, --reps, --graph, --copies)")
    ap.add_argument("--m", type=int, default=M_FULL)
    ap.add_argument("--n", type=int, default=0, help="case custom: N (with --k)")
    ap.add_argument("--k", type=int, default=0)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--copies", type=int, default=1, help="case: distinct weight copies cycled through (defeats L2)")
    ap.add_argument("--fp32-scales", action="store_true")
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--graph", action="store_true", help="case: time a CUDA graph of the reps")
    ap.add_argument("--w4a4", action="store_true",
                    help="case: the integer-exact W4A4 GEMM (gemm_int4) on quantize_int4 activations")
    ap.add_argument("--int8", action="store_true", help="case: the int8 (W8A16) kernel, per-channel scales")
    ap.add_argument("--attention-case", default=None,
                    choices=[f"{a}/{b}" for a in ("fp16", "int8", "int4") for b in ("fp16", "u8")],
                    help="time one fused-attention shape (with --tokens, --heads, --reps, --skip-below)")
    ap.add_argument("--tokens", type=int, default=4608)
    ap.add_argument("--heads", type=int, default=24)
    ap.add_argument("--skip-below", type=float, default=0.0)
    args = ap.parse_args()
    if args.attention_case is not None:
        run_attention_case(args)
        return
    if args.case is not None:
        run_case(args)
        return
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = setup_dist()
    if args.workload == "gemm" and M_FULL % world != 0:
        raise SystemExit(f"--gpus {world} must divide M={M_FULL}")
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
