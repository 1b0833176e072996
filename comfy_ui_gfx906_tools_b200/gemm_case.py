"""Run and time one W4A16 GEMM case (used for ncu captures and quick timing).

    python -m comfy_ui_gfx906_tools_b200.gemm_case --shape qkv --m 4608 [--reps 20] [--graph]
    python -m comfy_ui_gfx906_tools_b200.gemm_case --n 128 --k 256 --m 1 --graph   (any N, K)

Weights are the synthetic Q4_0 weights of the benchmark (fp16-exact scales,
used through an fp16 scale copy as Gfx906Int4Ops.Linear does), activations
bf16 N(0, 1). Prints one JSON line with the CUDA-event time per GEMM and the
algorithmic TFLOP/s and GB/s (bytes = N*K/2 + N*K/32*scale_bytes + 2*M*K + 2*M*N).
"""
from __future__ import annotations

import argparse
import json

import torch

from . import ops, synthetic

SHAPES = {name: (K, N) for name, K, N in synthetic.FLUX_SHAPES}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", default="qkv", choices=sorted(SHAPES))
    ap.add_argument("--n", type=int, default=0, help="custom N (with --k) instead of a named shape")
    ap.add_argument("--k", type=int, default=0)
    ap.add_argument("--m", type=int, default=4608)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--copies", type=int, default=1, help="distinct weight copies cycled through (defeats L2)")
    ap.add_argument("--fp32-scales", action="store_true")
    ap.add_argument("--splits", type=int, default=0, help="explicit split count (0 = automatic)")
    ap.add_argument("--graph", action="store_true", help="time a CUDA graph of the reps (launch-bound cases)")
    a = ap.parse_args()
    K, N = (a.k, a.n) if a.n and a.k else SHAPES[a.shape]
    if a.n and a.k:
        a.shape = f"{N}x{K}"
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ws = []
    for c in range(a.copies):
        raw, _, _ = synthetic.q4_0_weight(N, K, seed=10 + c)
        p, s = ops.repack_q4_0_native(raw.to(dev), N, K)
        if not a.fp32_scales:
            s = ops.scales_to_f16_if_exact(s)
        ws.append((p, s))
    x = synthetic.activations(a.m, K, seed=1).to(dev)
    stream = torch.cuda.Stream(dev)

    def run():
        for i in range(a.reps):
            p, s = ws[i % a.copies]
            ops.gemm_w4a16(x, p, s, None, torch.bfloat16, splits=a.splits)

    with torch.cuda.stream(stream):
        run()  # warm-up (also creates this stream's split-K workspace)
        torch.cuda.synchronize(dev)
        fn = run
        if a.graph:
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
    us = 1e3 * e0.elapsed_time(e1) / a.reps
    sb = ws[0][1].element_size()
    nbytes = N * K // 2 + N * (K // 32) * sb + 2 * a.m * K + 2 * a.m * N
    print(json.dumps({"shape": a.shape, "M": a.m, "N": N, "K": K, "us": us, "tflops": 2 * a.m * N * K / us / 1e6,
                      "GB_s": nbytes / us / 1e3, "scale_bytes": sb, "graph": a.graph, "copies": a.copies,
                      "splits": a.splits}))


if __name__ == "__main__":
    main()
