"""Build oracle/_ref/libgfx906_ref.so: the reference's own int4 / int8 GEMM and
quantizer kernels (nodes/ComfyUI-Gfx906Int4/csrc/int4_gemm_scaled.hip and
int8_gemm.hip), compiled where they lie under the reference checkout with
nvcc for sm_100a against the HIP stand-in headers in oracle/hip_shim/, plus
the C entry points of oracle/ref_kernels.cu. TEST INFRASTRUCTURE ONLY.

    python oracle/build_ref.py [--reference PATH]

Does nothing when the reference checkout is absent (the GPU box runs the
prebuilt library, which travels with the repository snapshot). No reference
source is copied: the .hip files are compiled in place, outputs go to
oracle/_ref/ only.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT_DIR, "libgfx906_ref.so")
DEFAULT_REF = "/root/reference"
SOURCES = ("nodes/ComfyUI-Gfx906Int4/csrc/int4_gemm_scaled.hip", "nodes/ComfyUI-Gfx906Int4/csrc/int8_gemm.hip",
           "nodes/ComfyUI-Gfx906Int4/csrc/int4_train_quant.hip")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17", "-Xcompiler", "-fPIC",
         "-I", os.path.join(HERE, "hip_shim")]


def nvcc() -> str:
    return os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")


def build(reference: str = DEFAULT_REF, force: bool = False) -> str | None:
    srcs = [os.path.join(reference, s) for s in SOURCES]
    if not all(os.path.exists(s) for s in srcs):
        return LIB if os.path.exists(LIB) else None
    deps = srcs + [os.path.join(HERE, "ref_kernels.cu"), os.path.abspath(__file__)] + [
        os.path.join(HERE, "hip_shim", "hip", f) for f in ("hip_runtime.h", "hip_fp16.h", "hip_bf16.h")]
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(d) for d in deps):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    objs = []
    for src in srcs + [os.path.join(HERE, "ref_kernels.cu")]:
        obj = os.path.join(OUT_DIR, os.path.basename(src).rsplit(".", 1)[0] + ".o")
        cmd = [nvcc(), "-x", "cu", *FLAGS, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        objs.append(obj)
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", LIB + ".tmp", *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=DEFAULT_REF)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.reference, a.force), file=sys.stdout)
