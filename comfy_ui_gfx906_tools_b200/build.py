"""Build the sm_100a shared library in-tree with nvcc (no torch extension JIT).

    python -m comfy_ui_gfx906_tools_b200.build [--force] [--verbose]

Produces ``comfy_ui_gfx906_tools_b200/lib/libgfx906_b200.so``: every ``csrc/*.cu``
compiled for ``-gencode arch=compute_100a,code=sm_100a`` and linked into one
C-ABI library (declarations in ``include/gfx906_b200.h``). nvcc cross-compiles
without a GPU, so this runs in the build container; the built ``.so`` travels
with the repository snapshot to the GPU box.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_ROOT, "include")
LIB_DIR = os.path.join(PKG_DIR, "lib")
OBJ_DIR = os.path.join(REPO_ROOT, "_build", "obj")
LIB_NAME = "libgfx906_b200.so"
LIB_PATH = os.path.join(LIB_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"]


def nvcc_path() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    if os.path.exists(cand):
        return cand
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found (set CUDA_HOME)")
    return found


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + glob.glob(os.path.join(INCLUDE, "*.h")))


def _newest(paths):
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    return _newest(_sources() + _headers() + [os.path.abspath(__file__)]) > os.path.getmtime(LIB_PATH)


def _compile(src: str, verbose: bool, extra=(), obj_dir: str = OBJ_DIR, force: bool = True) -> str:
    os.makedirs(obj_dir, exist_ok=True)
    obj = os.path.join(obj_dir, os.path.basename(src).replace(".cu", ".o"))
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= _newest(
            [src, *_headers(), os.path.abspath(__file__)]):
        return obj  # up to date (default flags only)
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, file=sys.stderr)
    return obj


def build(force: bool = False, verbose: bool = False, defines=(), out_path: str | None = None) -> str:
    """Compile and link the library; `defines` (e.g. ["-DNAME=1"]) and
    `out_path` build a variant elsewhere (the in-tree default is untouched)."""
    target = out_path or LIB_PATH
    if not force and not defines and out_path is None and not needs_build():
        return LIB_PATH
    os.makedirs(os.path.dirname(target), exist_ok=True)
    srcs = _sources()
    obj_dir = OBJ_DIR if not defines else os.path.join(OBJ_DIR, "variant_" + str(abs(hash(tuple(defines)))))
    incremental = not force and not defines and not verbose
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, tuple(defines), obj_dir, force=not incremental), srcs))
    tmp = target + ".tmp"
    cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-o", tmp, *objs, "-lrt", "-lpthread", "-ldl"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, target)
    return target


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register / spill / smem usage")
    ap.add_argument("-D", dest="defines", action="append", default=[], help="extra preprocessor define (variant build)")
    ap.add_argument("--out", default=None, help="output path for a variant build")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, defines=["-D" + d for d in a.defines], out_path=a.out))


if __name__ == "__main__":
    main()
