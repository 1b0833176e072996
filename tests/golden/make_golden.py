"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs the reference's OWN Python code (read-only checkout of
luna-niemitalo/comfy_ui_gfx906_tools) on seeded inputs and stores inputs and
outputs in ``tests/golden/*.npz``:

  * ``nodes/ComfyUI-Gfx906Int4/ops.py`` imported as a module with a one-class
    ``comfy.ops`` stub (``ops.py:194,199`` need only a base class):
    ``quantize_pack_int4``, ``repack_q4_0_native``, ``get_group_rotation``,
    ``apply_group_rotation``, ``choose_rotation_group``, and the
    quantize-on-load of ``Gfx906Int4Ops.Linear`` via ``make_load_quantizing_ops``;
  * functions extracted verbatim (AST) from files that cannot be imported
    here: ``nodes.py::quantize_dequantize_int4`` (nodes.py:43-52),
    ``int4_train_test.py::dequant`` (develop/experiments/2026-10-11/
    int4_train_test.py:46-52), ``bench_int8.py::dequant``
    (develop/harness/bench_int8.py:32-33), ``nodes.py::_quantize_module_weight``.

Usage (in the build container, where the reference is mounted):
    python tests/golden/make_golden.py [--reference PATH]
The fixtures are committed; the tests never read the reference at run time.
"""
from __future__ import annotations

import argparse
import ast
import importlib.util
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _stub_comfy():
    comfy = types.ModuleType("comfy")
    comfy_ops = types.ModuleType("comfy.ops")

    class disable_weight_init:  # the only name ops.py needs (ops.py:199)
        pass

    class manual_cast(disable_weight_init):
        pass

    class MixedPrecisionOp:
        pass

    comfy_ops.disable_weight_init = disable_weight_init
    comfy_ops.manual_cast = manual_cast
    comfy_ops.MixedPrecisionOp = MixedPrecisionOp
    comfy.ops = comfy_ops
    sys.modules["comfy"] = comfy
    sys.modules["comfy.ops"] = comfy_ops


def _load_module(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _extract_function(path, func_name, namespace):
    """Exec one top-level function's source from `path` into `namespace`."""
    src = open(path).read()
    tree = ast.parse(src)
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name == func_name:
            mod = ast.Module(body=[node], type_ignores=[])
            exec(compile(mod, path, "exec"), namespace)
            return namespace[func_name]
    raise KeyError(f"{func_name} not found in {path}")


_REPO_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _bf16_bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get(
        "GFX906_REFERENCE", os.path.join(os.path.dirname(_REPO_ROOT), "reference")))
    args = ap.parse_args()
    ref = args.reference
    node_dir = os.path.join(ref, "nodes", "ComfyUI-Gfx906Int4")
    _stub_comfy()
    ops = _load_module(os.path.join(node_dir, "ops.py"), "ref_gfx906_ops")

    ns = {"torch": torch, "BLOCK": 32}
    qdq = _extract_function(os.path.join(node_dir, "nodes.py"), "quantize_dequantize_int4", ns)
    ns_t = {"torch": torch}
    dequant_train = _extract_function(
        os.path.join(ref, "develop", "experiments", "2026-10-11", "int4_train_test.py"), "dequant", ns_t)
    ns_8 = {"torch": torch}
    dequant_int8 = _extract_function(os.path.join(ref, "develop", "harness", "bench_int8.py"), "dequant", ns_8)
    ns_q = {
        "torch": torch, "repack_q4_0_native": ops.repack_q4_0_native, "quantize_pack_int4": ops.quantize_pack_int4,
        "get_group_rotation": ops.get_group_rotation, "apply_group_rotation": ops.apply_group_rotation,
        "_get_gguf_dequant_module": lambda: None,
    }
    quantize_module_weight = _extract_function(os.path.join(node_dir, "nodes.py"), "_quantize_module_weight", ns_q)

    out = {}
    g = torch.Generator().manual_seed(20261201)

    # --- quantize_pack_int4 on fp32 / fp16 / bf16 weights, incl. edge blocks ---
    for name, dtype in (("f32", torch.float32), ("f16", torch.float16), ("bf16", torch.bfloat16)):
        w = (torch.randn(48, 256, generator=g) * 0.05).to(dtype)
        w[0, :32] = 0                      # all-zero block: amax clamps to 1e-8
        w[1, :32] = torch.arange(32) - 15.5  # exact .5 ratios: round-half-even
        w[2, 32:64] = 7.0                   # |x| == amax everywhere
        w[3, 64:96] = -1e-3
        w[4, :] *= 1000.0                   # large magnitudes
        packed, scale = ops.quantize_pack_int4(w.float() if dtype == torch.float32 else w)
        out[f"qp_{name}_in"] = w.float().numpy()
        out[f"qp_{name}_packed"] = packed.numpy()
        out[f"qp_{name}_scale"] = scale.numpy()
        deq = dequant_train(packed, scale, 32)
        out[f"qp_{name}_dequant_f32"] = deq.numpy()

    # --- Q4_0 ingest: synthetic ggml blocks (the benchmark generators), repacked by the reference ---
    N, K = 40, 192
    u = torch.randint(0, 16, (N, K), generator=g, dtype=torch.int32)
    d = (torch.randn(N, K // 32, generator=g).abs() * 0.02 / 7 + 1e-4).half()
    ub = u.to(torch.uint8).reshape(N * K // 32, 32)
    blocks = torch.empty(N * K // 32, 18, dtype=torch.uint8)
    blocks[:, :2] = d.reshape(-1, 1).view(torch.uint8).reshape(-1, 2)
    blocks[:, 2:] = (ub[:, :16] & 0xF) | ((ub[:, 16:] & 0xF) << 4)
    raw = blocks.reshape(-1).contiguous()
    packed, scale = ops.repack_q4_0_native(raw, N, K)
    out["q40_raw"] = raw.numpy()
    out["q40_u"] = u.numpy().astype(np.uint8)
    out["q40_d"] = d.numpy()
    out["q40_packed"] = packed.numpy()
    out["q40_scale"] = scale.numpy()
    out["q40_dequant_f32"] = dequant_train(packed, scale, 32).numpy()
    # the bf16 weight the W4A16 emulation multiplies with (nodes.py:51-52 semantics)
    out["q40_dequant_bf16_bits"] = _bf16_bits((dequant_train(packed, scale, 32)).to(torch.bfloat16))

    # --- quantize_dequantize_int4 (nodes.py:43-52) in bf16 and fp32 ---
    t = torch.randn(16, 128, generator=g) * 0.1
    out["qdq_in"] = t.numpy()
    out["qdq_f32"] = qdq(t).numpy()
    out["qdq_bf16_bits"] = _bf16_bits(qdq(t.to(torch.bfloat16)))
    out["qdq_bf16_in_bits"] = _bf16_bits(t.to(torch.bfloat16))

    # --- int8 dequant (bench_int8.py:32-33) on a hand-made int8 operand ---
    q8 = torch.clamp(torch.round(torch.randn(24, 128, generator=g) * 40), -127, 127).to(torch.int8)
    s8 = torch.rand(24, 4, generator=g) * 0.01 + 1e-4
    out["i8_q"] = q8.numpy()
    out["i8_s"] = s8.numpy()
    out["i8_dequant"] = dequant_int8(q8, s8).numpy()

    # --- small GEMM: fp32 dequant-then-matmul (bench_int8.py:43 pattern) ---
    M = 5
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    bias = torch.randn(N, generator=g).to(torch.bfloat16)
    w_f32 = dequant_train(out_t := torch.from_numpy(out["q40_packed"]), torch.from_numpy(out["q40_scale"]), 32)
    del out_t
    y = x.float() @ w_f32.t() + bias.float()
    out["gemm_x_bits"] = _bf16_bits(x)
    out["gemm_bias_bits"] = _bf16_bits(bias)
    out["gemm_y_f32"] = y.numpy()

    # --- rotation helpers (ops.py:43-105) ---
    for kin in (96, 256, 40):
        grp = ops.choose_rotation_group(kin)
        out[f"rot_group_{kin}"] = np.array(-1 if grp is None else grp)
    R = ops.get_group_rotation(256, 128, torch.device("cpu"))
    out["rot_R_256_128"] = R.numpy()
    v = torch.randn(6, 256, generator=g)
    out["rot_in"] = v.numpy()
    out["rot_out"] = ops.apply_group_rotation(v, R, 128).numpy()

    # --- Gfx906Int4Ops.Linear quantize-on-load (ops.py:228-246) with rotation ---
    LoadOps = ops.make_load_quantizing_ops(sys.modules["comfy.ops"].manual_cast, "cpu", True)
    lin = LoadOps.Linear(256, 24, bias=True)
    wl = torch.randn(24, 256, generator=g) * 0.05
    bl = torch.randn(24, generator=g)
    sd = {"weight": wl.clone(), "bias": bl.clone()}
    lin.load_state_dict(sd)
    out["load_w"] = wl.numpy()
    out["load_rotation_group"] = np.array(lin.rotation_group)
    out["load_q4"] = lin.weight_q4.numpy()
    out["load_scale"] = lin.weight_scale.numpy()

    # --- _quantize_module_weight (nodes.py:157-223): plain float route ---
    class _Fake:
        def __init__(self, w):
            self.weight = w
            self.out_features, self.in_features = w.shape
    wp = (torch.randn(16, 64, generator=g) * 0.05).to(torch.bfloat16)
    pk, sc, tag = quantize_module_weight(_Fake(wp), 32, 0)
    out["qmw_in_bits"] = _bf16_bits(wp)
    out["qmw_packed"] = pk.numpy()
    out["qmw_scale"] = sc.numpy()
    out["qmw_tag"] = np.array(tag)

    path = os.path.join(HERE, "reference_vectors.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
