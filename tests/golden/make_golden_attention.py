"""Generate tests/golden/attention_prep.npz: the reference's own attention
prepare step on seeded inputs.

Imports nodes/ComfyUI-Gfx906Int4/attention.py from the reference checkout as a
package module (its relative imports ``ops`` and ``block_sparse`` load from
the same directory; ``comfy.ops`` is stubbed as in make_golden.py) and runs
``_prepare_qk`` for the three Q.K modes and ``_prepare_v`` for both P.V modes
on CPU tensors (attention.py:31-75). The fixture pins
``comfy_ui_gfx906_tools_b200.attention.prepare_qk / prepare_v`` bit for bit,
and the inputs feed the oracle's restatement of the kernel.

Usage (where the reference is mounted):
    python tests/golden/make_golden_attention.py [--reference PATH]
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from make_golden import _REPO_ROOT, _stub_comfy  # noqa: E402


def _load_reference_package(node_dir: str):
    pkg = types.ModuleType("ref_gfx906_pkg")
    pkg.__path__ = [node_dir]
    sys.modules["ref_gfx906_pkg"] = pkg
    for name in ("ops", "block_sparse", "attention"):
        spec = importlib.util.spec_from_file_location(f"ref_gfx906_pkg.{name}", os.path.join(node_dir, f"{name}.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = mod
        spec.loader.exec_module(mod)
        setattr(pkg, name, mod)
    return pkg.attention


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get(
        "GFX906_REFERENCE", os.path.join(os.path.dirname(_REPO_ROOT), "reference")))
    args = ap.parse_args()
    _stub_comfy()
    att = _load_reference_package(os.path.join(args.reference, "nodes", "ComfyUI-Gfx906Int4"))

    g = torch.Generator().manual_seed(20261202)
    B, H, KVH, L = 1, 2, 1, 100
    q = (torch.randn(B, H, L, 128, generator=g) * 2).half()
    k = (torch.randn(B, KVH, L, 128, generator=g) * 2 + 0.5).half()  # a mean offset for the smoothing step
    v = torch.randn(B, KVH, L, 128, generator=g).half()
    q[0, 1, 7, 3] = 40.0   # outliers: the int4 rotation spreads them
    k[0, 0, 9, 100] = -35.0
    v[0, 0, 70, 5] = 12.0
    out = {"q": q.numpy(), "k": k.numpy(), "v": v.numpy()}
    for mode in ("fp16", "int8", "int4"):
        qb, qs, kb, ks = att._prepare_qk(q, k, mode)
        out[f"qk_{mode}_qb"] = qb.numpy()
        out[f"qk_{mode}_qs"] = qs.numpy()
        out[f"qk_{mode}_kb"] = kb.numpy()
        out[f"qk_{mode}_ks"] = ks.numpy()
    for mode in ("fp16", "u8"):
        vt, vs = att._prepare_v(v, mode)
        out[f"v_{mode}_vt"] = vt.numpy()
        out[f"v_{mode}_vs"] = vs.numpy()
    # block-sparse prediction and calibration (block_sparse.py:60-90) on structured q / k:
    # clustered keys so that the prediction keeps a strict subset of tiles
    bs = sys.modules["ref_gfx906_pkg.block_sparse"]
    # (runs of 64 keys / 32 queries around one of 6 centres, as neighbouring image tokens are alike)
    centers = torch.randn(6, 128, generator=g) * 3
    kid = torch.randint(0, 6, (1, 1, -(-450 // 64)), generator=g).repeat_interleave(64, -1)[..., :450]
    qid = torch.randint(0, 6, (1, 2, -(-300 // 32)), generator=g).repeat_interleave(32, -1)[..., :300]
    kc = centers[kid] + torch.randn(1, 1, 450, 128, generator=g) * 0.3
    qc = centers[qid] + torch.randn(1, 2, 300, 128, generator=g) * 0.3
    out["bs_q"], out["bs_k"] = qc.half().numpy(), kc.half().numpy()
    for tau, rows in ((0.9, 128), (0.995, 64)):
        keep = bs.predict_keep(qc.half(), kc.half(), tau, rows)
        out[f"bs_keep_{rows}"] = keep.numpy()
        out[f"bs_missed_{rows}"] = bs.missed_mass(qc.half(), kc.half(), keep, rows).numpy()
    path = os.path.join(HERE, "attention_prep.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays")


if __name__ == "__main__":
    main()
