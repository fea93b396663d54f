"""Generate tests/golden/golden.npz by running the REFERENCE's own unfused CPU path.

Runs ``rmsnorm_residual_qkv`` from the reference checkout (src/triton_fused_rmsnorm_qkv/
baseline.py, imported from ``--reference``) on the seeded inputs of ``oracle.make_case``
for every case in cases.py, and stores:
  <case>__out     full projection = torch.cat of the reference's three chunks
  <case>__hidden  x + residual as PyTorch computes it (baseline.py:48)
  <case>__digest  sha256 of the input tensors (so a test can tell regenerated inputs
                  differ, e.g. under another PyTorch version)
HAS_RESIDUAL=0 cases feed a zero residual (the reference raises on None; x + 0 == x).

Usage (in a checkout where the reference is present):
    python tests/golden/make_golden.py --reference /path/to/reference
"""
from __future__ import annotations

import argparse
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).resolve().parent))

from cases import CASES, as_bits, inputs_digest  # noqa: E402
from oracle import make_case  # noqa: E402


def load_reference_baseline(ref_root: Path):
    path = ref_root / "src" / "triton_fused_rmsnorm_qkv" / "baseline.py"
    spec = importlib.util.spec_from_file_location("_reference_baseline", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.rmsnorm_residual_qkv


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of a checkout of the reference repository")
    ap.add_argument("--out", default=str(Path(__file__).resolve().parent / "golden.npz"))
    a = ap.parse_args()
    ref_fn = load_reference_baseline(Path(a.reference))
    torch.set_num_threads(1)
    arrays = {"torch_version": np.array(torch.__version__)}
    for c in CASES:
        x, r, g, w = make_case(c["M"], c["H"], c["N"], c["dtype"], c["seed"], c["res"])
        r_eff = r if r is not None else torch.zeros_like(x)
        q, k, v = ref_fn(x[None], r_eff[None], g, w, c["eps"])
        out = torch.cat([q, k, v], dim=-1)[0]
        hidden = x + r_eff
        arrays[c["name"] + "__out"] = as_bits(out)
        arrays[c["name"] + "__hidden"] = as_bits(hidden)
        arrays[c["name"] + "__digest"] = np.array(inputs_digest(x, r, g, w))
        print(f"{c['name']}: out {tuple(out.shape)} {out.dtype}")
    np.savez(a.out, **arrays)
    print("wrote", a.out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
