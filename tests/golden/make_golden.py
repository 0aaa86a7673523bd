"""Generate golden attention vectors from the reference's own numpy model.

The reference ships no golden vectors: its GPU tests draw ``torch.randn`` on
the device (``test.py:5,8``). It does ship a CPU model of its pair kernel,
``attn_pair_model`` (``model_check.py:103-133``), which emulates the kernel's
per-lane head-dim slices, its cross-lane reduction and its tiled online
softmax (TILE_N = 16) in float64, and which the reference checks against
direct attention to 1e-5 (``model_check.py:136-153``).

This script imports that model from a checkout of the reference (by default
a ``reference`` directory beside this repository, or ``$GFX906_REFERENCE``),
runs it on small seeded inputs
that are exactly representable in fp16 (odd lengths, Sq != Skv, every head-dim
family the reference supports), and writes inputs and outputs to
``pair_model_cases.npz`` beside this file. The fixture is committed; the tests
only read it. Re-run this script only in a container that has the reference.

    python tests/golden/make_golden.py
"""

from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT = HERE / "pair_model_cases.npz"

# (name, B, H, Sq, Skv, D, scale, std, seed, SPLIT, ilv)
CASES = [
    ("d64_odd", 1, 2, 37, 83, 64, 0.125, 1.0, 11, 4, True),
    ("d128_odd", 1, 2, 37, 83, 128, 128 ** -0.5, 1.0, 12, 4, True),
    ("d128_cross", 1, 1, 257, 140, 128, 128 ** -0.5, 0.5, 13, 4, True),
    ("d64_tile_edges", 1, 1, 130, 129, 64, 0.125, 1.0, 14, 4, True),
    ("d32_strided", 1, 2, 29, 150, 32, 32 ** -0.5, 1.0, 15, 4, False),
    ("d16", 1, 1, 13, 40, 16, 0.25, 1.0, 16, 4, False),
    ("d8", 1, 1, 9, 33, 8, 8 ** -0.5, 1.0, 17, 4, False),
    ("d24", 1, 1, 11, 70, 24, 24 ** -0.5, 1.0, 18, 4, False),
    ("d512", 1, 1, 8, 40, 512, 512 ** -0.5, 1.0, 19, 4, True),
    ("single", 1, 1, 1, 1, 64, 0.125, 1.0, 20, 4, True),
    ("large_scores", 1, 1, 64, 300, 64, 0.125, 2.5, 21, 4, True),
]


def load_reference_model():
    default = Path(__file__).resolve().parents[2].parent / "reference"
    root = Path(os.environ.get("GFX906_REFERENCE", str(default)))
    path = root / "model_check.py"
    spec = importlib.util.spec_from_file_location("reference_model_check", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)  # module body only defines functions
    return mod


def main():
    ref = load_reference_model()
    arrays = {}
    names = []
    for (name, B, H, Sq, Skv, D, scale, std, seed, split, ilv) in CASES:
        rng = np.random.default_rng(seed)
        q = (rng.standard_normal((B, H, Sq, D)) * std).astype(np.float16)
        k = (rng.standard_normal((B, H, Skv, D)) * std).astype(np.float16)
        v = (rng.standard_normal((B, H, Skv, D)) * std).astype(np.float16)
        out = ref.attn_pair_model(q.astype(np.float64), k.astype(np.float64),
                                  v.astype(np.float64), scale, SPLIT=split, ilv=ilv)
        arrays[f"{name}.q"] = q
        arrays[f"{name}.k"] = k
        arrays[f"{name}.v"] = v
        arrays[f"{name}.out"] = out.astype(np.float32)
        arrays[f"{name}.scale"] = np.float64(scale)
        names.append(name)
        print(f"{name}: B{B} H{H} Sq{Sq} Skv{Skv} D{D} -> |out|max {np.abs(out).max():.4f}")
    arrays["names"] = np.array(names)
    np.savez_compressed(OUT, **arrays)
    print("wrote", OUT, OUT.stat().st_size, "bytes")


if __name__ == "__main__":
    sys.exit(main())
