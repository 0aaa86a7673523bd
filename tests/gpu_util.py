"""Shared helpers of the GPU tests (parity against the CPU oracle)."""

import torch

from oracle.sdpa_math import errors, sdpa_math_fp32

MAX_ABS = 2e-3   # tolerance on the fp16 output vs fp32 SDPA MATH
MEAN_ABS = 2e-4


def check_rows(out, q, k, v, scale, rows=None, max_abs=MAX_ABS, mean_abs=MEAN_ABS, what=""):
    """Compare out[:, :, rows] with the fp32 oracle on the same rows."""
    ref = sdpa_math_fp32(q, k, v, scale, rows=rows)
    got = out if rows is None else out[:, :, rows]
    mx, mean = errors(got, ref)
    assert mx <= max_abs and mean <= mean_abs, f"{what}: max-abs {mx:.3e} mean-abs {mean:.3e}"
    return mx, mean


def sample_rows(Sq, n_each=128, seed=0):
    """First and last rows (tile edges) plus a seeded random sample."""
    g = torch.Generator().manual_seed(seed)
    head = torch.arange(0, min(Sq, n_each))
    tail = torch.arange(max(0, Sq - n_each - 2), Sq)
    mid = torch.randint(0, Sq, (n_each,), generator=g)
    return torch.unique(torch.cat([head, tail, mid]))
