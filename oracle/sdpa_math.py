"""fp32 SDPA MATH on fp16 inputs: the reference's correctness oracle.

The reference checks its kernel against ``F.scaled_dot_product_attention`` on
the same fp16 tensors (``test.py:12``, ``test_variants.py:54-56``); on gfx906
that is the MATH backend (``deploy/gfx906_attention.py:17-18``). The B200
build evaluates the same formula in fp32 (inputs upcast from fp16), which is a
strictly more accurate target, and compares fp16 outputs to it with
max-abs <= 2e-3 and mean-abs <= 2e-4.

For long sequences the score matrix does not fit in memory, so query rows are
processed in chunks against the full K/V -- the reference's own slice trick
(``test.py:14-18``, ``test_d512.py:12-14``); each chunk is exact for its rows.
TEST INFRASTRUCTURE ONLY.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel


def sdpa_math_fp32(q, k, v, scale, q_chunk=None, rows=None):
    """Returns fp32 [B,H,Sq',D] = softmax(scale * q k^T) v, computed on the CPU.

    q, k, v: fp16 (or any float) tensors [B,H,S,D]; they are moved to the CPU
    and upcast to fp32. ``rows`` (a slice or index tensor over Sq) restricts
    the query rows; ``q_chunk`` bounds the rows per SDPA call (default: keep
    each chunk's score matrix under ~256 MiB).
    """
    q = q.detach().to("cpu", torch.float32)
    k = k.detach().to("cpu", torch.float32)
    v = v.detach().to("cpu", torch.float32)
    if rows is not None:
        q = q[:, :, rows]
    B, H, Sq, D = q.shape
    Skv = k.shape[2]
    if Skv == 0:
        return torch.zeros(B, H, Sq, v.shape[-1], dtype=torch.float32)
    if q_chunk is None:
        q_chunk = max(1, (64 << 20) // max(1, B * H * Skv))
    outs = []
    with sdpa_kernel(SDPBackend.MATH):
        for r0 in range(0, Sq, q_chunk):
            outs.append(F.scaled_dot_product_attention(
                q[:, :, r0:r0 + q_chunk], k, v, scale=scale))
    return torch.cat(outs, dim=2) if outs else torch.zeros(B, H, 0, D)


def errors(out_fp16, ref_fp32):
    """(max-abs, mean-abs) error of an fp16 output against the fp32 oracle."""
    d = (out_fp16.detach().to("cpu", torch.float32) - ref_fp32).abs()
    if d.numel() == 0:
        return 0.0, 0.0
    return d.max().item(), d.mean().item()
