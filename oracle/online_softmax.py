"""Numpy restatement of the reference kernel's tiled online softmax.

The reference streams keys in tiles (TILE_N = 16, ``attn_kernel.hip:62-68``)
and keeps, per query row, a running max ``m`` and running sum ``l``
(``attn_kernel.hip:357``). Per tile (``attn_kernel.hip:452-462, 491-492``):

    s      = scale * q . k_i            for the keys of the tile
    m_new  = max(m, max(s))
    e_i    = exp(s_i - m_new)
    rs     = exp(m - m_new) if l > 0 else 0
    acc    = acc * rs + sum_i e_i v_i
    l      = l * rs + sum_i e_i ;  m = m_new

and writes ``acc / l`` at the end (``attn_kernel.hip:497-511``); rows with
l == 0 (no keys) are left unwritten by the reference and are zero here.

``online_softmax_attention`` restates that loop with the tile size as a
parameter and an optional lazy-rescale threshold in log2 units: with
``threshold=t`` the running max is only moved when the new tile max exceeds
it by more than ``t / log2(e)``; the stale max cancels between acc and l, so
the result is the same attention (the sm_100a kernel uses BN=128, t=8).
TEST INFRASTRUCTURE ONLY.
"""

from __future__ import annotations

import numpy as np

LOG2E = 1.4426950408889634


def online_softmax_attention(q, k, v, scale, tile_n=16, threshold=0.0):
    """float64 attention over [..., Sq, D] x [..., Skv, D] via the tiled loop."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    lead = q.shape[:-2]
    Sq, D = q.shape[-2:]
    Skv = k.shape[-2]
    nb = int(np.prod(lead)) if lead else 1
    qf = q.reshape(nb, Sq, D)
    kf = k.reshape(nb, Skv, k.shape[-1])
    vf = v.reshape(nb, Skv, v.shape[-1])
    out = np.zeros((qf.shape[0], Sq, v.shape[-1]))
    thr = threshold / LOG2E  # natural-log units
    for b in range(qf.shape[0]):
        m = np.full(Sq, -np.inf)
        l = np.zeros(Sq)
        acc = np.zeros((Sq, v.shape[-1]))
        for n0 in range(0, Skv, tile_n):
            s = scale * (qf[b] @ kf[b, n0:n0 + tile_n].T)  # [Sq, tile]
            m_tile = s.max(axis=1)
            m_cand = np.maximum(m, m_tile)
            move = m_cand > m + thr
            m_new = np.where(move, m_cand, m)
            rs = np.where(l > 0, np.exp(np.where(np.isfinite(m), m - m_new, -np.inf)), 0.0)
            e = np.exp(s - m_new[:, None])
            acc = acc * rs[:, None] + e @ vf[b, n0:n0 + tile_n]
            l = l * rs + e.sum(axis=1)
            m = m_new
        live = l > 0
        out[b, live] = acc[live] / l[live, None]
    return out.reshape(*lead, Sq, v.shape[-1])


def direct_attention(q, k, v, scale):
    """float64 softmax(scale q k^T) v without tiling (reference for the model)."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    s = scale * (q @ np.swapaxes(k, -1, -2))
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    return (p @ v) / p.sum(axis=-1, keepdims=True)
