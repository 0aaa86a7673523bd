"""Size-independent properties at the benchmark configs' full sizes (needs a B200).

Where the CPU oracle cannot compare whole outputs in seconds, these hold for
any correct attention and are checked on every row: invariance under a joint
permutation of the keys and values, linearity in V, and agreement of a
query-row slice with the same rows of the full call. Sampled rows are also
compared with the oracle directly.
"""

import pytest
import torch

import gfx906_b200
from gfx906_b200.configs import CONFIGS, make_qkv
from tests.gpu_util import MAX_ABS, check_rows, sample_rows

pytestmark = pytest.mark.gpu


def attn(q, k, v, scale):
    return gfx906_b200.attn(q, k, v, scale)


def test_c5_full_size_rows_against_oracle():
    cfg = CONFIGS["C5"]
    q, k, v = make_qkv(cfg.B, cfg.H, cfg.Sq, cfg.Skv, cfg.D, seed=cfg.seed)
    out = attn(q.cuda(), k.cuda(), v.cuda(), cfg.scale).cpu()
    assert torch.isfinite(out.float()).all()
    check_rows(out, q, k, v, cfg.scale, sample_rows(cfg.Sq, n_each=16, seed=cfg.seed), what="C5 131072")


@pytest.mark.parametrize("name", ["C2", "C5"])
def test_key_permutation_invariance(name):
    cfg = CONFIGS[name]
    q, k, v = make_qkv(cfg.B, cfg.H, cfg.Sq, cfg.Skv, cfg.D, seed=cfg.seed, device="cuda")
    perm = torch.randperm(cfg.Skv, generator=torch.Generator().manual_seed(3)).cuda()
    a = attn(q, k, v, cfg.scale)
    b = attn(q, k[:, :, perm].contiguous(), v[:, :, perm].contiguous(), cfg.scale)
    # the same sums in another order: fp32 accumulation, fp16 P and output
    assert (a.float() - b.float()).abs().max().item() <= MAX_ABS


@pytest.mark.parametrize("name", ["C2", "C4"])
def test_linearity_in_v(name):
    cfg = CONFIGS[name]
    q, k, v1 = make_qkv(cfg.B, cfg.H, cfg.Sq, cfg.Skv, cfg.D, seed=cfg.seed, device="cuda")
    v2 = torch.randn(v1.shape, generator=torch.Generator().manual_seed(11)).half().cuda()
    both = attn(q, k, (v1.float() * 0.5 + v2.float() * 0.25).half(), cfg.scale).float()
    parts = attn(q, k, v1, cfg.scale).float() * 0.5 + attn(q, k, v2, cfg.scale).float() * 0.25
    assert (both - parts).abs().max().item() <= MAX_ABS


@pytest.mark.parametrize("name,rows", [("C2", (1024, 2048)), ("C3", (256, 4096)), ("C5s", (20480, 32768))])
def test_query_row_slice_matches_full_call(name, rows):
    cfg = CONFIGS[name]
    q, k, v = make_qkv(cfg.B, cfg.H, cfg.Sq, cfg.Skv, cfg.D, seed=cfg.seed, device="cuda")
    full = attn(q, k, v, cfg.scale)
    lo, hi = rows
    part = attn(q[:, :, lo:hi].contiguous(), k, v, cfg.scale)
    # whole 256-row blocks: same per-row arithmetic unless the schedule splits
    # the key range differently (then the combine order differs by rounding)
    assert (part.float() - full[:, :, lo:hi].float()).abs().max().item() <= 1e-3
