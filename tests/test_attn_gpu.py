"""Parity of the sm_100a kernel with the CPU oracle (needs a B200)."""

import numpy as np
import pytest
import torch

from gfx906_b200.configs import CONFIGS, config_inputs, make_qkv
from oracle.sdpa_math import sdpa_math_fp32
from tests.gpu_util import MAX_ABS, MEAN_ABS, check_rows, sample_rows

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def op():
    import gfx906_b200

    assert gfx906_b200.is_sm100(), "these tests need an sm_100 GPU"
    gfx906_b200.attn  # noqa: B018
    mod = gfx906_b200.load_attention()
    assert mod is not None, gfx906_b200.last_error()
    yield mod
    assert mod.device_status(True) == 0, "a kernel wait timed out during the tests"


def run(op, q, k, v, scale):
    out = op.attn(q.cuda(), k.cuda(), v.cuda(), scale)
    torch.cuda.synchronize()
    return out.cpu()


def test_golden_reference_model_cases(op, golden):
    """Kernel vs the reference's own pair-kernel model (model_check.py:103-133)."""
    for name, c in golden.items():
        q, k, v = (torch.from_numpy(c[x]) for x in ("q", "k", "v"))
        out = run(op, q, k, v, float(c["scale"])).float().numpy()
        ref = c["out"]
        # fp16 output: allow half an ulp of |ref| on top of the absolute bar
        big = max(1.0, float(np.abs(ref).max()))
        err = np.abs(out - ref)
        assert err.max() <= MAX_ABS * big, (name, err.max())
        assert err.mean() <= MEAN_ABS * big, (name, err.mean())


@pytest.mark.parametrize("S", [64, 256, 1024, 4096, 100, 1000])
def test_reference_test_py_shapes_d64(op, S):
    """test.py:23-24: B=2, H=8, D=64, scale 0.125."""
    q, k, v = make_qkv(2, 8, S, S, 64, seed=S)
    out = run(op, q, k, v, 0.125)
    rows = None if S <= 1024 else sample_rows(S)
    check_rows(out, q, k, v, 0.125, rows, what=f"S={S}")


@pytest.mark.parametrize("D", [32, 16, 8, 24, 40, 48, 56])
def test_small_head_dims(op, D):
    """test.py:26-27 (D=32, D=16 at S=512) plus every other D<64, D%8==0."""
    q, k, v = make_qkv(2, 8, 512, 512, D, seed=D)
    out = run(op, q, k, v, 0.125)
    check_rows(out, q, k, v, 0.125, what=f"D={D}")


@pytest.mark.parametrize("Sq,Skv,D", [(256, 256, 64), (1024, 1024, 64), (100, 300, 64),
                                      (256, 256, 128), (1024, 1024, 128), (77, 411, 128),
                                      (512, 512, 32), (512, 512, 512)])
def test_reference_variant_matrix(op, Sq, Skv, D):
    """test_variants.py:78-80 shapes (B=2, H=4, scale 0.125): Sq != Skv, odd lengths."""
    q, k, v = make_qkv(2, 4, Sq, Skv, D, seed=Sq + Skv + D)
    out = run(op, q, k, v, 0.125)
    check_rows(out, q, k, v, 0.125, what=f"{Sq}x{Skv} D{D}")


@pytest.mark.parametrize("Sq,Skv,D", [(1, 1, 64), (1, 7, 128), (7, 1, 64), (129, 1, 128),
                                      (255, 257, 128), (257, 255, 64), (513, 129, 128),
                                      (384, 640, 128)])
def test_ragged_edges(op, Sq, Skv, D):
    q, k, v = make_qkv(1, 3, Sq, Skv, D, seed=Sq * 7 + Skv)
    out = run(op, q, k, v, D ** -0.5)
    check_rows(out, q, k, v, D ** -0.5, what=f"{Sq}x{Skv} D{D}")


@pytest.mark.parametrize("name", ["C1", "C2", "C3", "C4", "C5s"])
def test_benchmark_configs(op, name):
    cfg = CONFIGS[name]
    q, k, v = config_inputs(cfg)
    out = run(op, q, k, v, cfg.scale)
    rows = None if cfg.Sq * cfg.B * cfg.H <= 8192 else sample_rows(cfg.Sq, seed=cfg.seed)
    check_rows(out, q, k, v, cfg.scale, rows, what=name)


def test_scale_edge_cases(op):
    q, k, v = make_qkv(1, 2, 300, 200, 64, seed=9)
    for scale in (-0.125, 0.0, 1.0, 1e-3):
        out = run(op, q, k, v, scale)
        check_rows(out, q, k, v, scale, what=f"scale={scale}")


def test_large_scores_exercise_rescale(op):
    """Scores growing along the keys force repeated max updates (lazy rescale)."""
    q, k, v = make_qkv(1, 2, 256, 1024, 128, seed=10)
    ramp = torch.linspace(0.1, 3.0, 1024).view(1, 1, -1, 1)
    k = (k.float() * ramp).half()
    q = (q.float() * 2).half()
    out = run(op, q, k, v, 128 ** -0.5)
    # Peaked rows have |O| > 1 here: fp16 P and fp16 output rounding scale with
    # |O|, so the bar is 2e-3 / 2e-4 times max(1, max|ref|) (as for the fixtures).
    ref_mag = max(1.0, float(sdpa_math_fp32(q, k, v, 128 ** -0.5).abs().max()))
    check_rows(out, q, k, v, 128 ** -0.5, max_abs=MAX_ABS * ref_mag, mean_abs=MEAN_ABS * ref_mag,
               what="ramp")


def test_empty_and_zero_keys(op):
    q, k, v = make_qkv(1, 2, 16, 0, 64)
    out = run(op, q, k, v, 0.125)
    assert out.shape == (1, 2, 16, 64) and torch.all(out == 0)
    q, k, v = make_qkv(1, 2, 0, 16, 64)
    out = run(op, q, k, v, 0.125)
    assert out.shape == (1, 2, 0, 64)


def test_non_contiguous_inputs(op):
    """test_d512.py:22-30 pattern: strided view and transposed [b, D, S] views."""
    g = torch.Generator().manual_seed(11)
    b, S, D = 1, 1024, 128
    qf = torch.randn(b, S, D * 2, generator=g).half()[:, :, ::2]
    kf = torch.randn(b, D, S, generator=g).half().transpose(1, 2)
    vf = torch.randn(b, D, S, generator=g).half().transpose(1, 2)
    q4, k4, v4 = qf.unsqueeze(1), kf.unsqueeze(1), vf.unsqueeze(1)
    out = op.attn(q4.cuda(), k4.cuda(), v4.cuda(), D ** -0.5).cpu()
    check_rows(out, q4.contiguous(), k4.contiguous(), v4.contiguous(), D ** -0.5, what="noncontig")


def test_deterministic(op):
    """dbg.py:22-23: two calls give bit-identical outputs."""
    q, k, v = make_qkv(2, 8, 1000, 777, 128, seed=12)
    q, k, v = q.cuda(), k.cuda(), v.cuda()
    a = op.attn(q, k, v, 0.1)
    b = op.attn(q, k, v, 0.1)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_input_checks_raise(op):
    q, k, v = make_qkv(1, 1, 8, 8, 64, device="cuda")
    with pytest.raises(RuntimeError):
        op.attn(q.float(), k, v, 0.1)
    with pytest.raises(RuntimeError):
        op.attn(q, k.float(), v, 0.1)
    with pytest.raises(RuntimeError):
        op.attn(q, k[:, :, :4], v, 0.1)
    q2, k2, v2 = make_qkv(1, 1, 8, 8, 96, device="cuda")
    with pytest.raises(RuntimeError, match="head_dim"):
        op.attn(q2, k2, v2, 0.1)


def test_current_stream_is_used(op):
    q, k, v = make_qkv(1, 4, 512, 512, 64, seed=13, device="cuda")
    ref = op.attn(q, k, v, 0.125)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out = op.attn(q, k, v, 0.125)
    s.synchronize()
    assert torch.equal(out, ref)


def test_long_sequence_memory_is_linear(op):
    """test.py:48-61: S=32768 at H=8, D=64 runs in O(S*D) memory (MATH would need 32 GiB)."""
    S = 32768
    q, k, v = make_qkv(1, 8, S, S, 64, seed=14, device="cuda")
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    out = op.attn(q, k, v, 0.125)
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated() - base
    # the output plus the split workspace, whose size depends on the SM count
    # and head dim, not on S (at most 48 MiB on a B200); S*S fp32 scores alone
    # would be 8 * 32768^2 * 4 B = 32 GiB
    assert peak <= out.numel() * 2 + (48 << 20), peak
    rows = sample_rows(S, n_each=64, seed=14)
    check_rows(out.cpu(), q.cpu(), k.cpu(), v.cpu(), 0.125, rows, what="S=32768")


@pytest.mark.parametrize("S", [256, 1024, 4096, 9216])
def test_reference_d512_shapes(op, S):
    """test_d512.py:19-20: D=512, one head, checked on a <=1024-row slice."""
    q, k, v = make_qkv(1, 1, S, S, 512, seed=S + 512)
    out = run(op, q, k, v, 512 ** -0.5)
    rows = None if S <= 1024 else sample_rows(S, seed=S)
    check_rows(out, q, k, v, 512 ** -0.5, rows, what=f"D512 S={S}")


@pytest.mark.parametrize("Sq,Skv", [(1, 1), (77, 411), (130, 129), (300, 1000), (1000, 64)])
def test_d512_ragged(op, Sq, Skv):
    q, k, v = make_qkv(2, 2, Sq, Skv, 512, seed=Sq * 3 + Skv)
    out = run(op, q, k, v, 512 ** -0.5)
    check_rows(out, q, k, v, 512 ** -0.5, what=f"D512 {Sq}x{Skv}")


def test_d512_non_contiguous_vae_layout(op):
    """test_d512.py:22-30: strided q and transposed [b, D, S] k/v views."""
    g = torch.Generator().manual_seed(21)
    b, S, D = 1, 1024, 512
    qf = torch.randn(b, S, D * 2, generator=g).half()[:, :, ::2]
    kf = torch.randn(b, D, S, generator=g).half().transpose(1, 2)
    vf = torch.randn(b, D, S, generator=g).half().transpose(1, 2)
    q4, k4, v4 = qf.unsqueeze(1), kf.unsqueeze(1), vf.unsqueeze(1)
    out = op.attn(q4.cuda(), k4.cuda(), v4.cuda(), D ** -0.5).cpu()
    check_rows(out, q4.contiguous(), k4.contiguous(), v4.contiguous(), D ** -0.5, what="d512 noncontig")


def test_d512_very_long_sequence(op):
    """bench_d512.py:63-79: S=129600 at D=512 (one head) in O(S*D) memory."""
    S = 129600
    q, k, v = make_qkv(1, 1, S, S, 512, seed=15, device="cuda")
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    out = op.attn(q, k, v, 512 ** -0.5)
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated() - base
    assert peak <= out.numel() * 2 + (1 << 20), peak  # the D=512 kernel uses no workspace
    rows = sample_rows(S, n_each=24, seed=15)
    check_rows(out.cpu(), q.cpu(), k.cpu(), v.cpu(), 512 ** -0.5, rows, what="S=129600 D512")
