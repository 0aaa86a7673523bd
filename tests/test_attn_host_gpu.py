"""attn_host: host tensors in, host tensor out, copies overlapped per block (needs a B200)."""

import pytest
import torch

import gfx906_b200
from gfx906_b200.configs import make_qkv
from tests.gpu_util import check_rows, sample_rows

pytestmark = pytest.mark.gpu

CASES = [((1, 24, 1024, 1024, 128), 8), ((2, 3, 300, 777, 64), 4), ((1, 1, 129, 5000, 16), None),
         ((3, 5, 256, 128, 32), 64), ((1, 4, 4096, 4096, 128), 3)]


@pytest.mark.parametrize("shape,blocks", CASES)
def test_attn_host_matches_oracle_and_device(shape, blocks):
    B, H, Sq, Skv, D = shape
    q, k, v = make_qkv(B, H, Sq, Skv, D, seed=Sq + D)
    hq, hk, hv = q.pin_memory(), k.pin_memory(), v.pin_memory()
    out = gfx906_b200.attn_host(hq, hk, hv, D ** -0.5, blocks=blocks)
    assert not out.is_cuda and out.shape == q.shape and out.dtype == torch.float16
    rows = None if B * H * Sq <= 8192 else sample_rows(Sq, n_each=48, seed=D)
    check_rows(out, q, k, v, D ** -0.5, rows, what=f"attn_host {shape} blocks={blocks}")
    dev = gfx906_b200.attn(q.cuda(), k.cuda(), v.cuda(), D ** -0.5).cpu()
    assert (out.float() - dev.float()).abs().max().item() <= 1e-3


def test_attn_host_reuses_out_and_accepts_pageable_inputs():
    q, k, v = make_qkv(2, 4, 512, 640, 64, seed=3)
    out = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    for _ in range(3):
        r = gfx906_b200.attn_host(q, k, v, 0.125, out=out, blocks=3)
        assert r is out
    check_rows(out, q, k, v, 0.125, None, what="pageable inputs")


def test_attn_host_non_blocking_then_synchronise():
    q, k, v = make_qkv(1, 6, 1024, 1024, 128, seed=4)
    hq, hk, hv = q.pin_memory(), k.pin_memory(), v.pin_memory()
    out = gfx906_b200.attn_host(hq, hk, hv, 128 ** -0.5, non_blocking=True)
    torch.cuda.current_stream().synchronize()
    check_rows(out, q, k, v, 128 ** -0.5, sample_rows(1024, n_each=32, seed=4), what="non_blocking")
    assert gfx906_b200.device_status(False) == 0


def test_attn_host_back_to_back_non_blocking_calls_keep_their_inputs():
    """Calls queued without a synchronisation in between: the uploads of a
    call overlap the previous call's kernels and downloads, and every call
    must still see its own inputs and write its own output."""
    shapes = [(1, 8, 1024, 1024, 128), (2, 3, 700, 900, 64), (1, 8, 1024, 1024, 128)]
    cases = []
    for i, (B, H, Sq, Skv, D) in enumerate(shapes):
        q, k, v = make_qkv(B, H, Sq, Skv, D, seed=40 + i)
        cases.append((q, k, v, D ** -0.5, q.pin_memory(), k.pin_memory(), v.pin_memory(),
                      torch.empty(q.shape, dtype=q.dtype, pin_memory=True)))
    for _ in range(2):
        for q, k, v, scale, hq, hk, hv, out in cases:
            gfx906_b200.attn_host(hq, hk, hv, scale, out=out, blocks=4, non_blocking=True)
    torch.cuda.current_stream().synchronize()
    for i, (q, k, v, scale, hq, hk, hv, out) in enumerate(cases):
        check_rows(out, q, k, v, scale, sample_rows(q.shape[2], n_each=24, seed=i), what=f"back-to-back call {i}")
    assert gfx906_b200.device_status(False) == 0


def test_attn_host_same_shape_calls_reuse_buffers_in_order():
    """Four queued calls of one shape cycle through the two device buffer sets;
    each must still read its own inputs and land in its own output."""
    cases = []
    for i in range(4):
        q, k, v = make_qkv(1, 6, 768, 1000, 64, seed=60 + i)
        cases.append((q, k, v, q.pin_memory(), k.pin_memory(), v.pin_memory(),
                      torch.empty(q.shape, dtype=q.dtype, pin_memory=True)))
    for q, k, v, hq, hk, hv, out in cases:
        gfx906_b200.attn_host(hq, hk, hv, 0.125, out=out, blocks=3, non_blocking=True)
    torch.cuda.current_stream().synchronize()
    for i, (q, k, v, hq, hk, hv, out) in enumerate(cases):
        check_rows(out, q, k, v, 0.125, sample_rows(768, n_each=24, seed=i), what=f"queued call {i}")


def test_attn_out_writes_into_given_tensor_and_checks_it():
    mod = gfx906_b200._module_or_raise()
    q, k, v = (t.cuda() for t in make_qkv(1, 2, 300, 400, 64, seed=7))
    o = torch.empty_like(q)
    mod.attn_out(q, k, v, 0.125, o)
    assert torch.equal(o, gfx906_b200.attn(q, k, v, 0.125))
    with pytest.raises(RuntimeError):
        mod.attn_out(q, k, v, 0.125, torch.empty(1, 2, 300, 32, dtype=torch.float16, device="cuda"))
    with pytest.raises(RuntimeError):
        mod.attn_out(q, k, v, 0.125, torch.empty_like(q, dtype=torch.float32))
