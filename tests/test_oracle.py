"""The CPU oracle, pinned against the reference's own model (no GPU)."""

import numpy as np
import pytest
import torch

from oracle.online_softmax import direct_attention, online_softmax_attention
from oracle.sdpa_math import errors, sdpa_math_fp32


def test_golden_fixture_present(golden):
    assert len(golden) >= 10
    for name, c in golden.items():
        assert c["q"].dtype == np.float16 and c["out"].dtype == np.float32, name


@pytest.mark.parametrize("tile_n,threshold", [(16, 0.0), (128, 8.0), (7, 8.0), (128, 0.0)])
def test_online_softmax_matches_reference_model(golden, tile_n, threshold):
    """Restated tiled loop == reference attn_pair_model outputs (model_check.py:103-133)."""
    for name, c in golden.items():
        out = online_softmax_attention(c["q"], c["k"], c["v"], float(c["scale"]), tile_n, threshold)
        np.testing.assert_allclose(out, c["out"], atol=1e-5, rtol=1e-5, err_msg=name)


def test_sdpa_math_matches_reference_model(golden):
    """fp32 SDPA MATH (the reference's oracle) == reference model on the same inputs."""
    for name, c in golden.items():
        q, k, v = (torch.from_numpy(c[x]) for x in ("q", "k", "v"))
        ref = sdpa_math_fp32(q, k, v, float(c["scale"]))
        np.testing.assert_allclose(ref.numpy(), c["out"], atol=2e-5, rtol=1e-5, err_msg=name)


def test_chunked_oracle_is_exact_per_row():
    g = torch.Generator().manual_seed(3)
    q = torch.randn(1, 2, 300, 64, generator=g).half()
    k = torch.randn(1, 2, 257, 64, generator=g).half()
    v = torch.randn(1, 2, 257, 64, generator=g).half()
    full = sdpa_math_fp32(q, k, v, 0.125)
    chunked = sdpa_math_fp32(q, k, v, 0.125, q_chunk=37)
    assert torch.allclose(full, chunked, atol=1e-6)
    rows = sdpa_math_fp32(q, k, v, 0.125, rows=slice(100, 140))
    assert torch.allclose(full[:, :, 100:140], rows, atol=1e-6)


def test_lazy_rescale_threshold_is_exact():
    """Large, growing scores force the lazy-rescale path of the sm_100a tiling."""
    rng = np.random.default_rng(5)
    q = rng.standard_normal((1, 1, 20, 64)) * 3
    k = rng.standard_normal((1, 1, 600, 64)) * np.linspace(0.2, 3.0, 600)[:, None]
    v = rng.standard_normal((1, 1, 600, 64))
    ref = direct_attention(q, k, v, 0.125)
    for thr in (0.0, 8.0, 20.0):
        out = online_softmax_attention(q, k, v, 0.125, tile_n=128, threshold=thr)
        np.testing.assert_allclose(out, ref, atol=1e-9, rtol=1e-9)


def test_empty_keys_give_zero_rows():
    q = np.ones((1, 1, 3, 8))
    k = np.ones((1, 1, 0, 8))
    v = np.ones((1, 1, 0, 8))
    assert np.all(online_softmax_attention(q, k, v, 0.3) == 0)
    out = sdpa_math_fp32(torch.ones(1, 1, 3, 8), torch.ones(1, 1, 0, 8), torch.ones(1, 1, 0, 8), 0.3)
    assert out.shape == (1, 1, 3, 8) and torch.all(out == 0)


def test_error_metric():
    ref = torch.zeros(2, 2)
    out = torch.tensor([[0.0, 1e-3], [0.0, -3e-3]]).half()
    mx, mean = errors(out, ref)
    assert abs(mx - 3e-3) < 1e-5 and abs(mean - 1e-3) < 1e-5
