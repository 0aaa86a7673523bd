"""attn_host argument checks that need no GPU."""

import pytest
import torch

import gfx906_b200


def _qkv(dtype=torch.float16):
    q = torch.zeros(1, 2, 8, 16, dtype=dtype)
    return q, q.clone(), q.clone()


def test_rejects_wrong_dtype_and_layout():
    q, k, v = _qkv(torch.float32)
    with pytest.raises(ValueError):
        gfx906_b200.attn_host(q, k, v, 0.25)
    q, k, v = _qkv()
    with pytest.raises(ValueError):
        gfx906_b200.attn_host(q.transpose(1, 2), k, v, 0.25)
    with pytest.raises(ValueError):
        gfx906_b200.attn_host(q, k[:, :1], v, 0.25)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path")
def test_fails_loudly_without_cuda():
    q, k, v = _qkv()
    with pytest.raises(RuntimeError):
        gfx906_b200.attn_host(q, k, v, 0.25)
