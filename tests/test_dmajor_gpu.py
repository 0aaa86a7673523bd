"""D=512 on transposed ("d-major") tensors: q [B,H,D,Sq], k, v [B,H,D,Skv], the
layout of a [b, c, h, w] VAE feature map (needs a B200)."""

import pytest
import torch

import gfx906_b200
from gfx906_b200 import build
from gfx906_b200.cabi import CABI, STATUS
from gfx906_b200.configs import make_qkv
from tests.gpu_util import check_rows, sample_rows

pytestmark = pytest.mark.gpu

# CTA pairs of 2 x 128 query rows: one tile (the odd CTA past Sq), three
# tiles (the second pair's odd CTA past Sq), ragged rows and keys, C4's heads
SHAPES = [(1, 1, 1024, 1024), (2, 1, 1000, 1000), (1, 2, 256, 1032), (1, 1, 8, 16), (1, 3, 136, 264),
          (1, 1, 4096, 4096), (1, 1, 384, 1000), (1, 4, 1024, 4096)]


def dmajor(t):  # [B,H,S,D] -> contiguous [B,H,D,S]
    return t.transpose(2, 3).contiguous()


@pytest.mark.parametrize("shape", SHAPES)
def test_dmajor_matches_oracle(shape):
    B, H, Sq, Skv = shape
    q, k, v = make_qkv(B, H, Sq, Skv, 512, seed=Sq + Skv)
    o = gfx906_b200.attn_dmajor(dmajor(q).cuda(), dmajor(k).cuda(), dmajor(v).cuda(), 512 ** -0.5)
    assert o.shape == (B, H, 512, Sq) and o.is_contiguous()
    out = o.cpu().transpose(2, 3)
    rows = None if B * H * Sq <= 4096 else sample_rows(Sq, n_each=48, seed=7)
    check_rows(out, q, k, v, 512 ** -0.5, rows, what=f"dmajor {shape}")
    # same kernel arithmetic as the row-major path, up to rounding of the final division
    ref = gfx906_b200.attn(q.cuda(), k.cuda(), v.cuda(), 512 ** -0.5).cpu()
    assert (out.float() - ref.float()).abs().max().item() <= 1e-3


def test_vae_hook_on_feature_maps():
    from gfx906_b200 import gfx906_attention as attention

    g = torch.Generator().manual_seed(9)
    b, c, h, w = 2, 512, 32, 24
    q, k, v = (torch.randn(b, c, h, w, generator=g).half().cuda() for _ in range(3))
    out = attention._vae_attn(q, k, v, lambda *a: pytest.fail("fallback used"))
    assert out.shape == (b, c, h, w) and out.dtype == torch.float16
    seq = lambda t: t.reshape(b, c, h * w).transpose(1, 2).unsqueeze(1).cpu()  # noqa: E731
    ref = gfx906_b200.attn(seq(q).cuda(), seq(k).cuda(), seq(v).cuda(), c ** -0.5)
    ref = ref.squeeze(1).transpose(1, 2).reshape(b, c, h, w)
    assert (out.float() - ref.float()).abs().max().item() <= 1e-3
    check_rows(seq(out.float()).half(), seq(q), seq(k), seq(v), c ** -0.5, sample_rows(h * w, n_each=32, seed=1),
               what="VAE feature maps")


def test_dmajor_argument_errors():
    lib = CABI(build.LIB_PATH)
    q = torch.zeros(1, 1, 512, 1024, dtype=torch.float16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    p = q.data_ptr()
    assert lib.launch_dmajor_status(p, p, p, p, 1, 1, 1020, 1024, 512, 0.1, st) == STATUS["EALIGN"]
    assert lib.launch_dmajor_status(p, p, p, p, 1, 1, 1024, 1020, 512, 0.1, st) == STATUS["EALIGN"]
    assert lib.launch_dmajor_status(p, p, p, p, 1, 1, 128, 128, 128, 0.1, st) == STATUS["EHEADDIM"]
    o = torch.full_like(q, 1.0)
    assert lib.launch_dmajor_status(p, None, None, o.data_ptr(), 1, 1, 1024, 0, 512, 0.1, st) == STATUS["OK"]
    torch.cuda.synchronize()
    assert o.abs().sum().item() == 0  # no keys: zeros
    with pytest.raises(RuntimeError):
        gfx906_b200.attn_dmajor(q[..., :1020], q[..., :1020], q[..., :1020], 0.1)
    assert lib.device_status(reset=False) == STATUS["OK"]
