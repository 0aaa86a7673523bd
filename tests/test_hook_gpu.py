"""The ComfyUI DiT seam on the real sm_100a operator (needs a B200).

``_container_attn`` is what ComfyUI's ``optimized_attention.container_function``
calls for every DiT attention once ``install()`` ran
(deploy/gfx906_attention.py:52-79 in the reference). Here it runs with the real
eligibility rules, the real lazy loader and the real kernel; only the ComfyUI
containers are stand-ins (``peek``/``take``) and the stock attention it would
fall back to raises, so a silent fallback fails the test. Checked: the default
scale (SDPA's 1/sqrt(D)) and an explicit one, the [B,H,S,D] output
(``skip_output_reshape``) and the [B,S,H*D] one, and the bf16 -> fp16 -> bf16
cast path (the reference checks that cast at test_d512.py:32-37), all against
fp32 SDPA MATH on the fp16 inputs the kernel saw.
"""

import pytest
import torch

from gfx906_b200 import gfx906_attention as hook
from gfx906_b200.configs import make_qkv
from oracle.sdpa_math import errors, sdpa_math_fp32
from tests.gpu_util import MAX_ABS, MEAN_ABS

pytestmark = pytest.mark.gpu


class Box:
    """Stand-in for a ComfyUI q/k/v container: peek() looks, take() hands over."""

    def __init__(self, t):
        self.t = t
        self.taken = False

    def peek(self):
        return self.t

    def take(self):
        self.taken = True
        return self.t


def _no_stock(*args, **kwargs):
    raise AssertionError("an eligible call fell back to stock attention")


@pytest.fixture(autouse=True)
def stock_raises(monkeypatch):
    import gfx906_b200

    assert gfx906_b200.load_attention() is not None, gfx906_b200.last_error()
    monkeypatch.setattr(hook, "_stock_attention", _no_stock)


# (B, H, S, D): the C2 head layout scaled down so the oracle is quick, a D=64
# and a D<64 case, and the wide-head D=512 case with Sq != Skv
SHAPES = [(1, 24, 512, 512, 128), (2, 4, 300, 700, 64), (1, 3, 129, 257, 40), (1, 2, 256, 384, 512)]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("skip_output_reshape", [True, False])
@pytest.mark.parametrize("explicit_scale", [False, True])
@pytest.mark.parametrize("shape", SHAPES)
def test_container_attn_on_kernel(shape, dtype, skip_output_reshape, explicit_scale):
    B, H, Sq, Skv, D = shape
    q, k, v = make_qkv(B, H, Sq, Skv, D, seed=B * H + Sq + D)
    if dtype == torch.bfloat16:
        q, k, v = q.to(dtype), k.to(dtype), v.to(dtype)
    boxes = [Box(t.cuda()) for t in (q, k, v)]
    kwargs = {"scale": 0.7 * D ** -0.5} if explicit_scale else {}
    scale = kwargs.get("scale", D ** -0.5)
    out = hook._container_attn(*boxes, heads=H, skip_reshape=True, skip_output_reshape=skip_output_reshape,
                               **kwargs)
    torch.cuda.synchronize()
    assert all(b.taken for b in boxes)
    assert out.dtype == dtype and out.is_cuda
    # what the kernel saw: the fp16 copies of the inputs (bf16 is cast first)
    qh, kh, vh = q.half(), k.half(), v.half()
    ref = sdpa_math_fp32(qh, kh, vh, scale)  # fp32 [B,H,Sq,D]
    if skip_output_reshape:
        assert out.shape == (B, H, Sq, D)
        got = out
    else:
        assert out.shape == (B, Sq, H * D)
        got = out.reshape(B, Sq, H, D).transpose(1, 2)
    mx, mean = errors(got.cpu(), ref)
    if dtype == torch.float16:
        assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)
    else:
        # the fp16 result rounded to bf16: the bar plus half a bf16 ulp of |O|
        half_ulp = 2.0 ** -9 * ref.abs().max().item()
        assert mx <= MAX_ABS + half_ulp and mean <= MEAN_ABS + half_ulp / 4, (mx, mean)
        # and exactly the operator's fp16 output cast to bf16
        import gfx906_b200

        direct = gfx906_b200.attn(qh.cuda(), kh.cuda(), vh.cuda(), scale).to(dtype)
        if not skip_output_reshape:
            direct = direct.transpose(1, 2).reshape(B, Sq, H * D)
        assert torch.equal(out, direct)


def test_ineligible_call_goes_to_stock(monkeypatch):
    """A masked call is not the kernel's: the stock callable gets the containers' tensors."""
    seen = {}

    def stock(q, k, v, heads, mask=None, **kw):
        seen["mask"] = mask
        return "stock"

    monkeypatch.setattr(hook, "_stock_attention", stock)
    q, k, v = (t.cuda() for t in make_qkv(1, 2, 64, 64, 64, seed=1))
    mask = torch.zeros(64, 64, device="cuda")
    assert hook._container_attn(Box(q), Box(k), Box(v), heads=2, mask=mask, skip_reshape=True) == "stock"
    assert seen["mask"] is mask
