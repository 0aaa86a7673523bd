"""The reference's own binding, restated for CUDA, on this library (needs a B200).

tests/ref_binding/attn_cuda_binding.cpp is the reference's attn.cpp (its
`extern "C" void launch(...)` declaration, checks, .contiguous() copies and
current-stream launch, attn.cpp:1-21) with the HIP names replaced by CUDA
ones. It links against libgfx906_b200_attn.so and calls the bare `launch`
symbol (attn_kernel.hip:710-711's signature), so these tests compute through
exactly the entry point a drop-in replacement of the reference's kernel object
must provide.
"""

import ctypes

import pytest
import torch

from gfx906_b200 import build
from gfx906_b200.cabi import CABI, STATUS
from gfx906_b200.configs import make_qkv
from tests.gpu_util import check_rows, sample_rows

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def binding():
    from tests.ref_binding import build_binding

    return build_binding.load()


@pytest.fixture(scope="module")
def lib():
    return CABI(build.LIB_PATH)


# the reference's test lists: test.py:23-27 (D=64, odd lengths, D=32/16),
# test_variants.py:78-80 (Sq != Skv), test_d512.py:19-20 (D=512), plus C2's heads
SHAPES = [(2, 8, 64, 64, 64), (2, 8, 1000, 1000, 64), (2, 8, 512, 512, 32), (2, 8, 512, 512, 16),
          (2, 4, 100, 300, 64), (2, 4, 77, 411, 128), (2, 4, 512, 512, 512), (1, 24, 4096, 4096, 128),
          (1, 1, 1024, 4096, 512)]


@pytest.mark.parametrize("shape", SHAPES)
def test_reference_binding_calls_launch(binding, lib, shape):
    B, H, Sq, Skv, D = shape
    q, k, v = make_qkv(B, H, Sq, Skv, D, seed=Sq * 3 + D)
    scale = D ** -0.5
    out = binding.attn(q.cuda(), k.cuda(), v.cuda(), scale)
    torch.cuda.synchronize()
    # launch() returns void; its status is kept for gfx906_b200_attn_last_error
    # on the calling thread (the binding and ctypes share the one library)
    assert lib.last_error() == STATUS["OK"]
    assert out.shape == (B, H, Sq, D) and out.dtype == torch.float16
    rows = None if B * H * Sq <= 16384 else sample_rows(Sq, n_each=64, seed=D)
    check_rows(out.cpu(), q, k, v, scale, rows, what=f"reference binding {shape}")


def test_reference_binding_noncontiguous_inputs(binding, lib):
    """test_d512.py:22-30: strided and transposed views go through .contiguous()."""
    g = torch.Generator().manual_seed(7)
    b, S, D = 1, 1024, 512
    q = torch.randn(b, S, 2 * D, generator=g).half()[:, :, ::2].unsqueeze(1)
    k = torch.randn(b, D, S, generator=g).half().transpose(1, 2).unsqueeze(1)
    v = torch.randn(b, D, S, generator=g).half().transpose(1, 2).unsqueeze(1)
    out = binding.attn(q.cuda(), k.cuda(), v.cuda(), D ** -0.5)
    torch.cuda.synchronize()
    assert lib.last_error() == STATUS["OK"]
    check_rows(out.cpu(), q.contiguous(), k.contiguous(), v.contiguous(), D ** -0.5, what="non-contiguous")


def test_bare_launch_status_on_bad_head_dim(lib):
    """The void launch() reports through last_error (the reference never checked)."""
    lib.dll.launch(None, None, None, None, 1, 1, 8, 8, 96, ctypes.c_float(0.1), None)
    assert lib.last_error() == STATUS["EHEADDIM"]


def test_reference_binding_rejects_like_the_reference(binding):
    q = torch.zeros(1, 1, 8, 96, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="head_dim"):
        binding.attn(q, q, q, 0.1)
    with pytest.raises(RuntimeError):
        binding.attn(q.float(), q, q, 0.1)
