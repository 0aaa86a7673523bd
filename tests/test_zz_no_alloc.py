"""The allocation-free entry point against the workspace entry point (needs a B200).

gfx906_b200_attn_launch_noalloc serves callers that cannot allocate device
memory: a plugin whose host runtime owns every device allocation and hands it
only tensors and a stream, an application that reserves a fixed memory budget
at start-up, or code on a latency-critical path where cudaMalloc/cudaFree take
a driver-wide lock or synchronise the device. It runs the same schedule as
gfx906_b200_attn_launch_ws with the scratch in a fixed array inside the
library, so for the same inputs it must give the same bits.

The shapes run back to back in one module on the one shared array, each twice
in a row, without clearing anything in between. This file is collected last
so that a failure here, in a run that stops at the first failure, comes after
every other test.
"""

import pytest
import torch

from gfx906_b200 import build
from gfx906_b200.cabi import CABI, STATUS
from gfx906_b200.configs import make_qkv
from tests.gpu_util import check_rows, sample_rows

pytestmark = pytest.mark.gpu

# Split shapes (the scratch array is used) of different sizes, then shapes
# that do not split (no scratch: the call forwards to the workspace entry
# with none).
SPLIT_SHAPES = [(1, 1, 16384, 16384, 64), (1, 3, 300, 2000, 128), (1, 4, 16384, 16384, 128),
                (1, 1, 4096, 32768, 64), (1, 2, 1024, 1024, 512), (1, 4, 512, 4096, 512)]
WHOLE_SHAPES = [(2, 16, 4096, 1024, 128), (1, 8, 1024, 1024, 64), (1, 1, 256, 100, 512), (1, 4, 4096, 4096, 512)]


@pytest.fixture(scope="module")
def lib():
    import gfx906_b200

    assert gfx906_b200.load_attention() is not None, gfx906_b200.last_error()
    return CABI(build.LIB_PATH)


def _launch_ws(lib, q, k, v, shape, st):
    B, H, Sq, Skv, D = shape
    need = lib.workspace_size(B, H, Sq, Skv, D)
    ws = torch.empty(max(need, 256), dtype=torch.uint8, device="cuda")
    ref = torch.empty_like(q)
    rc = lib.launch_ws_status(q.data_ptr(), k.data_ptr(), v.data_ptr(), ref.data_ptr(), B, H, Sq, Skv, D,
                              D ** -0.5, ws.data_ptr() if need else None, need, st)
    assert rc == STATUS["OK"], lib.error_string(rc)
    return ref, need


def _check_twice(lib, shape, expect_split):
    B, H, Sq, Skv, D = shape
    q, k, v = make_qkv(B, H, Sq, Skv, D, seed=Sq + D)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    st = torch.cuda.current_stream().cuda_stream
    ref, need = _launch_ws(lib, qd, kd, vd, shape, st)
    assert (need > 0) == expect_split
    assert need <= lib.dll.gfx906_b200_attn_noalloc_capacity()
    for _ in range(2):  # two calls in a row on the shared array
        out = torch.full_like(qd, float("nan"))
        rc = lib.launch_noalloc_status(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr(), B, H, Sq,
                                       Skv, D, D ** -0.5, st)
        assert rc == STATUS["OK"], lib.error_string(rc)
        assert lib.last_error() == STATUS["OK"]
        torch.cuda.synchronize()
        # same schedule, same deterministic combine: the same bits
        assert torch.equal(out, ref), shape
    rows = None if B * H * Sq <= 8192 else sample_rows(Sq, n_each=48, seed=D)
    check_rows(out.cpu(), q, k, v, D ** -0.5, rows, what=f"noalloc {shape}")
    assert lib.device_status(reset=False) == STATUS["OK"]


@pytest.mark.parametrize("shape", SPLIT_SHAPES)
def test_noalloc_split_matches_workspace_entry_twice(lib, shape):
    _check_twice(lib, shape, expect_split=True)


@pytest.mark.parametrize("shape", WHOLE_SHAPES)
def test_noalloc_unsplit_matches_workspace_entry_twice(lib, shape):
    _check_twice(lib, shape, expect_split=False)


def test_noalloc_rejects_bad_arguments(lib):
    assert lib.launch_noalloc_status(None, None, None, None, 1, 1, 8, 8, 100, 0.1) == STATUS["EHEADDIM"]
    assert lib.last_error() == STATUS["EHEADDIM"]
    assert lib.error_string(STATUS["ENOSPACE"]) != "unknown status"
