"""The allocation-free entry point against the workspace entry point (needs a B200).

gfx906_b200_attn_launch_noalloc serves callers that cannot allocate device
memory (their host runtime owns it, or their memory budget is fixed, or the
call sits on a latency-critical path where cudaMalloc/cudaFree lock or
synchronise). It runs the split schedule with its scratch in a fixed array
inside the library. This file is collected last so that a failure here, in a
run that stops at the first failure, comes after every other test.
"""

import pytest
import torch

from gfx906_b200 import build
from gfx906_b200.cabi import CABI, STATUS
from gfx906_b200.configs import make_qkv
from tests.gpu_util import MAX_ABS, MEAN_ABS

pytestmark = pytest.mark.gpu

# Shapes whose plan splits the key range (so the scratch array is used).
SHAPES = [(1, 1, 16384, 16384, 64), (1, 3, 300, 2000, 128), (1, 4, 16384, 16384, 128)]


@pytest.fixture(scope="module")
def lib():
    import gfx906_b200

    assert gfx906_b200.load_attention() is not None, gfx906_b200.last_error()
    return CABI(build.LIB_PATH)


@pytest.mark.parametrize("shape", SHAPES)
def test_noalloc_matches_workspace_entry_twice(lib, shape):
    B, H, Sq, Skv, D = shape
    need = lib.workspace_size(B, H, Sq, Skv, D)
    assert 0 < need <= lib.dll.gfx906_b200_attn_noalloc_capacity()
    q, k, v = make_qkv(B, H, Sq, Skv, D, seed=Sq + D, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    ref = torch.empty_like(q)
    assert lib.launch_ws_status(q.data_ptr(), k.data_ptr(), v.data_ptr(), ref.data_ptr(), B, H, Sq, Skv, D,
                                D ** -0.5, ws.data_ptr(), need, st) == STATUS["OK"]
    for _ in range(2):  # two calls in a row on the shared array
        out = torch.empty_like(q)
        rc = lib.launch_noalloc_status(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H, Sq, Skv, D,
                                       D ** -0.5, st)
        assert rc == STATUS["OK"], lib.error_string(rc)
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs()
        assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS
    assert lib.device_status(reset=False) == STATUS["OK"]


def test_noalloc_rejects_bad_arguments(lib):
    assert lib.launch_noalloc_status(None, None, None, None, 1, 1, 8, 8, 100, 0.1) == STATUS["EHEADDIM"]
    assert lib.error_string(STATUS["ENOSPACE"]) != "unknown status"
