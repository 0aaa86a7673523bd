"""Failure detection of the bounded mbarrier waits, without faulting the GPU.

A one-block kernel waits on an mbarrier that nothing arrives at; its wait has
a short limit, after which it sets the device status word and returns. The
host reads the status, and the context stays usable for real work.
"""

import pytest
import torch

from gfx906_b200 import build
from gfx906_b200.cabi import CABI, STATUS
from gfx906_b200.configs import make_qkv
from tests.gpu_util import check_rows

pytestmark = pytest.mark.gpu


def test_wait_timeout_sets_status_and_context_survives():
    import gfx906_b200

    mod = gfx906_b200.load_attention()
    assert mod is not None, gfx906_b200.last_error()
    lib = CABI(build.LIB_PATH)
    torch.cuda.synchronize()
    assert lib.device_status(reset=True) == STATUS["OK"]
    assert lib.dll.gfx906_b200_attn_selftest_wait_timeout(50_000_000, None) == STATUS["OK"]  # 50 ms
    assert lib.device_status(reset=False) == STATUS["ETIMEOUT"]
    rc, info = lib.timeout_info()
    assert rc == STATUS["OK"] and info[3] == 0  # barrier index 0 of the self-test block
    assert lib.device_status(reset=True) == STATUS["ETIMEOUT"]
    assert lib.device_status(reset=False) == STATUS["OK"]
    # the context is still usable
    q, k, v = make_qkv(1, 2, 300, 300, 64, seed=3)
    out = mod.attn(q.cuda(), k.cuda(), v.cuda(), 0.125).cpu()
    check_rows(out, q, k, v, 0.125, what="after timeout")
    assert mod.device_status(False) == 0
