"""The two schedules through the C ABI, against the CPU oracle (needs a B200).

gfx906_b200_attn_launch (no workspace): every CTA takes whole 256-row query
blocks. gfx906_b200_attn_launch_ws: the key range is split across CTAs and
partial results are combined on the GPU.
"""

import pytest
import torch

from gfx906_b200 import build
from gfx906_b200.cabi import CABI, STATUS
from gfx906_b200.configs import make_qkv
from tests.gpu_util import check_rows, sample_rows

pytestmark = pytest.mark.gpu

SHAPES = [(1, 8, 1024, 1024, 64), (1, 24, 4096, 4096, 128), (2, 16, 4096, 1024, 128),
          (1, 1, 16384, 16384, 64), (1, 3, 300, 2000, 128), (3, 5, 777, 1500, 32),
          (1, 2, 100, 129, 128), (1, 1, 129, 5000, 16),
          # D = 512 on CTA pairs: C4 (whole units over 74 clusters), one 8-GPU
          # rank's shard of C4 (16 units: split with a workspace), an odd
          # number of query tiles (the last pair's odd CTA past Sq), ragged keys
          (1, 4, 4096, 4096, 512), (1, 4, 512, 4096, 512), (1, 1, 384, 1000, 512), (3, 5, 640, 2000, 512),
          (2, 4, 77, 411, 512)]


@pytest.fixture(scope="module")
def lib():
    import gfx906_b200

    assert gfx906_b200.load_attention() is not None, gfx906_b200.last_error()
    return CABI(build.LIB_PATH)


def run(lib, q, k, v, scale, use_ws, ws_cache):
    B, H, Sq, D = q.shape
    Skv = k.shape[2]
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    o = torch.empty_like(qd)
    st = torch.cuda.current_stream().cuda_stream
    if use_ws:
        n = lib.workspace_size(B, H, Sq, Skv, D)
        if n and (ws_cache.get("t") is None or ws_cache["t"].numel() < n):
            ws_cache["t"] = torch.empty(n, dtype=torch.uint8, device="cuda")
        ws = ws_cache["t"].data_ptr() if n else None
        rc = lib.launch_ws_status(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), o.data_ptr(), B, H, Sq, Skv,
                                  D, scale, ws, n, st)
    else:
        rc = lib.launch_status(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), o.data_ptr(), B, H, Sq, Skv, D,
                               scale, st)
    assert rc == STATUS["OK"], lib.error_string(rc)
    torch.cuda.synchronize()
    return o.cpu()


@pytest.mark.parametrize("use_ws", [False, True])
@pytest.mark.parametrize("shape", SHAPES)
def test_schedules_match_oracle(lib, shape, use_ws):
    B, H, Sq, Skv, D = shape
    q, k, v = make_qkv(B, H, Sq, Skv, D, seed=Sq + Skv)
    cache = {}
    out = run(lib, q, k, v, D ** -0.5, use_ws, cache)
    rows = None if B * H * Sq <= 8192 else sample_rows(Sq, n_each=96, seed=D)
    check_rows(out, q, k, v, D ** -0.5, rows, what=f"{shape} ws={use_ws}")
    if use_ws:
        # the workspace is reusable: a second call on it gives the same bits
        out2 = run(lib, q, k, v, D ** -0.5, use_ws, cache)
        assert torch.equal(out, out2)


def test_workspace_size_and_checks(lib):
    assert lib.workspace_size(1, 1, 256, 100, 512) == 0  # D=512, one key tile: whole units
    assert lib.workspace_size(1, 4, 4096, 4096, 512) == 0  # D=512, C4: whole units on 74 clusters
    assert lib.workspace_size(1, 4, 512, 4096, 512) > 0  # D=512, 16 units < 74 clusters: split
    assert lib.workspace_size(1, 4, 1024, 0, 64) == 0
    assert lib.workspace_size(1, 4, 1024, 1024, 100) == 0
    assert lib.workspace_size(2, 16, 4096, 1024, 128) == 0  # 8 key tiles per unit: never split
    assert lib.workspace_size(1, 40, 2048, 2048, 128) == 0  # 16 key tiles: the partial last wave is not split
    assert lib.workspace_size(1, 24, 4096, 4096, 128) > 0  # 32 key tiles: the partial last wave is split
    assert lib.workspace_size(1, 1, 131072, 131072, 64) > 0  # 1024 key tiles: the tail is split
    n = lib.workspace_size(1, 8, 16384, 16384, 128)  # 512 units of 128 key tiles: tail split
    assert n > 0
    q, k, v = make_qkv(1, 8, 16384, 16384, 128, device="cuda")
    o = torch.empty_like(q)
    small = torch.zeros(256, dtype=torch.uint8, device="cuda")
    rc = lib.launch_ws_status(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), 1, 8, 16384, 16384, 128,
                              0.1, small.data_ptr(), 256, torch.cuda.current_stream().cuda_stream)
    assert rc == STATUS["EINVAL"]
    assert lib.device_status(reset=False) == STATUS["OK"]


def test_workspace_contents_do_not_matter(lib):
    """Garbage in the workspace (any bytes, earlier calls of other sizes) changes nothing."""
    shape = (1, 4, 16384, 16384, 128)
    B, H, Sq, Skv, D = shape
    q, k, v = make_qkv(B, H, Sq, Skv, D, seed=5)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    n = lib.workspace_size(B, H, Sq, Skv, D)
    assert n > 0
    st = torch.cuda.current_stream().cuda_stream
    outs = []
    for fill in ("zeros", "ones", "random", "other-size-call"):
        ws = torch.zeros(n + 4096, dtype=torch.uint8, device="cuda")
        if fill == "ones":
            ws.fill_(255)
        elif fill == "random":
            ws.random_(0, 256)
        elif fill == "other-size-call":
            q2, k2, v2 = make_qkv(2, 7, 900, 4100, 128, seed=6, device="cuda")
            o2 = torch.empty_like(q2)
            n2 = lib.workspace_size(2, 7, 900, 4100, 128)
            assert n2 <= ws.numel()
            assert lib.launch_ws_status(q2.data_ptr(), k2.data_ptr(), v2.data_ptr(), o2.data_ptr(), 2, 7, 900,
                                        4100, 128, 0.1, ws.data_ptr(), ws.numel(), st) == STATUS["OK"]
        o = torch.empty_like(qd)
        rc = lib.launch_ws_status(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), o.data_ptr(), B, H, Sq, Skv, D,
                                  D ** -0.5, ws.data_ptr(), ws.numel(), st)
        assert rc == STATUS["OK"]
        torch.cuda.synchronize()
        outs.append(o.cpu())
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    check_rows(outs[0], q, k, v, D ** -0.5, sample_rows(Sq, n_each=64, seed=3), what="ws garbage")


def test_workspace_shared_between_library_instances(lib, tmp_path):
    """A second copy of the library (its own launch epochs) reuses a workspace
    the first one left behind: its split counters must not be mistaken for
    the new launch's."""
    import shutil

    copy = tmp_path / "libgfx906_b200_attn_copy.so"
    shutil.copy(build.LIB_PATH, copy)
    lib2 = CABI(str(copy))
    shape = (1, 4, 16384, 16384, 128)
    B, H, Sq, Skv, D = shape
    q, k, v = make_qkv(B, H, Sq, Skv, D, seed=8)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    n = lib.workspace_size(B, H, Sq, Skv, D)
    assert n > 0 and lib2.workspace_size(B, H, Sq, Skv, D) == n
    ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    outs = []
    for which in (lib, lib2, lib, lib2):
        o = torch.full_like(qd, float("nan"))
        rc = which.launch_ws_status(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), o.data_ptr(), B, H, Sq, Skv, D,
                                    D ** -0.5, ws.data_ptr(), n, st)
        assert rc == STATUS["OK"]
        torch.cuda.synchronize()
        outs.append(o.cpu())
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    assert not torch.isnan(outs[0]).any()
    check_rows(outs[0], q, k, v, D ** -0.5, sample_rows(Sq, n_each=32, seed=8), what="two library instances")
    assert lib.device_status(reset=False) == STATUS["OK"]
    assert lib2.device_status(reset=False) == STATUS["OK"]


@pytest.mark.parametrize("limit", [140, 137])
def test_sm_limit_caps_the_grid(lib, limit):
    """With the SMs capped (as a sharded pipeline does to leave SMs to NCCL)
    every schedule plans at most `limit` CTAs (D = 512: limit // 2 clusters)
    and still matches the oracle, workspace sized for the capped plan."""
    shapes = [(1, 1, 4096, 32768, 64), (1, 24, 4096, 4096, 128), (1, 4, 512, 4096, 512), (1, 4, 4096, 4096, 512)]
    prev = lib.set_sm_limit(limit)
    try:
        for shape in shapes:
            B, H, Sq, Skv, D = shape
            rc, pl = lib.plan(B, H, Sq, Skv, D, with_workspace=True)
            assert rc == STATUS["OK"]
            assert pl["ctas"] <= (limit if D != 512 else 2 * (limit // 2)), (shape, pl)
            q, k, v = make_qkv(B, H, Sq, Skv, D, seed=limit + D)
            out = run(lib, q, k, v, D ** -0.5, True, {})
            check_rows(out, q, k, v, D ** -0.5, sample_rows(Sq, n_each=32, seed=D), what=f"{shape} limit={limit}")
    finally:
        assert lib.set_sm_limit(prev) == limit
    rc, pl = lib.plan(1, 24, 4096, 4096, 128, with_workspace=True)
    assert pl["ctas"] == torch.cuda.get_device_properties(0).multi_processor_count
