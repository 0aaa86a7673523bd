"""The C-ABI library loads and exports what include/gfx906_b200_attn.h declares.

Only argument validation is exercised here (it returns before any CUDA call);
compute calls need a GPU and live in the gpu-marked tests.
"""

import ctypes
import re

import pytest

from gfx906_b200 import build
from gfx906_b200.cabi import CABI, STATUS

HEADER = build.INCLUDE / "gfx906_b200_attn.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^GFX906_B200_API\s+[\w\s\*]*?\b(\w+)\s*\(", text, re.M)))


def declared_status_codes():
    return dict((m[0], int(m[1])) for m in re.findall(r"#define (GFX906_B200_E?\w+) (\d+)", HEADER.read_text()))


@pytest.fixture(scope="module")
def lib():
    return CABI(build.build_library())


def test_header_declares_the_reference_entry_point():
    names = declared_functions()
    assert "launch" in names and "gfx906_b200_attn_launch" in names
    assert len(names) >= 8


def test_every_declared_symbol_is_exported(lib):
    for name in declared_functions():
        assert hasattr(lib.dll, name), name


def test_status_codes_match_header():
    assert declared_status_codes() == {f"GFX906_B200_{k}": v for k, v in STATUS.items()}


def test_argument_validation_without_gpu(lib):
    # unsupported head dims return before touching CUDA
    for d in (0, 4, 12, 72, 96, 100, 256, 1024):
        assert lib.launch_status(None, None, None, None, 1, 1, 8, 8, d, 0.1) == STATUS["EHEADDIM"], d
    assert lib.launch_status(None, None, None, None, -1, 1, 8, 8, 64, 0.1) == STATUS["EINVAL"]
    assert lib.launch_status(None, None, None, None, 1, 1, 8, -8, 64, 0.1) == STATUS["EINVAL"]
    # empty problems are a no-op success
    assert lib.launch_status(None, None, None, None, 0, 4, 8, 8, 64, 0.1) == STATUS["OK"]
    assert lib.launch_status(None, None, None, None, 1, 4, 0, 8, 64, 0.1) == STATUS["OK"]
    # null or misaligned pointers on a non-empty problem
    assert lib.launch_status(None, None, None, None, 1, 1, 8, 8, 64, 0.1) == STATUS["EINVAL"]
    p, bad = 4096, 4096 + 8
    assert lib.launch_status(p, p, bad, p, 1, 1, 8, 8, 64, 0.1) == STATUS["EALIGN"]


def test_void_launch_records_last_error(lib):
    lib.dll.launch(None, None, None, None, 1, 1, 8, 8, 100, ctypes.c_float(0.1), None)
    assert lib.dll.gfx906_b200_attn_last_error() == STATUS["EHEADDIM"]
    lib.dll.launch(None, None, None, None, 0, 1, 8, 8, 64, ctypes.c_float(0.1), None)
    assert lib.dll.gfx906_b200_attn_last_error() == STATUS["OK"]


def test_error_strings_and_flops(lib):
    for code in STATUS.values():
        s = lib.error_string(code)
        assert s and s != "unknown status"
    assert lib.error_string(999) == "unknown status"
    assert lib.dll.gfx906_b200_attn_flops(1, 24, 4096, 4096, 128) == 4.0 * 24 * 4096 * 4096 * 128


B200_SMS = 148


def plan(lib, *shape, ws=True, sms=B200_SMS):
    rc, pl = lib.plan(*shape, with_workspace=ws, num_sms=sms)
    assert rc == STATUS["OK"], lib.error_string(rc)
    return pl


def test_plan_fills_a_b200_for_small_row_shards(lib):
    """One 8-GPU rank's shard of one long head (C5 at S=32768: 4096 query rows
    x 32768 keys, 16 units of 256 rows x 256 key tiles) gets every SM."""
    pl = plan(lib, 1, 1, 4096, 32768, 64)
    # ~9 CTAs per unit: the pieces are combined by a second kernel
    assert pl["split"] == 2 and pl["ctas"] == B200_SMS and pl["tail_ctas"] == B200_SMS
    assert pl["unit_rows"] == 256
    # C5 at S=131072 on 8 GPUs (64 units per rank) and on one GPU
    assert plan(lib, 1, 1, 16384, 131072, 64)["ctas"] == B200_SMS
    assert plan(lib, 1, 1, 131072, 131072, 64)["ctas"] == B200_SMS
    # two units: at most 31 CTAs share a unit's key range
    pl = plan(lib, 1, 1, 512, 4096, 64)
    assert pl["split"] == 2 and pl["ctas"] <= 31 * 2
    # C5 and C5 at S=32768 on one GPU: few pieces per unit, combined in the kernel
    assert plan(lib, 1, 1, 131072, 131072, 64)["split"] == 1
    assert plan(lib, 1, 1, 32768, 32768, 64)["split"] == 1


def test_plan_short_units(lib):
    # C1: 8 key tiles per unit, too few units for half the SMs: whole 128-row
    # units (64 CTAs; splitting them over 128 CTAs measured slower)
    for ws in (True, False):
        assert plan(lib, 1, 8, 1024, 1024, 64, ws=ws) == {"ctas": 64, "split": 0, "tail_ctas": 0, "unit_rows": 128}
    # C3: 512 units of 8 key tiles stay whole on every SM
    assert plan(lib, 2, 16, 4096, 1024, 128) == {"ctas": 148, "split": 0, "tail_ctas": 0, "unit_rows": 256}
    # C2: the partial last wave of 32-key-tile units is split
    pl = plan(lib, 1, 24, 4096, 4096, 128)
    assert pl["split"] == 1 and pl["ctas"] == 148
    # D=512 on CTA pairs: C4's 128 units (query-tile pairs x head-dim halves)
    # run whole on 74 clusters; one 8-GPU rank's shard of C4 (16 units) is split
    # over all 74
    for ws in (True, False):
        assert plan(lib, 1, 4, 4096, 4096, 512, ws=ws) == {"ctas": 148, "split": 0, "tail_ctas": 0, "unit_rows": 256}
    assert plan(lib, 1, 4, 512, 4096, 512) == {"ctas": 148, "split": 2, "tail_ctas": 148, "unit_rows": 256}
    assert plan(lib, 1, 4, 512, 4096, 512, ws=False)["ctas"] == 32
    # 4 units of one key tile: whole units, one cluster each
    assert plan(lib, 1, 1, 256, 100, 512) == {"ctas": 4, "split": 0, "tail_ctas": 0, "unit_rows": 256}


def test_plan_argument_checks(lib):
    buf = (ctypes.c_int * 4)()
    assert lib.dll.gfx906_b200_attn_plan(1, 1, 8, 8, 64, 1, 148, None) == STATUS["EINVAL"]
    assert lib.dll.gfx906_b200_attn_plan(1, 1, 8, 8, 100, 1, 148, buf) == STATUS["EHEADDIM"]
    assert lib.dll.gfx906_b200_attn_plan(1, 1, 8, 0, 64, 1, 148, buf) == STATUS["OK"] and list(buf) == [0] * 4


def test_noalloc_records_argument_errors(lib):
    assert lib.launch_noalloc_status(None, None, None, None, 1, 1, 8, 8, 100, 0.1) == STATUS["EHEADDIM"]
    assert lib.last_error() == STATUS["EHEADDIM"]
    assert lib.launch_noalloc_status(None, None, None, None, 0, 1, 8, 8, 64, 0.1) == STATUS["OK"]
    assert lib.last_error() == STATUS["OK"]


def test_sm_limit_round_trip(lib):
    """The SM cap is process-wide state: set returns the previous value and
    values <= 0 mean no cap (no GPU needed to set it)."""
    assert lib.set_sm_limit(100) == 0
    assert lib.set_sm_limit(-5) == 100
    assert lib.set_sm_limit(0) == 0
