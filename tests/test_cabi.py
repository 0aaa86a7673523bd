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
