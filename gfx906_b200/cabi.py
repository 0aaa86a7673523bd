"""ctypes binding of the C-ABI library (``include/gfx906_b200_attn.h``).

This is the stub a host application without torch would write to call the
library; the tests use it to check the exported surface and to drive the
C-ABI directly with device pointers.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

STATUS = {"OK": 0, "EINVAL": 1, "EHEADDIM": 2, "EALIGN": 3, "ENODEV": 4, "ECUDA": 5, "ETIMEOUT": 6,
          "ENOSPACE": 7}

_c_int, _c_void_p, _c_float = ctypes.c_int, ctypes.c_void_p, ctypes.c_float


class CABI:
    """Loaded ``libgfx906_b200_attn.so`` with typed entry points."""

    def __init__(self, path):
        self.path = Path(path)
        self.dll = ctypes.CDLL(str(self.path))
        d = self.dll
        sig = [_c_void_p] * 4 + [_c_int] * 5 + [_c_float, _c_void_p]
        d.launch.argtypes, d.launch.restype = sig, None
        d.gfx906_b200_attn_launch.argtypes, d.gfx906_b200_attn_launch.restype = sig, _c_int
        d.gfx906_b200_attn_last_error.argtypes, d.gfx906_b200_attn_last_error.restype = [], _c_int
        d.gfx906_b200_attn_error_string.argtypes = [_c_int]
        d.gfx906_b200_attn_error_string.restype = ctypes.c_char_p
        d.gfx906_b200_attn_device_status.argtypes = [_c_int]
        d.gfx906_b200_attn_device_status.restype = _c_int
        d.gfx906_b200_attn_timeout_info.argtypes = [ctypes.POINTER(_c_int)]
        d.gfx906_b200_attn_timeout_info.restype = _c_int
        d.gfx906_b200_attn_selftest_wait_timeout.argtypes = [ctypes.c_ulonglong, _c_void_p]
        d.gfx906_b200_attn_selftest_wait_timeout.restype = _c_int
        d.gfx906_b200_attn_workspace_size.argtypes = [_c_int] * 5
        d.gfx906_b200_attn_workspace_size.restype = ctypes.c_size_t
        d.gfx906_b200_attn_launch_ws.argtypes = sig[:-1] + [_c_void_p, ctypes.c_size_t, _c_void_p]
        d.gfx906_b200_attn_launch_ws.restype = _c_int
        d.gfx906_b200_attn_launch_dmajor.argtypes = sig
        d.gfx906_b200_attn_launch_dmajor.restype = _c_int
        d.gfx906_b200_attn_launch_noalloc.argtypes = sig
        d.gfx906_b200_attn_launch_noalloc.restype = _c_int
        d.gfx906_b200_attn_noalloc_capacity.argtypes = []
        d.gfx906_b200_attn_noalloc_capacity.restype = ctypes.c_size_t
        d.gfx906_b200_attn_plan.argtypes = [_c_int] * 7 + [ctypes.POINTER(_c_int)]
        d.gfx906_b200_attn_plan.restype = _c_int
        d.gfx906_b200_attn_set_sm_limit.argtypes, d.gfx906_b200_attn_set_sm_limit.restype = [_c_int], _c_int
        d.gfx906_b200_attn_flops.argtypes = [_c_int] * 5
        d.gfx906_b200_attn_flops.restype = ctypes.c_double

    def launch_status(self, q, k, v, o, B, H, Sq, Skv, D, scale, stream=None) -> int:
        return self.dll.gfx906_b200_attn_launch(q, k, v, o, B, H, Sq, Skv, D, _c_float(scale), stream)

    def launch_ws_status(self, q, k, v, o, B, H, Sq, Skv, D, scale, ws, ws_bytes, stream=None) -> int:
        return self.dll.gfx906_b200_attn_launch_ws(q, k, v, o, B, H, Sq, Skv, D, _c_float(scale), ws,
                                                   ws_bytes, stream)

    def launch_noalloc_status(self, q, k, v, o, B, H, Sq, Skv, D, scale, stream=None) -> int:
        return self.dll.gfx906_b200_attn_launch_noalloc(q, k, v, o, B, H, Sq, Skv, D, _c_float(scale), stream)

    def launch_dmajor_status(self, q, k, v, o, B, H, Sq, Skv, D, scale, stream=None) -> int:
        return self.dll.gfx906_b200_attn_launch_dmajor(q, k, v, o, B, H, Sq, Skv, D, _c_float(scale), stream)

    def workspace_size(self, B, H, Sq, Skv, D) -> int:
        return self.dll.gfx906_b200_attn_workspace_size(B, H, Sq, Skv, D)

    def plan(self, B, H, Sq, Skv, D, with_workspace=True, num_sms=0):
        """(status, {"ctas", "split", "tail_ctas", "unit_rows"}) of the schedule a launch
        would use on a GPU with num_sms SMs (0: the current device)."""
        buf = (_c_int * 4)()
        rc = self.dll.gfx906_b200_attn_plan(B, H, Sq, Skv, D, 1 if with_workspace else 0, num_sms, buf)
        return rc, dict(zip(("ctas", "split", "tail_ctas", "unit_rows"), list(buf)))

    def set_sm_limit(self, sms: int) -> int:
        """Caps the SMs the persistent kernels use (0: all); returns the previous cap."""
        return self.dll.gfx906_b200_attn_set_sm_limit(sms)

    def last_error(self) -> int:
        return self.dll.gfx906_b200_attn_last_error()

    def error_string(self, status: int) -> str:
        return self.dll.gfx906_b200_attn_error_string(status).decode()

    def device_status(self, reset: bool = False) -> int:
        return self.dll.gfx906_b200_attn_device_status(1 if reset else 0)

    def timeout_info(self):
        buf = (_c_int * 6)()
        rc = self.dll.gfx906_b200_attn_timeout_info(buf)
        return rc, list(buf)
