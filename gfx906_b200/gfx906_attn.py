"""Lazy loader for the sm_100a tiled attention operator.

Counterpart of the reference's ``deploy/gfx906_attn.py``: one load attempt per
process, an architecture gate, a rebuild of the native objects when they are
stale, a ``.build_failed`` marker so that a failed build is not retried on
every import, and a ``.prebuilt`` marker holding the compiler log of the last
successful build (``deploy/gfx906_attn.py:21-22, 40-59, 62-88``).

The differences are the target (``is_sm100`` instead of ``is_gfx906``; nvcc
for ``sm_100a`` instead of hipcc for gfx906) and the artefacts: an in-tree
C-ABI library plus a torch operator module linked to it (``build.py``),
instead of a HIP object handed to ``torch.utils.cpp_extension.load``.
"""

from __future__ import annotations

import importlib
import logging

import torch

from . import build as _build

logger = logging.getLogger("SeedVR2-LongVideo")

_BUILD_FAILED = _build.PKG_DIR / ".build_failed"
_PREBUILT = _build.PKG_DIR / ".prebuilt"

_module = None
_attempted = False
_last_error = None  # why the last load returned None (for error messages)


def is_sm100() -> bool:
    """True when the current CUDA device is an sm_100 GPU (B200)."""
    if not torch.cuda.is_available():
        return False
    try:
        return torch.cuda.get_device_capability(torch.cuda.current_device()) == (10, 0)
    except Exception:  # noqa: BLE001 - no usable device
        return False


def _build_kernel_obj() -> bool:
    """Make sure the library and the operator module are built and current.

    Mirrors ``deploy/gfx906_attn.py:40-59``: stale artefacts are rebuilt, a
    failed build leaves ``.build_failed`` (with the compiler output) and later
    calls return False without retrying; delete the marker to retry.
    """
    if _BUILD_FAILED.is_file():
        return False
    try:
        _build.build_library()
        _build.build_extension()
    except Exception as exc:  # noqa: BLE001 - record and fall back
        _BUILD_FAILED.write_text(str(exc)[-4000:])
        logger.warning("sm_100 attention kernel build failed: %s", str(exc)[-500:])
        return False
    log = _build.PKG_DIR / ".nvcc.log"
    if log.is_file():
        _PREBUILT.write_text(log.read_text()[-8000:])
    return True


def import_extension():
    """Import the built operator module (raises ImportError if it is absent)."""
    return importlib.import_module(f"{__package__}.{_build.EXT_NAME}")


def load_attention():
    """Return the operator module (has ``attn(q, k, v, scale)``) or None.

    q/k/v are [B, H, S, D] fp16 CUDA tensors; Sq may differ from Skv, and D
    must be <= 64 and a multiple of 8, or exactly 128, or exactly 512.
    Returns None off sm_100, on build failure, or after a failed first
    attempt. Never raises.
    """
    global _module, _attempted, _last_error
    if _attempted:
        return _module
    _attempted = True
    try:
        if not is_sm100():
            _last_error = "current device is not an sm_100 (B200) GPU"
            return None
        if not _build_kernel_obj():
            _last_error = "build failed: " + (
                _BUILD_FAILED.read_text()[-500:] if _BUILD_FAILED.is_file() else "?")
            return None
        _module = import_extension()
        logger.info("sm_100 attention kernel loaded")
    except Exception as exc:  # noqa: BLE001 - fall back to stock attention
        logger.warning("sm_100 attention kernel unavailable: %s", exc)
        _last_error = str(exc)
        _module = None
    return _module


def last_error():
    """Why the last ``load_attention()`` returned None (or None if it did not)."""
    return _last_error


def _reset_for_tests() -> None:
    global _module, _attempted, _last_error
    _module, _attempted, _last_error = None, False, None
