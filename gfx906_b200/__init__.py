"""B200 (sm_100a) flash-attention forward with the gfx906 extension's surface.

Public entry points:

* ``attn(q, k, v, scale)``: the operator itself (fp16 [B,H,S,D] CUDA tensors).
  Raises if the native operator cannot be loaded; there is no fallback.
* ``load_attention()`` / ``is_sm100()``: the lazy loader, as in the
  reference's ``deploy/gfx906_attn.py`` (returns None instead of raising).
* ``gfx906_attention.install()``: the ComfyUI hook with eligibility gating and
  stock fallback, as in the reference's ``deploy/gfx906_attention.py``.
* ``attn_host(q, k, v, scale)``: the same operator for q, k, v in (pinned)
  host memory, uploads and downloads overlapped with the kernel per block of
  (batch x head) units (``host.py``).
* ``set_sm_limit(n)`` / ``sm_limit(n)``: cap the SMs the persistent kernels
  use, leaving the rest to kernels of other streams (NCCL collectives of a
  sharded pipeline, ``shard.attention_by_rows_pipelined``).
"""

import contextlib

from .gfx906_attn import is_sm100, last_error, load_attention

__all__ = ["attn", "attn_dmajor", "attn_host", "device_status", "is_sm100", "load_attention", "last_error",
           "set_sm_limit", "sm_limit"]


def _module_or_raise():
    mod = load_attention()
    if mod is None:
        raise RuntimeError(f"gfx906_b200: sm_100 attention operator unavailable: {last_error()}")
    return mod


def attn(q, k, v, scale):
    """O = softmax(scale * q @ k^T) @ v on the sm_100a kernel (fp16 [B,H,S,D])."""
    return _module_or_raise().attn(q, k, v, scale)


def attn_dmajor(q, k, v, scale):
    """The operator on transposed fp16 tensors: q [B,H,D,Sq], k, v [B,H,D,Skv],
    D = 512, sequence innermost (a [b, c, h, w] feature map is [b, 1, c, h*w]);
    returns o as [B,H,D,Sq]. Sq and Skv must be multiples of 8."""
    return _module_or_raise().attn_dmajor(q, k, v, scale)


def device_status(reset: bool = False) -> int:
    """0 unless a kernel wait timed out since the last reset (synchronises)."""
    return _module_or_raise().device_status(reset)


def attn_host(q, k, v, scale, out=None, device=None, blocks=None, non_blocking=False):
    """The operator on host tensors with the PCIe copies overlapped (see ``host.attn_host``)."""
    from .host import attn_host as _attn_host

    return _attn_host(q, k, v, scale, out=out, device=device, blocks=blocks, non_blocking=non_blocking)


def set_sm_limit(sms: int) -> int:
    """Caps, process-wide, the SMs the persistent kernels plan for (0: all of
    the device's); returns the previous cap. D = 512 uses sms // 2 two-CTA
    clusters (at least one)."""
    return int(_module_or_raise().set_sm_limit(int(sms)))


@contextlib.contextmanager
def sm_limit(sms: int):
    """``set_sm_limit(sms)`` for the duration of a ``with`` block."""
    prev = set_sm_limit(sms)
    try:
        yield
    finally:
        set_sm_limit(prev)
