"""Route eligible ComfyUI attention calls to the sm_100a tiled kernel.

Counterpart of the reference's ``deploy/gfx906_attention.py``. ``install()``
sets ``optimized_attention.container_function``, the seam
``comfy/ldm/modules/attention.py`` reserves for containerised q/k/v
(``deploy/gfx906_attention.py:140-163``). A call runs the kernel when it is
eligible (the ``_eligible`` rules below, identical to
``deploy/gfx906_attention.py:38-49``) and the operator loaded; every other call
goes to the stock callable unchanged. There is no CPU path: off sm_100 nothing
is installed, and ineligible shapes keep their original (GPU) attention.

With ``SEEDVR2_GFX906_VAE=1`` the VAE mid-block attention factory is wrapped
too (``deploy/gfx906_attention.py:82-137``): [b, 512, h, w] fp16/bf16 CUDA
inputs become one [b, 1, h*w, 512] attention; a kernel error falls back to the
function the factory selected. ``SEEDVR2_GFX906_LOG_SHAPES=1`` logs each new
eligible shape once. ``GFX906_B200_STRICT=1`` makes an eligible call raise
instead of falling back when the operator cannot be loaded.
"""

from __future__ import annotations

import logging
import os

import torch

from . import gfx906_attn

logger = logging.getLogger("SeedVR2-LongVideo")
_LOG_SHAPES = os.environ.get("SEEDVR2_GFX906_LOG_SHAPES") == "1"
_VAE_HOOK = os.environ.get("SEEDVR2_GFX906_VAE") == "1"
_STRICT = os.environ.get("GFX906_B200_STRICT") == "1"
_seen_shapes: set = set()

_stock_attention = None  # the optimized_attention callable that was wrapped
_stock_normal_attention = None  # diffusionmodules.model.normal_attention at install


def _head_dim_ok(d: int) -> bool:
    return d == 128 or d == 512 or (d <= 64 and d % 8 == 0)


def _eligible(qt, kt, vt, heads, mask, kwargs) -> bool:
    """Whether a [B,H,S,D] call can run on the kernel (same rules as the reference)."""
    if mask is not None or kwargs.get("enable_gqa"):
        return False
    if qt.dtype not in (torch.float16, torch.bfloat16) or not qt.is_cuda:
        return False
    if qt.ndim != 4 or kt.shape != vt.shape:
        return False
    same_bhd = (qt.shape[0] == kt.shape[0] and qt.shape[1] == kt.shape[1]
                and qt.shape[3] == kt.shape[3])
    if not same_bhd or qt.shape[1] != heads:
        return False
    return _head_dim_ok(qt.shape[3])


def _load_or_raise():
    mod = gfx906_attn.load_attention()
    if mod is None and _STRICT:
        raise RuntimeError("sm_100 attention operator unavailable: "
                           f"{gfx906_attn.last_error()}")
    return mod


def _container_attn(q, k, v, heads, mask=None, attn_precision=None,
                    skip_reshape=False, skip_output_reshape=False, **kwargs):
    """``container_function`` body: kernel for eligible calls, else stock."""
    qt, kt, vt = q.peek(), k.peek(), v.peek()
    mod = None
    if skip_reshape and _eligible(qt, kt, vt, heads, mask, kwargs):
        mod = _load_or_raise()
    if mod is None:
        return _stock_attention(
            q.take(), k.take(), v.take(), heads, mask=mask,
            attn_precision=attn_precision, skip_reshape=skip_reshape,
            skip_output_reshape=skip_output_reshape, **kwargs)
    shape = tuple(qt.shape)
    if _LOG_SHAPES and shape not in _seen_shapes:
        _seen_shapes.add(shape)
        logger.info("sm_100 attention: %s %s", shape, qt.dtype)
    qt, kt, vt = q.take(), k.take(), v.take()
    scale = kwargs.get("scale")
    if scale is None:  # what scaled_dot_product_attention uses without a scale
        scale = qt.shape[-1] ** -0.5
    out_dtype = qt.dtype
    if out_dtype != torch.float16:
        qt, kt, vt = qt.half(), kt.half(), vt.half()
    out = mod.attn(qt, kt, vt, scale)
    if out_dtype != torch.float16:
        out = out.to(out_dtype)
    if skip_output_reshape:
        return out
    b = out.shape[0]
    return out.transpose(1, 2).reshape(b, -1, heads * out.shape[-1])


def _vae_attn(q, k, v, fallback):
    """Drop-in for the VAE ``normal_attention`` ([b, c, h, w] -> same shape).

    Eligible calls (CUDA fp16/bf16, equal shapes, c == 512) run as one
    attention over the h*w positions: on the feature maps as they are (the
    kernel's transposed layout) when h*w is a multiple of 8, else as
    [b, 1, h*w, c]; the rest, and any kernel error, use ``fallback``.
    """
    mod = None
    if (q.is_cuda and q.dtype in (torch.float16, torch.bfloat16)
            and q.dim() == 4 and q.shape == k.shape == v.shape
            and q.shape[1] == 512):
        mod = gfx906_attn.load_attention()
    if mod is None:
        return fallback(q, k, v)
    b, c, h, w = q.shape
    out_dtype = q.dtype
    qt, kt, vt = q, k, v
    if out_dtype != torch.float16:
        qt, kt, vt = qt.half(), kt.half(), vt.half()

    def to_seq(t):  # [b, c, h, w] -> [b, 1, h*w, c] (a strided view)
        return t.reshape(b, c, h * w).transpose(1, 2).unsqueeze(1)

    # The feature maps are already the kernel's transposed layout [b, 1, c, h*w]
    # (sequence innermost): no transpose in or out when h*w % 8 == 0.
    dmajor = getattr(mod, "attn_dmajor", None) if (h * w) % 8 == 0 else None
    try:
        if dmajor is not None:
            out = dmajor(qt.reshape(b, 1, c, h * w), kt.reshape(b, 1, c, h * w),
                         vt.reshape(b, 1, c, h * w), c ** -0.5).reshape(b, c, h, w)
        else:
            out = mod.attn(to_seq(qt), to_seq(kt), to_seq(vt), c ** -0.5)
            out = out.squeeze(1).transpose(1, 2).reshape(b, c, h, w)
    except Exception:  # noqa: BLE001 - a kernel error must not abort the decode
        logger.warning("sm_100 VAE attention raised; the call goes to %s instead",
                       getattr(fallback, "__name__", fallback))
        return fallback(q, k, v)
    if out_dtype != torch.float16:
        out = out.to(out_dtype)
    return out


def _install_vae_hook():
    """Replace the ``vae_attention`` factory with one whose returned callable
    runs eligible calls on the kernel whenever the original factory chose the
    sliced ``normal_attention`` or ``pytorch_attention``; any other choice
    (xformers, say) is returned untouched."""
    global _stock_normal_attention
    try:
        from comfy.ldm.modules.diffusionmodules import model as _model
    except Exception as exc:  # noqa: BLE001 - ComfyUI is not on the import path
        logger.warning("no VAE hook installed (ComfyUI model module unavailable: %s)", exc)
        return
    if _stock_normal_attention is not None:
        return
    _stock_normal_attention = _model.normal_attention
    intercepted = {_model.normal_attention, getattr(_model, "pytorch_attention", None)}
    orig_factory = _model.vae_attention

    def factory():
        fn = orig_factory()
        if fn not in intercepted:
            return fn  # a backend this hook does not replace
        return lambda q, k, v: _vae_attn(q, k, v, fn)

    _model.vae_attention = factory
    logger.info("VAE mid-block attention (D=512) now runs on the sm_100 kernel")


def install():
    """Claim ``optimized_attention.container_function`` for this module, once.

    Does nothing unless the current GPU is an sm_100 part and ComfyUI's
    attention module imports; refuses (with a warning) when another extension
    already owns the seam."""
    global _stock_attention
    if not gfx906_attn.is_sm100():
        return
    try:
        from comfy.ldm.modules import attention as _attn
    except Exception as exc:  # noqa: BLE001 - ComfyUI is not on the import path
        logger.warning("no attention hook installed (ComfyUI attention module unavailable: %s)", exc)
        return
    opt = _attn.optimized_attention
    if _stock_attention is opt:
        return
    if not hasattr(opt, "container_function"):
        return
    if opt.container_function is not None:
        logger.warning("another extension owns optimized_attention.container_function; "
                       "leaving it in place")
        return
    _stock_attention = opt
    opt.container_function = _container_attn
    logger.info("DiT attention now runs on the sm_100 kernel when eligible")
    if _VAE_HOOK:
        _install_vae_hook()
