"""Loader and ComfyUI-hook semantics on the CPU, with fake ComfyUI modules.

Mirrors the reference's test_vae_hook.py (fake ``comfy.*`` modules in
``sys.modules``, a mocked kernel raising to test the fallback) and adds the
eligibility rules of deploy/gfx906_attention.py:38-49, the container-function
flow (:52-79), install() (:140-163) and the loader's marker protocol
(deploy/gfx906_attn.py:40-88). The kernel is replaced by a test double here;
the real kernel is exercised by the gpu-marked tests.
"""

import sys
import types
from unittest import mock

import pytest
import torch
import torch.nn.functional as F

from gfx906_b200 import gfx906_attention as attention
from gfx906_b200 import gfx906_attn


class FakeT:
    """Just the attributes _eligible reads."""

    def __init__(self, shape, dtype=torch.float16, cuda=True):
        self.shape = tuple(shape)
        self.dtype = dtype
        self.is_cuda = cuda
        self.ndim = len(shape)


def elig(q, k=None, v=None, heads=None, mask=None, **kw):
    k = k or FakeT(q.shape)
    v = v or FakeT(k.shape)
    return attention._eligible(q, k, v, heads if heads is not None else q.shape[1], mask, kw)


@pytest.mark.parametrize("d,ok", [(8, True), (16, True), (24, True), (40, True), (56, True),
                                  (64, True), (128, True), (512, True), (4, False), (12, False),
                                  (72, False), (96, False), (256, False), (1024, False)])
def test_eligible_head_dims(d, ok):
    assert elig(FakeT((2, 4, 100, d))) is ok


def test_eligible_rejections():
    q = FakeT((2, 4, 100, 64))
    assert elig(q) is True
    assert elig(q, mask=object()) is False
    assert elig(q, enable_gqa=True) is False
    assert elig(FakeT((2, 4, 100, 64), dtype=torch.float32)) is False
    assert elig(FakeT((2, 4, 100, 64), dtype=torch.bfloat16)) is True
    assert elig(FakeT((2, 4, 100, 64), cuda=False)) is False
    assert elig(FakeT((2, 100, 64))) is False
    assert elig(q, FakeT((2, 4, 50, 64)), FakeT((2, 4, 51, 64))) is False  # k != v
    assert elig(q, FakeT((1, 4, 50, 64))) is False  # batch
    assert elig(q, FakeT((2, 3, 50, 64))) is False  # heads
    assert elig(q, FakeT((2, 4, 50, 32))) is False  # head dim
    assert elig(q, heads=8) is False
    assert elig(q, FakeT((2, 4, 7, 64))) is True  # Sq != Skv is fine


class Box:
    """A ComfyUI-style container: peek() looks, take() hands over."""

    def __init__(self, t):
        self.t = t
        self.taken = False

    def peek(self):
        return self.t

    def take(self):
        self.taken = True
        return self.t


def sdpa_module():
    calls = []

    def attn(q, k, v, scale):
        calls.append((q.dtype, tuple(q.shape), scale))
        return F.scaled_dot_product_attention(q.float(), k.float(), v.float(), scale=scale).half()

    return types.SimpleNamespace(attn=attn), calls


def stock(q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False,
          skip_output_reshape=False, **kwargs):
    return ("stock", heads, skip_reshape, skip_output_reshape, tuple(sorted(kwargs)))


def qkv(dtype=torch.float16, B=2, H=3, S=5, D=16):
    g = torch.Generator().manual_seed(0)
    return [torch.randn(B, H, S, D, generator=g).to(dtype) for _ in range(3)]


@pytest.fixture
def hooked(monkeypatch):
    monkeypatch.setattr(attention, "_stock_attention", stock)
    monkeypatch.setattr(attention, "_eligible", lambda *a: True)
    mod, calls = sdpa_module()
    monkeypatch.setattr(attention.gfx906_attn, "load_attention", lambda: mod)
    return calls


def test_container_eligible_runs_kernel_with_default_scale(hooked):
    q, k, v = qkv()
    boxes = [Box(t) for t in (q, k, v)]
    out = attention._container_attn(*boxes, heads=3, skip_reshape=True, skip_output_reshape=True)
    assert all(b.taken for b in boxes)
    assert hooked == [(torch.float16, (2, 3, 5, 16), 16 ** -0.5)]
    ref = F.scaled_dot_product_attention(q.float(), k.float(), v.float())
    assert torch.allclose(out.float(), ref, atol=2e-3)


def test_container_output_reshape_and_bf16_roundtrip(hooked):
    q, k, v = qkv(torch.bfloat16)
    out = attention._container_attn(Box(q), Box(k), Box(v), heads=3, skip_reshape=True, scale=0.3)
    assert out.dtype == torch.bfloat16 and out.shape == (2, 5, 3 * 16)
    assert hooked[0][0] == torch.float16 and hooked[0][2] == 0.3
    ref = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), scale=0.3)
    assert torch.allclose(out.float(), ref.transpose(1, 2).reshape(2, 5, 48), atol=2e-2)


def test_container_without_skip_reshape_uses_stock(hooked):
    q, k, v = qkv()
    out = attention._container_attn(Box(q), Box(k), Box(v), heads=3, skip_reshape=False, foo=1)
    assert out == ("stock", 3, False, False, ("foo",)) and hooked == []


def test_container_ineligible_or_unloadable_uses_stock(monkeypatch):
    monkeypatch.setattr(attention, "_stock_attention", stock)
    q, k, v = qkv()
    # CPU tensors are not eligible
    assert attention._container_attn(Box(q), Box(k), Box(v), heads=3, skip_reshape=True)[0] == "stock"
    monkeypatch.setattr(attention, "_eligible", lambda *a: True)
    monkeypatch.setattr(attention.gfx906_attn, "load_attention", lambda: None)
    assert attention._container_attn(Box(q), Box(k), Box(v), heads=3, skip_reshape=True)[0] == "stock"
    monkeypatch.setattr(attention, "_STRICT", True)
    with pytest.raises(RuntimeError, match="unavailable"):
        attention._container_attn(Box(q), Box(k), Box(v), heads=3, skip_reshape=True)


# ---- port of the reference's test_vae_hook.py -----------------------------

def fake_comfy(model):
    modules = {name: types.ModuleType(name) for name in (
        "comfy", "comfy.ldm", "comfy.ldm.modules", "comfy.ldm.modules.diffusionmodules")}
    modules["comfy.ldm.modules.diffusionmodules"].model = model
    return modules


def test_vae_factory_preserves_selected_fallback():
    def normal(q, k, v):
        return "normal"

    def pytorch(q, k, v):
        return "pytorch"

    def other(q, k, v):
        return "other"

    for selected in (normal, pytorch, other):
        model = types.SimpleNamespace(normal_attention=normal, pytorch_attention=pytorch,
                                      vae_attention=lambda s=selected: s)
        with mock.patch.dict(sys.modules, fake_comfy(model)), \
                mock.patch.object(attention, "_stock_normal_attention", None):
            attention._install_vae_hook()
            fn = model.vae_attention()
            if selected is other:
                assert fn is other
            assert fn(torch.zeros(1), None, None) == selected(None, None, None)


def test_vae_kernel_error_uses_selected_fallback():
    class Tensor:
        is_cuda = True
        dtype = torch.float16
        shape = (1, 512, 2, 2)

        def dim(self):
            return 4

        def reshape(self, *args):
            return self

        def transpose(self, *args):
            return self

        def unsqueeze(self, *args):
            return self

    t = Tensor()
    kernel = types.SimpleNamespace(attn=mock.Mock(side_effect=RuntimeError))
    with mock.patch.object(attention.gfx906_attn, "load_attention", return_value=kernel):
        assert attention._vae_attn(t, t, t, lambda q, k, v: "fallback") == "fallback"


def test_vae_eligible_layout_and_scale(monkeypatch):
    mod, calls = sdpa_module()
    monkeypatch.setattr(attention.gfx906_attn, "load_attention", lambda: mod)
    g = torch.Generator().manual_seed(1)
    b, c, h, w = 1, 512, 3, 4
    q, k, v = (torch.randn(b, c, h, w, generator=g).to(torch.bfloat16) for _ in range(3))

    class Cuda(torch.Tensor):  # a CPU tensor that claims to be on CUDA for the gate
        @property
        def is_cuda(self):
            return True

    qc, kc, vc = (t.as_subclass(Cuda) for t in (q, k, v))
    out = attention._vae_attn(qc, kc, vc, lambda *a: "fallback")
    assert calls and calls[0][1] == (b, 1, h * w, c) and calls[0][2] == c ** -0.5
    assert out.shape == (b, c, h, w) and out.dtype == torch.bfloat16
    seq = lambda t: t.float().reshape(b, c, h * w).transpose(1, 2).unsqueeze(1)  # noqa: E731
    ref = F.scaled_dot_product_attention(seq(q), seq(k), seq(v), scale=c ** -0.5)
    ref = ref.squeeze(1).transpose(1, 2).reshape(b, c, h, w)
    assert torch.allclose(out.float(), ref, atol=3e-2)
    # not 512 channels: fallback
    small = torch.zeros(1, 64, 2, 2).as_subclass(Cuda)
    assert attention._vae_attn(small, small, small, lambda *a: "fallback") == "fallback"


def test_vae_feature_maps_use_the_transposed_layout(monkeypatch):
    """h*w % 8 == 0: the [b, c, h, w] maps go to attn_dmajor as [b, 1, c, h*w] views
    (no transpose on the way in or out); the result matches SDPA on [b, 1, h*w, c]."""
    calls = []

    def attn_dmajor(q, k, v, scale):
        calls.append((q.dtype, tuple(q.shape), scale, q.is_contiguous()))
        t = lambda x: x.float().transpose(2, 3)  # noqa: E731  [B,H,D,S] -> [B,H,S,D]
        return F.scaled_dot_product_attention(t(q), t(k), t(v), scale=scale).transpose(2, 3).half()

    mod = types.SimpleNamespace(attn=mock.Mock(side_effect=AssertionError("row-major path used")),
                                attn_dmajor=attn_dmajor)
    monkeypatch.setattr(attention.gfx906_attn, "load_attention", lambda: mod)
    g = torch.Generator().manual_seed(2)
    b, c, h, w = 2, 512, 4, 6

    class Cuda(torch.Tensor):
        @property
        def is_cuda(self):
            return True

    q, k, v = (torch.randn(b, c, h, w, generator=g).half().as_subclass(Cuda) for _ in range(3))
    out = attention._vae_attn(q, k, v, lambda *a: "fallback")
    assert calls == [(torch.float16, (b, 1, c, h * w), c ** -0.5, True)]
    seq = lambda t: t.float().reshape(b, c, h * w).transpose(1, 2).unsqueeze(1)  # noqa: E731
    ref = F.scaled_dot_product_attention(seq(q), seq(k), seq(v), scale=c ** -0.5)
    ref = ref.squeeze(1).transpose(1, 2).reshape(b, c, h, w)
    assert out.shape == (b, c, h, w) and torch.allclose(out.float(), ref, atol=2e-3)


# ---- install() --------------------------------------------------------------

def fake_attention_module(container=None):
    opt = types.SimpleNamespace(container_function=container)
    mods = {name: types.ModuleType(name) for name in ("comfy", "comfy.ldm", "comfy.ldm.modules",
                                                      "comfy.ldm.modules.attention")}
    mods["comfy.ldm.modules.attention"].optimized_attention = opt
    mods["comfy.ldm.modules"].attention = mods["comfy.ldm.modules.attention"]
    return mods, opt


def test_install_is_noop_off_sm100(monkeypatch):
    mods, opt = fake_attention_module()
    monkeypatch.setattr(attention.gfx906_attn, "is_sm100", lambda: False)
    with mock.patch.dict(sys.modules, mods):
        attention.install()
    assert opt.container_function is None


def test_install_sets_seam_once_and_respects_existing(monkeypatch):
    monkeypatch.setattr(attention.gfx906_attn, "is_sm100", lambda: True)
    monkeypatch.setattr(attention, "_stock_attention", None)
    mods, opt = fake_attention_module()
    with mock.patch.dict(sys.modules, mods):
        attention.install()
        assert opt.container_function is attention._container_attn
        assert attention._stock_attention is opt
        attention.install()  # idempotent
        assert opt.container_function is attention._container_attn
    monkeypatch.setattr(attention, "_stock_attention", None)
    other = object()
    mods2, opt2 = fake_attention_module(container=other)
    with mock.patch.dict(sys.modules, mods2):
        attention.install()
    assert opt2.container_function is other


# ---- loader -------------------------------------------------------------------

@pytest.fixture
def fresh_loader(monkeypatch, tmp_path):
    gfx906_attn._reset_for_tests()
    monkeypatch.setattr(gfx906_attn, "_BUILD_FAILED", tmp_path / ".build_failed")
    monkeypatch.setattr(gfx906_attn, "_PREBUILT", tmp_path / ".prebuilt")
    yield tmp_path
    gfx906_attn._reset_for_tests()


def test_loader_off_sm100_returns_none_once(fresh_loader, monkeypatch):
    probe = mock.Mock(return_value=False)
    monkeypatch.setattr(gfx906_attn, "is_sm100", probe)
    assert gfx906_attn.load_attention() is None
    assert "sm_100" in gfx906_attn.last_error()
    assert gfx906_attn.load_attention() is None
    assert probe.call_count == 1  # one attempt per process


def test_loader_build_failure_marker_stops_retries(fresh_loader, monkeypatch):
    monkeypatch.setattr(gfx906_attn, "is_sm100", lambda: True)
    build = mock.Mock(side_effect=RuntimeError("nvcc exploded"))
    monkeypatch.setattr(gfx906_attn._build, "build_library", build)
    assert gfx906_attn.load_attention() is None
    marker = fresh_loader / ".build_failed"
    assert marker.is_file() and "nvcc exploded" in marker.read_text()
    gfx906_attn._reset_for_tests()
    assert gfx906_attn._build_kernel_obj() is False
    assert build.call_count == 1  # the marker prevents a rebuild


def test_loader_success_path_imports_extension(fresh_loader, monkeypatch):
    monkeypatch.setattr(gfx906_attn, "is_sm100", lambda: True)
    monkeypatch.setattr(gfx906_attn._build, "build_library", lambda: None)
    monkeypatch.setattr(gfx906_attn._build, "build_extension", lambda: None)
    mod = gfx906_attn.load_attention()
    assert mod is not None and hasattr(mod, "attn") and hasattr(mod, "device_status")
    assert gfx906_attn.load_attention() is mod


def test_strict_entry_raises_without_operator(fresh_loader, monkeypatch):
    import gfx906_b200

    monkeypatch.setattr(gfx906_attn, "is_sm100", lambda: False)
    with pytest.raises(RuntimeError, match="unavailable"):
        gfx906_b200.attn(None, None, None, 1.0)
