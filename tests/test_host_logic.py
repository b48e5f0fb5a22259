"""Host-side surface of the plug-in: env semantics, install idempotence,
plug-in entry point (fused_moe.py:76-118, 1245-1315; plugin.py:47-124)."""
import pytest

from wisp_b200.integrations.vllm import fused_moe as fm
from wisp_b200.integrations.vllm import plugin


@pytest.mark.parametrize("raw,mode", [(None, "paged"), ("paged", "paged"), ("RESIDENT", "resident"),
                                      (" copy ", "copy"), ("day1", "copy"), ("day2a", "resident"),
                                      ("day2b", "paged"), ("bogus", "paged")])
def test_resolve_mode(monkeypatch, raw, mode):
    if raw is None:
        monkeypatch.delenv("WISP_MODE", raising=False)
    else:
        monkeypatch.setenv("WISP_MODE", raw)
    assert fm._resolve_mode() == mode


@pytest.mark.parametrize("raw,E,cap", [(None, 128, 24), (None, 8, 8), ("16", 128, 16), ("1", 128, 2),
                                       ("999", 128, 128), ("x", 128, 128), ("-5", 8, 2)])
def test_resolve_cap(monkeypatch, raw, E, cap):
    if raw is None:
        monkeypatch.delenv("WISP_CAP_EXPERTS", raising=False)
    else:
        monkeypatch.setenv("WISP_CAP_EXPERTS", raw)
    assert fm._resolve_cap_experts(E) == cap


def _fake_cls():
    class FakeMethod:
        def create_weights(self, *a, **k):
            return "orig_cw"

        def process_weights_after_loading(self, layer):
            return "orig_pw"

        def forward_cuda(self, layer, x, *a):
            return "orig_fwd"
    return FakeMethod


def test_install_is_idempotent_and_keeps_originals(monkeypatch):
    cls = _fake_cls()
    orig = cls.forward_cuda
    monkeypatch.setenv("WISP_MODE", "paged")
    assert fm.install_wisp_moe(_cls=cls) is True
    assert fm.is_installed(_cls=cls)
    assert cls._wisp_original_forward_cuda is orig
    assert cls.forward_cuda is fm._patched_forward_cuda
    assert cls.create_weights is fm._patched_create_weights
    assert fm._WISP_RUNTIME_CONFIG["mode"] == "paged"
    # second call: no re-patch, runtime config refreshed only
    assert fm.install_wisp_moe(mode="resident", cap_experts=12, _cls=cls) is False
    assert cls._wisp_original_forward_cuda is orig
    assert fm._WISP_RUNTIME_CONFIG == {"mode": "resident", "cap_experts_override": 12}


def test_unpatched_layer_passes_through():
    cls = _fake_cls()
    fm.install_wisp_moe(_cls=cls)

    class Layer:
        pass
    assert cls().forward_cuda(Layer(), None, None, None) == "orig_fwd"


def test_plugin_disable(monkeypatch):
    called = []
    monkeypatch.setenv("WISP_PLUGIN_DISABLE", "1")
    monkeypatch.setattr(fm, "install_wisp_moe", lambda **k: called.append(1))
    plugin.register()
    assert not called


@pytest.mark.slow
def test_install_on_the_installed_vllm_class():
    """Patches the real vLLM UnquantizedFusedMoEMethod (imports vLLM, ~25 s)."""
    pytest.importorskip("vllm")
    from vllm.model_executor.layers.fused_moe.unquantized_fused_moe_method import (
        UnquantizedFusedMoEMethod as U,
    )
    import inspect
    applied = fm.install_wisp_moe()
    assert fm.is_installed()
    assert U.forward_cuda is fm._patched_forward_cuda
    assert fm.install_wisp_moe() is False
    # the patched forward keeps the installed vLLM's argument list
    want = list(inspect.signature(U._wisp_original_forward_cuda).parameters)
    got = list(inspect.signature(fm._patched_forward_cuda).parameters)
    assert want == got, (want, got)
    assert applied in (True, False)
