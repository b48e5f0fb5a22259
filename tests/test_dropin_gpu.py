"""The drop-in boundary exercised the way vLLM drives it.

vLLM's ``FusedMoE`` layer calls its quant method's ``create_weights`` at model
construction, its weight loader fills the returned parameters, then
``process_weights_after_loading`` runs once, and every forward goes through
``forward_cuda(layer, x, topk_weights, topk_ids, shared_experts,
shared_experts_input)``.  Here a stand-in method class (the attributes the
patch reads: ``moe.has_bias`` / ``moe.is_act_and_mul``, and the three
methods ``install_wisp_moe`` replaces) is patched by ``install_wisp_moe`` and
driven through that sequence at Qwen3-30B-A3B layer shapes, in each
``WISP_MODE``, against the CPU oracle (reference fused_moe.py:673-759,
762-927, 930-987; the controller helpers :537-593).
"""
import pytest
import torch

from oracle.moe import compare, moe_reference
from oracle.pager import PagerOracle, forward_pager
from wisp_b200 import workloads as wl

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
SHAPE = wl.QWEN3_30B
E = 64


class _MoEConfig:
    has_bias = False
    is_act_and_mul = True


def _method_class():
    """A fresh stand-in for vLLM's UnquantizedFusedMoEMethod (patched per test)."""

    class FakeUnquantizedFusedMoEMethod:
        original_calls = []

        def __init__(self):
            self.moe = _MoEConfig()

        def create_weights(self, layer, num_experts, hidden_size, intermediate_size_per_partition,
                           params_dtype, **extra_weight_attrs):
            raise AssertionError("the patch replaces create_weights")

        def process_weights_after_loading(self, layer):
            type(self).original_calls.append("process_weights_after_loading")

        def forward_cuda(self, layer, x, topk_weights, topk_ids, shared_experts=None,
                         shared_experts_input=None):
            type(self).original_calls.append("forward_cuda")
            return "original"

    return FakeUnquantizedFusedMoEMethod


@pytest.fixture(scope="module")
def weights():
    g = torch.Generator().manual_seed(7)
    w13 = (torch.randn(E, 2 * SHAPE.inter, SHAPE.hidden, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, SHAPE.hidden, SHAPE.inter, generator=g) * 0.02).to(torch.bfloat16)
    return w13, w2


@pytest.fixture()
def registry():
    """Isolate the module-level layer registry the controller helpers read."""
    from wisp_b200.integrations.vllm import fused_moe as fm
    saved = (list(fm._LAYER_STATES), dict(fm._LAYER_BY_ID), dict(fm._WISP_RUNTIME_CONFIG))
    fm._LAYER_STATES.clear()
    fm._LAYER_BY_ID.clear()
    yield fm
    for st in fm._LAYER_STATES:
        st.close()
    fm._LAYER_STATES[:] = saved[0]
    fm._LAYER_BY_ID.clear()
    fm._LAYER_BY_ID.update(saved[1])
    fm._WISP_RUNTIME_CONFIG.clear()
    fm._WISP_RUNTIME_CONFIG.update(saved[2])


def _load_layer(fm, cls, w13, w2):
    """create_weights -> weight loader fills the CPU params -> process_weights_after_loading."""
    method = cls()
    layer = torch.nn.Module()
    loaded = []
    cls.create_weights(method, layer, E, SHAPE.hidden, SHAPE.inter, torch.bfloat16,
                       weight_loader=lambda *a: loaded.append(a))
    assert layer.w13_weight.device.type == "cpu" and layer.w2_weight.device.type == "cpu"
    assert tuple(layer.w13_weight.shape) == (E, 2 * SHAPE.inter, SHAPE.hidden)
    assert tuple(layer.w2_weight.shape) == (E, SHAPE.hidden, SHAPE.inter)
    assert layer.w13_weight.weight_loader is not None      # set_weight_attrs carried the loader
    layer.w13_weight.data.copy_(w13)
    layer.w2_weight.data.copy_(w2)
    method.process_weights_after_loading(layer)
    assert "process_weights_after_loading" in cls.original_calls
    return method, layer


def _routing(T, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, SHAPE.hidden, generator=g).to(torch.bfloat16)
    w, ids = wl.softmax_topk(torch.randn(T, E, generator=g), SHAPE.top_k)
    return x, w, ids


def _check(out, x, w13, w2, w, ids):
    c = compare(out.cpu(), moe_reference(x, w13, w2, w, ids))
    assert c["max_abs"] <= 1e-2 and c["mean_rel"] <= 1e-3, c


def test_paged_mode_through_the_patch(weights, registry):
    fm = registry
    w13, w2 = weights
    cls = _method_class()
    assert fm.install_wisp_moe(mode="paged", cap_experts=16, _cls=cls) is True
    assert fm.is_installed(_cls=cls)
    method, layer = _load_layer(fm, cls, w13, w2)
    st = layer._wisp_state
    assert st is not None and st.mode == "paged" and st.cap_experts == 16
    # the Parameters are 0-element placeholders on the GPU; the masters are pinned
    assert layer.w13_weight.numel() == 0 and layer.w13_weight.device.type == "cuda"
    assert layer.w2_weight.numel() == 0 and layer.w2_weight.device.type == "cuda"
    assert layer._wisp_cpu_pin_w13.is_pinned() and layer._wisp_cpu_pin_w2.is_pinned()
    # a second process_weights_after_loading is a no-op (same state object)
    method.process_weights_after_loading(layer)
    assert layer._wisp_state is st and fm.num_registered_layers() == 1
    oracle = PagerOracle(E, 16)
    steps = [(1, 3), (4, 4), (16, 5), (2, 6)]                 # 16 tokens route to > 16 experts: sub-batched
    for T, seed in steps:
        x, w, ids = _routing(T, seed)
        out = cls.forward_cuda(method, layer, x.to(DEV), w.to(DEV), ids.to(DEV), None, None)
        torch.cuda.synchronize()
        _check(out, x, w13, w2, w, ids)
        forward_pager(oracle, ids.numpy())
    assert "forward_cuda" not in cls.original_calls
    s2e, tick, clock, stats = st._read()
    assert (s2e, tick, clock, stats) == (oracle.slot_to_expert, oracle.lru_tick, oracle.lru_clock,
                                         oracle.stats())
    assert st.stats_forward == len(steps)                     # counted once per forward (:1017)
    # controller surface (:537-593)
    assert fm.current_layer_cap() == 16 and fm.num_experts_per_layer() == E
    assert fm.expert_bytes_per_cap() == 3 * SHAPE.hidden * SHAPE.inter * 2
    snap = fm.snapshot_expert_stats(reset=True)
    assert (snap["forward"], snap["miss"], snap["hit"]) == (len(steps), oracle.stats_miss, oracle.stats_hits)
    assert snap["ws"] == len(set(ids.reshape(-1).tolist()))   # unique experts of the last forward
    snap2 = fm.snapshot_expert_stats(reset=False)
    assert (snap2["forward"], snap2["miss"], snap2["hit"]) == (0, 0, 0)
    # hot resize of every registered layer at a drained barrier
    assert fm.resize_layer_caps(24) == 1 and fm.current_layer_cap() == 24
    oracle.resize_cap(24)
    x, w, ids = _routing(8, 9)
    out = cls.forward_cuda(method, layer, x.to(DEV), w.to(DEV), ids.to(DEV), None, None)
    torch.cuda.synchronize()
    _check(out, x, w13, w2, w, ids)
    forward_pager(oracle, ids.numpy())
    assert st._read()[:3] == (oracle.slot_to_expert, oracle.lru_tick, oracle.lru_clock)


def test_resident_mode_through_the_patch(weights, registry):
    fm = registry
    w13, w2 = weights
    cls = _method_class()
    fm.install_wisp_moe(mode="resident", _cls=cls)
    method, layer = _load_layer(fm, cls, w13, w2)
    st = layer._wisp_state
    assert st.mode == "resident" and st.cap_experts == E
    assert st.slot_to_expert == list(range(E))                # primed identity map (:242-258)
    for i, (T, seed) in enumerate([(1, 11), (16, 12), (3, 13)]):
        x, w, ids = _routing(T, seed)
        out = cls.forward_cuda(method, layer, x.to(DEV), w.to(DEV), ids.to(DEV), None, None)
        st.synchronize()
        _check(out, x, w13, w2, w, ids)
        assert st.stats_forward == i + 1                      # resident forwards count (:974-976)
    assert st.stats_miss == 0 and st.stats_evict == 0


def test_copy_mode_through_the_patch(weights, registry):
    fm = registry
    w13, w2 = weights
    cls = _method_class()
    fm.install_wisp_moe(mode="copy", _cls=cls)
    method, layer = _load_layer(fm, cls, w13, w2)
    assert layer._wisp_state is None and layer._wisp_cpu_w13 is not None
    assert fm.num_registered_layers() == 0                    # copy mode registers no paging layer
    for T, seed in [(2, 21), (16, 22)]:
        x, w, ids = _routing(T, seed)
        out = cls.forward_cuda(method, layer, x.to(DEV), w.to(DEV), ids.to(DEV), None, None)
        torch.cuda.synchronize()
        _check(out, x, w13, w2, w, ids)


def test_untouched_layer_passes_through(registry):
    fm = registry
    cls = _method_class()
    fm.install_wisp_moe(mode="paged", _cls=cls)
    method = cls()
    layer = torch.nn.Module()                                 # no WiSP state: the original forward
    assert cls.forward_cuda(method, layer, None, None, None, None, None) == "original"
    assert cls.original_calls == ["forward_cuda"]
