"""Block-quantised FP8 paging (the reference's fused_moe_fp8.py).

* CPU: the FP8 oracle (oracle/moe_fp8.py) against golden outputs of vLLM's
  own block-FP8 fused_experts (tests/golden/make_vllm_fp8_golden.py); the
  FP8 cap rule; the install surface on a stand-in method class.
* GPU: the FP8 layer (resident and paged) against vLLM's outputs and the
  oracle, its pager state against the LRU oracle (the FP8 path pages with the
  same policy), byte identity across caps, and the drop-in sequence
  create_weights -> process_weights_after_loading -> apply on a stand-in
  Fp8MoEMethod.

The oracle reproduces vLLM's FP8 outputs bit for bit on every golden case
(its quantiser's scale is amax / 448 as a division; the product with 1/448
differs in the last bit for some groups and moves their codes).  The layer
differs from vLLM only in the fp32 accumulation order; tolerance, as for
every parity test: max-abs <= 1e-2 and mean-rel <= 1e-3."""
import os

import numpy as np
import pytest
import torch

from oracle.moe import compare
from oracle.moe_fp8 import moe_reference_fp8
from oracle.pager import PagerOracle, forward_pager
from tests.golden.make_vllm_fp8_golden import CASES, case_tensors, checksum

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "vllm_fp8_fused_experts.npz")
MAX_ABS, MEAN_REL = 1e-2, 1e-3
DEV = torch.device("cuda:0")


def _case(case):
    name, E, H, I, T, K, cap, seed = case
    d = np.load(GOLD)
    tensors = case_tensors(E, H, I, T, K, cap, seed)
    np.testing.assert_array_equal(checksum(*tensors), d[name + "/checksum"],
                                  err_msg="seeded inputs differ from the ones vLLM saw")
    return tensors, torch.from_numpy(d[name + "/out"]).view(torch.bfloat16)


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_fp8_oracle_matches_vllm(case):
    (w13, w2, s13, s2, x, w, ids, _), vout = _case(case)
    out = moe_reference_fp8(x, w13, w2, s13, s2, w, ids)
    assert torch.equal(out.to(torch.bfloat16), vout), compare(vout, out)


def test_fp8_cap_rule(monkeypatch):
    from wisp_b200.integrations.vllm.fused_moe_fp8 import _resolve_cap_experts
    monkeypatch.delenv("WISP_CAP_EXPERTS", raising=False)
    assert _resolve_cap_experts(256) == 24 and _resolve_cap_experts(16) == 16
    for raw, want in (("4", 8), ("100", 100), ("999", 256), ("x", 24)):
        monkeypatch.setenv("WISP_CAP_EXPERTS", raw)
        assert _resolve_cap_experts(256) == want, raw


class _MoEConfig:
    has_bias = False
    is_act_and_mul = True


def _fp8_method_class():
    class FakeFp8MoEMethod:
        calls = []

        def __init__(self, block=True):
            self.moe = _MoEConfig()
            self.block_quant = block
            self.weight_block_size = [128, 128] if block else None

        def create_weights(self, layer, *a, **k):
            type(self).calls.append("create_weights")

        def process_weights_after_loading(self, layer):
            type(self).calls.append("process_weights_after_loading")

        def apply(self, layer, x, topk_weights, topk_ids, shared_experts=None, shared_experts_input=None):
            type(self).calls.append("apply")
            return "original"

    return FakeFp8MoEMethod


def test_fp8_install_is_idempotent_and_leaves_other_fp8_layers_alone():
    from wisp_b200.integrations.vllm.fused_moe_fp8 import install_wisp_fp8, is_fp8_installed
    cls = _fp8_method_class()
    assert not is_fp8_installed(_cls=cls)
    assert install_wisp_fp8(_cls=cls) is True and install_wisp_fp8(_cls=cls) is False
    assert is_fp8_installed(_cls=cls)
    m = cls(block=False)                           # per-tensor FP8: vLLM's own path
    layer = torch.nn.Module()
    cls.create_weights(m, layer, 4, 128, 128, torch.bfloat16)
    cls.process_weights_after_loading(m, layer)
    assert cls.apply(m, layer, None, None, None) == "original"
    assert cls.calls == ["create_weights", "process_weights_after_loading", "apply"]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_fp8_layer_matches_vllm(case):
    from wisp_b200.integrations.vllm.fused_moe_fp8 import WispMoEStateFP8
    name, E, H, I, T, K, cap, seed = case
    (w13, w2, s13, s2, x, w, ids, _), vout = _case(case)
    ref = moe_reference_fp8(x, w13, w2, s13, s2, w, ids)
    outs = []
    for mode, c_exp in (("resident", E), ("paged", cap), ("paged", max(K, 8))):
        st = WispMoEStateFP8(w13.clone(), w2.clone(), s13, s2, c_exp, DEV, 0, mode=mode)
        if mode == "resident":
            st.prime_identity()
        out = st.forward(x.to(DEV), w.to(DEV), ids.to(DEV))
        st.synchronize()
        for what, want in (("vllm", vout.float()), ("oracle", ref)):
            c = compare(out.cpu(), want)
            assert c["max_abs"] <= MAX_ABS and c["mean_rel"] <= MEAN_REL, (mode, c_exp, what, c)
        if mode == "paged":
            o = PagerOracle(E, c_exp)
            forward_pager(o, ids.numpy())
            assert st._read() == (o.slot_to_expert, o.lru_tick, o.lru_clock, o.stats()), (mode, c_exp)
        outs.append(out.cpu())
        st.close()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])            # byte-identical across caps and modes


@pytest.mark.gpu
def test_fp8_dropin_through_the_patch():
    from wisp_b200.integrations.vllm import fused_moe_fp8 as f8
    name, E, H, I, T, K, cap, seed = CASES[1]
    (w13, w2, s13, s2, x, w, ids, _), vout = _case(CASES[1])
    cls = _fp8_method_class()
    f8.install_wisp_fp8(_cls=cls)
    m = cls()
    layer = torch.nn.Module()
    saved = list(f8._FP8_LAYER_STATES)
    try:
        cls.create_weights(m, layer, E, H, I, torch.bfloat16, weight_loader=lambda *a: None)
        assert layer.w13_weight.dtype == torch.float8_e4m3fn and layer.w13_weight.device.type == "cpu"
        assert tuple(layer.w13_weight_scale_inv.shape) == (E, 2 * I // 128, H // 128)
        layer.w13_weight.data.copy_(w13)
        layer.w2_weight.data.copy_(w2)
        layer.w13_weight_scale_inv.data.copy_(s13)
        layer.w2_weight_scale_inv.data.copy_(s2)
        os.environ["WISP_CAP_EXPERTS"] = str(cap)
        try:
            cls.process_weights_after_loading(m, layer)
        finally:
            del os.environ["WISP_CAP_EXPERTS"]
        st = layer._wisp_fp8_state
        assert st.cap_experts == cap and layer.w13_weight.numel() == 0
        out = cls.apply(m, layer, x.to(DEV), w.to(DEV), ids.to(DEV), None, None)
        st.synchronize()
        c = compare(out.cpu(), vout.float())
        assert c["max_abs"] <= MAX_ABS and c["mean_rel"] <= MEAN_REL, c
        assert st.stats_forward == 1
        st.close()
    finally:
        f8._FP8_LAYER_STATES[:] = saved
