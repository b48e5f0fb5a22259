"""The other model shapes of the benchmark configurations, at their exact
layer sizes: Mixtral-8x7B (config 4: hidden 4096, intermediate 14336, 8
experts, top-2; decode runs the generic kernels since the intermediate size is
beyond the decode fast path, prefill-sized calls the tensor-core GEMMs) and
Qwen3-235B-A22B (config 5: hidden 4096, intermediate 1536, top-8), paged at
small caps.  Tolerance as in the other parity tests: mean-rel <= 1e-3 and per
element <= max(1e-2, 2 ulp(out) + sum over k of 2 ulp(y_k)) against the fp32
oracle with the reference's bf16 storage points."""
import pytest
import torch

from oracle.moe import compare, moe_reference
from oracle.pager import PagerOracle, forward_pager
from tests.test_moe_gpu import MEAN_REL, MAX_ABS, fwd, state

pytestmark = pytest.mark.gpu


def _ulp(v):  # bf16: 8 significand bits
    return torch.ldexp(torch.ones_like(v), torch.frexp(v.abs().clamp_min(1e-30))[1] - 8)


def _check(out, x, w13, w2, w, ids):
    ref, Y = moe_reference(x, w13, w2, w, ids, return_partials=True)
    c = compare(out, ref)
    assert c["mean_rel"] <= MEAN_REL, c
    bound = torch.clamp_min(2 * _ulp(ref) + (2 * _ulp(Y)).sum(dim=1), MAX_ABS)
    assert bool(((out.float() - ref).abs() <= bound).all()), c


def _weights(E, H, I, seed):
    g = torch.Generator().manual_seed(seed)
    w13 = torch.empty(E, 2 * I, H, dtype=torch.bfloat16)
    w2 = torch.empty(E, H, I, dtype=torch.bfloat16)
    for e in range(E):  # per expert, to keep the fp32 temporaries small
        w13[e] = (torch.randn(2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
        w2[e] = (torch.randn(H, I, generator=g) * 0.02).to(torch.bfloat16)
    return w13, w2, g


@pytest.fixture(scope="module")
def mixtral():
    return _weights(8, 4096, 14336, 8)


@pytest.mark.parametrize("cap", [2, 4])
def test_mixtral_decode_paged(mixtral, cap):
    w13, w2, g = mixtral
    st = state(w13, w2, cap)
    oracle = PagerOracle(8, cap)
    for T in (1, 8, 3):
        x = torch.randn(T, 4096, generator=g).to(torch.bfloat16)
        logits = torch.randn(T, 8, generator=g)
        w, ids = torch.softmax(logits, -1).topk(2, -1)
        w = (w / w.sum(-1, keepdim=True)).float()
        ids = ids.to(torch.int32)
        out = fwd(st, x, w, ids)
        _check(out, x, w13, w2, w, ids)
        forward_pager(oracle, ids.numpy())
        s2e, tick, clock, stats = st._read()
        assert s2e == oracle.slot_to_expert and tick == oracle.lru_tick and stats == oracle.stats()
    st.close()


def test_mixtral_prefill_tensor_core_path(mixtral):
    w13, w2, g = mixtral
    st = state(w13, w2, 8, "resident")
    T = 264  # 528 (token, k) pairs: beyond the weight-stationary range
    x = torch.randn(T, 4096, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, 8, generator=g)
    w, ids = torch.softmax(logits, -1).topk(2, -1)
    w = (w / w.sum(-1, keepdim=True)).float()
    launches0 = st.telemetry()["kernel_launches"]
    out = fwd(st, x, w, ids.to(torch.int32))
    # resident: routing-and-gather, gate-up, down, combine
    assert st.telemetry()["kernel_launches"] - launches0 == 4
    _check(out, x, w13, w2, w, ids)
    st.close()


def test_qwen3_235b_decode_paged():
    E, H, I, K = 16, 4096, 1536, 8  # the 235B layer's hidden / intermediate sizes, 16 of its experts
    w13, w2, g = _weights(E, H, I, 235)
    st = state(w13, w2, 8)
    for T in (1, 4):
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        logits = torch.randn(T, E, generator=g)
        w, ids = torch.softmax(logits, -1).topk(K, -1)
        w = (w / w.sum(-1, keepdim=True)).float()
        out = fwd(st, x, w, ids.to(torch.int32))
        _check(out, x, w13, w2, w, ids)
    st.close()
