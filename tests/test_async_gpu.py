"""The single-launch forward with asynchronous page-in (default path):
byte-identical to the host-synchronous path, pager bit-exact with the
reference's traces, and device-side failures reported to the host without
a GPU fault (a bounded wait on a flag that is never raised)."""
import numpy as np
import pytest
import torch

from oracle.moe import compare, moe_reference
from oracle.pager import PagerOracle, forward_pager
from tests.conftest import GOLDEN, split_forwards
from wisp_b200 import _lib
from wisp_b200 import workloads as wl

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _state(w13, w2, cap, asynchronous=True):
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState
    st = WispMoEState(w13, w2, cap, "paged", DEV, 0)
    st.configure(asynchronous=asynchronous)
    return st


def _weights(E, H, I, seed):
    g = torch.Generator().manual_seed(seed)
    return ((torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16),
            (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16), g)


def test_async_and_sync_paths_are_byte_identical():
    E, H, I, K = 64, 512, 256, 8
    w13, w2, g = _weights(E, H, I, 5)
    a, b = _state(w13, w2, 12, True), _state(w13, w2, 12, False)
    for T in (1, 4, 16, 1, 9, 2, 16, 1):
        x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
        w, ids = wl.softmax_topk(torch.randn(T, E, generator=g), K)
        oa = a.forward(x, w.to(DEV), ids.to(DEV))
        ob = b.forward(x, w.to(DEV), ids.to(DEV))
        a.synchronize()
        b.synchronize()
        assert torch.equal(oa, ob), T
    assert a._read() == b._read()
    ref = moe_reference(x.cpu(), w13, w2, w, ids)
    c = compare(oa.cpu(), ref)
    assert c["max_abs"] <= 1e-2 and c["mean_rel"] <= 1e-3, c
    a.close()
    b.close()


REPLAY = ["cfg1_b1_cap8", "cfg2_b4_cap16_l0", "cfg2_b16_cap8_l1", "cfg3_chunk0_cap32",
          "cfg4_b8_cap2", "cfg5_local64_cap16_b64", "ragged_e16_cap5"]


@pytest.mark.parametrize("name", REPLAY)
def test_async_forward_replays_reference_trace(golden, name):
    """The pager inside the single-launch forward (block 0) against the
    reference's recorded state after every forward."""
    case = golden[name]
    E, cap = int(case["E"]), int(case["cap"])
    H, I = 64, 32
    w13, w2, g = _weights(E, H, I, 1)
    st = _state(w13, w2, cap, True)
    fws, _ = split_forwards(case)
    for i, ids in enumerate(fws):
        T, K = ids.shape
        x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
        w = torch.full((T, K), 1.0 / K).to(DEV)
        st.forward(x, w, torch.from_numpy(np.ascontiguousarray(ids)).to(DEV))
        if i % 7 == 0 or i == len(fws) - 1:
            st.synchronize()
            s2e, tick, clock, stats = st._read()
            assert s2e == case["s2e"][i].tolist(), f"fwd {i}"
            assert tick == case["tick"][i].tolist(), f"fwd {i}"
            assert clock == int(case["clock"][i]) and stats == case["stats"][i].tolist(), f"fwd {i}"
    st.close()


def test_async_bad_expert_reported_at_sync_then_recovers():
    E, H, I, K = 16, 256, 128, 4
    w13, w2, g = _weights(E, H, I, 2)
    st = _state(w13, w2, 8)
    x = torch.randn(2, H, generator=g).to(torch.bfloat16).to(DEV)
    w = torch.full((2, K), 0.25, device=DEV)
    st.forward(x, w, torch.tensor([[0, 1, 2, 3], [4, 5, 6, 99]], dtype=torch.int32, device=DEV))
    with pytest.raises(_lib.WispError) as ei:
        st.synchronize()
    assert ei.value.code == _lib.WISP_ERR_BAD_EXPERT
    assert st.stats() == [0, 0, 0, 0]                   # rejected before any bookkeeping
    ids = torch.tensor([[0, 1, 2, 3], [4, 5, 6, 7]], dtype=torch.int32)
    out = st.forward(x, w, ids.to(DEV))
    st.synchronize()
    c = compare(out.cpu(), moe_reference(x.cpu(), w13, w2, w.cpu(), ids))
    assert c["max_abs"] <= 1e-2 and c["mean_rel"] <= 1e-3, c
    st.close()


def test_dropped_pagein_times_out_without_fault_and_layer_recovers():
    """Host-side fault: the page-in engine skips one page-in, so the kernel
    waits on a slot flag nobody raises; the wait runs out after 0.3 s, the
    kernel returns, the host reads WISP_ERR_TIMEOUT and the layer restarts
    cold and computes correctly again."""
    E, H, I, K = 16, 256, 128, 4
    w13, w2, g = _weights(E, H, I, 3)
    st = _state(w13, w2, 8)
    st.configure(wait_ns=300_000_000, drop_pageins=1)
    x = torch.randn(1, H, generator=g).to(torch.bfloat16).to(DEV)
    w = torch.full((1, K), 0.25, device=DEV)
    ids = torch.tensor([[3, 1, 4, 5]], dtype=torch.int32)
    st.forward(x, w, ids.to(DEV))
    with pytest.raises(_lib.WispError) as ei:
        st.synchronize()
    assert ei.value.code == _lib.WISP_ERR_TIMEOUT
    assert st.slot_to_expert == [-1] * 8                 # cold restart
    out = st.forward(x, w, ids.to(DEV))
    st.synchronize()
    c = compare(out.cpu(), moe_reference(x.cpu(), w13, w2, w.cpu(), ids))
    assert c["max_abs"] <= 1e-2 and c["mean_rel"] <= 1e-3, c
    torch.cuda.synchronize()
    st.close()


def test_workspace_growth_while_another_layer_pages_in():
    """A forward that grows its workspace (more rows than any earlier call)
    right after another layer's forward that is still waiting for page-ins:
    the reallocation waits for the device first, so it does not stall the
    page-in thread (that forward would otherwise wait until its limit and
    restart cold)."""
    E, H, I, K = 16, 512, 256, 1
    w13, w2, g = _weights(E, H, I, 21)
    a, b = _state(w13, w2, 3, True), _state(w13, w2, 3, True)
    for st in (a, b):
        st.configure(wait_ns=2_000_000_000)
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState
    full = WispMoEState(w13, w2, E, "resident", DEV, 0)
    full.prime_identity()
    for T in (8, 40, 90):
        xa, xb = (torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV) for _ in range(2))
        ia, ib = (torch.randint(0, E, (T, K), generator=g).to(torch.int32).to(DEV) for _ in range(2))
        wa, wb = (torch.rand(T, K, generator=g).to(DEV) for _ in range(2))
        oa = a.forward(xa, wa, ia)   # pages in, waits on the page-in thread
        ob = b.forward(xb, wb, ib)   # grows b's workspace meanwhile
        a.synchronize()
        b.synchronize()
        assert torch.equal(oa, full.forward(xa, wa, ia)), T
        assert torch.equal(ob, full.forward(xb, wb, ib)), T
    for st in (a, b, full):
        st.close()


def test_paged_layers_default_to_the_synchronous_path():
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState
    E, H, I, K = 16, 256, 128, 4
    w13, w2, g = _weights(E, H, I, 22)
    paged = WispMoEState(w13, w2, 6, "paged", DEV, 0)
    res = WispMoEState(w13, w2, E, "resident", DEV, 0)
    res.prime_identity()
    x = torch.randn(5, H, generator=g).to(torch.bfloat16).to(DEV)
    w, ids = wl.softmax_topk(torch.randn(5, E, generator=g), K)
    out = paged.forward(x, w.to(DEV), ids.to(DEV))
    paged.synchronize()
    # synchronous path: pager kernel + two kernels per group; resident: one launch
    res.forward(x, w.to(DEV), ids.to(DEV))
    assert paged.telemetry()["kernel_launches"] == 1 + 2 * paged.telemetry()["groups"]
    assert res.telemetry()["kernel_launches"] == 1
    assert torch.equal(out, res.forward(x, w.to(DEV), ids.to(DEV)))
    paged.close()
    res.close()
