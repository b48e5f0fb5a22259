"""The allocation-free expert compute (``wisp_expert_compute_noalloc``).

It serves callers that may not call cudaMalloc themselves (a plug-in inside a
serving engine that has reserved the free HBM for its KV cache, or a decode
loop that cannot take cudaMalloc's implicit device synchronisation): its
intermediates live in one static device array.  Here it is called through
the C ABI on a layer's slot scratch and compared with the regular entry point
(``wisp_moe_forward``) on two calls in a row, within the parity tolerance of
the other tests (max-abs 1e-2, mean-rel 1e-3).  This file is collected last
so that a run stopping at its first failure has run every other test.
"""
import pytest
import torch

from oracle.moe import compare
from wisp_b200 import _lib
from wisp_b200 import workloads as wl

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _noalloc(st, x, w, slots, out):
    L = _lib.lib()
    rc = L.wisp_expert_compute_noalloc(
        DEV.index, x.data_ptr(), st.scratch_w13.data_ptr(), st.scratch_w2.data_ptr(),
        st.cap_experts, slots.data_ptr(), w.data_ptr(), x.shape[0], slots.shape[1],
        st.hidden_size, st.intermediate_size, out.data_ptr(),
        _lib.stream_ptr(torch.cuda.current_stream(DEV)))
    _lib.check(rc, "wisp_expert_compute_noalloc")


def _case(E, H, I, T, K, seed):
    g = torch.Generator().manual_seed(seed)
    w13 = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
    return w13, w2, g


def test_noalloc_matches_forward_on_two_calls_resident():
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState
    E, H, I, K = 32, 512, 256, 4
    w13, w2, g = _case(E, H, I, 8, K, seed=21)
    st = WispMoEState(w13, w2, E, "resident", DEV, 0)
    st.prime_identity()
    for T in (8, 3):                               # two calls in a row
        x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
        w, ids = wl.softmax_topk(torch.randn(T, E, generator=g), K)
        w, ids = w.to(DEV), ids.to(DEV)
        ref = st.forward(x, w, ids)
        out = torch.full_like(x, float("nan"))
        _noalloc(st, x, w, ids.to(torch.int32).contiguous(), out)   # identity map: slot == expert
        torch.cuda.synchronize()
        c = compare(out.cpu(), ref.cpu().float())
        assert c["max_abs"] <= 1e-2 and c["mean_rel"] <= 1e-3, c
    st.close()


def test_noalloc_matches_forward_on_two_calls_paged():
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState
    shape = wl.QWEN3_30B
    E, K = 32, 8
    cap = E                                        # one group; LRU-placed, non-identity slots
    w13, w2, g = _case(E, shape.hidden, shape.inter, 16, K, seed=22)
    st = WispMoEState(w13, w2, cap, "paged", DEV, 0)
    for T in (16, 1):                              # two calls in a row
        x = torch.randn(T, shape.hidden, generator=g).to(torch.bfloat16).to(DEV)
        w, ids = wl.softmax_topk(torch.randn(T, E, generator=g), K)
        w, ids = w.to(DEV), ids.to(DEV)
        slots = st.pager_step(ids)                 # pages the routed experts in (one group: cap == E)
        ref = st.forward(x, w, ids)                # all hits now: same slots
        out = torch.full_like(x, float("nan"))
        _noalloc(st, x, w, slots.to(DEV).contiguous(), out)
        torch.cuda.synchronize()
        c = compare(out.cpu(), ref.cpu().float())
        assert c["max_abs"] <= 1e-2 and c["mean_rel"] <= 1e-3, c
    st.close()


def test_noalloc_takes_no_device_memory_after_setup():
    """A zero-token call places the static array and the kernels' code on the
    device; after it (and a first compute call), a call leaves the device's
    free memory and torch's allocator untouched.  The largest call the array
    admits, 128 pairs at top_k 1, matches the regular forward."""
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState
    E, H, I, K, T = 64, 1024, 512, 1, 128
    w13, w2, g = _case(E, H, I, T, K, seed=23)
    st = WispMoEState(w13, w2, E, "resident", DEV, 0)
    st.prime_identity()
    L = _lib.lib()
    _lib.check(L.wisp_expert_compute_noalloc(DEV.index, None, None, None, 0, None, None, 0, 0, 0, 0,
                                             None, None), "set-up call")
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    w, ids = wl.softmax_topk(torch.randn(T, E, generator=g), K)
    w, ids = w.to(DEV), ids.to(DEV)
    slots = ids.to(torch.int32).contiguous()
    ref = st.forward(x, w, ids)
    out = torch.full_like(x, float("nan"))
    _noalloc(st, x, w, slots, out)                 # first compute call
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(DEV)
    alloc0 = torch.cuda.memory_allocated(DEV)
    out.fill_(float("nan"))
    _noalloc(st, x, w, slots, out)                 # second call: nothing may be allocated
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(DEV)
    assert (free1, torch.cuda.memory_allocated(DEV)) == (free0, alloc0)
    c = compare(out.cpu(), ref.cpu().float())
    assert c["max_abs"] <= 1e-2 and c["mean_rel"] <= 1e-3, c
    st.close()


def test_noalloc_rejects_sizes_beyond_the_static_scratch():
    L = _lib.lib()
    rc = L.wisp_expert_compute_noalloc(0, None, None, None, 8, None, None, 17, 8, 2048, 768, None,
                                       None)
    assert rc == _lib.WISP_ERR_INVALID
    assert b"static scratch" in L.wisp_last_error()
    rc = L.wisp_expert_compute_noalloc(0, None, None, None, 8, None, None, 1, 8, 16384, 768, None,
                                       None)
    assert rc == _lib.WISP_ERR_INVALID
