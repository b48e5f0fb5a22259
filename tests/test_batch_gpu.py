"""Decode batches on the weight-stationary tensor-core path (calls of
tc_min_pairs <= T * k <= 512 pairs): parity with the fp32 CPU oracle under
the same bounds as the prefill path (mean-rel <= 1e-3; per element
|out - ref| <= max(1e-2, 2 ulp(ref) + sum over k of 2 ulp(y_k)), the stored
bf16 values may each round the other way with another fp32 accumulation
order), byte identity across caps, modes and slot placements, agreement with
the token-major GEMMs on the same pairs, the pager state unchanged by the
path, the kernel count (resident: one persistent kernel that routes the call
itself, counts the forward and combines, with no pager launch and no host
round trip; paged: pager + gather and the persistent kernel per group), the
threshold knob, and a routed id out of range reported at
synchronize with no counter changed."""
import pytest
import torch

from oracle.moe import compare, moe_reference
from oracle.pager import PagerOracle, forward_pager
from tests.test_moe_gpu import MAX_ABS, MEAN_REL, fwd, rand_case, state
from wisp_b200 import _lib
from wisp_b200 import workloads as wl

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _bf16_ulp(v):
    return torch.ldexp(torch.ones_like(v), torch.frexp(v.abs().clamp_min(1e-30))[1] - 8)


def assert_parity(out, x, w13, w2, w, ids):
    ref, Y = moe_reference(x, w13, w2, w, ids, return_partials=True)
    c = compare(out, ref)
    assert c["mean_rel"] <= MEAN_REL, c
    bound = torch.clamp_min(2 * _bf16_ulp(ref) + (2 * _bf16_ulp(Y)).sum(dim=1), MAX_ABS)
    d = (out.float() - ref).abs()
    assert bool((d <= bound).all()), (c, float((d - bound).max()))
    return c


@pytest.mark.parametrize("E,H,I,T,K,cap,mode", [
    (128, 2048, 768, 16, 8, 128, "resident"),   # Qwen3-30B-A3B decode, batch 16
    (128, 2048, 768, 8, 8, 128, "resident"),    # batch 8 (64 pairs)
    (128, 2048, 768, 3, 8, 128, "resident"),    # batch 3 (24 pairs, above the default 22)
    (128, 2048, 768, 64, 8, 128, "resident"),   # batch 64 (512 pairs: the largest call on this path)
    (128, 2048, 768, 40, 8, 64, "paged"),       # 320 pairs, paged groups
    (128, 2048, 768, 16, 8, 40, "paged"),       # paged, several groups
    (8, 4096, 1536, 32, 2, 8, "resident"),      # Qwen3-235B hidden/inter, top-2, 8 tokens/expert
    (16, 256, 128, 64, 4, 16, "resident"),      # small shapes, > 32 pairs per expert (several token blocks)
    (32, 512, 256, 40, 4, 12, "paged"),
])
def test_batch_matches_oracle(E, H, I, T, K, cap, mode):
    w13, w2, x, w, ids = rand_case(E, H, I, T, K, seed=T * K + H)
    st = state(w13, w2, cap, mode)
    out = fwd(st, x, w, ids)
    assert_parity(out, x, w13, w2, w, ids)
    assert torch.equal(fwd(st, x, w, ids), out)
    st.close()


def test_batch_byte_identical_across_caps_modes_and_placements():
    E, H, I, T, K = 32, 512, 256, 24, 4
    w13, w2, x, w, ids = rand_case(E, H, I, T, K, seed=17)
    outs = []
    for cap, mode in ((32, "resident"), (32, "paged"), (20, "paged"), (9, "paged")):
        st = state(w13, w2, cap, mode)
        if mode == "paged":  # a different slot placement first
            st.ensure_resident(torch.arange(E - 1, E - 1 - min(cap, E), -1, dtype=torch.int32))
        outs.append(fwd(st, x, w, ids))
        st.close()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


def test_batch_agrees_with_token_major_gemm():
    """512 pairs run weight-stationary, 520 pairs token-major: the first 64
    tokens' outputs (the same pairs) are byte-identical, so the two
    tensor-core paths are one numeric class."""
    E, H, I, K = 32, 512, 256, 8
    w13, w2, x, w, ids = rand_case(E, H, I, 65, K, seed=23)
    st = state(w13, w2, E, "resident")
    big = fwd(st, x, w, ids)                    # 520 pairs: token-major GEMMs
    small = fwd(st, x[:64], w[:64], ids[:64])   # 512 pairs: weight-stationary
    assert torch.equal(big[:64], small)
    st.close()


def test_default_threshold_follows_the_expert_shape():
    """Default: the smallest call whose tiles (I/128 + H/256 per pair) could
    fill the GPU twice over; the same for every E (expert-parallel shards)."""
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    for E, H, I in ((128, 2048, 768), (16, 2048, 768), (16, 512, 256), (4, 4096, 1536)):
        w13 = torch.zeros(E, 2 * I, H, dtype=torch.bfloat16)
        w2 = torch.zeros(E, H, I, dtype=torch.bfloat16)
        st = state(w13, w2, E, "paged")
        per = I // 128 + H // 256
        assert st.tc_min_pairs == min(max(-(-2 * sms // per), 1), 513), (E, H, I)
        st.close()


def test_batch_pager_state_and_kernel_count():
    E, H, I, T, K, cap = 32, 256, 128, 20, 4, 10
    w13, w2, x, _, _ = rand_case(E, H, I, T, K, seed=29)
    st = state(w13, w2, cap)
    st.configure(tc_min_pairs=1)
    oracle = PagerOracle(E, cap)
    for step in range(3):
        g = torch.Generator().manual_seed(200 + step)
        w, ids = wl.softmax_topk(torch.randn(T, E, generator=g), K)
        l0, g0 = st.telemetry()["kernel_launches"], st.telemetry()["groups"]
        out = fwd(st, x, w, ids)
        groups, _, _ = forward_pager(oracle, ids.numpy())
        tel = st.telemetry()
        assert tel["groups"] - g0 == len(groups)
        assert tel["kernel_launches"] - l0 == 1 + 2 * len(groups)
        s2e, tick, clock, stats = st._read()
        assert s2e == oracle.slot_to_expert and tick == oracle.lru_tick and clock == oracle.lru_clock
        assert stats == oracle.stats()
        assert_parity(out, x, w13, w2, w, ids)
    st.close()
    res = state(w13, w2, E, "resident")
    res.configure(tc_min_pairs=1)
    l0 = res.telemetry()["kernel_launches"]
    res.forward(x.to(DEV), w.to(DEV), ids.to(DEV))
    res.synchronize()
    tel = res.telemetry()
    assert tel["kernel_launches"] - l0 == 1
    assert res.stats() == [1, 0, 0, 0]
    assert tel["groups"] == 1 and tel["unique_experts"] == len(set(ids.reshape(-1).tolist()))
    res.close()


def test_threshold_knob_selects_the_path():
    E, H, I, T, K = 16, 256, 128, 8, 4   # 32 pairs: CUDA-core kernels by default (threshold 148)
    w13, w2, x, w, ids = rand_case(E, H, I, T, K, seed=31)
    st = state(w13, w2, E, "resident")
    assert st.tc_min_pairs > T * K
    l0 = st.telemetry()["kernel_launches"]
    a = fwd(st, x, w, ids)
    assert st.telemetry()["kernel_launches"] - l0 == 1      # one-launch forward
    st.configure(tc_min_pairs=32)
    l0 = st.telemetry()["kernel_launches"]
    b = fwd(st, x, w, ids)
    assert st.telemetry()["kernel_launches"] - l0 == 1      # the routing persistent kernel
    for o in (a, b):
        assert_parity(o, x, w13, w2, w, ids)
    with pytest.raises(_lib.WispError):
        st.configure(tc_min_pairs=0)
    st.close()


def test_batch_bad_expert_reported_at_sync_then_recovers():
    E, H, I, T, K = 16, 256, 128, 16, 4
    w13, w2, x, w, ids = rand_case(E, H, I, T, K, seed=37)
    st = state(w13, w2, E, "resident")
    st.configure(tc_min_pairs=1)
    bad = ids.clone()
    bad[3, 1] = E + 5
    st.forward(x.to(DEV), w.to(DEV), bad.to(torch.int32).to(DEV))
    with pytest.raises(_lib.WispError) as ei:
        st.synchronize()
    assert ei.value.code == _lib.WISP_ERR_BAD_EXPERT
    assert st.stats()[0] == 0                               # rejected before any bookkeeping
    out = fwd(st, x, w, ids)
    assert_parity(out, x, w13, w2, w, ids)
    st.close()


def test_resident_forward_before_prime_is_rejected():
    """A resident layer's slots are filled by prime_identity only: a forward
    before it is an argument error on the host, not a read of empty slots."""
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState
    E, H, I, T, K = 16, 256, 128, 16, 4
    w13, w2, x, w, ids = rand_case(E, H, I, T, K, seed=41)
    st = WispMoEState(w13, w2, E, "resident", DEV, 0)
    for t in (1, T):   # the CUDA-core and the tensor-core class
        with pytest.raises(_lib.WispError) as ei:
            st.forward(x[:t].to(DEV), w[:t].to(DEV), ids[:t].to(DEV))
        assert ei.value.code == _lib.WISP_ERR_INVALID
    st.prime_identity()
    st.configure(tc_min_pairs=1)
    assert_parity(fwd(st, x, w, ids), x, w13, w2, w, ids)
    st.close()

