"""Device pager (K1) + page-in against the reference's recorded traces and
the reference's own unit tests (tests/test_wisp_state.py:71-175)."""
import numpy as np
import pytest
import torch

from tests.conftest import GOLDEN, split_forwards

pytestmark = pytest.mark.gpu

GOLDEN_NAMES = [str(n) for n in np.load(GOLDEN)["names"]]
DEV = "cuda:0"


def make_state(E=8, cap=4, mode="paged"):
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState
    # each expert's weights hold its own id, so content checks are exact
    w13 = torch.empty((E, 4, 2), dtype=torch.float32)
    w2 = torch.empty((E, 2, 4), dtype=torch.float32)
    for e in range(E):
        w13[e].fill_(float(e))
        w2[e].fill_(float(e))
    return WispMoEState(w13, w2, cap, mode, torch.device(DEV), 0)


def need(st, experts):
    st.ensure_resident(torch.tensor(experts, dtype=torch.long, device=DEV))


def emap(st):
    torch.cuda.synchronize()
    return st.expert_map_device.cpu().tolist()


def assert_consistent(st):
    torch.cuda.synchronize()
    m = emap(st)
    s2e = st.slot_to_expert
    e2s = {e: s for s, e in enumerate(s2e) if e != -1}
    for e, s in e2s.items():
        assert m[e] == s
        assert torch.all(st.scratch_w13[s].cpu() == float(e)), f"expert {e} slot {s} w13"
        assert torch.all(st.scratch_w2[s].cpu() == float(e)), f"expert {e} slot {s} w2"
    for e in range(st.num_experts):
        if e not in e2s:
            assert m[e] == -1


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_device_pager_replays_reference_trace(golden, name):
    case = golden[name]
    E, cap = int(case["E"]), int(case["cap"])
    st = make_state(E, cap)
    fws, offs = split_forwards(case)
    for i, ids in enumerate(fws):
        t = torch.from_numpy(np.ascontiguousarray(ids))
        if case["err"][i]:
            with pytest.raises(RuntimeError, match="sub-batch"):
                st.pager_step(t)
        else:
            slots = st.pager_step(t).numpy()
            np.testing.assert_array_equal(slots, case["slots"][offs[i]:offs[i + 1]], err_msg=f"fwd {i}")
        s2e, tick, clock, stats = st._read()
        assert s2e == case["s2e"][i].tolist(), f"fwd {i}"
        assert tick == case["tick"][i].tolist(), f"fwd {i}"
        assert clock == int(case["clock"][i])
        assert stats == case["stats"][i].tolist(), f"fwd {i}"
        np.testing.assert_array_equal(np.array(emap(st), np.int32), case["emap"][i])
    assert_consistent(st)
    st.close()


@pytest.mark.parametrize("E,cap,T,K,steps,seed", [
    (128, 8, 1, 8, 300, 1), (128, 32, 16, 8, 60, 2), (512, 40, 4, 8, 80, 3),
    (1024, 64, 2, 16, 60, 4), (8, 2, 8, 2, 200, 5), (256, 200, 32, 8, 20, 6)])
def test_device_pager_matches_oracle_random(E, cap, T, K, steps, seed):
    """Long random traces (ids beyond the set-table size, ids64, large E)."""
    from oracle.pager import PagerOracle, forward_pager
    rng = np.random.default_rng(seed)
    st = make_state(E, cap)
    p = PagerOracle(E, cap)
    for step in range(steps):
        ids = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int64)
        _, slots_ref, _ = forward_pager(p, ids)
        slots = st.pager_step(torch.from_numpy(ids)).numpy()
        np.testing.assert_array_equal(slots, slots_ref, err_msg=f"step {step}")
    s2e, tick, clock, stats = st._read()
    assert (s2e, tick, clock, stats) == (p.slot_to_expert, p.lru_tick, p.lru_clock, p.stats())
    assert_consistent(st)
    st.close()


def test_bad_expert_id_rejected_without_state_change():
    from wisp_b200._lib import WispError, WISP_ERR_BAD_EXPERT
    st = make_state(8, 4)
    need(st, [0, 1])
    before = st._read()
    with pytest.raises(WispError) as ei:
        st.pager_step(torch.tensor([[0, 9]]))
    assert ei.value.code == WISP_ERR_BAD_EXPERT
    assert st._read()[:3] == before[:3]


# ---- the reference's unit tests, on the device pager --------------------------

def test_miss_then_hit():
    st = make_state()
    need(st, [0, 1])
    assert st.stats_miss == 2 and st.stats_hits == 0
    assert_consistent(st)
    need(st, [0, 1])
    assert st.stats_miss == 2 and st.stats_hits == 2 and st.stats_evict == 0
    assert_consistent(st)


def test_lru_eviction_order():
    st = make_state()
    need(st, [0, 1])
    need(st, [2, 3])
    assert st.slot_to_expert == [3, 2, 1, 0]
    need(st, [4])
    # lowest tick, ties to the lower slot: slot 2 (expert 1)
    assert st.slot_to_expert == [3, 2, 4, 0]
    assert emap(st)[4] == 2 and st.stats_evict == 1
    assert_consistent(st)


def test_needed_set_never_evicted():
    st = make_state()
    need(st, [0, 1, 2, 3])
    need(st, [0, 1, 4])
    e2s = st.expert_to_slot
    assert 0 in e2s and 1 in e2s and 4 in e2s
    assert (2 in e2s) != (3 in e2s)
    assert_consistent(st)


def test_working_set_overflow_raises():
    st = make_state()
    with pytest.raises(RuntimeError, match="sub-batch"):
        need(st, [0, 1, 2, 3, 4])


def test_map_consistency_random_walk():
    torch.manual_seed(0)
    st = make_state()
    for _ in range(50):
        k = int(torch.randint(1, 5, ()).item())
        experts = torch.randperm(8)[:k].tolist()
        need(st, experts)
        e2s = st.expert_to_slot
        for e in experts:
            assert e in e2s
    assert_consistent(st)


def test_resize_grow_preserves_residents():
    st = make_state()
    need(st, [0, 1, 2, 3])
    st.resize_cap(6)
    assert st.cap_experts == 6
    s2e = st.slot_to_expert
    assert len(s2e) == 6 and len(st.lru_tick) == 6 and s2e[4:] == [-1, -1]
    assert_consistent(st)
    ev = st.stats_evict
    need(st, [4, 5])
    assert st.stats_evict == ev
    assert_consistent(st)


def test_resize_shrink_drops_tail_and_repages():
    st = make_state()
    need(st, [0, 1, 2, 3])
    tail = [e for e in st.slot_to_expert[2:] if e != -1]
    st.resize_cap(2)
    assert st.cap_experts == 2 and len(st.slot_to_expert) == 2
    m = emap(st)
    for e in tail:
        assert e not in st.expert_to_slot and m[e] == -1
    assert_consistent(st)
    need(st, [tail[0]])
    assert tail[0] in st.expert_to_slot
    assert_consistent(st)


def test_resize_noop_and_clamps():
    st = make_state()
    need(st, [0, 1])
    st.resize_cap(4)
    assert st.cap_experts == 4
    st.resize_cap(1)
    assert st.cap_experts == 2
    st.resize_cap(999)
    assert st.cap_experts == 8
    assert_consistent(st)


def test_prime_identity_resident_mode():
    st = make_state(cap=8, mode="resident")
    st.prime_identity()
    torch.cuda.synchronize()
    assert emap(st) == list(range(8))
    assert_consistent(st)
