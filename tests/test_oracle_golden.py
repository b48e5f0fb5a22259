"""The CPU oracle pager against traces recorded from the reference itself."""
import numpy as np
import pytest

from oracle.pager import PagerOracle, PagerOverflow, forward_pager
from tests.conftest import split_forwards


def replay(case):
    E, cap = int(case["E"]), int(case["cap"])
    p = PagerOracle(E, cap)
    fws, offs = split_forwards(case)
    for i, ids in enumerate(fws):
        if case["err"][i]:
            with pytest.raises(PagerOverflow):
                forward_pager(p, ids)
        else:
            _, slots, _ = forward_pager(p, ids)
            np.testing.assert_array_equal(slots, case["slots"][offs[i]:offs[i + 1]])
        assert p.slot_to_expert == case["s2e"][i].tolist(), i
        assert p.lru_tick == case["tick"][i].tolist(), i
        assert p.lru_clock == int(case["clock"][i])
        assert p.stats() == case["stats"][i].tolist(), i
        np.testing.assert_array_equal(p.expert_map(), case["emap"][i])


def test_golden_cases_present(golden):
    assert len(golden) >= 30
    assert "cfg1_b1_cap8" in golden and "overflow_cap4" in golden


@pytest.mark.parametrize("name", [
    "cfg1_b1_cap8", "cfg2_b1_cap8_l0", "cfg2_b4_cap16_l1", "cfg2_b16_cap8_l0",
    "cfg2_b16_cap32_l1", "cfg3_chunk0_cap32", "cfg3_chunk1_cap32", "cfg4_b1_cap2",
    "cfg4_b8_cap4", "cfg5_local64_cap16_b64", "overflow_cap4", "ragged_e16_cap5"])
def test_oracle_matches_reference_trace(golden, name):
    replay(golden[name])


def test_oracle_matches_every_golden_case(golden):
    for name, case in golden.items():
        replay(case)


# --- the reference's own unit tests (tests/test_wisp_state.py:71-175), on the oracle

def test_miss_then_hit():
    p = PagerOracle(8, 4)
    p.ensure_resident([0, 1])
    assert (p.stats_miss, p.stats_hits) == (2, 0)
    p.ensure_resident([0, 1])
    assert (p.stats_miss, p.stats_hits, p.stats_evict) == (2, 2, 0)


def test_lru_eviction_order_exact():
    p = PagerOracle(8, 4)
    p.ensure_resident([0, 1])
    p.ensure_resident([2, 3])
    # LIFO pops from free [0,1,2,3]: 0->3, 1->2, then 2->1, 3->0
    assert p.slot_to_expert == [3, 2, 1, 0]
    rec = p.ensure_resident([4])
    # lowest tick first, ties to the lower slot: slot 2 (expert 1, tick 1)
    assert rec.victims == [(2, 1)] and rec.placed == [(4, 2)]
    assert p.stats_evict == 1 and p.slot_to_expert == [3, 2, 4, 0]


def test_needed_set_never_evicted():
    p = PagerOracle(8, 4)
    p.ensure_resident([0, 1, 2, 3])
    p.ensure_resident([0, 1, 4])
    assert 0 in p.expert_to_slot and 1 in p.expert_to_slot and 4 in p.expert_to_slot
    assert (2 in p.expert_to_slot) != (3 in p.expert_to_slot)


def test_working_set_overflow_raises():
    p = PagerOracle(8, 4)
    with pytest.raises(PagerOverflow, match="sub-batch"):
        p.ensure_resident([0, 1, 2, 3, 4])


def test_resize_semantics():
    p = PagerOracle(8, 4)
    p.ensure_resident([0, 1, 2, 3])
    p.resize_cap(6)
    assert p.cap == 6 and p.slot_to_expert[4:] == [-1, -1]
    ev = p.stats_evict
    p.ensure_resident([4, 5])
    assert p.stats_evict == ev
    p.resize_cap(2)
    assert len(p.slot_to_expert) == 2
    p.resize_cap(1)
    assert p.cap == 2
    p.resize_cap(999)
    assert p.cap == 8
