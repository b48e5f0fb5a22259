"""The set-iteration-order model against the interpreter itself."""
import random

from oracle.setorder import set_order


def test_setorder_matches_interpreter_exhaustive_small():
    # every subset of range(12), inserted ascending
    for mask in range(1, 1 << 12):
        ks = [i for i in range(12) if mask >> i & 1]
        assert set_order(ks) == list(set(int(k) for k in ks))


def test_setorder_matches_interpreter_random_large():
    rng = random.Random(7)
    for E in (16, 64, 128, 256, 512):
        for size in range(1, E + 1):
            for _ in range(4):
                ks = sorted(rng.sample(range(E), size))
                assert set_order(ks) == list(set(int(k) for k in ks)), (E, ks)


def test_setorder_known_unsorted_case():
    # ascending insertion (what torch.unique feeds the reference) is not sorted
    # once ids reach the table size; another insertion order gives another order
    ks = [3, 10, 35, 42, 67, 74, 99, 106]
    assert set_order(ks) == [67, 35, 3, 99, 10, 42, 74, 106] == list(set(ks))
    other = [3, 35, 67, 99, 10, 42, 74, 106]
    assert set_order(other) == [99, 35, 67, 3, 10, 42, 74, 106] == list(set(other))
