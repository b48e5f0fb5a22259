"""The prefetch path's host logic and the oracle against traces recorded from
the reference itself (tests/golden/make_prefetch_golden.py): the package's
co-occurrence table and predictor must issue the same predictions, in the
same order, and the oracle pager's prefetch_async must leave every layer in
the recorded state after every forward.  Also checks that the table's JSON
form matches the reference's schema and round-trips."""
import os

import numpy as np
import pytest

from oracle.pager import PagerOracle, forward_pager
from wisp_b200.integrations.vllm.cooccur import CooccurTable, NativeCooccurTable, predict_layer

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "prefetch_golden.npz")


def load_cases():
    z = np.load(GOLDEN)
    names = [str(n) for n in z["names"]]
    return {n: {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(n + "/")} for n in names}


CASES = load_cases()


def unique_set(ids):
    """The reference's ``{int(e) for e in torch.unique(topk_ids).tolist()}``:
    a set built from the ascending unique ids."""
    return {int(e) for e in np.unique(np.asarray(ids)).tolist()}


@pytest.mark.parametrize("table_cls", [CooccurTable, NativeCooccurTable], ids=["python", "native"])
@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_and_predictor_replay_reference_prefetch(name, table_cls):
    """Both tables -- the Python restatement and the library's host C++ one
    the plug-in uses -- issue the reference's predictions."""
    c = CASES[name]
    E, cap, L, S = int(c["E"]), int(c["cap"]), int(c["L"]), int(c["S"])
    pagers = [PagerOracle(E, cap) for _ in range(L)]
    last = [set() for _ in range(L)]
    table, obs = table_cls(), {}
    f = 0
    for _s in range(S):
        for l in range(L):
            forward_pager(pagers[l], c["ids"][f])
            last[l] = unique_set(c["ids"][f])
            assert sorted(last[l]) == np.nonzero(c["last"][f])[0].tolist()
            obs[l] = last[l]
            issued = None
            if l + 1 < L:
                k = max(8, pagers[l + 1].cap // 2)
                predicted = predict_layer(table, obs, l + 1, k=k, normalize=True, decay=0.5)
                if predicted:
                    issued = list(set(predicted))
                    pagers[l + 1].prefetch_async(issued, last[l + 1])
            if l == L - 1:
                table.observe_step(obs)
                obs.clear()
            n = int(c["npred"][f])
            if issued is None:
                assert n == 0, (f, "the reference prefetched")
            else:
                assert int(c["ptarget"][f]) == l + 1
                assert issued == c["pred"][f][:n].tolist(), (f, "prediction or its order")
            for j in range(L):
                p = pagers[j]
                assert p.slot_to_expert == c["s2e"][f][j].tolist(), (f, j)
                assert p.lru_tick == c["tick"][f][j].tolist(), (f, j)
                assert p.lru_clock == int(c["clock"][f][j]), (f, j)
                assert p.stats() == c["stats"][f][j].tolist(), (f, j)
            f += 1


def test_cooccur_table_schema_round_trip(tmp_path):
    t = CooccurTable()
    t.observe_step({0: {3, 1}, 1: {2}, 2: {1, 5}})
    t.observe_step({0: {1}, 2: {5}})
    d = t.to_dict()
    assert d["schema_version"] == 1 and d["num_steps_observed"] == 2
    assert sorted(map(tuple, d["marginals"])) == [(0, 1, 2), (0, 3, 1), (1, 2, 1), (2, 1, 1), (2, 5, 2)]
    assert [0, 1, 2, 5, 2] in d["pairs"] and [1, 2, 2, 1, 1] in d["pairs"]
    for name in ("t.json", "t.json.gz"):
        t.save(tmp_path / name)
        u = CooccurTable.load(tmp_path / name)
        e = u.to_dict()
        # (a source with no later-layer partner has a key only before saving,
        # as in the reference's table; the stats block is informational)
        assert {k: e[k] for k in ("schema_version", "num_steps_observed", "pairs", "marginals")} == \
            {k: d[k] for k in ("schema_version", "num_steps_observed", "pairs", "marginals")}
    assert predict_layer(t, {0: {1}}, 2, k=2) == [5, 1]
    assert predict_layer(t, {}, 2) == []


def test_native_table_matches_python_table():
    """Random steps (layers in any order, empty layers, repeated ids): the same
    serialisation, sizes and predictions under every predictor option."""
    import random
    rnd = random.Random(7)
    py, nat = CooccurTable(), NativeCooccurTable()
    L, E = 7, 24
    for _ in range(40):
        obs = {l: [rnd.randrange(E) for _ in range(rnd.randint(0, 6))]
               for l in rnd.sample(range(L), rnd.randint(1, L))}
        py.observe_step(obs)
        nat.observe_step(obs)
    assert py.to_dict() == nat.to_dict()
    assert (py.n_source_keys, py.n_pairs, py.num_steps_observed) == \
        (nat.n_source_keys, nat.n_pairs, nat.num_steps_observed)
    for _ in range(300):
        seen = {l: [rnd.randrange(E) for _ in range(rnd.randint(0, 6))]
                for l in rnd.sample(range(L), rnd.randint(0, L))}
        tgt = rnd.randrange(L + 1)
        for kw in ({}, {"normalize": False}, {"decay": 0.5}, {"decay": 0.3, "only_prev_layer": True},
                   {"k": 3, "decay": 0.7}):
            assert predict_layer(py, seen, tgt, **kw) == predict_layer(nat, seen, tgt, **kw)
    d = py.to_dict()
    assert CooccurTable.from_dict(d).to_dict() == NativeCooccurTable.from_dict(d).to_dict()
