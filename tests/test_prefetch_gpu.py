"""The device prefetch path against traces recorded from the reference itself
(tests/golden/make_prefetch_golden.py): paged layers registered like vLLM's,
each forward's pager step on the GPU, then the package's post-forward block
(predict with the co-occurrence table learned online, prefetch the next
layer on its copy stream).  After every forward, every layer's slot map,
ticks, clock and counters must equal the reference's, and every prediction
(and its order) must match."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "prefetch_golden.npz")


def load_cases():
    z = np.load(GOLDEN)
    names = [str(n) for n in z["names"]]
    return {n: {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(n + "/")} for n in names}


CASES = load_cases()


@pytest.fixture()
def fm(monkeypatch):
    from wisp_b200.integrations.vllm import fused_moe as m
    saved = list(m._LAYER_STATES)
    m._LAYER_STATES.clear()
    monkeypatch.setenv("WISP_PREFETCH", "1")
    monkeypatch.setenv("WISP_COOCCUR_ONLINE", "1")
    monkeypatch.delenv("WISP_COOCCUR_PATH", raising=False)
    monkeypatch.setattr(m, "_COOCCUR_TABLE", None)
    m._CURRENT_STEP_OBS.clear()
    yield m
    for st in m._LAYER_STATES:
        st.close()
    m._LAYER_STATES[:] = saved
    m._CURRENT_STEP_OBS.clear()


def _paging_layer(m, E, cap, idx):
    # each expert's weights hold its own id, so the slot contents can be checked
    w13 = torch.empty((E, 4, 2), dtype=torch.float32)
    w2 = torch.empty((E, 2, 4), dtype=torch.float32)
    for e in range(E):
        w13[e].fill_(float(e))
        w2[e].fill_(float(e))
    return m.WispMoEState(w13, w2, cap, "paged", DEV, idx)


@pytest.mark.parametrize("name", sorted(CASES))
def test_device_prefetch_replays_reference(fm, name):
    c = CASES[name]
    E, cap, L, S = int(c["E"]), int(c["cap"]), int(c["L"]), int(c["S"])
    states = [_paging_layer(fm, E, cap, l) for l in range(L)]
    fm._LAYER_STATES.extend(states)
    issued = []
    for st in states:
        orig = st.prefetch_async

        def rec(pred, st=st, orig=orig):
            issued.append((st.layer_idx, list(pred)))
            return orig(pred)
        st.prefetch_async = rec
    f = 0
    for _s in range(S):
        for l in range(L):
            issued.clear()
            states[l].pager_step(torch.from_numpy(np.ascontiguousarray(c["ids"][f])))
            last = states[l].last_unique_experts
            assert sorted(last) == np.nonzero(c["last"][f])[0].tolist(), f
            fm._post_forward(states[l], last)
            n = int(c["npred"][f])
            if n:
                assert issued == [(int(c["ptarget"][f]), c["pred"][f][:n].tolist())], f
            else:
                assert not issued, f
            for j in range(L):
                s2e, tick, clock, stats = states[j]._read()
                assert s2e == c["s2e"][f][j].tolist(), (f, j)
                assert tick == c["tick"][f][j].tolist(), (f, j)
                assert clock == int(c["clock"][f][j]), (f, j)
                assert stats == c["stats"][f][j].tolist(), (f, j)
            f += 1
    # slot contents: every resident expert's weights landed in its slot
    torch.cuda.synchronize()
    for st in states:
        for s, e in enumerate(st.slot_to_expert):
            if e >= 0:
                assert torch.all(st.scratch_w13[s].cpu() == float(e)), (s, e)
                assert torch.all(st.scratch_w2[s].cpu() == float(e)), (s, e)
    assert states[1].stats_pred_total > 0


def test_prefetch_rejects_out_of_range_ids(fm):
    from wisp_b200 import _lib
    st = _paging_layer(fm, 8, 4, 0)
    with pytest.raises(_lib.WispError):
        st.prefetch_async({1, 9})
    assert st._read()[2] == 0          # nothing changed, not even the clock
    st.close()
