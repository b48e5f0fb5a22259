"""Record golden traces of the reference's prefetch path by running the
REFERENCE itself on CPU.

    python tests/golden/make_prefetch_golden.py /path/to/reference/src

Same stand-ins as ``make_golden.py`` (no-op CUDA streams / events, a
recording ``fused_experts``).  A stack of paged layers is registered in the
reference's ``_LAYER_STATES`` and decoded step by step with
``WISP_PREFETCH=1`` and ``WISP_COOCCUR_ONLINE=1`` (a cold co-occurrence table
that learns online), so the reference's own post-forward block
(src/wisp/integrations/vllm/fused_moe.py:1170-1233) observes each step,
predicts the next layer's experts (src/wisp/oracle/cooccur.py:228-292) and
calls ``prefetch_async`` (fused_moe.py:360-433).  After every layer forward
the pager state of every layer is snapshotted, and every ``prefetch_async``
call is recorded with its argument in the order the reference iterates it.

Output: ``tests/golden/prefetch_golden.npz``.  The GPU box never runs this
script; tests read only the ``.npz``.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from make_golden import _Layer, _Method, load_reference  # noqa: E402
from wisp_b200 import workloads as wl  # noqa: E402

MAX_PRED = 64


def run_stack(fm, E, cap, L, steps):
    """steps: [S][L] int32 [T, k] arrays."""
    os.environ["WISP_PREFETCH"] = "1"
    os.environ["WISP_COOCCUR_ONLINE"] = "1"
    os.environ.pop("WISP_COOCCUR_PATH", None)
    fm._COOCCUR_TABLE = None
    fm._CURRENT_STEP_OBS.clear()
    fm._LAYER_STATES.clear()
    states = [fm.WispMoEState(torch.zeros(E, 2, 1), torch.zeros(E, 1, 1), cap, "paged", torch.device("cpu"), l)
              for l in range(L)]
    fm._LAYER_STATES.extend(states)
    preds = []
    orig = fm.WispMoEState.prefetch_async

    def recording(self, predicted_experts):
        preds.append((self.layer_idx, list(predicted_experts)))   # the reference's iteration order
        return orig(self, predicted_experts)

    fm.WispMoEState.prefetch_async = recording
    rec = {k: [] for k in ("s2e", "tick", "clock", "stats", "last", "pred", "npred", "ptarget", "ids")}
    try:
        for s in range(len(steps)):
            for l in range(L):
                ids_t = torch.from_numpy(np.ascontiguousarray(steps[s][l])).to(torch.int32)
                T, K = ids_t.shape
                layer = _Layer()
                layer.select_experts = lambda ids_t=ids_t, T=T, K=K, **kw: (torch.ones(T, K) / K, ids_t, None)
                preds.clear()
                fm._wisp_forward_cuda_paged(_Method(), layer, torch.zeros(T, 1), states[l], False, K, None, True)
                rec["s2e"].append([list(st.slot_to_expert) for st in states])
                rec["tick"].append([list(st.lru_tick) for st in states])
                rec["clock"].append([st.lru_clock for st in states])
                rec["stats"].append([[st.stats_forward, st.stats_miss, st.stats_hits, st.stats_evict]
                                     for st in states])
                last = np.full(E, 0, np.int8)
                last[sorted(states[l].last_unique_experts)] = 1
                rec["last"].append(last)
                p = np.full(MAX_PRED, -1, np.int32)
                assert len(preds) <= 1
                if preds:
                    target, lst = preds[0]
                    p[:len(lst)] = lst
                    rec["npred"].append(len(lst))
                    rec["ptarget"].append(target)
                else:
                    rec["npred"].append(0)
                    rec["ptarget"].append(-1)
                rec["pred"].append(p)
                rec["ids"].append(ids_t.numpy())
    finally:
        fm.WispMoEState.prefetch_async = orig
        fm._LAYER_STATES.clear()
    return {
        "s2e": np.array(rec["s2e"], np.int32), "tick": np.array(rec["tick"], np.int64),
        "clock": np.array(rec["clock"], np.int64), "stats": np.array(rec["stats"], np.int64),
        "last": np.array(rec["last"], np.int8), "pred": np.array(rec["pred"], np.int32),
        "npred": np.array(rec["npred"], np.int32), "ptarget": np.array(rec["ptarget"], np.int32),
        "ids": np.stack(rec["ids"]).astype(np.int32),
        "E": np.int32(E), "cap": np.int32(cap), "L": np.int32(L), "S": np.int32(len(steps)),
    }


def correlated_trace(S, L, B, E, k, seed):
    """Zipf routing whose layer-l+1 experts follow layer l's (a fixed random
    map per layer pair), so the co-occurrence table has a signal to learn."""
    ids, _ = wl.zipf_trace(S, L, B, E, k, 1.1, 0.3, seed=seed)
    rng = np.random.default_rng(seed + 1)
    follow = [rng.permutation(E) for _ in range(L)]
    out = ids.copy()
    for s in range(S):
        for l in range(1, L):
            for b in range(B):
                if rng.random() < 0.7:
                    cand = follow[l][out[s, l - 1, b]]
                    seen, row = set(), []
                    for e in list(cand) + list(out[s, l, b]):
                        if int(e) not in seen:
                            seen.add(int(e))
                            row.append(int(e))
                    out[s, l, b] = np.array(row[:k], np.int32)
    return [[out[s, l] for l in range(L)] for s in range(S)]


def cases():
    return [
        ("pf_e16_cap6_l4_b2", 16, 6, 4, correlated_trace(24, 4, 2, 16, 2, seed=1)),
        ("pf_e32_cap12_l3_b4", 32, 12, 3, correlated_trace(20, 3, 4, 32, 4, seed=2)),
        ("pf_e128_cap32_l4_b1", 128, 32, 4, correlated_trace(16, 4, 1, 128, 8, seed=3)),
        ("pf_e64_cap16_l3_b2", 64, 16, 3, correlated_trace(16, 3, 2, 64, 8, seed=4)),
    ]


def main():
    src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get(
        "WISP_REFERENCE_SRC", os.path.join(os.path.dirname(REPO), "reference", "src"))
    fm, _calls = load_reference(src)
    blob, names = {}, []
    for name, E, cap, L, steps in cases():
        res = run_stack(fm, E, cap, L, steps)
        for k, v in res.items():
            blob[f"{name}/{k}"] = v
        names.append(name)
        print(f"{name}: forwards={len(res['npred'])} prefetches={int((res['npred'] > 0).sum())} "
              f"final stats={res['stats'][-1].tolist()}")
    blob["names"] = np.array(names)
    path = os.path.join(HERE, "prefetch_golden.npz")
    np.savez_compressed(path, **blob)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
