"""Record golden pager traces by running the REFERENCE itself on CPU.

Run in a container that has the reference checkout (default
``$WISP_REFERENCE_SRC`` or ``../reference/src`` relative to the repo root):

    python tests/golden/make_golden.py /path/to/reference/src

It imports the reference's ``WispMoEState`` and ``_wisp_forward_cuda_paged``
(src/wisp/integrations/vllm/fused_moe.py:126-490, 990-1237) with three
no-op stand-ins for ``torch.cuda.Stream`` / ``Event`` / ``current_stream``
and a recording stand-in for vLLM's ``fused_experts``.  The reference's own
code then performs the first-fit sub-batching and every ``ensure_resident``
call; the stand-in ``fused_experts`` records, per call, the slot each
``(t, k)`` reads (``expert_map[topk_ids]`` at call time).  After every
forward the pager state is snapshotted.

Output: ``tests/golden/pager_golden.npz`` (a few hundred KB).  The GPU box
never runs this script; tests read only the ``.npz``.
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, REPO)

from wisp_b200 import workloads as wl  # noqa: E402


class _NoStream:
    def __init__(self, *a, **k):
        pass

    def wait_event(self, *a, **k):
        pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


class _NoEvent:
    def __init__(self, *a, **k):
        pass

    def record(self, *a, **k):
        pass


def load_reference(src: str):
    torch.cuda.Stream = _NoStream
    torch.cuda.Event = _NoEvent
    torch.cuda.current_stream = lambda *a, **k: _NoStream()
    torch.cuda.stream = lambda s: _NoStream()
    sys.path.insert(0, src)
    calls: list = []
    fake = types.ModuleType("vllm.model_executor.layers.fused_moe.fused_moe")

    def fused_experts(hidden_states, w1, w2, topk_weights, topk_ids, inplace=False,
                      expert_map=None, **kw):
        calls.append((topk_ids.clone(), expert_map[topk_ids.long()].clone()))
        return torch.zeros_like(hidden_states)

    fake.fused_experts = fused_experts
    sys.modules["vllm.model_executor.layers.fused_moe.fused_moe"] = fake
    from wisp.integrations.vllm import fused_moe as fm
    return fm, calls


class _Layer:
    num_fused_shared_experts = 0


class _Method:
    topk_indices_dtype = None
    moe_quant_config = None


def run_trace(fm, calls, E, cap, forwards):
    """forwards: list of int32 [T, k] arrays (one per forward)."""
    st = fm.WispMoEState(torch.zeros(E, 2, 1), torch.zeros(E, 1, 1), cap, "paged",
                         torch.device("cpu"), 0)
    rec = {k: [] for k in ("s2e", "tick", "clock", "stats", "emap", "slots",
                            "ids", "ncalls", "T", "err")}
    for ids in forwards:
        ids_t = torch.from_numpy(np.ascontiguousarray(ids)).to(torch.int32)
        T, K = ids_t.shape
        layer = _Layer()
        layer.select_experts = lambda **kw: (torch.ones(T, K) / K, ids_t, None)
        calls.clear()
        err = 0
        try:
            fm._wisp_forward_cuda_paged(_Method(), layer, torch.zeros(T, 1), st,
                                        False, K, None, True)
        except RuntimeError as e:
            assert "sub-batch" in str(e)
            err = 1
        slots = np.full((T, K), -1, np.int32)
        row = 0
        for tid, sl in calls:
            n = tid.shape[0]
            slots[row:row + n] = sl.numpy()
            row += n
        rec["s2e"].append(list(st.slot_to_expert))
        rec["tick"].append(list(st.lru_tick))
        rec["clock"].append(st.lru_clock)
        rec["stats"].append([st.stats_forward, st.stats_miss, st.stats_hits, st.stats_evict])
        rec["emap"].append(st.expert_map_device.numpy().copy())
        rec["slots"].append(slots)
        rec["ids"].append(ids_t.numpy())
        rec["ncalls"].append(len(calls))
        rec["T"].append(T)
        rec["err"].append(err)
        if err:
            break
    out = {
        "s2e": np.array(rec["s2e"], np.int32),
        "tick": np.array(rec["tick"], np.int64),
        "clock": np.array(rec["clock"], np.int64),
        "stats": np.array(rec["stats"], np.int64),
        "emap": np.array(rec["emap"], np.int32),
        "slots": np.concatenate(rec["slots"]).astype(np.int32),
        "ids": np.concatenate(rec["ids"]).astype(np.int32),
        "ncalls": np.array(rec["ncalls"], np.int32),
        "T": np.array(rec["T"], np.int32),
        "err": np.array(rec["err"], np.int32),
        "E": np.int32(E), "cap": np.int32(cap),
    }
    return out


def cases():
    """(name, E, cap, list of per-forward [T,k] id arrays)."""
    out = []
    # config 1: Qwen3-30B layer, logits routing, 256 decode tokens at B=1, cap 8
    _, ids = wl.logits_routing(256, 128, 8, seed=0)
    out.append(("cfg1_b1_cap8", 128, 8, [ids[t:t + 1].numpy() for t in range(256)]))
    # config 2 shape: Zipf(1.1), reuse 0.6, B in {1,4,16}, caps 8..32 (2 layers, 48 steps)
    for B in (1, 4, 16):
        tids, _ = wl.zipf_trace(48, 2, B, 128, 8, 1.1, 0.6, seed=2)
        for cap in (8, 16, 24, 32):
            for layer in range(2):
                out.append((f"cfg2_b{B}_cap{cap}_l{layer}", 128, cap,
                            [tids[t, layer] for t in range(48)]))
    # config 3 shape: uniform top-8 of 128, chunks of 256 tokens, cap 32
    for c in range(2):
        tids, _ = wl.uniform_topk(256, 128, 8, seed=30 + c)
        out.append((f"cfg3_chunk{c}_cap32", 128, 32, [tids]))
    # config 4 shape: Mixtral E=8 top-2, Zipf(0.8), B in {1,8}, caps {2,4}
    for B in (1, 8):
        tids, _ = wl.zipf_trace(64, 1, B, 8, 2, 0.8, 0.0, seed=4)
        for cap in (2, 4):
            out.append((f"cfg4_b{B}_cap{cap}", 8, cap, [tids[t, 0] for t in range(64)]))
    # config 5 shape (per-rank local pager): 64 local experts (P=2), cap 16, B=64
    tids, _ = wl.zipf_trace(8, 1, 64, 64, 8, 1.1, 0.5, seed=5)
    out.append(("cfg5_local64_cap16_b64", 64, 16, [tids[t, 0] for t in range(8)]))
    # overflow: a single token with more unique experts than the cap
    rng = np.random.default_rng(9)
    # (duplicated ids inside a token are legal and collapse in the needed set)
    fw = [np.array([[0, 1, 1, 0, 0]], np.int32), np.array([[2, 3, 3, 2, 2]], np.int32),
          np.array([[0, 4, 5, 6, 7]], np.int32)]
    out.append(("overflow_cap4", 8, 4, fw))
    # small random walk with repeated / ragged batches (T from 1 to 6)
    fw = []
    for _ in range(40):
        T = int(rng.integers(1, 7))
        fw.append(np.stack([rng.permutation(16)[:3] for _ in range(T)]).astype(np.int32))
    out.append(("ragged_e16_cap5", 16, 5, fw))
    return out


def main():
    src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get(
        "WISP_REFERENCE_SRC", os.path.join(os.path.dirname(REPO), "reference", "src"))
    fm, calls = load_reference(src)
    blob = {}
    names = []
    for name, E, cap, fw in cases():
        res = run_trace(fm, calls, E, cap, fw)
        for k, v in res.items():
            blob[f"{name}/{k}"] = v
        names.append(name)
        print(f"{name}: forwards={len(res['T'])} calls={int(res['ncalls'].sum())} "
              f"stats={res['stats'][-1].tolist()} err={int(res['err'].max())}")
    blob["names"] = np.array(names)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "pager_golden.npz")
    np.savez_compressed(path, **blob)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
