"""Cross-layer expert co-activation table and the prefetch predictor.

Host-side logic of the reference's speculative prefetch (off by default
there too): src/wisp/oracle/cooccur.py:44-236 (``CooccurTable``) and
:228-292 (``predict_layer``), driven by the paged forward's post-forward
block (src/wisp/integrations/vllm/fused_moe.py:1170-1233).

* ``observe_step({layer: experts})`` counts, for one decode step, every
  cross-layer pair ``(L_src, e_src) -> (L_dst, e_dst)`` with ``L_dst > L_src``
  (once per step) and the marginal ``(L, e)``.
* ``predict_layer(table, seen, target)`` scores every expert of the target
  layer by ``sum over conditioning (L_src, e_src)`` of
  ``decay ** (target - L_src - 1) * count / marginal`` and returns the top
  ``k`` by (score descending, id ascending).

The table is serialised in the reference's JSON schema (version 1:
``pairs = [L_src, e_src, L_dst, e_dst, n]``, ``marginals = [L, e, n]``,
optionally gzipped) so a warm table recorded for the reference loads here
unchanged.  The arithmetic order of the scores matches the reference's
(sources in the order they were observed, destinations in first-seen
order), so the ranking -- ties included -- is the same.
"""
from __future__ import annotations

import gzip
import json
import os
from typing import Iterable, Mapping

SCHEMA_VERSION = 1


class CooccurTable:
    """Per-layer-pair expert co-activation counts.

    ``count[(L_src, e_src)][L_dst][e_dst]`` = steps in which both fired;
    ``layer_total[(L, e)]`` = steps in which ``e`` fired at ``L``."""

    def __init__(self) -> None:
        self.count: dict[tuple[int, int], dict[int, dict[int, int]]] = {}
        self.layer_total: dict[tuple[int, int], int] = {}
        self.num_steps_observed = 0

    def observe_step(self, expert_ids_by_layer: Mapping[int, Iterable[int]]) -> None:
        layers = [(int(L), [int(e) for e in es]) for L, es in expert_ids_by_layer.items()]
        layers = [(L, es) for L, es in layers if es]
        for L, es in layers:
            for e in es:
                self.layer_total[(L, e)] = self.layer_total.get((L, e), 0) + 1
        for L_src, src in layers:
            for e_src in src:
                per_dst = self.count.setdefault((L_src, e_src), {})
                for L_dst, dst in layers:
                    if L_dst <= L_src:
                        continue
                    row = per_dst.setdefault(L_dst, {})
                    for e_dst in dst:
                        row[e_dst] = row.get(e_dst, 0) + 1
        self.num_steps_observed += 1

    @property
    def n_source_keys(self) -> int:
        return len(self.count)

    @property
    def n_pairs(self) -> int:
        return sum(len(row) for per in self.count.values() for row in per.values())

    # ---- serialisation (the reference's schema) ---------------------------------
    def to_dict(self) -> dict:
        pairs = [[L_src, e_src, L_dst, e_dst, n]
                 for (L_src, e_src), per in self.count.items()
                 for L_dst, row in per.items() for e_dst, n in row.items() if n > 0]
        marg = [[L, e, n] for (L, e), n in self.layer_total.items() if n > 0]
        return {"schema_version": SCHEMA_VERSION, "num_steps_observed": self.num_steps_observed,
                "pairs": pairs, "marginals": marg,
                "stats": {"n_source_keys": self.n_source_keys, "n_pairs": self.n_pairs,
                          "memory_estimate_bytes": 40 * self.n_pairs}}

    @classmethod
    def from_dict(cls, data: Mapping) -> "CooccurTable":
        if int(data.get("schema_version", 1)) != SCHEMA_VERSION:
            raise ValueError(f"cooccur table schema_version {data.get('schema_version')} unsupported")
        t = cls()
        for L_src, e_src, L_dst, e_dst, n in data.get("pairs") or []:
            t.count.setdefault((int(L_src), int(e_src)), {}).setdefault(int(L_dst), {})[int(e_dst)] = int(n)
        for L, e, n in data.get("marginals") or []:
            t.layer_total[(int(L), int(e))] = int(n)
        t.num_steps_observed = int(data.get("num_steps_observed", 0))
        return t

    def save(self, path) -> None:
        path = os.fspath(path)
        os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
        text = json.dumps(self.to_dict(), separators=(",", ":"))
        opener = gzip.open if path.endswith(".gz") else open
        with opener(path, "wt", encoding="utf-8") as f:
            f.write(text)

    @classmethod
    def load(cls, path) -> "CooccurTable":
        path = os.fspath(path)
        opener = gzip.open if path.endswith(".gz") else open
        with opener(path, "rt", encoding="utf-8") as f:
            return cls.from_dict(json.load(f))


def predict_layer(table: CooccurTable, seen_so_far: Mapping[int, Iterable[int]], target_layer: int, *,
                  k: int = 8, normalize: bool = True, decay: float = 1.0,
                  only_prev_layer: bool = False) -> list[int]:
    """Top-``k`` expert ids for ``target_layer`` given the experts seen at
    earlier layers of the current step; ``[]`` when nothing conditions."""
    scores: dict[int, float] = {}
    for L_src, src in seen_so_far.items():
        if L_src >= target_layer or (only_prev_layer and L_src != target_layer - 1):
            continue
        w = decay ** (target_layer - L_src - 1)
        for e_src in src:
            row = table.count.get((L_src, e_src), {}).get(target_layer)
            if not row:
                continue
            total = table.layer_total.get((L_src, e_src), 0) if normalize else 1
            denom = total if normalize and total > 0 else 1
            for e_dst, c in row.items():
                scores[e_dst] = scores.get(e_dst, 0.0) + w * c / denom
    if not scores:
        return []
    return [e for e, _ in sorted(scores.items(), key=lambda kv: (-kv[1], kv[0]))[:k]]


__all__ = ["CooccurTable", "predict_layer", "SCHEMA_VERSION"]
