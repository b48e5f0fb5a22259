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


def _csr(layers_map: Mapping[int, Iterable[int]]):
    """{layer: experts} in its own order as ctypes CSR arrays (layers, offsets, experts)."""
    import ctypes
    ls, offs, es = [], [0], []
    for L, xs in layers_map.items():
        ls.append(int(L))
        es.extend(int(e) for e in xs)
        offs.append(len(es))
    n = len(ls)
    return (n, (ctypes.c_int32 * max(n, 1))(*ls), (ctypes.c_int32 * (n + 1))(*offs),
            (ctypes.c_int32 * max(len(es), 1))(*es))


class NativeCooccurTable:
    """The same table in the library's host C++ (``wisp_cooccur_*``): the same
    counts, serialisation order and scores as :class:`CooccurTable`, so the
    same rankings, at native speed (the prediction walks every earlier layer's
    experts once per layer of a decode step)."""

    def __init__(self) -> None:
        import ctypes
        from wisp_b200 import _lib
        self._lib = _lib
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().wisp_cooccur_create(ctypes.byref(h)), "wisp_cooccur_create")
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                self._lib.lib().wisp_cooccur_destroy(h)
            except Exception:  # interpreter shutdown: the library may be gone already
                pass
            self._h = None

    def observe_step(self, expert_ids_by_layer: Mapping[int, Iterable[int]]) -> None:
        n, ls, offs, es = _csr(expert_ids_by_layer)
        self._lib.check(self._lib.lib().wisp_cooccur_observe_step(self._h, n, ls, offs, es),
                        "wisp_cooccur_observe_step")

    def predict(self, seen_so_far: Mapping[int, Iterable[int]], target_layer: int, *, k: int = 8,
                normalize: bool = True, decay: float = 1.0, only_prev_layer: bool = False) -> list[int]:
        import ctypes
        n, ls, offs, es = _csr(seen_so_far)
        out = (ctypes.c_int32 * max(int(k), 1))()
        m = ctypes.c_int32(0)
        self._lib.check(self._lib.lib().wisp_cooccur_predict(
            self._h, n, ls, offs, es, int(target_layer), int(k), int(bool(normalize)), float(decay),
            int(bool(only_prev_layer)), out, ctypes.byref(m)), "wisp_cooccur_predict")
        return list(out[:m.value])

    def _sizes(self):
        import ctypes
        v = [ctypes.c_int64(0) for _ in range(4)]
        self._lib.check(self._lib.lib().wisp_cooccur_sizes(self._h, *[ctypes.byref(x) for x in v]),
                        "wisp_cooccur_sizes")
        return [x.value for x in v]

    @property
    def n_source_keys(self) -> int:
        return self._sizes()[0]

    @property
    def n_pairs(self) -> int:
        return self._sizes()[1]

    @property
    def num_steps_observed(self) -> int:
        return self._sizes()[3]

    def to_dict(self) -> dict:
        import ctypes
        n_src, n_pairs, n_marg, steps = self._sizes()
        pairs = (ctypes.c_int64 * max(5 * n_pairs, 1))()
        marg = (ctypes.c_int64 * max(3 * n_marg, 1))()
        npo, nmo = ctypes.c_int64(0), ctypes.c_int64(0)
        self._lib.check(self._lib.lib().wisp_cooccur_export(self._h, pairs, n_pairs, ctypes.byref(npo), marg,
                                                             n_marg, ctypes.byref(nmo)), "wisp_cooccur_export")
        P = [list(pairs[5 * i:5 * i + 5]) for i in range(npo.value)]
        M = [list(marg[3 * i:3 * i + 3]) for i in range(nmo.value)]
        return {"schema_version": SCHEMA_VERSION, "num_steps_observed": steps, "pairs": P, "marginals": M,
                "stats": {"n_source_keys": n_src, "n_pairs": n_pairs, "memory_estimate_bytes": 40 * n_pairs}}

    @classmethod
    def from_dict(cls, data: Mapping) -> "NativeCooccurTable":
        if int(data.get("schema_version", 1)) != SCHEMA_VERSION:
            raise ValueError(f"cooccur table schema_version {data.get('schema_version')} unsupported")
        t = cls()
        L = t._lib.lib()
        for L_src, e_src, L_dst, e_dst, n in data.get("pairs") or []:
            t._lib.check(L.wisp_cooccur_set_pair(t._h, int(L_src), int(e_src), int(L_dst), int(e_dst), int(n)),
                         "wisp_cooccur_set_pair")
        for Lm, e, n in data.get("marginals") or []:
            t._lib.check(L.wisp_cooccur_set_marginal(t._h, int(Lm), int(e), int(n)), "wisp_cooccur_set_marginal")
        t._lib.check(L.wisp_cooccur_set_steps(t._h, int(data.get("num_steps_observed", 0))),
                     "wisp_cooccur_set_steps")
        return t

    def save(self, path) -> None:
        CooccurTable.from_dict(self.to_dict()).save(path)

    @classmethod
    def load(cls, path) -> "NativeCooccurTable":
        return cls.from_dict(CooccurTable.load(path).to_dict())


def predict_layer(table, seen_so_far: Mapping[int, Iterable[int]], target_layer: int, *,
                  k: int = 8, normalize: bool = True, decay: float = 1.0,
                  only_prev_layer: bool = False) -> list[int]:
    """Top-``k`` expert ids for ``target_layer`` given the experts seen at
    earlier layers of the current step; ``[]`` when nothing conditions."""
    if isinstance(table, NativeCooccurTable):
        return table.predict(seen_so_far, target_layer, k=k, normalize=normalize, decay=decay,
                             only_prev_layer=only_prev_layer)
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


__all__ = ["CooccurTable", "NativeCooccurTable", "predict_layer", "SCHEMA_VERSION"]
