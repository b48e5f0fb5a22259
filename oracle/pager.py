"""Restatement of the reference's paged-MoE bookkeeping (CPU oracle).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Follows, in order of the reference source:
  * ``WispMoEState.__init__`` state: src/wisp/integrations/vllm/fused_moe.py:161-236
  * ``ensure_resident``:               fused_moe.py:264-358
  * ``prime_identity``:                fused_moe.py:242-258
  * ``resize_cap``:                    fused_moe.py:439-490
  * ``prefetch_async``:                fused_moe.py:360-433
  * first-fit token sub-batching and the per-forward call sequence of
    ``_wisp_forward_cuda_paged``:      fused_moe.py:1017, 1102-1168

The needed set is a real Python ``set`` built from the ascending unique ids,
exactly as the reference builds it, so its iteration order is the
interpreter's (the device pager reproduces it with ``oracle.setorder``).
Pinned by ``tests/test_oracle_golden.py`` against traces recorded by running
the reference's own ``WispMoEState`` and forward on CPU.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

OVERFLOW_MSG = ("per-kernel-call working set ({n} unique experts) exceeds cap_experts "
                "({cap}); the forward path failed to sub-batch correctly")


class PagerOverflow(RuntimeError):
    """Raised when one call's unique experts cannot fit (fused_moe.py:313-327)."""


@dataclass
class StepRecord:
    needed: list            # needed set, interpreter iteration order
    missing: list           # missing experts, in that order
    victims: list           # evicted (slot, expert), in eviction order
    placed: list            # (expert, slot) for each miss, in order


@dataclass
class PagerOracle:
    num_experts: int
    cap: int
    slot_to_expert: list = field(default_factory=list)
    expert_to_slot: dict = field(default_factory=dict)
    lru_tick: list = field(default_factory=list)
    lru_clock: int = 0
    stats_forward: int = 0
    stats_miss: int = 0
    stats_evict: int = 0
    stats_hits: int = 0

    def __post_init__(self):
        if not self.slot_to_expert:
            self.slot_to_expert = [-1] * self.cap
            self.lru_tick = [0] * self.cap

    # fused_moe.py:264-358
    def ensure_resident(self, needed_ids) -> StepRecord:
        needed = sorted({int(e) for e in np.asarray(needed_ids).reshape(-1).tolist()})
        needed_set = set(int(e) for e in needed)
        missing = [e for e in needed_set if e not in self.expert_to_slot]
        self.stats_hits += len(needed_set) - len(missing)
        rec = StepRecord(list(needed_set), list(missing), [], [])
        if not missing:
            self.lru_clock += 1
            for e in needed_set:
                self.lru_tick[self.expert_to_slot[e]] = self.lru_clock
            return rec
        free_slots = [s for s in range(self.cap) if self.slot_to_expert[s] == -1]
        cands = sorted(((self.lru_tick[s], s) for s in range(self.cap)
                        if self.slot_to_expert[s] != -1
                        and self.slot_to_expert[s] not in needed_set),
                       key=lambda x: x[0])
        need_slot = len(missing) - len(free_slots)
        if need_slot > 0:
            if need_slot > len(cands):
                raise PagerOverflow(OVERFLOW_MSG.format(n=len(needed_set), cap=self.cap))
            for _tick, s in cands[:need_slot]:
                ev = self.slot_to_expert[s]
                self.expert_to_slot.pop(ev, None)
                self.slot_to_expert[s] = -1
                free_slots.append(s)
                self.stats_evict += 1
                rec.victims.append((s, ev))
        self.lru_clock += 1
        for e in missing:
            slot = free_slots.pop()
            self.slot_to_expert[slot] = e
            self.expert_to_slot[e] = slot
            self.lru_tick[slot] = self.lru_clock
            self.stats_miss += 1
            rec.placed.append((e, slot))
        for e in needed_set:
            self.lru_tick[self.expert_to_slot[e]] = self.lru_clock
        return rec

    # fused_moe.py:360-433
    def prefetch_async(self, predicted, last_unique) -> StepRecord:
        """Speculative load of ``predicted`` (an iterable in the order the
        reference iterates its set) with the history bias: slots holding an
        expert of ``last_unique`` or of the prediction are not victims; a
        prediction larger than the free slots plus the victims is cut short;
        the clock moves only when something loads; evictions count, misses
        do not."""
        predicted = list(predicted)
        pred_set = set(predicted)
        last = set(last_unique)
        rec = StepRecord(predicted, [], [], [])
        to_load = [e for e in predicted if e not in self.expert_to_slot]
        if not to_load:
            return rec
        free_slots = [s for s in range(self.cap) if self.slot_to_expert[s] == -1]
        cands = sorted(((self.lru_tick[s], s) for s in range(self.cap)
                        if self.slot_to_expert[s] != -1
                        and self.slot_to_expert[s] not in last
                        and self.slot_to_expert[s] not in pred_set),
                       key=lambda x: x[0])
        need_slot = len(to_load) - len(free_slots)
        if need_slot > 0:
            if need_slot > len(cands):
                to_load = to_load[: len(cands) + len(free_slots)]
                need_slot = len(to_load) - len(free_slots)
            for _tick, s in cands[:need_slot]:
                ev = self.slot_to_expert[s]
                self.expert_to_slot.pop(ev, None)
                self.slot_to_expert[s] = -1
                free_slots.append(s)
                self.stats_evict += 1
                rec.victims.append((s, ev))
        self.lru_clock += 1
        for e in to_load:
            if not free_slots:
                break
            slot = free_slots.pop()
            self.slot_to_expert[slot] = int(e)
            self.expert_to_slot[int(e)] = slot
            self.lru_tick[slot] = self.lru_clock
            rec.placed.append((int(e), slot))
        rec.missing = [e for e, _ in rec.placed]
        return rec

    # fused_moe.py:242-258
    def prime_identity(self) -> None:
        assert self.cap == self.num_experts
        for i in range(self.num_experts):
            self.slot_to_expert[i] = i
            self.expert_to_slot[i] = i

    # fused_moe.py:439-490
    def resize_cap(self, new_cap: int) -> None:
        new_cap = max(2, min(int(new_cap), self.num_experts))
        if new_cap == self.cap:
            return
        if new_cap < self.cap:
            for s in range(new_cap, self.cap):
                e = self.slot_to_expert[s]
                if e != -1:
                    self.expert_to_slot.pop(e, None)
            del self.slot_to_expert[new_cap:]
            del self.lru_tick[new_cap:]
        else:
            self.slot_to_expert.extend([-1] * (new_cap - self.cap))
            self.lru_tick.extend([0] * (new_cap - self.cap))
        self.cap = new_cap

    def expert_map(self) -> np.ndarray:
        m = np.full(self.num_experts, -1, np.int32)
        for e, s in self.expert_to_slot.items():
            m[e] = s
        return m

    def stats(self) -> list:
        return [self.stats_forward, self.stats_miss, self.stats_hits, self.stats_evict]


def first_fit_groups(topk_ids, cap: int) -> list:
    """Token groups of the paged forward as ``[t0, t1)`` ranges.

    fused_moe.py:1102-1140: the whole batch is one call when its unique
    experts fit the cap; otherwise tokens join the current group, in index
    order, while the union stays within the cap or the group is empty.  (The
    fast path is the first-fit result when the union fits, so one loop
    covers both.)"""
    ids = np.asarray(topk_ids).reshape(len(topk_ids), -1)
    groups, start, cur = [], 0, set()
    for t in range(ids.shape[0]):
        tok = {int(e) for e in ids[t].tolist()}
        merged = cur | tok
        if len(merged) <= cap or t == start:
            cur = merged
        else:
            groups.append((start, t))
            start, cur = t, tok
    if ids.shape[0] > start:
        groups.append((start, ids.shape[0]))
    return groups


def forward_pager(p: PagerOracle, topk_ids):
    """Pager side of one paged forward (fused_moe.py:1017, 1102-1168).

    Returns ``(groups, slots, records)``: the token groups, the slot each
    ``(t, k)`` reads after its group's ``ensure_resident`` (``[T, k]`` int32),
    and the per-group step records."""
    ids = np.asarray(topk_ids).reshape(len(topk_ids), -1)
    p.stats_forward += 1
    groups = first_fit_groups(ids, p.cap)
    slots = np.full(ids.shape, -1, np.int32)
    recs = []
    for t0, t1 in groups:
        recs.append(p.ensure_resident(ids[t0:t1]))
        for t in range(t0, t1):
            for j in range(ids.shape[1]):
                slots[t, j] = p.expert_to_slot[int(ids[t, j])]
    return groups, slots, recs
