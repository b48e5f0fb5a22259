"""Iteration order of a CPython ``set`` of small non-negative ints.

TEST INFRASTRUCTURE ONLY: this module is part of the CPU oracle. Only the
tests, ``__graft_entry__.smoke()`` and ``bench.py``'s reference arm may use it.

Why it exists: the reference pager walks ``needed_set`` (a Python ``set``
built from the ascending output of ``torch.unique``) to produce its
``missing`` list, and then hands out slots with a LIFO ``pop()``
(src/wisp/integrations/vllm/fused_moe.py:279-283 and :346-347).  Slot
placement therefore depends on the interpreter's hash-table order.  The
device pager reproduces that order with the model below; this Python copy
is the readable statement of it and is checked exhaustively against the
interpreter in ``tests/test_setorder.py``.

Model (CPython 3.x ``set`` behaviour for keys whose hash equals the key):
  * the table starts with 8 entries; ``mask = size - 1``;
  * a key starts at index ``h & mask``; if that entry is taken it tries the
    next 9 entries in a row (only when ``i + 9 <= mask``), then jumps to
    ``(5*i + 1 + perturb) & mask`` with ``perturb`` (initially ``h``)
    shifted right by 5 before each jump, and repeats;
  * after an insert, when ``5*fill >= 3*mask`` the table is rebuilt with the
    smallest power of two (>= 8) that is larger than ``4*used``; the old
    entries are re-inserted in old-table index order;
  * iteration walks the table in index order.
"""
from __future__ import annotations

LINEAR_RUN = 9
PERTURB_SHIFT = 5
MIN_SIZE = 8


def _place(table: list, mask: int, key: int) -> None:
    i = key & mask
    perturb = key
    while True:
        run = LINEAR_RUN if i + LINEAR_RUN <= mask else 0
        j = i
        for _ in range(run + 1):
            if table[j] is None:
                table[j] = key
                return
            j += 1
        perturb >>= PERTURB_SHIFT
        i = (i * 5 + 1 + perturb) & mask


def table_size_for(used: int) -> int:
    size = MIN_SIZE
    while size <= used * 4:
        size <<= 1
    return size


def set_order(keys_in_insert_order) -> list[int]:
    """Return ``list(set(keys))`` as CPython would, for distinct ints >= 0
    inserted one at a time in the given order."""
    table: list = [None] * MIN_SIZE
    mask = MIN_SIZE - 1
    used = 0
    for k in keys_in_insert_order:
        _place(table, mask, int(k))
        used += 1
        if used * 5 >= mask * 3:
            new_size = table_size_for(used)
            old = [e for e in table if e is not None]
            table = [None] * new_size
            mask = new_size - 1
            for e in old:
                _place(table, mask, e)
    return [e for e in table if e is not None]
