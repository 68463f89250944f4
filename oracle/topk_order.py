"""CPU ORACLE — test infrastructure, never the product: the tie order of ``torch.topk`` on the CPU.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may import this module.

The reference's router is the ``transformers`` block it builds
(``tarfa/engine/channel.py:19-30``).  It selects experts with
``torch.topk(softmax_fp32(logits), 8)`` (``transformers`` 5.5.0,
``models/qwen3_5_moe/modeling_qwen3_5_moe.py:767``).  When probabilities tie at
or inside the top-k, which ids ``torch.topk`` returns, and in which order, is a
property of its CPU implementation.  This module restates that implementation.

PyTorch 2.11.0's CPU top-k (``aten/src/ATen/native/TopKImpl.h``,
``topk_impl_loop``) fills a vector of ``(value, index)`` pairs for each row.
Then, with ``comp(x, y) = x.value > y.value`` (``largest=True``, NaN first):

* if ``k * 64 <= n``: ``std::partial_sort(first, first + k, last, comp)``;
* else: ``std::nth_element(first, first + k - 1, last, comp)``, then
  ``std::sort(first, first + k - 1, comp)``.

The comparator looks at values only, so equal values come out in whatever
order the standard-library algorithms leave them.  Those algorithms are
libstdc++'s from GCC 13.3, the compiler torch 2.11.0 was built with
(``torch.__config__.show()``).  They are the textbook ones:

* ``nth_element``: introselect.  A median-of-three pivot taken from
  ``first + 1``, the middle and ``last - 1`` is swapped into ``first``.  A
  Hoare partition then runs with unguarded scans.  After ``2 * floor(log2 n)``
  partitions the search falls back to heap select.  A range of 3 or fewer
  elements gets an insertion sort.
* ``sort``: introsort with the same partition, stopping at ranges of 16 or
  fewer, then an insertion sort.  For ``k <= 17`` the ``k - 1`` elements are
  sorted by insertion alone, which is stable.
* ``partial_sort``: heap select (a heap of the first ``k`` under ``comp``, each
  later element that beats the heap top replaces it), then heap sort.

The restatement is pinned against ``torch.topk`` itself by
``tests/test_topk_order.py``.  That test uses random tie-heavy rows, structured
orders, and adversarial rows that exhaust the introselect depth limit.
``adversarial_row`` builds those last ones with McIlroy's lazy-comparator
method ("A Killer Adversary for Quicksort", 1999).
"""
from __future__ import annotations

import math

import numpy as np


class _Row:
    """One row under selection: parallel lists of keys and expert ids.

    ``gt(a, b)`` is the comparator on keys ("a ranks before b"); the default
    compares numbers, NaN first (``TopKImpl.h``'s ``largest`` comparator).
    """

    def __init__(self, keys, gt=None):
        self.key = list(keys)
        self.ids = list(range(len(self.key)))
        self.gt = gt or _gt_number

    # -- element moves ----------------------------------------------------
    def _before(self, p: int, q: int) -> bool:
        return self.gt(self.key[p], self.key[q])

    def _swap(self, p: int, q: int):
        k, i = self.key, self.ids
        k[p], k[q] = k[q], k[p]
        i[p], i[q] = i[q], i[p]

    def _take(self, p: int):
        return self.key[p], self.ids[p]

    def _put(self, p: int, item):
        self.key[p], self.ids[p] = item

    # -- pivot and partition -----------------------------------------------
    def _pivot_to_front(self, front: int, a: int, b: int, c: int):
        """Swap the median of positions a, b, c into ``front`` (the comparison
        sequence decides which of equal keys is taken)."""
        if self._before(a, b):
            pick = b if self._before(b, c) else (c if self._before(a, c) else a)
        elif self._before(a, c):
            pick = a
        elif self._before(b, c):
            pick = c
        else:
            pick = b
        self._swap(front, pick)

    def _hoare(self, lo: int, hi: int, piv: int) -> int:
        """Unguarded Hoare partition of [lo, hi) around the key at ``piv``;
        returns the first position of the right part."""
        while True:
            while self._before(lo, piv):
                lo += 1
            hi -= 1
            while self._before(piv, hi):
                hi -= 1
            if lo >= hi:
                return lo
            self._swap(lo, hi)
            lo += 1

    def _split(self, lo: int, hi: int) -> int:
        self._pivot_to_front(lo, lo + 1, lo + (hi - lo) // 2, hi - 1)
        return self._hoare(lo + 1, hi, lo)

    # -- insertion sort ------------------------------------------------------
    def _insertion(self, lo: int, hi: int):
        """Insertion sort of [lo, hi): an element that ranks before the first
        one moves to the front in one shift; the others walk left."""
        for p in range(lo + 1, hi):
            item = self._take(p)
            if self.gt(item[0], self.key[lo]):
                for q in range(p, lo, -1):
                    self._put(q, self._take(q - 1))
                self._put(lo, item)
            else:
                self._walk_left(p, item)

    def _walk_left(self, p: int, item):
        """Shift ``item`` left from ``p`` past every element it ranks before
        (unguarded: something to its left stops it)."""
        q = p
        while self.gt(item[0], self.key[q - 1]):
            self._put(q, self._take(q - 1))
            q -= 1
        self._put(q, item)

    # -- heaps (the top is the element every other one ranks before) ----------
    def _sift(self, base: int, hole: int, n: int, item):
        top = hole
        child = hole
        while child < (n - 1) // 2:
            child = 2 * (child + 1)
            if self._before(base + child, base + child - 1):
                child -= 1
            self._put(base + hole, self._take(base + child))
            hole = child
        if n % 2 == 0 and child == (n - 2) // 2:
            child = 2 * (child + 1)
            self._put(base + hole, self._take(base + child - 1))
            hole = child - 1
        parent = (hole - 1) // 2
        while hole > top and self.gt(self.key[base + parent], item[0]):
            self._put(base + hole, self._take(base + parent))
            hole = parent
            parent = (hole - 1) // 2
        self._put(base + hole, item)

    def _heapify(self, lo: int, hi: int):
        n = hi - lo
        if n < 2:
            return
        for parent in range((n - 2) // 2, -1, -1):
            self._sift(lo, parent, n, self._take(lo + parent))

    def _pop_into(self, lo: int, hi: int, dst: int):
        item = self._take(dst)
        self._put(dst, self._take(lo))
        self._sift(lo, 0, hi - lo, item)

    def _heap_select(self, lo: int, mid: int, hi: int):
        self._heapify(lo, mid)
        for p in range(mid, hi):
            if self._before(p, lo):
                self._pop_into(lo, mid, p)

    def _heap_sort(self, lo: int, hi: int):
        while hi - lo > 1:
            hi -= 1
            self._pop_into(lo, hi, hi)

    # -- the three algorithms -----------------------------------------------
    def nth_element(self, nth: int, lo: int = 0, hi: int | None = None):
        hi = len(self.key) if hi is None else hi
        if lo == hi or nth == hi:
            return
        budget = 2 * int(math.floor(math.log2(hi - lo)))
        while hi - lo > 3:
            if budget == 0:
                self._heap_select(lo, nth + 1, hi)
                self._swap(lo, nth)
                return
            budget -= 1
            cut = self._split(lo, hi)
            if cut <= nth:
                lo = cut
            else:
                hi = cut
        self._insertion(lo, hi)

    def sort(self, lo: int, hi: int):
        if hi - lo < 2:
            return
        self._introsort(lo, hi, 2 * int(math.floor(math.log2(hi - lo))))
        if hi - lo > 16:
            self._insertion(lo, lo + 16)
            for p in range(lo + 16, hi):
                self._walk_left(p, self._take(p))
        else:
            self._insertion(lo, hi)

    def _introsort(self, lo: int, hi: int, budget: int):
        while hi - lo > 16:
            if budget == 0:
                self._heap_select(lo, hi, hi)
                self._heap_sort(lo, hi)
                return
            budget -= 1
            cut = self._split(lo, hi)
            self._introsort(cut, hi, budget)
            hi = cut

    def partial_sort(self, mid: int):
        self._heap_select(0, mid, len(self.key))
        self._heap_sort(0, mid)


def _gt_number(a, b) -> bool:
    an, bn = a != a, b != b
    return (an and not bn) or a > b


def topk_ids(keys, k: int) -> list[int]:
    """Ids ``torch.topk(keys, k)`` returns on the CPU (largest, sorted)."""
    n = len(keys)
    k = min(k, n)
    if k == 0:
        return []
    row = _Row(keys)
    if k * 64 <= n:
        row.partial_sort(k)
    else:
        row.nth_element(k - 1)
        row.sort(0, k - 1)
    return row.ids[:k]


def topk_rows(keys: np.ndarray, k: int) -> np.ndarray:
    """``topk_ids`` for every row of a ``[T, n]`` array (int64 ``[T, k]``).

    A row whose top ``k + 1`` keys are all distinct has one possible answer, the
    top ``k`` by key; only rows with an equality there run the restatement.
    """
    keys = np.asarray(keys)
    T, n = keys.shape
    k = min(k, n)
    order = np.argsort(-keys, axis=-1, kind="stable")
    out = order[:, :k].astype(np.int64).copy()
    m = min(k + 1, n)
    srt = np.take_along_axis(keys, order[:, :m], axis=-1)
    tied = (srt[:, 1:] == srt[:, :-1]).any(axis=-1) | np.isnan(srt).any(axis=-1)
    for t in np.nonzero(tied)[0]:
        out[t] = topk_ids(keys[t].tolist(), k)
    return out


def adversarial_row(n: int, k: int) -> list[int]:
    """Integer keys on which introselect (for ``k``) uses its whole partition
    budget, built with McIlroy's lazy comparator: items start as "gas" (above
    every frozen value); when two gas items meet, one is frozen to the next
    value up, preferring the current pivot candidate.  Gas left at the end
    takes one value above all frozen ones (a block of ties at the top)."""
    gas = object()
    val = [gas] * n
    nxt = [0]
    cand = [-1]

    def freeze(x):
        val[x] = nxt[0]
        nxt[0] += 1

    def gt(x, y):
        if val[x] is gas and val[y] is gas:
            freeze(x if x == cand[0] else y)
        if val[x] is gas:
            cand[0] = x
            return True
        if val[y] is gas:
            cand[0] = y
            return False
        return val[x] > val[y]

    row = _Row(range(n), gt)          # keys are item numbers, compared lazily
    row.nth_element(k - 1)
    top = nxt[0]
    return [top if v is gas else v for v in val]
