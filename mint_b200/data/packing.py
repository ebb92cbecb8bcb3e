"""BOS best-fit packing of documents into rows (mint/data/dist/pretrain.py:218-257).

Each row of ``T + 1`` tokens is filled by repeatedly taking the longest buffered document that
fits the remaining space (the earliest-buffered one among equal lengths); when none fits, the
shortest document is cropped to the remaining space. The reference scans the whole buffer per
pick (O(buffer)); this index keeps one FIFO per length plus a sorted list of lengths, so a pick
is O(log #distinct lengths) and yields the identical sequence of picks.
"""

from __future__ import annotations

import bisect
from collections import deque


class BestFitBuffer:
    def __init__(self) -> None:
        self._by_len: dict[int, deque] = {}
        self._lengths: list[int] = []  # sorted distinct lengths present
        self._count = 0

    def __len__(self) -> int:
        return self._count

    def add(self, doc: list[int]) -> None:
        n = len(doc)
        q = self._by_len.get(n)
        if q is None:
            q = deque()
            self._by_len[n] = q
            bisect.insort(self._lengths, n)
        q.append(doc)
        self._count += 1

    def _take(self, n: int) -> list[int]:
        q = self._by_len[n]
        doc = q.popleft()
        if not q:
            del self._by_len[n]
            self._lengths.pop(bisect.bisect_left(self._lengths, n))
        self._count -= 1
        return doc

    def pop_best_fit(self, remaining: int) -> list[int] | None:
        """Longest doc with ``len <= remaining`` (len > 0), or None."""
        i = bisect.bisect_right(self._lengths, remaining) - 1
        if i < 0 or self._lengths[i] <= 0:
            return None
        return self._take(self._lengths[i])

    def pop_shortest(self) -> list[int]:
        return self._take(self._lengths[0])

    def clear(self) -> None:
        self._by_len.clear()
        self._lengths.clear()
        self._count = 0


def pack_row(buffer: BestFitBuffer, capacity: int, refill) -> tuple[list[int], list[int]]:  # noqa: ANN001
    """Fill one row; returns (tokens, doc ids). ``refill()`` tops the buffer up when it runs low."""
    toks: list[int] = []
    docs: list[int] = []
    doc_id = 0
    while len(toks) < capacity:
        refill()
        remaining = capacity - len(toks)
        doc = buffer.pop_best_fit(remaining)
        if doc is None:
            doc = buffer.pop_shortest()[:remaining]
        toks.extend(doc)
        docs.extend([doc_id] * len(doc))
        doc_id += 1
    return toks, docs
