"""Sequence sharding of batched decode across GPUs (one process per GPU).

Decode sequences are independent: each sequence's pages, block-table row and
output live on exactly one GPU, so sharding needs no collective on the data
path.  Sequences go to ranks by LPT (longest processing time first) on their
token counts, which balances the bytes each GPU streams.
"""
from __future__ import annotations

import heapq

import numpy as np


def lpt_assign(lengths, n_ranks: int) -> list[np.ndarray]:
    """Indices of the sequences each rank owns (sorted), balanced by tokens.

    Deterministic: ties break on the lower sequence index and the lower rank."""
    if n_ranks < 1:
        raise ValueError("n_ranks must be >= 1")
    lengths = np.asarray(lengths, dtype=np.int64)
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    heap = [(0, r) for r in range(n_ranks)]
    owned: list[list[int]] = [[] for _ in range(n_ranks)]
    for i in order:
        load, r = heapq.heappop(heap)
        owned[r].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), r))
    return [np.array(sorted(o), dtype=np.int64) for o in owned]


def rank_loads(lengths, shards) -> np.ndarray:
    lengths = np.asarray(lengths, dtype=np.int64)
    return np.array([int(lengths[s].sum()) for s in shards], dtype=np.int64)
