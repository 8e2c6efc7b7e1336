"""Request sharding across the GPUs of one box.

Requests of a micro-batch are independent (no cross-request attention), so
the multi-GPU path partitions them by request with no collective on the hot
path and gathers outputs on the host. Assignment is LPT (longest processing
time first) on each request's kept (q,k) pairs -- the attention FLOPs.
"""
from __future__ import annotations

import heapq
from typing import List, Sequence

PREFIX, WINDOW, SPARSE_MAX_SEQ = 176, 432, 8192


def kept_pairs(length: int, sparse: bool, prefix: int = PREFIX, window: int = WINDOW) -> int:
    """Kept pairs of one request under the keep rule of src/webgpu/ops.ts:220."""
    if not sparse:
        return length * (length + 1) // 2
    total = 0
    # closed form per query: |[0, min(prefix, q+1))  U  (q-window, q]|
    for q in range(length):
        lo = max(0, q - window + 1)
        pre = min(prefix, q + 1)
        total += pre + (q + 1 - lo) - max(0, pre - lo)
    return total


def resolve_sparse(mode: int, lengths: Sequence[int]) -> bool:
    if mode == 1:
        return False
    if mode == 2:
        return True
    return (max(lengths) if lengths else 0) <= SPARSE_MAX_SEQ


def lpt_shard(lengths: Sequence[int], world: int, mode: int = 0) -> List[List[int]]:
    """Assign request indices to ``world`` ranks, balancing kept pairs.

    Deterministic: ties broken by request index, then rank index. Each rank's
    list is returned in ascending request order (the host gather restores the
    batch order from these indices)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    sparse = resolve_sparse(mode, lengths)
    order = sorted(range(len(lengths)), key=lambda i: (-kept_pairs(lengths[i], sparse), i))
    heap = [(0, r) for r in range(world)]
    heapq.heapify(heap)
    out: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + kept_pairs(lengths[i], sparse), r))
    return [sorted(x) for x in out]


def gather_order(assignment: List[List[int]]) -> List[int]:
    """Concatenation order of per-rank outputs -> original request order."""
    flat = [i for rank in assignment for i in rank]
    pos = {req: n for n, req in enumerate(flat)}
    return [pos[i] for i in range(len(flat))]
