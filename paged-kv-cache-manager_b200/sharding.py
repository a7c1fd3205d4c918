"""Request sharding across the GPUs of one box.

Every sequence's attention and KV mutations touch only its own blocks, so requests are partitioned across
GPUs with no collective on the data path: each GPU owns its own block pool, its own KVManager shard and its
own streams.  Requests that share blocks (a prefix parent and its children, a fork leader and its samples)
must live on the same GPU, because block ids are local to a pool.

assign_requests() balances the per-GPU bytes read per decode step (proportional to context tokens) with the
longest-processing-time-first greedy rule: groups sorted by total context, largest first, each to the
currently lightest GPU.  Ties go to the lowest rank, so the result is deterministic.
"""
from __future__ import annotations

import heapq
from typing import Dict, List, Optional, Sequence


def assign_requests(context_tokens: Sequence[int], world: int,
                    group_of: Optional[Sequence[int]] = None) -> List[int]:
    """Rank of each request.  `group_of[i]` (optional) names the sharing group of request i (requests of one
    group share blocks and go to the same rank); by default every request is its own group."""
    n = len(context_tokens)
    if world < 1:
        raise ValueError("world must be >= 1")
    groups: Dict[int, List[int]] = {}
    for i in range(n):
        g = group_of[i] if group_of is not None else i
        groups.setdefault(g, []).append(i)
    order = sorted(groups.items(), key=lambda kv: (-sum(context_tokens[i] for i in kv[1]), kv[0]))
    heap = [(0, r) for r in range(world)]
    rank = [0] * n
    for _, members in order:
        load, r = heapq.heappop(heap)
        for i in members:
            rank[i] = r
        heapq.heappush(heap, (load + sum(context_tokens[i] for i in members), r))
    return rank


def shard_of(rank_of: Sequence[int], rank: int) -> List[int]:
    """Indices of the requests assigned to `rank`, in their original order."""
    return [i for i, r in enumerate(rank_of) if r == rank]


def imbalance(context_tokens: Sequence[int], rank_of: Sequence[int], world: int) -> float:
    """max rank load / mean rank load (1.0 = perfect balance)."""
    loads = [0] * world
    for t, r in zip(context_tokens, rank_of):
        loads[r] += t
    mean = sum(loads) / world
    return max(loads) / mean if mean else 1.0
