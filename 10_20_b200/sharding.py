"""Request sharding across GPUs for the query path.

Requests are independent (one query row each, with its own pages), so N GPUs
split a batch by request and run with no data-path collective.  The cost of a
request is its compulsory HBM traffic (`row_bytes`), which grows with the
context length; a longest-processing-time assignment with a per-GPU request
count keeps every GPU's batch the same size (weak scaling) while balancing the
bytes each one streams.
"""
from __future__ import annotations

import heapq


def row_bytes(n: int, heads: int, take: int, window: int, topk: int, latent_row_bytes: int = 0,
              outputs: int = 1, staging: bool = True) -> dict:
    """Compulsory bytes of one request of token length n (each input byte once,
    each output byte once): q/w, centre keys (132 B per centre, 8 per built
    page), sink/tail staging (read + write; only for the operator sequence that
    copies those keys into the fine pool -- the fused selection scores them in
    place, `staging=False`), fine keys (selected pages and the sink/tail
    tokens) + members of the selected pages, the three int32 Top-k outputs and
    the latent gather (read once, written `outputs` times)."""
    pages = max(n - 1, 0) // 1024 * 16
    tk = min(pages, take)
    sink = min(64, n)
    tail = max(sink, min(max(n - 1, 0) // 1024 * 1024, max(sink, n - window)))
    count = sink + n - tail
    q = heads * (128 + 4)
    centres = pages * 8 * 132
    staging = count * 132 * 2 if staging else 0
    fine = (tk * 64 + count) * 132 + tk * 64 * 4
    out = topk * 4 * 3
    gather = topk * latent_row_bytes * (1 + outputs) if latent_row_bytes else 0
    return dict(q=q, centres=centres, staging=staging, fine=fine, topk_out=out, gather=gather,
                total=q + centres + staging + fine + out + gather)


def shard_requests(costs, world: int, per_rank: int | None = None):
    """Assign request indices to `world` ranks, heaviest first, each to the least
    loaded rank that still has room (`per_rank` requests each if given, which
    requires len(costs) == world * per_rank).  Deterministic: every rank computes
    the same assignment.  Returns one ascending index list per rank."""
    n = len(costs)
    if world < 1:
        raise ValueError("world must be >= 1")
    if per_rank is not None and n != world * per_rank:
        raise ValueError(f"{n} requests cannot fill {world} ranks of {per_rank}")
    cap = per_rank if per_rank is not None else n
    order = sorted(range(n), key=lambda i: (-costs[i], i))
    heap = [(0, r) for r in range(world)]
    shards = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        if len(shards[r]) < cap:       # a full rank leaves the heap
            heapq.heappush(heap, (load + costs[i], r))
    return [sorted(s) for s in shards]
