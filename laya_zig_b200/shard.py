"""Sharding independent decisions over ranks (one process per GPU).

Decisions never interact, so the model is replicated and the work is split
without any collective on the data path: the decisions are packed into
length-sorted buckets of at most `max_tokens` tokens (synth.bucket), and the
buckets go to ranks longest-processing-time first, with the cost of a bucket
estimated from its projection and attention FLOPs. Results come back to the
host per rank.
"""
from __future__ import annotations

import heapq
from typing import List, Sequence

GEMM_FLOPS_PER_TOKEN = 2 * 124_452_864


def attention_flops(L: int) -> float:
    """4 * 768 * (10 L^2 + 14 S(L)): 8 global encoder layers + 2 head layers
    over all keys, 14 sliding layers over |i - j| <= 64."""
    s = sum(min(L, i + 65) - max(0, i - 64) for i in range(L))
    return 4.0 * 768 * (10 * L * L + 14 * s)


def bucket_cost(lengths: Sequence[int]) -> float:
    return sum(GEMM_FLOPS_PER_TOKEN * L + attention_flops(L) for L in lengths)


def lpt_assign(costs: Sequence[float], world: int) -> List[List[int]]:
    """Bucket indices per rank, longest first onto the least-loaded rank.
    Ties go to the lowest rank, so every rank computes the same answer."""
    heap = [(0.0, r) for r in range(world)]
    out: List[List[int]] = [[] for _ in range(world)]
    for b in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        load, r = heapq.heappop(heap)
        out[r].append(b)
        heapq.heappush(heap, (load + costs[b], r))
    return out


def gather(local: dict, n_total: int, group=None):
    """Host-side gather of {decision index: result} from every rank (a
    torch.distributed object gather; no device data moves). Returns the list
    in decision order on every rank; raises if an index is missing or twice."""
    import torch.distributed as dist
    parts = [None] * dist.get_world_size(group)
    dist.all_gather_object(parts, local, group=group)
    merged = {}
    for p in parts:
        for k, v in p.items():
            if k in merged:
                raise RuntimeError("decision %d computed by two ranks" % k)
            merged[k] = v
    if len(merged) != n_total:
        raise RuntimeError("%d of %d decisions came back" % (len(merged), n_total))
    return [merged[i] for i in range(n_total)]


def shard(decisions, world: int, rank: int, max_tokens: int = 32768):
    """(this rank's buckets as lists of decision indices, every rank's load)."""
    from .synth import bucket
    buckets = bucket(decisions, max_tokens)
    costs = [bucket_cost([len(decisions[i].ids) for i in b]) for b in buckets]
    plan = lpt_assign(costs, world)
    loads = [sum(costs[b] for b in plan[r]) for r in range(world)]
    return [buckets[b] for b in plan[rank]], loads
