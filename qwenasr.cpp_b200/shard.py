"""Stream sharding across GPUs (one process per GPU, no data-path collective).

Each utterance stream's KV cache lives on one GPU, so streams are partitioned
up front.  Predicted cost of a stream = the KV bytes its decode steps read,
i.e. the sum over its steps of its context length; streams are assigned
longest-first to the least-loaded rank (greedy LPT).  torch.distributed is
used only for timing: the barrier and the max (or sum) over ranks.
"""
from __future__ import annotations

import heapq

import numpy as np


def stream_cost(prompt_len: int, new_tokens: int) -> int:
    """Tokens read by all decode steps of one stream: sum_{t<n} (P + t + 1)."""
    return int(new_tokens * prompt_len + new_tokens * (new_tokens + 1) // 2)


def lpt_partition(costs, n_ranks: int, cap: int | None = None) -> list[list[int]]:
    """Indices of `costs` per rank, greedy longest-processing-time first: each
    stream, costliest first, goes to the least-loaded rank (ties: lowest rank).
    With `cap`, a rank that holds `cap` streams takes no more (a fixed batch
    per GPU); n_ranks * cap must cover all streams."""
    costs = np.asarray(costs, dtype=np.int64)
    if cap is not None and cap * n_ranks < len(costs):
        raise ValueError("cap * n_ranks is smaller than the number of streams")
    order = np.argsort(-costs, kind="stable")
    heap = [(0, r) for r in range(n_ranks)]
    out: list[list[int]] = [[] for _ in range(n_ranks)]
    for i in order:
        load, r = heapq.heappop(heap)
        out[r].append(int(i))
        if cap is None or len(out[r]) < cap:
            heapq.heappush(heap, (load + int(costs[i]), r))
    return [sorted(x) for x in out]


def reduce_max(dist, value: float, device=None) -> float:
    """Max of a scalar over ranks (dist = torch.distributed or None)."""
    if dist is None:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reduce_sum(dist, value: float, device=None) -> float:
    if dist is None:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())
