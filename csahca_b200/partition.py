"""Partitioning of decode batches over the GPUs of one node (one process per GPU).

The batched decode paths shard with no collective on the data path: every
rank owns a disjoint share of the work and the K/V (or paged caches) of that
share, decodes it with the single-GPU kernels, and is done.

* CSA batches (configs 1-3): requests are independent (b, h) rows.  A batch of
  requests is split greedily by context length (longest first onto the least
  loaded rank), because the scorer's time is proportional to the K rows it
  reads, i.e. to sum(L_b) of the rank's requests.  A batch of one request with
  few heads (config 1: 8 heads) is split by head.
* DSV4 batches (configs 4/5): queries carry equal slot counts, so ranks get
  contiguous, equal query ranges.

``gather_rows`` reassembles per-rank outputs into the full batch for callers
that want every output on every rank (an all-gather; not part of a timed
decode step).  The reference runs on one GPU only; its callers' process model
(one process per GPU) is integrations/sglang_dsv4/scripts/launch_patched_dsv4.sh:17,76.
"""

from __future__ import annotations

from typing import Sequence

import torch
import torch.distributed as dist


def shard_requests_by_length(lengths: Sequence[int], world: int) -> list[list[int]]:
    """Greedy longest-first split of requests over ``world`` ranks, balancing
    the sum of context lengths.  Returns each rank's request ids in ascending
    order.  Ties go to the lower request id and to the lower rank, so every
    rank computes the same split."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    load = [0] * world
    shares: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (load[j], len(shares[j]), j))
        shares[r].append(i)
        load[r] += int(lengths[i])
    return [sorted(s) for s in shares]


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous, near-equal range ``[lo, hi)`` of ``n`` items for ``rank``."""
    return (n * rank) // world, (n * (rank + 1)) // world


def shard_heads(heads: int, rank: int, world: int) -> tuple[int, int]:
    """Head range of ``rank`` for a head-sharded decode (config 1: 8 heads)."""
    return shard_range(heads, rank, world)


def shard_queries(num_queries: int, rank: int, world: int) -> list[int]:
    """Query ids of ``rank`` for a DSV4 batch (equal slot counts per query)."""
    lo, hi = shard_range(num_queries, rank, world)
    return list(range(lo, hi))


def imbalance(lengths: Sequence[int], shares: list[list[int]]) -> float:
    """max over ranks of the share's summed length / the mean (1.0 = perfect)."""
    loads = [sum(int(lengths[i]) for i in s) for s in shares]
    mean = sum(loads) / max(1, len(loads))
    return max(loads) / mean if mean else 1.0


def gather_rows(local: torch.Tensor, ids: Sequence[int], total: int, group=None) -> torch.Tensor:
    """Every rank's rows ``local[i]`` (request ``ids[i]``) assembled into a
    ``[total, ...]`` tensor on every rank.  Ranks may own different numbers of
    rows: shares are padded to the largest one for the all-gather."""
    world = dist.get_world_size(group)
    counts = [0] * world
    dist.all_gather_object(counts, len(ids), group=group)
    id_lists: list = [None] * world
    dist.all_gather_object(id_lists, list(map(int, ids)), group=group)
    width = max(counts)
    pad = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    out = torch.empty((total,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    seen = 0
    for r in range(world):
        if counts[r]:
            out[torch.tensor(id_lists[r], device=local.device)] = parts[r][: counts[r]]
        seen += counts[r]
    if seen != total:
        raise RuntimeError(f"gather_rows: ranks own {seen} rows, expected {total}")
    return out
