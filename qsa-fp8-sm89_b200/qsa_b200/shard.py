"""Request sharding across GPUs (one process per GPU, no data-path collective).

Requests of a decode batch are independent -- each Top-K row reads only its
own block-table row and K/V pages -- so the batch is partitioned by request:

* ``contiguous_shards`` -- equal contiguous ranges;
* ``lpt_bins`` -- longest-processing-time-first bins on per-request Top-K
  lengths, for ragged batches;

Each rank then holds only the pages its requests reference (its block table
remapped to local page ids) and runs the decode on its own stream. Outputs
stay on their rank; ``gather_rows`` is the optional copy of every shard's
output to one rank, outside the hot path.
"""

from __future__ import annotations

import heapq

import torch


def contiguous_shards(n_rows: int, world: int) -> list[tuple[int, int]]:
    """[start, end) row range of each rank; sizes differ by at most one."""
    if world < 1:
        raise ValueError("world must be >= 1")
    base, extra = divmod(n_rows, world)
    out, start = [], 0
    for r in range(world):
        end = start + base + (1 if r < extra else 0)
        out.append((start, end))
        start = end
    return out


def lpt_bins(lengths, world: int) -> list[list[int]]:
    """Longest-processing-time-first assignment of requests to ``world`` bins.

    Requests are taken longest first and each goes to the bin with the least
    total length so far (ties: lowest bin id); within a bin, requests keep the
    longest-first order, which also serves as the in-GPU work order. The
    result is deterministic, so every rank computes the same plan.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    lens = [int(x) for x in (lengths.tolist() if hasattr(lengths, "tolist") else lengths)]
    order = sorted(range(len(lens)), key=lambda i: (-lens[i], i))
    heap = [(0, b) for b in range(world)]
    bins: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, b = heapq.heappop(heap)
        bins[b].append(i)
        heapq.heappush(heap, (load + lens[i], b))
    return bins


def bin_loads(lengths, bins) -> list[int]:
    lens = [int(x) for x in (lengths.tolist() if hasattr(lengths, "tolist") else lengths)]
    return [sum(lens[i] for i in b) for b in bins]


def gather_rows(local: torch.Tensor, counts: list[int], dst: int = 0, group=None):
    """Copies each rank's output rows to rank ``dst`` (torch.distributed).

    ``counts[r]`` is the number of rows rank r holds. Shards are padded to the
    largest count for one ``all_gather``; rank ``dst`` returns the rows in rank
    order, other ranks return None. Not part of the timed decode.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    width = max(counts)
    pad = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    if rank != dst:
        return None
    return torch.cat([p[:c] for p, c in zip(parts, counts)], dim=0)
