"""Multi-GPU partitioning of the compressed-KV path.

Two strategies, one process per GPU (``torch.distributed``):

* batch x KV-head sharding -- independent sequences go to ranks by greedy
  longest-processing-time on their cache bytes; no data-path collective.
* sequence-split-KV -- one long sequence's packed 128-token blocks are split
  into contiguous ranges, one per rank; the last rank also owns the exact
  residual window.  Each rank produces (m, l, o) partials with the same
  kernel (``partial=True``), the partials are all-gathered over NCCL, and the
  log-sum-exp rule of ``models/compressed_kv_kernels.py:85-89`` merges them.

The reference is single-GPU (``models/compressed_kv_attention.py:10``); both
strategies are new.
"""
from __future__ import annotations

import heapq
from typing import Sequence

import torch

Q_BYTES_PER_TOKEN = {8: 560, 4: 304}   # per KV head at D=256: codes + meta


def view_bytes(packed_tokens: int, residual: int, heads_kv: int = 4, head_dim: int = 256,
               bits: int = 8) -> int:
    """Algorithmic bytes one attention call streams for a view (codes, meta,
    exact residual); the per-token figures of the layout in ``include/ckv.h``."""
    codes = 2 * head_dim * bits // 8
    meta = head_dim * 8 // 128 + (head_dim // 64) * 8
    return heads_kv * (packed_tokens * (codes + meta) + residual * 4 * head_dim)


def lpt_partition(costs: Sequence[float], parts: int) -> list[list[int]]:
    """Greedy longest-processing-time: indices of ``costs`` per part.

    Items are placed largest first on the least-loaded part; ties go to the
    lowest part index, so every rank computes the same plan.
    """
    if parts < 1:
        raise ValueError('parts must be >= 1')
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0.0, p) for p in range(parts)]
    out: list[list[int]] = [[] for _ in range(parts)]
    for i in order:
        load, p = heapq.heappop(heap)
        out[p].append(i)
        heapq.heappush(heap, (load + costs[i], p))
    for items in out:
        items.sort()
    return out


def split_kv_range(units: int, residual: int, world: int, rank: int) -> list[int]:
    """(unit_begin, unit_end, resid_begin, resid_end) of ``rank``'s shard.

    Packed blocks are split as evenly as whole blocks allow; the residual
    window belongs to the last rank, which gets correspondingly fewer blocks.
    """
    if not 0 <= rank < world:
        raise ValueError('rank out of range')
    # A residual token costs about 1024/560 of a packed token; express the
    # residual in block units so the last rank's total load matches the rest.
    resid_blocks = residual * 1024 / (128 * 560)
    total = units + resid_blocks
    bounds = []
    for r in range(world + 1):
        b = round(total * r / world)
        bounds.append(min(units, max(0, b)))
    bounds[world] = units
    ub, ue = bounds[rank], bounds[rank + 1]
    if rank == world - 1:
        return [ub, ue, 0, residual]
    return [ub, ue, 0, 0]


def gather_partials(partial: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather [rows, D+2] partials -> [world, rows, D+2] (rank order)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    out = torch.empty((world * partial.shape[0], partial.shape[1]), dtype=partial.dtype,
                      device=partial.device)
    dist.all_gather_into_tensor(out, partial.contiguous(), group=group)
    return out.view(world, *partial.shape)


def split_kv_attention(query: torch.Tensor, view, scale: float, group=None) -> torch.Tensor:
    """Attention of one sequence split across the ranks of ``group``.

    Every rank passes the same query and a view of the same cache (each rank
    only reads its own block range and, on the last rank, the residual).
    Returns the full output on every rank.
    """
    import torch.distributed as dist
    from . import compressed_kv_kernels as K
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    rng = split_kv_range(view.packed_tokens // 128, view.keys.shape[2], world, rank)
    part = K.attention([query], [view], scale, ranges=[rng], partial=True)[0]
    parts = gather_partials(part, group)
    out = K.combine(parts, query.dtype)
    return out.view(query.shape)
