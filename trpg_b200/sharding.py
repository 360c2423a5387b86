"""Multi-GPU partitioning of the compressed-KV path.

Two strategies, one process per GPU (``torch.distributed``):

* batch x KV-head sharding -- independent sequences go to ranks by greedy
  longest-processing-time on their cache bytes; no data-path collective.
* sequence-split-KV -- one long sequence's packed 128-token blocks are split
  into contiguous ranges, one per rank; the last rank also owns the exact
  residual window.  Each rank produces (m, l, o) partials with the same
  kernel (``partial=True``); the log-sum-exp rule of
  ``models/compressed_kv_kernels.py:85-89`` merges them.  The partials cross
  GPUs either through ``PeerExchange`` (one launch per rank writes its
  partial into every rank's buffer over NVLink peer mappings and merges once
  all have arrived, no collective library) or through an NCCL all-gather
  followed by the merge kernel (``gather_partials``).

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


class PeerExchange:
    """Exchange of split-KV partials over peer memory between the ranks of a
    process group (one process per GPU), the ``ckv_exchange_*`` calls of
    ``include/ckv.h``.

    Each rank allocates one buffer, the ranks swap its CUDA IPC handle
    (``all_gather_object`` on ``group``, once), and every rank maps the
    others' buffers.  ``combine(partial)`` is then one launch per rank and
    step: publish this rank's partial into every buffer, wait for all ranks'
    partials of the step (bounded), merge.  It never synchronises the host,
    keeps its step count on the device (so it can be captured in a CUDA
    graph), and every rank must call it the same number of times.
    ``close()`` waits for the device and for the other ranks before it
    unmaps and frees.
    """

    def __init__(self, rows: int, head_dim: int, group=None, spin_limit: int = 0):
        import ctypes
        import torch.distributed as dist
        from . import _native
        self.group = group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.rows, self.head_dim, self.spin_limit = rows, head_dim, spin_limit
        lib = self._lib = _native.library()
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        _check(lib, lib.ckv_exchange_alloc(self.world, rows, head_dim, ctypes.byref(own), handle))
        self._own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self._peers = []
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(self._own)
                continue
            peer = ctypes.c_void_p()
            _check(lib, lib.ckv_exchange_open(h, ctypes.byref(peer)))
            self._peers.append(peer.value)
            ptrs.append(peer.value)
        self.buffers = ptrs

    def combine(self, partial: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        """This rank's partial [rows, D+2] fp32 in, the merged [rows, D] out."""
        from ._native import ops
        return ops().exchange_combine(partial, self.buffers, self.rank, 3, self.spin_limit, dtype)

    def error(self) -> int:
        """1 if a wait of this rank's launches gave up since the last check."""
        import ctypes
        flag = ctypes.c_int(0)
        stream = torch.cuda.current_stream().cuda_stream
        _check(self._lib, self._lib.ckv_exchange_error(self._own, ctypes.byref(flag), stream))
        return flag.value

    def close(self) -> None:
        import torch.distributed as dist
        if self._own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)        # no rank still writes into a buffer
        for p in self._peers:
            _check(self._lib, self._lib.ckv_exchange_close(p))
        dist.barrier(group=self.group)        # no rank still maps this one
        _check(self._lib, self._lib.ckv_exchange_free(self._own))
        self._own, self._peers, self.buffers = None, [], []


def _check(lib, status: int) -> None:
    if status != 0:
        raise RuntimeError(f'ckv: {lib.ckv_status_string(status).decode()}: '
                           f'{lib.ckv_last_error().decode()}')


def split_kv_attention(query: torch.Tensor, view, scale: float, group=None,
                       exchange: PeerExchange | None = None) -> torch.Tensor:
    """Attention of one sequence split across the ranks of ``group``.

    Every rank passes the same query and a view of the same cache (each rank
    only reads its own block range and, on the last rank, the residual).
    Returns the full output on every rank.  With ``exchange`` the partials
    cross GPUs through peer memory; without it, through an NCCL all-gather.
    """
    import torch.distributed as dist
    from . import compressed_kv_kernels as K
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    rng = split_kv_range(view.packed_tokens // 128, view.keys.shape[2], world, rank)
    part = K.attention([query], [view], scale, ranges=[rng], partial=True)[0]
    if exchange is not None:
        out = exchange.combine(part, query.dtype)
    else:
        out = K.combine(gather_partials(part, group), query.dtype)
    return out.view(query.shape)
