"""Drop-in for ``models/compressed_kv_kernels.py``: attention over packed views.

``decode(query, view, scale)`` keeps the reference signature and return
convention (``models/compressed_kv_kernels.py:93``): a new tensor shaped and
typed like ``query``; the view is not modified.  It runs one launch of the
hand-written sm_100a kernel behind ``ckv_attention`` (``include/ckv.h``):
split-KV over (KV head, 128-token block) work items, in-register dequant of
the Q8/Q4 history next to the exact residual window, and the log-sum-exp
merge of the splits inside the same launch.

Beyond the reference:

* ``verify(query, view, scale)`` -- 2..4 (up to 16 rows per KV head) queries
  with lower-right causal masking, the semantics of dequantize + SDPA with
  ``causal_lower_right(q, L)`` (``models/quantized_kv.py:126-134``;
  ``models/compressed_prefill_kernels.py:81,90``);
* ``attention(queries, views, scale)`` -- many sequences (ragged lengths) in
  one launch;
* ``partial=True`` / ``ranges`` -- split-KV partials (m, l, o) of a shard of
  the packed blocks and residual, merged by ``combine``.
"""
from __future__ import annotations

from typing import Sequence

import torch

from . import _native
from ._native import ops

MAX_SEQS = 64   # CKV_MAX_SEQS in include/ckv.h

DEQUANT_MODES = _native.DEQUANT_MODES


def set_dequant(mode: str) -> str:
    """Select the dequantization rule of every attention call in this process
    (decode, verify, batched, split-KV); returns the previous one.

    * ``'exact'`` -- each code becomes ``round_to_query_dtype(fma(code,
      scale, low))`` before it meets the query or the probabilities, the
      rounding of the reference's own kernel
      (``models/compressed_kv_kernels.py:47,68``, pinned by the reference's
      fused-multiply-add known-answer test).
    * ``'folded'`` -- the scales are multiplied into the query and the
      probabilities instead (``sum_d (q_d scale_d) code_d + sum_d q_d low_d``,
      and per token for the values), and the codes reach the tensor cores as
      exact fp16 values.  Several times fewer instructions per code; the
      results differ from the exact rule by fp16 rounding of q*scale and
      p*scale (finer than the bf16 rounding of each dequantized value) and
      meet the same tolerances against dequantize + SDPA.  Head dims 128 and
      256; 64 uses the exact rule.

    The environment variable ``TRPG_CKV_DEQUANT`` sets the rule when the
    library loads (default ``'exact'``).
    """
    return _native.set_dequant(mode)


def dequant() -> str:
    """The dequantization rule in force (see ``set_dequant``)."""
    return _native.dequant()


def _inner_dense(t: torch.Tensor) -> torch.Tensor:
    """Banks need dense inner two dims and 16-byte aligned rows."""
    if t.stride(-1) != 1 or t.stride(-2) != t.shape[-1]:
        t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone(memory_format=torch.contiguous_format)
    return t


def _dense_rows(t: torch.Tensor) -> torch.Tensor:
    """Value banks: each token's groups contiguous (TMA boxes / bulk copies of 32 tokens)."""
    if (t.stride(-1) != 1 or t.stride(-2) != t.shape[-1]
            or t.stride(-3) != t.shape[-2] * t.shape[-1] or t.data_ptr() % 16):
        t = t.contiguous()
        if t.data_ptr() % 16:
            t = t.clone()
    return t


def _residual(t: torch.Tensor) -> torch.Tensor:
    if t.stride(-1) != 1 or t.stride(-2) % 8 or t.stride(-3) % 8 or t.data_ptr() % 16:
        t = t.contiguous()
        if t.data_ptr() % 16:
            t = t.clone()
    return t


def full_range(view) -> list[int]:
    """(unit_begin, unit_end, resid_begin, resid_end) covering the whole view."""
    return [0, view.packed_tokens // 128, 0, view.keys.shape[2]]


def attention(queries: Sequence[torch.Tensor], views: Sequence, scale: float, *,
              ranges: Sequence[Sequence[int]] | None = None, partial: bool = False):
    """One launch over every (query, view) pair.

    queries[i]: [1, Hq, nq, D] (bf16/fp16, last dim dense); views[i]: a
    ``QuantizedKVView``.  Returns a list of outputs shaped like the queries,
    or, with ``partial=True``, float32 [Hq*nq, D+2] partials (o, m, l).
    """
    if len(queries) != len(views) or not queries:
        raise ValueError('need one view per query')
    bits = views[0].bits
    kd, km, vd, vm, rk, rv, packed, lengths, flat = [], [], [], [], [], [], [], [], []
    for i, (q, v) in enumerate(zip(queries, views)):
        if v.bits != bits:
            raise ValueError('all views of one call must share bits')
        rng = list(ranges[i]) if ranges is not None else full_range(v)
        has_packed = rng[1] > rng[0]
        kd.append(_inner_dense(v.key_data) if has_packed else None)
        km.append(_inner_dense(v.key_meta) if has_packed else None)
        vd.append(_dense_rows(v.value_data) if has_packed else None)
        vm.append(_dense_rows(v.value_meta) if has_packed else None)
        has_resid = rng[3] > rng[2]
        rk.append(_residual(v.keys) if has_resid else None)
        rv.append(_residual(v.values) if has_resid else None)
        packed.append(int(v.packed_tokens))
        lengths.append(int(v.length))
        flat.extend(int(x) for x in rng)
    out = []
    for c in range(0, len(queries), MAX_SEQS):      # the kernel takes 64 sequences per launch
        sl = slice(c, c + MAX_SEQS)
        out += ops().attention(list(queries[sl]), kd[sl], km[sl], vd[sl], vm[sl], rk[sl], rv[sl],
                               packed[sl], lengths[sl], flat[4 * c:4 * (c + MAX_SEQS)], int(bits),
                               float(scale), bool(partial))
    return out


_decode_op = None


def _single(query, view, scale):
    """One sequence over its whole view; the op fixes any bank or window
    layout the kernel cannot read directly."""
    global _decode_op
    if view.packed_tokens < 128 or view.keys.shape[2] == 0:
        return attention([query], [view], scale)[0]
    if _decode_op is None:
        _decode_op = ops().decode
    return _decode_op(query, view.key_data, view.key_meta, view.value_data, view.value_meta,
                      view.keys, view.values, view.packed_tokens, view.length, view.bits, scale)


def decode(query: torch.Tensor, view, scale: float) -> torch.Tensor:
    """Single-query GQA decode over a packed view (``compressed_kv_kernels.py:93``)."""
    return _single(query, view, scale)


def verify(query: torch.Tensor, view, scale: float) -> torch.Tensor:
    """Multi-query verify: lower-right causal attention of query [1,Hq,n,D]."""
    return _single(query, view, scale)


def attention_error(device=None) -> int:
    """1 if an attention call on ``device`` gave up waiting inside the kernel
    (its outputs are then invalid) since the last check, else 0; clears it.

    The kernels bound every wait (about a second) instead of hanging; this
    reports such an event.  It waits for the device's streams that ran
    attention calls.
    """
    dev = torch.device('cuda', torch.cuda.current_device()) if device is None else torch.device(device)
    return int(ops().attention_error(torch.empty(0, device=dev)))


def combine(partials: Sequence[torch.Tensor] | torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Log-sum-exp merge of split-KV partials (``compressed_kv_kernels.py:85-89``).

    partials: list of [rows, D+2] float32 (or one [parts, rows, D+2] tensor).
    Returns [rows, D] of ``dtype``.
    """
    if not isinstance(partials, torch.Tensor):
        partials = torch.stack(list(partials))
    return ops().combine_partials(partials, dtype)
