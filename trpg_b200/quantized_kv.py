"""Hybrid Q4/Q8 KV cache over the B200 kernels (mirror of ``models/quantized_kv.py``).

Same classes, names, tensor layout and state machine as the reference cache,
so ``HybridCacheTransaction``, prefix snapshots and the generation loops keep
working unchanged:

* ``_PackedBank`` (``models/quantized_kv.py:36-78``): slabs grow by 32 key
  units / 4096 value tokens and copy the history only when they grow; rows
  below ``units`` are never written again.
* ``QuantizedKVView`` (``:81-90``) and ``QuantizedAttentionLayer``
  (``:93-159``): exact residual window, append / compact / update.
* ``make_cache`` / ``cache_bytes`` (``:162-188``).

Two steps change:

* quantize-on-append: ``compact_residual`` quantizes the compacted tokens
  straight into the bank slabs with one launch (``ckv_pack_append``) instead
  of packing into temporaries and copying.  The bytes written are identical
  to packing the same rows with ``_pack``.
* the exact window: instead of ``torch.cat`` of the whole window on every
  token (``models/quantized_kv.py:109-110``), the window lives in a buffer
  with spare capacity and new tokens are written in place, K and V in one
  launch (``ckv_residual_append``).  ``keys`` / ``values`` are views of its
  first R rows; earlier views are never written again (appends go past
  their end, and compaction moves the rest to a new buffer), so snapshots
  taken by ``HybridCacheTransaction`` stay valid.  The layer keeps only
  plain integers about the buffer (its address, capacity and the rows
  written so far), so the transaction's snapshot of ``vars(layer)`` --
  tensors only under ``keys`` / ``values`` -- captures the whole state:
  after a rollback the restored integers and views agree, and the next
  append takes the place of the discarded tokens.  A view that is not the
  end of the rows this layer wrote (a snapshot restored by other means, a
  tensor set from outside) is copied to a new buffer before any append.

CUDA tensors only: the quantizer and dequantizer have no CPU path here.
"""
from __future__ import annotations

from typing import NamedTuple

import torch
from transformers import DynamicCache
from transformers.cache_utils import DynamicLayer

from . import quantized_kv_kernels as _kernels
from ._native import ROUNDING, ops

KEY_SLAB_UNITS = 32       # models/quantized_kv.py:48
WINDOW_MIN = 512          # tokens of exact-window capacity (compaction keeps it under 256)
VALUE_SLAB_TOKENS = 4096  # models/quantized_kv.py:51


_window_op = None


def _window_append(keys_new, values_new, keys, values, capacity):
    """One launch writes the new key and value rows after the window views
    ``keys`` / ``values`` (buffers of ``capacity`` rows per head) and returns
    the views of the rows written so far."""
    global _window_op
    if _window_op is None:
        _window_op = ops().window_append
    return _window_op(keys_new, values_new, keys, values, capacity)


def _pack(rows, bits, rounding=None):
    """``models/quantized_kv.py:15``; CUDA only."""
    return _kernels.pack(rows, bits, rounding or _kernels.DEFAULT_ROUNDING)


def _unpack(data, meta, bits, dtype):
    """``models/quantized_kv.py:28``; CUDA only."""
    return _kernels.unpack(data, meta, bits, dtype)


def _bank_shapes(kind, bits, b, h, d):
    """(data inner dims, meta inner dims) of one bank row."""
    if kind == 'key':
        return (d, 128 * bits // 8), (d, 2)
    return (d // 64, 64 * bits // 8), (d // 64, 2)


class _PackedBank:
    """Grow packed storage in slabs, never re-quantize historical blocks."""

    def __init__(self, bits, kind, rounding=None):
        self.bits, self.kind = bits, kind
        self.rounding = rounding or _kernels.DEFAULT_ROUNDING
        self.data = self.meta = None
        self.units = 0

    def _rows_per_unit(self):
        return 1 if self.kind == 'key' else 128

    def reserve(self, units_needed, like, b, h, d):
        """Ensure capacity for ``units_needed`` units (128 tokens each)."""
        per = self._rows_per_unit()
        end = units_needed * per
        if self.data is not None and end <= self.data.shape[2]:
            return
        slab = KEY_SLAB_UNITS if self.kind == 'key' else VALUE_SLAB_TOKENS
        capacity = ((end + slab - 1) // slab) * slab
        dshape, mshape = _bank_shapes(self.kind, self.bits, b, h, d)
        new_data = torch.empty((b, h, capacity, *dshape), device=like.device, dtype=torch.uint8)
        new_meta = torch.empty((b, h, capacity, *mshape), device=like.device, dtype=torch.float32)
        if self.units:
            used = self.units * per
            new_data[:, :, :used].copy_(self.data[:, :, :used])
            new_meta[:, :, :used].copy_(self.meta[:, :, :used])
        self.data, self.meta = new_data, new_meta

    def append(self, x):
        """Reference-compatible append of [B,H,T,D] tokens (T a multiple of 128)."""
        b, h, t, d = x.shape
        if self.kind == 'key':
            rows = x.reshape(b, h, t // 128, 128, d).transpose(-1, -2).contiguous()
        else:
            rows = x.reshape(b, h, t, d // 64, 64).contiguous()
        data, meta = _pack(rows, self.bits, self.rounding)
        units = t // 128
        self.reserve(self.units + units, x, b, h, d)
        per = self._rows_per_unit()
        lo, hi = self.units * per, (self.units + units) * per
        self.data[:, :, lo:hi].copy_(data)
        self.meta[:, :, lo:hi].copy_(meta)
        self.units += units

    def unpack(self, dtype):
        per = self._rows_per_unit()
        rows = _unpack(self.data[:, :, :self.units * per].contiguous(),
                       self.meta[:, :, :self.units * per].contiguous(), self.bits, dtype)
        b, h = rows.shape[:2]
        if self.kind == 'key':
            return rows.transpose(-1, -2).reshape(b, h, -1, rows.shape[-2])
        return rows.flatten(-2)

    def bytes(self):
        return sum(t.numel() * t.element_size() for t in (self.data, self.meta) if t is not None)


class QuantizedKVView(NamedTuple):
    key_data: torch.Tensor | None
    key_meta: torch.Tensor | None
    value_data: torch.Tensor | None
    value_meta: torch.Tensor | None
    packed_tokens: int
    keys: torch.Tensor
    values: torch.Tensor
    bits: int
    length: int


class QuantizedAttentionLayer(DynamicLayer):
    is_croppable = False

    def __init__(self, bits, rounding=None):
        super().__init__()
        self.bits = bits
        self.rounding = rounding or _kernels.DEFAULT_ROUNDING
        self.cumulative_length = 0
        # The exact window's buffers: key / value base addresses, rows per
        # head, and rows written by this layer (0: no buffer).
        self._window_kptr = self._window_vptr = 0
        self._window_cap = self._window_rows = 0
        self.key_bank = _PackedBank(bits, 'key', self.rounding)
        self.value_bank = _PackedBank(bits, 'value', self.rounding)

    def append_for_attention(self, key_states, value_states):
        """``models/quantized_kv.py:103-114``, appending in place to the window buffer."""
        n = key_states.shape[-2]
        cap, rows = self._window_cap, self._window_rows
        if cap and rows + n <= cap:
            keys, values = self.keys, self.values
            if (keys.shape[2] == rows and keys.data_ptr() == self._window_kptr
                    and values.data_ptr() == self._window_vptr):
                # Fast path: the views end at the rows this layer wrote (the op
                # checks dtype, device and the buffer geometry).
                self.keys, self.values = _window_append(key_states, value_states, keys, values, cap)
                self._window_rows = rows + n
                self.cumulative_length += n
                kb, vb = self.key_bank, self.value_bank
                return QuantizedKVView(kb.data, kb.meta, vb.data, vb.meta, kb.units * 128,
                                       self.keys, self.values, self.bits, self.cumulative_length)
        if key_states.shape[-1] % 64 or value_states.shape[-1] % 64:
            raise ValueError('quantized KV needs head_dim to be a multiple of 64')
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        self.cumulative_length += n
        if not (key_states.is_cuda and key_states.dim() == 4 and key_states.shape[0] == 1
                and key_states.dtype in (torch.bfloat16, torch.float16)
                and value_states.shape == key_states.shape and value_states.dtype == key_states.dtype
                and (self.keys.dim() != 4 or (self.keys.dtype == key_states.dtype
                                              and self.keys.shape[1] == key_states.shape[1]
                                              and self.keys.shape[3] == key_states.shape[3]))):
            self.keys = torch.cat((self.keys, key_states), dim=-2)
            self.values = torch.cat((self.values, value_states), dim=-2)
            self._forget_window()
        else:
            r = self.keys.shape[-2] if self.keys.dim() == 4 else 0
            self._new_window(key_states, r + n, self.keys if r else None, self.values if r else None)
            self.keys, self.values = _window_append(key_states, value_states, self.keys, self.values,
                                                    self._window_cap)
            self._window_rows = r + n
        return QuantizedKVView(self.key_bank.data, self.key_bank.meta,
                               self.value_bank.data, self.value_bank.meta,
                               self.key_bank.units * 128, self.keys, self.values,
                               self.bits, self.cumulative_length)

    def _forget_window(self):
        self._window_kptr = self._window_vptr = 0
        self._window_cap = self._window_rows = 0

    def _new_window(self, like, need, keys=None, values=None):
        """Fresh window buffers with room for ``need`` rows plus 256 more; the
        rows of ``keys`` / ``values`` (if given) are copied to their start and
        ``self.keys`` / ``self.values`` become the views of those rows."""
        b, h, _, d = like.shape
        cap = max(WINDOW_MIN, -(-need // 128) * 128 + 256)
        kb = torch.empty((b, h, cap, d), dtype=like.dtype, device=like.device)
        vb = torch.empty_like(kb)
        r = 0
        if keys is not None:
            r = keys.shape[2]
            kb[:, :, :r].copy_(keys)
            vb[:, :, :r].copy_(values)
        self.keys, self.values = kb.narrow(2, 0, r), vb.narrow(2, 0, r)
        self._window_kptr, self._window_vptr = kb.data_ptr(), vb.data_ptr()
        self._window_cap, self._window_rows = cap, r

    def compact_residual(self):
        """``models/quantized_kv.py:116-124``, quantizing straight into the slabs."""
        count = max(0, (self.keys.shape[-2] - 128) // 128 * 128)
        if not count:
            return
        b, h, r, d = self.keys.shape
        if b != 1:
            raise NotImplementedError('the quantized hybrid cache holds a single session')
        units = self.key_bank.units
        self.key_bank.reserve(units + count // 128, self.keys, b, h, d)
        self.value_bank.reserve(units + count // 128, self.keys, b, h, d)
        ops().pack_append(self.keys, self.values, self.key_bank.data, self.key_bank.meta,
                          self.value_bank.data, self.value_bank.meta, count, units, self.bits,
                          ROUNDING[self.rounding])
        self.key_bank.units = units + count // 128
        self.value_bank.units = units + count // 128
        # The rest moves to a new window (the reference clones it); the old
        # buffer, and every view of it handed out, stays as it was.
        self._new_window(self.keys, r - count, self.keys[..., count:, :], self.values[..., count:, :])

    def update(self, key_states, value_states, *args, **kwargs):
        """``models/quantized_kv.py:126-134``: dequantized history + residual."""
        self.append_for_attention(key_states, value_states)
        if self.key_bank.units:
            keys = torch.cat((self.key_bank.unpack(self.dtype), self.keys), dim=-2)
            values = torch.cat((self.value_bank.unpack(self.dtype), self.values), dim=-2)
        else:
            keys, values = self.keys, self.values
        self.compact_residual()
        return keys, values

    def get_seq_length(self):
        return self.cumulative_length

    def bytes(self):
        return self.key_bank.bytes() + self.value_bank.bytes() + sum(
            t.numel() * t.element_size() for t in (self.keys, self.values) if t is not None)

    def reset(self):
        self.__init__(self.bits, self.rounding)

    def reorder_cache(self, beam_idx):
        raise NotImplementedError('the quantized hybrid cache holds a single session; no beam reorder')

    def offload(self):
        raise NotImplementedError('the quantized hybrid cache does not support CPU offload')

    def crop(self, *args, **kwargs):
        raise NotImplementedError('hybrid state must be rebuilt as a whole; KV cannot be cropped')

    def batch_repeat_interleave(self, *args, **kwargs):
        raise NotImplementedError('the quantized hybrid cache holds a single session')

    def batch_select_indices(self, *args, **kwargs):
        raise NotImplementedError('the quantized hybrid cache holds a single session')


def make_cache(config, mode='q8'):
    """``models/quantized_kv.py:162-170``."""
    if mode not in ('bf16', 'q8', 'q4'):
        raise ValueError('KV mode must be bf16, q8 or q4')
    cache = DynamicCache(config=config)
    if mode != 'bf16':
        for index, kind in enumerate(config.layer_types):
            if kind == 'full_attention':
                cache.layers[index] = QuantizedAttentionLayer(int(mode[1:]))
    return cache


def cache_bytes(cache):
    """``models/quantized_kv.py:173-188``: retained storage, shared views once."""
    seen = set()

    def retained(value):
        if isinstance(value, torch.Tensor):
            storage = value.untyped_storage()
            key = (value.device, storage.data_ptr())
            if key in seen:
                return 0
            seen.add(key)
            return storage.nbytes()
        if isinstance(value, dict):
            return sum(retained(v) for v in value.values())
        if isinstance(value, (list, tuple)):
            return sum(retained(v) for v in value)
        if isinstance(value, _PackedBank):
            return sum(retained(v) for v in vars(value).values())
        return 0

    return sum(retained(vars(layer)) for layer in cache.layers)
