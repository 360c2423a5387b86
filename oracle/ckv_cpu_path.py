"""CPU restatement of the reference's PyTorch CPU path, for timing only.

TEST / BASELINE INFRASTRUCTURE ONLY: imported by ``bench.py``'s CPU legs
(``cpu_baseline`` and ``--impl reference``), never by ``trpg_b200``.

The reference cannot travel to the GPU host, so this module restates its CPU
code path with torch CPU ops (multi-threaded through torch's intra-op pool),
step for step:

* quantize a residual block: min/max per group, IEEE division, round half
  to even, clamp, Q4 nibble pack (``models/quantized_kv.py:19-25``);
* bank layout and slab-free append (``:43-66``, rows appended by cat);
* dequantize: code * scale + low, then cast (``:32-33``, ``:68-75``);
* attention: ``update`` + ``scaled_dot_product_attention(enable_gqa=True)``
  (``:126-134``; ``scripts/profile_compressed_kv.py:39-42``).

Parity of this restatement with the numpy oracle is checked in
``tests/test_oracle_golden.py``.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def _quantize(rows: torch.Tensor, bits: int):
    rows = rows.float()
    low = rows.amin(-1)
    scale = ((rows.amax(-1) - low) / float((1 << bits) - 1)).clamp_min(1e-8)
    codes = ((rows - low.unsqueeze(-1)) / scale.unsqueeze(-1)).round().clamp(0, (1 << bits) - 1)
    codes = codes.to(torch.uint8)
    if bits == 4:
        codes = codes[..., 0::2] | (codes[..., 1::2] << 4)
    return codes, torch.stack((scale, low), -1)


def _dequantize(codes: torch.Tensor, meta: torch.Tensor, bits: int, dtype):
    if bits == 4:
        codes = torch.stack((codes & 15, codes >> 4), -1).flatten(-2)
    return (codes.float() * meta[..., :1] + meta[..., 1:]).to(dtype)


class CpuLayer:
    """The reference cache state machine on CPU tensors."""

    def __init__(self, bits: int):
        self.bits = bits
        self.kd = self.km = self.vd = self.vm = None
        self.keys = self.values = None
        self.length = 0

    @property
    def units(self):
        return 0 if self.kd is None else self.kd.shape[2]

    def _append_bank(self, k, v):
        b, h, t, d = k.shape
        kd, km = _quantize(k.reshape(b, h, t // 128, 128, d).transpose(-1, -2), self.bits)
        vd, vm = _quantize(v.reshape(b, h, t, d // 64, 64), self.bits)
        if self.kd is None:
            self.kd, self.km, self.vd, self.vm = kd, km, vd, vm
        else:
            self.kd = torch.cat((self.kd, kd), 2)
            self.km = torch.cat((self.km, km), 2)
            self.vd = torch.cat((self.vd, vd), 2)
            self.vm = torch.cat((self.vm, vm), 2)

    def append_for_attention(self, k, v):
        self.length += k.shape[-2]
        self.keys = k if self.keys is None else torch.cat((self.keys, k), -2)
        self.values = v if self.values is None else torch.cat((self.values, v), -2)

    def compact_residual(self):
        count = max(0, (self.keys.shape[-2] - 128) // 128 * 128)
        if count:
            self._append_bank(self.keys[..., :count, :], self.values[..., :count, :])
            self.keys = self.keys[..., count:, :].clone()
            self.values = self.values[..., count:, :].clone()

    def full_kv(self):
        if not self.units:
            return self.keys, self.values
        dtype = self.keys.dtype
        k = _dequantize(self.kd, self.km, self.bits, dtype)
        b, h = k.shape[:2]
        k = k.transpose(-1, -2).reshape(b, h, -1, k.shape[-2])
        v = _dequantize(self.vd, self.vm, self.bits, dtype).flatten(-2)
        return torch.cat((k, self.keys), -2), torch.cat((v, self.values), -2)

    def update(self, k, v):
        self.append_for_attention(k, v)
        out = self.full_kv()
        self.compact_residual()
        return out


def attend(q, layer: CpuLayer, scale: float):
    """Reference attention over a layer's current view (decode or verify)."""
    keys, values = layer.full_kv()
    mask = None
    if q.shape[2] > 1:
        from torch.nn.attention.bias import causal_lower_right
        mask = causal_lower_right(q.shape[2], keys.shape[2])
    return F.scaled_dot_product_attention(q, keys, values, attn_mask=mask, enable_gqa=True,
                                          scale=scale)


def decode_step(layer: CpuLayer, q, k_new, v_new, scale: float):
    """One decode step of one layer: append, attend, compact."""
    layer.append_for_attention(k_new, v_new)
    out = attend(q, layer, scale)
    layer.compact_residual()
    return out
