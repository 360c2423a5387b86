"""CPU oracle for the compressed-KV path.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` may
import it.  Nothing in ``trpg_b200`` imports it, and the CUDA path has no CPU
fallback that could route through it.

It restates, in numpy, the reference algorithm for every step of the path:

* quantizer   -- ``models/quantized_kv.py:15-25`` (CPU ``_pack``: IEEE fp32
  division, round half to even) and ``models/quantized_kv_kernels.py:7-22``
  (``_pack_kernel``: the same arithmetic with ``floor(t + 0.5)``);
* dequantizer -- ``models/quantized_kv.py:28-33`` (separate multiply and add)
  and ``models/quantized_kv_kernels.py:25-36`` (fused multiply-add, which the
  GPU decode kernels of the reference also use,
  ``models/compressed_kv_kernels.py:47,68``);
* bank layout -- ``models/quantized_kv.py:43-75`` (K grouped per channel over
  128 tokens, V per token over 64 channels);
* cache state machine -- ``models/quantized_kv.py:103-134``;
* attention   -- ``torch.nn.functional.scaled_dot_product_attention`` with
  ``enable_gqa=True`` and an optional ``causal_lower_right`` mask, the
  reference's own oracle (``scripts/profile_compressed_kv.py:39-42``,
  ``tests/test_compressed_prefill_attention.py:44-47``).  SDPA is third-party
  (torch; the reference pins 2.9.0 / 2.14.0); its published definition
  ``softmax(q k^T * scale + mask) v`` is restated here in float64.

Parity pin: ``tests/golden/make_golden.py`` runs the reference itself (CPU
``_pack``/``_unpack``, the Triton ``pack`` under the Triton interpreter, and
``QuantizedAttentionLayer.update`` + SDPA) and commits the results as
fixtures; ``tests/test_oracle_golden.py`` checks this module against them.
"""
from __future__ import annotations

import hashlib

import numpy as np

# --------------------------------------------------------------------------
# 16-bit float helpers (bit-exact round-to-nearest-even conversions)
# --------------------------------------------------------------------------


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    lsb = (u >> 16) & 1
    rounded = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    if nan.any():
        rounded = np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), rounded)
    return rounded


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 values to ``dtype`` ('bfloat16' | 'float16' | 'float32');
    return them as fp32 (exactly representable)."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == 'bfloat16':
        return bf16_bits_to_f32(f32_to_bf16_bits(x))
    if dtype == 'float16':
        return x.astype(np.float16).astype(np.float32)
    if dtype == 'float32':
        return x
    raise ValueError(dtype)


def seeded_normal(seed: int, shape, dtype: str = 'bfloat16', scale: float = 1.0) -> np.ndarray:
    """Deterministic N(0, 1) values rounded to ``dtype`` (returned as fp32).

    Uses numpy's PCG64 so that fixtures, tests and benchmarks regenerate the
    same inputs on any machine without depending on torch's RNG streams.
    """
    rng = np.random.Generator(np.random.PCG64(seed))
    return round_to(rng.standard_normal(size=shape, dtype=np.float32) * np.float32(scale), dtype)


def outlier_channels(seed: int, heads: int, dim: int, fraction: float = 0.01) -> np.ndarray:
    """Per KV head, ceil(fraction*dim) channels chosen by a seeded permutation."""
    rng = np.random.Generator(np.random.PCG64(seed + 7919))
    count = int(np.ceil(fraction * dim))
    return np.stack([rng.permutation(dim)[:count] for _ in range(heads)])


# --------------------------------------------------------------------------
# Quantizer / dequantizer
# --------------------------------------------------------------------------


def pack_rows(rows: np.ndarray, bits: int, rounding: str = 'half_even'):
    """Affine-quantize each row (last axis = one group).

    Follows ``models/quantized_kv.py:19-25`` (rounding='half_even') and
    ``models/quantized_kv_kernels.py:11-21`` (rounding='half_up').
    Returns (codes uint8 [..., G or G/2], meta float32 [..., 2] = (scale, low)).
    """
    if bits not in (4, 8):
        raise ValueError('bits must be 4 or 8')
    rows = np.asarray(rows, dtype=np.float32)
    levels = np.float32((1 << bits) - 1)
    low = rows.min(-1)
    scale = np.maximum((rows.max(-1) - low) / levels, np.float32(1e-8)).astype(np.float32)
    t = ((rows - low[..., None]) / scale[..., None]).astype(np.float32)
    if rounding == 'half_even':
        r = np.rint(t)
    elif rounding == 'half_up':
        r = np.floor((t + np.float32(0.5)).astype(np.float32))
    else:
        raise ValueError(rounding)
    codes = np.clip(r, 0, levels).astype(np.uint8)
    if bits == 4:
        codes = (codes[..., ::2] | (codes[..., 1::2] << 4)).astype(np.uint8)
    meta = np.stack((scale, low), -1).astype(np.float32)
    return codes, meta


def unpack_rows(codes: np.ndarray, meta: np.ndarray, bits: int, dtype: str = 'bfloat16',
                fused: bool = True) -> np.ndarray:
    """Dequantize rows; values are rounded to ``dtype`` and returned as fp32.

    fused=True  -> one rounding of code*scale+low (the reference's CUDA
                   unpack and decode kernels, ``quantized_kv_kernels.py:36``);
    fused=False -> product rounded to fp32, then the sum (CPU ``_unpack``,
                   ``quantized_kv.py:32-33``).
    """
    codes = np.asarray(codes, dtype=np.uint8)
    if bits == 4:
        codes = np.stack((codes & 15, codes >> 4), -1).reshape(*codes.shape[:-1], -1)
    c = codes.astype(np.float64)
    scale = meta[..., :1].astype(np.float64)
    low = meta[..., 1:].astype(np.float64)
    if fused:
        # code (8 bits) * scale (24 bits) is exact in float64; the sum is
        # exact unless the exponents of scale and low differ by more than 21.
        value = (c * scale + low).astype(np.float32)
    else:
        product = (c * scale).astype(np.float32).astype(np.float64)
        value = (product + low).astype(np.float32)
    return round_to(value, dtype)


# --------------------------------------------------------------------------
# Bank layout (models/quantized_kv.py:43-75)
# --------------------------------------------------------------------------


def key_rows(x: np.ndarray) -> np.ndarray:
    """[B,H,T,D] -> [B,H,T/128,D,128]: one row per channel per 128-token block."""
    b, h, t, d = x.shape
    return np.ascontiguousarray(x.reshape(b, h, t // 128, 128, d).transpose(0, 1, 2, 4, 3))


def value_rows(x: np.ndarray) -> np.ndarray:
    """[B,H,T,D] -> [B,H,T,D/64,64]: one row per token per 64-channel group."""
    b, h, t, d = x.shape
    return np.ascontiguousarray(x.reshape(b, h, t, d // 64, 64))


def unpack_key_bank(data, meta, bits, dtype='bfloat16', fused=True):
    rows = unpack_rows(data, meta, bits, dtype, fused)          # [B,H,U,D,128]
    b, h = rows.shape[:2]
    return np.ascontiguousarray(rows.transpose(0, 1, 2, 4, 3)).reshape(b, h, -1, rows.shape[-2])


def unpack_value_bank(data, meta, bits, dtype='bfloat16', fused=True):
    rows = unpack_rows(data, meta, bits, dtype, fused)          # [B,H,T,D/64,64]
    return rows.reshape(*rows.shape[:3], -1)


class OracleLayer:
    """CPU restatement of ``QuantizedAttentionLayer`` (``quantized_kv.py:93-134``).

    Holds the packed banks as plain arrays (units rows only, no slab padding)
    plus the exact residual window.
    """

    def __init__(self, bits: int, rounding: str = 'half_even', dtype: str = 'bfloat16'):
        self.bits, self.rounding, self.dtype = bits, rounding, dtype
        self.kd = self.km = self.vd = self.vm = None
        self.keys = self.values = None
        self.length = 0

    @property
    def units(self) -> int:
        return 0 if self.kd is None else self.kd.shape[2]

    @property
    def packed_tokens(self) -> int:
        return 128 * self.units

    def _append_bank(self, k: np.ndarray, v: np.ndarray):
        kd, km = pack_rows(key_rows(k), self.bits, self.rounding)
        vd, vm = pack_rows(value_rows(v), self.bits, self.rounding)
        if self.kd is None:
            self.kd, self.km, self.vd, self.vm = kd, km, vd, vm
        else:
            self.kd = np.concatenate((self.kd, kd), 2)
            self.km = np.concatenate((self.km, km), 2)
            self.vd = np.concatenate((self.vd, vd), 2)
            self.vm = np.concatenate((self.vm, vm), 2)

    def append_for_attention(self, k: np.ndarray, v: np.ndarray):
        """``quantized_kv.py:103-114``: concatenate into the residual."""
        if k.shape[-1] % 64:
            raise ValueError('head_dim must be a multiple of 64')
        self.length += k.shape[-2]
        self.keys = k.copy() if self.keys is None else np.concatenate((self.keys, k), -2)
        self.values = v.copy() if self.values is None else np.concatenate((self.values, v), -2)
        return self.view()

    def view(self):
        return dict(key_data=self.kd, key_meta=self.km, value_data=self.vd, value_meta=self.vm,
                    packed_tokens=self.packed_tokens, keys=self.keys, values=self.values,
                    bits=self.bits, length=self.length)

    def compact_residual(self):
        """``quantized_kv.py:116-124``: pack floor((R-128)/128)*128 tokens."""
        count = max(0, (self.keys.shape[-2] - 128) // 128 * 128)
        if count:
            self._append_bank(self.keys[..., :count, :], self.values[..., :count, :])
            self.keys = self.keys[..., count:, :].copy()
            self.values = self.values[..., count:, :].copy()

    def full_kv(self, fused: bool = True):
        """Dequantized history followed by the exact residual (``update``'s cat)."""
        if self.units:
            keys = np.concatenate((unpack_key_bank(self.kd, self.km, self.bits, self.dtype, fused),
                                   self.keys), -2)
            values = np.concatenate((unpack_value_bank(self.vd, self.vm, self.bits, self.dtype, fused),
                                     self.values), -2)
            return keys, values
        return self.keys, self.values

    def update(self, k: np.ndarray, v: np.ndarray, fused: bool = True):
        """``quantized_kv.py:126-134``: append, dequantize, compact."""
        self.append_for_attention(k, v)
        keys, values = self.full_kv(fused)
        self.compact_residual()
        return keys, values

    def fill(self, k: np.ndarray, v: np.ndarray):
        """The state ``update`` leaves (append, then compact) without
        dequantizing the history, for long contexts whose dequantized copy
        would not fit in memory."""
        self.append_for_attention(k, v)
        self.compact_residual()

    def head_kv(self, head: int, t0: int, t1: int, fused: bool = True):
        """Keys and values [t1 - t0, D] of one KV head for absolute positions
        [t0, t1): dequantized packed tokens, then the exact window."""
        parts_k, parts_v = [], []
        p = self.packed_tokens
        if t0 < p:
            a, b = t0, min(t1, p)
            u0, u1 = a // 128, -(-b // 128)
            kh = unpack_key_bank(self.kd[:, head:head + 1, u0:u1], self.km[:, head:head + 1, u0:u1],
                                 self.bits, self.dtype, fused)[0, 0]
            vh = unpack_value_bank(self.vd[:, head:head + 1, u0 * 128:u1 * 128],
                                   self.vm[:, head:head + 1, u0 * 128:u1 * 128],
                                   self.bits, self.dtype, fused)[0, 0]
            parts_k.append(kh[a - u0 * 128:b - u0 * 128])
            parts_v.append(vh[a - u0 * 128:b - u0 * 128])
        if t1 > p:
            a, b = max(t0, p) - p, t1 - p
            parts_k.append(self.keys[0, head, a:b])
            parts_v.append(self.values[0, head, a:b])
        return np.concatenate(parts_k, 0), np.concatenate(parts_v, 0)


# --------------------------------------------------------------------------
# Attention (restated SDPA with GQA and a lower-right causal mask)
# --------------------------------------------------------------------------


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float,
              causal_lower_right: bool = False) -> np.ndarray:
    """softmax(q k^T * scale [+ lower-right causal mask]) v, in float64.

    q [B,Hq,n,D]; k,v [B,Hkv,L,D]; query head h reads KV head h // (Hq/Hkv).
    Lower-right alignment: query i may see key j iff j <= L - n + i.
    """
    b, hq, n, d = q.shape
    hkv, length = k.shape[1], k.shape[2]
    group = hq // hkv
    kk = np.repeat(k.astype(np.float64), group, axis=1)
    vv = np.repeat(v.astype(np.float64), group, axis=1)
    logits = np.einsum('bhnd,bhld->bhnl', q.astype(np.float64), kk) * scale
    if causal_lower_right:
        i = np.arange(n)[:, None]
        j = np.arange(length)[None, :]
        logits = np.where(j <= length - n + i, logits, -np.inf)
    logits -= logits.max(-1, keepdims=True)
    p = np.exp(logits)
    p /= p.sum(-1, keepdims=True)
    return np.einsum('bhnl,bhld->bhnd', p, vv)


def decode_reference(q: np.ndarray, layer: OracleLayer, scale: float, fused: bool = True,
                     causal_lower_right: bool | None = None) -> np.ndarray:
    """The reference's attention over a view: dequantize + cat + SDPA."""
    keys, values = layer.full_kv(fused)
    if causal_lower_right is None:
        causal_lower_right = q.shape[2] > 1
    return attention(q, keys, values, scale, causal_lower_right)


def decode_reference_chunked(q: np.ndarray, layer: OracleLayer, scale: float, fused: bool = True,
                             causal_lower_right: bool | None = None, chunk: int = 8192,
                             t0: int = 0, t1: int | None = None):
    """``decode_reference`` with bounded memory: one KV head and ``chunk``
    positions at a time, softmax merged across chunks in float64 (the same
    log-sum-exp rule as ``combine_partials``).

    With ``t0`` / ``t1`` it covers only positions [t0, t1) and returns the
    unnormalised (m, l, o) of that range in the log2 domain instead (the
    split-KV partial of a shard).  Query row i of n may see position j iff
    j <= L - n + i when ``causal_lower_right``.
    """
    b, hq, n, d = q.shape
    length = layer.length
    if causal_lower_right is None:
        causal_lower_right = n > 1
    partial = t1 is not None
    t1 = length if t1 is None else t1
    heads = layer.kd.shape[1] if layer.kd is not None else layer.keys.shape[1]
    group = hq // heads
    log2e = np.log2(np.e)
    m = np.full((hq, n), -np.inf)
    l = np.zeros((hq, n))
    o = np.zeros((hq, n, d))
    for h in range(heads):
        qh = q[0, h * group:(h + 1) * group].astype(np.float64).reshape(group * n, d)
        rows = np.arange(group * n) % n
        for a in range(t0, t1, chunk):
            e = min(t1, a + chunk)
            kh, vh = layer.head_kv(h, a, e, fused)
            s2 = (qh @ kh.astype(np.float64).T) * (scale * log2e)
            if causal_lower_right:
                pos = np.arange(a, e)[None, :]
                s2 = np.where(pos <= length - n + rows[:, None], s2, -np.inf)
            mm = m[h * group:(h + 1) * group].reshape(-1)
            mc = np.maximum(mm, s2.max(-1))
            safe = np.where(np.isfinite(mc), mc, 0.0)
            alpha = np.where(np.isfinite(mm), np.exp2(mm - safe), 0.0)
            p = np.where(np.isfinite(s2), np.exp2(s2 - safe[:, None]), 0.0)
            sl = slice(h * group, (h + 1) * group)
            l[sl] = (l[sl].reshape(-1) * alpha + p.sum(-1)).reshape(group, n)
            o[sl] = (o[sl].reshape(-1, d) * alpha[:, None] + p @ vh.astype(np.float64)).reshape(group, n, d)
            m[sl] = mc.reshape(group, n)
    if partial:
        return m[None], l[None], o[None]
    return (o / l[..., None])[None]


# --------------------------------------------------------------------------
# Split-KV partial combine (compressed_kv_kernels.py:80-90)
# --------------------------------------------------------------------------


def partial_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float):
    """Unnormalised single-query attention over one KV range.

    Returns (m, l, o) in the log2 domain used by ``_partial``: m = max logit
    times log2(e), l = sum 2^(logit - m), o = sum 2^(logit - m) v.  An empty
    range gives m = -inf, l = 0, o = 0.
    """
    b, hq, n, d = q.shape
    group = hq // k.shape[1]
    if k.shape[2] == 0:
        return (np.full((b, hq, n), -np.inf), np.zeros((b, hq, n)), np.zeros((b, hq, n, d)))
    kk = np.repeat(k.astype(np.float64), group, axis=1)
    vv = np.repeat(v.astype(np.float64), group, axis=1)
    logits = np.einsum('bhnd,bhld->bhnl', q.astype(np.float64), kk) * scale * np.log2(np.e)
    m = logits.max(-1)
    p = np.exp2(logits - m[..., None])
    return m, p.sum(-1), np.einsum('bhnl,bhld->bhnd', p, vv)


def combine_partials(ms, ls, os_):
    """Log-sum-exp merge of partials (``compressed_kv_kernels.py:85-89``)."""
    ms = np.stack(ms)
    top = ms.max(0)
    safe = np.where(np.isfinite(top), top, 0.0)
    w = np.where(np.isfinite(ms), np.exp2(ms - safe), 0.0)
    num = (w[..., None] * np.stack(os_)).sum(0)
    den = (w * np.stack(ls)).sum(0)
    return num / den[..., None]


# --------------------------------------------------------------------------
# Misc
# --------------------------------------------------------------------------


def digest(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def cache_state(seed: int, heads: int, length: int, dim: int, bits: int, new_tokens: int = 1,
                dtype: str = 'bfloat16', rounding: str = 'half_even', outliers: bool = False):
    """Reference-reachable cache state (``scripts/profile_compressed_kv.py:31-36``).

    ``update`` with the first length-new_tokens tokens, then
    ``append_for_attention`` with the last new_tokens.  Returns
    (layer, k, v) where k, v are the full [1,H,length,D] inputs.
    """
    k = seeded_normal(seed, (1, heads, length, dim), dtype)
    v = seeded_normal(seed + 1, (1, heads, length, dim), dtype)
    if outliers:
        idx = outlier_channels(seed, heads, dim)
        for h in range(heads):
            k[:, h, :, idx[h]] = round_to(k[:, h, :, idx[h]] * 8, dtype)
            v[:, h, :, idx[h]] = round_to(v[:, h, :, idx[h]] * 8, dtype)
    layer = OracleLayer(bits, rounding, dtype)
    if length > 16384:
        layer.fill(k[:, :, :length - new_tokens], v[:, :, :length - new_tokens])
    else:
        layer.update(k[:, :, :length - new_tokens], v[:, :, :length - new_tokens])
    layer.append_for_attention(k[:, :, length - new_tokens:], v[:, :, length - new_tokens:])
    return layer, k, v
