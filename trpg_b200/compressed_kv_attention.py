"""Guarded compressed-KV attention entry points and the attention-module patch.

Mirror of ``models/compressed_kv_attention.py`` over the B200 kernels:

* ``compressed_kv_decode(query, view, scale)`` -- the same eligibility rules
  as the reference (``:8-29``), applied in C++ in the same op call as the
  kernel; returns ``None`` for anything the kernel does not cover so the
  caller falls back to SDPA.
* ``compressed_kv_verify(query, view, scale)`` -- new: the multi-query
  (MTP verify) variant, up to 16 query rows per KV head, lower-right causal.
* ``_supported_mask`` (``:32-37``), ``_forward`` (``:40-82``),
  ``configure_compressed_kv_attention`` (``:85-95``) and
  ``compressed_kv_info`` (``:98-103``).  ``_forward`` additionally routes
  2..4-token calls to ``compressed_kv_verify`` inside
  ``mtp_verification_scope`` (``trpg_b200.mtp_verification_kernels``, which
  shares the reference's flag once ``trpg_b200.install`` has run), and
  chunks over a packed history to ``compressed_kv_prefill``
  (``trpg_b200.compressed_prefill_attention``) where the packed kernel is
  faster than dequantize + SDPA: by default 16..4096 tokens at head_dim 128
  and 256 (the tcgen05 kernel) and 16..1024 at head_dim 64 (the mma.sync
  kernel); 16..4096 with ``prefill=True``, none with ``prefill=False``.  The
  reference only exposes that kernel as a standalone API.

Kernel launch errors raise; only "unsupported" returns ``None``.
"""
from __future__ import annotations

import sys
from types import MethodType

import torch

from . import mtp_verification_kernels as _scope
from .quantized_kv import QuantizedAttentionLayer

BACKEND = 'b200-affine-q4-q8-cuda'


DECODE_ROUTE, VERIFY_ROUTE = 0, 1   # Route in trpg_b200/csrc/ckv_torch.cpp

_guarded_ops = {}


def _quantized_layer(layer):
    """This package's cache layer, or the reference's own (``models.quantized_kv``
    loaded before ``install()`` ran): both hand out the same view and keep
    the same layout, so the kernels serve either."""
    if isinstance(layer, QuantizedAttentionLayer):
        return True
    cls = type(layer)
    if cls.__name__ != 'QuantizedAttentionLayer':
        return False
    module = sys.modules.get(cls.__module__)
    return getattr(module, 'QuantizedAttentionLayer', None) is cls and hasattr(layer, 'key_bank')


def _run_guarded(query, view, scale, route):
    """The view's plain fields are type-checked here; the acceptance rules of
    the kernels (the reference's guard, ``:8-29``) and the launch run in one
    C++ op call, which returns None when the call is not covered."""
    length, bits, packed = view.length, view.bits, view.packed_tokens
    if (type(length) is not int or type(packed) is not int or type(bits) is not int
            or not isinstance(scale, (int, float)) or isinstance(scale, bool)):
        return None
    op = _guarded_ops.get(route)
    if op is None:
        from ._native import ops
        op = _guarded_ops[route] = (ops().decode_guarded if route == DECODE_ROUTE
                                    else ops().attention_guarded)
    if route == DECODE_ROUTE:
        return op(query, view.key_data, view.key_meta, view.value_data, view.value_meta,
                  view.keys, view.values, packed, length, bits, float(scale))
    return op(query, view.key_data, view.key_meta, view.value_data, view.value_meta,
              view.keys, view.values, packed, length, bits, float(scale), route)


def compressed_kv_decode(query, view, scale):
    """Single-query decode over a packed view, or None when unsupported
    (reference ``:8-29``); launch errors raise."""
    return _run_guarded(query, view, scale, DECODE_ROUTE)


def compressed_kv_verify(query, view, scale):
    """Multi-query verify over a packed view, or None when unsupported.

    query [1, Hq, n, D] holds the last n positions (already appended to the
    view's window); the n * Hq/Hkv query rows of a KV head must not exceed 16.
    """
    return _run_guarded(query, view, scale, VERIFY_ROUTE)


def _supported_mask(mask, length, queries=1):
    """Masks the kernels reproduce exactly (reference ``:32-37``).

    One query: None or a lower-right causal bias of 1 x ``length``.  Several
    queries: only the lower-right causal bias of ``queries`` x ``length``.
    Upstream attention given no mask for several queries aligns its causal
    mask top-left (SDPA ``is_causal``), which is not the kernels' rule, so
    that call stays on the upstream path.
    """
    if mask is None:
        return queries == 1
    from torch.nn.attention.bias import CausalBias, CausalVariant
    return (type(mask) is CausalBias and mask.variant == CausalVariant.LOWER_RIGHT
            and mask.seq_len_q == queries and mask.seq_len_kv == length)


def _forward(self, hidden_states, position_embeddings, attention_mask, past_key_values=None, **kwargs):
    """Patched ``Qwen3_5Attention.forward`` (reference ``:40-82``)."""
    layer = None
    if past_key_values is not None and self.layer_idx < len(past_key_values.layers):
        layer = past_key_values.layers[self.layer_idx]
    q_len = hidden_states.shape[1] if hidden_states.ndim == 3 else 0
    verify = q_len > 1 and q_len <= 4 and _scope.mtp_verification_enabled()
    prefill = 16 <= q_len <= getattr(self, '_direct_kv_prefill_max', 0)
    eligible = (self._direct_kv_enabled and not self.training and not torch.is_grad_enabled()
                and not torch.is_autocast_enabled('cuda') and hidden_states.is_cuda
                and hidden_states.shape[0] == 1 and (q_len == 1 or verify or prefill)
                and hidden_states.dtype in (torch.bfloat16, torch.float16)
                and _quantized_layer(layer) and layer.key_bank.units > 0
                and self.head_dim in (64, 128, 256) and self.config._attn_implementation == 'sdpa'
                and not kwargs.get('output_attentions', False) and kwargs.get('head_mask') is None
                and all(value is None or name in ('is_causal', 'output_attentions', 'use_cache', 'position_ids')
                        for name, value in kwargs.items())
                and _supported_mask(attention_mask, layer.get_seq_length() + q_len, q_len))
    if not eligible:
        return self._direct_kv_original(hidden_states, position_embeddings, attention_mask,
                                        past_key_values=past_key_values, **kwargs)
    from transformers.models.qwen3_5.modeling_qwen3_5 import apply_rotary_pos_emb
    shape = hidden_states.shape[:-1]
    head_shape = (*shape, -1, self.head_dim)
    query, gate = torch.chunk(self.q_proj(hidden_states).view(*shape, -1, self.head_dim * 2), 2, -1)
    gate = gate.reshape(*shape, -1)
    query = self.q_norm(query.reshape(head_shape)).transpose(1, 2)
    key = self.k_norm(self.k_proj(hidden_states).view(head_shape)).transpose(1, 2)
    value = self.v_proj(hidden_states).view(head_shape).transpose(1, 2)
    query, key = apply_rotary_pos_emb(query, key, *position_embeddings)
    view = layer.append_for_attention(key, value)
    if q_len == 1:
        output = compressed_kv_decode(query, view, self.scaling)
    elif verify:
        output = compressed_kv_verify(query, view, self.scaling)
    else:
        from .compressed_prefill_attention import compressed_kv_prefill
        output = compressed_kv_prefill(query, view, self.scaling)
    if output is None:
        # State was appended once: finish the same operation with SDPA rather
        # than running upstream and appending these tokens a second time.
        keys = torch.cat((layer.key_bank.unpack(layer.dtype), view.keys), -2)
        values = torch.cat((layer.value_bank.unpack(layer.dtype), view.values), -2)
        mask = None
        if q_len > 1:
            from torch.nn.attention.bias import causal_lower_right
            mask = causal_lower_right(q_len, view.length)
        output = torch.nn.functional.scaled_dot_product_attention(query, keys, values, attn_mask=mask,
                                                                  enable_gqa=True, scale=self.scaling)
    else:
        self._direct_kv_calls += 1
        if verify:
            self._direct_kv_verify_calls += 1
        elif q_len > 1:
            self._direct_kv_prefill_calls += 1
        self._direct_kv_last_length = view.length
    layer.compact_residual()
    output = output.transpose(1, 2).reshape(*shape, -1).contiguous()
    return self.o_proj(output * torch.sigmoid(gate)), None


def configure_compressed_kv_attention(model, enabled=True, prefill=None):
    """Patch every ``Qwen3_5Attention`` (reference ``:85-95``).

    Prefill chunks over a packed history go to the packed prefill kernel
    instead of dequantize + SDPA: by default (``prefill=None``) 16..4096
    tokens at head_dim 128 / 256 and 16..1024 at head_dim 64, where each
    kernel is the faster; 16..4096 with ``prefill=True``, none with
    ``prefill=False``.
    """
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5Attention
    for module in model.modules():
        if type(module) is not Qwen3_5Attention:
            continue
        if not hasattr(module, '_direct_kv_original'):
            module._direct_kv_original = module.forward
            module._direct_kv_calls = module._direct_kv_last_length = 0
            module._direct_kv_verify_calls = module._direct_kv_prefill_calls = 0
            module.forward = MethodType(_forward, module)
        module._direct_kv_enabled = bool(enabled)
        default = 4096 if getattr(module, 'head_dim', 0) >= 128 else 1024
        module._direct_kv_prefill_max = default if prefill is None else (4096 if prefill else 0)
    return compressed_kv_info(model)


def compressed_kv_info(model):
    """Dispatch counters (reference ``:98-103``)."""
    modules = [m for m in model.modules() if hasattr(m, '_direct_kv_enabled')]
    return dict(backend=BACKEND, configured_layers=sum(m._direct_kv_enabled for m in modules),
                direct_decode_calls=sum(m._direct_kv_calls for m in modules),
                direct_verify_calls=sum(getattr(m, '_direct_kv_verify_calls', 0) for m in modules),
                direct_prefill_calls=sum(getattr(m, '_direct_kv_prefill_calls', 0) for m in modules),
                longest_decode=max((m._direct_kv_last_length for m in modules), default=0),
                fallback='SDPA for a first chunk (no packed history), chunks of 5..15 tokens or '
                         'above the prefill limit, arbitrary masks, unsupported shapes or precision')
