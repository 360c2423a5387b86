"""Guarded packed prefill: lower-right causal attention of a query chunk.

Drop-in for ``models/compressed_prefill_attention.py:6-52``: the same
function name and signature, the same accept/reject set, ``None`` for a call
the kernel does not cover (the caller then runs dequantize + SDPA) and the
kernel's output otherwise.  The acceptance rules run in C++
(``torch.ops.ckv.attention_guarded``, the chunk route, which also serves the
decode and verify routes), next to the kernel they protect; only the plain
Python types of the view's fields are checked here.  Launch errors raise, and
a missing native library raises instead of returning ``None``.
"""
from __future__ import annotations

PREFILL_ROUTE = 2   # Route::kPrefill in trpg_b200/csrc/ckv_torch.cpp

_guarded = None


def compressed_kv_prefill(query, view, scale):
    """Lower-right causal attention of ``query`` [1, Hq, n, D] (16 <= n <= 4096)
    over the whole packed history plus the exact window, or ``None``.

    Call after appending the chunk (the window holds its n positions) and
    before ``compact_residual()``.  The caller must reject custom masks.
    """
    global _guarded
    length, bits, packed = view.length, view.bits, view.packed_tokens
    if (type(length) is not int or type(packed) is not int or type(bits) is not int
            or not isinstance(scale, (int, float)) or isinstance(scale, bool)):
        return None
    if _guarded is None:
        from ._native import ops
        _guarded = ops().attention_guarded
    return _guarded(query, view.key_data, view.key_meta, view.value_data, view.value_meta,
                    view.keys, view.values, packed, length, bits, float(scale), PREFILL_ROUTE)
