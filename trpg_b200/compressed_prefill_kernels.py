"""Packed prefill launcher over the B200 kernel (``ckv_prefill``).

Mirror of ``models/compressed_prefill_kernels.py:98-111``: ``prefill(query,
view, scale)`` runs after the public eligibility checks of
``trpg_b200.compressed_prefill_attention.compressed_kv_prefill`` and reads
the whole history once per CTA of 128 query rows (position-major over the G
query heads of a KV head), never materialising the dequantized history.  For
head_dim 128 and 256 the CTA's products run on tcgen05 (operands staged in
shared memory by producer warps that dequantize the codes, logits and output
accumulated in tensor memory); for head_dim 64, and when
``trpg_b200._native.set_prefill_tensor_cores(0)`` selects it, on mma.sync
(8 warps of 16 rows, ``BM`` in ``csrc/ckv_prefill.cu``).
"""
from __future__ import annotations

_prefill_op = None


def prefill(query, view, scale):
    """Lower-right causal attention of ``query`` [1, Hq, qlen, D] over the view.

    Returns a new [1, Hq, qlen, D] tensor in the query dtype.  Raises when the
    CUDA extension is missing or the launch fails.
    """
    global _prefill_op
    if _prefill_op is None:
        from ._native import ops
        _prefill_op = ops().prefill
    return _prefill_op(query, view.key_data, view.key_meta, view.value_data, view.value_meta,
                       view.keys, view.values, int(view.packed_tokens), int(view.length),
                       int(view.bits), float(scale))
