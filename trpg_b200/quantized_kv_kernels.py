"""Drop-in for ``models/quantized_kv_kernels.py``: affine pack/unpack.

Same call signatures as the reference (``pack(rows, bits)`` at
``models/quantized_kv_kernels.py:39`` and ``unpack(data, meta, bits, dtype)``
at ``:50``), backed by hand-written sm_100a CUDA (``ckv_pack_rows`` /
``ckv_unpack_rows`` in ``include/ckv.h``).  CUDA tensors only, as in the
reference (``models/quantized_kv.py:16,29`` only routes CUDA tensors here).

``pack`` defaults to round-half-to-even with IEEE division, which reproduces
the reference CPU quantizer (``models/quantized_kv.py:19-25``) bit for bit;
``rounding='half_up'`` follows the tie rule of the reference Triton kernel
(``floor(t + 0.5)``, ``models/quantized_kv_kernels.py:14``) with IEEE
division.  It is pinned to fixtures that the reference's Triton kernel
produced under the Triton interpreter on CPU, whose fp32 divide is IEEE;
the same kernel compiled for a GPU may lower that divide differently and
so differ where a quotient lies within an ulp of a rounding boundary.  No
fixture from the compiled kernel exists: the reference's package install
ships only its ``src/`` tree, so its ``models/`` kernels never reach a GPU
host.  ``unpack`` rounds one fused multiply-add to ``dtype`` like the
reference CUDA unpack (``:36``).
"""
from __future__ import annotations

import torch

from ._native import ROUNDING, ops

DEFAULT_ROUNDING = 'half_even'


def pack(rows: torch.Tensor, bits: int, rounding: str = DEFAULT_ROUNDING):
    """rows [..., G] (G = 64 or 128, bf16/fp16) -> (codes uint8 [..., G*bits/8], meta f32 [..., 2])."""
    if not rows.is_cuda:
        raise RuntimeError('trpg_b200 pack runs on CUDA tensors only')
    return ops().pack_rows(rows, int(bits), ROUNDING[rounding])


def unpack(data: torch.Tensor, meta: torch.Tensor, bits: int, dtype: torch.dtype) -> torch.Tensor:
    """codes + (scale, low) -> values of ``dtype`` with the last dim expanded for Q4."""
    if not data.is_cuda:
        raise RuntimeError('trpg_b200 unpack runs on CUDA tensors only')
    return ops().unpack_rows(data, meta, int(bits), dtype)
