"""B200-native compressed-KV attention (the Uyizi/trpg KV hot path).

Modules mirror the reference's own, with the same names and signatures:

* ``trpg_b200.quantized_kv_kernels``    -- ``pack`` / ``unpack``
* ``trpg_b200.compressed_kv_kernels``   -- ``decode`` (+ ``verify``,
  batched ``attention``, split-KV ``combine``)
* ``trpg_b200.quantized_kv``            -- the hybrid Q4/Q8 cache
* ``trpg_b200.compressed_kv_attention`` -- guards and the attention patch
* ``trpg_b200.mtp_verification_kernels`` -- request-local verify scope
* ``trpg_b200.sharding``                -- multi-GPU work partitioning
* ``trpg_b200.install``                 -- route the reference's kernel
  modules to this package

Kernels live in ``libtrpg_ckv.so`` (C ABI, ``include/ckv.h``) and are
registered as ``torch.ops.ckv``; build them with ``python -m trpg_b200.build``.
"""
from ._native import load as load_native  # noqa: F401

__all__ = ['load_native']
