"""Packed prefill on the host: the public guard's CPU behaviour
(tests/test_compressed_prefill_attention.py:11-19) and the C ABI's argument
checks, which return before any CUDA call (these run without a GPU)."""
import ctypes
import sys
from unittest.mock import patch

import torch

from trpg_b200 import _native

from tests.test_zz_no_alloc import Seq

I32 = ctypes.c_int32
P, R, QLEN, D = 256, 48, 32, 64


class PrefillArgs(ctypes.Structure):
    """``ckv_prefill_args`` of include/ckv.h."""
    _fields_ = [('seq', Seq), ('heads_q', I32), ('heads_kv', I32), ('head_dim', I32),
                ('qlen', I32), ('bits', I32), ('dtype', I32), ('scale', ctypes.c_float)]


def _lib():
    lib = _native.library()
    lib.ckv_prefill.argtypes = [ctypes.POINTER(PrefillArgs), ctypes.c_void_p, ctypes.c_size_t,
                                ctypes.c_void_p]
    lib.ckv_prefill.restype = ctypes.c_int
    lib.ckv_prefill_workspace.argtypes = [ctypes.POINTER(PrefillArgs), ctypes.POINTER(ctypes.c_size_t)]
    lib.ckv_prefill_workspace.restype = ctypes.c_int
    return lib


def _args(**over):
    base = 0x10000000          # fake, aligned; validation reads no memory
    seq = Seq(base, QLEN * D, D, base, 2 * D * 128, D * 128, base, 2 * D * 2, D * 2,
              base, 512 * D, D, base, 512 * 2, 2, base, R * D, D, base, R * D, D,
              P, P + R, 0, P // 128, 0, R, base)
    for k, v in over.items():
        if hasattr(seq, k):
            setattr(seq, k, v)
    a = PrefillArgs(seq, 4, 2, D, QLEN, 8, 0, .125)
    for k, v in over.items():
        if k in dict(PrefillArgs._fields_):
            setattr(a, k, v)
    return a


def test_cpu_query_never_imports_or_launches_the_kernel():
    from trpg_b200.compressed_prefill_attention import compressed_kv_prefill
    from trpg_b200.quantized_kv import QuantizedKVView
    x = torch.randn(1, 1, 256, 64)
    view = QuantizedKVView(None, None, None, None, 128, x, x, 4, 384)
    with torch.inference_mode(), patch.dict(sys.modules, {'trpg_b200.compressed_prefill_kernels': None}):
        assert compressed_kv_prefill(x[:, :, :16], view, .125) is None


def test_prefill_rejects_bad_arguments_before_any_launch():
    lib = _lib()
    assert lib.ckv_prefill(None, None, 0, None) == 1
    bad = {
        'qlen': R + 1,                 # the window must hold the chunk
        'packed_tokens': 0,            # needs packed history
        'bits': 5,
        'heads_q': 3,                  # not a multiple of heads_kv
        'scale': float('nan'),
        'q_stride_pos': D + 4,         # rows not 16-byte aligned
        'keys': 0x10000008,            # residual base not 16-byte aligned
    }
    for k, v in bad.items():
        assert lib.ckv_prefill(ctypes.byref(_args(**{k: v})), None, 0, None) == 1, k
    assert lib.ckv_prefill(ctypes.byref(_args(head_dim=96)), None, 0, None) == 2
    assert lib.ckv_prefill(ctypes.byref(_args(resid_begin=8)), None, 0, None) == 2   # a shard


def test_short_chunks_split_the_history_and_need_a_workspace():
    """32 queries x 2 group heads = 1 tile per KV head, 2 CTAs: the history
    (256 packed tokens = 4 tiles of 64) splits 4 ways, one (o, m, l) record of
    D + 2 floats per split and output row.  Without a GPU the plan assumes
    148 SMs.  A missing workspace is refused before any launch."""
    lib = _lib()
    nbytes = ctypes.c_size_t()
    assert lib.ckv_prefill_workspace(ctypes.byref(_args()), ctypes.byref(nbytes)) == 0
    assert nbytes.value == 4 * (4 * QLEN) * (D + 2) * 4
    assert lib.ckv_prefill(ctypes.byref(_args()), None, 0, None) == 3
    # 1184 queries x 2 = 19 tiles per KV head, 38 CTAs: 3 splits by SM count,
    # but a 128-token history has only 2 tiles of 64, so 2.
    big = _args(qlen=1184, packed_tokens=128, length=128 + 1200, unit_end=1, resid_end=1200)
    assert lib.ckv_prefill_workspace(ctypes.byref(big), ctypes.byref(nbytes)) == 0
    assert nbytes.value == 2 * (4 * 1184) * (D + 2) * 4
    # 4096 queries x 2 = 64 tiles x 2 heads = 128 CTAs fill 86% of a wave, and
    # 2..4 splits fill 256/296, 384/444, 512/592 just the same: no split.
    full = _args(qlen=4096, length=P + 4096, resid_end=4096)
    assert lib.ckv_prefill_workspace(ctypes.byref(full), ctypes.byref(nbytes)) == 0
    assert nbytes.value == 0
    # 4 KV heads: 256 CTAs are 1.73 waves; 4 splits make 1024 CTAs, 7 waves
    # less 12 slots (99% full).
    wide = _args(qlen=4096, length=P + 4096, resid_end=4096, heads_q=8, heads_kv=4)
    assert lib.ckv_prefill_workspace(ctypes.byref(wide), ctypes.byref(nbytes)) == 0
    assert nbytes.value == 4 * (8 * 4096) * (D + 2) * 4


def test_install_routes_the_reference_prefill_kernel_module():
    """``install()`` maps the reference's ``compressed_prefill_kernels`` (whose
    ``prefill`` its guard imports, models/compressed_prefill_attention.py:46-51)
    to this package's, and ``uninstall()`` restores the previous entry."""
    from trpg_b200 import compressed_prefill_kernels, install
    name = 'refpkg_for_test.compressed_prefill_kernels'
    assert name not in sys.modules
    install.install('refpkg_for_test')
    try:
        assert sys.modules[name] is compressed_prefill_kernels
        assert callable(sys.modules[name].prefill)
    finally:
        install.uninstall('refpkg_for_test')
    assert name not in sys.modules


def test_patch_prefill_limits():
    """Prefill routing limits of the attention patch: by default 1024 tokens
    at head_dim 64 and 4096 at head_dim 256, 4096 with ``prefill=True``,
    none with ``prefill=False``."""
    from transformers import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5Attention
    from trpg_b200.compressed_kv_attention import compressed_kv_info, configure_compressed_kv_attention
    config = Qwen3_5TextConfig(hidden_size=128, intermediate_size=256, num_hidden_layers=1,
                               num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                               layer_types=['full_attention'])
    config._attn_implementation = 'sdpa'
    module = Qwen3_5Attention(config, 0)
    limits = []
    configure_compressed_kv_attention(module)
    limits.append(module._direct_kv_prefill_max)
    for prefill in (True, False):
        configure_compressed_kv_attention(module, prefill=prefill)
        limits.append(module._direct_kv_prefill_max)
    assert limits == [1024, 4096, 0]
    assert compressed_kv_info(module)['direct_prefill_calls'] == 0
    wide = Qwen3_5Attention(Qwen3_5TextConfig(hidden_size=128, intermediate_size=256,
                                              num_hidden_layers=1, num_attention_heads=4,
                                              num_key_value_heads=2, head_dim=256,
                                              layer_types=['full_attention']), 0)
    configure_compressed_kv_attention(wide)
    assert wide._direct_kv_prefill_max == 4096
