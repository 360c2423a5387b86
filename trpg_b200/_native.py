"""Loader for the in-tree native libraries.

``libtrpg_ckv.so`` holds the CUDA kernels behind the C ABI of
``include/ckv.h``; ``_ckv_torch.so`` registers them as ``torch.ops.ckv.*``.
There is no CPU implementation and no fallback: if either library is
missing, every op raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / 'libtrpg_ckv.so'
TORCH_LIB_PATH = PKG / '_ckv_torch.so'

# Symbols of include/ckv.h, in declaration order.
EXPORTS = ('ckv_status_string', 'ckv_last_error', 'ckv_version', 'ckv_pack_rows',
           'ckv_unpack_rows', 'ckv_pack_append', 'ckv_residual_append', 'ckv_attention_workspace',
           'ckv_attention_error', 'ckv_attention', 'ckv_attention_static',
           'ckv_combine_partials', 'ckv_prefill_workspace', 'ckv_prefill', 'ckv_prefill_error',
           'ckv_prefill_set_tensor_cores', 'ckv_exchange_bytes',
           'ckv_exchange_alloc', 'ckv_exchange_open', 'ckv_exchange_close', 'ckv_exchange_free',
           'ckv_exchange_combine', 'ckv_exchange_error')

ROUNDING = {'half_even': 0, 'half_up': 1}
DEQUANT_MODES = ('exact', 'folded')

_lib = None
_loaded = False
_dequant = 'exact'


def library() -> ctypes.CDLL:
    """The C-ABI library (ctypes handle)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f'{LIB_PATH.name} is not built; run `python -m trpg_b200.build`')
        _lib = ctypes.CDLL(str(LIB_PATH))
        _lib.ckv_status_string.restype = ctypes.c_char_p
        _lib.ckv_last_error.restype = ctypes.c_char_p
        _lib.ckv_exchange_bytes.restype = ctypes.c_size_t
        _lib.ckv_exchange_bytes.argtypes = [ctypes.c_int, ctypes.c_int64, ctypes.c_int]
        _lib.ckv_exchange_alloc.argtypes = [ctypes.c_int, ctypes.c_int64, ctypes.c_int,
                                            ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]
        _lib.ckv_exchange_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
        _lib.ckv_exchange_close.argtypes = [ctypes.c_void_p]
        _lib.ckv_exchange_free.argtypes = [ctypes.c_void_p]
        _lib.ckv_exchange_error.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
    return _lib


def load() -> None:
    """Register ``torch.ops.ckv``; raises ImportError when not built."""
    global _loaded
    if _loaded:
        return
    library()
    if not TORCH_LIB_PATH.exists():
        raise ImportError(f'{TORCH_LIB_PATH.name} is not built; run `python -m trpg_b200.build`')
    torch.ops.load_library(str(TORCH_LIB_PATH))
    _loaded = True
    set_dequant(os.environ.get('TRPG_CKV_DEQUANT', 'exact'))
    set_prefill_tensor_cores(int(os.environ.get('TRPG_CKV_PREFILL_TC', '2')))


_prefill_tc = 2


def set_prefill_tensor_cores(mode: int) -> None:
    """Packed-prefill kernel at head_dim 128 / 256, process-wide: 0 mma.sync,
    1 tcgen05 with its phases in order, 2 tcgen05 pipelined (producer warps
    dequantize ahead, two logit buffers)."""
    global _prefill_tc
    mode = int(mode)
    if library().ckv_prefill_set_tensor_cores(mode) != 0:
        raise ValueError(f'prefill kernel mode must be 0, 1 or 2, not {mode}')
    _prefill_tc = mode


def prefill_tensor_cores() -> int:
    return _prefill_tc


def set_dequant(mode: str) -> str:
    """Dequantization rule of the attention ops ('exact' or 'folded'); returns
    the previous one.  See ``compressed_kv_kernels.set_dequant``."""
    global _dequant
    if mode not in DEQUANT_MODES:
        raise ValueError(f'dequantization rule must be one of {DEQUANT_MODES}, not {mode!r}')
    load()
    torch.ops.ckv.set_dequant(DEQUANT_MODES.index(mode))
    old, _dequant = _dequant, mode
    return old


def dequant() -> str:
    load()
    return _dequant


def ops():
    load()
    return torch.ops.ckv
