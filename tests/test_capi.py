"""The C-ABI library loads, exports every declared symbol and validates its
arguments on the host (no kernel launches: these run without a GPU)."""
import ctypes
import re
from pathlib import Path

import pytest

from trpg_b200 import _native

HEADER = Path(__file__).resolve().parents[1] / 'include' / 'ckv.h'


def declared_functions():
    text = re.sub(r'/\*.*?\*/', '', HEADER.read_text(), flags=re.S)
    names = re.findall(r'^\s*(?:const\s+)?\w+\s*\*?\s*(ckv_\w+)\s*\(', text, flags=re.M)
    return [n for n in names if n != 'ckv_partial_row']


def test_header_and_loader_agree():
    assert sorted(declared_functions()) == sorted(_native.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = _native.library()
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_version_and_status_strings():
    lib = _native.library()
    assert lib.ckv_version() >> 16 == 1
    assert lib.ckv_status_string(0) == b'ok'
    assert b'unsupported' in lib.ckv_status_string(2)


def test_pack_rows_rejects_bad_arguments_before_any_launch():
    lib = _native.library()
    lib.ckv_pack_rows.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int,
                                  ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                  ctypes.c_void_p]
    bad_group = lib.ckv_pack_rows(None, 0, 4, 96, 8, 0, None, None, None)
    bad_bits = lib.ckv_pack_rows(None, 0, 4, 64, 5, 0, None, None, None)
    null_ptr = lib.ckv_pack_rows(None, 0, 4, 64, 8, 0, None, None, None)
    empty = lib.ckv_pack_rows(None, 0, 0, 64, 8, 0, None, None, None)
    assert (bad_group, bad_bits, null_ptr, empty) == (1, 1, 1, 0)


def test_attention_rejects_null_and_oversized_requests():
    lib = _native.library()
    lib.ckv_attention.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    assert lib.ckv_attention(None, None, 0, None) == 1


def test_torch_ops_register_without_cuda():
    _native.load()
    import torch
    for op in ('pack_rows', 'unpack_rows', 'pack_append', 'attention', 'combine_partials', 'decode',
               'attention_error', 'prefill'):
        assert hasattr(torch.ops.ckv, op)


def test_cpu_tensors_raise_instead_of_falling_back():
    import torch
    from trpg_b200 import quantized_kv_kernels as Q
    with pytest.raises(RuntimeError):
        Q.pack(torch.zeros(4, 64, dtype=torch.bfloat16), 8)


def test_exchange_sizes_and_arguments_are_checked_on_the_host():
    lib = _native.library()
    rows, d = 16, 256
    want = 256 + 2 * 2 * rows * (d + 2) * 8
    assert lib.ckv_exchange_bytes(2, rows, d) == (want + 255) // 256 * 256
    assert lib.ckv_exchange_bytes(0, rows, d) == 0
    assert lib.ckv_exchange_bytes(9, rows, d) == 0           # above CKV_EXCHANGE_MAX_WORLD
    assert lib.ckv_exchange_bytes(2, rows, 255) == 0         # odd head_dim
    lib.ckv_exchange_combine.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                         ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p,
                                         ctypes.c_void_p]
    assert lib.ckv_exchange_combine(None, rows, d, None, 2, 0, 3, 0, 0, None, None) == 1
    bufs = (ctypes.c_void_p * 2)(256, 512)
    assert lib.ckv_exchange_combine(None, rows, d, bufs, 2, 2, 3, 0, 0, None, None) == 1  # rank
    assert lib.ckv_exchange_combine(None, rows, d, bufs, 2, 0, 4, 0, 0, None, None) == 1  # phases
    assert lib.ckv_exchange_combine(None, rows, d, bufs, 2, 0, 1, 0, 0, None, None) == 1  # no partial
