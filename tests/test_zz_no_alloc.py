"""``ckv_attention_static``: attention through the C ABI with the library's own
scratch array instead of a caller workspace (include/ckv.h).

The GPU cases call the entry point through ctypes, twice in a row on one
stream, and compare each result with the workspace entry point
(``ckv_attention`` behind ``torch.ops.ckv``) on the same inputs.  The file
name sorts last so that it also runs after every other test has used the
device.
"""
import ctypes

import numpy as np
import pytest
import torch

from trpg_b200 import _native

from tests._util import gpu_cache_state

RTOL, ATOL = .025, .004
STATIC_BYTES = 4 << 20          # CKV_STATIC_SCRATCH_BYTES
CKV_ERR_INVALID, CKV_ERR_WORKSPACE = 1, 3
DTYPE = {torch.bfloat16: 0, torch.float16: 1}

I64, I32, VP = ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p


class Seq(ctypes.Structure):
    """``ckv_seq`` of include/ckv.h (strides in elements)."""
    _fields_ = [('query', VP), ('q_stride_head', I64), ('q_stride_pos', I64),
                ('key_data', VP), ('kd_stride_head', I64), ('kd_stride_unit', I64),
                ('key_meta', VP), ('km_stride_head', I64), ('km_stride_unit', I64),
                ('value_data', VP), ('vd_stride_head', I64), ('vd_stride_token', I64),
                ('value_meta', VP), ('vm_stride_head', I64), ('vm_stride_token', I64),
                ('keys', VP), ('rk_stride_head', I64), ('rk_stride_token', I64),
                ('values', VP), ('rv_stride_head', I64), ('rv_stride_token', I64),
                ('packed_tokens', I64), ('length', I64),
                ('unit_begin', I32), ('unit_end', I32), ('resid_begin', I32), ('resid_end', I32),
                ('out', VP)]


class AttnArgs(ctypes.Structure):
    """``ckv_attn_args`` of include/ckv.h."""
    _fields_ = [('seqs', ctypes.POINTER(Seq)), ('num_seqs', I32), ('heads_q', I32),
                ('heads_kv', I32), ('head_dim', I32), ('nq', I32), ('bits', I32), ('dtype', I32),
                ('scale', ctypes.c_float), ('partial', I32), ('flags', I32)]


def _lib():
    lib = _native.library()
    lib.ckv_attention_static.argtypes = [ctypes.POINTER(AttnArgs), VP]
    lib.ckv_attention_static.restype = ctypes.c_int
    lib.ckv_attention_workspace.argtypes = [ctypes.POINTER(AttnArgs), ctypes.POINTER(ctypes.c_size_t)]
    lib.ckv_attention_workspace.restype = ctypes.c_int
    return lib


def _seq(query, view, out):
    from trpg_b200.compressed_kv_kernels import _dense_rows, _inner_dense, _residual
    kd, km = _inner_dense(view.key_data), _inner_dense(view.key_meta)
    vd, vm = _dense_rows(view.value_data), _dense_rows(view.value_meta)
    rk, rv = _residual(view.keys), _residual(view.values)
    s = Seq(query.data_ptr(), query.stride(1), query.stride(2),
            kd.data_ptr(), kd.stride(1), kd.stride(2), km.data_ptr(), km.stride(1), km.stride(2),
            vd.data_ptr(), vd.stride(1), vd.stride(2), vm.data_ptr(), vm.stride(1), vm.stride(2),
            rk.data_ptr(), rk.stride(1), rk.stride(2), rv.data_ptr(), rv.stride(1), rv.stride(2),
            int(view.packed_tokens), int(view.length), 0, int(view.packed_tokens) // 128,
            0, int(view.keys.shape[2]), out.data_ptr())
    return s, (kd, km, vd, vm, rk, rv)     # keep any copies alive for the call


CKV_DEQUANT_FOLDED = 2


def _args(queries, views, outs, scale):
    from trpg_b200 import compressed_kv_kernels as K
    seqs, keep = zip(*(_seq(q, v, o) for q, v, o in zip(queries, views, outs)))
    arr = (Seq * len(seqs))(*seqs)
    q = queries[0]
    flags = CKV_DEQUANT_FOLDED if K.dequant() == 'folded' else 0   # the rule the torch ops use
    args = AttnArgs(arr, len(seqs), q.shape[1], views[0].keys.shape[1], q.shape[3], q.shape[2],
                    views[0].bits, DTYPE[q.dtype], scale, 0, flags)
    return args, (arr, keep)


def _static(queries, views, scale):
    outs = [torch.empty_like(q) for q in queries]
    args, keep = _args(queries, views, outs, scale)
    rc = _lib().ckv_attention_static(ctypes.byref(args), VP(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, _native.library().ckv_last_error()
    return outs, keep


def _batch(seed, lengths, bits, nq, dtype='bfloat16'):
    views, queries = [], []
    gen = torch.Generator().manual_seed(seed)
    for i, length in enumerate(lengths):
        _, view, _ = gpu_cache_state(seed + i, 4, length, 256, bits, new_tokens=nq, dtype=dtype)
        views.append(view)
        queries.append(torch.randn((1, 16, nq, 256), generator=gen).to('cuda', view.keys.dtype))
    return queries, views


def test_static_entry_rejects_null_args():
    assert _lib().ckv_attention_static(None, None) == CKV_ERR_INVALID


@pytest.mark.gpu
@pytest.mark.parametrize('bits,nq,lengths', [(8, 1, [32767]), (8, 1, [1500, 4097, 9000]),
                                             (4, 2, [3000, 700]), (8, 4, [5000])])
def test_static_matches_workspace_entry_twice(bits, nq, lengths, both_rules):
    from trpg_b200 import compressed_kv_kernels as K
    queries, views = _batch(11 * bits + nq, lengths, bits, nq)
    scale = 256 ** -.5
    with torch.inference_mode():
        first, keep1 = _static(queries, views, scale)
        second, keep2 = _static(queries, views, scale)        # no sync in between
        expected = K.attention(queries, views, scale)
        torch.cuda.synchronize()
    for a, b, e in zip(first, second, expected):
        e = e.float().cpu().numpy()
        np.testing.assert_allclose(a.float().cpu().numpy(), e, rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(b.float().cpu().numpy(), e, rtol=RTOL, atol=ATOL)
    assert _static_gave_up() == 0


def _static_gave_up():
    """The static array's give-up word, read through ckv_attention_error with
    no workspace (0: no bounded wait of the last static call ran out)."""
    lib = _native.library()
    lib.ckv_attention_error.argtypes = [VP, ctypes.POINTER(ctypes.c_int), VP]
    lib.ckv_attention_error.restype = ctypes.c_int
    flag = ctypes.c_int(-1)
    rc = lib.ckv_attention_error(None, ctypes.byref(flag),
                                 VP(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.ckv_last_error()
    return flag.value


@pytest.mark.gpu
def test_static_back_to_back_different_shapes():
    """A call with another shape right after one batch: tickets start at zero."""
    from trpg_b200 import compressed_kv_kernels as K
    qa, va = _batch(5, [2048, 6000], 8, 1)
    qb, vb = _batch(6, [4000], 4, 3)
    scale = 256 ** -.5
    with torch.inference_mode():
        out_a, ka = _static(qa, va, scale)
        out_b, kb = _static(qb, vb, scale)
        exp_a, exp_b = K.attention(qa, va, scale), K.attention(qb, vb, scale)
        torch.cuda.synchronize()
    for a, e in zip(out_a + out_b, exp_a + exp_b):
        np.testing.assert_allclose(a.float().cpu().numpy(), e.float().cpu().numpy(), rtol=RTOL, atol=ATOL)


@pytest.mark.gpu
def test_static_rejects_request_beyond_scratch():
    queries, views = _batch(7, [5000], 8, 4)
    q, v = queries[0], views[0]
    n = 64                                                    # one view, many sequences
    outs = [torch.empty_like(q) for _ in range(n)]
    args, keep = _args([q] * n, [v] * n, outs, 256 ** -.5)
    need = ctypes.c_size_t()
    assert _lib().ckv_attention_workspace(ctypes.byref(args), ctypes.byref(need)) == 0
    assert need.value > STATIC_BYTES
    rc = _lib().ckv_attention_static(ctypes.byref(args), VP(torch.cuda.current_stream().cuda_stream))
    assert rc == CKV_ERR_WORKSPACE
    assert b'static buffer' in _native.library().ckv_last_error()
