"""Pin the CPU oracle to fixtures produced by the reference itself.

The fixtures come from ``tests/golden/make_golden.py`` (reference CPU
``_pack``/``_unpack``, the reference Triton ``pack`` under the Triton
interpreter, and ``QuantizedAttentionLayer.update`` + SDPA).
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import ckv_oracle as O

GOLDEN = Path(__file__).resolve().parent / 'golden'
Q = np.load(GOLDEN / 'quantizer.npz')
A = np.load(GOLDEN / 'attention.npz')
CASES = sorted({k[:-len('_spec')] for k in A.files if k.endswith('_spec')})


@pytest.mark.parametrize('bits', [8, 4])
@pytest.mark.parametrize('group', [128, 64])
def test_quantizer_matches_reference_cpu_pack_bit_exact(bits, group):
    key = f'b{bits}_g{group}'
    codes, meta = O.pack_rows(Q[f'{key}_rows'], bits, 'half_even')
    np.testing.assert_array_equal(codes, Q[f'{key}_cpu_codes'])
    np.testing.assert_array_equal(meta.view(np.uint32), Q[f'{key}_cpu_meta'].view(np.uint32))


@pytest.mark.parametrize('bits', [8, 4])
@pytest.mark.parametrize('group', [128, 64])
def test_quantizer_matches_reference_triton_pack_bit_exact(bits, group):
    key = f'b{bits}_g{group}'
    codes, meta = O.pack_rows(Q[f'{key}_rows'], bits, 'half_up')
    np.testing.assert_array_equal(codes, Q[f'{key}_triton_codes'])
    np.testing.assert_array_equal(meta.view(np.uint32), Q[f'{key}_triton_meta'].view(np.uint32))


def test_the_two_reference_rounding_rules_really_differ_on_ties():
    diffs = sum(int((Q[f'b{b}_g{g}_cpu_codes'] != Q[f'b{b}_g{g}_triton_codes']).sum())
                for b in (8, 4) for g in (128, 64))
    assert diffs > 0


@pytest.mark.parametrize('bits', [8, 4])
@pytest.mark.parametrize('group', [128, 64])
def test_dequantizer_matches_reference_cpu_unpack_bit_exact(bits, group):
    key = f'b{bits}_g{group}'
    values = O.unpack_rows(Q[f'{key}_cpu_codes'], Q[f'{key}_cpu_meta'], bits, 'bfloat16', fused=False)
    np.testing.assert_array_equal(values.view(np.uint32), Q[f'{key}_cpu_unpack_bf16'].view(np.uint32))


def test_fused_dequant_known_answer():
    """Crafted values of tests/test_compressed_kv_attention.py:124-157 (reference):
    code 204 with scale 0.020067401230335236 and low -1.9765625 lands on
    2.109375 with one rounding and on 2.125 with a rounded product."""
    codes = np.array([[204, 0, 255]], np.uint8)
    meta = np.array([[0.020067401230335236, -1.9765625]], np.float32)
    fused = O.unpack_rows(codes, meta, 8, 'bfloat16', fused=True)
    split = O.unpack_rows(codes, meta, 8, 'bfloat16', fused=False)
    assert fused[0, 0] == np.float32(2.109375)
    assert split[0, 0] == np.float32(2.125)


@pytest.mark.parametrize('name', CASES)
def test_cache_state_and_attention_match_reference(name):
    bits, hkv, hq, length, dim, n, seed, outliers = (int(x) for x in A[f'{name}_spec'])
    dtype = str(A[f'{name}_dtype'])
    scale = float(A[f'{name}_scale'])
    layer, _, _ = O.cache_state(seed, hkv, length, dim, bits, n, dtype, outliers=bool(outliers))
    assert layer.packed_tokens == int(A[f'{name}_packed'])
    assert layer.keys.shape[2] == int(A[f'{name}_residual'])
    assert O.digest(layer.kd, layer.km, layer.vd, layer.vm) == str(A[f'{name}_bank_digest'])
    assert O.digest(layer.keys, layer.values) == str(A[f'{name}_residual_digest'])
    q = O.seeded_normal(seed + 2, (1, hq, n, dim), dtype)
    # The reference dequantizes on CPU with a separate multiply and add.
    got = O.decode_reference(q, layer, scale, fused=False)
    want = A[f'{name}_output']
    np.testing.assert_allclose(got, want, rtol=1e-2, atol=4e-3)


@pytest.mark.parametrize('name', ['c1_q8_l2048', 'q4_l2048', 'verify_q8_n4_l1500'])
def test_cpu_timing_path_matches_reference(name):
    """The torch-CPU restatement used for CPU timings reproduces the reference."""
    import torch
    from oracle import ckv_cpu_path as P
    bits, hkv, hq, length, dim, n, seed, outliers = (int(x) for x in A[f'{name}_spec'])
    dtype = str(A[f'{name}_dtype'])
    tdt = getattr(torch, dtype)
    _, k, v = O.cache_state(seed, hkv, length, dim, bits, n, dtype, outliers=bool(outliers))
    layer = P.CpuLayer(bits)
    kt, vt = torch.from_numpy(k).to(tdt), torch.from_numpy(v).to(tdt)
    layer.update(kt[:, :, :length - n], vt[:, :, :length - n])
    layer.append_for_attention(kt[:, :, length - n:], vt[:, :, length - n:])
    assert O.digest(layer.kd.numpy(), layer.km.numpy(), layer.vd.numpy(),
                    layer.vm.numpy()) == str(A[f'{name}_bank_digest'])
    q = torch.from_numpy(O.seeded_normal(seed + 2, (1, hq, n, dim), dtype)).to(tdt)
    out = P.attend(q, layer, float(A[f'{name}_scale'])).float().numpy()
    np.testing.assert_array_equal(out, A[f'{name}_output'])


@pytest.mark.parametrize('bits,nq,length', [(8, 1, 3000), (4, 4, 1500), (8, 3, 700)])
def test_chunked_oracle_equals_the_whole_history_oracle(bits, nq, length):
    """The bounded-memory attention used at full sizes agrees with the
    dequantize + cat + SDPA restatement, whole and as merged shards."""
    layer, _, _ = O.cache_state(31 + bits, 2, length, 64, bits, new_tokens=nq)
    q = O.seeded_normal(37, (1, 6, nq, 64))
    want = O.decode_reference(q, layer, .125)
    got = O.decode_reference_chunked(q, layer, .125, chunk=256)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-12)
    if nq == 1:
        cut = [0, 1024, 1300, layer.length]
        parts = [O.decode_reference_chunked(q, layer, .125, chunk=200, t0=a, t1=b)
                 for a, b in zip(cut, cut[1:])]
        merged = O.combine_partials(*zip(*parts))
        np.testing.assert_allclose(merged, want, rtol=0, atol=1e-12)


def test_fill_leaves_the_state_update_leaves():
    k = O.seeded_normal(41, (1, 2, 900, 64))
    v = O.seeded_normal(42, (1, 2, 900, 64))
    a, b = O.OracleLayer(8), O.OracleLayer(8)
    a.update(k, v)
    b.fill(k, v)
    assert O.digest(a.kd, a.km, a.vd, a.vm, a.keys, a.values) == \
        O.digest(b.kd, b.km, b.vd, b.vm, b.keys, b.values)
