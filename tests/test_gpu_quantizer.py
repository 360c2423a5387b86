"""Quantizer parity on the GPU: bit-exact against the oracle and the
reference's own fixtures (codes and scales, both rounding rules)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import ckv_oracle as O
from tests._util import bank_arrays, gpu_cache_state, to_torch

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / 'golden'


@pytest.fixture(scope='module', autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip('CUDA required')
    from trpg_b200 import _native
    _native.load()


@pytest.mark.parametrize('bits', [8, 4])
@pytest.mark.parametrize('group', [128, 64])
@pytest.mark.parametrize('rounding', ['half_even', 'half_up'])
def test_pack_matches_reference_fixtures_bit_exact(bits, group, rounding):
    from trpg_b200.quantized_kv_kernels import pack
    q = np.load(GOLDEN / 'quantizer.npz')
    key = f'b{bits}_g{group}'
    rows = to_torch(q[f'{key}_rows'], 'bfloat16')
    codes, meta = pack(rows, bits, rounding)
    tag = 'cpu' if rounding == 'half_even' else 'triton'
    np.testing.assert_array_equal(codes.cpu().numpy(), q[f'{key}_{tag}_codes'])
    np.testing.assert_array_equal(meta.cpu().numpy().view(np.uint32),
                                  q[f'{key}_{tag}_meta'].view(np.uint32))


@pytest.mark.parametrize('dtype', ['bfloat16', 'float16'])
@pytest.mark.parametrize('bits', [8, 4])
def test_pack_unpack_bit_exact_on_large_seeded_rows(dtype, bits):
    from trpg_b200.quantized_kv_kernels import pack, unpack
    rows = O.seeded_normal(77 + bits, (4096, 128), dtype) * np.float32(3)
    rows = O.round_to(rows, dtype)
    for rounding in ('half_even', 'half_up'):
        codes, meta = pack(to_torch(rows, dtype), bits, rounding)
        want_c, want_m = O.pack_rows(rows, bits, rounding)
        np.testing.assert_array_equal(codes.cpu().numpy(), want_c)
        np.testing.assert_array_equal(meta.cpu().numpy().view(np.uint32), want_m.view(np.uint32))
        out = unpack(codes, meta, bits, getattr(torch, dtype)).float().cpu().numpy()
        want = O.unpack_rows(want_c, want_m, bits, dtype, fused=True)
        np.testing.assert_array_equal(out.view(np.uint32), want.view(np.uint32))


def test_unpack_known_answer_single_rounding():
    from trpg_b200.quantized_kv_kernels import unpack
    codes = torch.tensor([[204, 0, 255] + [0] * 61], dtype=torch.uint8, device='cuda')
    meta = torch.tensor([[0.020067401230335236, -1.9765625]], device='cuda')
    out = unpack(codes, meta, 8, torch.bfloat16).float().cpu()
    assert out[0, 0].item() == 2.109375


@pytest.mark.parametrize('case', ['c1_q8_l2048', 'q4_l2048', 'q8_fp16_l1000_d128',
                                  'q4_l4097_d64_gqa3', 'q8_outliers_l3000', 'verify_q8_n4_l1500'])
def test_gpu_cache_banks_match_reference_digests(case):
    """The direct-to-slab append produces the reference CPU quantizer's bytes."""
    a = np.load(GOLDEN / 'attention.npz')
    bits, hkv, hq, length, dim, n, seed, outliers = (int(x) for x in a[f'{case}_spec'])
    dtype = str(a[f'{case}_dtype'])
    layer, view, olayer = gpu_cache_state(seed, hkv, length, dim, bits, n, dtype, bool(outliers))
    assert view.packed_tokens == int(a[f'{case}_packed'])
    assert O.digest(*bank_arrays(layer)) == str(a[f'{case}_bank_digest'])


@pytest.mark.parametrize('rounding', ['half_even', 'half_up'])
def test_growth_across_slabs_keeps_history_and_matches_oracle(rounding):
    """Several compactions across the 32-unit key slab boundary."""
    from trpg_b200.quantized_kv import QuantizedAttentionLayer
    k = O.seeded_normal(91, (1, 2, 4500, 64))
    v = O.seeded_normal(92, (1, 2, 4500, 64))
    layer = QuantizedAttentionLayer(8, rounding)
    ol = O.OracleLayer(8, rounding)
    pos = 0
    with torch.inference_mode():
        for chunk in (1000, 1000, 1000, 1000, 300, 200):
            layer.update(to_torch(k[:, :, pos:pos + chunk], 'bfloat16'),
                         to_torch(v[:, :, pos:pos + chunk], 'bfloat16'))
            ol.update(k[:, :, pos:pos + chunk], v[:, :, pos:pos + chunk])
            pos += chunk
    assert layer.key_bank.data.shape[2] == 64      # grew past one 32-unit slab
    got = bank_arrays(layer)
    for g, w in zip(got, (ol.kd, ol.km, ol.vd, ol.vm)):
        np.testing.assert_array_equal(g.view(np.uint8), w.view(np.uint8))
