"""Attention parity on the GPU: the B200 kernels against the oracle
(dequantize + cat + softmax attention) and the reference's own outputs."""
import copy
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import ckv_oracle as O
from tests._util import gpu_cache_state, max_abs, to_torch

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / 'golden'
# Reference test tolerance (tests/test_compressed_kv_attention.py:76) and the
# acceptance bound: max-abs 2e-2 / rel 1e-2 against dequantize + SDPA.
RTOL, ATOL, MAX_ABS = .025, .004, 2e-2


@pytest.fixture(scope='module', autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip('CUDA required')
    from trpg_b200 import _native
    _native.load()


def run(q, view, scale):
    from trpg_b200.compressed_kv_attention import compressed_kv_decode, compressed_kv_verify
    with torch.inference_mode():
        if q.shape[2] == 1:
            return compressed_kv_decode(q, view, scale)
        return compressed_kv_verify(q, view, scale)


def check(actual, expected):
    a = actual.float().cpu().numpy()
    assert np.isfinite(a).all()
    assert max_abs(a, expected) <= MAX_ABS
    np.testing.assert_allclose(a, expected, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize('case', sorted({k[:-5] for k in np.load(GOLDEN / 'attention.npz').files
                                         if k.endswith('_spec')}))
def test_matches_reference_outputs_and_oracle(case, both_rules):
    a = np.load(GOLDEN / 'attention.npz')
    bits, hkv, hq, length, dim, n, seed, outliers = (int(x) for x in a[f'{case}_spec'])
    dtype, scale = str(a[f'{case}_dtype']), float(a[f'{case}_scale'])
    layer, view, olayer = gpu_cache_state(seed, hkv, length, dim, bits, n, dtype, bool(outliers))
    qn = O.seeded_normal(seed + 2, (1, hq, n, dim), dtype)
    out = run(to_torch(qn, dtype), view, scale)
    assert out is not None and out.shape == (1, hq, n, dim) and out.dtype == view.keys.dtype
    check(out, a[f'{case}_output'])                      # the reference itself
    check(out, O.decode_reference(qn, olayer, scale))    # oracle, fused dequant


@pytest.mark.parametrize('bits', [8, 4])
@pytest.mark.parametrize('residual', [1, 16, 64, 128, 129, 255, 256, 300])
def test_residual_window_sweep(bits, residual, both_rules):
    """Hand-built views: any residual length next to 3 packed blocks."""
    from trpg_b200.quantized_kv import QuantizedAttentionLayer, QuantizedKVView
    k = O.seeded_normal(5, (1, 4, 384 + residual, 256))
    v = O.seeded_normal(6, (1, 4, 384 + residual, 256))
    layer = QuantizedAttentionLayer(bits)
    with torch.inference_mode():
        layer.key_bank.reserve(3, to_torch(k[:, :, :1], 'bfloat16'), 1, 4, 256)
        layer.value_bank.reserve(3, to_torch(k[:, :, :1], 'bfloat16'), 1, 4, 256)
        layer.key_bank.append(to_torch(k[:, :, :384], 'bfloat16'))
        layer.value_bank.append(to_torch(v[:, :, :384], 'bfloat16'))
    keys, values = to_torch(k[:, :, 384:], 'bfloat16'), to_torch(v[:, :, 384:], 'bfloat16')
    view = QuantizedKVView(layer.key_bank.data, layer.key_bank.meta, layer.value_bank.data,
                           layer.value_bank.meta, 384, keys, values, bits, 384 + residual)
    ol = O.OracleLayer(bits)
    ol._append_bank(k[:, :, :384], v[:, :, :384])
    ol.keys, ol.values, ol.length = k[:, :, 384:], v[:, :, 384:], 384 + residual
    q = O.seeded_normal(7, (1, 16, 1, 256))
    check(run(to_torch(q, 'bfloat16'), view, 1 / 16), O.decode_reference(q, ol, 1 / 16))


@pytest.mark.parametrize('nq', [2, 3, 4])
@pytest.mark.parametrize('bits', [8, 4])
def test_verify_lower_right_causal(nq, bits, both_rules):
    layer, view, ol = gpu_cache_state(40 + nq, 4, 1000 + 77 * nq, 256, bits, nq)
    q = O.seeded_normal(50 + nq, (1, 16, nq, 256))
    check(run(to_torch(q, 'bfloat16'), view, 1 / 16), O.decode_reference(q, ol, 1 / 16))


def test_verify_sixteen_rows_with_fp16_and_d128(both_rules):
    layer, view, ol = gpu_cache_state(61, 2, 2222, 128, 8, 2, 'float16')
    q = O.seeded_normal(62, (1, 16, 2, 128), 'float16')      # 8 groups x 2 queries = 16 rows
    check(run(to_torch(q, 'float16'), view, 128 ** -.5), O.decode_reference(q, ol, 128 ** -.5))


def test_large_logits_stay_finite_and_unsupported_inputs_return_none(both_rules):
    layer, view, ol = gpu_cache_state(71, 2, 512, 64, 4)
    keys = view.keys
    q = keys[..., :1, :].repeat_interleave(2, dim=1) * 80
    expected = O.decode_reference(q.float().cpu().numpy(), ol, .125)
    check(run(q, view, .125), expected)
    from trpg_b200.compressed_kv_attention import compressed_kv_decode
    with torch.inference_mode():
        assert compressed_kv_decode(q.expand(2, -1, -1, -1), view, .125) is None
        assert compressed_kv_decode(q.expand(-1, -1, 2, -1), view, .125) is None
        assert compressed_kv_decode(q.float(), view, .125) is None
        assert compressed_kv_decode(q, view, float('nan')) is None
    with torch.enable_grad():
        assert compressed_kv_decode(q, view, .125) is None


@pytest.mark.parametrize('bank', ['value', 'key'])
def test_fused_dequant_rounding_known_answer(bank):
    """tests/test_compressed_kv_attention.py:124-157 of the reference: crafted
    metadata where a fused and a split multiply-add round to opposite bf16
    neighbours (2.109375 vs 2.125); the kernel must follow the fused one."""
    from trpg_b200.quantized_kv import QuantizedAttentionLayer
    with torch.inference_mode():
        layer = QuantizedAttentionLayer(8)
        zero = torch.zeros(1, 1, 256, 64, device='cuda', dtype=torch.bfloat16)
        layer.update(zero, zero)
        b = getattr(layer, bank + '_bank')
        if bank == 'value':
            b.data[:, :, :128].fill_(204)
            b.data[:, :, :128, :, -2] = 0
            b.data[:, :, :128, :, -1] = 255
            b.meta[:, :, :128, :, 0] = .020067401230335236
            b.meta[:, :, :128, :, 1] = -1.9765625
        else:
            b.data[:, :, 0, 0].fill_(204)
            b.data[:, :, 0, 0, 0] = 0
            b.data[:, :, 0, 0, 1] = 255
            b.meta[:, :, 0, 0, 0] = .020067401230335236
            b.meta[:, :, 0, 0, 1] = -1.9765625
            layer.keys[..., 0] = 2.125
            layer.value_bank.data[:, :, :128].zero_()
            layer.value_bank.meta[:, :, :128, :, 1] = 1.
        view = layer.append_for_attention(layer.keys[:, :, :1].clone(), layer.values[:, :, :1].clone())
        keys = torch.cat((layer.key_bank.unpack(zero.dtype), view.keys), -2)
        values = torch.cat((layer.value_bank.unpack(zero.dtype), view.values), -2)
        q = torch.zeros(1, 1, 1, 64, device='cuda', dtype=torch.bfloat16)
        if bank == 'key':
            q[..., 0] = 16
        expected = torch.nn.functional.scaled_dot_product_attention(q, keys, values)
        actual = run(q, view, .125)
    torch.testing.assert_close(actual[..., :1], expected[..., :1], rtol=0, atol=.002)


def test_batched_ragged_call_equals_per_sequence_calls(both_rules):
    from trpg_b200.compressed_kv_kernels import attention
    qs, views, want = [], [], []
    for i, length in enumerate((700, 1900, 2600, 3333, 5000)):
        layer, view, ol = gpu_cache_state(100 + i, 4, length, 256, 8)
        q = O.seeded_normal(200 + i, (1, 16, 1, 256))
        qs.append(to_torch(q, 'bfloat16'))
        views.append(view)
        want.append(O.decode_reference(q, ol, 1 / 16))
    with torch.inference_mode():
        outs = attention(qs, views, 1 / 16)
    for out, w in zip(outs, want):
        check(out, w)


@pytest.mark.parametrize('world', [2, 3, 8])
def test_split_kv_partials_combine_to_the_full_result(world, both_rules):
    from trpg_b200 import sharding
    from trpg_b200.compressed_kv_kernels import attention, combine
    layer, view, ol = gpu_cache_state(81, 4, 9000, 256, 4)
    q = to_torch(O.seeded_normal(82, (1, 16, 1, 256)), 'bfloat16')
    with torch.inference_mode():
        parts = [attention([q], [view], 1 / 16, partial=True,
                           ranges=[sharding.split_kv_range(view.packed_tokens // 128,
                                                           view.keys.shape[2], world, r)])[0]
                 for r in range(world)]
        out = combine(parts, torch.bfloat16).view(1, 16, 1, 256)
        full = attention([q], [view], 1 / 16)[0]
    torch.testing.assert_close(out, full, rtol=.01, atol=2e-3)


def test_decode_does_not_modify_the_view_and_reuses_across_lengths():
    layer, view, _ = gpu_cache_state(90, 2, 1025, 64, 8)
    before = [t.clone() for t in (view.keys, view.values, view.key_data, view.key_meta)]
    q = torch.randn(1, 4, 1, 64, device='cuda', dtype=torch.bfloat16)
    x = torch.randn(1, 2, 1, 64, device='cuda', dtype=torch.bfloat16)
    assert run(q, view, .125) is not None
    for t, b in zip((view.keys, view.values, view.key_data, view.key_meta), before):
        assert torch.equal(t, b)
    with torch.inference_mode():
        for _ in range(300):    # crosses a compaction boundary
            v = layer.append_for_attention(x, x)
            assert run(q, v, .125) is not None
            layer.compact_residual()
    assert layer.get_seq_length() == 1325


def test_long_decode_loop_never_gives_up_a_wait():
    """Thousands of decode launches through append / decode / compact (the
    bench's 32K-context step on 4 layers): no kernel may abort a wait.  An
    abort means a pipeline barrier lost track of its phase (it used to
    happen about once in 8000 launches when one team of warps ran a stage
    ahead of the other), and that call's output would be wrong."""
    from trpg_b200.compressed_kv_kernels import attention_error, decode
    from trpg_b200.quantized_kv import QuantizedAttentionLayer
    gen = torch.Generator(device='cuda').manual_seed(21)
    attention_error()   # clear anything left by earlier tests
    with torch.inference_mode():
        layers = []
        for _ in range(4):
            k = torch.randn(1, 4, 32767, 256, generator=gen, device='cuda').bfloat16()
            v = torch.randn(1, 4, 32767, 256, generator=gen, device='cuda').bfloat16()
            layer = QuantizedAttentionLayer(8)
            layer.update(k, v)
            layers.append(layer)
        q = torch.randn(64, 1, 16, 1, 256, generator=gen, device='cuda').bfloat16()
        kn = torch.randn(64, 1, 4, 1, 256, generator=gen, device='cuda').bfloat16()
        for step in range(2500):
            for layer in layers:
                view = layer.append_for_attention(kn[step % 64], kn[(step + 1) % 64])
                decode(q[step % 64], view, 1 / 16)
                layer.compact_residual()
        torch.cuda.synchronize()
    assert attention_error() == 0


def test_window_appends_in_place_and_keeps_earlier_views():
    """The exact window is written in place (no torch.cat per token).  It must
    equal the concatenation the reference keeps, views handed out earlier
    must not change, and a rolled-back snapshot must be appendable again."""
    from trpg_b200.quantized_kv import QuantizedAttentionLayer
    gen = torch.Generator(device='cuda').manual_seed(8)
    with torch.inference_mode():
        k0 = torch.randn(1, 2, 700, 128, generator=gen, device='cuda').bfloat16()
        layer = QuantizedAttentionLayer(8)
        layer.update(k0, -k0)
        ref_k, ref_v = layer.keys.clone(), layer.values.clone()
        views = []
        for step in range(300):        # crosses compactions
            x = torch.randn(1, 2, 1, 128, generator=gen, device='cuda').bfloat16()
            view = layer.append_for_attention(x, 2 * x)
            ref_k, ref_v = torch.cat((ref_k, x), -2), torch.cat((ref_v, 2 * x), -2)
            assert torch.equal(view.keys, ref_k) and torch.equal(view.values, ref_v)
            views.append((view.keys, view.keys.clone()))
            before = layer.keys.shape[-2]
            layer.compact_residual()
            drop = before - layer.keys.shape[-2]
            ref_k, ref_v = ref_k[..., drop:, :], ref_v[..., drop:, :]
        for live, copy in views:
            assert torch.equal(live, copy)
        # rollback: restore an earlier window view and append different tokens
        snap = (layer.keys, layer.values, layer.cumulative_length)
        y = torch.randn(1, 2, 1, 128, generator=gen, device='cuda').bfloat16()
        first = layer.append_for_attention(y, y).keys.clone()
        layer.keys, layer.values, layer.cumulative_length = snap
        z = torch.randn(1, 2, 1, 128, generator=gen, device='cuda').bfloat16()
        again = layer.append_for_attention(z, z)
        assert torch.equal(again.keys[..., :-1, :], first[..., :-1, :])
        assert torch.equal(again.keys[..., -1:, :], z)


@pytest.mark.parametrize('bits', [8, 4])
def test_folded_rule_follows_value_and_key_ranges_across_blocks(bits):
    """Blocks whose value and key magnitudes differ by up to 10^6 from one
    another (and a block of exact zeros): the folded rule's range exponent
    moves with them.  The folded rule never rounds a dequantized value, so
    the reference here is dequantize + SDPA without that rounding (at |v| ~
    3000 the bf16 rounding of the other rule alone moves outputs by ~1)."""
    from trpg_b200 import compressed_kv_kernels as K
    from trpg_b200.quantized_kv import QuantizedAttentionLayer, QuantizedKVView
    blocks, resid = 24, 200
    k = O.seeded_normal(81, (1, 4, 128 * blocks + resid, 256))
    v = O.seeded_normal(82, (1, 4, 128 * blocks + resid, 256))
    for b in range(blocks):
        sl = slice(128 * b, 128 * (b + 1))
        v[:, :, sl] = O.round_to(v[:, :, sl] * np.float32(10.0 ** ((b % 7) - 3)), 'bfloat16')
        k[:, :, sl] = O.round_to(k[:, :, sl] * np.float32(2.0 ** ((b % 5) - 2)), 'bfloat16')
    v[:, :, 128 * 5:128 * 6] = 0
    layer = QuantizedAttentionLayer(bits)
    with torch.inference_mode():
        layer.key_bank.reserve(blocks, to_torch(k[:, :, :1], 'bfloat16'), 1, 4, 256)
        layer.value_bank.reserve(blocks, to_torch(k[:, :, :1], 'bfloat16'), 1, 4, 256)
        layer.key_bank.append(to_torch(k[:, :, :128 * blocks], 'bfloat16'))
        layer.value_bank.append(to_torch(v[:, :, :128 * blocks], 'bfloat16'))
    keys = to_torch(k[:, :, 128 * blocks:], 'bfloat16')
    values = to_torch(v[:, :, 128 * blocks:], 'bfloat16')
    view = QuantizedKVView(layer.key_bank.data, layer.key_bank.meta, layer.value_bank.data,
                           layer.value_bank.meta, 128 * blocks, keys, values, bits,
                           128 * blocks + resid)
    ol = O.OracleLayer(bits, dtype='float32')    # dequantized values not rounded to bf16
    ol._append_bank(k[:, :, :128 * blocks], v[:, :, :128 * blocks])
    ol.keys, ol.values, ol.length = k[:, :, 128 * blocks:], v[:, :, 128 * blocks:], 128 * blocks + resid
    q = O.seeded_normal(83, (1, 16, 1, 256))
    expected = O.decode_reference(q, ol, 1 / 16)
    err = {}
    old = K.dequant()
    try:
        for rule in ('exact', 'folded'):
            K.set_dequant(rule)
            out = run(to_torch(q, 'bfloat16'), view, 1 / 16).float().cpu().numpy()
            assert np.isfinite(out).all()
            err[rule] = max_abs(out, expected)
    finally:
        K.set_dequant(old)
    # Outputs average values of magnitude up to ~4000 with heavy cancellation;
    # a 16-bit rounding anywhere moves them by ~1e-4 of that magnitude.
    vmax = float(np.abs(v).max())
    assert err['folded'] <= 1e-3 * vmax, (err, vmax)
    assert err['folded'] <= 1.5 * err['exact'] + 1e-3, err
