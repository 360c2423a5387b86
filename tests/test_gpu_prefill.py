"""Packed prefill parity on the GPU: ``compressed_kv_prefill`` (the B200
``ckv_prefill`` kernels: tcgen05 and mma.sync for head_dim 128 / 256) against
the oracle's dequantize + cat + lower-right
causal softmax attention, on the reference's own cases
(tests/test_compressed_prefill_attention.py:26-53) and the edges around them.
"""
import numpy as np
import pytest
import torch

from oracle import ckv_oracle as O
from tests._util import gpu_cache_state, max_abs, to_torch

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures('both_prefill_kernels')]
# Reference test tolerance (tests/test_compressed_prefill_attention.py:49)
# and the acceptance bound, max-abs 2e-2 against dequantize + SDPA.
RTOL, ATOL, MAX_ABS = .03, .004, 2e-2


@pytest.fixture(scope='module', autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip('CUDA required')
    from trpg_b200 import _native
    _native.load()


def prefill(q, view, scale):
    from trpg_b200.compressed_prefill_attention import compressed_kv_prefill
    with torch.inference_mode():
        return compressed_kv_prefill(q, view, scale)


def check(actual, expected):
    assert actual is not None
    a = actual.float().cpu().numpy()
    assert np.isfinite(a).all()
    assert max_abs(a, expected) <= MAX_ABS
    np.testing.assert_allclose(a, expected, rtol=RTOL, atol=ATOL)


def query(seed, heads, qlen, dim, dtype):
    """[1, heads, qlen, D] as the transpose of [1, qlen, heads, D] (strided)."""
    q = O.seeded_normal(seed, (1, qlen, heads, dim), dtype)
    return q.transpose(0, 2, 1, 3), to_torch(q, dtype).transpose(1, 2)


# (bits, history, qlen, D, dtype): incomplete query tiles and residual/packed
# transition points, 6 query heads over 2 KV heads.
REFERENCE_CASES = [(4, 257, 16, 64, 'bfloat16'), (8, 385, 17, 128, 'float16'),
                   (4, 1025, 63, 256, 'bfloat16'), (8, 4096, 129, 256, 'bfloat16')]


@pytest.mark.parametrize('bits,history,qlen,dim,dtype', REFERENCE_CASES)
def test_q4_q8_exact_residual_causal_and_noncontiguous_queries(bits, history, qlen, dim, dtype):
    layer, view, ol = gpu_cache_state(104 + history, 2, history + qlen, dim, bits, qlen, dtype)
    qn, qt = query(7 + qlen, 6, qlen, dim, dtype)
    assert not qt.is_contiguous()
    scale = dim ** -.5
    check(prefill(qt, view, scale), O.decode_reference(qn, ol, scale, causal_lower_right=True))
    # Current attention keeps the exact residual until the caller compacts.
    assert layer.keys.shape[2] == view.keys.shape[2]
    assert layer.key_bank.units * 128 == view.packed_tokens


@pytest.mark.parametrize('bits,groups,qlen,dim,dtype', [
    (8, 16, 160, 128, 'float16'), (4, 1, 700, 64, 'bfloat16'),
    (8, 4, 333, 256, 'bfloat16'), (4, 8, 250, 128, 'float16')])
def test_group_sizes_dtypes_and_a_long_chunk(bits, groups, qlen, dim, dtype):
    hkv = 2
    layer, view, ol = gpu_cache_state(200 + groups, hkv, 1536 + qlen, dim, bits, qlen, dtype)
    qn, qt = query(300 + groups, hkv * groups, qlen, dim, dtype)
    check(prefill(qt.contiguous(), view, dim ** -.5),
          O.decode_reference(qn, ol, dim ** -.5, causal_lower_right=True))


def test_chunk_after_a_long_residual_window():
    """A window much longer than the chunk: rows see earlier window tokens too."""
    layer, view, ol = gpu_cache_state(401, 2, 2048, 128, 8, 16)
    from trpg_b200.quantized_kv import QuantizedAttentionLayer
    assert isinstance(layer, QuantizedAttentionLayer)
    qn, qt = query(402, 4, 16, 128, 'bfloat16')
    assert view.keys.shape[2] >= 16
    check(prefill(qt, view, 128 ** -.5), O.decode_reference(qn, ol, 128 ** -.5, causal_lower_right=True))


def test_large_logits_and_unsupported_inputs():
    layer, view, ol = gpu_cache_state(71, 1, 256 + 32, 64, 8, 32)
    q = (view.keys * 40).contiguous()
    expected = O.decode_reference(q.float().cpu().numpy(), ol, .125, causal_lower_right=True)
    out = prefill(q, view, .125)
    assert torch.isfinite(out).all()
    check(out, expected)
    for bad_q in (q[:, :, :15], q.float(), q.expand(2, -1, -1, -1)):
        assert prefill(bad_q, view, .125) is None
    assert prefill(q, view._replace(packed_tokens=0), .125) is None
    assert prefill(q, view, float('nan')) is None
    assert prefill(q, view._replace(keys=view.keys[:, :, :16]), .125) is None
    with torch.enable_grad():
        from trpg_b200.compressed_prefill_attention import compressed_kv_prefill
        assert compressed_kv_prefill(q, view, .125) is None


def test_growing_lengths_and_slab_strides():
    """Histories that grow the slab capacity (strided banks) in one process."""
    for history in (4096, 4224, 8320):
        layer, view, ol = gpu_cache_state(history, 2, history + 33, 64, 8, 33)
        qn, qt = query(history + 1, 4, 33, 64, 'bfloat16')
        check(prefill(qt, view, .125), O.decode_reference(qn, ol, .125, causal_lower_right=True))


def test_prefill_then_decode_on_the_same_layer():
    """The caller's sequence: append the chunk, prefill, compact, then decode."""
    from trpg_b200.compressed_kv_attention import compressed_kv_decode
    layer, view, ol = gpu_cache_state(501, 2, 1000 + 64, 128, 4, 64)
    qn, qt = query(502, 4, 64, 128, 'bfloat16')
    check(prefill(qt, view, 128 ** -.5), O.decode_reference(qn, ol, 128 ** -.5, causal_lower_right=True))
    with torch.inference_mode():
        layer.compact_residual()
        ol.compact_residual()
        k = O.seeded_normal(503, (1, 2, 1, 128))
        v = O.seeded_normal(504, (1, 2, 1, 128))
        dview = layer.append_for_attention(to_torch(k, 'bfloat16'), to_torch(v, 'bfloat16'))
        ol.append_for_attention(k, v)
        q1 = O.seeded_normal(505, (1, 4, 1, 128))
        out = compressed_kv_decode(to_torch(q1, 'bfloat16'), dview, 128 ** -.5)
    check(out, O.decode_reference(q1, ol, 128 ** -.5))


def test_real_qwen_attention_routes_a_prefill_chunk_and_keeps_the_cache():
    """A second prefill chunk through the patched ``Qwen3_5Attention`` matches
    the unpatched module (dequantize + SDPA via the cache's ``update``) and
    leaves the same cache state (after the reference's real-attention test,
    tests/test_compressed_kv_attention.py:159-187)."""
    import copy
    from transformers import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5Attention
    from torch.nn.attention.bias import causal_lower_right
    from trpg_b200.compressed_kv_attention import compressed_kv_info, configure_compressed_kv_attention
    from trpg_b200.quantized_kv import make_cache
    torch.manual_seed(0)
    config = Qwen3_5TextConfig(hidden_size=128, intermediate_size=256, num_hidden_layers=1,
                               num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                               layer_types=['full_attention'])
    config._attn_implementation = 'sdpa'
    module = Qwen3_5Attention(config, 0).cuda().bfloat16().eval().requires_grad_(False)
    configure_compressed_kv_attention(module, False)
    cache = make_cache(config, 'q8')
    n0, n1 = 384, 64
    x = torch.randn(1, n0 + n1, 128, device='cuda', dtype=torch.bfloat16)
    angle = torch.randn(1, n0 + n1, 64, device='cuda')
    pos = (angle.cos().bfloat16(), angle.sin().bfloat16())
    with torch.inference_mode():
        module(x[:, :n0], tuple(t[:, :n0] for t in pos), causal_lower_right(n0, n0), past_key_values=cache)
        ref, direct = copy.deepcopy(cache), copy.deepcopy(cache)
        hidden = x[:, n0:].contiguous()
        positions = tuple(t[:, n0:].contiguous() for t in pos)
        mask = causal_lower_right(n1, n0 + n1)
        expected, _ = module(hidden, positions, mask, past_key_values=ref)
        plain = copy.deepcopy(direct)
        configure_compressed_kv_attention(module, True, prefill=False)   # prefill routing off
        module(hidden, positions, mask, past_key_values=plain)
        assert compressed_kv_info(module)['direct_prefill_calls'] == 0
        configure_compressed_kv_attention(module, True)          # default: chunks up to 1024
        actual, weights = module(hidden, positions, mask, past_key_values=direct)
    assert weights is None
    torch.testing.assert_close(actual, expected, rtol=.03, atol=.004)
    info = compressed_kv_info(module)
    assert info['direct_prefill_calls'] == 1 and info['direct_verify_calls'] == 0
    assert direct.get_seq_length() == ref.get_seq_length()
    assert torch.equal(direct.layers[0].keys, ref.layers[0].keys)
    u = ref.layers[0].key_bank.units
    assert direct.layers[0].key_bank.units == u
    assert torch.equal(direct.layers[0].key_bank.data[:, :, :u], ref.layers[0].key_bank.data[:, :, :u])


@pytest.mark.parametrize('bits,dtype', [(8, 'bfloat16'), (4, 'float16')])
def test_short_history_long_chunk_splits_into_residual_only_shares(bits, dtype):
    """128 packed tokens under a 600-token chunk (one query head per KV head):
    10 CTAs split the history 2 ways, and the second share holds only
    residual tiles, so its early query rows see no token there (m = -inf in
    their partial records)."""
    layer, view, ol = gpu_cache_state(601 + bits, 2, 900, 64, bits, 600, dtype)
    assert view.packed_tokens == 128
    qn, qt = query(602, 2, 600, 64, dtype)
    check(prefill(qt, view, .125), O.decode_reference(qn, ol, .125, causal_lower_right=True))
