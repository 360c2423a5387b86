"""The model patch end to end on real attention modules (GPU).

Ports of the reference's integration tests to this package's patch
(``trpg_b200.compressed_kv_attention``) and cache (``trpg_b200.quantized_kv``):

* decode through a real ``Qwen3_5Attention``: the patched call matches the
  unpatched module, leaves the same cache, and custom masks / extra biases
  fall back to upstream with bit-identical outputs
  (tests/test_compressed_kv_attention.py:159-204);
* greedy generation through a tiny causal LM gives the same tokens with and
  without the patch, and every decode step takes the direct path (:206-229);
* a 2-token verify call inside the request scope takes the verify kernel,
  outside it falls back (models/mtp_generation.py:82-88);
* an append transaction rolled back over the in-place window leaves a cache
  that continues exactly like one that never took the appended tokens
  (models/hybrid_cache_transaction.py:39-56,105-119).
"""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


def _attention_module(heads=4, kv_heads=2, dim=64, hidden=128):
    from transformers import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5Attention
    config = Qwen3_5TextConfig(hidden_size=hidden, intermediate_size=256, num_hidden_layers=1,
                               num_attention_heads=heads, num_key_value_heads=kv_heads,
                               head_dim=dim, layer_types=['full_attention'])
    config._attn_implementation = 'sdpa'
    torch.manual_seed(0)
    module = Qwen3_5Attention(config, 0).cuda().bfloat16().eval().requires_grad_(False)
    return config, module


def _positions(n, dim=64, seed=1):
    gen = torch.Generator(device='cuda').manual_seed(seed)
    angle = torch.randn(1, n, dim, device='cuda', generator=gen)
    return angle.cos().bfloat16(), angle.sin().bfloat16()


def test_real_attention_decode_matches_upstream_and_keeps_the_cache():
    from torch.nn.attention.bias import causal_lower_right
    from trpg_b200.compressed_kv_attention import compressed_kv_info, configure_compressed_kv_attention
    from trpg_b200.quantized_kv import make_cache
    config, module = _attention_module()
    configure_compressed_kv_attention(module, False)
    cache = make_cache(config, 'q4')
    x = torch.randn(1, 384, 128, device='cuda', dtype=torch.bfloat16)
    pos = (torch.ones(1, 384, 64, device='cuda', dtype=torch.bfloat16),
           torch.zeros(1, 384, 64, device='cuda', dtype=torch.bfloat16))
    with torch.inference_mode():
        module(x, pos, causal_lower_right(384, 384), past_key_values=cache)
        ref, direct = copy.deepcopy(cache), copy.deepcopy(cache)
        hidden = x[:, :1].contiguous()
        positions = tuple(t[:, :1].contiguous() for t in pos)
        expected, _ = module(hidden, positions, causal_lower_right(1, 385), past_key_values=ref)
        configure_compressed_kv_attention(module, True)
        actual, weights = module(hidden, positions, causal_lower_right(1, 385), past_key_values=direct)
        assert weights is None
        torch.testing.assert_close(actual, expected, rtol=.03, atol=.004)
        assert compressed_kv_info(module)['direct_decode_calls'] == 1
        assert direct.get_seq_length() == ref.get_seq_length()
        assert torch.equal(direct.layers[0].keys, ref.layers[0].keys)
        u = ref.layers[0].key_bank.units
        assert direct.layers[0].key_bank.units == u
        assert torch.equal(direct.layers[0].key_bank.data[:, :, :u], ref.layers[0].key_bank.data[:, :, :u])
        # A masked history must go upstream, not to the all-visible kernel.
        custom = torch.zeros(1, 1, 1, 386, device='cuda', dtype=torch.bfloat16)
        custom[..., 10:200] = -float('inf')
        configure_compressed_kv_attention(module, False)
        expected, _ = module(hidden, positions, custom, past_key_values=ref)
        configure_compressed_kv_attention(module, True)
        actual, _ = module(hidden, positions, custom, past_key_values=direct)
        torch.testing.assert_close(actual, expected, rtol=0, atol=0)
        assert compressed_kv_info(module)['direct_decode_calls'] == 1
        bias = torch.zeros(1, 1, 1, 387, device='cuda', dtype=torch.bfloat16)
        bias[..., 100:250] = -30
        configure_compressed_kv_attention(module, False)
        expected, _ = module(hidden, positions, None, past_key_values=ref, position_bias=bias)
        configure_compressed_kv_attention(module, True)
        actual, _ = module(hidden, positions, None, past_key_values=direct, position_bias=bias)
        torch.testing.assert_close(actual, expected, rtol=0, atol=0)
        assert compressed_kv_info(module)['direct_decode_calls'] == 1


def _greedy(model, cache, ids, new_tokens, chunk=128):
    """Chunked prefill then greedy decode, one token per call."""
    out_tokens = []
    n = ids.shape[1]
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        out = model(input_ids=ids[:, s:e], position_ids=torch.arange(s, e, device='cuda')[None],
                    past_key_values=cache, use_cache=True, logits_to_keep=1)
        cache = out.past_key_values
    tok = int(out.logits[0, -1].argmax())
    for i in range(new_tokens - 1):
        out_tokens.append(tok)
        out = model(input_ids=torch.tensor([[tok]], device='cuda'),
                    position_ids=torch.tensor([[n + i]], device='cuda'),
                    past_key_values=cache, use_cache=True, logits_to_keep=1)
        cache = out.past_key_values
        tok = int(out.logits[0, -1].argmax())
    out_tokens.append(tok)
    return out_tokens


def test_greedy_generation_tokens_are_identical_with_the_patch():
    from transformers import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForCausalLM
    from trpg_b200.compressed_kv_attention import compressed_kv_info, configure_compressed_kv_attention
    from trpg_b200.quantized_kv import make_cache
    config = Qwen3_5TextConfig(vocab_size=64, hidden_size=128, intermediate_size=256,
                               num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                               head_dim=64, layer_types=['linear_attention', 'full_attention'],
                               max_position_embeddings=1024)
    config._attn_implementation = 'sdpa'
    torch.manual_seed(0)
    model = Qwen3_5ForCausalLM(config).cuda().bfloat16().eval().requires_grad_(False)
    ids = (torch.arange(384, device='cuda') % 64)[None]
    with torch.inference_mode():
        configure_compressed_kv_attention(model, False)
        expected = _greedy(model, make_cache(config, 'q8'), ids, 4)
        configure_compressed_kv_attention(model, True)
        actual = _greedy(model, make_cache(config, 'q8'), ids, 4)
    assert actual == expected
    assert compressed_kv_info(model)['direct_decode_calls'] == 3


def test_verify_route_inside_the_request_scope():
    from torch.nn.attention.bias import causal_lower_right
    from trpg_b200.compressed_kv_attention import compressed_kv_info, configure_compressed_kv_attention
    from trpg_b200.mtp_verification_kernels import mtp_verification_scope
    from trpg_b200.quantized_kv import make_cache
    config, module = _attention_module()
    configure_compressed_kv_attention(module, False)
    cache = make_cache(config, 'q8')
    n0 = 400
    x = torch.randn(1, n0 + 2, 128, device='cuda', dtype=torch.bfloat16)
    pos = _positions(n0 + 2)
    with torch.inference_mode():
        module(x[:, :n0], tuple(t[:, :n0] for t in pos), causal_lower_right(n0, n0), past_key_values=cache)
        ref, direct, plain = copy.deepcopy(cache), copy.deepcopy(cache), copy.deepcopy(cache)
        hidden = x[:, n0:].contiguous()
        positions = tuple(t[:, n0:].contiguous() for t in pos)
        mask = causal_lower_right(2, n0 + 2)
        expected, _ = module(hidden, positions, mask, past_key_values=ref)
        configure_compressed_kv_attention(module, True)
        module(hidden, positions, mask, past_key_values=plain)      # no scope: upstream
        assert compressed_kv_info(module)['direct_verify_calls'] == 0
        with mtp_verification_scope():
            actual, _ = module(hidden, positions, mask, past_key_values=direct)
            # Several queries without a mask: upstream aligns top-left; stays upstream.
            module(hidden, positions, None, past_key_values=copy.deepcopy(cache))
    assert compressed_kv_info(module)['direct_verify_calls'] == 1
    torch.testing.assert_close(actual, expected, rtol=.03, atol=.004)
    assert direct.get_seq_length() == ref.get_seq_length()
    assert torch.equal(direct.layers[0].keys, ref.layers[0].keys)


class _AppendTransaction:
    """The append transaction's contract (models/hybrid_cache_transaction.py):
    keys / values kept by reference, the banks' data / meta by reference,
    every other attribute copied as plain metadata; rollback restores the
    attribute dictionaries."""

    def __init__(self, cache):
        plain = (bool, int, float, str, torch.dtype, torch.device, type, type(None))
        self.states = []
        for layer in cache.layers:
            state = dict(vars(layer))
            for name, value in state.items():
                if name in ('key_bank', 'value_bank'):
                    bank = dict(vars(value))
                    assert all(k in ('data', 'meta') or isinstance(v, plain) for k, v in bank.items())
                    self.states.append((value, bank))
                else:
                    assert name in ('keys', 'values') or isinstance(value, plain), name
            self.states.append((layer, state))

    def rollback(self):
        for obj, state in self.states:
            vars(obj).clear()
            vars(obj).update(state)


def test_rollback_over_the_in_place_window_continues_like_a_fresh_cache():
    from torch.nn.attention.bias import causal_lower_right
    from trpg_b200.compressed_kv_attention import configure_compressed_kv_attention
    from trpg_b200.mtp_verification_kernels import mtp_verification_scope
    from trpg_b200.quantized_kv import make_cache
    config, module = _attention_module()
    configure_compressed_kv_attention(module, True)
    cache = make_cache(config, 'q8')
    n0 = 300
    x = torch.randn(1, n0 + 4, 128, device='cuda', dtype=torch.bfloat16)
    pos = _positions(n0 + 4)
    sl = lambda a, b: (x[:, a:b].contiguous(), tuple(t[:, a:b].contiguous() for t in pos))
    with torch.inference_mode():
        module(*sl(0, n0), causal_lower_right(n0, n0), past_key_values=cache)
        module(*sl(n0, n0 + 1), None, past_key_values=cache)        # window fast path
        twin = copy.deepcopy(cache)
        layer = cache.layers[0]
        base = layer.keys.data_ptr()
        tx = _AppendTransaction(cache)
        with mtp_verification_scope():                               # 2 rejected draft tokens
            module(*sl(n0 + 1, n0 + 3), causal_lower_right(2, n0 + 3), past_key_values=cache)
        assert cache.get_seq_length() == n0 + 3
        tx.rollback()
        assert cache.get_seq_length() == n0 + 1
        assert layer.keys.data_ptr() == base
        out, _ = module(*sl(n0 + 3, n0 + 4), None, past_key_values=cache)
        assert layer.keys.data_ptr() == base      # appended in place over the discarded rows
        want, _ = module(*sl(n0 + 3, n0 + 4), None, past_key_values=twin)
    torch.testing.assert_close(out, want, rtol=0, atol=0)
    assert torch.equal(layer.keys, twin.layers[0].keys)
    assert torch.equal(layer.values, twin.layers[0].values)
