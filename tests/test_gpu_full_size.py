"""Parity at the full size of every workload the benchmark names.

Each case builds the cache the reference's way (``update`` of L - n tokens,
then ``append_for_attention`` of n, ``scripts/profile_compressed_kv.py:31-36``)
with this package's kernels, runs the CUDA attention through the public
entry points, and compares with the oracle's dequantize + SDPA restatement
(``oracle.ckv_oracle.decode_reference_chunked``: float64, one KV head and a
bounded chunk of positions at a time).

Tolerances: the reference tests' own ``assert_allclose(rtol=.025,
atol=.004)`` (tests/test_compressed_kv_attention.py:76) and the looser
max-abs 2e-2 / rel 1e-2 of the workload definition, both asserted.

The sizes matter because the launch plan changes shape with them: one wave
of 37 CTAs per KV head for few (sequence, head) pairs (the 32K and 131K
single-sequence cases), several waves of about 8 items per CTA for many
pairs (the 64-sequence batch and the 16 x 4-query verify), the 16-row
two-tile variant for 4 queries, and the merge copying records in chunks
when a pair's records exceed shared memory (16-row records, about 18 CTAs
per pair in the verify case).
"""
import numpy as np
import pytest
import torch

from oracle import ckv_oracle as O
from tests._util import gpu_cache_state, to_torch

pytestmark = pytest.mark.gpu

HQ, HKV, D = 16, 4, 256
SCALE = 1 / 16
RTOL, ATOL = .025, .004          # reference tests
MAX_ABS, REL = 2e-2, 1e-2        # workload definition (max-abs, relative to max |expected|)


def check(actual, expected):
    a = actual.float().cpu().numpy().astype(np.float64).reshape(expected.shape)
    np.testing.assert_allclose(a, expected, rtol=RTOL, atol=ATOL)
    err = np.abs(a - expected).max()
    assert err <= MAX_ABS, err
    assert err <= REL * max(1.0, np.abs(expected).max()), err


def query(seed, nq=1, dtype='bfloat16'):
    qn = O.seeded_normal(seed, (1, HQ, nq, D), dtype)
    return qn, to_torch(qn, dtype)


def test_single_sequence_32k_q8_outliers_across_compaction(both_rules):
    """32768 tokens (32512 packed + 256 window) with 1% of channels x8, then
    160 decode steps on the same layer (a compaction at the 256th window
    token), checked against the oracle at the first step, just before and
    just after the compaction, and at the last step."""
    from trpg_b200.compressed_kv_kernels import decode
    layer, view, ol = gpu_cache_state(2, HKV, 32768, D, 8, outliers=True)
    assert view.packed_tokens == 32512 and view.keys.shape[2] == 256
    qn, qt = query(20)
    with torch.inference_mode():
        check(decode(qt, view, SCALE), O.decode_reference_chunked(qn, ol, SCALE))
        layer.compact_residual()
        ol.compact_residual()
        units0 = layer.key_bank.units
        for step in range(1, 161):
            kn = O.seeded_normal(3000 + step, (1, HKV, 1, D))
            vn = O.seeded_normal(5000 + step, (1, HKV, 1, D))
            view = layer.append_for_attention(to_torch(kn, 'bfloat16'), to_torch(vn, 'bfloat16'))
            ol.append_for_attention(kn, vn)
            if step in (1, 127, 128, 129, 160):
                qn, qt = query(7000 + step)
                check(decode(qt, view, SCALE), O.decode_reference_chunked(qn, ol, SCALE))
            layer.compact_residual()
            ol.compact_residual()
    assert layer.key_bank.units == ol.units == units0 + 1


def test_two_32k_layers_back_to_back(both_rules):
    """Two distinct 32K caches decoded one after the other on one stream (the
    benchmark's layer loop), each checked."""
    from trpg_b200.compressed_kv_kernels import decode
    states = [gpu_cache_state(40 + i, HKV, 32768, D, 8, outliers=True) for i in range(2)]
    queries = [query(60 + i) for i in range(2)]
    with torch.inference_mode():
        outs = [decode(qt, view, SCALE) for (qn, qt), (_, view, _) in zip(queries, states)]
    for out, (qn, _), (_, _, ol) in zip(outs, queries, states):
        check(out, O.decode_reference_chunked(qn, ol, SCALE))


def test_batch_of_64_ragged_sequences_in_one_launch(both_rules):
    """64 sequences, contexts uniform in [1024, 8192], one query each, Q8:
    one kernel launch over all (sequence, KV head) pairs."""
    from trpg_b200.compressed_kv_kernels import MAX_SEQS, attention
    rng = np.random.Generator(np.random.PCG64(3))
    lengths = rng.integers(1024, 8193, size=64).tolist()
    assert len(lengths) == MAX_SEQS
    states = [gpu_cache_state(300 + i, HKV, L, D, 8) for i, L in enumerate(lengths)]
    queries = [query(400 + i) for i in range(64)]
    with torch.inference_mode():
        outs = attention([q[1] for q in queries], [s[1] for s in states], SCALE)
    for out, (qn, _), (_, _, ol) in zip(outs, queries, states):
        check(out, O.decode_reference_chunked(qn, ol, SCALE))


def test_verify_16_sequences_4_queries_16k(both_rules):
    """16 sequences x 4 query positions (lower-right causal among them) over
    16384 tokens, Q8: 16 query rows per KV head, the two-tile variant."""
    from trpg_b200.compressed_kv_kernels import attention
    states = [gpu_cache_state(500 + i, HKV, 16384, D, 8, new_tokens=4) for i in range(16)]
    queries = [query(600 + i, nq=4) for i in range(16)]
    with torch.inference_mode():
        outs = attention([q[1] for q in queries], [s[1] for s in states], SCALE)
    for out, (qn, _), (_, _, ol) in zip(outs, queries, states):
        check(out, O.decode_reference_chunked(qn, ol, SCALE, causal_lower_right=True))


@pytest.fixture(scope='module')
def long_q4():
    layer, view, ol = gpu_cache_state(5, HKV, 131072, D, 4)
    qn, qt = query(55)
    expected = O.decode_reference_chunked(qn, ol, SCALE, chunk=16384)
    return layer, view, ol, qn, qt, expected


def test_long_context_q4_131k_whole(long_q4, both_rules):
    from trpg_b200.compressed_kv_kernels import decode
    layer, view, ol, qn, qt, expected = long_q4
    assert view.packed_tokens == 130816 and view.keys.shape[2] == 256
    with torch.inference_mode():
        check(decode(qt, view, SCALE), expected)


@pytest.mark.parametrize('world', [2, 4, 8])
def test_long_context_q4_131k_split_kv_shards(long_q4, world, both_rules):
    """The split-KV partitioning of the multi-GPU path, emulated on one GPU:
    each shard's (o, m, l) partial from its own launch, merged by the
    combine kernel."""
    from trpg_b200.compressed_kv_kernels import attention, combine
    from trpg_b200.sharding import split_kv_range
    layer, view, ol, qn, qt, expected = long_q4
    units, resid = view.packed_tokens // 128, view.keys.shape[2]
    with torch.inference_mode():
        parts = [attention([qt], [view], SCALE, ranges=[split_kv_range(units, resid, world, r)],
                           partial=True)[0] for r in range(world)]
        out = combine(parts, torch.bfloat16)
    check(out.view(1, HQ, 1, D), expected)
