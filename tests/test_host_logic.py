"""Host-side logic that needs no GPU: guards, mask whitelist, request scope,
multi-GPU planning, and the split-KV exchange over gloo ranks."""
import os
import threading

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import ckv_oracle as O
from trpg_b200 import sharding
from trpg_b200.compressed_kv_attention import (_supported_mask, compressed_kv_decode,
                                               compressed_kv_verify)
from trpg_b200.mtp_verification_kernels import mtp_verification_enabled, mtp_verification_scope
from trpg_b200.quantized_kv import QuantizedKVView


def cpu_view(packed=256, residual=129, heads=2, dim=64):
    z = torch.zeros
    return QuantizedKVView(z(1, heads, 4, dim, 128, dtype=torch.uint8), z(1, heads, 4, dim, 2),
                           z(1, heads, 512, dim // 64, 64, dtype=torch.uint8),
                           z(1, heads, 512, dim // 64, 2),
                           packed, z(1, heads, residual, dim, dtype=torch.bfloat16),
                           z(1, heads, residual, dim, dtype=torch.bfloat16), 8, packed + residual)


def test_cpu_inputs_return_none_so_callers_fall_back():
    view = cpu_view()
    q = torch.zeros(1, 4, 1, 64, dtype=torch.bfloat16)
    with torch.inference_mode():
        assert compressed_kv_decode(q, view, .125) is None
        assert compressed_kv_verify(q.expand(-1, -1, 2, -1), view, .125) is None


def test_only_lower_right_causal_masks_are_eligible():
    from torch.nn.attention.bias import causal_lower_right, causal_upper_left
    assert _supported_mask(None, 512)
    # Several queries without a mask: upstream aligns its causal mask top-left,
    # which the kernels do not reproduce, so the call stays upstream.
    assert not _supported_mask(None, 512, 2)
    assert not _supported_mask(None, 512, 64)
    assert _supported_mask(causal_lower_right(1, 512), 512)
    assert not _supported_mask(causal_upper_left(1, 512), 512)
    assert not _supported_mask(causal_lower_right(2, 512), 512)
    assert _supported_mask(causal_lower_right(2, 512), 512, 2)
    assert not _supported_mask(causal_lower_right(1, 511), 512)
    assert not _supported_mask(torch.zeros(1, 1, 1, 512), 512)


def test_verification_scope_nests_and_isolates_threads():
    assert not mtp_verification_enabled()
    with mtp_verification_scope():
        assert mtp_verification_enabled()
        with mtp_verification_scope(False):
            assert not mtp_verification_enabled()
        assert mtp_verification_enabled()
        seen = []
        t = threading.Thread(target=lambda: seen.append(mtp_verification_enabled()))
        t.start(); t.join()
        assert seen == [False]
    with pytest.raises(KeyError):
        with mtp_verification_scope():
            raise KeyError
    assert not mtp_verification_enabled()


def test_lpt_partition_balances_ragged_batches():
    rng = np.random.Generator(np.random.PCG64(3))
    lengths = rng.integers(1024, 8193, size=64)
    costs = [sharding.view_bytes(int(L) // 128 * 128, int(L) % 128 + 128) for L in lengths]
    for parts in (1, 2, 4, 8):
        plan = sharding.lpt_partition(costs, parts)
        assert sorted(i for p in plan for i in p) == list(range(64))
        loads = [sum(costs[i] for i in p) for p in plan]
        assert max(loads) <= sum(costs) / parts * 1.05 + max(costs)


def test_split_kv_ranges_cover_every_block_once():
    for units in (0, 1, 7, 254, 1022):
        for world in (1, 2, 3, 4, 8):
            ranges = [sharding.split_kv_range(units, 256, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == units
            for a, b in zip(ranges, ranges[1:]):
                assert a[1] == b[0]
            assert sum(r[3] - r[2] for r in ranges) == 256
            assert ranges[-1][2:] == [0, 256]


def test_view_bytes_matches_the_layout_figures():
    # 560 B per token per KV head for Q8 at D=256, 304 for Q4, 1024 residual.
    assert sharding.view_bytes(128, 0, 1) == 128 * 560
    assert sharding.view_bytes(128, 0, 1, bits=4) == 128 * 304
    assert sharding.view_bytes(0, 1, 1) == 1024


def _split_kv_rank(rank, world, port, result):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world,
                            timeout=__import__('datetime').timedelta(seconds=60))
    try:
        layer, _, _ = O.cache_state(21, 2, 1500, 64, 8)
        q = O.seeded_normal(23, (1, 4, 1, 64))
        keys, values = layer.full_kv()
        units, resid = layer.units, layer.keys.shape[2]
        ub, ue, rb, re = sharding.split_kv_range(units, resid, world, rank)
        idx = np.r_[np.arange(ub * 128, ue * 128), layer.packed_tokens + np.arange(rb, re)]
        m, l, o = O.partial_attention(q, keys[:, :, idx], values[:, :, idx], 0.125)
        part = torch.from_numpy(np.concatenate(
            (o.reshape(-1, 64), m.reshape(-1, 1), l.reshape(-1, 1)), 1).astype(np.float32))
        parts = sharding.gather_partials(part).numpy()
        out = O.combine_partials([p[:, 64] for p in parts], [p[:, 65] for p in parts],
                                 [p[:, :64] for p in parts])
        want = O.attention(q, keys, values, 0.125).reshape(-1, 64)
        result[rank] = float(np.abs(out - want).max())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('world', [2])
def test_split_kv_exchange_over_gloo_matches_full_attention(world):
    ctx = mp.get_context('spawn')
    manager = ctx.Manager()
    result = manager.dict()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_split_kv_rank, args=(r, world, port, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert len(result) == world
    assert max(result.values()) < 1e-5


FAKE_SCOPE = """
from contextlib import contextmanager
from contextvars import ContextVar
_MTP_VERIFICATION_ENABLED = ContextVar('fake_flag', default=False)
@contextmanager
def mtp_verification_scope(enabled=True):
    token = _MTP_VERIFICATION_ENABLED.set(bool(enabled))
    try:
        yield
    finally:
        _MTP_VERIFICATION_ENABLED.reset(token)
"""
FAKE_CACHE = """
class QuantizedAttentionLayer:
    pass
def make_cache(config, mode='q8'):
    return 'reference cache'
def cache_bytes(cache):
    return -1
"""
FAKE_CALLER = """
from .quantized_kv import make_cache, cache_bytes, QuantizedAttentionLayer
from .mtp_verification_kernels import mtp_verification_scope
"""


def test_install_routes_every_module_and_shares_the_verify_flag(tmp_path, monkeypatch):
    """A package laid out like the reference: a caller imported before
    install() gets this package's functions and classes, one imported after
    gets them through the module table, and the caller's verify scope turns
    on the flag the patched forward reads."""
    import importlib
    import sys
    from trpg_b200 import install as I
    from trpg_b200 import compressed_kv_attention as A
    from trpg_b200 import mtp_verification_kernels as S
    from trpg_b200 import quantized_kv as Q
    pkg = tmp_path / 'fakeref'
    pkg.mkdir()
    (pkg / '__init__.py').write_text('')
    (pkg / 'mtp_verification_kernels.py').write_text(FAKE_SCOPE)
    (pkg / 'quantized_kv.py').write_text(FAKE_CACHE)
    (pkg / 'early_caller.py').write_text(FAKE_CALLER)
    (pkg / 'late_caller.py').write_text(FAKE_CALLER)
    monkeypatch.syspath_prepend(str(tmp_path))
    own_flag = S._MTP_VERIFICATION_ENABLED
    early = importlib.import_module('fakeref.early_caller')
    assert early.make_cache(None) == 'reference cache'
    try:
        I.install('fakeref')
        assert sys.modules['fakeref.quantized_kv'] is Q
        for name in I.MODULES:
            assert sys.modules[f'fakeref.{name}'].__name__ == f'trpg_b200.{name}'
        assert early.make_cache is Q.make_cache and early.cache_bytes is Q.cache_bytes
        assert early.QuantizedAttentionLayer is Q.QuantizedAttentionLayer
        late = importlib.import_module('fakeref.late_caller')
        assert late.make_cache is Q.make_cache
        for scope in (early.mtp_verification_scope, late.mtp_verification_scope):
            assert not A._scope.mtp_verification_enabled()
            with scope():
                assert A._scope.mtp_verification_enabled()
            assert not A._scope.mtp_verification_enabled()
    finally:
        I.uninstall('fakeref')
        S.bind(own_flag)
        for name in list(sys.modules):
            if name == 'fakeref' or name.startswith('fakeref.'):
                del sys.modules[name]


def test_layer_state_is_what_a_cache_transaction_can_snapshot():
    """The reference transaction (models/hybrid_cache_transaction.py:74-99)
    keeps tensors of a quantized layer only under keys / values (by
    reference) and the banks' data / meta; every other attribute must be
    plain metadata.  The in-place window therefore lives in integers."""
    from trpg_b200.quantized_kv import QuantizedAttentionLayer
    plain = (bool, int, float, str, torch.dtype, torch.device, type, type(None))
    layer = QuantizedAttentionLayer(8)
    x = torch.zeros(1, 2, 5, 64, dtype=torch.bfloat16)
    with torch.inference_mode():
        layer.append_for_attention(x, x)        # CPU tensors: the concatenating path
    for name, value in vars(layer).items():
        if name in ('keys', 'values'):
            assert isinstance(value, torch.Tensor)
        elif name in ('key_bank', 'value_bank'):
            for bname, bvalue in vars(value).items():
                assert bname in ('data', 'meta') or isinstance(bvalue, plain), bname
        else:
            assert isinstance(value, plain), (name, type(value))
