"""Split-KV partials exchanged over peer memory (``ckv_exchange_*``, GPU).

* Two ranks' buffers driven from one process on one GPU (publish launches,
  then wait-and-merge launches, so no launch waits on another launch):
  every rank's merge equals ``ckv_combine_partials`` of the same partials
  bit for bit, over several steps (both slots, partial shapes with a rank
  that saw no token).
* A wait that nothing satisfies gives up after its bound, sets the error
  word, and leaves the context usable.
* On two GPUs (skipped with fewer), two processes map each other's buffers
  through CUDA IPC; each rank's merged split-KV decode equals the merge of
  the gathered partials.
"""
import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

ROWS, D = 16, 256


def _partials(seed, world, empty_rank=None):
    g = torch.Generator(device='cuda').manual_seed(seed)
    p = torch.randn(world, ROWS, D + 2, generator=g, device='cuda')
    p[:, :, D] = torch.rand(world, ROWS, generator=g, device='cuda') * 10 - 5     # m (log2 domain)
    p[:, :, D + 1] = torch.rand(world, ROWS, generator=g, device='cuda') * 50 + 1  # l > 0
    if empty_rank is not None:
        p[empty_rank, :, :D] = 0
        p[empty_rank, :, D] = -float('inf')
        p[empty_rank, :, D + 1] = 0
    return p


def _alloc(world):
    from trpg_b200 import _native
    lib = _native.library()
    buf = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    assert lib.ckv_exchange_alloc(world, ROWS, D, ctypes.byref(buf), handle) == 0
    return lib, buf.value


def _error(lib, buf):
    flag = ctypes.c_int(0)
    assert lib.ckv_exchange_error(buf, ctypes.byref(flag), torch.cuda.current_stream().cuda_stream) == 0
    return flag.value


@pytest.mark.parametrize('world', [2, 3])
def test_ranks_on_one_gpu_merge_like_combine_partials(world):
    from trpg_b200._native import ops
    allocs = [_alloc(world) for _ in range(world)]
    lib, bufs = allocs[0][0], [b for _, b in allocs]
    try:
        for step in range(5):
            parts = _partials(100 + step, world, empty_rank=(step % world) if step == 3 else None)
            want = ops().combine_partials(parts, torch.bfloat16)
            for r in range(world):
                ops().exchange_combine(parts[r].contiguous(), bufs, r, 1, 0, torch.bfloat16)
            outs = [ops().exchange_combine(parts[r].contiguous(), bufs, r, 2, 0, torch.bfloat16)
                    for r in range(world)]
            for out in outs:
                assert torch.equal(out, want), step
        assert all(_error(lib, b) == 0 for b in bufs)
    finally:
        torch.cuda.synchronize()
        for _, b in allocs:
            lib.ckv_exchange_free(b)


def test_a_wait_nothing_satisfies_gives_up_and_reports_it():
    from trpg_b200._native import ops
    lib, b0 = _alloc(2)
    _, b1 = _alloc(2)
    try:
        parts = _partials(7, 2)
        # Rank 0 publishes; rank 1 never does, so rank 0's wait runs out
        # after about 2^20 cycles (half a millisecond).
        ops().exchange_combine(parts[0].contiguous(), [b0, b1], 0, 3, 1 << 20, torch.bfloat16)
        assert _error(lib, b0) == 1
        assert _error(lib, b0) == 0                      # read and cleared
        # The context is still usable.
        x = torch.arange(10, device='cuda', dtype=torch.float32)
        assert float((x * 2).sum()) == 90.0
    finally:
        torch.cuda.synchronize()
        lib.ckv_exchange_free(b0)
        lib.ckv_exchange_free(b1)


def _two_gpu_rank(rank, world, port, result):
    os.environ.setdefault('NCCL_NVLS_ENABLE', '0')
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group('gloo', init_method=f'tcp://127.0.0.1:{port}', rank=rank, world_size=world)
    ok = False
    try:
        from oracle import ckv_oracle as O
        from tests._util import gpu_cache_state, to_torch
        from trpg_b200 import compressed_kv_kernels as K
        from trpg_b200.sharding import PeerExchange, split_kv_range
        ex = PeerExchange(ROWS, D)
        layer, view, _ = gpu_cache_state(9, 4, 20000, D, 8)
        good = True
        for step in range(4):
            q = to_torch(O.seeded_normal(50 + step, (1, 16, 1, D)), 'bfloat16')
            rng = split_kv_range(view.packed_tokens // 128, view.keys.shape[2], world, rank)
            with torch.inference_mode():
                part = K.attention([q], [view], 1 / 16, ranges=[rng], partial=True)[0]
                out = ex.combine(part, torch.bfloat16)
            gathered = [None] * world
            dist.all_gather_object(gathered, part.cpu())
            want = K.combine(torch.stack([g.cuda() for g in gathered]), torch.bfloat16)
            good = good and torch.equal(out, want)
        good = good and ex.error() == 0
        ex.close()
        ok = good
    finally:
        result[rank] = ok
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason='needs two GPUs')
def test_two_gpus_exchange_through_peer_mappings():
    import torch.multiprocessing as mp
    world = 2
    with mp.get_context('spawn').Manager() as m:
        result = m.dict()
        mp.start_processes(_two_gpu_rank, args=(world, 29617, result), nprocs=world,
                           start_method='spawn', join=True)
        assert [result.get(r) for r in range(world)] == [True, True]
