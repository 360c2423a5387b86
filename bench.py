"""Benchmark: Q8-KV decode attention at 32K context (8 full-attention layers).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (per GPU): one sequence whose 8 full-attention layers each hold a
distinct Q8 cache of 32768 tokens (32512 packed + 256 exact residual; the
reference-reachable state), 16 query heads / 4 KV heads x 256, bf16.  K and V
are seeded N(0,1) with 1% of channels per KV head scaled x8.  One step =
for each layer: append the new token (residual), decode attention over the
whole cache, compact (one 128-token block is quantized into the banks every
128 steps).  Every 128 steps the cache is rolled back to its starting state
(reference swap, no device work) so the context stays at 32768..32895.

Reported: ``value`` = tokens/s through the 8 attention layers summed over all
GPUs, device-timed with CUDA events (inputs resident in HBM; the 8 caches,
591 MB, exceed L2); ``e2e`` = the same through the public API with the step's
inputs copied from pinned host memory and outputs read back every step;
``roofline`` = achieved HBM GB/s of the decode kernel (algorithmic bytes per
launch / mean launch time) against the measured copy bandwidth;
``cpu_baseline`` = the reference's PyTorch CPU path (restated in
``oracle/ckv_cpu_path.py``) on this host.  With N > 1 every rank runs its own
sequence (weak scaling: sequences are independent, no collective on the data
path).  ``--impl reference`` times that CPU path alone.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
METRIC = ('Q8-KV decode attn µs/step & HBM GB/s (% peak) at 32K ctx; '
          '1/2/4/8-GPU tok/s')
HQ, HKV, D, LAYERS, CONTEXT, BITS = 16, 4, 256, 8, 32768, 8
SCALE = 1 / 16
ROLLBACK = 128


def peaks():
    path = ROOT / 'MEASURED_PEAKS.json'
    if path.exists():
        data = json.loads(path.read_text())
        return float(data['hbm_gbs']), 'measured'
    return 6650.0, 'fallback'


# ---------------------------------------------------------------------------
# Distributed plumbing
# ---------------------------------------------------------------------------
def init_dist():
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if world > 1:
        import datetime
        import torch.distributed as dist
        # NCCL's communicator set-up lines (stderr) name the ranks and the
        # transport each run used.
        os.environ.setdefault('NCCL_DEBUG', 'INFO')
        os.environ.setdefault('NCCL_DEBUG_SUBSYS', 'INIT')
        torch.cuda.set_device(local)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device('cuda', local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], device='cuda', dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# Clocks sampled during the timed region
# ---------------------------------------------------------------------------
# A child process samples the SM clock and the clock-event reasons through
# NVML (read-only queries) every 20 ms and writes one flushed line per sample:
# "<unix time> <MHz> <max MHz> <reason mask>".
_SAMPLER = r"""
import sys, time, pynvml as nv
nv.nvmlInit()
uuid, out = sys.argv[1], sys.argv[2]
handle = None
for i in range(nv.nvmlDeviceGetCount()):
    h = nv.nvmlDeviceGetHandleByIndex(i)
    u = nv.nvmlDeviceGetUUID(h)
    u = u.decode() if isinstance(u, bytes) else u
    if u.replace('GPU-', '') == uuid:
        handle = h
if handle is None:
    handle = nv.nvmlDeviceGetHandleByIndex(0)
mx = nv.nvmlDeviceGetMaxClockInfo(handle, nv.NVML_CLOCK_SM)
with open(out, 'w') as f:
    while True:
        mhz = nv.nvmlDeviceGetClockInfo(handle, nv.NVML_CLOCK_SM)
        mask = nv.nvmlDeviceGetCurrentClocksEventReasons(handle)
        f.write(f'{time.time()} {mhz} {mx} {mask}\n')
        f.flush()
        time.sleep(0.02)
"""


class Clocks:
    """SM clock and clock-event reasons during a time window, sampled by a
    child process so that the benchmark's own launches are not slowed."""
    REASONS = (('hw_slowdown', 0x8), ('sw_power_cap', 0x4), ('hw_thermal_slowdown', 0x40),
               ('sw_thermal_slowdown', 0x20), ('hw_power_brake', 0x80))

    def __init__(self, device: int):
        import subprocess
        import tempfile
        self.path = tempfile.mktemp(prefix='bench_clocks_', suffix='.txt')
        self.proc = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.proc = subprocess.Popen([sys.executable, '-c', _SAMPLER, uuid, self.path],
                                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except (OSError, RuntimeError, AttributeError):
            self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        self.t0 = time.time()

    def stop(self):
        self.t1 = time.time()

    def summary(self):
        if self.proc is None:
            return {'samples': 0}
        time.sleep(0.05)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except Exception:
            self.proc.kill()
        rows = []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = line.split()
                    if len(parts) == 4:
                        rows.append((float(parts[0]), float(parts[1]), float(parts[2]), int(parts[3])))
            os.unlink(self.path)
        except OSError:
            pass
        inside = [r for r in rows if self.t0 is not None and self.t0 <= r[0] <= self.t1]
        if not inside:
            return {'samples': 0, 'samples_total': len(rows)}
        reasons = sorted({name for _, _, _, mask in inside for name, bit in self.REASONS if mask & bit})
        return {'sm_mhz': statistics.median(r[1] for r in inside), 'sm_max_mhz': max(r[2] for r in inside),
                'reasons': reasons, 'samples': len(inside)}


# ---------------------------------------------------------------------------
# Workload
# ---------------------------------------------------------------------------
def synthetic_kv(gen, length, device):
    """K, V ~ N(0,1) bf16 with 1% of channels per KV head scaled x8."""
    k = torch.randn(1, HKV, length, D, generator=gen, device=device, dtype=torch.float32)
    v = torch.randn(1, HKV, length, D, generator=gen, device=device, dtype=torch.float32)
    count = -(-D // 100)
    for h in range(HKV):
        idx = torch.randperm(D, generator=gen, device=device)[:count]
        k[:, h, :, idx] *= 8
        v[:, h, :, idx] *= 8
    return k.bfloat16(), v.bfloat16()


def algorithmic_bytes(view) -> int:
    """Codes + meta of every packed token, the exact residual, q and output."""
    packed, resid = view.packed_tokens, view.keys.shape[2]
    per_token = 2 * D * BITS // 8 + D * 8 // 128 + (D // 64) * 8      # 560 at Q8, D=256
    return HKV * (packed * per_token + resid * 2 * D * 2) + 2 * HQ * D * 2


class Sequence:
    """8 layer caches of one sequence plus per-step inputs.

    The caches are built with ``update`` of 32767 tokens and then one decode
    step (append + compaction), so the timed state starts right after a
    compaction: 32640 packed tokens and a 128-token exact window, and the
    first timed step attends over 32769 tokens.  Every ``ROLLBACK`` (128)
    steps the layers return to that state; the compaction that the 128th step
    of a cycle would do is therefore never timed inside the loop and is
    charged separately (``compaction_seconds``).
    """

    def __init__(self, seed, steps, device):
        from trpg_b200.quantized_kv import QuantizedAttentionLayer
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        self.layers = []
        with torch.inference_mode():
            for _ in range(LAYERS):
                k, v = synthetic_kv(gen, CONTEXT - 1, device)
                layer = QuantizedAttentionLayer(BITS)
                layer.update(k, v)
                del k, v
                kn = torch.randn(1, HKV, 1, D, generator=gen, device=device).bfloat16()
                layer.append_for_attention(kn, kn)
                layer.compact_residual()
                assert layer.keys.shape[2] == 128
                self.layers.append(layer)
        torch.cuda.synchronize()
        n = min(steps, ROLLBACK - 1)
        self.q = torch.randn(n, LAYERS, 1, HQ, 1, D, generator=gen, device=device).bfloat16()
        self.kn = torch.randn(n, LAYERS, 1, HKV, 1, D, generator=gen, device=device).bfloat16()
        self.vn = torch.randn(n, LAYERS, 1, HKV, 1, D, generator=gen, device=device).bfloat16()
        # Per (step, layer) input tensors, as a model's projections would hand
        # them over (no indexing inside the timed loop).
        self.qs = [list(self.q[i].unbind(0)) for i in range(n)]
        self.kns = [list(self.kn[i].unbind(0)) for i in range(n)]
        self.vns = [list(self.vn[i].unbind(0)) for i in range(n)]
        self.snap = [self._snapshot(l) for l in self.layers]

    @staticmethod
    def _snapshot(layer):
        # Every attribute of the layer and its banks (tensors by reference),
        # as an append transaction keeps them: the in-place window's integers
        # come back with its views, so appends after a rollback stay in place.
        return dict(vars(layer)), dict(vars(layer.key_bank)), dict(vars(layer.value_bank))

    def rollback(self):
        for layer, (state, kb, vb) in zip(self.layers, self.snap):
            vars(layer).clear()
            vars(layer).update(state)
            vars(layer.key_bank).clear()
            vars(layer.key_bank).update(kb)
            vars(layer.value_bank).clear()
            vars(layer.value_bank).update(vb)


def run_steps(seq, decode, steps, start=0, outs=None):
    """Run ``steps`` decode steps (all layers); returns #kernel launches.

    A cycle is ROLLBACK - 1 steps from the snapshot (the window grows from
    128 to 255 tokens, so no step compacts); then the layers roll back."""
    launches = 0
    cycle = ROLLBACK - 1
    for s in range(start, start + steps):
        i = s % cycle
        if i == 0 and s:
            seq.rollback()
        qs, kns, vns = seq.qs[i], seq.kns[i], seq.vns[i]
        for li, layer in enumerate(seq.layers):
            view = layer.append_for_attention(kns[li], vns[li])
            out = decode(qs[li], view, SCALE)
            launches += 2
            units = layer.key_bank.units
            layer.compact_residual()
            launches += layer.key_bank.units != units
            if outs is not None:
                outs[li] = out
    return launches


def capture_steps(seq, decode, count, inputs, stream, out, before=None, after=None):
    """One CUDA graph per step position i < count of the rollback cycle, each
    holding step i's 8 layers (append of the new key/value row into the
    exact window, then decode) and the stack of the 8 outputs into `out`;
    ``before(i)`` / ``after(i)`` add work captured ahead of / behind the
    layers (the end-to-end loop's input and output copies).

    A serving loop replays the graph of the step it is at; the row a step
    appends and the length it attends over are fixed per position, so the
    graphs are captured in cycle order from the snapshot state and replaying
    graph i reproduces step i of every cycle (graph 0 after graph count - 1
    is the rollback).  ``inputs(i)`` gives step i's per-layer (q, k, v)."""
    graphs = []
    pool = torch.cuda.graph_pool_handle()
    seq.rollback()
    with torch.inference_mode():
        for i in range(count):
            qs, kns, vns = inputs(i)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream, pool=pool):
                if before is not None:
                    before(i)
                outs = []
                for li, layer in enumerate(seq.layers):
                    view = layer.append_for_attention(kns[li], vns[li])
                    outs.append(decode(qs[li], view, SCALE))
                    layer.compact_residual()       # a no-op within the cycle
                torch.stack(outs, out=out)
                if after is not None:
                    after(i)
            graphs.append(g)
    seq.rollback()
    return graphs


def warm_stream(seq, decode, stream):
    """One eager step on `stream` (its attention workspace is made outside
    any capture), then back to the snapshot."""
    stream.wait_stream(torch.cuda.current_stream())
    with torch.inference_mode(), torch.cuda.stream(stream):
        run_steps(seq, decode, 1)
    stream.synchronize()
    seq.rollback()


def compaction_seconds(seq, repeats=8):
    """Device seconds of one layer's compaction (quantize 128 tokens into the
    banks and move the rest of the window), the work every 128th decode step
    of a layer adds: each layer is brought to a 256-token window, compacted
    between CUDA events, and rolled back."""
    total, count = 0.0, 0
    with torch.inference_mode():
        for r in range(repeats):
            for layer in seq.layers:
                kn = seq.kn[0, 0].expand(1, HKV, 128, D).contiguous()
                layer.append_for_attention(kn, kn)
                assert layer.keys.shape[2] == 256
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                layer.compact_residual()
                b.record()
                b.synchronize()
                if r:                       # the first round warms the allocator
                    total += a.elapsed_time(b) * 1e-3
                    count += 1
            seq.rollback()
    return total / count


def time_kernel(seq, decode, min_seconds=0.6):
    """Mean device time of one decode launch.

    The 8 layers' decode launches (one token appended to each cache) are
    captured once in a CUDA graph and replayed back to back on one stream,
    between CUDA events on that stream, so host launch overhead is excluded;
    the 8 distinct caches (591 MB) keep every launch reading from HBM.  The
    replays run for at least ``min_seconds`` so that the clock sampler sees
    the kernel under load.
    """
    with torch.inference_mode():
        views = [layer.append_for_attention(seq.kn[0, li], seq.vn[0, li])
                 for li, layer in enumerate(seq.layers)]
        sizes = [algorithmic_bytes(v) for v in views]
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for li, v in enumerate(views):     # the stream's workspace is made outside capture
                decode(seq.q[0, li], v, SCALE)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for li, v in enumerate(views):
                decode(seq.q[0, li], v, SCALE)

        def replay(n):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                graph.replay()
                a.record(stream)
                for _ in range(n):
                    graph.replay()
                b.record(stream)
            stream.synchronize()
            return a.elapsed_time(b) * 1e-3

        probe = replay(32) / 32
        replays = max(32, int(min_seconds / probe) + 1)
        sec = replay(replays) / (replays * LAYERS)
        del graph
    seq.rollback()
    return sec, statistics.mean(sizes), replays


def cpu_reference(steps, warmup, one_thread_steps=0):
    """The reference CPU path on one layer per step (a bounded sample)."""
    from oracle import ckv_cpu_path as P
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(12)
    layer = P.CpuLayer(BITS)
    k, v = synthetic_kv(gen, CONTEXT - 1, 'cpu')
    layer.update(k, v)
    del k, v
    snap = (layer.keys, layer.values, layer.length, layer.kd, layer.km, layer.vd, layer.vm)
    q = torch.randn(1, HQ, 1, D, generator=gen).bfloat16()
    kn = torch.randn(1, HKV, 1, D, generator=gen).bfloat16()
    def timed(n):
        times = []
        for i in range(n):
            if i and i % ROLLBACK == 0:
                layer.keys, layer.values, layer.length, layer.kd, layer.km, layer.vd, layer.vm = snap
            t = time.perf_counter()
            P.decode_step(layer, q, kn, kn, SCALE)
            times.append(time.perf_counter() - t)
        return statistics.mean(times)

    for i in range(warmup):
        P.decode_step(layer, q, kn, kn, SCALE)
    per_layer = timed(steps)
    out = {'value': 1.0 / (LAYERS * per_layer), 'unit': 'tok/s', 'cores': threads,
           'kind': 'port', 'ms_per_layer': per_layer * 1e3,
           'sample': f'{steps} decode steps of 1 of the 8 identical 32K-token Q8 layers '
                     f'(append + dequantize + SDPA + compact), torch CPU ops, {threads} threads; '
                     f'tok/s = 1 / (8 x mean layer time)'}
    if one_thread_steps:
        torch.set_num_threads(1)
        try:
            single = timed(one_thread_steps)
        finally:
            torch.set_num_threads(threads)
        out['one_thread'] = {'value': 1.0 / (LAYERS * single), 'unit': 'tok/s', 'cores': 1,
                             'ms_per_layer': single * 1e3, 'sample': f'{one_thread_steps} decode steps'}
    return out


# ---------------------------------------------------------------------------
# Arms
# ---------------------------------------------------------------------------
def reference_arm(args, world, rank):
    if rank != 0:
        return
    base = cpu_reference(args.steps, args.warmup)
    line = {'impl': 'reference', 'metric': METRIC, 'value': base['value'], 'unit': 'tok/s',
            'n_gpus': args.gpus, 'steps': args.steps, 'warmup': args.warmup,
            'ms_per_step': base['ms_per_layer'] * LAYERS, 'higher_is_better': True,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'u8/bf16', 'data': 'synthetic',
            'config': config(args, world),
            'cpu_baseline': {k: base[k] for k in ('value', 'unit', 'cores', 'kind', 'sample')},
            'e2e': {'value': base['value'], 'unit': 'tok/s', 'h2d_bytes_per_step': 0,
                    'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)


def config(args, world):
    return {'workload': 'single-sequence Q8 decode, 8 layers x 32K context (32640 packed + '
                        '129..255 bf16 recent tokens: 32769..32895 in all), 16q/4kv x 256, '
                        'append + decode per layer; the 128-token compaction every 128 steps '
                        'is timed separately and charged per step',
            'model': 'attention only (no weights)', 'global_batch': world, 'seq_len': CONTEXT,
            'parallelism': f'dp{world} (independent sequences)', 'layers': LAYERS,
            'heads_q': HQ, 'heads_kv': HKV, 'head_dim': D, 'bits': BITS,
            'l2': 'inputs larger than L2 (8 distinct caches, 591 MB per GPU)',
            'clocks_window': 'the timed loop plus the roofline replays (at least 0.6 s)'}


def b200_arm(args, world, rank, local):
    from trpg_b200 import _native
    from trpg_b200.compressed_kv_kernels import decode
    _native.load()
    device = torch.device('cuda', local)
    torch.cuda.set_device(device)
    clocks = Clocks(local)          # the sampler starts while the caches are built
    seq = Sequence(1000 + rank, args.steps + args.warmup, device)
    cycle = ROLLBACK - 1
    count = min(cycle, max(args.steps, args.warmup))
    stream = torch.cuda.Stream(device)
    warm_stream(seq, decode, stream)
    step_out = torch.empty(LAYERS, 1, HQ, 1, D, dtype=torch.bfloat16, device=device)
    graphs = capture_steps(seq, decode, count, lambda i: (seq.qs[i], seq.kns[i], seq.vns[i]),
                           stream, step_out)
    # The graphs compute what the eager calls compute: step 0 both ways.
    with torch.inference_mode(), torch.cuda.stream(stream):
        graphs[0].replay()
        got = step_out.clone()
        want = [None] * LAYERS
        run_steps(seq, decode, 1, outs=want)
        want = torch.stack(want)
    stream.synchronize()
    seq.rollback()
    if not torch.equal(got, want):
        raise RuntimeError('step graph and eager step disagree')

    def replay_steps(first, k):
        for s in range(first, first + k):
            graphs[(s % cycle) % count].replay()

    # untimed warm-up: every graph once (its first launch uploads it to the
    # device), then the warm-up steps
    with torch.cuda.stream(stream):
        for g in graphs:
            g.replay()
        replay_steps(0, args.warmup)
    stream.synchronize()

    # ---- device-timed region: K steps, one graph replay each -------------------
    barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push('timed')      # lets a profiler keep to the timed launches
    with torch.cuda.stream(stream):
        start.record(stream)
        replay_steps(0, args.steps)
        stop.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier(world)
    loop_ms = max_over_ranks(start.elapsed_time(stop), world)
    launches = 2 * LAYERS * args.steps       # append + decode per layer per step
    del graphs

    # The same steps issued eagerly from Python (no graphs), for comparison.
    seq.rollback()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    eager_steps = min(args.steps, 4 * cycle)
    start.record()
    run_steps(seq, decode, eager_steps)
    stop.record()
    torch.cuda.synchronize()
    eager_ms = max_over_ranks(start.elapsed_time(stop), world) / eager_steps
    seq.rollback()

    # ---- roofline of the decode kernel (the clock window extends over it) ----
    from trpg_b200.compressed_kv_kernels import dequant, set_dequant
    rule = dequant()
    sec, bytes_per_launch, replays = time_kernel(seq, decode)
    clocks.stop()
    sec = max_over_ranks(sec, world)
    # The same launches under the other dequantization rule, for comparison.
    other = 'exact' if rule == 'folded' else 'folded'
    set_dequant(other)
    sec_other = max_over_ranks(time_kernel(seq, decode, min_seconds=0.2)[0], world)
    set_dequant(rule)
    peak, peak_kind = peaks()
    achieved = bytes_per_launch / sec / 1e9
    traffic = None
    tfile = ROOT / 'profiles' / 'traffic_attn_q8_decode.json'
    if tfile.exists():
        traffic = json.loads(tfile.read_text()).get('bytes_per_launch')

    # ---- the compaction every 128th step adds, charged per step -------------
    compact_s = max_over_ranks(compaction_seconds(seq), world)
    amortised_ms = LAYERS * compact_s * 1e3 / ROLLBACK
    ms = loop_ms / args.steps + amortised_ms          # per step

    # ---- end to end through the public API with host buffers -----------------
    e2e = e2e_run(seq, args, world, device, decode, stream)
    e2e_ms = e2e['ms'] + amortised_ms

    value = world / (ms * 1e-3)
    line = {'metric': METRIC, 'value': value, 'unit': 'tok/s', 'n_gpus': world,
            'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': ms,
            'us_per_step': ms * 1e3, 'us_per_layer': ms * 1e3 / LAYERS,
            'us_per_step_loop': loop_ms * 1e3 / args.steps,
            'us_per_step_eager': eager_ms * 1e3,
            'step_issue': 'one CUDA graph per step position of the cycle (append + decode per '
                          'layer, outputs stacked), replayed once per step; us_per_step_eager '
                          'issues the same calls from Python',
            'compaction_us_per_layer': compact_s * 1e6,
            'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None,
            'dtype': 'u8/bf16', 'data': 'synthetic (seeded N(0,1), 1% outlier channels x8)',
            'config': config(args, world),
            'roofline': {'bound': 'hbm', 'achieved': achieved, 'peak': peak, 'unit': 'GB/s',
                         'frac': achieved / peak, 'traffic': traffic, 'peak_source': peak_kind,
                         'kernel': 'attn_kernel<8,256,1,bf16>',
                         'bytes_per_launch': bytes_per_launch, 'us_per_launch': sec * 1e6,
                         'launches_timed': replays * LAYERS, 'dequant': rule,
                         'other_rule': {'dequant': other, 'us_per_launch': sec_other * 1e6,
                                        'frac': bytes_per_launch / sec_other / 1e9 / peak}},
            'hbm_gbs_step': LAYERS * bytes_per_launch / (ms * 1e-3) / 1e9,
            'clocks': clocks.summary(),
            'e2e': {'value': world / (e2e_ms * 1e-3), 'unit': 'tok/s',
                    'h2d_bytes_per_step': e2e['h2d'], 'd2h_bytes_per_step': e2e['d2h'],
                    'us_per_step': e2e_ms * 1e3,
                    'eager': {'value': world / ((e2e['eager_ms'] + amortised_ms) * 1e-3),
                              'us_per_step': (e2e['eager_ms'] + amortised_ms) * 1e3}},
            'gpu_launches': launches}
    del seq
    torch.cuda.empty_cache()
    # The partitionings the multi-GPU path is built for, at every N.
    line['batch_sharded'] = measure_extra('c3', args, world, rank, device)
    line['split_kv'] = measure_extra('c5', args, world, rank, device)
    # The long-context Q4 launch under the other rule (the folded rule's
    # fewer instructions per code matter most at 4 bits).
    set_dequant(other)
    alt = measure_extra('c5', args, world, rank, device, min_steps=5)
    set_dequant(rule)
    line['split_kv']['other_rule'] = {'dequant': other,
                                      'us_per_launch_max_rank': alt['roofline']['us_per_launch_max_rank'],
                                      'frac_rank0': alt['roofline']['frac_rank0']}
    if rank == 0 and world == 1 and not args.no_cpu:
        torch.cuda.empty_cache()
        base = cpu_reference(args.cpu_steps, 1, one_thread_steps=args.cpu_one_thread_steps)
        line['cpu_baseline'] = {k: base[k] for k in ('value', 'unit', 'cores', 'kind', 'sample')}
        if 'one_thread' in base:
            line['cpu_baseline']['one_thread'] = base['one_thread']
    if rank == 0:
        print(json.dumps(line), flush=True)


def e2e_run(seq, args, world, device, decode, stream):
    """The decode step end to end: every step copies its query and new
    key/value rows from pinned host memory into a device staging buffer
    (one host-to-device copy), runs the 8 layers through the public API
    (``append_for_attention`` + ``compressed_kv_decode``) and reads the 8
    outputs back into host memory (one device-to-host copy the host waits
    for); warmed up, then ``args.steps`` steps timed (wall clock around a
    synchronised loop, max over ranks).

    The step runs as its CUDA graph, captured from those API calls with the
    two copies inside it (a memcpy node from step i's pinned input row at
    the head, one into the pinned output buffer at the tail), the way a
    serving loop replays a decode step; the host waits on an event recorded
    after the replay.  The same loop issuing the copies and the API calls
    eagerly from Python is reported beside it."""
    n = seq.q.shape[0]
    # One pinned buffer per step: q, k, v of all layers back to back.
    parts = (seq.q, seq.kn, seq.vn)
    flat = torch.cat([t.reshape(n, -1) for t in parts], 1).cpu().pin_memory()
    sizes = [t[0].numel() for t in parts]
    shapes = [t.shape[1:] for t in parts]
    dev_in = torch.empty(flat.shape[1], dtype=flat.dtype, device=device)
    q, kn, vn = (list(x.view(shape).unbind(0)) for x, shape in zip(dev_in.split(sizes), shapes))
    host_out = torch.empty(LAYERS, 1, HQ, 1, D, dtype=torch.bfloat16).pin_memory()
    dev_out = torch.empty(host_out.shape, dtype=host_out.dtype, device=device)
    cycle = ROLLBACK - 1
    count = min(cycle, n, max(args.steps, args.warmup, 3))
    rows = [flat[i] for i in range(n)]          # the steps' pinned input rows, made once
    graphs = capture_steps(seq, decode, count, lambda i: (q, kn, vn), stream, dev_out,
                           before=lambda i: dev_in.copy_(rows[i], non_blocking=True),
                           after=lambda i: host_out.copy_(dev_out, non_blocking=True))
    done = torch.cuda.Event()

    def wait_done():
        # Spin on the event: the host resumes as soon as the copy lands
        # instead of after a blocking wake-up.
        done.record(stream)
        while not done.query():
            pass

    def graph_steps(k):
        with torch.cuda.stream(stream):
            for s in range(k):
                graphs[(s % cycle) % count].replay()
                wait_done()

    outs = [None] * LAYERS

    def eager_steps(k):
        with torch.cuda.stream(stream):
            for s in range(k):
                i = s % cycle
                if i == 0 and s:
                    seq.rollback()
                dev_in.copy_(rows[i], non_blocking=True)
                with torch.inference_mode():
                    for li, layer in enumerate(seq.layers):
                        view = layer.append_for_attention(kn[li], vn[li])
                        outs[li] = compressed_kv_decode(q[li], view, SCALE)
                        layer.compact_residual()
                    torch.stack(outs, out=dev_out)
                host_out.copy_(dev_out, non_blocking=True)
                wait_done()

    from trpg_b200.compressed_kv_attention import compressed_kv_decode

    def timed(fn, k):
        fn(max(3, args.warmup, count))     # every graph replayed (uploaded) once
        seq.rollback()
        barrier(world)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        fn(k)
        ms = max_over_ranks((time.perf_counter() - t0) * 1e3, world)
        seq.rollback()
        return ms / k

    graph_ms = timed(graph_steps, args.steps)
    del graphs
    eager_ms = timed(eager_steps, min(args.steps, 4 * cycle))
    return {'ms': graph_ms, 'eager_ms': eager_ms, 'h2d': flat[0].numel() * 2,
            'd2h': host_out.numel() * 2}


# ---------------------------------------------------------------------------
# The other configurations (parity-test cases; measured on request)
# ---------------------------------------------------------------------------
WORKLOADS = {
    'c3': 'batched decode: 64 sequences, ragged contexts uniform in [1024, 8192], Q8, one query '
          'token each, 16q/4kv x 256, one launch per GPU; sequences sharded over GPUs by LPT on bytes',
    'c4': 'MTP verification: 16 sequences x 4 query tokens (lower-right causal), 16384 context, Q8, '
          '16q/4kv x 256, one launch per GPU; sequences sharded over GPUs',
    'c5': 'long-context Q4 decode: 1 sequence, 131072 context, 16q/4kv x 256; split-KV over GPUs, '
          '(m, l, o) partials all-gathered over NCCL and merged',
    'prefill': 'packed prefill: one query chunk (--qlen, default 4096) over a quantized history '
               '(--history, default 32768; --bits, default 8), 16q/4kv x 256, lower-right causal; '
               'replicas only across GPUs',
}


def build_view(gen, length, n_new, bits, device):
    """Reference-reachable cache state: update(L - n) then append(n)."""
    from trpg_b200.quantized_kv import QuantizedAttentionLayer
    with torch.inference_mode():
        k, v = synthetic_kv(gen, length - n_new, device)
        layer = QuantizedAttentionLayer(bits)
        layer.update(k, v)
        del k, v
        kn = torch.randn(1, HKV, n_new, D, generator=gen, device=device).bfloat16()
        vn = torch.randn(1, HKV, n_new, D, generator=gen, device=device).bfloat16()
        view = layer.append_for_attention(kn, vn)
    return layer, view


def view_bytes_q(view, nq=1) -> int:
    """Algorithmic bytes of one attention call over `view`: codes + meta,
    exact window, query and output."""
    bits = view.bits
    per_token = 2 * D * bits // 8 + D * 8 // 128 + (D // 64) * 8
    return HKV * (view.packed_tokens * per_token + view.keys.shape[2] * 2 * D * 2) + 2 * HQ * nq * D * 2


def graph_seconds(fn, replays=20, align=None):
    """Device seconds per call of `fn`, from a CUDA graph of one call replayed
    back to back between events on the capturing stream.  ``align`` runs
    before the timed replays (a barrier, when the call waits for other
    ranks, so that no rank's time counts another rank's late start)."""
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.inference_mode():
        with torch.cuda.stream(stream):
            fn()
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            fn()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            for _ in range(3):
                graph.replay()
        if align is not None:
            stream.synchronize()
            align()
        with torch.cuda.stream(stream):
            a.record(stream)
            for _ in range(replays):
                graph.replay()
            b.record(stream)
        stream.synchronize()
        del graph
    return a.elapsed_time(b) * 1e-3 / replays


def measure_extra(w, args, world, rank, device, min_steps=20):
    """One of the other configurations at ``world`` GPUs, as a dict.

    c3 / c4: the sequences are sharded over the ranks by LPT on bytes and
    each rank runs one launch over its share (no collective); c5: each rank
    computes the (o, m, l) partial of its contiguous share of the 131072-token
    history, the partials are all-gathered over NCCL and merged.  Kernel time
    comes from CUDA-graph replays of one launch; the step (for c5 on several
    GPUs: partial, all-gather and merge, each between CUDA events) is timed
    over at least ``min_steps`` steps; every figure is the max over ranks."""
    from trpg_b200.compressed_kv_kernels import attention, combine
    from trpg_b200.sharding import lpt_partition, split_kv_range, view_bytes
    gen = torch.Generator(device=device)
    peak, peak_kind = peaks()
    if w in ('c3', 'c4'):
        if w == 'c3':
            cpu = torch.Generator().manual_seed(3)
            lengths = torch.randint(1024, 8193, (64,), generator=cpu).tolist()
            nq, bits = 1, 8
        else:
            lengths, nq, bits = [16384] * 16, 4, 8
        # Shard by bytes (the state rule gives P and R from L).
        def pr(length):
            p = 128 * max(0, (length - nq - 128) // 128)
            return p, length - p
        parts = lpt_partition([view_bytes(*pr(L), HKV, D, bits) for L in lengths], world)
        mine = parts[rank]
        gen.manual_seed(1000 * (3 if w == 'c3' else 4) + rank)
        views, queries = [], []
        for i in mine:
            _, view = build_view(gen, lengths[i], nq, bits, device)
            views.append(view)
            queries.append(torch.randn(1, HQ, nq, D, generator=gen, device=device).bfloat16())
        fn = lambda: attention(queries, views, SCALE)
        nbytes = sum(view_bytes_q(v, nq) for v in views)
        tokens = len(lengths) * nq
    elif w == 'c5':
        gen.manual_seed(5)
        _, view = build_view(gen, 131072, 1, 4, device)
        q = torch.randn(1, HQ, 1, D, generator=gen, device=device).bfloat16()
        units, resid = view.packed_tokens // 128, view.keys.shape[2]
        rng = split_kv_range(units, resid, world, rank)
        if world == 1:
            fn = lambda: attention([q], [view], SCALE)
        else:
            fn = lambda: attention([q], [view], SCALE, ranges=[rng], partial=True)
        per_token = 2 * D * 4 // 8 + D * 8 // 128 + (D // 64) * 8
        nbytes = HKV * ((rng[1] - rng[0]) * 128 * per_token + (rng[3] - rng[2]) * 2 * D * 2) + 2 * HQ * D * 2
        tokens = 1
    else:
        raise SystemExit(f'unknown workload {w}')
    sec_kernel = graph_seconds(fn)
    steps = max(min_steps, args.steps)
    exchange = w == 'c5' and world > 1
    if exchange:
        import torch.distributed as dist
        gathered = None

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    with torch.inference_mode():
        def step(e=None):
            nonlocal gathered
            if e:
                e[0].record()
            out = fn()
            if exchange:
                part = out[0]
                if e:
                    e[1].record()
                if gathered is None:
                    gathered = torch.empty((world * part.shape[0], part.shape[1]), dtype=part.dtype,
                                           device=device)
                dist.all_gather_into_tensor(gathered, part)
                out = combine(gathered.view(world, *part.shape), torch.bfloat16)
            if e:
                e[2].record()
            return out
        for _ in range(max(3, args.warmup)):
            step()
        torch.cuda.synchronize()
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for i in range(steps):
            step(ev[i] if exchange else None)
        b.record()
        torch.cuda.synchronize()
        barrier(world)
    eager_ms = max_over_ranks(a.elapsed_time(b) / steps, world)
    k_us = max_over_ranks(sec_kernel * 1e6, world)
    achieved = nbytes / sec_kernel / 1e9
    # c3 / c4: the step is the one launch, issued as a replayed CUDA graph
    # (the 64- or 16-sequence argument table costs about 7 us of host time
    # per sequence when issued eagerly, which 'ms_per_step_eager' shows).
    ms = eager_ms if w == 'c5' else k_us * 1e-3
    out = {'workload': WORKLOADS[w], 'value': tokens / (ms * 1e-3), 'unit': 'tok/s',
           'n_gpus': world, 'steps': steps, 'ms_per_step': ms, 'ms_per_step_eager': eager_ms,
           'scaling': 'strong' if w == 'c5' else 'strong (fixed batch sharded)',
           'dtype': 'u4/bf16' if w == 'c5' else 'u8/bf16',
           'roofline': {'bound': 'hbm', 'achieved_rank0': achieved, 'peak': peak, 'unit': 'GB/s',
                        'frac_rank0': achieved / peak, 'peak_source': peak_kind,
                        'bytes_per_launch_rank0': nbytes, 'us_per_launch_max_rank': k_us}}
    if exchange:
        compute = statistics.median(e[0].elapsed_time(e[1]) for e in ev) * 1e3
        combine_us = statistics.median(e[1].elapsed_time(e[2]) for e in ev) * 1e3
        out['us_partial_max_rank'] = max_over_ranks(compute, world)
        out['us_allgather_combine_max_rank'] = max_over_ranks(combine_us, world)
        # The same exchange over NVLink peer mappings instead of NCCL: one
        # launch per rank publishes its partial into every rank's buffer and
        # merges once all have arrived.  Timed as CUDA-graph replays of the
        # step (partial + exchange) and of the exchange alone.
        from trpg_b200.sharding import PeerExchange
        with torch.inference_mode():
            part0 = fn()[0]
        px = PeerExchange(part0.shape[0], D)
        try:
            # One checked exchange first: the merged output must equal the
            # NCCL path's and no wait may give up, before any timing.
            with torch.inference_mode():
                dist.all_gather_into_tensor(gathered, part0)
                want = combine(gathered.view(world, *part0.shape), torch.bfloat16)
                got = px.combine(part0, torch.bfloat16)
            bad = float(px.error() != 0 or not torch.equal(got, want))
            bad = max_over_ranks(bad, world)
            if bad:
                out['peer_exchange'] = {'unavailable': 'the checked exchange disagreed with NCCL or gave up'}
            else:
                align = lambda: (barrier(world), torch.cuda.synchronize())
                step_s = graph_seconds(lambda: px.combine(fn()[0], torch.bfloat16), replays=200, align=align)
                ex_s = graph_seconds(lambda: px.combine(part0, torch.bfloat16), replays=200, align=align)
                failed = px.error()
                step_us = max_over_ranks(step_s * 1e6, world)
                out['peer_exchange'] = {'us_per_step_max_rank': step_us,
                                        'us_exchange_combine_max_rank': max_over_ranks(ex_s * 1e6, world),
                                        'value': tokens / (step_us * 1e-6), 'unit': 'tok/s',
                                        'wait_gave_up': bool(max_over_ranks(float(failed), world))}
        finally:
            px.close()
    return out


def extra_workload(args, world, rank, local):
    from trpg_b200 import _native
    _native.load()
    device = torch.device('cuda', local)
    torch.cuda.set_device(device)
    clocks = Clocks(local)
    clocks.start()
    line = measure_extra(args.workload, args, world, rank, device)
    clocks.stop()
    line = {'metric': f'{args.workload}: decode attention tokens/s', **line,
            'warmup': args.warmup, 'higher_is_better': True, 'data': 'synthetic',
            'clocks': clocks.summary()}
    if rank == 0:
        print(json.dumps(line), flush=True)


def prefill_workload(args, world, rank, local):
    """Packed prefill (``compressed_kv_prefill``) against dequantize + SDPA on
    the same view, both device-timed from CUDA-graph replays: the shapes of
    the reference's prefill profile (scripts/profile_compressed_prefill.py:36-47)."""
    from torch.nn.attention.bias import causal_lower_right
    from torch.nn import functional as F
    from trpg_b200 import _native
    from trpg_b200.compressed_prefill_attention import compressed_kv_prefill
    _native.load()
    device = torch.device('cuda', local)
    torch.cuda.set_device(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(104 + rank)
    qlen, history, bits = args.qlen, args.history, args.bits
    layer, view = build_view(gen, history + qlen, qlen, bits, device)
    q = torch.randn(1, qlen, HQ, D, generator=gen, device=device).bfloat16().transpose(1, 2)
    bias = causal_lower_right(qlen, view.length)

    def packed():
        out = compressed_kv_prefill(q, view, SCALE)
        assert out is not None
        return out

    def unpack_sdpa():
        keys = torch.cat((layer.key_bank.unpack(q.dtype), view.keys), -2)
        values = torch.cat((layer.value_bank.unpack(q.dtype), view.values), -2)
        return F.scaled_dot_product_attention(q, keys, values, attn_mask=bias, enable_gqa=True,
                                              scale=SCALE)

    with torch.inference_mode():
        err = (packed().float() - unpack_sdpa().float()).abs().max().item()
    clocks = Clocks(local)
    clocks.start()
    sec = max_over_ranks(graph_seconds(packed, replays=max(3, args.steps)), world)
    clocks.stop()
    sec_ref = max_over_ranks(graph_seconds(unpack_sdpa, replays=max(3, args.steps)), world)
    P, R = view.packed_tokens, view.keys.shape[2]
    visible = qlen * P + qlen * (R - qlen) + qlen * (qlen + 1) // 2
    flops = 4 * HQ * D * visible
    path = ROOT / 'MEASURED_PEAKS.json'
    peak = json.loads(path.read_text()).get('bf16_tflops') if path.exists() else None
    peak, kind = (float(peak), 'measured') if peak else (1590.0, 'fallback')
    achieved = flops / sec / 1e12
    line = {'metric': 'prefill: query tokens/s', 'workload': WORKLOADS['prefill'],
            'value': world * qlen / sec, 'unit': 'tok/s', 'n_gpus': world, 'steps': args.steps,
            'higher_is_better': True, 'scaling': 'weak (replicas)', 'dtype': f'u{bits}/bf16',
            'data': 'synthetic', 'ms_per_call': sec * 1e3, 'history': P + R - qlen, 'qlen': qlen,
            'dequant_sdpa_ms': sec_ref * 1e3, 'speedup_vs_dequant_sdpa': sec_ref / sec,
            'max_abs_vs_dequant_sdpa': err,
            'roofline': {'bound': 'tensor', 'achieved': achieved, 'peak': peak, 'unit': 'TFLOP/s',
                         'frac': achieved / peak, 'peak_source': kind, 'flops_per_launch': flops},
            'clocks': clocks.summary()}
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=1024)
    ap.add_argument('--warmup', type=int, default=16)
    ap.add_argument('--impl', choices=('b200', 'reference'), default='b200')
    ap.add_argument('--dequant', choices=('exact', 'folded'), default=None,
                    help='dequantization rule of the attention kernel (default: the library '
                         'default, TRPG_CKV_DEQUANT or exact)')
    ap.add_argument('--cpu-steps', type=int, default=24)
    ap.add_argument('--cpu-one-thread-steps', type=int, default=3)
    ap.add_argument('--no-cpu', action='store_true')
    ap.add_argument('--workload', choices=('c2',) + tuple(WORKLOADS), default='c2',
                    help='c2 (default) is the headline 32K decode step; c3/c4/c5 measure the '
                         'other configurations')
    ap.add_argument('--history', type=int, default=32768, help='prefill: history tokens')
    ap.add_argument('--qlen', type=int, default=4096, help='prefill: query chunk length')
    ap.add_argument('--bits', type=int, choices=(4, 8), default=8, help='prefill: code width')
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error('--warmup must be >= 3')
    world, rank, local = init_dist()
    if args.dequant and args.impl == 'b200':
        from trpg_b200.compressed_kv_kernels import set_dequant
        set_dequant(args.dequant)
    try:
        if args.impl == 'reference':
            reference_arm(args, world, rank)
        elif args.workload == 'prefill':
            prefill_workload(args, world, rank, local)
        elif args.workload != 'c2':
            extra_workload(args, world, rank, local)
        else:
            b200_arm(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == '__main__':
    sys.path.insert(0, str(ROOT))
    main()
