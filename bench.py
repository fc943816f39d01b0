"""Benchmark of ma_deform_attn on B200: device-timed microseconds per call, roofline, CPU baseline, end to end.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c1h] [--mode auto] [--impl ours|reference]
    python bench.py --sweep [--dtype ...]        # the fused/project crossover table that fits FUSED_LIMIT_SM100

A step is one ma_deform_attn call on one batch of the workload (default c1h: RT-DETR 640x640 decoder layer, float16,
B=1 image per GPU, Q=300, C=256, H=8, D=32, L=3, P=4). Timing follows upstream bench/bench.py:40-61 (calls captured
in a CUDA graph, device-timed with CUDA events), with one change: every call reads a different input set from a pool
whose total size exceeds twice the 126 MB L2, so each call's memory comes from HBM ("l2": "rotating inputs > 2x L2").
With --gpus N under torchrun each rank runs its own images (batch sharding, no collective in the data path), the
timed region is bracketed by barriers and synchronisation, and the slowest rank's time is reported.

--layer times the whole deformable attention layer instead (deform_attn_layer: query -> offsets and softmaxed
weights -> attention -> output_proj), beside the same layer with the producer in torch operators on the GPU (two
nn.Linear, softmax, location arithmetic; then this library's ma_deform_attn) and the all-torch layer on the GPU
(deform_attn_layer_reference: grid_sample), on the same rotating inputs.

--backward times training steps instead: forward + backward of ma_deform_attn (gradients of memory, value_weight,
value_bias, sampling_locations and attention_weights), beside the same through the torch reference (nn.Linear +
grid_sample, autograd) on the GPU, both captured in CUDA graphs on rotating inputs; plus the backward kernel alone
with its roofline. --layer --backward times a training step of the whole layer (every gradient, this library's
kernels only) beside the all-torch layer under autograd.

--output-proj adds the decoder's output_proj to every call; --outproj-plan chooses whether it runs in the sampler's
cluster epilogue or as a chained GEMM (default: the library's automatic plan).

--impl reference times the CPU implementation of the same call: upstream's algorithm (nn.Linear + grid_sample, the
oracle's torch_port on torch's CPU operators) with all host threads, on rank 0 only.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from marearts_tinydeform_b200 import (_native, choose_mode, deform_attn_layer, ma_deform_attn,  # noqa: E402
                                      ma_deform_attn_reference, sampling_producer_reference, workloads)
from marearts_tinydeform_b200 import _pick_with_outproj  # noqa: E402

L2_BYTES = 126 * 2 ** 20
METRIC = 'µs per ma_deform_attn call (device-timed) and achieved HBM GB/s vs peak'


def peaks():
    path = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p['hbm_gbs']), 'measured'
    except (OSError, KeyError, ValueError):
        return 6650.0, 'fallback'


def committed_traffic(kernel, config):
    """DRAM bytes per launch from the committed ncu summary (profiles/traffic.json), or None."""
    try:
        with open(os.path.join(ROOT, 'profiles', 'traffic.json')) as f:
            return json.load(f).get(f'{kernel}@{config}')
    except (OSError, ValueError):
        return None


class ClockSampler:
    """nvidia-smi samples (SM clock, throttle reasons) taken every 100 ms while the timed region runs."""

    QUERY = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
             'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
             'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--id={self.index}', f'--query-gpu={self.QUERY}',
                                          '--format=csv,noheader,nounits', '-lms', '100'],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(',')])

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['nvidia-smi unavailable'], 'samples': 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace('.', '').isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace('.', '').isdigit()]
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[5:9]) if v.lower() == 'active'})
        return {'sm_mhz': statistics.median(sm) if sm else None, 'sm_max_mhz': max(mx) if mx else None,
                'reasons': reasons, 'samples': len(self.rows)}


def input_pool(cfg_name, B, device, min_bytes):
    """Distinct input sets (memory, loc, attn per set; weights shared) totalling at least min_bytes."""
    base = workloads.make_inputs(cfg_name, seed=0, B=B, device=device, generate_on_device=True)
    per_set = sum(t.numel() * t.element_size() for t in (base[0], base[5], base[6]))
    n = max(2, -(-min_bytes // per_set))
    g = torch.Generator(device=device).manual_seed(1234)
    pool = []
    B_, Q_, H_, L_, P_ = base[6].shape
    for i in range(n):
        mem = torch.randn(base[0].shape, generator=g, device=device).to(base[0].dtype)
        loc = torch.rand(base[5].shape, generator=g, device=device).to(base[5].dtype)
        logits = torch.randn(B_, Q_, H_, L_ * P_, generator=g, device=device)
        attn = logits.softmax(-1).view(base[6].shape).to(base[6].dtype)
        pool.append((mem, loc, attn))
    pool[0] = (base[0], base[5], base[6])
    return base, pool


def graph_time_us(fn, steps, warmup):
    """Device time per call of `fn(i)`, i = 0 .. steps-1, captured as one CUDA graph (upstream bench.py:40-61)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(max(warmup, 3)):
            fn(i)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    before = _native.launch_count()
    with torch.cuda.graph(g):
        for i in range(steps):
            fn(i)
    launches = _native.launch_count() - before
    g.replay()
    torch.cuda.synchronize()
    return g, launches


def replay_times(g, steps, reps=1):
    """Device time per call (µs) of each of `reps` replays of a graph of `steps` calls, CUDA events on the current
    stream. Before each start event a short spin kernel keeps the stream busy while the host submits the graph, so
    the timed region holds the calls only, not the host's submission latency."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    out = []
    for _ in range(reps):
        torch.cuda.synchronize()
        torch.cuda._sleep(100_000)
        start.record()
        g.replay()
        end.record()
        end.synchronize()
        out.append(start.elapsed_time(end) * 1e3 / steps)
    return out


def time_graph(g, steps, reps=1):
    """Median device time per call (µs) over `reps` replays (see replay_times)."""
    return statistics.median(replay_times(g, steps, reps))


def l2_gather_peak(dev, kinds, visits=1 << 24, reps=10):
    """Measured L2 random-row gather rate of this GPU for each (row_bytes, wide) in kinds: td_probe_row_gather over
    an 8 MiB buffer (L2-resident; the c1h value and memory are 4.3 MB each) with every SM, `reps` launches timed
    with CUDA events after two warm-up launches. Returns {key: {'GBps', 'G_rows_per_s'}}, key '64B' or '128B_v8'."""
    buf = torch.randint(0, 255, (8 << 20,), dtype=torch.uint8, device=dev)
    grid = torch.cuda.get_device_properties(dev).multi_processor_count * 8
    sink = torch.empty(grid * 1024, dtype=torch.int32, device=dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    out = {}
    for row_bytes, wide in kinds:
        for _ in range(2):
            n = _native.probe_row_gather(buf, row_bytes, visits, wide, grid=grid, sink=sink)
        torch.cuda.synchronize()
        start.record()
        for _ in range(reps):
            _native.probe_row_gather(buf, row_bytes, visits, wide, grid=grid, sink=sink)
        end.record()
        end.synchronize()
        t = start.elapsed_time(end) * 1e-3 / reps
        out[probe_key(row_bytes, wide)] = {'GBps': round(n * row_bytes / t / 1e9, 1),
                                           'G_rows_per_s': round(n / t / 1e9, 3)}
    return out


def probe_key(row_bytes, wide):
    return f'{row_bytes}B' + ('_v8' if wide else '')


def gather_kind(kind, C, D, e):
    """(row_bytes, 32-byte loads) of the corner rows a gather kernel reads: the sampler reads D-wide head slices
    (32-byte loads from 128 bytes on), the fused kernel C-wide memory rows (16-byte loads)."""
    if kind == 'sample':
        rb = D * e
        return rb, rb >= 128 and rb % 32 == 0
    return C * e, False


def dist_setup(n_gpus):
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device('cuda', local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier_max(value, world):
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device='cuda')
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cpu_time_us(cfg_name, budget_s=10.0, max_calls=50):
    """The CPU path (oracle torch_port = upstream's nn.Linear + grid_sample) on all host threads, bounded."""
    from oracle import deform_oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    args = workloads.make_inputs(cfg_name, seed=0)
    with torch.inference_mode():
        for _ in range(2):
            deform_oracle.torch_port(*args)
        times, t_end = [], time.perf_counter() + budget_s
        while len(times) < max_calls and time.perf_counter() < t_end:
            t0 = time.perf_counter()
            deform_oracle.torch_port(*args)
            times.append(time.perf_counter() - t0)
    return statistics.median(times) * 1e6, threads, len(times)


def resolved_mode(cfg_name, mode):
    """The order `mode` runs on B200 for this workload ('auto' resolved with FUSED_LIMIT_SM100, the table compute
    capability 10.x uses), so that the CPU arm names the configuration of the GPU arm."""
    if mode != 'auto':
        return mode
    import marearts_tinydeform_b200 as td
    a = workloads.make_inputs(cfg_name, seed=0, device='meta')
    return td._pick(a[0], a[1], a[5].shape[1], a[5].shape[2], a[5].shape[3], a[5].shape[4],
                    limits=td.FUSED_LIMIT_SM100)


def run_reference_arm(args):
    rank = int(os.environ.get('RANK', '0'))
    world = int(os.environ.get('WORLD_SIZE', '1'))
    if rank != 0:
        return
    # exactly W untimed and K timed calls of the CPU path (the upstream algorithm on torch's CPU operators, all host
    # threads), one call of the workload per step
    from oracle import deform_oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    inputs = workloads.make_inputs(args.config, seed=0)
    with torch.inference_mode():
        for _ in range(args.warmup):
            deform_oracle.torch_port(*inputs)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            deform_oracle.torch_port(*inputs)
        us = (time.perf_counter() - t0) / max(1, args.steps) * 1e6
    n = args.steps
    cfg = workloads.CONFIGS[args.config]
    line = {
        'metric': METRIC, 'value': round(us, 2), 'unit': 'us', 'impl': 'reference', 'n_gpus': args.gpus,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(us / 1e3, 4), 'higher_is_better': False,
        'scaling': 'weak', 'vs_baseline': None, 'dtype': str(cfg['dtype']).replace('torch.', ''),
        'data': 'synthetic (seeded, BASELINE config shapes)',
        'config': config_dict(args.config, world, resolved_mode(args.config, args.mode)),
        'cpu_baseline': {'value': round(us, 2), 'unit': 'us', 'cores': threads, 'kind': 'port',
                         'sample': f'{n} timed calls of {args.config} (B={cfg["B"]}), mean, torch CPU ops, '
                                   f'{threads} threads'},
        'e2e': {'value': round(us, 2), 'unit': 'us', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)


def config_dict(name, world, mode, where='GPU'):
    c = workloads.CONFIGS[name]
    return {'workload': f'{name}: B={c["B"]} per {where}, Q={c["Q"]}, C={c["C"]}, H={c["H"]}, D={c["D"]}, '
                        f'levels={c["levels"]}, P={c["P"]}',
            'global_batch': c['B'] * world, 'queries': c['Q'], 'mode': mode,
            'parallelism': f'batch-shard x{world}' if world > 1 else 'single GPU',
            'l2': 'rotating inputs > 2x L2 (126 MB) between calls'}


def kernel_bytes(kind, B, Q, N, C, H, D, L, P, e, bias=True):
    HD = H * D
    if kind == 'fused':
        return workloads.algorithmic_bytes(B, Q, N, C, H, D, L, P, e, bias)
    if kind == 'proj':
        return e * (B * N * C + HD * C + (HD if bias else 0) + B * N * HD)
    if kind == 'sample':
        return e * (B * N * HD + 3 * B * Q * H * L * P + B * Q * HD)
    raise ValueError(kind)


def call_roofline(kernels, t_call, hbm, peak_kind, l2_peaks, config, B, Q, N, C, H, D, L, P, e, bias, gather,
                  gather_row_bytes, l2_key):
    """The call's roofline: its compulsory HBM bytes (memory and weights read once, locations and weights read,
    output written) over its device time, against the measured HBM peak; beside it each kernel's own algorithmic
    bytes over its standalone time, and the gather kernel's corner-row bytes over its time against the measured L2
    random-row gather rate for rows of that size."""
    alg = workloads.algorithmic_bytes(B, Q, N, C, H, D, L, P, e, bias)
    achieved = alg / (t_call * 1e-6) / 1e9
    per = {}
    traffic = 0
    for k, t in kernels.items():
        kb = kernel_bytes(k, B, Q, N, C, H, D, L, P, e, bias)
        tr = committed_traffic(k, config)
        traffic = None if tr is None or traffic is None else traffic + tr
        d = {'us': round(t, 3), 'algorithmic_bytes': kb, 'achieved': round(kb / (t * 1e-6) / 1e9, 1),
             'frac': round(kb / (t * 1e-6) / 1e9 / hbm, 4), 'traffic': tr}
        if k == gather:
            gb = B * Q * H * L * P * 4 * gather_row_bytes
            l2a = gb / (t * 1e-6) / 1e9
            d.update({'bound': 'l2 gather', 'gather_bytes': gb, 'gather_row_bytes': gather_row_bytes,
                      'l2_achieved': round(l2a, 1), 'l2_peak': l2_peaks[l2_key]['GBps'], 'l2_peak_rows': l2_key,
                      'l2_frac': round(l2a / l2_peaks[l2_key]['GBps'], 4)})
        else:
            d['bound'] = 'hbm'
        per[k] = d
    return {'bound': 'hbm', 'scope': 'whole call: compulsory HBM bytes / device time per call',
            'achieved': round(achieved, 1), 'peak': hbm, 'unit': 'GB/s', 'frac': round(achieved / hbm, 4),
            'peak_source': peak_kind, 'algorithmic_bytes': alg, 'traffic': traffic,
            'traffic_source': 'profiles/traffic.json (ncu dram bytes per launch, summed over the call)',
            'kernels': per, 'l2_frac': per[gather]['l2_frac'], 'l2_peak': per[gather]['l2_peak'],
            'l2_peak_source': 'measured in this run (td_probe_row_gather, 8 MiB L2-resident buffer, all SMs)'}


def run_ours(args):
    rank, world, local = dist_setup(args.gpus)
    dev = torch.device('cuda', local)
    _native.load()
    cfg = workloads.CONFIGS[args.config]
    B = cfg['B']
    base, pool = input_pool(args.config, B, dev, 2 * L2_BYTES)
    W, bias, shapes, starts = base[1], base[2], base[3], base[4]
    mode = args.mode if args.mode != 'auto' else choose_mode(base[0], W, base[5])
    N, C, H, D, L, P, Q = base[0].shape[1], cfg['C'], cfg['H'], cfg['D'], len(cfg['levels']), cfg['P'], cfg['Q']
    e = base[0].element_size()
    outs = [torch.empty(B, Q, H * D, dtype=base[0].dtype, device=dev) for _ in range(2)]
    # optional value padding mask: a seeded random fraction of every image's tokens padded
    mask = None
    if args.padding_mask > 0:
        gm = torch.Generator(device=dev).manual_seed(77)
        mask = torch.rand(B, N, generator=gm, device=dev) < args.padding_mask

    # optional output_proj (the decoder's nn.Linear on the result, [C, H * D]), chained behind the attention
    wo = bo = None
    if args.output_proj:
        go = torch.Generator(device=dev).manual_seed(78)
        wo = ((torch.rand(C, H * D, generator=go, device=dev) * 2 - 1) * (6 / (C + H * D)) ** 0.5).to(W.dtype)
        bo = torch.zeros(C, dtype=W.dtype, device=dev)
        if args.mode == 'auto':  # the order auto takes with output_proj
            mode = _pick_with_outproj(base[0], W, Q, H, L, P, wo)

    def call(i):
        mem, loc, attn = pool[i % len(pool)]
        return ma_deform_attn(mem, W, bias, shapes, starts, loc, attn, mode=args.mode, value_padding_mask=mask,
                              output_weight=wo, output_bias=bo)

    with torch.inference_mode():
        g, launches = graph_time_us(call, args.steps, args.warmup)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()
        with ClockSampler(local) as clocks:
            time.sleep(0.25)
            replays = replay_times(g, args.steps, reps=max(1, args.reps))
        t_call = barrier_max(statistics.median(replays), world)
        t_min = barrier_max(min(replays), world)
        del g

        # per-kernel times of the path the call took (same rotation, same stream), for the roofline
        kernels = {}
        if mode == 'fused':
            kernels['fused'] = t_call
        else:
            hm = [_native.value_proj(pool[j][0], W, bias, H, head_major=True) for j in range(len(pool))]
            gp, _ = graph_time_us(lambda i: _native.value_proj(pool[i % len(pool)][0], W, bias, H, head_major=True),
                                  args.steps, args.warmup)
            kernels['proj'] = time_graph(gp, args.steps, reps=max(1, args.reps))
            del gp
            gs, _ = graph_time_us(lambda i: _native.sample_head_major(hm[i % len(pool)], shapes, starts,
                                                                      pool[i % len(pool)][1], pool[i % len(pool)][2]),
                                  args.steps, args.warmup)
            kernels['sample'] = time_graph(gs, args.steps, reps=max(1, args.reps))
            del gs, hm
        hbm, peak_kind = peaks()
        gather = 'fused' if mode == 'fused' else 'sample'
        g_rb, g_wide = gather_kind(gather, C, D, e)
        probe_rb = min(512, 1 << (g_rb.bit_length() - 1))  # the probe reads power-of-two rows of at most 512 bytes
        l2_peaks = l2_gather_peak(dev, [(probe_rb, g_wide and probe_rb >= 32)])
        roofline = call_roofline(kernels, t_call, hbm, peak_kind, l2_peaks, args.config, B, Q, N, C, H, D, L, P, e,
                                 bias is not None, gather, g_rb, probe_key(probe_rb, g_wide and probe_rb >= 32))

        # hot-L2 time (upstream's method: one input set replayed)
        gh, _ = graph_time_us(lambda i: ma_deform_attn(base[0], W, bias, shapes, starts, base[5], base[6],
                                                       mode=args.mode, value_padding_mask=mask,
                                                       output_weight=wo, output_bias=bo),
                              args.steps, args.warmup)
        t_hot = barrier_max(time_graph(gh, args.steps, reps=3), world)
        del gh

        # end to end through the public API: pinned host inputs copied in, result copied out, every step. A serving
        # loop stages a step's inputs in one pinned host buffer (each tensor at a 256-byte aligned offset) and copies
        # it in with one transfer: a small pinned copy costs ~10-20 us of latency whatever its size, so seven copies
        # per step took ~2.4x the time of the one 4.3 MB transfer that dominates.
        parts = [t for t in (base[0], W, bias, shapes, starts, base[5], base[6]) if t is not None]
        offs, total = [], 0
        for t in parts:
            offs.append(total)
            total += (t.numel() * t.element_size() + 255) // 256 * 256
        host_buf = torch.empty(total, dtype=torch.uint8).pin_memory()
        for t, o in zip(parts, offs):
            nb = t.numel() * t.element_size()
            host_buf[o:o + nb].copy_(t.detach().contiguous().view(-1).view(torch.uint8).cpu())
        h2d = sum(t.numel() * t.element_size() for t in parts)
        out_host = torch.empty((B, Q, C if wo is not None else H * D), dtype=base[0].dtype).pin_memory()
        d2h = out_host.numel() * out_host.element_size()
        e2e_steps = max(10, min(args.steps, 200))

        # A serving loop double-buffers: step k's inputs are copied in on a copy stream while step k - 1 computes
        # (two device buffers; a buffer is refilled only after the step that read it has finished), and each
        # step's result is copied out on the compute stream. Every copy of every step is inside the timed region.
        compute = torch.cuda.current_stream()
        copy_stream = torch.cuda.Stream()
        dev_bufs = [torch.empty(total, dtype=torch.uint8, device=dev) for _ in range(2)]
        views = [[buf[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape) for t, o in zip(parts, offs)]
                 for buf in dev_bufs]
        ready = [torch.cuda.Event() for _ in range(2)]
        free = [torch.cuda.Event() for _ in range(2)]
        for ev in free:
            ev.record(compute)

        def e2e_step(k):
            j = k % 2
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(free[j])
                dev_bufs[j].copy_(host_buf, non_blocking=True)
                ready[j].record(copy_stream)
            compute.wait_event(ready[j])
            dev_in = list(views[j])
            if bias is None:
                dev_in.insert(2, None)
            out = ma_deform_attn(*dev_in, mode=args.mode, value_padding_mask=mask, output_weight=wo, output_bias=bo)
            free[j].record(compute)
            out_host.copy_(out, non_blocking=True)

        for k in range(3):
            e2e_step(k)
        torch.cuda.synchronize()
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(compute)
        for ev in free:  # no copy of the timed steps starts before the timed region
            ev.record(compute)
        for k in range(e2e_steps):
            e2e_step(k)
        end.record(compute)
        end.synchronize()
        t_e2e = barrier_max(start.elapsed_time(end) * 1e3 / e2e_steps, world)

    sharded = None if args.no_sharded else sharded_record(args, world, dev)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        us, threads, n = cpu_time_us(args.config)
        cpu = {'value': round(us, 2), 'unit': 'us', 'cores': threads, 'kind': 'port',
               'sample': f'{n} calls of {args.config} (B=1) on torch CPU ops (oracle torch_port), median'}
    if rank == 0:
        line = {
            'metric': METRIC, 'value': round(t_call, 3), 'unit': 'us', 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': round(t_call / 1e3, 6), 'higher_is_better': False,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': str(cfg['dtype']).replace('torch.', ''),
            'data': 'synthetic (seeded, BASELINE config shapes)',
            'config': dict(config_dict(args.config, world, mode),
                           **({'value_padding_mask': args.padding_mask} if mask is not None else {}),
                           **({'output_proj': [C, H * D], 'outproj_plan': args.outproj_plan}
                              if wo is not None else {})),
            'mode': mode, 'queries_per_s': round(B * Q * world / (t_call * 1e-6), 1),
            'replays': {'n': len(replays), 'steps_each': args.steps, 'median_us': round(t_call, 3),
                        'min_us': round(t_min, 3), 'value_is': 'median over replays (max over ranks)'},
            'hot_l2_us': round(t_hot, 3), 'kernel_us': {k: round(v, 3) for k, v in kernels.items()},
            'roofline': roofline,
            'cpu_baseline': cpu,
            'e2e': {'value': round(t_e2e, 2), 'unit': 'us', 'h2d_bytes_per_step': h2d, 'd2h_bytes_per_step': d2h},
            'gpu_launches': launches,
            'clocks': clocks.summary(),
        }
        if sharded is not None:
            line['sharded'] = sharded
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def sharded_record(args, world, dev, cfg_name='c3'):
    """The batch-sharded configuration: c3 (bfloat16, 8 images, Q=300) split over the ranks by batch_range, each
    step one ma_deform_attn_sharded call per rank with gather=True (the outputs all-gathered to every rank over NCCL;
    no collective at one rank), K steps in one CUDA graph on rotating inputs, device-timed, max over ranks; beside
    it the same steps without the gather, so the all-gather's share of the step is measured, not inferred."""
    from marearts_tinydeform_b200.shard import batch_range, ma_deform_attn_sharded
    rank = int(os.environ.get('RANK', '0'))
    cfg = workloads.CONFIGS[cfg_name]
    Bg = cfg['B']
    start, stop = batch_range(Bg, world, rank)
    b = stop - start
    base, pool = input_pool(cfg_name, b, dev, 2 * L2_BYTES)
    W, bias, shapes, starts = base[1], base[2], base[3], base[4]
    gather = world > 1

    def step(i, with_gather):
        mem, loc, attn = pool[i % len(pool)]
        return ma_deform_attn_sharded(mem, W, bias, shapes, starts, loc, attn, gather=with_gather,
                                      global_batch=Bg)

    times = {}
    with torch.inference_mode():
        for name, flag in (('no_gather', False), ('gather', gather)):
            if world > 1:
                import torch.distributed as dist
                dist.barrier()
            g, _ = graph_time_us(lambda i, f=flag: step(i, f), args.steps, args.warmup)
            if world > 1:
                dist.barrier()
            times[name] = barrier_max(time_graph(g, args.steps, reps=max(5, args.reps // 5)), world)
            del g
        out = step(0, gather)
        # the all-gather fused into the sampler (rows stored into every rank's output over NVLink): PeerGather; at
        # one rank the same kernel storing into the one output (nothing crosses NVLink)
        from marearts_tinydeform_b200.shard import PeerGather
        pg = PeerGather(Bg, cfg['Q'], cfg['H'], cfg['D'], cfg['dtype'])
        try:
            if world > 1:
                dist.barrier()
            g, _ = graph_time_us(lambda i: pg(*pool[i % len(pool)][:1], W, bias, shapes, starts,
                                              *pool[i % len(pool)][1:]), args.steps, args.warmup)
            if world > 1:
                dist.barrier()
            times['peer'] = barrier_max(time_graph(g, args.steps, reps=max(5, args.reps // 5)), world)
            del g
            torch.cuda.synchronize()
            peer = torch.equal(pg(*pool[0][:1], W, bias, shapes, starts, *pool[0][1:]).clone(), out)
            torch.cuda.synchronize()
            if _native.device_error(clear=True) != 0:
                peer = False
        finally:
            pg.close()
    N, C, H, D, L, P, Q = base[0].shape[1], cfg['C'], cfg['H'], cfg['D'], len(cfg['levels']), cfg['P'], cfg['Q']
    e = base[0].element_size()
    hbm, _ = peaks()
    alg = workloads.algorithmic_bytes(b, Q, N, C, H, D, L, P, e, bias is not None)
    t = times['gather']
    return {'workload': f'{cfg_name}: {cfg["dtype"]} B={Bg} global, {b} image(s) on rank {rank} of {world}, Q={Q}, '
                        f'C={C}, H={H}, D={D}, levels={cfg["levels"]}, P={P}',
            'global_batch': Bg, 'images_per_rank': b, 'scaling': 'strong', 'us_per_step': round(t, 3),
            'us_per_step_without_gather': round(times['no_gather'], 3),
            'allgather_share': round(max(0.0, t - times['no_gather']) / t, 4) if gather else 0.0,
            'queries_per_s': round(Bg * Q / (t * 1e-6), 1), 'gathered_shape': list(out.shape),
            'gathered_bytes_per_rank': out.numel() * out.element_size() if gather else 0,
            'per_gpu_roofline_frac': round(alg / (times['no_gather'] * 1e-6) / 1e9 / hbm, 4),
            **({'us_per_step_peer_gather': round(times['peer'], 3), 'peer_gather_equals_nccl': peer,
                'peer_gather': ('rows stored into every rank\'s output over NVLink by the sampler (PeerGather)'
                                if world > 1 else 'the same sampler storing into the one output (PeerGather, '
                                                  'one rank: nothing crosses NVLink)')}
               if 'peer' in times else {}),
            'timing': 'CUDA graph of K steps (NCCL all-gather captured), median of replays, max over ranks'}


def run_layer(args):
    """One deformable attention layer per step (see the module docstring); prints one JSON line."""
    torch.cuda.set_device(0)
    dev = torch.device('cuda', 0)
    _native.load()
    cfg = workloads.CONFIGS[args.config]
    B, Q, C, H, D, P, dtype = cfg['B'], cfg['Q'], cfg['C'], cfg['H'], cfg['D'], cfg['P'], cfg['dtype']
    L = len(cfg['levels'])
    base, pool = input_pool(args.config, B, dev, 2 * L2_BYTES)
    W, bias, shapes, starts = base[1], base[2], base[3], base[4]
    g = torch.Generator(device=dev).manual_seed(91)
    LP = H * L * P
    sw = torch.cat([torch.randn(2 * LP, C, generator=g, device=dev) * (2.0 / C ** 0.5),
                    torch.randn(LP, C, generator=g, device=dev) / C ** 0.5]).to(dtype)
    sb = (torch.randn(3 * LP, generator=g, device=dev) * 0.5).to(dtype)
    wo = ((torch.rand(C, H * D, generator=g, device=dev) * 2 - 1) * (6 / (C + H * D)) ** 0.5).to(dtype)
    bo = torch.zeros(C, dtype=dtype, device=dev)
    sets = []
    for mem, _, _ in pool:
        q = torch.randn(B, Q, C, generator=g, device=dev).to(dtype)
        ref = torch.rand(B, Q, L, args.ref_dim, generator=g, device=dev)
        if args.ref_dim == 4:
            ref[..., 2:] = 0.05 + 0.45 * ref[..., 2:]
        sets.append((q, ref.to(dtype), mem))
    mode = args.mode if args.mode != 'auto' else _pick_with_outproj(base[0], W, Q, H, L, P, wo)
    kw = dict(output_weight=wo, output_bias=bo)

    def ours(i):
        q, ref, mem = sets[i % len(sets)]
        return deform_attn_layer(q, ref, mem, shapes, starts, H, P, sw, sb, W, bias, mode=args.mode, **kw)

    def torch_producer(i):
        q, ref, mem = sets[i % len(sets)]
        proj = torch.nn.functional.linear(q, sw, sb)
        off = proj[..., :2 * LP].view(B, Q, H, L, P, 2)
        attn = proj[..., 2 * LP:].view(B, Q, H, L * P).softmax(-1).view(B, Q, H, L, P)
        if args.ref_dim == 2:
            norm = torch.stack([shapes[:, 1], shapes[:, 0]], -1).to(dtype)
            loc = ref[:, :, None, :, None, :] + off / norm[None, None, None, :, None, :]
        else:
            loc = ref[:, :, None, :, None, :2] + off / P * ref[:, :, None, :, None, 2:] * 0.5
        return ma_deform_attn(mem, W, bias, shapes, starts, loc, attn, mode=args.mode, **kw)

    shapes_host, starts_host = shapes.cpu(), starts.cpu()  # grid_sample callers read the level geometry on the host

    def all_torch(i):
        q, ref, mem = sets[i % len(sets)]
        loc, attn = sampling_producer_reference(q, ref, shapes, H, P, sw, sb)
        out = ma_deform_attn_reference(mem, W, bias, shapes_host, starts_host, loc, attn)
        return torch.nn.functional.linear(out, wo, bo)

    times = {}
    with torch.inference_mode():
        for name, fn in (('ours', ours), ('torch_producer', torch_producer), ('all_torch', all_torch)):
            gr, launches = graph_time_us(fn, args.steps, args.warmup)
            if name == 'ours':
                ours_launches = launches
                torch.cuda.synchronize()
                with ClockSampler(0) as clocks:
                    time.sleep(0.25)
                    times[name] = time_graph(gr, args.steps, reps=max(1, args.reps))
            else:
                times[name] = time_graph(gr, args.steps, reps=max(1, args.reps))
            del gr
        gq, _ = graph_time_us(lambda i: _native.linear(sets[i % len(sets)][0], sw, sb), args.steps, args.warmup)
        t_qproj = time_graph(gq, args.steps, reps=max(1, args.reps))
        del gq
        # parity of the timed configuration: ours against the all-torch layer on the first input set
        diff = (ours(0).float() - all_torch(0).float()).abs().max().item()
    line = {
        'metric': 'µs per deformable attention layer (device-timed)', 'value': round(times['ours'], 3), 'unit': 'us',
        'n_gpus': 1, 'steps': args.steps, 'warmup': args.warmup, 'higher_is_better': False,
        'dtype': str(dtype).replace('torch.', ''), 'data': 'synthetic (seeded, BASELINE config shapes)',
        'config': dict(config_dict(args.config, 1, mode), query_dim=C, reference_points=args.ref_dim,
                       output_proj=[C, H * D]),
        'torch_producer_us': round(times['torch_producer'], 3), 'all_torch_us': round(times['all_torch'], 3),
        'query_proj_us': round(t_qproj, 3), 'max_abs_diff_vs_all_torch': diff,
        'gpu_launches': ours_launches, 'clocks': clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def run_layer_backward(args):
    """A training step of the whole layer per step (--layer --backward): forward (producer, attention, output_proj)
    and the gradients of every float input -- query, reference points, memory and the four projections' weights and
    biases -- on this library's kernels, beside the same step in torch operators (grid_sample, F.linear, autograd) on
    the GPU; prints one JSON line."""
    torch.cuda.set_device(0)
    dev = torch.device('cuda', 0)
    _native.load()
    cfg = workloads.CONFIGS[args.config]
    B, Q, C, H, D, P, dtype = cfg['B'], cfg['Q'], cfg['C'], cfg['H'], cfg['D'], cfg['P'], cfg['dtype']
    L = len(cfg['levels'])
    base, pool = input_pool(args.config, B, dev, 2 * L2_BYTES)
    shapes, starts = base[3], base[4]
    shapes_host, starts_host = shapes.cpu(), starts.cpu()
    g = torch.Generator(device=dev).manual_seed(92)
    LP = H * L * P
    params = [torch.cat([torch.randn(2 * LP, C, generator=g, device=dev) * (2.0 / C ** 0.5),
                         torch.randn(LP, C, generator=g, device=dev) / C ** 0.5]).to(dtype),
              (torch.randn(3 * LP, generator=g, device=dev) * 0.5).to(dtype),
              base[1].detach().clone(), base[2].detach().clone(),
              ((torch.rand(C, H * D, generator=g, device=dev) * 2 - 1) * (6 / (C + H * D)) ** 0.5).to(dtype),
              torch.zeros(C, dtype=dtype, device=dev)]
    params = [t.requires_grad_(True) for t in params]
    sets = []
    for mem, _, _ in pool:
        q = torch.randn(B, Q, C, generator=g, device=dev).to(dtype)
        ref = torch.rand(B, Q, L, args.ref_dim, generator=g, device=dev)
        if args.ref_dim == 4:
            ref[..., 2:] = 0.05 + 0.45 * ref[..., 2:]
        sets.append(tuple(t.requires_grad_(True) for t in (q, ref.to(dtype), mem.detach().clone())))
    gouts = [torch.randn(B, Q, C, generator=g, device=dev).to(dtype) for _ in range(4)]
    mode = args.mode if args.mode != 'auto' else _pick_with_outproj(base[0], base[1], Q, H, L, P, params[4])

    def ours(i):
        q, ref, mem = sets[i % len(sets)]
        sw, sb, W, bias, wo, bo = params
        out = deform_attn_layer(q, ref, mem, shapes, starts, H, P, sw, sb, W, bias, output_weight=wo,
                                output_bias=bo, mode=args.mode)
        return torch.autograd.grad(out, (q, ref, mem, *params), gouts[i % len(gouts)])

    def all_torch(i):
        q, ref, mem = sets[i % len(sets)]
        sw, sb, W, bias, wo, bo = params
        loc, attn = sampling_producer_reference(q, ref, shapes, H, P, sw, sb)
        out = torch.nn.functional.linear(ma_deform_attn_reference(mem, W, bias, shapes_host, starts_host, loc, attn),
                                         wo, bo)
        return torch.autograd.grad(out, (q, ref, mem, *params), gouts[i % len(gouts)])

    times = {}
    gr, launches = graph_time_us(ours, args.steps, args.warmup)
    torch.cuda.synchronize()
    with ClockSampler(0) as clocks:
        time.sleep(0.25)
        times['ours'] = time_graph(gr, args.steps, reps=max(1, args.reps))
    del gr
    gr, _ = graph_time_us(all_torch, args.steps, args.warmup)
    times['all_torch'] = time_graph(gr, args.steps, reps=max(1, args.reps))
    del gr
    # gradients of ours against the all-torch step in float32 on the first input set (upcast inputs; the half-precision
    # torch step is itself too coarse to judge by): the largest |diff| over max |grad|, per tensor
    q0, r0, m0 = sets[0]
    up = [t.detach().float().requires_grad_(True) for t in (q0, r0, m0, *params)]
    loc32, attn32 = sampling_producer_reference(up[0], up[1], shapes, H, P, up[3], up[4])
    out32 = torch.nn.functional.linear(ma_deform_attn_reference(up[2], up[5], up[6], shapes_host, starts_host, loc32,
                                                                attn32), up[7], up[8])
    want = torch.autograd.grad(out32, up, gouts[0].float())
    names = ('query', 'reference_points', 'memory', 'sampling_weight', 'sampling_bias', 'value_weight', 'value_bias',
             'output_weight', 'output_bias')
    rel = {n: round(float((a.float() - b).abs().max()) / max(float(b.abs().max()), 1e-30), 5)
           for n, a, b in zip(names, ours(0), want)}
    line = {
        'metric': 'µs per training step of the deformable attention layer (forward + every gradient, device-timed)',
        'value': round(times['ours'], 3), 'unit': 'us', 'n_gpus': 1, 'steps': args.steps, 'warmup': args.warmup,
        'higher_is_better': False, 'dtype': str(dtype).replace('torch.', ''),
        'data': 'synthetic (seeded, BASELINE config shapes)',
        'config': dict(config_dict(args.config, 1, mode), query_dim=C, reference_points=args.ref_dim,
                       output_proj=[C, H * D]),
        'all_torch_us': round(times['all_torch'], 3),
        'grad_max_rel_diff_vs_float32_torch': rel,  # per input: max |diff| / max |grad|
        'gpu_launches': launches, 'clocks': clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def run_backward(args):
    """Forward + backward per step (see the module docstring); prints one JSON line."""
    torch.cuda.set_device(0)
    dev = torch.device('cuda', 0)
    _native.load()
    cfg = workloads.CONFIGS[args.config]
    B, Q, C, H, D, P = cfg['B'], cfg['Q'], cfg['C'], cfg['H'], cfg['D'], cfg['P']
    L = len(cfg['levels'])
    base, pool = input_pool(args.config, B, dev, 2 * L2_BYTES)
    shapes, starts = base[3], base[4]
    shapes_host, starts_host = shapes.cpu(), starts.cpu()
    W = base[1].detach().clone().requires_grad_(True)
    bias = base[2].detach().clone().requires_grad_(True)
    sets = [tuple(t.detach().clone().requires_grad_(True) for t in s) for s in pool]
    g = torch.Generator(device=dev).manual_seed(5)
    gouts = [torch.randn(B, Q, H * D, generator=g, device=dev).to(W.dtype) for _ in range(4)]
    N = base[0].shape[1]
    e = base[0].element_size()
    mode = args.mode if args.mode != 'auto' else choose_mode(base[0], base[1], base[5])

    def step(fn, i, **kw):
        mem, loc, attn = sets[i % len(sets)]
        out = fn(mem, W, bias, kw.get('shapes', shapes), kw.get('starts', starts), loc, attn, **kw.get('extra', {}))
        return torch.autograd.grad(out, (mem, W, bias, loc, attn), gouts[i % len(gouts)])

    times = {}
    gr, launches = graph_time_us(lambda i: step(ma_deform_attn, i, extra={'mode': args.mode}), args.steps,
                                 args.warmup)
    torch.cuda.synchronize()
    with ClockSampler(0) as clocks:
        time.sleep(0.25)
        times['ours'] = time_graph(gr, args.steps, reps=max(1, args.reps))
    del gr
    gr, _ = graph_time_us(lambda i: step(ma_deform_attn_reference, i, shapes=shapes_host, starts=starts_host),
                          args.steps, args.warmup)
    times['torch'] = time_graph(gr, args.steps, reps=max(1, args.reps))
    del gr
    with torch.no_grad():
        plain = [tuple(t.detach() for t in s_) for s_ in sets]
        gf, _ = graph_time_us(lambda i: ma_deform_attn(plain[i % len(plain)][0], base[1], base[2], shapes, starts,
                                                       *plain[i % len(plain)][1:], mode=args.mode),
                              args.steps, args.warmup)
        times['forward_only'] = time_graph(gf, args.steps, reps=max(1, args.reps))
        del gf
        # the backward kernel alone, on the values of the rotating sets in the layout the backward uses (the
        # project order's own head-major value; the fused order recomputes it in the nn.Linear layout)
        if mode == 'project':
            vals = [_native.value_proj(p_[0], base[1], base[2], H, head_major=True) for p_ in plain]
            heads = None
        else:
            vals = [torch.nn.functional.linear(p_[0], base[1], base[2]) for p_ in plain]
            heads = H
        gk, _ = graph_time_us(lambda i: _native.sample_backward(vals[i % len(vals)], shapes, starts,
                                                                *plain[i % len(plain)][1:], gouts[i % len(gouts)],
                                                                heads=heads),
                              args.steps, args.warmup)
        t_kernel = time_graph(gk, args.steps, reps=max(1, args.reps))
        del gk, vals
    # algorithmic bytes of one backward-kernel launch: value, locations, weights and grad_out read, grad_value
    # (float32, zeroed then accumulated: written once and read once by the atomics), the small gradients written
    S = B * Q * H * L * P
    alg = e * (B * N * H * D + 3 * S + B * Q * H * D) + 4 * (2 * B * N * H * D) + e * 3 * S
    hbm, peak_kind = peaks()
    achieved = alg / (t_kernel * 1e-6) / 1e9
    line = {
        'metric': 'µs per forward + backward of ma_deform_attn (device-timed)', 'value': round(times['ours'], 3),
        'unit': 'us', 'n_gpus': 1, 'steps': args.steps, 'warmup': args.warmup, 'higher_is_better': False,
        'dtype': str(cfg['dtype']).replace('torch.', ''), 'data': 'synthetic (seeded, BASELINE config shapes)',
        'config': dict(config_dict(args.config, 1, mode), grads=['memory', 'value_weight', 'value_bias',
                                                                 'sampling_locations', 'attention_weights']),
        'torch_reference_us': round(times['torch'], 3), 'forward_only_us': round(times['forward_only'], 3),
        'backward_kernel_us': round(t_kernel, 3),
        'roofline': {'bound': 'hbm', 'kernel': 'sample_backward', 'achieved': round(achieved, 1), 'peak': hbm,
                     'unit': 'GB/s', 'frac': round(achieved / hbm, 4), 'peak_source': peak_kind,
                     'algorithmic_bytes': alg},
        'gpu_launches': launches, 'clocks': clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def load_upstream(path):
    """Upstream's package from an installed checkout (with its compiled CUDA extension), imported under the name
    upstream_marearts_tinydeform so that it does not shadow this repository's alias package. (module, None) or
    (None, why)."""
    import importlib.util
    pkg = os.path.join(path, 'marearts_tinydeform')
    init = os.path.join(pkg, '__init__.py')
    if not os.path.exists(init):
        return None, f'no installed marearts_tinydeform package under {path}'
    spec = importlib.util.spec_from_file_location('upstream_marearts_tinydeform', init,
                                                  submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    try:
        spec.loader.exec_module(mod)
    except Exception as exc:  # an extension built for another torch or CUDA
        return None, f'upstream package failed to import: {type(exc).__name__}: {exc}'
    if getattr(mod, '_C', None) is None:
        return None, 'upstream CUDA extension is not built in ' + pkg
    return mod, None


REFERENCE_CUDA_CASES = [  # (config, overrides)
    ('c1h', {}), ('c1h', {'Q': 100}), ('c1h', {'B': 8}), ('c1', {}), ('c3', {}), ('c4', {})]


def run_reference_cuda(args):
    """Upstream's own CUDA operator (its fused_forward; its project order = F.linear + sample_forward) against this
    library's ma_deform_attn (auto), same B200, same harness: a graph of K calls over inputs rotating through a pool
    larger than 2x L2, median of replays, TF32 off. One JSON line per case; a line with 'unavailable' when upstream's
    extension is not installed (python -m pip install --no-index --no-build-isolation --no-deps --target
    baseline/_ref <upstream checkout>, built with TORCH_CUDA_ARCH_LIST=10.0)."""
    mod, why = load_upstream(args.ref_path)
    if mod is None:
        print(json.dumps({'impl': 'reference-cuda', 'unavailable': why}), flush=True)
        return
    torch.cuda.set_device(0)
    dev = torch.device('cuda', 0)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    _native.load()
    for name, over in REFERENCE_CUDA_CASES:
        cfg = dict(workloads.CONFIGS[name], **over)
        saved = workloads.CONFIGS[name]
        workloads.CONFIGS[name] = cfg
        try:
            base, pool = input_pool(name, cfg['B'], dev, 2 * L2_BYTES)
        finally:
            workloads.CONFIGS[name] = saved
        W, bias, shapes, starts = base[1], base[2], base[3], base[4]
        res = {}
        with torch.inference_mode():
            for label, fn, mode in (('upstream_fused', mod.ma_deform_attn, 'fused'),
                                    ('upstream_project', mod.ma_deform_attn, 'project'),
                                    ('ours_auto', ma_deform_attn, 'auto')):
                def call(i, fn=fn, mode=mode):
                    mem, loc, attn = pool[i % len(pool)]
                    return fn(mem, W, bias, shapes, starts, loc, attn, mode=mode)
                g, _ = graph_time_us(call, args.steps, args.warmup)
                res[label] = round(time_graph(g, args.steps, reps=max(5, args.reps // 5)), 3)
                del g
            mem, loc, attn = pool[0]
            ours = ma_deform_attn(mem, W, bias, shapes, starts, loc, attn).double()
            theirs = mod.ma_deform_attn(mem, W, bias, shapes, starts, loc, attn, mode='project').double()
            diff = (ours - theirs).abs().max().item()
            picked = choose_mode(mem, W, loc)
        best_ref = min(res['upstream_fused'], res['upstream_project'])
        print(json.dumps({'impl': 'reference-cuda', 'case': f'{name} {over}' if over else name,
                          'dtype': str(cfg['dtype']).replace('torch.', ''), 'B': cfg['B'], 'Q': cfg['Q'],
                          'us_per_call': res, 'ours_mode': picked,
                          'speedup_vs_upstream_faster': round(best_ref / res['ours_auto'], 3),
                          'max_abs_diff_vs_upstream_project': diff, 'steps': args.steps,
                          'l2': 'rotating inputs > 2x L2 between calls'}), flush=True)


def run_l2_peak(args):
    """The L2 random-row gather rates (td_probe_row_gather) for every row size the gather kernels read; one line."""
    torch.cuda.set_device(0)
    dev = torch.device('cuda', 0)
    _native.load()
    kinds = [(16, False), (32, False), (64, False), (128, False), (128, True), (256, False), (256, True),
             (512, False), (512, True)]
    with ClockSampler(0) as clocks:
        time.sleep(0.25)
        rates = l2_gather_peak(dev, kinds)
    hbm, kind = peaks()
    print(json.dumps({'metric': 'L2 random-row gather rate (td_probe_row_gather, 8 MiB buffer, all SMs)',
                      'rates': rates, 'hbm_peak_gbs': hbm, 'hbm_peak_source': kind,
                      'sm_count': torch.cuda.get_device_properties(dev).multi_processor_count,
                      'clocks': clocks.summary()}), flush=True)


def run_sweep(args):
    """Fused vs project over upstream's sweep grid (bench/results/rtx4090.md) and the c5 grid; prints a table."""
    torch.cuda.set_device(0)
    _native.load()
    rows = []
    grids = [('c1', dtype, B, Q) for dtype in args.dtype for B in (1, 4, 8) for Q in (50, 100, 200, 300, 600, 900)]
    grids += [('c5', dtype, B, Q) for dtype in args.dtype for B in workloads.C5_BATCHES for Q in workloads.C5_QUERIES]
    grids += [('c4', dtype, B, Q) for dtype in args.dtype for B in (1, 8) for Q in (300, 900)]
    clocks = ClockSampler(0)
    with torch.inference_mode(), clocks:
        for cfg, dname, B, Q in grids:
            dtype = getattr(torch, dname)
            a = workloads.make_inputs(cfg, seed=0, B=B, Q=Q, dtype=dtype, device='cuda', generate_on_device=True)
            t = {}
            for mode in ('fused', 'project'):
                g, _ = graph_time_us(lambda i, m=mode: ma_deform_attn(*a, mode=m), 50, 3)
                t[mode] = time_graph(g, 50, reps=5)
                del g
            pick = choose_mode(a[0], a[1], a[5])
            c = workloads.CONFIGS[cfg]
            N, L, P, D = a[0].shape[1], len(c['levels']), c['P'], c['D']
            ratio = Q * L * P * 4 / (N * D)
            row = {'config': cfg, 'dtype': dname, 'B': B, 'Q': Q, 'ratio': ratio, 'fused_us': t['fused'],
                   'project_us': t['project'], 'auto': pick, 'auto_us': t[pick],
                   'best': min(t, key=t.get), 'auto_within_10pct': t[pick] <= 1.1 * min(t.values())}
            rows.append(row)
            print(json.dumps(row), flush=True)
            del a
            torch.cuda.empty_cache()
    ok = sum(r['auto_within_10pct'] for r in rows)
    print(json.dumps({'sweep_cases': len(rows), 'auto_within_10pct': ok, 'clocks': clocks.summary()}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=200)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--reps', type=int, default=50)
    ap.add_argument('--config', default='c1h', choices=sorted(workloads.CONFIGS))
    ap.add_argument('--mode', default='auto', choices=('auto', 'fused', 'project'))
    ap.add_argument('--impl', default='ours', choices=('ours', 'reference', 'reference-cuda'),
                    help="reference: upstream's algorithm on the host CPU; reference-cuda: upstream's own CUDA "
                         "operator from an installed checkout (--ref-path), timed beside this library")
    ap.add_argument('--ref-path', default=os.path.join(ROOT, 'baseline', '_ref'),
                    help='--impl reference-cuda: where upstream is installed (pip --target)')
    ap.add_argument('--no-cpu', action='store_true')
    ap.add_argument('--no-sharded', action='store_true', help='skip the batch-sharded c3 record')
    ap.add_argument('--l2-peak', action='store_true', help='print the L2 random-row gather rates and exit')
    ap.add_argument('--output-proj', action='store_true',
                    help='chain the decoder output_proj ([C, H*D] nn.Linear) behind the attention')
    ap.add_argument('--outproj-plan', default='auto', choices=('auto', 'chained', 'cluster'),
                    help="--output-proj / --layer: output_proj in the sampler's cluster kernel or chained as a GEMM")
    ap.add_argument('--padding-mask', type=float, default=0.0,
                    help='fraction of tokens padded by a random value padding mask (0: no mask)')
    ap.add_argument('--sweep', action='store_true')
    ap.add_argument('--layer', action='store_true', help='time the whole deformable attention layer')
    ap.add_argument('--backward', action='store_true',
                    help='time forward + backward (training); with --layer, the whole layer\'s training step')
    ap.add_argument('--ref-dim', type=int, default=4, choices=(2, 4),
                    help='--layer: reference points (2) or reference boxes (4)')
    ap.add_argument('--dtype', nargs='+', default=['float16', 'bfloat16', 'float32'])
    ap.add_argument('--as-dtype', choices=('float32', 'float16', 'bfloat16', 'float64'),
                    help='run the config in this dtype instead of its own (profiling the other kernels)')
    args = ap.parse_args()
    if args.outproj_plan != 'auto':
        _native.set_output_proj_plan({'chained': _native.OUTPROJ_CHAINED, 'cluster': _native.OUTPROJ_CLUSTER}[
            args.outproj_plan])
    if args.as_dtype:
        workloads.CONFIGS[args.config] = dict(workloads.CONFIGS[args.config], dtype=getattr(torch, args.as_dtype))
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == 'reference':
        run_reference_arm(args)
    elif args.impl == 'reference-cuda':
        run_reference_cuda(args)
    elif args.l2_peak:
        run_l2_peak(args)
    elif args.sweep:
        run_sweep(args)
    elif args.layer and args.backward:
        run_layer_backward(args)
    elif args.layer:
        run_layer(args)
    elif args.backward:
        run_backward(args)
    else:
        run_ours(args)


if __name__ == '__main__':
    main()
