#!/usr/bin/env python
"""Benchmark of the B200 grouped-convolution engine (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...
    python bench.py --impl reference ...     # the reference's CPU implementation

A step is one gc_cuda_conv call (implementation 3, the production choice)
over one batch of synthetic input already resident in HBM.  Default workload:
the depthwise N32 C256 56x56 convolution, one batch per GPU ("weak": every
rank runs its own batch, no collective on the data path).  ``--workload
config5_g32 --scaling strong`` shards the N1024 batch across the ranks.

Reported: ``value`` (GB/s of algorithmic bytes, whole job, device time of K
back-to-back steps, max over ranks), ``e2e`` (same metric through the C ABI
with the batch in pinned host memory and both copies inside the timed
region), ``roofline`` of the kernel, ``cudnn`` (torch.nn.functional.conv2d,
TF32 off, benchmark mode, same buffers), ``cpu_baseline`` (the reference's CPU
library on the host cores), ``clocks`` sampled through NVML while timing.
"""
from __future__ import annotations

import argparse
import ctypes as ct
import datetime
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

METRIC = 'grouped-conv GB/s & GFLOP/s (% of B200 roofline), latency ratio vs cuDNN, 1/2/4/8 GPU'
UNIT = 'GB/s'
L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {'hbm_gbs': 6650.0, 'bf16_tflops': 1590.0}


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=2000)
    ap.add_argument('--warmup', type=int, default=20)
    ap.add_argument('--impl', choices=['ours', 'reference'], default='ours')
    ap.add_argument('--workload', default='config2',
                    choices=['config1', 'config2', 'config4_leaf', 'config5_g32', 'config5_g4', 'config4_block',
                             'config3', 'atlas', 'model_layers'])
    ap.add_argument('--scaling', choices=['weak', 'strong'], default=None,
                    help='weak: each rank runs the full workload batch; strong: the batch is sharded')
    ap.add_argument('--shape', default=None,
                    help='N,C,H,W,CPG: a custom 3x3/s1/p1 shape (uniform inputs) instead of --workload')
    ap.add_argument('--batch', type=int, default=None,
                    help='override the workload batch (small cases for profiling)')
    ap.add_argument('--e2e-steps', type=int, default=20)
    ap.add_argument('--no-e2e', action='store_true')
    ap.add_argument('--no-cudnn', action='store_true')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--cpu-seconds', type=float, default=10.0, help='CPU baseline sample budget')
    ap.add_argument('--atlas-batches', type=int, default=10, help='atlas: paired batches per shape')
    ap.add_argument('--atlas-samples', type=int, default=30, help='atlas: samples per batch and implementation')
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error('--warmup must be at least 3')
    if args.shape:
        args.workload = 'custom:' + args.shape
    if args.scaling is None:
        args.scaling = 'strong' if args.workload.startswith('config5') else 'weak'
    return args


def measured_peaks():
    path = ROOT / 'MEASURED_PEAKS.json'
    if path.exists():
        data = json.loads(path.read_text())
        return {'hbm_gbs': float(data['hbm_gbs']), 'bf16_tflops': float(data.get('bf16_tflops', 0))}, 'measured'
    return dict(FALLBACK_PEAKS), 'fallback'


def recorded_traffic(workload):
    """DRAM bytes per launch of the dominant kernel, from a committed ncu summary."""
    path = ROOT / 'profiles' / 'traffic.json'
    if not path.exists():
        return None
    entry = json.loads(path.read_text()).get(workload)
    return None if entry is None else entry.get('dram_bytes_per_launch')


class ClockSampler:
    """Samples SM clock, power and clock-event reasons through NVML (read only)."""
    REASONS = {
        'hw_slowdown': 'nvmlClocksEventReasonHwSlowdown',
        'hw_thermal_slowdown': 'nvmlClocksEventReasonHwThermalSlowdown',
        'sw_thermal_slowdown': 'nvmlClocksEventReasonSwThermalSlowdown',
        'sw_power_cap': 'nvmlClocksEventReasonSwPowerCap',
        'hw_power_brake_slowdown': 'nvmlClocksEventReasonHwPowerBrakeSlowdown',
    }

    def __init__(self, device_index, period=0.005):
        self.period = period
        self.samples = []
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            # NVML enumerates physical GPUs; map through CUDA_VISIBLE_DEVICES if set.
            visible = os.environ.get('CUDA_VISIBLE_DEVICES')
            index = device_index
            if visible:
                ids = [v.strip() for v in visible.split(',') if v.strip()]
                if device_index < len(ids) and ids[device_index].isdigit():
                    index = int(ids[device_index])
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # no NVML: report why instead of clocks
            self.nvml = None
            self.error = str(exc)

    def _run(self):
        n = self.nvml
        while not self._stop.is_set():
            try:
                sm = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
                reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                power = n.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
                self.samples.append((sm, reasons, power))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if self.nvml is None:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': [], 'error': self.error}
        if not self.samples:
            return {'sm_mhz': None, 'sm_max_mhz': self.max_mhz, 'reasons': [], 'samples': 0}
        active = set()
        for _, mask, _ in self.samples:
            for name, const in self.REASONS.items():
                if mask & getattr(self.nvml, const):
                    active.add(name)
        return {'sm_mhz': statistics.median(s[0] for s in self.samples), 'sm_max_mhz': self.max_mhz,
                'reasons': sorted(active), 'samples': len(self.samples),
                'power_w_max': max(s[2] for s in self.samples)}


def dist_setup():
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    return rank, world, local


def barrier():
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def workload_host(name, images_first, images_count):
    """Host arrays (x for images [first, first+count), w) of a workload."""
    from groupconv_atlas_b200 import workloads
    wl = workloads.by_name(name, with_x=False)
    x = workloads.images(wl.shape, wl.seed, wl.dist, images_first, images_count)
    return wl, x, wl.w


# ---------------------------------------------------------------------------------------
# The reference arm: the reference's CPU implementation on the host cores.
# ---------------------------------------------------------------------------------------
def cpu_reference_runner(shape, x, w):
    """Returns (run(out), kind, cores): the reference library compiled from the
    reference's sources (kind 'reference') or the oracle's C restatement of it
    (kind 'port'), GC_BLOCKED schedule on every host thread."""
    from oracle import oracle as orc
    cores = os.cpu_count() or 1
    if orc.reference_available():
        return (lambda out: orc.reference_conv(shape, x, w, impl=2, threads=cores, out=out)), 'reference', cores
    return (lambda out: orc.conv_f32_blocked(shape, x, w, threads=cores)), 'port', cores


def sample_images(name, total_images, budget_s):
    """Largest image count (<= total) whose one blocked CPU pass stays within
    budget_s, measured on one image."""
    wl, x1, w = workload_host(name, 0, 1)
    import dataclasses
    one = dataclasses.replace(wl.shape, n=1)
    run, _, _ = cpu_reference_runner(one, x1, w)
    out = np.empty(one.output, np.float32)
    run(out)
    t0 = time.perf_counter()
    run(out)
    per_image = max(time.perf_counter() - t0, 1e-6)
    return int(max(1, min(total_images, budget_s // per_image or 1)))


def cpu_baseline(name, images_total, seconds):
    """Times the reference CPU implementation on a bounded sample of the workload."""
    import dataclasses
    m = sample_images(name, images_total, seconds / 4)
    wl, x, w = workload_host(name, 0, m)
    shape = dataclasses.replace(wl.shape, n=m)
    run, kind, cores = cpu_reference_runner(shape, x, w)
    out = np.empty(shape.output, np.float32)
    run(out)  # warm-up
    passes, t0 = 0, time.perf_counter()
    while True:
        run(out)
        passes += 1
        elapsed = time.perf_counter() - t0
        if elapsed >= seconds or passes >= 200:
            break
    bytes_per_pass = 4 * (math.prod(shape.input) + math.prod(shape.weight) + math.prod(shape.output))
    return {'value': bytes_per_pass * passes / elapsed / 1e9, 'unit': UNIT, 'cores': cores, 'kind': kind,
            'sample': f'{m} of {images_total} images x {passes} passes ({elapsed:.1f} s), GC_BLOCKED, '
                      f'{cores} threads'}


def run_reference(args):
    rank, world, _ = dist_setup()
    if rank != 0:
        return 0  # the CPU reference runs on rank 0 only
    import dataclasses
    from groupconv_atlas_b200 import workloads
    wl = workloads.by_name(args.workload, with_x=False)
    m = sample_images(args.workload, wl.shape.n, 0.25)
    wl, x, w = workload_host(args.workload, 0, m)
    shape = dataclasses.replace(wl.shape, n=m)
    run, kind, cores = cpu_reference_runner(shape, x, w)
    out = np.empty(shape.output, np.float32)
    for _ in range(args.warmup):
        run(out)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run(out)
    elapsed = time.perf_counter() - t0
    step_bytes = 4 * (math.prod(shape.input) + math.prod(shape.weight) + math.prod(shape.output))
    step_flops = 2 * math.prod(shape.output) * shape.cpg * 9
    value = step_bytes * args.steps / elapsed / 1e9
    line = {'impl': 'reference', 'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': args.gpus,
            'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': elapsed / args.steps * 1e3,
            'higher_is_better': True, 'scaling': args.scaling, 'vs_baseline': None, 'dtype': 'f32',
            'data': 'synthetic (seeded, per-image generators)',
            'gflops': step_flops * args.steps / elapsed / 1e9,
            'config': {'workload': args.workload, 'shape': dataclasses.asdict(wl.shape),
                       'step': f'{m} images of the batch per step'},
            'cpu_baseline': {'value': value, 'unit': UNIT, 'cores': cores, 'kind': kind,
                             'sample': f'{m} images per step, GC_BLOCKED, {cores} threads'},
            'e2e': {'value': value, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------------
# Our arm.
# ---------------------------------------------------------------------------------------
class Call:
    """Pre-built C ABI arguments of one gc_cuda_conv call (descriptors built once)."""

    def __init__(self, native, shape, x, w, y, stream, impl=3):
        from groupconv_atlas_b200.api import cshape, tensor
        self.fn = native.lib.gc_cuda_conv
        self.native = native
        self.p, self.xd, self.wd, self.yd = cshape(shape), tensor(x), tensor(w), tensor(y)
        self.args = (ct.byref(self.p), ct.byref(self.xd), ct.byref(self.wd), ct.byref(self.yd), impl,
                     ct.c_void_p(stream))

    def __call__(self):
        status = self.fn(*self.args)
        if status:
            self.native.check(status)


def run_ours(args):
    import dataclasses
    import torch
    import torch.distributed as dist
    from groupconv_atlas_b200 import api, shard, workloads
    from oracle import oracle as orc

    rank, world, local = dist_setup()
    torch.cuda.set_device(local)
    if world > 1:
        # NCCL's own log lines (its version banner, when the environment asks
        # for it) go to stderr unless the caller chose a file: stdout carries
        # only the JSON line
        os.environ.setdefault('NCCL_DEBUG_FILE', '/dev/stderr')
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device('cuda', local))
    native = api.Native()
    full = workloads.by_name(args.workload, batch=args.batch, with_x=False)
    if args.scaling == 'weak':
        units = [shard.Unit(0, full.shape.n, 0, full.shape.cin)]
        first_image = rank * full.shape.n  # each rank: its own batch of the same shape
        job_images = full.shape.n * world
    else:
        units = shard.units_for_rank(full.shape, world, rank)
        first_image = units[0].n0 if units else 0
        job_images = full.shape.n
    n_images = sum(u.images() for u in units) if args.scaling == 'strong' else full.shape.n
    local_shape = dataclasses.replace(full.shape, n=max(1, units[-1].n1 - units[0].n0) if args.scaling == 'strong'
                                      else full.shape.n)
    # Host data of this rank's images (pinned), weights.
    x_host = workloads.images(full.shape, full.seed, full.dist, first_image, local_shape.n)
    w_host = full.w
    xh = torch.from_numpy(x_host).pin_memory()
    wh = torch.from_numpy(w_host).pin_memory()
    set_bytes = 4 * (math.prod(local_shape.input) + math.prod(local_shape.output))
    sets = int(min(4096, max(1, math.ceil(3 * L2_BYTES / set_bytes))))
    stream = torch.cuda.Stream()
    dw = wh.to('cuda')
    xs = [xh.to('cuda') for _ in range(sets)]
    ys = [torch.empty(local_shape.output, device='cuda') for _ in range(sets)]
    torch.cuda.synchronize()

    def unit_views(xt, yt):
        out = []
        for u in units if args.scaling == 'strong' else [shard.Unit(0, local_shape.n, 0, local_shape.cin)]:
            if args.scaling == 'strong':
                u = shard.Unit(u.n0 - units[0].n0, u.n1 - units[0].n0, u.c0, u.c1)
            sub = u.shape(local_shape)
            ox, ow, oy = u.offsets(local_shape)
            xv = xt.view(-1)[ox:ox + math.prod(sub.input)].view(sub.input)
            wv = dw.view(-1)[ow:ow + math.prod(sub.weight)].view(sub.weight)
            yv = yt.view(-1)[oy:oy + math.prod(sub.output)].view(sub.output)
            out.append((sub, xv, wv, yv))
        return out

    calls = [[Call(native, sub, xv, wv, yv, stream.cuda_stream) for sub, xv, wv, yv in unit_views(xs[i], ys[i])]
             for i in range(sets)]
    launches_per_step = len(calls[0])
    step_bytes = sum(4 * (math.prod(s.input) + math.prod(s.weight) + math.prod(s.output))
                     for s, *_ in unit_views(xs[0], ys[0]))
    step_flops = sum(2 * math.prod(s.output) * s.cpg * 9 for s, *_ in unit_views(xs[0], ys[0]))

    # Correctness gate before timing: 64 FP64 points of this rank's output.
    with torch.cuda.stream(stream):
        for c in calls[0]:
            c()
    plan = native.last_plan()
    stream.synchronize()
    y0 = ys[0].cpu().numpy()
    check = orc.check_points(local_shape, x_host, w_host, y0)
    if not check['passed']:
        raise SystemExit(f'correctness gate failed on rank {rank}: {check["failed_points"]} points [{plan}]')
    if native.device_status(clear=True):
        raise SystemExit('device status word set after the correctness gate')

    # Device-timed region: K back-to-back steps, events around every step.
    with torch.cuda.stream(stream):
        for k in range(args.warmup):
            for c in calls[k % sets]:
                c()
    stream.synchronize()
    region0, region1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    with sampler, torch.cuda.stream(stream):
        region0.record(stream)
        for k in range(args.steps):
            for c in calls[k % sets]:
                c()
        region1.record(stream)
        stream.synchronize()
    torch.cuda.synchronize()
    barrier()
    elapsed_ms = region0.elapsed_time(region1)
    # Average launch duration for the roofline: the events bracketing the
    # timed region on the launch stream, over the launches inside it.
    # (Consecutive launches overlap prologue and tail through programmatic
    # dependent launch, so the region, not an event pair per launch, is the
    # per-launch cost; an event between launches would break that overlap.)
    kernel_ms = elapsed_ms / (args.steps * launches_per_step)

    def graph_step(k):
        for c in calls[k % sets]:
            c()
    with torch.cuda.stream(stream):
        graph_kernel_ms = graph_step_ms(torch, stream, graph_step, min(args.steps, 50)) / launches_per_step
    max_elapsed = shard.max_over_ranks(elapsed_ms)
    job_bytes = shard.sum_over_ranks(step_bytes)
    job_flops = shard.sum_over_ranks(step_flops)
    value = job_bytes * args.steps / (max_elapsed / 1e3) / 1e9
    gflops = job_flops * args.steps / (max_elapsed / 1e3) / 1e9

    # End to end through the C ABI: pinned host batch -> device -> conv -> host,
    # pipelined in chunks over three streams, copies inside the timed region.
    e2e = None
    if not args.no_e2e:
        e2e = end_to_end(args, native, local_shape, units, xh, wh, torch, api, shard)

    cudnn = None
    if not args.no_cudnn and rank == 0:
        cudnn = cudnn_baseline(args, torch, local_shape, xs, dw, sets,
                               (elapsed_ms / args.steps, graph_kernel_ms * launches_per_step))

    cpu = None
    if not args.no_cpu_baseline and rank == 0 and world == 1:
        cpu = cpu_baseline(args.workload, local_shape.n, args.cpu_seconds)

    status = native.device_status(clear=True)
    if status:
        raise SystemExit(f'device status word set during timing: {status:#x}')
    peaks, peak_kind = measured_peaks()
    achieved = (step_bytes / launches_per_step) / (kernel_ms / 1e3) / 1e9
    fp32_tflops = (step_flops / launches_per_step) / (kernel_ms / 1e3) / 1e12
    if plan.startswith('kernel=tf32x3'):
        # Tensor-bound: FP32 work against the 3xTF32 ceiling = measured bf16
        # GEMM rate / 2 (TF32 issues at half the bf16 rate) / 3 (products).
        peak_tensor = peaks['bf16_tflops'] / 2 / 3
        roofline = {'bound': 'tensor', 'achieved': fp32_tflops, 'peak': peak_tensor, 'unit': 'TFLOP/s',
                    'frac': fp32_tflops / peak_tensor,
                    'peak_source': f'{peak_kind} bf16 dense GEMM / 2 (TF32 rate) / 3 (3xTF32 products)',
                    'hbm_achieved_gbs': achieved, 'hbm_frac': achieved / peaks['hbm_gbs']}
    else:
        roofline = {'bound': 'hbm', 'achieved': achieved, 'peak': peaks['hbm_gbs'], 'unit': 'GB/s',
                    'frac': achieved / peaks['hbm_gbs'], 'peak_source': f'{peak_kind} copy bandwidth'}
        if rank == 0 and xs[0].numel() == ys[0].numel():
            # Context for launch-sized transfers: a device copy x -> y of the
            # same bytes per launch, same rotating sets, back to back.
            copy_ms = copy_same_bytes_ms(torch, stream, xs, ys, args.steps)
            copy_gbs = 2 * xs[0].numel() * 4 / (copy_ms / 1e3) / 1e9
            roofline['same_size_copy'] = {'gbs': copy_gbs, 'ms': copy_ms, 'frac_of_it': achieved / copy_gbs,
                                          'what': 'torch copy_ of x into y (read + write bytes), '
                                                  'same rotating sets, K back-to-back copies'}
    traffic = recorded_traffic(args.workload)
    clocks = sampler.summary()
    if world > 1:
        import torch.distributed as dist
        gathered = [None] * world
        dist.all_gather_object(gathered, clocks)
        clocks = gathered[0] | {'per_rank_reasons': [g.get('reasons') for g in gathered]}
    if rank == 0:
        line = {
            'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': max_elapsed / args.steps, 'higher_is_better': True,
            'scaling': args.scaling, 'vs_baseline': None, 'dtype': 'f32',
            'data': 'synthetic (seeded per-image generators, distributions of the workload definition)',
            'gflops': gflops,
            'config': {'workload': args.workload, 'shape': dataclasses.asdict(full.shape),
                       'images_per_step': job_images, 'implementation': 3, 'kernel_plan': plan,
                       'l2': f'{sets} rotating input/output sets per rank, {sets * set_bytes / 2**20:.0f} MiB '
                             f'> L2 {L2_BYTES / 2**20:.0f} MiB',
                       'parallelism': f'{args.scaling} batch sharding over {world} GPU(s), no collective'},
            'roofline': {**roofline, 'traffic': traffic, 'kernel_ms': kernel_ms,
                         'kernel_ms_timing': 'CUDA events bracketing the timed region on the launch stream / launches',
                         'graph_kernel_ms': graph_kernel_ms,
                         'algorithmic_bytes_per_launch': step_bytes / launches_per_step,
                         'algorithmic_flops_per_launch': step_flops / launches_per_step,
                         'fp32_tflops': fp32_tflops},
            'e2e': e2e, 'gpu_launches': args.steps * launches_per_step, 'clocks': clocks,
            'cudnn': cudnn, 'cpu_baseline': cpu,
        }
        print(json.dumps(line), flush=True)
    del calls
    if world > 1:
        dist.destroy_process_group()
    return 0


def end_to_end(args, native, shape, units, xh, wh, torch, api, shard):
    """Same metric, through the C ABI with host buffers: per step the batch is
    copied host->device in chunks (pinned), convolved chunk by chunk as soon
    as its copy lands, and copied back; three streams overlap the two copy
    directions with compute, and two device buffer sets alternate between
    steps, so the copies of step k+1 never wait for the convolutions of
    step k."""
    import dataclasses
    n = shape.n
    chunks = max(1, min(8, n))
    bounds = [(i * n // chunks, (i + 1) * n // chunks) for i in range(chunks)]
    bounds = [b for b in bounds if b[1] > b[0]]
    dws = [torch.empty(shape.weight, device='cuda') for _ in range(2)]
    dxs = [torch.empty(shape.input, device='cuda') for _ in range(2)]
    dys = [torch.empty(shape.output, device='cuda') for _ in range(2)]
    yh = torch.empty(shape.output, pin_memory=True)
    s_in, s_cmp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    calls = [[Call(native, dataclasses.replace(shape, n=hi - lo), dxs[b][lo:hi], dws[b], dys[b][lo:hi],
                   s_cmp.cuda_stream) for lo, hi in bounds] for b in range(2)]
    ev_in = [[torch.cuda.Event() for _ in bounds] for _ in range(2)]
    ev_cmp = [[torch.cuda.Event() for _ in bounds] for _ in range(2)]
    ev_out = [[torch.cuda.Event() for _ in bounds] for _ in range(2)]
    used = [False, False]

    def step(k):
        b = k & 1
        dx, dy = dxs[b], dys[b]
        with torch.cuda.stream(s_in):
            if used[b]:
                s_in.wait_event(ev_cmp[b][-1])  # step k-2 finished reading these weights
            dws[b].copy_(wh, non_blocking=True)
            for j, (lo, hi) in enumerate(bounds):
                if used[b]:
                    s_in.wait_event(ev_cmp[b][j])  # step k-2 finished reading this dx chunk
                dx[lo:hi].copy_(xh[lo:hi], non_blocking=True)
                ev_in[b][j].record(s_in)
        for j in range(len(bounds)):
            s_cmp.wait_event(ev_in[b][j])
            if used[b]:
                s_cmp.wait_event(ev_out[b][j])  # step k-2 finished reading this dy chunk
            calls[b][j]()
            ev_cmp[b][j].record(s_cmp)
        with torch.cuda.stream(s_out):
            for j, (lo, hi) in enumerate(bounds):
                s_out.wait_event(ev_cmp[b][j])
                yh[lo:hi].copy_(dy[lo:hi], non_blocking=True)
                ev_out[b][j].record(s_out)
        used[b] = True

    for i in range(3):
        step(i)
    torch.cuda.synchronize()
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(s_in)
    for i in range(args.e2e_steps):
        step(3 + i)
    t1.record(s_out)
    torch.cuda.synchronize()
    barrier()
    ms = shard.max_over_ranks(t0.elapsed_time(t1))
    # the host result of the last step equals that step's device output
    consistent = bool(torch.equal(yh, dys[(2 + args.e2e_steps) & 1].cpu()))
    step_bytes = 4 * (math.prod(shape.input) + math.prod(shape.weight) + math.prod(shape.output))
    job_bytes = shard.sum_over_ranks(step_bytes)
    # The link's bound: the same bytes copied in both directions at once
    # (the step's input host->device while its output goes device->host),
    # with no convolution.
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    c0.record(s_in)
    for _ in range(5):
        s_out.wait_event(c0)
        with torch.cuda.stream(s_in):
            dxs[0].copy_(xh, non_blocking=True)
        with torch.cuda.stream(s_out):
            yh.copy_(dys[0], non_blocking=True)
        s_in.wait_stream(s_out)
    c1.record(s_in)
    torch.cuda.synchronize()
    link_ms = shard.max_over_ranks(c0.elapsed_time(c1) / 5)
    bound = job_bytes / (link_ms / 1e3) / 1e9
    e2e_value = job_bytes * args.e2e_steps / (ms / 1e3) / 1e9
    return {'value': e2e_value, 'unit': UNIT,
            'link_bound': {'value': bound, 'unit': UNIT, 'frac': e2e_value / bound, 'ms_per_step': link_ms,
                           'what': 'the step\'s input host->device and output device->host copied at once '
                                   '(pinned), no convolution'},
            'h2d_bytes_per_step': 4 * (math.prod(shape.input) + math.prod(shape.weight)),
            'd2h_bytes_per_step': 4 * math.prod(shape.output), 'steps': args.e2e_steps,
            'ms_per_step': ms / args.e2e_steps, 'chunks': len(bounds),
            'path': 'pinned host -> gc_cuda_conv per chunk (C ABI via ctypes) -> pinned host',
            'host_matches_device': consistent}


def copy_same_bytes_ms(torch, stream, xs, ys, steps):
    """Average duration of a device copy x -> y over the rotating sets."""
    sets = len(xs)
    with torch.cuda.stream(stream):
        for k in range(3):
            ys[k % sets].view(-1).copy_(xs[k % sets].view(-1))
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for k in range(steps):
            ys[k % sets].view(-1).copy_(xs[k % sets].view(-1))
        b.record(stream)
        stream.synchronize()
    return a.elapsed_time(b) / steps


def graph_step_ms(torch, stream, step, count, replays=3):
    """Device time of one step from CUDA-graph replay: `count` steps captured
    back to back (host launch cost excluded, as the reference's graph timing
    bench/cuda_run.py:92-121), mean over `replays` replays."""
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for k in range(count):
            step(k)
    graph.replay()
    stream.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(replays):
        graph.replay()
    b.record(stream)
    stream.synchronize()
    ms = a.elapsed_time(b) / (replays * count)
    del graph
    return ms


def cudnn_baseline(args, torch, shape, xs, dw, sets, our_step_ms):
    """torch.nn.functional.conv2d on the same device buffers: TF32 off and read
    back, cudnn.benchmark on, device time of back-to-back calls."""
    import torch.nn.functional as F
    if hasattr(torch.backends, 'fp32_precision'):
        for target in (torch.backends, torch.backends.cuda.matmul, torch.backends.cudnn,
                       torch.backends.cudnn.conv):
            target.fp32_precision = 'ieee'
        tf32 = torch.backends.cudnn.conv.fp32_precision != 'ieee'
    else:
        torch.backends.cuda.matmul.allow_tf32 = False
        torch.backends.cudnn.allow_tf32 = False
        tf32 = torch.backends.cudnn.allow_tf32
    if tf32:
        raise SystemExit('could not disable TF32 for the cuDNN baseline')
    torch.backends.cudnn.benchmark = True
    stream = torch.cuda.Stream()
    steps = max(20, min(args.steps, 200))
    with torch.inference_mode(), torch.cuda.stream(stream):
        for k in range(10):
            F.conv2d(xs[k % sets], dw, padding=1, groups=shape.groups)
        stream.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for k in range(steps):
            F.conv2d(xs[k % sets], dw, padding=1, groups=shape.groups)
        b.record(stream)
        stream.synchronize()
        eager_ms = a.elapsed_time(b) / steps
        outs = [None] * sets

        def step(k):
            outs[k % sets] = F.conv2d(xs[k % sets], dw, padding=1, groups=shape.groups)
        graph_ms = graph_step_ms(torch, stream, step, min(steps, 50))
    return {'ms_per_step': eager_ms, 'graph_ms_per_step': graph_ms, 'ours_ms_per_step': our_step_ms[0],
            'ours_graph_ms_per_step': our_step_ms[1], 'speedup_vs_cudnn': eager_ms / our_step_ms[0],
            'speedup_vs_cudnn_graph': graph_ms / our_step_ms[1],
            'timing': 'back-to-back calls on one stream (eager) and CUDA-graph replay, both sides',
            'api': 'torch.nn.functional.conv2d', 'tf32': False, 'benchmark': True,
            'cudnn_version': torch.backends.cudnn.version()}


def set_fp32_precision(torch):
    """TF32 off everywhere (cuDNN and matmul), read back."""
    if hasattr(torch.backends, 'fp32_precision'):
        for target in (torch.backends, torch.backends.cuda.matmul, torch.backends.cudnn,
                       torch.backends.cudnn.conv):
            target.fp32_precision = 'ieee'
        if torch.backends.cudnn.conv.fp32_precision != 'ieee':
            raise SystemExit('could not disable TF32')
    else:
        torch.backends.cuda.matmul.allow_tf32 = False
        torch.backends.cudnn.allow_tf32 = False


GRAPH_STEPS, GRAPH_REPLAYS = 50, 3  # the block's graph timing: calls captured, replays timed


def run_block(args):
    """Config 4: torchvision MobileNetV2 features[3] (random Kaiming-normal
    init, seed 2, eval), N4 input N(0,1); the reference block runs every conv
    on cuDNN, the candidate replaces only the depthwise 3x3 by gc_cuda_conv
    (implementation 3), as the reference's bench/module_run.py:215-235 does.
    Reports block latency from CUDA-graph replay (device) and synchronized
    per-call wall time (API), both blocks, same inputs."""
    import copy
    import torch
    import torchvision
    from groupconv_atlas_b200 import api, torch_module
    from oracle import oracle as orc
    rank, world, local = dist_setup()
    if rank != 0:
        return 0
    torch.cuda.set_device(local)
    set_fp32_precision(torch)
    torch.backends.cudnn.benchmark = True
    torch.manual_seed(2)
    block = torchvision.models.mobilenet_v2(weights=None).features[3].eval().cuda()
    cand = copy.deepcopy(block)
    native = api.Native()
    replaced = torch_module.substitute(cand, torch_module.is_depthwise_3x3, native)
    x = torch.randn((4, 24, 56, 56), generator=torch.Generator().manual_seed(2)).cuda()
    stream = torch.cuda.Stream()
    with torch.inference_mode(), torch.cuda.stream(stream):
        ref = block(x)
        out = cand(x)
        stream.synchronize()
        check = orc.error_metrics(out.cpu().numpy(), ref.cpu().numpy())
        if not check['passed']:
            raise SystemExit(f'substituted block does not match the cuDNN block: {check}')
        plan = native.last_plan()
        results = {}
        mods = (('ours', cand), ('cudnn', block))
        for name, mod in mods:
            for _ in range(20):
                mod(x)
            results[name + '_graph_us'] = graph_step_ms(torch, stream, lambda k, m=mod: m(x), GRAPH_STEPS,
                                                        GRAPH_REPLAYS) * 1e3
        # Synchronized API time: rounds alternate between the two blocks (host
        # timing drifts over seconds); per block the median over rounds.
        rounds, per_round = 10, max(1, args.steps // 10)
        api_rounds = {name: [] for name, _ in mods}
        for r in range(rounds):
            for name, mod in (mods if r % 2 == 0 else mods[::-1]):
                stream.synchronize()
                t0 = time.perf_counter()
                for _ in range(per_round):
                    mod(x)
                    stream.synchronize()
                api_rounds[name].append((time.perf_counter() - t0) / per_round * 1e6)
        for name, _ in mods:
            results[name + '_api_us'] = statistics.median(api_rounds[name])
            results[name + '_api_rounds_us'] = api_rounds[name]
        # end to end: pinned host input -> block -> pinned host output
        xh = x.cpu().pin_memory()
        yh = torch.empty(tuple(out.shape), pin_memory=True)
        xd = torch.empty_like(x)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.e2e_steps):
            xd.copy_(xh, non_blocking=True)
            yh.copy_(cand(xd), non_blocking=True)
        b.record(stream)
        stream.synchronize()
        e2e_us = a.elapsed_time(b) / args.e2e_steps * 1e3
    line = {'metric': 'MobileNetV2 features[3] block latency, depthwise 3x3 on gc_cuda_conv (config 4)',
            'value': results['ours_graph_us'], 'unit': 'us', 'n_gpus': 1, 'steps': args.steps,
            'warmup': 20, 'ms_per_step': results['ours_graph_us'] / 1e3, 'higher_is_better': False,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic N(0,1) input, seed 2',
            'config': {'workload': 'config4_block', 'replaced': replaced, 'kernel_plan': plan,
                       'input': [4, 24, 56, 56]},
            'block': results, 'speedup_graph': results['cudnn_graph_us'] / results['ours_graph_us'],
            'speedup_api': results['cudnn_api_us'] / results['ours_api_us'], 'check': check,
            'e2e': {'value': e2e_us, 'unit': 'us', 'h2d_bytes_per_step': x.numel() * 4,
                    'd2h_bytes_per_step': out.numel() * 4},
            # the timed region of `value`: GRAPH_REPLAYS replays of GRAPH_STEPS
            # block calls, one gc_cuda_conv launch each
            'gpu_launches': GRAPH_STEPS * GRAPH_REPLAYS * len(replaced)}
    print(json.dumps(line), flush=True)
    return 0


def run_sweep(args):
    """Config 3: the 80-shape sweep.  Per shape: device time of gc_cuda_conv
    (implementation 3) and of torch.nn.functional.conv2d (TF32 off, benchmark
    mode), both by CUDA-graph replay over rotating buffers larger than L2 where
    the shape allows; a 64-point FP64 check of our output; the roofline
    fraction of the bound that applies to the chosen kernel."""
    import torch
    import torch.nn.functional as F
    from groupconv_atlas_b200 import api, workloads
    from oracle import oracle as orc
    rank, world, local = dist_setup()
    if rank != 0:
        return 0
    torch.cuda.set_device(local)
    set_fp32_precision(torch)
    torch.backends.cudnn.benchmark = True
    native = api.Native()
    peaks, peak_kind = measured_peaks()
    props = torch.cuda.get_device_properties(local)
    ffma_peak = props.multi_processor_count * 128 * 2 * 1.965e9 / 1e12  # TFLOP/s at max SM clock
    tensor_peak = peaks['bf16_tflops'] / 6
    stream = torch.cuda.Stream()
    rows = []
    for s in workloads.sweep_shapes():
        x_host, w_host = workloads.sweep_inputs(s, 0, 1)
        nbytes = 4 * (2 * math.prod(s.input) + math.prod(s.weight))
        sets = int(max(1, min(8, math.ceil(3 * L2_BYTES / nbytes))))
        g = torch.Generator(device='cuda').manual_seed(int(s.id[3:11], 16))
        with torch.cuda.stream(stream):
            xs = [torch.rand(s.input, device='cuda', generator=g) * 2 - 1 for _ in range(sets)]
            ys = [torch.empty(s.output, device='cuda') for _ in range(sets)]
            w = torch.from_numpy(w_host).cuda()
            native.cuda(s, xs[0], w, ys[0], 3, stream.cuda_stream)
            plan = native.last_plan()
            stream.synchronize()
            check = orc.check_points(s, xs[0].cpu().numpy(), w_host, ys[0].cpu().numpy())
            reps = 20
            ours = graph_step_ms(torch, stream, lambda k: native.cuda(s, xs[k % sets], w, ys[k % sets], 3,
                                                                      stream.cuda_stream), reps)
            with torch.inference_mode():
                for k in range(3):
                    F.conv2d(xs[k % sets], w, padding=1, groups=s.groups)
                theirs = graph_step_ms(torch, stream,
                                       lambda k: F.conv2d(xs[k % sets], w, padding=1, groups=s.groups), reps)
        flops = 2 * math.prod(s.output) * s.cpg * 9
        gbs = nbytes / (ours / 1e3) / 1e9
        tflops = flops / (ours / 1e3) / 1e12
        if plan.startswith('kernel=tf32x3'):
            bound, frac = 'tensor', tflops / tensor_peak
        elif s.cpg >= 4:
            bound, frac = 'fp32', max(tflops / ffma_peak, gbs / peaks['hbm_gbs'])
        else:
            bound, frac = 'hbm', gbs / peaks['hbm_gbs']
        rows.append({'shape': [s.n, s.cin, s.h, s.w, s.cpg], 'us': ours * 1e3, 'cudnn_us': theirs * 1e3,
                     'speedup_vs_cudnn': theirs / ours, 'gbs': gbs, 'tflops': tflops, 'bound': bound,
                     'frac': frac, 'points_ok': check['passed'], 'kernel': plan.split()[0].split('=')[1]})
        del xs, ys
        torch.cuda.empty_cache()
    geo = lambda v: math.exp(statistics.fmean(math.log(max(x, 1e-12)) for x in v))
    line = {'metric': 'config-3 sweep: geomean speedup of gc_cuda_conv over torch/cuDNN (TF32 off), 80 shapes',
            'value': geo(r['speedup_vs_cudnn'] for r in rows), 'unit': 'x', 'n_gpus': 1, 'steps': 20,
            'warmup': 3, 'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32',
            'data': 'synthetic uniform[-1,1) inputs, weights uniform[-1,1)/sqrt(9 cpg)',
            'config': {'workload': 'config3', 'shapes': len(rows), 'timing': 'CUDA-graph replay, both sides'},
            'wins': sum(r['speedup_vs_cudnn'] > 1.05 for r in rows),
            'losses': sum(r['speedup_vs_cudnn'] < 1 / 1.05 for r in rows),
            'all_points_ok': all(r['points_ok'] for r in rows),
            'geomean_roofline_frac': geo(r['frac'] for r in rows),
            'peaks': {'hbm_gbs': peaks['hbm_gbs'], 'ffma_tflops': ffma_peak, 'tf32x3_tflops': tensor_peak,
                      'source': peak_kind},
            'rows': rows}
    print(json.dumps(line), flush=True)
    return 0 if line['all_points_ok'] else 1


def paired_shape_rows(args, entries):
    """Per shape of `entries` ((Shape, extra row fields) pairs): paired
    batches of device timings of gc_cuda_conv (implementation 3, or 0 for
    layers outside B geometry) and
    torch.nn.functional.conv2d (TF32 off, benchmark mode), the two run in a
    seeded random order within each batch (bench/cuda_run.py:231-248); a
    sample is one CUDA-graph replay of `repeats` calls (about 1 ms of work, at
    most 20 calls) over rotating buffers larger than L2 where the shape
    allows; the speed-up and its 95 % interval come from the paired
    batch-median bootstrap (bench/stats.py).  Inputs are the reference's
    seeded per-shape inputs; every output is checked at 64 FP64 points before
    timing, against the reference's fixed tolerances and against the
    1e-5 * sum|x*w| bound.  Returns one row per shape."""
    import random
    import torch
    import torch.nn.functional as F
    from groupconv_atlas_b200 import api, stats
    from oracle import oracle as orc
    native = api.Native()
    stream = torch.cuda.Stream()
    batches, samples = args.atlas_batches, args.atlas_samples
    rows = []
    for s, extra in entries:
        # implementations 1-3 serve B geometry (3x3, stride 1, pad 1, Cin ==
        # Cout) only; every other layer runs on implementation 0
        impl = 3 if (s.r, s.s, s.sh, s.sw, s.ph, s.pw, s.dh, s.dw, s.cin) == (3, 3, 1, 1, 1, 1, 1, 1, s.cout) else 0
        x_host, w_host = api.inputs(s)
        nbytes = 4 * (math.prod(s.input) + math.prod(s.output) + math.prod(s.weight))
        sets = int(max(1, min(8, math.ceil(3 * L2_BYTES / nbytes))))
        g = torch.Generator(device='cuda').manual_seed(int(s.id[3:11], 16))
        with torch.cuda.stream(stream):
            xs = [torch.from_numpy(x_host).cuda()] + [torch.rand(s.input, device='cuda', generator=g) * 2 - 1
                                                      for _ in range(sets - 1)]
            ys = [torch.empty(s.output, device='cuda') for _ in range(sets)]
            w = torch.from_numpy(w_host).cuda()
            native.cuda(s, xs[0], w, ys[0], impl, stream.cuda_stream)
            plan = native.last_plan()
            stream.synchronize()
            y0 = ys[0].cpu().numpy()
        check = orc.check_points(s, x_host, w_host, y0)
        abs_sum = orc.oracle_points(s, np.abs(x_host), np.abs(w_host), check['points'])
        got = np.array([float(y0[p]) for p in check['points']])
        expected = orc.oracle_points(s, x_host, w_host, check['points'])
        bound_ok = bool(np.all(np.abs(got - expected) <= orc.BOUND_FACTOR * abs_sum))
        del x_host, y0
        conv = dict(stride=(s.sh, s.sw), padding=(s.ph, s.pw), dilation=(s.dh, s.dw), groups=s.groups)
        calls = {'ours': lambda k: native.cuda(s, xs[k % sets], w, ys[k % sets], impl, stream.cuda_stream),
                 'cudnn': lambda k: F.conv2d(xs[k % sets], w, **conv)}
        graphs, repeats = {}, {}
        with torch.cuda.stream(stream), torch.inference_mode():
            for name, call in calls.items():
                for k in range(10):
                    call(k)
                pilot = graph_step_ms(torch, stream, call, 3) * 1e3
                repeats[name] = max(1, min(20, int(1000.0 / max(pilot, 1.0))))
                graph = torch.cuda.CUDAGraph()
                stream.synchronize()
                with torch.cuda.graph(graph, stream=stream):
                    for k in range(repeats[name]):
                        call(k)
                graph.replay()
                graphs[name] = graph
            stream.synchronize()
            medians = {name: [] for name in calls}
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * samples)]
            for b in range(batches):
                order = list(calls)
                random.Random(f'{stats.SEED}:{s.id}:{b}').shuffle(order)
                for name in order:
                    for i in range(samples):
                        ev[2 * i].record(stream)
                        graphs[name].replay()
                        ev[2 * i + 1].record(stream)
                    stream.synchronize()
                    us = [ev[2 * i].elapsed_time(ev[2 * i + 1]) * 1e3 / repeats[name] for i in range(samples)]
                    medians[name].append(statistics.median(us))
        cmp = stats.compare_batches(medians['cudnn'], medians['ours'])
        rows.append({**extra, 'shape': [s.n, s.cin, s.h, s.w, s.cpg], 'stride': s.sh, 'implementation': impl,
                     'shape_id': s.id,
                     'kernel': plan.split()[0].split('=')[1], 'us': statistics.median(medians['ours']),
                     'cudnn_us': statistics.median(medians['cudnn']), 'speedup_vs_cudnn': cmp['speedup'],
                     'ci95': cmp['ci95'], 'classification': cmp['classification'],
                     'repeats': repeats, 'points_ok': check['passed'], 'bound_ok': bound_ok,
                     'max_abs_err': check['max_abs'], 'reduction_terms': s.cpg * s.r * s.s})
        del graphs, xs, ys
        torch.cuda.empty_cache()
    return rows


def shape_set_line(args, workload, metric, rows, data, extra=None):
    geo = lambda v: math.exp(statistics.fmean(math.log(max(x, 1e-12)) for x in v))
    counts = {c: sum(r['classification'] == c for r in rows) for c in ('WIN', 'TIE', 'LOSS', 'UNCERTAIN')}
    ok = all(r['bound_ok'] and (r['points_ok'] or r['reduction_terms'] > 576) for r in rows)
    line = {'metric': metric, 'value': geo(r['speedup_vs_cudnn'] for r in rows), 'unit': 'x', 'n_gpus': 1,
            'steps': args.atlas_batches * args.atlas_samples, 'warmup': 10, 'higher_is_better': True,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32', 'data': data,
            'config': {'workload': workload, 'shapes': len(rows), 'batches': args.atlas_batches,
                       'samples_per_batch': args.atlas_samples,
                       'timing': 'CUDA-graph replay, both sides, seeded random order per batch',
                       'l2': 'rotating input/output sets, 3x L2 where the shape allows'},
            'classification': counts, 'all_checks_ok': ok, **(extra or {}), 'rows': rows}
    print(json.dumps(line), flush=True)
    return 0 if ok else 1


def run_atlas(args):
    """The reference's 80-shape Atlas (C256, N{1,32} x H=W{7..112} x
    cpg{1..64,256}) measured the reference's way (paired_shape_rows)."""
    import torch
    from groupconv_atlas_b200 import workloads
    rank, world, local = dist_setup()
    if rank != 0:
        return 0
    torch.cuda.set_device(local)
    set_fp32_precision(torch)
    torch.backends.cudnn.benchmark = True
    rows = paired_shape_rows(args, [(s, {}) for s in workloads.atlas_shapes()])
    return shape_set_line(args, 'atlas', 'atlas: geomean speedup of gc_cuda_conv over torch/cuDNN (TF32 off), '
                          '80 shapes', rows, 'synthetic: the reference seeding per shape id, x, w ~U[-1,1)')


def run_model_layers(args):
    """The reference's 12 frozen model-layer operations: the 8 without bias
    measured like the Atlas; the 4 biased ConvNeXt layers reported as
    unsupported (the ABI has no bias), as bench/model_run.py does."""
    import torch
    from groupconv_atlas_b200 import workloads
    rank, world, local = dist_setup()
    if rank != 0:
        return 0
    torch.cuda.set_device(local)
    set_fp32_precision(torch)
    torch.backends.cudnn.benchmark = True
    layers = workloads.model_layers()
    rows = paired_shape_rows(args, [(l.shape, {'model': l.model, 'module_path': l.module_path})
                                    for l in layers if not l.bias])
    unsupported = [{'model': l.model, 'module_path': l.module_path, 'n': l.shape.n, 'status': 'UNSUPPORTED',
                    'reason': 'bias not implemented'} for l in layers if l.bias]
    return shape_set_line(args, 'model_layers', 'model layers: geomean speedup of gc_cuda_conv over torch/cuDNN '
                          '(TF32 off), 8 no-bias layers', rows,
                          'synthetic: the reference seeding per shape id, x, w ~U[-1,1)',
                          {'unsupported': unsupported})


def main(argv=None):
    args = parse_args(argv)
    if args.impl == 'reference':
        return run_reference(args)
    if args.workload == 'config4_block':
        return run_block(args)
    if args.workload == 'config3':
        return run_sweep(args)
    if args.workload == 'atlas':
        return run_atlas(args)
    if args.workload == 'model_layers':
        return run_model_layers(args)
    return run_ours(args)


if __name__ == '__main__':
    raise SystemExit(main())
