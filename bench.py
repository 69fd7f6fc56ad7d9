#!/usr/bin/env python
"""Benchmark of the B200 grouped-convolution engine (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...
    python bench.py --impl reference ...     # the reference's CPU implementation

A step is one pass of gc_cuda_conv (implementation 3, the production choice)
over one batch of synthetic input already resident in HBM.  Default
workload: the large-batch ResNeXt-style layer N1024 C256 56x56, 32 groups
(8 channels per group), strong-scaled: the batch is split across the ranks
by ``shard.units_for_rank`` (contiguous image ranges passed to the unchanged
C ABI by pointer offset; group blocks when there are fewer images than
ranks), no collective on the data path.  The same line carries secondary
blocks measured the same way (``--blocks``; default the 64-channel-group
variant of that layer on the tensor-core path and the depthwise N32 C256
56x56 layer), each with its own roofline, cuDNN ratio and end-to-end figure.

Reported per workload: ``value`` (GB/s of algorithmic bytes, whole job,
device time of K back-to-back steps, max over ranks) and ``gflops``,
``e2e`` (same metric through the C ABI with the batch in pinned host memory
and both copies inside the timed region), ``roofline`` of the kernel against
the bound that applies (HBM copy rate, FP32 FFMA rate or the 3xTF32
tensor-core ceiling, each measured), ``cudnn`` (torch.nn.functional.conv2d in
a fresh process, TF32 off, benchmark mode), ``cpu_baseline`` (the
reference's CPU library on the host cores), ``clocks`` sampled through NVML
while timing.
"""
from __future__ import annotations

import argparse
import ctypes as ct
import dataclasses
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

from groupconv_atlas_b200.clocks import ClockSampler  # noqa: E402

METRIC = 'grouped-conv GB/s & GFLOP/s (% of B200 roofline), latency ratio vs cuDNN, 1/2/4/8 GPU'
UNIT = 'GB/s'
L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {'hbm_gbs': 6650.0, 'bf16_tflops': 1590.0}
WORKLOADS = ['config1', 'config2', 'config4_leaf', 'config5_g32', 'config5_g4', 'config4_block', 'config3', 'atlas',
             'model_layers', 'kernels', 'nhwc']
DEFAULT_BLOCKS = 'config5_g4,config2'


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=20)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', choices=['ours', 'reference'], default='ours')
    ap.add_argument('--workload', default='config5_g32', choices=WORKLOADS)
    ap.add_argument('--scaling', choices=['weak', 'strong'], default=None,
                    help='weak: each rank runs the full workload batch; strong: the batch is sharded '
                         '(default: strong for the N1024 layers, weak otherwise)')
    ap.add_argument('--blocks', default=None,
                    help='comma-separated secondary workloads measured into the same line '
                         f'(default {DEFAULT_BLOCKS} with the default workload, none otherwise; "" for none)')
    ap.add_argument('--shape', default=None,
                    help='N,C,H,W,CPG: a custom 3x3/s1/p1 shape (uniform inputs) instead of --workload')
    ap.add_argument('--batch', type=int, default=None,
                    help='override the workload batch (small cases for profiling)')
    ap.add_argument('--e2e-steps', type=int, default=10)
    ap.add_argument('--no-e2e', action='store_true')
    ap.add_argument('--no-cudnn', action='store_true')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-autotune', action='store_true',
                    help='skip gc_b200_autotune (the library\'s benchmark mode, run once per shape before timing, '
                         'as cuDNN runs with cudnn.benchmark)')
    ap.add_argument('--cpu-seconds', type=float, default=10.0, help='CPU baseline sample budget')
    ap.add_argument('--atlas-batches', type=int, default=10, help='atlas: paired batches per shape')
    ap.add_argument('--atlas-samples', type=int, default=30, help='atlas: samples per batch and implementation')
    ap.add_argument('--shapes', default='16,512,112,112,16;32,256,56,56,16;32,256,56,56,32',
                    help='kernels workload: N,C,H,W,CPG shapes separated by ";"')
    ap.add_argument('--families', default='tf32x3,direct_tma',
                    help='kernels workload: gc_b200_conv kernel families to compare')
    ap.add_argument('--cudnn-leg', default=None, help=argparse.SUPPRESS)  # internal: the fresh cuDNN process
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error('--warmup must be at least 3')
    if args.shape:
        args.workload = 'custom:' + args.shape
    if args.scaling is None:
        args.scaling = default_scaling(args.workload)
    if args.blocks is None:
        args.blocks = DEFAULT_BLOCKS if (args.workload == 'config5_g32' and not args.shape and args.batch is None) else ''
    args.block_list = [b for b in args.blocks.split(',') if b]
    return args


def default_scaling(workload):
    return 'strong' if workload.startswith('config5') else 'weak'


def _json(path):
    return json.loads(path.read_text()) if path.exists() else None


def peaks():
    """Roofline denominators.  HBM: the driver-measured copy rate of this
    pool's B200s (MEASURED_PEAKS.json).  FP32 FFMA and the tensor core's TF32
    rate: this library's own probes (gc_b200_probe_*), measured on a B200 of
    the same pool and committed in profiles/peaks.json.  Each has a labelled
    fallback when its file is absent."""
    out = {}
    mp = _json(ROOT / 'MEASURED_PEAKS.json')
    if mp:
        out['hbm_gbs'], out['hbm_source'] = float(mp['hbm_gbs']), 'measured copy bandwidth (MEASURED_PEAKS.json)'
        bf16 = float(mp.get('bf16_tflops', 0)) or FALLBACK_PEAKS['bf16_tflops']
    else:
        out['hbm_gbs'], out['hbm_source'] = FALLBACK_PEAKS['hbm_gbs'], 'fallback copy bandwidth'
        bf16 = FALLBACK_PEAKS['bf16_tflops']
    pk = _json(ROOT / 'profiles' / 'peaks.json')
    if pk:
        out['ffma_tflops'] = float(pk['ffma_tflops'])
        out['ffma_source'] = f"measured FFMA probe (profiles/peaks.json, {pk['when']})"
        out['tf32x3_tflops'] = float(pk['tf32x3_tflops'])
        out['tf32x3_source'] = (f"measured tcgen05 TF32 MMA probe / 3 (three TF32 products per FP32 product; "
                                f"profiles/peaks.json, {pk['when']})")
    else:
        out['ffma_tflops'] = 148 * 128 * 2 * 1.965e9 / 1e12
        out['ffma_source'] = 'nominal: 148 SMs x 128 FMA/clk x 2 x 1.965 GHz (no probe record)'
        out['tf32x3_tflops'] = bf16 / 2 / 3
        out['tf32x3_source'] = 'bf16 dense GEMM rate / 2 (TF32 rate) / 3 (no probe record)'
    return out


def recorded_traffic(workload):
    """DRAM bytes per launch of the dominant kernel, from a committed ncu summary."""
    data = _json(ROOT / 'profiles' / 'traffic.json')
    entry = (data or {}).get(workload)
    return None if entry is None else entry.get('dram_bytes_per_launch')


def roofline_of(plan, step_bytes, step_flops, launches, kernel_ms, pk):
    """Roofline of the dominant kernel: algorithmic bytes and FLOPs per launch
    over the average launch duration, against the bound that applies.  The
    tensor-core plans are bound by the 3xTF32 ceiling; the others by HBM or
    by the FP32 FFMA rate, whichever gives the longer minimum time."""
    achieved_gbs = (step_bytes / launches) / (kernel_ms / 1e3) / 1e9
    achieved_tflops = (step_flops / launches) / (kernel_ms / 1e3) / 1e12
    t_hbm = (step_bytes / launches) / (pk['hbm_gbs'] * 1e9)
    t_ffma = (step_flops / launches) / (pk['ffma_tflops'] * 1e12)
    common = {'hbm_achieved_gbs': achieved_gbs, 'hbm_frac': achieved_gbs / pk['hbm_gbs'],
              'fp32_tflops': achieved_tflops}
    if plan.startswith('kernel=tf32x3'):
        return {'bound': 'tensor', 'achieved': achieved_tflops, 'peak': pk['tf32x3_tflops'], 'unit': 'TFLOP/s',
                'frac': achieved_tflops / pk['tf32x3_tflops'], 'peak_source': pk['tf32x3_source'],
                'ffma_frac': achieved_tflops / pk['ffma_tflops'], **common}
    if t_ffma > t_hbm:
        return {'bound': 'fp32', 'achieved': achieved_tflops, 'peak': pk['ffma_tflops'], 'unit': 'TFLOP/s',
                'frac': achieved_tflops / pk['ffma_tflops'], 'peak_source': pk['ffma_source'], **common}
    return {'bound': 'hbm', 'achieved': achieved_gbs, 'peak': pk['hbm_gbs'], 'unit': 'GB/s',
            'frac': achieved_gbs / pk['hbm_gbs'], 'peak_source': pk['hbm_source'],
            'ffma_frac': achieved_tflops / pk['ffma_tflops'], **common}


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


def workload_config(name, shape):
    """The `config` object of a line: the same keys and values in both arms
    (the workload, its full shape, how the timing keeps L2 from serving
    re-reads).  Launch plans and the parallel split go elsewhere."""
    n, c, h, w = shape.input
    batch_bytes = 4 * 2 * n * c * h * w
    l2 = (f'inputs larger than L2: one step reads and writes {batch_bytes / 2**30:.2f} GiB > L2 126 MiB'
          if batch_bytes > 3 * L2_BYTES else
          'rotating input/output sets larger than 3x the 126 MiB L2 (GPU arm); one set per step')
    return {'workload': name, 'shape': dataclasses.asdict(shape), 'l2': l2}


def run_reference(args):
    rank, world, _ = dist_setup()
    if rank != 0:
        return 0  # the CPU reference runs on rank 0 only
    from groupconv_atlas_b200 import workloads
    wl = workloads.by_name(args.workload, batch=args.batch, with_x=False)
    m = sample_images(args.workload, wl.shape.n, 0.25)
    _, x, w = workload_host(args.workload, 0, m)
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
    sample = f'{m} of the workload\'s {wl.shape.n} images per step, GC_BLOCKED schedule, {cores} threads'
    line = {'impl': 'reference', 'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': args.gpus,
            'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': elapsed / args.steps * 1e3,
            'higher_is_better': True, 'scaling': args.scaling, 'vs_baseline': None, 'dtype': 'f32',
            'data': 'synthetic (seeded per-image generators, distributions of the workload definition)',
            'gflops': step_flops * args.steps / elapsed / 1e9,
            'config': workload_config(args.workload, wl.shape),
            'cpu_baseline': {'value': value, 'unit': UNIT, 'cores': cores, 'kind': kind, 'sample': sample},
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


@dataclasses.dataclass
class Piece:
    """One gc_cuda_conv call of a rank: a unit of ``shard.units_for_rank``
    (or a chunk of one) as a sub-shape with element offsets into the
    rank-local x, the full weights and the rank-local y."""
    shape: object
    x_off: int
    w_off: int
    y_off: int

    @property
    def x_len(self):
        return math.prod(self.shape.input)

    @property
    def w_len(self):
        return math.prod(self.shape.weight)

    @property
    def y_len(self):
        return math.prod(self.shape.output)

    @property
    def bytes(self):
        return 4 * (self.x_len + self.w_len + self.y_len)

    @property
    def flops(self):
        return 2 * self.y_len * self.shape.cpg * self.shape.r * self.shape.s


def rank_work(full, scaling, world, rank):
    """(first image, image count, units relative to that first image) of this
    rank: weak scaling gives every rank its own batch of the workload's shape
    (images rank*N .. rank*N+N-1 of the seeded stream); strong scaling splits
    the one batch with shard.units_for_rank."""
    from groupconv_atlas_b200 import shard
    if scaling == 'weak':
        return rank * full.n, full.n, [shard.Unit(0, full.n, 0, full.cin)]
    units = shard.units_for_rank(full, world, rank)
    if not units:
        return 0, 0, []
    first = units[0].n0
    return first, units[-1].n1 - first, [shard.Unit(u.n0 - first, u.n1 - first, u.c0, u.c1) for u in units]


def pieces_of(units, local_shape, chunks=1):
    """Pieces of the rank's units; with chunks > 1 a unit of several images
    is split into up to `chunks` image ranges (the end-to-end pipeline)."""
    from groupconv_atlas_b200 import shard
    out = []
    for u in units:
        n = u.images()
        parts = max(1, min(chunks, n))
        for i in range(parts):
            lo, hi = u.n0 + i * n // parts, u.n0 + (i + 1) * n // parts
            if hi <= lo:
                continue
            v = shard.Unit(lo, hi, u.c0, u.c1)
            out.append(Piece(v.shape(local_shape), *v.offsets(local_shape)))
    return out


def gate(pieces, x_local, w_full, y_local):
    """The correctness gate before timing: 64 FP64 points of every piece's
    output, each checked on the piece's own sub-shape and views (outputs of
    channels or images the rank does not compute are never read).  x_local,
    w_full and y_local are the rank-local input, the weights and the
    rank-local output (numpy arrays or tensors, flattened here).  Returns the
    failures as (piece index, failed point count); empty when all pass."""
    from oracle import oracle as orc
    xf, wf, yf = x_local.reshape(-1), w_full.reshape(-1), y_local.reshape(-1)
    failed = []
    for i, p in enumerate(pieces):
        xv = xf[p.x_off:p.x_off + p.x_len].reshape(p.shape.input)
        wv = wf[p.w_off:p.w_off + p.w_len].reshape(p.shape.weight)
        yv = yf[p.y_off:p.y_off + p.y_len].reshape(p.shape.output)
        check = orc.check_points(p.shape, xv, wv, yv)
        if not check['passed']:
            failed.append((i, check['failed_points']))
    return failed


def measure_workload(args, name, scaling, ctx, primary):
    """Everything one workload reports: correctness gate, device-timed
    steps, roofline, end to end, cuDNN and CPU baselines."""
    import torch
    from groupconv_atlas_b200 import shard, workloads
    native, rank, world, local = ctx['native'], ctx['rank'], ctx['world'], ctx['local']
    full = workloads.by_name(name, batch=args.batch if primary else None, with_x=False)
    first, local_n, units = rank_work(full.shape, scaling, world, rank)
    local_shape = dataclasses.replace(full.shape, n=max(1, local_n))
    x_host = workloads.images(full.shape, full.seed, full.dist, first, local_shape.n)
    w_host = full.w
    xh = torch.from_numpy(x_host).pin_memory()
    wh = torch.from_numpy(w_host).pin_memory()
    del x_host
    pieces = pieces_of(units, local_shape)
    set_bytes = 4 * (math.prod(local_shape.input) + math.prod(local_shape.output))
    sets = int(min(4096, max(1, math.ceil(3 * L2_BYTES / set_bytes))))
    stream = torch.cuda.Stream()
    dw = wh.to('cuda')
    xs = [xh.to('cuda') for _ in range(sets)]
    ys = [torch.empty(local_shape.output, device='cuda') for _ in range(sets)]
    torch.cuda.synchronize()

    def view(t, off, shape):
        return t.view(-1)[off:off + math.prod(shape)].view(shape)

    calls = [[Call(native, p.shape, view(xs[i], p.x_off, p.shape.input), view(dw, p.w_off, p.shape.weight),
                   view(ys[i], p.y_off, p.shape.output), stream.cuda_stream) for p in pieces] for i in range(sets)]
    launches = len(pieces)
    step_bytes = sum(p.bytes for p in pieces)
    step_flops = sum(p.flops for p in pieces)

    # Benchmark mode once per piece shape (the library's own plan search, as
    # the cuDNN baseline runs with cudnn.benchmark), outside the timed region.
    if not args.no_autotune:
        with torch.cuda.stream(stream):
            for p in pieces:
                native.autotune(p.shape, view(xs[0], p.x_off, p.shape.input), view(dw, p.w_off, p.shape.weight),
                                view(ys[0], p.y_off, p.shape.output), stream=stream.cuda_stream)
        stream.synchronize()
    # Correctness gate before timing: 64 FP64 points of every piece's output
    # (each unit's own sub-shape and views).
    plan = ''
    with torch.cuda.stream(stream):
        for c in calls[0]:
            c()
            plan = native.last_plan()
    stream.synchronize()
    failed = gate(pieces, xh.numpy(), wh.numpy(), ys[0])  # y indexed point by point on the device
    if failed:
        raise SystemExit(f'{name}: correctness gate failed on rank {rank}: {failed} [{plan}]')
    if native.device_status(clear=True):
        raise SystemExit('device status word set after the correctness gate')

    # Device-timed region: K back-to-back steps.
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
    # timed region on the launch stream, over the launches inside it
    # (consecutive launches overlap prologue and tail through programmatic
    # dependent launch, so the region, not an event pair per launch, is the
    # per-launch cost).
    kernel_ms = elapsed_ms / (args.steps * max(1, launches))

    def graph_step(k):
        for c in calls[k % sets]:
            c()
    graph_kernel_ms = None
    if launches:
        with torch.cuda.stream(stream):
            graph_kernel_ms = graph_step_ms(torch, stream, graph_step, min(args.steps, 50)) / launches
    max_elapsed = shard.max_over_ranks(elapsed_ms)
    job_bytes = shard.sum_over_ranks(step_bytes)
    job_flops = shard.sum_over_ranks(step_flops)
    value = job_bytes * args.steps / (max_elapsed / 1e3) / 1e9
    gflops = job_flops * args.steps / (max_elapsed / 1e3) / 1e9

    e2e = None
    if not args.no_e2e:
        e2e = end_to_end(args, native, local_shape, units, xh, wh, torch)
    pk = peaks()
    roof = roofline_of(plan, step_bytes, step_flops, max(1, launches), kernel_ms, pk) if launches else None
    if roof is not None and roof['bound'] == 'hbm' and rank == 0 and sets > 1:
        # Context for launch-sized transfers: a device copy x -> y of the
        # same bytes per launch, same rotating sets, back to back.
        copy_ms = copy_same_bytes_ms(torch, stream, xs, ys, args.steps)
        copy_gbs = 2 * xs[0].numel() * 4 / (copy_ms / 1e3) / 1e9
        roof['same_size_copy'] = {'gbs': copy_gbs, 'ms': copy_ms, 'frac_of_it': roof['achieved'] / copy_gbs,
                                  'what': 'torch copy_ of x into y (read + write bytes), same rotating sets, '
                                          'K back-to-back copies'}
    cudnn = None
    if not args.no_cudnn and rank == 0 and launches:
        cudnn = cudnn_fresh_process(args, local_shape, local, sets,
                                    (elapsed_ms / args.steps, graph_kernel_ms * launches))
    cpu = None
    if not args.no_cpu_baseline and rank == 0 and world == 1:
        cpu = cpu_baseline(name, local_shape.n, args.cpu_seconds if primary else args.cpu_seconds / 2)
    status = native.device_status(clear=True)
    if status:
        raise SystemExit(f'device status word set during timing: {status:#x}')
    clocks = sampler.summary()
    if world > 1:
        import torch.distributed as dist
        gathered = [None] * world
        dist.all_gather_object(gathered, clocks)
        clocks = gathered[0] | {'per_rank_reasons': [g.get('reasons') for g in gathered]}
    if roof is not None:
        roof.update({'traffic': recorded_traffic(name), 'kernel_ms': kernel_ms,
                     'kernel_ms_timing': 'CUDA events bracketing the timed region on the launch stream / launches',
                     'graph_kernel_ms': graph_kernel_ms,
                     'algorithmic_bytes_per_launch': step_bytes / launches,
                     'algorithmic_flops_per_launch': step_flops / launches})
    del calls, xs, ys
    torch.cuda.empty_cache()
    return {'workload': name, 'value': value, 'unit': UNIT, 'gflops': gflops, 'ms_per_step': max_elapsed / args.steps,
            'scaling': scaling, 'config': workload_config(name, full.shape),
            'run': {'implementation': 3, 'kernel_plan': plan, 'images_this_rank': local_n if units else 0,
                    'units_this_rank': len(units), 'launches_per_step': launches,
                    'rotating_sets': sets,
                    'parallelism': f'{scaling} scaling over {world} GPU(s): '
                                   + ('each rank its own batch' if scaling == 'weak'
                                      else 'shard.units_for_rank (batch ranges, group blocks when N < ranks)')
                                   + ', no collective on the data path'},
            'roofline': roof, 'e2e': e2e, 'gpu_launches': args.steps * launches, 'clocks': clocks,
            'cudnn': cudnn, 'cpu_baseline': cpu}


def run_ours(args):
    import torch
    import torch.distributed as dist
    from groupconv_atlas_b200 import api

    rank, world, local = dist_setup()
    torch.cuda.set_device(local)
    if world > 1:
        # NCCL's own log lines go to stderr unless the caller chose a file:
        # stdout carries only the JSON line
        os.environ.setdefault('NCCL_DEBUG_FILE', '/dev/stderr')
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device('cuda', local))
    ctx = {'native': api.Native(), 'rank': rank, 'world': world, 'local': local}
    main_result = measure_workload(args, args.workload, args.scaling, ctx, primary=True)
    blocks = [measure_workload(args, b, default_scaling(b), ctx, primary=False) for b in args.block_list]
    if rank == 0:
        m = main_result
        line = {
            'metric': METRIC, 'value': m['value'], 'unit': UNIT, 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': m['ms_per_step'], 'higher_is_better': True,
            'scaling': m['scaling'], 'vs_baseline': None, 'dtype': 'f32',
            'data': 'synthetic (seeded per-image generators, distributions of the workload definition)',
            'gflops': m['gflops'], 'config': m['config'], 'run': m['run'], 'roofline': m['roofline'],
            'e2e': m['e2e'], 'gpu_launches': m['gpu_launches'], 'clocks': m['clocks'], 'cudnn': m['cudnn'],
            'cpu_baseline': m['cpu_baseline'],
            'blocks': blocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def end_to_end(args, native, shape, units, xh, wh, torch):
    """Same metric, through the C ABI with host buffers: per step each piece
    of the rank's units (batch units in up to 8 image chunks) is copied
    host->device (pinned), convolved as soon as its copy lands, and copied
    back; three streams overlap the two copy directions with compute, and two
    device buffer sets alternate between steps, so the copies of step k+1
    never wait for the convolutions of step k."""
    from groupconv_atlas_b200 import shard
    pieces = pieces_of(units, shape, chunks=8)
    if not pieces:  # a rank without work still takes every collective step of the others
        barrier()
        barrier()
        shard.max_over_ranks(0.0)
        shard.sum_over_ranks(0.0)
        return None
    dws = [torch.empty(shape.weight, device='cuda') for _ in range(2)]
    dxs = [torch.empty(shape.input, device='cuda') for _ in range(2)]
    dys = [torch.empty(shape.output, device='cuda') for _ in range(2)]
    yh = torch.empty(shape.output, pin_memory=True)
    s_in, s_cmp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()

    def flat(t, off, n):
        return t.view(-1)[off:off + n]

    calls = [[Call(native, p.shape, flat(dxs[b], p.x_off, p.x_len).view(p.shape.input),
                   flat(dws[b], p.w_off, p.w_len).view(p.shape.weight),
                   flat(dys[b], p.y_off, p.y_len).view(p.shape.output), s_cmp.cuda_stream) for p in pieces]
             for b in range(2)]
    ev_in = [[torch.cuda.Event() for _ in pieces] for _ in range(2)]
    ev_cmp = [[torch.cuda.Event() for _ in pieces] for _ in range(2)]
    ev_out = [[torch.cuda.Event() for _ in pieces] for _ in range(2)]
    used = [False, False]

    def step(k):
        b = k & 1
        with torch.cuda.stream(s_in):
            if used[b]:
                s_in.wait_event(ev_cmp[b][-1])  # step k-2 finished reading these weights
            dws[b].copy_(wh, non_blocking=True)
            for j, p in enumerate(pieces):
                if used[b]:
                    s_in.wait_event(ev_cmp[b][j])  # step k-2 finished reading this x piece
                flat(dxs[b], p.x_off, p.x_len).copy_(flat(xh, p.x_off, p.x_len), non_blocking=True)
                ev_in[b][j].record(s_in)
        for j in range(len(pieces)):
            s_cmp.wait_event(ev_in[b][j])
            if used[b]:
                s_cmp.wait_event(ev_out[b][j])  # step k-2 finished reading this y piece
            calls[b][j]()
            ev_cmp[b][j].record(s_cmp)
        with torch.cuda.stream(s_out):
            for j, p in enumerate(pieces):
                s_out.wait_event(ev_cmp[b][j])
                flat(yh, p.y_off, p.y_len).copy_(flat(dys[b], p.y_off, p.y_len), non_blocking=True)
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
    s_in.wait_stream(s_out)
    torch.cuda.synchronize()
    barrier()
    ms = shard.max_over_ranks(t0.elapsed_time(t1))
    last = dys[(2 + args.e2e_steps) & 1]
    consistent = all(torch.equal(flat(yh, p.y_off, p.y_len), flat(last, p.y_off, p.y_len).cpu()) for p in pieces)
    step_bytes = sum(p.bytes for p in pieces)
    job_bytes = shard.sum_over_ranks(step_bytes)
    e2e_value = job_bytes * args.e2e_steps / (ms / 1e3) / 1e9
    del calls, dxs, dys, dws
    torch.cuda.empty_cache()
    return {'value': e2e_value, 'unit': UNIT,
            'h2d_bytes_per_step': sum(4 * p.x_len for p in pieces) + 4 * math.prod(shape.weight),
            'd2h_bytes_per_step': sum(4 * p.y_len for p in pieces), 'steps': args.e2e_steps,
            'ms_per_step': ms / args.e2e_steps, 'pieces_per_step': len(pieces),
            'path': 'pinned host -> gc_cuda_conv per piece (C ABI via ctypes) -> pinned host, '
                    'copies and calls overlapped on three streams',
            'host_matches_device': bool(consistent)}


def cudnn_fresh_process(args, shape, device, sets, ours):
    """torch.nn.functional.conv2d on the same shape in a fresh process (so
    cuDNN's benchmark search is not hidden by a cache warmed in this one, as
    the reference's bench/cuda_run.py:124-156 does): TF32 off and read back,
    cudnn.benchmark, device time of back-to-back calls (eager) and of
    CUDA-graph replay, rotating inputs as large as ours."""
    spec = json.dumps({'shape': dataclasses.asdict(shape), 'device': device, 'sets': sets,
                       'steps': max(20, min(args.steps, 200))})
    env = dict(os.environ)
    for k in ('RANK', 'WORLD_SIZE', 'LOCAL_RANK', 'MASTER_ADDR', 'MASTER_PORT', 'LOCAL_WORLD_SIZE',
              'GROUP_RANK', 'TORCHELASTIC_RUN_ID'):
        env.pop(k, None)
    proc = subprocess.run([sys.executable, str(ROOT / 'bench.py'), '--cudnn-leg', spec], capture_output=True,
                          text=True, env=env, timeout=600)
    if proc.returncode != 0:
        return {'error': (proc.stderr or proc.stdout)[-400:]}
    res = json.loads(proc.stdout.strip().splitlines()[-1])
    res.update({'ours_ms_per_step': ours[0], 'ours_graph_ms_per_step': ours[1],
                'speedup_vs_cudnn': res['ms_per_step'] / ours[0],
                'speedup_vs_cudnn_graph': res['graph_ms_per_step'] / ours[1]})
    return res


def cudnn_leg(spec):
    """The fresh cuDNN process (see cudnn_fresh_process)."""
    import torch
    import torch.nn.functional as F
    from groupconv_atlas_b200.api import Shape
    cfg = json.loads(spec)
    shape = Shape(**cfg['shape'])
    torch.cuda.set_device(cfg['device'])
    set_fp32_precision(torch)
    torch.backends.cudnn.benchmark = True
    sets, steps = cfg['sets'], cfg['steps']
    g = torch.Generator(device='cuda').manual_seed(3)
    stream = torch.cuda.Stream()
    with torch.inference_mode(), torch.cuda.stream(stream):
        xs = [torch.rand(shape.input, device='cuda', generator=g) * 2 - 1 for _ in range(sets)]
        w = torch.rand(shape.weight, device='cuda', generator=g) * 2 - 1
        conv = lambda k: F.conv2d(xs[k % sets], w, padding=1, groups=shape.groups)
        for k in range(10):
            conv(k)
        stream.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for k in range(steps):
            conv(k)
        b.record(stream)
        stream.synchronize()
        eager_ms = a.elapsed_time(b) / steps
        outs = [None] * sets

        def step(k):
            outs[k % sets] = conv(k)
        graph_ms = graph_step_ms(torch, stream, step, min(steps, 50))
    print(json.dumps({'ms_per_step': eager_ms, 'graph_ms_per_step': graph_ms,
                      'timing': 'fresh process; back-to-back calls on one stream (eager) and CUDA-graph replay',
                      'api': 'torch.nn.functional.conv2d', 'tf32': False, 'benchmark': True,
                      'cudnn_version': torch.backends.cudnn.version()}))
    return 0


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
    init, seed 2, eval; batch-norm running statistics drawn from a seeded
    distribution so that they are not the identity), N4 input N(0,1).  Three
    blocks on the same input: the reference block (every layer on
    PyTorch/cuDNN); the candidate with only the depthwise 3x3 replaced by
    gc_cuda_conv (implementation 3), as the reference's
    bench/module_run.py:215-235 does; and the fused candidate, whose
    depthwise conv + batch norm + ReLU6 run as one gc_b200_conv_ex call (the
    normalisation folded into the weights and a bias, ReLU6 in the epilogue).
    Reported per block: latency from CUDA-graph replay (device) and the
    synchronized per-call wall time (API); the API speed-up of each candidate
    over the reference block with the reference's paired batch-median
    bootstrap (bench/stats.py) over alternating rounds."""
    import copy
    import torch
    import torchvision
    from groupconv_atlas_b200 import api, stats, torch_module
    from oracle import oracle as orc
    rank, world, local = dist_setup()
    if rank != 0:
        return 0
    torch.cuda.set_device(local)
    set_fp32_precision(torch)
    torch.backends.cudnn.benchmark = True
    torch.manual_seed(2)
    block = torchvision.models.mobilenet_v2(weights=None).features[3].eval()
    g = torch.Generator().manual_seed(2)
    for m in block.modules():
        if isinstance(m, torch.nn.BatchNorm2d):
            m.running_mean.copy_(torch.randn(m.num_features, generator=g) * 0.1)
            m.running_var.copy_(torch.rand(m.num_features, generator=g) * 0.5 + 0.75)
            m.weight.data.copy_(torch.rand(m.num_features, generator=g) * 0.5 + 0.75)
            m.bias.data.copy_(torch.randn(m.num_features, generator=g) * 0.1)
    block = block.cuda()
    cand = copy.deepcopy(block)
    fused = copy.deepcopy(block)
    native = api.Native()
    replaced = torch_module.substitute(cand, torch_module.is_depthwise_3x3, native)
    fused_names = torch_module.fuse_conv_bn_act(fused, torch_module.is_depthwise, native)
    x = torch.randn((4, 24, 56, 56), generator=torch.Generator().manual_seed(2)).cuda()
    stream = torch.cuda.Stream()
    mods = (('ours', cand), ('fused', fused), ('cudnn', block))
    with torch.inference_mode(), torch.cuda.stream(stream):
        ref = block(x)
        checks, plans = {}, {}
        for name, mod in mods[:2]:
            out = mod(x)
            plans[name] = native.last_plan()
            stream.synchronize()
            checks[name] = orc.error_metrics(out.cpu().numpy(), ref.cpu().numpy())
            if not checks[name]['passed']:
                raise SystemExit(f'{name} block does not match the cuDNN block: {checks[name]}')
        results = {}
        for name, mod in mods:
            for _ in range(20):
                mod(x)
            results[name + '_graph_us'] = graph_step_ms(torch, stream, lambda k, m=mod: m(x), GRAPH_STEPS,
                                                        GRAPH_REPLAYS) * 1e3
        # Synchronized API time: rounds alternate the order of the blocks
        # (host timing drifts over seconds); per round the median call.
        rounds, per_round = 10, max(3, args.steps // 10)
        api_rounds = {name: [] for name, _ in mods}
        for r in range(rounds):
            order = list(mods) if r % 2 == 0 else list(mods)[::-1]
            for name, mod in order:
                samples = []
                for _ in range(per_round):
                    stream.synchronize()
                    t0 = time.perf_counter()
                    mod(x)
                    stream.synchronize()
                    samples.append((time.perf_counter() - t0) * 1e6)
                api_rounds[name].append(statistics.median(samples))
        for name, _ in mods:
            results[name + '_api_us'] = statistics.median(api_rounds[name])
            results[name + '_api_rounds_us'] = api_rounds[name]
        api_cmp = {name: stats.compare_batches(api_rounds['cudnn'], api_rounds[name]) for name in ('ours', 'fused')}
        # end to end: pinned host input -> fused block -> pinned host output
        xh = x.cpu().pin_memory()
        yh = torch.empty(tuple(ref.shape), pin_memory=True)
        xd = torch.empty_like(x)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.e2e_steps):
            xd.copy_(xh, non_blocking=True)
            yh.copy_(fused(xd), non_blocking=True)
        b.record(stream)
        stream.synchronize()
        e2e_us = a.elapsed_time(b) / args.e2e_steps * 1e3
    line = {'metric': 'MobileNetV2 features[3] block latency with the depthwise conv on this library (config 4)',
            'value': results['fused_graph_us'], 'unit': 'us', 'n_gpus': 1, 'steps': args.steps,
            'warmup': 20, 'ms_per_step': results['fused_graph_us'] / 1e3, 'higher_is_better': False,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32',
            'data': 'synthetic N(0,1) input, seed 2; Kaiming-normal weights, seeded batch-norm statistics',
            'config': {'workload': 'config4_block', 'replaced': replaced, 'fused': fused_names,
                       'kernel_plans': plans, 'input': [4, 24, 56, 56]},
            'block': results,
            'speedup_graph': {n: results['cudnn_graph_us'] / results[n + '_graph_us'] for n in ('ours', 'fused')},
            'speedup_api': {n: api_cmp[n]['speedup'] for n in ('ours', 'fused')},
            'api_classification': {n: api_cmp[n]['classification'] for n in ('ours', 'fused')},
            'api_ci95': {n: api_cmp[n]['ci95'] for n in ('ours', 'fused')},
            'check': checks,
            'e2e': {'value': e2e_us, 'unit': 'us', 'h2d_bytes_per_step': x.numel() * 4,
                    'd2h_bytes_per_step': ref.numel() * 4, 'block': 'fused'},
            # the timed region of `value`: GRAPH_REPLAYS replays of GRAPH_STEPS
            # fused-block calls, one gc_b200_conv_ex launch each
            'gpu_launches': GRAPH_STEPS * GRAPH_REPLAYS * len(fused_names)}
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
    pk = peaks()
    ffma_peak, tensor_peak = pk['ffma_tflops'], pk['tf32x3_tflops']
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
            if not args.no_autotune:
                native.autotune(s, xs[0], w, ys[0], stream=stream.cuda_stream)
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
            bound, frac = 'fp32', max(tflops / ffma_peak, gbs / pk['hbm_gbs'])
        else:
            bound, frac = 'hbm', gbs / pk['hbm_gbs']
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
            'peaks': pk,
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
        with_bias = bool(extra.pop('with_bias', False))
        b_host = (np.random.default_rng(int(s.id[3:11], 16)).uniform(-1, 1, s.cout).astype(np.float32)
                  if with_bias else None)
        nbytes = 4 * (math.prod(s.input) + math.prod(s.output) + math.prod(s.weight))
        sets = int(max(1, min(8, math.ceil(3 * L2_BYTES / nbytes))))
        g = torch.Generator(device='cuda').manual_seed(int(s.id[3:11], 16))
        with torch.cuda.stream(stream):
            xs = [torch.from_numpy(x_host).cuda()] + [torch.rand(s.input, device='cuda', generator=g) * 2 - 1
                                                      for _ in range(sets - 1)]
            ys = [torch.empty(s.output, device='cuda') for _ in range(sets)]
            w = torch.from_numpy(w_host).cuda()
            db = torch.from_numpy(b_host).cuda() if with_bias else None
            if not args.no_autotune and not with_bias:
                native.autotune(s, xs[0], w, ys[0], stream=stream.cuda_stream)
            if with_bias:
                native.conv_ex(s, xs[0], w, ys[0], bias=db, stream=stream.cuda_stream)
            else:
                native.cuda(s, xs[0], w, ys[0], impl, stream.cuda_stream)
            plan = native.last_plan()
            stream.synchronize()
            y0 = ys[0].cpu().numpy()
        if with_bias:  # the convolution part of the output is what the oracle checks
            y0 = y0 - b_host[None, :, None, None]
        check = orc.check_points(s, x_host, w_host, y0)
        abs_sum = orc.oracle_points(s, np.abs(x_host), np.abs(w_host), check['points'])
        got = np.array([float(y0[p]) for p in check['points']])
        expected = orc.oracle_points(s, x_host, w_host, check['points'])
        bound_ok = bool(np.all(np.abs(got - expected) <= orc.BOUND_FACTOR * abs_sum))
        del x_host, y0
        conv = dict(stride=(s.sh, s.sw), padding=(s.ph, s.pw), dilation=(s.dh, s.dw), groups=s.groups)
        if with_bias:
            calls = {'ours': lambda k: native.conv_ex(s, xs[k % sets], w, ys[k % sets], bias=db,
                                                      stream=stream.cuda_stream),
                     'cudnn': lambda k: F.conv2d(xs[k % sets], w, db, **conv)}
        else:
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
        rows.append({**extra, 'shape': [s.n, s.cin, s.h, s.w, s.cpg], 'stride': s.sh,
                     'implementation': 'gc_b200_conv_ex (bias)' if with_bias else impl,
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
    """The reference's 12 frozen model-layer operations measured like the
    Atlas: the 8 without bias through gc_cuda_conv, the 4 biased ConvNeXt
    7x7 depthwise layers (which the reference reports as unsupported,
    bench/model_run.py:46-49) through gc_b200_conv_ex with their bias, against
    torch's conv2d with the same bias."""
    import torch
    from groupconv_atlas_b200 import workloads
    rank, world, local = dist_setup()
    if rank != 0:
        return 0
    torch.cuda.set_device(local)
    set_fp32_precision(torch)
    torch.backends.cudnn.benchmark = True
    layers = workloads.model_layers()
    rows = paired_shape_rows(args, [(l.shape, {'model': l.model, 'module_path': l.module_path,
                                               'bias': l.bias, 'with_bias': l.bias}) for l in layers])
    return shape_set_line(args, 'model_layers', 'model layers: geomean speedup over torch/cuDNN (TF32 off), '
                          '12 layers: 8 through gc_cuda_conv, the 4 biased ConvNeXt 7x7 depthwise layers '
                          'through gc_b200_conv_ex', rows,
                          'synthetic: the reference seeding per shape id, x, w ~U[-1,1), bias ~U[-1,1) seeded per '
                          'shape id')


def run_kernels(args):
    """Per shape and kernel family (gc_b200_conv), the device time of K
    back-to-back calls between CUDA events on the launching stream, after W
    warm-up calls; uniform inputs generated on the device.  The evidence for
    the production choice between kernel families."""
    import torch
    from groupconv_atlas_b200 import api
    from groupconv_atlas_b200.api import Shape
    rank, world, local = dist_setup()
    if rank != 0:
        return 0
    torch.cuda.set_device(local)
    native = api.Native()
    pk = peaks()
    stream = torch.cuda.Stream()
    rows = []
    for spec in args.shapes.split(';'):
        n, c, h, w, cpg = (int(v) for v in spec.split(','))
        s = Shape(n=n, cin=c, cout=c, h=h, w=w, groups=c // cpg)
        flops = 2 * n * c * h * w * cpg * 9
        nbytes = 4 * (2 * n * c * h * w + c * cpg * 9)
        with torch.cuda.stream(stream):
            x = torch.rand(s.input, device='cuda') * 2 - 1
            wt = (torch.rand(s.weight, device='cuda') * 2 - 1) / math.sqrt(9 * cpg)
            y = torch.empty(s.output, device='cuda')
            row = {'shape': [n, c, h, w, cpg]}
            for fam in args.families.split(','):
                try:
                    native.b200(s, x, wt, y, fam, stream.cuda_stream)
                except api.NativeError as e:
                    row[fam] = {'status': e.status, 'error': str(e)}
                    continue
                plan = native.last_plan()
                for _ in range(args.warmup):
                    native.b200(s, x, wt, y, fam, stream.cuda_stream)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(args.steps):
                    native.b200(s, x, wt, y, fam, stream.cuda_stream)
                b.record(stream)
                stream.synchronize()
                ms = a.elapsed_time(b) / args.steps
                row[fam] = {'us': ms * 1e3, 'tflops': flops / (ms / 1e3) / 1e12, 'gbs': nbytes / (ms / 1e3) / 1e9,
                            'plan': plan}
            times = {f: v['us'] for f, v in row.items() if isinstance(v, dict) and 'us' in v}
            row['fastest'] = min(times, key=times.get) if times else None
            rows.append(row)
        del x, y
        torch.cuda.empty_cache()
    print(json.dumps({'metric': 'device time per call of gc_b200_conv kernel families', 'unit': 'us',
                      'n_gpus': 1, 'steps': args.steps, 'warmup': args.warmup, 'dtype': 'f32',
                      'data': 'synthetic uniform inputs on the device', 'peaks': pk,
                      'config': {'workload': 'kernels', 'families': args.families}, 'rows': rows}), flush=True)
    return 0


def run_nhwc(args):
    """Channels-last layers: gc_b200_conv_ex with layout NHWC against
    torch.nn.functional.conv2d on channels_last tensors (cuDNN, TF32 off,
    benchmark mode) - the reference's torch_tuned_channels_last variant
    (bench/cuda_boundaries.py:17) - and against this library's own NCHW path on
    the same layer.  Device time: K calls captured in one CUDA graph, replayed
    between CUDA events (host overheads of either API left out); 'api_us' is
    the same K calls issued from Python one by one."""
    import torch
    import torch.nn.functional as F
    from groupconv_atlas_b200 import api
    from groupconv_atlas_b200.api import Shape
    from oracle import oracle as orc
    rank, world, local = dist_setup()
    if rank != 0:
        return 0
    torch.cuda.set_device(local)
    set_fp32_precision(torch)
    torch.backends.cudnn.benchmark = True
    native = api.Native()
    stream = torch.cuda.Stream()
    rows = []
    for spec in args.shapes.split(';'):
        n, c, h, w, cpg = (int(v) for v in spec.split(','))
        s = Shape(n=n, cin=c, cout=c, h=h, w=w, groups=c // cpg)
        with torch.cuda.stream(stream), torch.inference_mode():
            g = torch.Generator(device='cuda').manual_seed(n * 7 + c)
            x = torch.rand(s.input, device='cuda', generator=g) * 2 - 1
            wt = (torch.rand(s.weight, device='cuda', generator=g) * 2 - 1) / math.sqrt(9 * cpg)
            xcl = x.contiguous(memory_format=torch.channels_last)
            wcl = wt.contiguous(memory_format=torch.channels_last)
            ycl = torch.empty(s.output, device='cuda').contiguous(memory_format=torch.channels_last)
            y = torch.empty(s.output, device='cuda')
            calls = {
                'ours_nhwc': lambda: native.conv_ex(s, xcl, wt, ycl, layout='nhwc',
                                                    stream=torch.cuda.current_stream().cuda_stream),
                'ours_nchw': lambda: native.cuda(s, x, wt, y, 3, torch.cuda.current_stream().cuda_stream),
                'cudnn_channels_last': lambda: F.conv2d(xcl, wcl, padding=1, groups=s.groups),
                'cudnn_nchw': lambda: F.conv2d(x, wt, padding=1, groups=s.groups),
            }
            row = {'shape': [n, c, h, w, cpg]}
            for name, call in calls.items():
                for _ in range(max(3, args.warmup)):
                    call()
                plan = native.last_plan() if name.startswith('ours') else None
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(args.steps):
                    call()
                b.record(stream)
                stream.synchronize()
                api_us = a.elapsed_time(b) / args.steps * 1e3
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    for _ in range(args.steps):
                        call()
                graph.replay()
                a.record(stream)
                graph.replay()
                b.record(stream)
                stream.synchronize()
                row[name] = {'us': a.elapsed_time(b) / args.steps * 1e3, 'api_us': api_us,
                             **({'plan': plan} if plan else {})}
                del graph
            # the NHWC result equals the NCHW production result within the FP32 acceptance gate
            m = orc.error_metrics(ycl.contiguous().cpu().numpy(), y.cpu().numpy())
            row['nhwc_matches_nchw'] = m['passed']
            row['speedup_vs_cudnn_channels_last'] = row['cudnn_channels_last']['us'] / row['ours_nhwc']['us']
            rows.append(row)
        del x, xcl, y, ycl
        torch.cuda.empty_cache()
    geo = math.exp(statistics.fmean(math.log(r['speedup_vs_cudnn_channels_last']) for r in rows))
    print(json.dumps({'metric': 'channels-last layers: speed-up of gc_b200_conv_ex (NHWC) over cuDNN channels_last',
                      'value': geo, 'unit': 'x', 'n_gpus': 1, 'steps': args.steps, 'dtype': 'f32',
                      'data': 'synthetic uniform inputs on the device', 'higher_is_better': True,
                      'config': {'workload': 'nhwc'}, 'all_match': all(r['nhwc_matches_nchw'] for r in rows),
                      'rows': rows}), flush=True)
    return 0 if all(r['nhwc_matches_nchw'] for r in rows) else 1


def main(argv=None):
    args = parse_args(argv)
    if args.cudnn_leg:
        return cudnn_leg(args.cudnn_leg)
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
    if args.workload == 'kernels':
        return run_kernels(args)
    if args.workload == 'nhwc':
        return run_nhwc(args)
    return run_ours(args)


if __name__ == '__main__':
    raise SystemExit(main())
