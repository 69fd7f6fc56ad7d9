"""Measures the B200's peak rates with the library's own probes (the roofline
denominators this repository reports against) and writes them, with the
clock record taken while they ran, to ``profiles/peaks.json``.

    python -m groupconv_atlas_b200.peaks [--out profiles/peaks.json] [--device 0]

Probes (``gc_b200_probe_*``, csrc/kernel_probe.cuh):
  ffma      FP32 FMA issue rate: 8 independent FMA chains per thread, 2048
            threads per SM (2 FLOP per FMA);
  tf32_mma  tensor-core TF32 rate: one CTA per SM issuing back-to-back
            tcgen05.mma.kind::tf32 of M = 128, N = 256, K = 8 (the MMA shape
            of the 3xTF32 path), and with two CTAs per SM as a check that one
            issuer saturates the tensor core;
  copy      HBM copy rate: 16-byte loads and stores over 1 GiB (read + write).

Each probe runs 3 untimed launches and then `--repeats` launches, each timed
by CUDA events on the launching stream; the best and the median rate are
kept.  Clocks are sampled through NVML (read only) during every timed run.
Derived ceilings:
  tf32x3_tflops  = tf32_mma / 3   (the usual 3xTF32 ceiling: three TF32
                   products per FP32 product);
  tf32x3_issued  = tf32_mma / 4   (the ceiling of this library's formulation:
                   [w_hi; w_lo] stacked along M times x_hi and x_lo, four
                   TF32 products per FP32 product).
"""
from __future__ import annotations

import argparse
import datetime
import json
import statistics
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _timed(torch, stream, launch, repeats):
    """(per-launch ms list) of `repeats` launches, each between two events."""
    for _ in range(3):
        launch()
    stream.synchronize()
    times = []
    for _ in range(repeats):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        launch()
        b.record(stream)
        b.synchronize()
        times.append(a.elapsed_time(b))
    return times


def measure(device=0, repeats=10):
    import torch
    from . import api
    from .clocks import ClockSampler
    native = api.Native()
    torch.cuda.set_device(device)
    props = torch.cuda.get_device_properties(device)
    sms = props.multi_processor_count
    stream = torch.cuda.Stream()
    results = {'gpu_name': props.name, 'sms': sms,
               'when': datetime.datetime.now(datetime.timezone.utc).strftime('%Y-%m-%dT%H:%M:%SZ'),
               'timing': f'3 untimed launches, then {repeats} launches each between CUDA events on the '
                         'launching stream; best and median', 'probes': {}}

    def record(name, work, unit, launch, what, scale):
        sampler = ClockSampler(device, period=0.002)
        with sampler, torch.cuda.stream(stream):
            times = _timed(torch, stream, launch, repeats)
        stat = native.device_status(clear=True)
        if stat:
            raise RuntimeError(f'{name} probe: device status word {stat:#x}')
        rates = [work / (t / 1e3) / scale for t in times]
        results['probes'][name] = {'best': max(rates), 'median': statistics.median(rates), 'unit': unit,
                                   'ms_median': statistics.median(times), 'work_per_launch': work,
                                   'what': what, 'clocks': sampler.summary()}

    out = torch.empty(sms * 8 * 256, device='cuda')
    ffma_blocks, ffma_iters = sms * 8, 16384
    with torch.cuda.stream(stream):
        flops = native.probe_ffma(out, ffma_blocks, ffma_iters, stream.cuda_stream)
    record('ffma', flops, 'TFLOP/s', lambda: native.probe_ffma(out, ffma_blocks, ffma_iters, stream.cuda_stream),
           f'{ffma_blocks} blocks x 256 threads, 8 FMA chains, {ffma_iters} x 16 FMAs per chain', 1e12)

    status = torch.zeros(2 * sms, dtype=torch.int32, device='cuda')
    mma_iters = 1 << 18
    for per_sm in (1, 2):
        blocks = per_sm * sms
        with torch.cuda.stream(stream):
            flops = native.probe_tf32_mma(status, blocks, mma_iters, stream.cuda_stream)
        record('tf32_mma' if per_sm == 1 else 'tf32_mma_2cta', flops, 'TFLOP/s',
               lambda b=blocks: native.probe_tf32_mma(status, b, mma_iters, stream.cuda_stream),
               f'{blocks} CTAs, one thread each issuing {mma_iters} tcgen05.mma.kind::tf32 M128 N256 K8', 1e12)
        torch.cuda.synchronize()
        if int(status[:blocks].sum().item()) != 0:
            raise RuntimeError('tf32 MMA probe: a bounded wait gave up')

    src = torch.empty(1 << 28, device='cuda')  # 1 GiB
    dst = torch.empty_like(src)
    src.fill_(1.0)
    copy_blocks = sms * 8
    with torch.cuda.stream(stream):
        nbytes = native.probe_copy(src, dst, copy_blocks, stream.cuda_stream)
    record('copy', nbytes, 'GB/s', lambda: native.probe_copy(src, dst, copy_blocks, stream.cuda_stream),
           f'1 GiB copied by {copy_blocks} blocks x 256 threads, 16-byte accesses (read + write bytes)', 1e9)
    del src, dst
    torch.cuda.synchronize()

    p = results['probes']
    results['ffma_tflops'] = p['ffma']['best']
    results['tf32_mma_tflops'] = p['tf32_mma']['best']
    results['tf32x3_tflops'] = p['tf32_mma']['best'] / 3
    results['tf32x3_issued_tflops'] = p['tf32_mma']['best'] / 4
    results['copy_gbs'] = p['copy']['best']
    mhz = p['ffma']['clocks'].get('sm_mhz')
    if mhz:
        results['ffma_flop_per_clk_per_sm'] = p['ffma']['best'] * 1e12 / (mhz * 1e6) / sms
    mhz = p['tf32_mma']['clocks'].get('sm_mhz')
    if mhz:
        results['tf32_flop_per_clk_per_sm'] = p['tf32_mma']['best'] * 1e12 / (mhz * 1e6) / sms
    return results


def markdown(results):
    rows = ['| probe | best | median | unit | SM MHz (median) | reasons | what |', '|---|---|---|---|---|---|---|']
    for name, r in results['probes'].items():
        c = r['clocks']
        rows.append(f"| {name} | {r['best']:.1f} | {r['median']:.1f} | {r['unit']} | {c.get('sm_mhz')} | "
                    f"{','.join(c.get('reasons', [])) or 'none'} | {r['what']} |")
    return '\n'.join(rows)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument('--out', default=str(ROOT / 'profiles' / 'peaks.json'))
    ap.add_argument('--device', type=int, default=0)
    ap.add_argument('--repeats', type=int, default=10)
    args = ap.parse_args(argv)
    results = measure(args.device, args.repeats)
    Path(args.out).write_text(json.dumps(results, indent=1) + '\n')
    print(markdown(results))
    print(json.dumps({k: v for k, v in results.items() if k != 'probes'}))
    return 0


if __name__ == '__main__':
    sys.exit(main())
