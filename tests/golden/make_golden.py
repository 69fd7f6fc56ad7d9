"""Generate the golden fixtures that pin the oracle to the reference.

Run in a checkout where the reference tree is available (it is read, never
copied):

    make -C oracle ref REF=<reference checkout>   # compile the reference CPU library
    GC_REFERENCE_TREE=<reference checkout> python tests/golden/make_golden.py

It writes, next to this script:

  golden_cases.npz  per case: geometry, the inputs produced by the reference's
                    own seeding (bench/api.py:156-158), the reference
                    library's FP32 serial output (csrc/cpu GC_SERIAL) and its
                    FP64 oracle output on the same inputs widened to FP64.
  golden_meta.json  Shape ids (bench/api.py:43-45) and the reference's 64-point
                    FP64 selections (bench/fp64_points.py:38-75) for a set of
                    shapes, plus the provenance of every case.

Cases: the reference's boundary suite (bench/check.py:65-78, every shape), its
four special input patterns (check.py:210-227), the native CUDA runner's
B-geometry matrix subset and general-geometry sweep (tests/native_cuda.cu:
233-250), and small B-geometry shapes for cpg 8/16/32.
"""
from __future__ import annotations

import os
import argparse
import ctypes as ct
import dataclasses
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument('--reference', default=os.environ.get('GC_REFERENCE_TREE'),
                        help='the reference checkout (default: $GC_REFERENCE_TREE)')
    args = parser.parse_args()
    if not args.reference:
        raise SystemExit('name the reference checkout: --reference PATH or GC_REFERENCE_TREE')
    sys.path.insert(0, args.reference)
    sys.path.insert(0, str(REPO))
    from bench.api import Shape, inputs  # the reference's own Python
    from bench.check import boundary_shapes
    from bench.fp64_points import select_points
    from oracle import oracle as orc

    if not orc.reference_available():
        raise SystemExit('build the reference library first: make -C oracle ref')

    cases = []  # (name, shape, x, w)

    def add(name, shape, x, w):
        cases.append((name, shape, np.ascontiguousarray(x, np.float32), np.ascontiguousarray(w, np.float32)))

    seed = 20260908
    for i, s in enumerate(boundary_shapes()):
        x, w = inputs(s, seed)
        add(f'boundary{i:02d}', s, x, w)
    special = boundary_shapes()[4]
    for pattern in ('zeros', 'impulse', 'group_isolation', 'cancellation'):
        x, w = inputs(special, seed)
        if pattern == 'zeros':
            x.fill(0)
        elif pattern == 'impulse':
            x.fill(0)
            x[0, 0, 0, special.w // 2] = 1
            w.fill(1)
        elif pattern == 'group_isolation':
            x.fill(0)
            x[:, :special.cin // special.groups] = 1
            w.fill(1)
        else:
            x.fill(1)
            w.reshape(-1)[::2] = 1
            w.reshape(-1)[1::2] = -1
        add(f'pattern_{pattern}', special, x, w)
    # B geometry, two groups, the native runner's spatial set (native_cuda.cu:233-243).
    for cpg in (1, 2, 3, 4, 8):
        for h, w_ in ((1, 1), (1, 19), (11, 1), (7, 13), (9, 17), (17, 33), (8, 16)):
            s = Shape(n=2 if (h * w_) % 2 else 1, cin=2 * cpg, cout=2 * cpg, h=h, w=w_, groups=2)
            x, w = inputs(s, 17)
            add(f'b_cpg{cpg}_{h}x{w_}', s, x, w)
    for cpg in (16, 32):
        s = Shape(n=1, cin=2 * cpg, cout=2 * cpg, h=12, w=20, groups=2)
        x, w = inputs(s, 101)
        add(f'b_cpg{cpg}_12x20', s, x, w)
    # General geometry sweep (native_cuda.cu:244-250).
    for k in (3, 5, 7):
        for st in (1, 2):
            for d in (1, 2):
                for pad in (0, 3):
                    s = Shape(n=1, cin=4, cout=6, h=17, w=23, r=k, s=k, groups=2, sh=st, sw=st, ph=pad,
                              pw=pad, dh=d, dw=d)
                    x, w = inputs(s, seed)
                    add(f'general_r{k}_s{st}_d{d}_p{pad}', s, x, w)
    s = Shape(n=1, cin=4, cout=6, h=17, w=23, r=3, s=5, groups=2, sh=2, sw=1, ph=1, pw=3, dh=1, dw=2)
    add('general_asymmetric', s, *inputs(s, seed))
    s = Shape(n=4, cin=3, cout=6, h=7, w=13, groups=3)
    add('general_depthwise_multiplier2', s, *inputs(s, seed))

    arrays, meta = {}, {'cases': [], 'shape_ids': {}, 'points': {}}
    for name, s, x, w in cases:
        y32 = orc.reference_conv(s, x, w, impl=0, threads=1)
        y64 = orc.reference_conv(s, x.astype(np.float64), w.astype(np.float64), impl=0, threads=1)
        arrays[f'{name}__x'] = x
        arrays[f'{name}__w'] = w
        arrays[f'{name}__y32'] = y32
        arrays[f'{name}__y64'] = y64
        meta['cases'].append({'name': name, 'shape': dataclasses.asdict(s),
                              'y32': 'reference gc_cpu_conv GC_SERIAL FP32',
                              'y64': 'reference gc_cpu_conv GC_SERIAL FP64 oracle'})
    for s in [Shape(), Shape(n=32, cin=256, cout=256, h=56, w=56, groups=256),
              Shape(n=1, cin=32, cout=32, h=56, w=56, groups=8),
              Shape(n=1024, cin=256, cout=256, h=56, w=56, groups=32),
              Shape(n=4, cin=144, cout=144, h=56, w=56, groups=144)] + boundary_shapes()[:6]:
        meta['shape_ids'][json.dumps(dataclasses.asdict(s), sort_keys=True)] = s.id
        meta['points'][s.id] = [list(p) for p in select_points(s, 64, seed)]
    np.savez_compressed(HERE / 'golden_cases.npz', **arrays)
    (HERE / 'golden_meta.json').write_text(json.dumps(meta, indent=1, sort_keys=True) + '\n')
    print(f'{len(cases)} cases -> {HERE / "golden_cases.npz"}')


if __name__ == '__main__':
    main()
