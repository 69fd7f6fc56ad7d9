"""The checker: CPU oracle for grouped 2-D cross-correlation.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, ``__graft_entry__.smoke()`` and
the cpu_baseline / reference legs of ``bench.py``; never by the product
package.  It wraps

  * ``liboracle.so``  - ``gc_oracle.c``, the C restatement of the reference's
    CPU convolution (csrc/cpu/cpu_internal.h:7-22, openmp.cpp:5-43,
    reference.cpp:5-26), built by ``make -C oracle``;
  * ``_ref/libgroupconv_ref.so`` - the reference's own CPU library compiled
    from its sources by ``make -C oracle ref`` (present where the reference
    tree was available at build time);

and restates in Python the reference's acceptance checks:
``error_metrics`` (bench/api.py:167-176), ``oracle_points``
(bench/api.py:178-192) and the 64-point FP64 selection/evaluation of
bench/fp64_points.py:38-119.  The B200 acceptance bound is
``|y - y_fp64| <= 1e-5 * sum|x*w|`` per output element.
"""
from __future__ import annotations

import ctypes as ct
import math
import operator
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBORACLE = HERE / 'liboracle.so'
LIBREF = HERE / '_ref' / 'libgroupconv_ref.so'
FIELDS = ('n', 'cin', 'cout', 'h', 'w', 'r', 's', 'groups', 'sh', 'sw', 'ph', 'pw', 'dh', 'dw')
BOUND_FACTOR = 1e-5
ATOL = RTOL = 1e-4


class _Shape(ct.Structure):
    _fields_ = [(f, ct.c_int64) for f in FIELDS]


def _cs(shape):
    return _Shape(*[int(getattr(shape, f)) for f in FIELDS])


def output_dims(shape):
    ho = (shape.h + 2 * shape.ph - shape.dh * (shape.r - 1) - 1) // shape.sh + 1
    wo = (shape.w + 2 * shape.pw - shape.dw * (shape.s - 1) - 1) // shape.sw + 1
    return (shape.n, shape.cout, ho, wo)


def build_oracle():
    """Compile liboracle.so from gc_oracle.c when it is missing or stale."""
    src = HERE / 'gc_oracle.c'
    if LIBORACLE.exists() and LIBORACLE.stat().st_mtime >= src.stat().st_mtime:
        return LIBORACLE
    subprocess.run(['make', '-s', '-C', str(HERE), 'all'], check=True)
    return LIBORACLE


_lib = None


def lib():
    global _lib
    if _lib is None:
        build_oracle()
        l = ct.CDLL(str(LIBORACLE))
        fp, dp, sp = ct.POINTER(ct.c_float), ct.POINTER(ct.c_double), ct.POINTER(_Shape)
        l.gco_conv_f32_serial.argtypes = [sp, fp, fp, fp]
        l.gco_conv_f32_blocked.argtypes = [sp, fp, fp, fp, ct.c_int]
        l.gco_conv_f64.argtypes = [sp, dp, dp, dp]
        l.gco_conv_f64_bound.argtypes = [sp, fp, fp, dp, dp, ct.c_int]
        for f in ('gco_conv_f32_serial', 'gco_conv_f32_blocked', 'gco_conv_f64', 'gco_conv_f64_bound'):
            getattr(l, f).restype = None
        _lib = l
    return _lib


def _ptr(a, ctype):
    assert a.flags['C_CONTIGUOUS']
    return a.ctypes.data_as(ct.POINTER(ctype))


def _threads(threads):
    return int(threads or os.cpu_count() or 1)


def conv_f32_serial(shape, x, w):
    """FP32, one reduction per output in the reference's order (bit-exact to it)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    y = np.empty(output_dims(shape), np.float32)
    lib().gco_conv_f32_serial(ct.byref(_cs(shape)), _ptr(x, ct.c_float), _ptr(w, ct.c_float), _ptr(y, ct.c_float))
    return y


def conv_f32_blocked(shape, x, w, threads=None):
    """FP32 c2 'blocked' OpenMP schedule; same per-output order as serial."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    y = np.empty(output_dims(shape), np.float32)
    lib().gco_conv_f32_blocked(ct.byref(_cs(shape)), _ptr(x, ct.c_float), _ptr(w, ct.c_float),
                               _ptr(y, ct.c_float), _threads(threads))
    return y


def conv_f64(shape, x, w):
    """FP64 oracle on FP64 inputs (reference csrc/cpu/reference.cpp:5-19)."""
    x = np.ascontiguousarray(x, np.float64)
    w = np.ascontiguousarray(w, np.float64)
    y = np.empty(output_dims(shape), np.float64)
    lib().gco_conv_f64(ct.byref(_cs(shape)), _ptr(x, ct.c_double), _ptr(w, ct.c_double), _ptr(y, ct.c_double))
    return y


def conv_f64_bound(shape, x, w, threads=None):
    """(FP64 result of FP32 inputs, per-output sum |x*w|)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    y = np.empty(output_dims(shape), np.float64)
    b = np.empty(output_dims(shape), np.float64)
    lib().gco_conv_f64_bound(ct.byref(_cs(shape)), _ptr(x, ct.c_float), _ptr(w, ct.c_float),
                             _ptr(y, ct.c_double), _ptr(b, ct.c_double), _threads(threads))
    return y, b


def bound_check(actual, expected64, abs_sum, factor=BOUND_FACTOR):
    """North-star acceptance: |y - y64| <= factor * sum|x*w| for every element
    (finite required).  Returns a JSON-safe summary."""
    a = np.asarray(actual, np.float64)
    err = np.abs(a - expected64)
    finite = np.isfinite(a)
    limit = factor * abs_sum
    bad = (~finite) | (err > limit)
    ratio = np.where(limit > 0, err / np.where(limit > 0, limit, 1.0), np.where(err > 0, np.inf, 0.0))
    return {'passed': bool(not bad.any()), 'failed_elements': int(bad.sum()), 'elements': int(a.size),
            'max_abs': float(err[finite].max()) if finite.any() else None,
            'max_ratio_to_bound': float(ratio[finite].max()) if finite.any() else None,
            'factor': factor}


def error_metrics(actual, reference, atol=ATOL, rtol=RTOL, eps=1e-12):
    """Elementwise atol+rtol gate with finite values required (reference bench/api.py:167-176)."""
    a = np.asarray(actual, dtype=np.float64)
    b = np.asarray(reference, dtype=np.float64)
    if a.shape != b.shape:
        raise ValueError('reference shape mismatch')
    finite = np.isfinite(a) & np.isfinite(b)
    diff = np.abs(a - b)
    bad = (diff > atol + rtol * np.abs(b)) | ~finite
    return {'passed': bool(not bad.any()), 'max_abs': float(np.max(diff)) if finite.all() else None,
            'max_rel': float(np.max(diff / (np.abs(b) + eps))) if finite.all() else None,
            'rms': float(np.sqrt(np.mean(diff * diff))) if finite.all() else None,
            'failed_elements': int(bad.sum()), 'elements': int(a.size), 'epsilon': eps,
            'atol': atol, 'rtol': rtol}


def oracle_points(shape, x, w, positions):
    """Scalar FP64 value at each (n, co, oh, ow) (reference bench/api.py:178-192)."""
    values = []
    opg, cpg = shape.cout // shape.groups, shape.cin // shape.groups
    for n, co, oh, ow in positions:
        acc = 0.0
        base = (co // opg) * cpg
        for ci in range(cpg):
            for r in range(shape.r):
                ih = oh * shape.sh - shape.ph + r * shape.dh
                for s in range(shape.s):
                    iw = ow * shape.sw - shape.pw + s * shape.dw
                    if 0 <= ih < shape.h and 0 <= iw < shape.w:
                        acc += float(x[n, base + ci, ih, iw]) * float(w[co, ci, r, s])
        values.append(acc)
    return np.array(values, dtype=np.float64)


def select_points(shape, count=64, seed=20260908):
    """Deterministic unique output points: batch/channel endpoints x corners and
    centre, group boundaries, then a seeded fill (reference fp64_points.py:38-75)."""
    count = operator.index(count)
    if count <= 0:
        raise ValueError('count must be positive')
    dims = output_dims(shape)
    total = math.prod(dims)
    target = min(count, total)
    points, seen = [], set()

    def add(point):
        if len(points) < target and point not in seen:
            seen.add(point)
            points.append(point)

    n, c, h, w = dims
    for batch in dict.fromkeys((0, n - 1)):
        for channel in dict.fromkeys((0, c - 1)):
            for row, col in ((0, 0), (h - 1, w - 1), (0, w - 1), (h - 1, 0), (h // 2, w // 2)):
                add((batch, channel, row, col))
    opg = c // shape.groups
    for group in range(shape.groups):
        for channel in dict.fromkeys((group * opg, (group + 1) * opg - 1)):
            add((group % n, channel, h // 2, w // 2))
        if len(points) == target:
            break
    rng = np.random.default_rng(seed)
    while len(points) < target and target < total // 2:
        add(tuple(int(rng.integers(d)) for d in dims))
    if len(points) < target:
        for point in np.ndindex(dims):
            add(point)
            if len(points) == target:
                break
    return points


def check_points(shape, x, w, actual, count=64, seed=20260908, atol=ATOL, rtol=RTOL):
    """64-point FP64 spot check of an output (reference fp64_points.py:78-119)."""
    points = select_points(shape, count, seed)
    expected = oracle_points(shape, x, w, points)
    got = np.array([float(actual[p]) for p in points])
    finite = np.isfinite(got) & np.isfinite(expected)
    err = np.abs(got - expected)
    ok = finite & (err <= atol + rtol * np.abs(expected))
    return {'passed': bool(ok.all()), 'failed_points': int((~ok).sum()), 'point_count': len(points),
            'max_abs': float(err[finite].max()) if finite.any() else None, 'points': points}


# ---- the reference's own CPU library, compiled from its sources -----------------------------

class _RefTensor(ct.Structure):
    _fields_ = [('data', ct.c_void_p), ('bytes', ct.c_uint64), ('dtype', ct.c_int32),
                ('device', ct.c_int32), ('device_index', ct.c_int32), ('rank', ct.c_int32),
                ('dims', ct.c_int64 * 4), ('strides', ct.c_int64 * 4)]


def _ref_desc(a):
    dtype = {np.dtype('float32'): 0, np.dtype('float64'): 1}[a.dtype]
    strides = tuple(s // a.itemsize for s in a.strides)
    return _RefTensor(a.ctypes.data, a.nbytes, dtype, 0, 0, 4, (ct.c_int64 * 4)(*a.shape),
                      (ct.c_int64 * 4)(*strides))


_ref = None


def reference_available():
    return LIBREF.exists()


def reference_lib():
    """The reference's CPU library (GC_SERIAL=0, GC_OPENMP=1, GC_BLOCKED=2)."""
    global _ref
    if _ref is None:
        if not LIBREF.exists():
            raise FileNotFoundError(f'{LIBREF} is not built (make -C oracle ref)')
        l = ct.CDLL(str(LIBREF))
        l.gc_cpu_conv.argtypes = [ct.POINTER(_Shape)] + [ct.POINTER(_RefTensor)] * 3 + [ct.c_int, ct.c_int]
        l.gc_last_error.restype = ct.c_char_p
        _ref = l
    return _ref


def reference_conv(shape, x, w, impl=2, threads=None, out=None):
    """Run the reference's gc_cpu_conv; raises on a non-zero status."""
    y = out if out is not None else np.empty(output_dims(shape), x.dtype)
    status = reference_lib().gc_cpu_conv(ct.byref(_cs(shape)), ct.byref(_ref_desc(x)), ct.byref(_ref_desc(w)),
                                         ct.byref(_ref_desc(y)), int(impl), _threads(threads))
    if status:
        raise RuntimeError(f'reference gc_cpu_conv status {status}: {reference_lib().gc_last_error().decode()}')
    return y
