"""Helpers shared by the GPU tests: run the library on device tensors through
the C ABI and check the output against the oracle."""
from __future__ import annotations

import numpy as np

from oracle import oracle as orc


def run(native, torch, shape, x, w, impl=None, kernel=None, stream=None, sentinel=True):
    """Copy x, w to the device, fill y with NaN (so unwritten outputs fail),
    call gc_cuda_conv (impl) or gc_b200_conv (kernel) on a non-default
    stream, and return (y as numpy, launch plan)."""
    stream = stream or torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dx = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        dw = torch.from_numpy(np.ascontiguousarray(w)).cuda()
        dy = torch.full(shape.output, float('nan') if sentinel else 0.0, device='cuda')
        if kernel is None:
            native.cuda(shape, dx, dw, dy, 3 if impl is None else impl, stream.cuda_stream)
        else:
            native.b200(shape, dx, dw, dy, kernel, stream.cuda_stream)
        plan = native.last_plan()
        stream.synchronize()
        return dy.cpu().numpy(), plan


# Reduction length up to which the reference's fixed 1e-4 tolerances (its
# FP32-against-FP32 gate and its FP64 spot check) are meaningful: they are
# sized for the reference's shapes (at most 64 channels per group, 576 terms
# per output).  Longer sums (wide groups, dense layers) legitimately move an
# FP32 result near a cancelling output by more than 1e-4, so there the
# per-element bound |y - y64| <= 1e-5 sum|x*w| against FP64 decides alone.
REFERENCE_GATES_MAX_TERMS = 576


def assert_matches(shape, x, w, y, y32=None, label='', points=True):
    """The acceptance checks: |y - y64| <= 1e-5 sum|x*w| for every element,
    and - for reductions of at most 576 terms - the reference's 1e-4/1e-4
    gate against its FP32 output and its 64-point FP64 spot check."""
    y64, bound = orc.conv_f64_bound(shape, x, w)
    res = orc.bound_check(y, y64, bound)
    assert res['passed'], f'{label}: bound check {res}'
    if shape.cpg * shape.r * shape.s > REFERENCE_GATES_MAX_TERMS:
        return res
    ref32 = y32 if y32 is not None else orc.conv_f32_blocked(shape, x, w)
    m = orc.error_metrics(y, ref32)
    assert m['passed'], f'{label}: fp32 gate {m}'
    if points:
        p = orc.check_points(shape, x, w, y)
        assert p['passed'], f'{label}: fp64 points {p["failed_points"]}'
    return res
