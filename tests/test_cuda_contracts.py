"""GPU contract tests of gc_cuda_conv, after the reference's native CUDA runner
(tests/native_cuda.cu: --contracts :167-197, --graph :122-154, --stress
:223-229) and bench/check.py's status mapping.  No test here faults, traps or
hangs the GPU: invalid pointers are rejected on the host before any launch,
and the bounded-wait self-test waits on a barrier nothing completes for a
few milliseconds, then returns."""
import ctypes as ct

import numpy as np
import pytest

from groupconv_atlas_b200 import api
from groupconv_atlas_b200.api import (Shape, NativeError, cshape, tensor, inputs, GC_OK, GC_INVALID,
                                      GC_UNSUPPORTED, GC_DEVICE_ERROR)
from oracle import oracle as orc
from tests.gpu_helpers import run, assert_matches

pytestmark = pytest.mark.gpu


def bshape(n, h, w, cpg, groups=2):
    return Shape(n=n, cin=cpg * groups, cout=cpg * groups, h=h, w=w, groups=groups)


def device_tensors(torch, s, seed=3):
    x, w = inputs(s, seed)
    dx, dw = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    dy = torch.full(s.output, float('nan'), device='cuda')
    return x, w, dx, dw, dy


def call(native, s, xd, wd, yd, impl=0, stream=0):
    p = cshape(s)
    return native.lib.gc_cuda_conv(ct.byref(p), ct.byref(xd), ct.byref(wd), ct.byref(yd), impl, stream)


def test_pointer_and_descriptor_contracts(native, torch_cuda):
    torch = torch_cuda
    s = bshape(1, 7, 13, 2)
    x, w, dx, dw, dy = device_tensors(torch, s)
    xd, wd, yd = tensor(dx), tensor(dw), tensor(dy)
    # host pointers in CUDA descriptors (reference native_cuda.cu:182-188)
    pinned = torch.from_numpy(x).pin_memory()
    bad = tensor(pinned); bad.device, bad.device_index = 1, 0
    assert call(native, s, bad, wd, yd) == GC_INVALID
    pageable = np.ascontiguousarray(x)
    bad = tensor(pageable); bad.device, bad.device_index = 1, 0
    assert call(native, s, bad, wd, yd) in (GC_INVALID, GC_DEVICE_ERROR)
    # descriptor device index differs from the pointer's device (:176-178)
    for t in (xd, wd, yd):
        t.device_index += 1
    assert call(native, s, xd, wd, yd) == GC_INVALID
    for t in (xd, wd, yd):
        t.device_index -= 1
    # rejected calls left no work behind: the sentinel output is untouched
    torch.cuda.synchronize()
    assert torch.isnan(dy).all()
    # a valid call still works afterwards (no sticky error)
    assert call(native, s, xd, wd, yd, 3) == GC_OK
    torch.cuda.synchronize()
    assert_matches(s, x, w, dy.cpu().numpy())
    assert native.device_status(clear=True) == 0


def test_misaligned_and_offset_pointers(native, torch_cuda):
    """Element-aligned but not 16-byte-aligned sub-tensors are valid: the
    engine falls back to cp.async staging and scalar stores, never faults."""
    torch = torch_cuda
    s = bshape(2, 9, 16, 4)
    x, w = inputs(s, 9)
    big_x = torch.zeros(x.size + 3, device='cuda')
    big_y = torch.full((int(np.prod(s.output)) + 3,), float('nan'), device='cuda')
    big_x[1:1 + x.size] = torch.from_numpy(x.reshape(-1)).cuda()
    dx = big_x[1:1 + x.size].view(s.input)
    dy = big_y[1:1 + int(np.prod(s.output))].view(s.output)
    dw = torch.from_numpy(w).cuda()
    for impl in (0, 1, 2, 3):
        native.cuda(s, dx, dw, dy, impl, 0)
        torch.cuda.synchronize()
        assert_matches(s, x, w, dy.cpu().numpy(), label=f'offset impl{impl} {native.last_plan()}')
    assert torch.isnan(big_y[0]) and torch.isnan(big_y[-2:]).all()


def test_nondefault_stream(native, torch_cuda):
    """reference tests/test_correctness.py:46-64 with implementation 2."""
    torch = torch_cuda
    s = Shape(cin=4, cout=4, groups=2, h=9, w=17)
    x, w = inputs(s)
    y, plan = run(native, torch, s, x, w, impl=2)
    pos = [(n, c, i, j) for n in range(s.n) for c in range(s.cout) for i in range(s.output[2]) for j in range(s.output[3])]
    assert orc.error_metrics(np.array([y[p] for p in pos]), orc.oracle_points(s, x, w, pos))['passed']


@pytest.mark.parametrize('impl,shape', [(0, bshape(1, 7, 13, 2)), (1, bshape(1, 7, 13, 2)), (2, bshape(1, 7, 13, 2)),
                                        (3, bshape(1, 7, 13, 2)), (3, bshape(2, 14, 16, 1)),
                                        (3, bshape(1, 12, 16, 16))])
def test_graph_capture(native, torch_cuda, impl, shape):
    """The ABI call captured into a CUDA graph and replayed gives the eager
    result (reference native_cuda.cu:122-154)."""
    torch = torch_cuda
    x, w, dx, dw, dy = device_tensors(torch, shape, 73)
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        native.cuda(shape, dx, dw, dy, impl, stream.cuda_stream)
    graph.replay()
    torch.cuda.synchronize()
    assert_matches(shape, x, w, dy.cpu().numpy(), label=f'graph impl{impl}')
    dy.fill_(float('nan'))
    graph.replay()
    torch.cuda.synchronize()
    assert not torch.isnan(dy).any()


@pytest.mark.parametrize('cpg', [1, 2, 4])
def test_stress_many_tiles(native, torch_cuda, cpg):
    """More than 65,535 work items, so every persistent CTA reuses its shared
    memory stages many times (reference native_cuda.cu:223-229)."""
    torch = torch_cuda
    s = bshape(65535 // (cpg * 4) + 1, 1, 17, cpg)
    x = (np.arange(np.prod(s.input)) // (s.h * s.w) % 7 - 3).astype(np.float32).reshape(s.input) * 0.25
    w = ((np.arange(np.prod(s.weight)) % 5) - 2).astype(np.float32).reshape(s.weight) * 0.125
    for impl in (1, 2, 3):
        y, plan = run(native, torch, s, x, w, impl=impl)
        y64, bound = orc.conv_f64_bound(s, x, w)
        res = orc.bound_check(y, y64, bound)
        assert res['passed'], (impl, plan, res)


def test_patterns_zero_impulse_isolation_cancellation(native, torch_cuda):
    """reference native_cuda.cu:74-93 patterns, every implementation."""
    torch = torch_cuda
    for cpg in (1, 2, 4, 3, 8, 16):
        s = bshape(1, 7, 13, cpg)
        x, w = inputs(s, 1)
        pats = {}
        pats['zero'] = (np.zeros_like(x), w)
        xi = np.zeros_like(x); xi[0, 0, s.h // 2, s.w // 2] = 1
        pats['impulse'] = (xi, w)
        pats['isolation'] = (xi, np.ones_like(w))
        xc = np.where(np.arange(x.size) % 2, -1.0, 1.0).astype(np.float32).reshape(x.shape)
        pats['cancellation'] = (xc, np.full_like(w, 0.125))
        for name, (xx, ww) in pats.items():
            for impl in (0, 1, 3):
                y, plan = run(native, torch, s, xx, ww, impl=impl)
                assert_matches(s, xx, ww, y, label=f'{name} cpg{cpg} impl{impl} {plan}')
                if name in ('impulse', 'isolation'):
                    assert np.all(y[:, cpg:] == 0), 'group leak'


def test_bounded_wait_selftest(native, torch_cuda):
    """A wait nothing completes gives up after its limit, records the
    timeout in the status word and returns; the context stays usable."""
    torch = torch_cuda
    assert native.device_status(clear=True) == 0
    native.selftest_wait_timeout(2000)  # 2 ms
    assert native.device_status(clear=True) & api.STATUS_TMA_TIMEOUT
    assert native.device_status(clear=True) == 0
    s = bshape(1, 8, 16, 2)
    x, w = inputs(s, 4)
    y, _ = run(native, torch, s, x, w, impl=3)
    assert_matches(s, x, w, y)


def test_unsupported_requests_launch_nothing(native, torch_cuda):
    torch = torch_cuda
    s = Shape(cin=4, cout=4, groups=2, h=9, w=11, sh=2, sw=2, ph=0, pw=0)
    x, w, dx, dw, dy = device_tensors(torch, s)
    for impl in (1, 2, 3, 4, -1):
        with pytest.raises(NativeError) as err:
            native.cuda(s, dx, dw, dy, impl, 0)
        assert err.value.status == GC_UNSUPPORTED
    torch.cuda.synchronize()
    assert torch.isnan(dy).all()
