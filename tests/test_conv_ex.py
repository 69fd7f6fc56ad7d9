"""gc_b200_conv_ex: a per-output-channel bias (the four ConvNeXt 7x7
depthwise layers the reference reports as unsupported, bench/model_run.py:
46-49, and any other geometry) and channels-last (NHWC) tensors (which the
reference times only through cuDNN, bench/cuda_boundaries.py:17).
Acceptance with a bias: |y - (y_fp64 + b)| <= 1e-5 * (sum|x*w| + |b|) per
element, plus the reference's 1e-4 gate against torch's conv2d with bias.
NHWC results are compared in NCHW order against the same oracle."""
import ctypes as ct

import numpy as np
import pytest

from groupconv_atlas_b200 import api, workloads
from groupconv_atlas_b200.api import GC_INVALID, GC_UNSUPPORTED, NativeError, Shape, inputs
from oracle import oracle as orc


def _desc(shape4, strides, dtype=0, device=1, index=0, data=1 << 20):
    n = int(np.prod(shape4))
    return api.Tensor(data, 4 * n, dtype, device, index, len(shape4), (ct.c_int64 * 4)(*shape4),
                      (ct.c_int64 * 4)(*strides))


def _dense(dims):
    n, c, h, w = dims
    return (c * h * w, h * w, w, 1)


def _cl(dims):
    n, c, h, w = dims
    return (h * w * c, 1, w * c, c)


def _call(native, s, x, w, b, y, layout, act=0):
    return native.lib.gc_b200_conv_ex(ct.byref(api.cshape(s)), ct.byref(x), ct.byref(w),
                                      ct.byref(b) if b is not None else None, ct.byref(y), layout, act, None)


def test_validation_without_a_device(native):
    """Descriptor errors are reported before any device work (no GPU needed):
    a malformed bias is GC_INVALID, a non-dense bias GC_UNSUPPORTED; NHWC
    with NCHW strides is GC_UNSUPPORTED after every GC_INVALID check; an
    unknown layout is GC_UNSUPPORTED."""
    s = Shape(n=2, cin=8, cout=8, h=5, w=6, groups=4)
    x = _desc(s.input, _cl(s.input), data=1 << 20)
    w = _desc(s.weight, _dense(s.weight), data=1 << 24)
    y = _desc(s.output, _cl(s.output), data=1 << 28)
    good_b = api.Tensor(1 << 30, 32, 0, 1, 0, 1, (ct.c_int64 * 4)(8), (ct.c_int64 * 4)(1))
    for dims, stride, nbytes, dtype in (((7,), (1,), 32, 0), ((8,), (1,), 16, 0), ((8,), (1,), 32, 1)):
        bad = api.Tensor(1 << 30, nbytes, dtype, 1, 0, 1, (ct.c_int64 * 4)(*dims), (ct.c_int64 * 4)(*stride))
        assert _call(native, s, x, w, bad, y, 1) == GC_INVALID, native.lib.gc_last_error()
    strided = api.Tensor(1 << 30, 64, 0, 1, 0, 1, (ct.c_int64 * 4)(8), (ct.c_int64 * 4)(2))
    assert _call(native, s, x, w, strided, y, 1) == GC_UNSUPPORTED
    xn = _desc(s.input, _dense(s.input), data=1 << 20)
    assert _call(native, s, xn, w, good_b, y, 1) == GC_UNSUPPORTED  # NCHW strides under the NHWC layout
    assert b'channels-last' in native.lib.gc_last_error()
    assert _call(native, s, x, w, good_b, y, 7) == GC_UNSUPPORTED
    assert _call(native, s, x, w, good_b, y, 1, act=5) == GC_UNSUPPORTED
    short = _desc(s.input, _cl(s.input))
    short.bytes = 8
    assert _call(native, s, short, w, None, y, 1) == GC_INVALID  # too small, before the layout check


def _bias_bound_check(s, x, w, b, y):
    y64, bound = orc.conv_f64_bound(s, x, w)
    bb = np.broadcast_to(np.asarray(b, np.float64)[None, :, None, None], y64.shape)
    res = orc.bound_check(y, y64 + bb, bound + np.abs(bb))
    assert res['passed'], res
    return res


@pytest.mark.gpu
@pytest.mark.parametrize('index', range(4))
def test_convnext_biased_layers(native, torch_cuda, index):
    torch = torch_cuda
    layer = [l for l in workloads.model_layers() if l.bias][index]
    s = layer.shape
    x, w = inputs(s)
    b = np.random.default_rng(index).uniform(-1, 1, s.cout).astype(np.float32)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dx, dw, db = (torch.from_numpy(a).cuda() for a in (x, w, b))
        dy = torch.full(s.output, float('nan'), device='cuda')
        native.conv_ex(s, dx, dw, dy, bias=db, stream=stream.cuda_stream)
        plan = native.last_plan()
        ref = torch.nn.functional.conv2d(dx, dw, db, padding=(s.ph, s.pw), groups=s.groups)
        stream.synchronize()
    assert plan.startswith('kernel=general engine=depthwise'), plan
    y = dy.cpu().numpy()
    _bias_bound_check(s, x, w, b, y)
    assert orc.error_metrics(y, ref.cpu().numpy())['passed']


BIAS_SHAPES = [
    dict(n=2, cin=32, cout=32, h=20, w=24, groups=32),                  # 3x3 s1 depthwise (cell kernel)
    dict(n=2, cin=16, cout=16, h=17, w=19, groups=16, sh=2, sw=2),      # 3x3 s2 depthwise
    dict(n=1, cin=8, cout=8, h=15, w=13, r=5, s=5, groups=8, ph=2, pw=2, dh=2, dw=2),  # dilated 5x5
    dict(n=2, cin=32, cout=32, h=14, w=14, groups=4),                   # grouped B geometry (general kernel)
    dict(n=1, cin=16, cout=32, h=9, w=11, groups=4, sh=2, sw=2),        # Cin != Cout
]


@pytest.mark.gpu
@pytest.mark.parametrize('geo', BIAS_SHAPES, ids=lambda g: '-'.join(f'{k}{v}' for k, v in g.items()))
def test_bias_any_geometry(native, torch_cuda, geo):
    torch = torch_cuda
    s = Shape(**geo)
    x, w = inputs(s, 3)
    b = np.linspace(-2, 2, s.cout).astype(np.float32)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dx, dw, db = (torch.from_numpy(a).cuda() for a in (x, w, b))
        dy = torch.full(s.output, float('nan'), device='cuda')
        native.conv_ex(s, dx, dw, dy, bias=db, stream=stream.cuda_stream)
        stream.synchronize()
    _bias_bound_check(s, x, w, b, dy.cpu().numpy())


@pytest.mark.gpu
def test_nchw_without_bias_is_the_production_path(native, torch_cuda):
    torch = torch_cuda
    s = Shape(n=3, cin=64, cout=64, h=28, w=28, groups=16)
    x, w = inputs(s, 5)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dx, dw = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
        a = torch.empty(s.output, device='cuda')
        b = torch.empty(s.output, device='cuda')
        native.conv_ex(s, dx, dw, a, stream=stream.cuda_stream)
        native.cuda(s, dx, dw, b, 3, stream.cuda_stream)
        stream.synchronize()
    assert torch.equal(a, b)


NHWC_SHAPES = [
    # (geometry, bias): the vector kernels (3x3 s1 p1, C % 4 == 0; one group per warp for groups
    # of 2, 4 and 8) at each group width, and the scalar kernel for other geometries and
    # channel counts
    (dict(n=4, cin=144, cout=144, h=56, w=56, groups=144), False),
    (dict(n=2, cin=64, cout=64, h=13, w=15, groups=32), True),
    (dict(n=2, cin=64, cout=64, h=14, w=17, groups=16), False),
    (dict(n=2, cin=128, cout=128, h=9, w=10, groups=16), True),
    (dict(n=1, cin=64, cout=64, h=12, w=12, groups=4), False),
    (dict(n=1, cin=48, cout=48, h=7, w=9, groups=1), True),
    (dict(n=3, cin=96, cout=96, h=17, w=30, groups=12), False),              # groups of 8, ragged quads
    (dict(n=2, cin=32, cout=32, h=5, w=6, groups=8), False),                 # groups of 4, 2 pixels past the row
    (dict(n=1, cin=24, cout=24, h=8, w=9, groups=12), False),                # groups of 2, 9 pixel columns
    (dict(n=2, cin=256, cout=256, h=7, w=7, groups=64), True),               # groups of 4, item tail
    (dict(n=8, cin=256, cout=256, h=56, w=54, groups=256), False),           # depthwise, strips of 2 rows
    (dict(n=4, cin=960, cout=960, h=7, w=7, groups=960), True),              # depthwise, weights per item
    (dict(n=16, cin=128, cout=128, h=63, w=64, groups=64), True),            # groups of 2, ragged last strip
    (dict(n=2, cin=6, cout=6, h=9, w=9, groups=2), True),                    # C % 4 != 0
    (dict(n=2, cin=96, cout=96, h=23, w=21, groups=96, sh=2, sw=2), False),  # strided depthwise
    (dict(n=1, cin=16, cout=32, h=11, w=10, r=5, s=5, groups=4, ph=2, pw=2), True),
    # groups of more than 16 channels: the tensor-core path reading and writing channels-last
    (dict(n=2, cin=64, cout=64, h=13, w=15, groups=2), False),     # 32 channels per group
    (dict(n=1, cin=256, cout=256, h=12, w=14, groups=1), False),   # dense: output-channel blocks, split K
    (dict(n=3, cin=128, cout=128, h=7, w=7, groups=2), False),     # 64 per group, images stacked in a strip
    (dict(n=2, cin=96, cout=96, h=11, w=13, groups=2), False),     # 48 per group
    (dict(n=4, cin=256, cout=256, h=28, w=28, groups=4), False),   # two strips per item
    (dict(n=2, cin=64, cout=64, h=9, w=10, groups=2), True),       # bias: the FFMA kernel
]


@pytest.mark.gpu
@pytest.mark.parametrize('geo,with_bias', NHWC_SHAPES, ids=lambda v: str(v) if isinstance(v, bool) else
                         '-'.join(f'{k}{x}' for k, x in v.items()))
def test_nhwc(native, torch_cuda, geo, with_bias):
    torch = torch_cuda
    s = Shape(**geo)
    x, w = inputs(s, 6)
    b = np.linspace(-1, 1, s.cout).astype(np.float32) if with_bias else None
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dx = torch.from_numpy(x).cuda().contiguous(memory_format=torch.channels_last)
        dw = torch.from_numpy(w).cuda()
        db = torch.from_numpy(b).cuda() if with_bias else None
        dy = torch.full(s.output, float('nan'), device='cuda').contiguous(memory_format=torch.channels_last)
        native.conv_ex(s, dx, dw, dy, bias=db, layout='nhwc', stream=stream.cuda_stream)
        plan = native.last_plan()
        stream.synchronize()
    tensor = s.b_geometry and s.cpg >= 16 and s.cpg % 8 == 0 and not with_bias
    if tensor:
        assert plan.startswith('kernel=tf32x3') and 'layout=nhwc' in plan, plan
    else:
        assert plan.startswith('kernel=nhwc'), plan
        vector = s.b_geometry and s.cin % 4 == 0 and (s.cpg in (1, 2) or s.cpg % 4 == 0)
        engine = {1: 'dw_tma', 2: 'dw_tma', 4: 'grp_tma', 8: 'grp_tma'}.get(s.cpg, 'vector4x4')
        assert (f'engine={engine}' in plan) == vector, plan
    y = dy.contiguous().cpu().numpy()  # back to NCHW order
    if with_bias:
        _bias_bound_check(s, x, w, b, y)
    else:
        y64, bound = orc.conv_f64_bound(s, x, w)
        assert orc.bound_check(y, y64, bound)['passed']


@pytest.mark.gpu
def test_nhwc_unaligned_takes_the_scalar_kernel(native, torch_cuda):
    torch = torch_cuda
    s = Shape(n=1, cin=16, cout=16, h=6, w=7, groups=4)
    x, w = inputs(s, 8)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        buf = torch.empty(int(np.prod(s.input)) + 1, device='cuda')
        xcl = torch.from_numpy(x).cuda().contiguous(memory_format=torch.channels_last)
        buf[1:].copy_(xcl.permute(0, 2, 3, 1).reshape(-1))
        dx = buf[1:].view(1, 6, 7, 16).permute(0, 3, 1, 2)  # channels-last strides, 4-byte offset
        dw = torch.from_numpy(w).cuda()
        dy = torch.full(s.output, float('nan'), device='cuda').contiguous(memory_format=torch.channels_last)
        native.conv_ex(s, dx, dw, dy, layout='nhwc', stream=stream.cuda_stream)
        plan = native.last_plan()
        stream.synchronize()
    assert 'engine=scalar' in plan, plan
    y64, bound = orc.conv_f64_bound(s, x, w)
    assert orc.bound_check(dy.contiguous().cpu().numpy(), y64, bound)['passed']


@pytest.mark.gpu
@pytest.mark.parametrize('groups', [32, 16, 8, 4])
def test_nhwc_unaligned_weights_take_the_strip_kernel(native, torch_cuda, groups):
    """Groups of 1, 2, 4 and 8 channels whose weights are not 16-byte aligned
    cannot use the TMA-staged kernels (they load weights as 16-byte vectors):
    the strip kernel serves them."""
    torch = torch_cuda
    s = Shape(n=2, cin=32, cout=32, h=10, w=12, groups=groups)
    x, w = inputs(s, 9)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dx = torch.from_numpy(x).cuda().contiguous(memory_format=torch.channels_last)
        buf = torch.empty(int(np.prod(s.weight)) + 1, device='cuda')
        buf[1:].copy_(torch.from_numpy(w).cuda().reshape(-1))
        dw = buf[1:].view(s.weight)  # dense, 4-byte offset
        dy = torch.full(s.output, float('nan'), device='cuda').contiguous(memory_format=torch.channels_last)
        native.conv_ex(s, dx, dw, dy, layout='nhwc', stream=stream.cuda_stream)
        plan = native.last_plan()
        stream.synchronize()
    assert 'engine=strip' in plan, plan
    y64, bound = orc.conv_f64_bound(s, x, w)
    assert orc.bound_check(dy.contiguous().cpu().numpy(), y64, bound)['passed']


EPI_SHAPES = [
    # B geometry on the direct engines (depthwise TMA kernel, grouped warp-specialized kernel,
    # cp.async staging for an odd width), the register-cell depthwise kernel, the general kernel
    dict(n=4, cin=144, cout=144, h=56, w=56, groups=144),
    dict(n=2, cin=64, cout=64, h=28, w=28, groups=16),
    dict(n=2, cin=32, cout=32, h=13, w=15, groups=8),
    dict(n=2, cin=16, cout=16, h=14, w=14, groups=16),
    dict(n=1, cin=64, cout=64, h=10, w=12, groups=2),
    dict(n=1, cin=96, cout=96, h=23, w=21, groups=96, sh=2, sw=2),
]


@pytest.mark.gpu
@pytest.mark.parametrize('act', ['relu', 'relu6'])
@pytest.mark.parametrize('geo', EPI_SHAPES, ids=lambda g: '-'.join(f'{k}{v}' for k, v in g.items()))
def test_bias_and_activation_epilogue(native, torch_cuda, geo, act):
    """act(conv + b) against the FP64 oracle with the same bias and clamp
    (the clamp can only shrink the error), on whichever kernel serves it."""
    torch = torch_cuda
    s = Shape(**geo)
    x, w = inputs(s, 12)
    x = x * 4.0  # outputs spread beyond 6 so that ReLU6 clamps both ends
    b = np.linspace(-1.5, 1.5, s.cout).astype(np.float32)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dx, dw, db = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (x, w, b))
        dy = torch.full(s.output, float('nan'), device='cuda')
        native.conv_ex(s, dx, dw, dy, bias=db, activation=act, stream=stream.cuda_stream)
        plan = native.last_plan()
        stream.synchronize()
    y64, bound = orc.conv_f64_bound(s, x, w)
    bb = np.broadcast_to(b.astype(np.float64)[None, :, None, None], y64.shape)
    hi = 6.0 if act == 'relu6' else np.inf
    expected = np.clip(y64 + bb, 0.0, hi)
    y = dy.cpu().numpy()
    res = orc.bound_check(y, expected, bound + np.abs(bb))
    assert res['passed'], (plan, res)
    assert (y >= 0).all() and (y <= hi).all()
    if act == 'relu6':
        assert (y == 6.0).any() and (y == 0.0).any()


NHWC_EPI_SHAPES = [
    # channels-last kernels carrying the epilogue: TMA-tiled (groups of 1, 2, 4), strip
    # (groups of 8), vector (groups of 12), scalar (strided depthwise)
    dict(n=4, cin=144, cout=144, h=56, w=56, groups=144),
    dict(n=2, cin=64, cout=64, h=28, w=28, groups=32),
    dict(n=2, cin=64, cout=64, h=28, w=28, groups=16),
    dict(n=2, cin=64, cout=64, h=13, w=16, groups=8),
    dict(n=1, cin=48, cout=48, h=9, w=10, groups=4),
    dict(n=1, cin=96, cout=96, h=23, w=21, groups=96, sh=2, sw=2),
]


@pytest.mark.gpu
@pytest.mark.parametrize('act', ['relu', 'relu6'])
@pytest.mark.parametrize('geo', NHWC_EPI_SHAPES, ids=lambda g: '-'.join(f'{k}{v}' for k, v in g.items()))
def test_nhwc_bias_and_activation_epilogue(native, torch_cuda, geo, act):
    """Channels-last act(conv + b) against the FP64 oracle, on whichever kernel serves it."""
    torch = torch_cuda
    s = Shape(**geo)
    x, w = inputs(s, 14)
    x = x * 4.0
    b = np.linspace(-1.5, 1.5, s.cout).astype(np.float32)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dx = torch.from_numpy(x).cuda().contiguous(memory_format=torch.channels_last)
        dw, db = torch.from_numpy(w).cuda(), torch.from_numpy(b).cuda()
        dy = torch.full(s.output, float('nan'), device='cuda').contiguous(memory_format=torch.channels_last)
        native.conv_ex(s, dx, dw, dy, bias=db, layout='nhwc', activation=act, stream=stream.cuda_stream)
        plan = native.last_plan()
        stream.synchronize()
    assert plan.startswith('kernel=nhwc'), plan
    y64, bound = orc.conv_f64_bound(s, x, w)
    bb = np.broadcast_to(b.astype(np.float64)[None, :, None, None], y64.shape)
    hi = 6.0 if act == 'relu6' else np.inf
    expected = np.clip(y64 + bb, 0.0, hi)
    y = dy.contiguous().cpu().numpy()
    res = orc.bound_check(y, expected, bound + np.abs(bb))
    assert res['passed'], (plan, res)
    assert (y >= 0).all() and (y <= hi).all()
    if act == 'relu6':
        assert (y == 6.0).any() and (y == 0.0).any()


@pytest.mark.gpu
def test_activation_without_bias_on_the_production_kernel(native, torch_cuda):
    torch = torch_cuda
    s = Shape(n=2, cin=64, cout=64, h=28, w=28, groups=8)
    x, w = inputs(s, 13)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dx, dw = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
        plain = torch.empty(s.output, device='cuda')
        relu = torch.empty(s.output, device='cuda')
        native.cuda(s, dx, dw, plain, 3, stream.cuda_stream)
        production = native.last_plan().split()[0]
        native.conv_ex(s, dx, dw, relu, activation='relu', stream=stream.cuda_stream)
        plan = native.last_plan()
        stream.synchronize()
    assert plan.split()[0] == production, (plan, production)
    assert torch.equal(relu, torch.clamp_min(plain, 0.0))


def test_autotune_validation_without_a_device(native):
    """gc_b200_autotune validates like gc_cuda_conv, then its own argument."""
    s = Shape(n=2, cin=8, cout=8, h=5, w=6, groups=4)
    x = _desc(s.input, _dense(s.input), data=1 << 20)
    w = _desc(s.weight, _dense(s.weight), data=1 << 24)
    y = _desc(s.output, _dense(s.output), data=1 << 28)
    call = lambda cand, yy=y: native.lib.gc_b200_autotune(ct.byref(api.cshape(s)), ct.byref(x), ct.byref(w),
                                                          ct.byref(yy), cand, None)
    assert call(0) == GC_INVALID and b'candidates' in native.lib.gc_last_error()
    assert call(65) == GC_INVALID
    bad = _desc(s.output, _dense(s.output), dtype=1, data=1 << 28)
    assert call(8, bad) == GC_INVALID
