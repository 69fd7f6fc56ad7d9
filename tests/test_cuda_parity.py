"""GPU parity: every kernel family, through the C ABI, against the oracle on
the same seeded inputs.  Acceptance per output element:
|y - y_fp64| <= 1e-5 * sum|x*w| (FP64 oracle), plus the reference's own gates
(1e-4 atol/rtol vs its FP32 output, 64 FP64 points)."""
import re

import numpy as np
import pytest

from groupconv_atlas_b200.api import Shape, NativeError, inputs, GC_UNSUPPORTED
from groupconv_atlas_b200 import workloads
from oracle import oracle as orc
from tests.gpu_helpers import run, assert_matches

pytestmark = pytest.mark.gpu


def expected_support(shape, impl):
    """The reference's support matrix (bench/check.py:106-112)."""
    if impl == 0:
        return True
    return shape.b_geometry and (impl != 2 or shape.cpg in (1, 2, 4))


def test_golden_all_implementations(native, torch_cuda, golden_cases):
    """Reference boundary suite, special patterns, native-runner matrix and the
    general-geometry sweep, through gc_cuda_conv implementations 0-3."""
    for c in golden_cases:
        for impl in range(4):
            if not expected_support(c.shape, impl):
                with pytest.raises(NativeError) as err:
                    run(native, torch_cuda, c.shape, c.x, c.w, impl=impl)
                assert err.value.status == GC_UNSUPPORTED, (c.name, impl)
                continue
            y, plan = run(native, torch_cuda, c.shape, c.x, c.w, impl=impl)
            assert_matches(c.shape, c.x, c.w, y, c.y32, label=f'{c.name} impl{impl} [{plan}]')


def tf32_co(cpg):
    """Output channels per tensor-path item: the widest multiple of 8 up to 64
    dividing the group; 0: not served."""
    return next((co for co in range(64, 7, -8) if cpg % co == 0), 0)


def tf32_fits(cpg, w):
    """A 256-pixel strip plus its 2 * (W + 2) + 2 halo rows must fit the
    converters' 1024 rows and the shared memory: weights staged twice, A tiles
    of 64 or 128 rows twice, four pixel tiles, the epilogue buffers and the
    barriers."""
    co = tf32_co(cpg)
    rows_b = -(-(256 + 2 * (w + 2) + 2) // 8) * 8
    smem = 2 * co * 288 + 2 * 9 * (128 if 2 * co > 64 else 64) * 32 + 4 * rows_b * 32 + 8 * 16 * 33 * 4 + 128
    return rows_b <= 1024 and smem <= 227 * 1024


def tf32_eligible(s):
    return s.b_geometry and tf32_co(s.cpg) > 0 and tf32_fits(s.cpg, s.w)


TF32_WIDEST_CPG16 = max(w for w in range(1, 1024) if tf32_fits(16, w))


@pytest.mark.parametrize('kernel', ['general', 'direct_ldg', 'direct_tma', 'tf32x3', 'small'])
def test_golden_kernel_families(native, torch_cuda, golden_cases, kernel):
    """Each kernel family on every golden case it serves; the others must be
    refused with GC_UNSUPPORTED, never silently rerouted."""
    ran = 0
    for c in golden_cases:
        eligible = kernel == 'general' or c.shape.b_geometry
        if kernel == 'direct_tma':
            eligible = eligible and c.shape.w % 4 == 0
        if kernel == 'tf32x3':
            eligible = tf32_eligible(c.shape)
        if kernel == 'small':
            eligible = c.shape.b_geometry and c.shape.h * c.shape.w <= 512
        if not eligible:
            with pytest.raises(NativeError) as err:
                run(native, torch_cuda, c.shape, c.x, c.w, kernel=kernel)
            assert err.value.status == GC_UNSUPPORTED
            continue
        y, plan = run(native, torch_cuda, c.shape, c.x, c.w, kernel=kernel)
        assert plan.startswith(f'kernel={kernel}'), plan
        assert_matches(c.shape, c.x, c.w, y, c.y32, label=f'{c.name} {kernel}')
        ran += 1
    assert ran > 0


SMALL_B = [
    # (n, c, h, w, cpg): tails in both axes, multi-band items, wide cpg
    (1, 8, 56, 56, 1), (3, 12, 30, 44, 2), (2, 16, 57, 60, 4), (2, 32, 23, 40, 8),
    (1, 48, 19, 28, 16), (1, 64, 14, 16, 32), (1, 128, 9, 12, 64), (2, 6, 33, 17, 3),
    (1, 10, 70, 72, 5), (1, 24, 112, 112, 1), (1, 16, 112, 112, 4), (1, 8, 7, 7, 8),
    (5, 4, 14, 14, 2), (1, 2, 200, 248, 1), (1, 4, 5, 252, 2),
    # 16-channel groups on the warp-specialized direct kernel: tails, several groups per item
    (2, 64, 30, 56, 16), (1, 32, 9, 12, 16), (3, 128, 17, 28, 16), (1, 16, 112, 112, 16),
]


@pytest.mark.parametrize('n,c,h,w,cpg', SMALL_B)
@pytest.mark.parametrize('kernel', ['direct_ldg', 'direct_tma', 'small', 'auto'])
def test_b_geometry_shapes(native, torch_cuda, n, c, h, w, cpg, kernel):
    s = Shape(n=n, cin=c, cout=c, h=h, w=w, groups=c // cpg)
    x, wt = inputs(s, 7)
    if kernel == 'direct_tma' and w % 4:
        pytest.skip('TMA staging needs width % 4 == 0')
    if kernel == 'direct_tma' and w + 8 > 256:
        pytest.skip('TMA box is at most 256 columns')
    if kernel == 'small' and h * w > 512:
        pytest.skip('small-image kernel serves at most 512 pixels per plane')
    y, plan = run(native, torch_cuda, s, x, wt, kernel=kernel)
    assert_matches(s, x, wt, y, label=f'{s} {plan}')


def test_config1_full(native, torch_cuda):
    """Config 1 (N1 C32 56x56, 8 groups of 4 channels), full output, all implementations."""
    wl = workloads.config1()
    for impl in (0, 1, 2, 3):
        y, plan = run(native, torch_cuda, wl.shape, wl.x, wl.w, impl=impl)
        assert_matches(wl.shape, wl.x, wl.w, y, label=f'config1 impl{impl} {plan}')


def test_config4_leaf_full(native, torch_cuda):
    """MobileNetV2 depthwise leaf of config 4 (N4 C144 56x56), full output."""
    s = Shape(n=4, cin=144, cout=144, h=56, w=56, groups=144)
    x, w = inputs(s, 2)
    y, plan = run(native, torch_cuda, s, x, w, impl=3)
    assert_matches(s, x, w, y, label=f'config4 leaf {plan}')


@pytest.mark.parametrize('name', ['config2', 'config5_g32', 'config5_g4'])
def test_config_batch_slices(native, torch_cuda, name):
    """Configs 2 and 5 at their channel/spatial sizes on a 2-image batch slice
    (full outputs checked against the FP64 oracle)."""
    wl = workloads.by_name(name, batch=2)
    y, plan = run(native, torch_cuda, wl.shape, wl.x, wl.w, impl=3)
    assert_matches(wl.shape, wl.x, wl.w, y, label=f'{name} slice {plan}')


def test_sweep_config3(native, torch_cuda):
    """All 80 shapes of the config-3 sweep.  Shapes whose oracle finishes
    quickly are checked in full; the others on a one-image slice of the same
    channels and spatial size plus 64 FP64 points of the full batch."""
    shapes = workloads.sweep_shapes()
    assert len(shapes) == 80
    for s in shapes:
        work = s.n * s.cout * s.h * s.w * s.cpg * 9
        check = s if work <= 3e8 else Shape(**{**s.__dict__, 'n': 1})
        x, w = workloads.sweep_inputs(check)
        y, plan = run(native, torch_cuda, check, x, w, impl=3)
        assert_matches(check, x, w, y, label=f'sweep {s} {plan}', points=check is s)
        if check is not s:
            x, w = workloads.sweep_inputs(s)
            y, _ = run(native, torch_cuda, s, x, w, impl=3)
            p = orc.check_points(s, x, w, y)
            assert p['passed'], f'sweep points {s}'


TF32_SHAPES = [
    # (n, c, h, w, cpg): one/many strips, partial last strip, tails, N > 1
    (1, 16, 8, 16, 8), (2, 32, 12, 20, 16), (1, 64, 9, 12, 32), (1, 128, 9, 12, 64),
    (3, 64, 30, 28, 32), (2, 128, 56, 56, 64), (1, 256, 14, 16, 8), (4, 96, 7, 8, 16),
    (1, 64, 112, 112, 16), (2, 64, 33, 44, 64),
    # widths that are not a multiple of 4, tiny planes
    (3, 128, 7, 7, 64), (2, 64, 14, 14, 32), (1, 32, 13, 11, 16), (4, 16, 9, 5, 8), (1, 64, 30, 30, 64),
    # widest row that fits, several strips per row
    (1, 16, 6, TF32_WIDEST_CPG16, 16), (2, 8, 3, 300, 8),
    # images stacked into one strip: batch not a multiple of the block, 1x1 planes
    (5, 64, 5, 6, 32), (7, 32, 3, 3, 16), (3, 64, 1, 1, 64), (9, 128, 10, 9, 64),
    # many groups: every CTA crosses group boundaries
    (3, 512, 9, 10, 16), (2, 512, 12, 12, 32), (1, 256, 20, 30, 8),
    # 24/40/48/56-channel groups; wide groups and dense layers in output-channel blocks
    (2, 96, 11, 13, 48), (2, 48, 10, 9, 24), (1, 80, 12, 11, 40), (1, 112, 9, 8, 56),
    (2, 256, 9, 10, 128), (1, 256, 12, 14, 256), (2, 192, 8, 9, 96), (1, 160, 7, 9, 80), (1, 144, 8, 8, 72),
    # two 256-pixel strips per item: 32- and 48-channel groups of large planes
    (2, 64, 112, 112, 32), (3, 96, 64, 100, 48),
]


def test_tf32x3_refuses_unserved_group_width(native, torch_cuda):
    s = Shape(n=1, cin=40, cout=40, h=6, w=7, groups=2)  # 20 channels per group
    x, wt = inputs(s, 5)
    with pytest.raises(NativeError) as err:
        run(native, torch_cuda, s, x, wt, kernel='tf32x3')
    assert err.value.status == GC_UNSUPPORTED


def test_tf32x3_refuses_rows_beyond_reach(native, torch_cuda):
    s = Shape(n=1, cin=16, cout=16, h=4, w=TF32_WIDEST_CPG16 + 1, groups=1)
    x, wt = inputs(s, 5)
    with pytest.raises(NativeError) as err:
        run(native, torch_cuda, s, x, wt, kernel='tf32x3')
    assert err.value.status == GC_UNSUPPORTED


@pytest.mark.parametrize('n,c,h,w,cpg', [(2, 64, 112, 112, 32), (3, 96, 64, 100, 48)])
def test_tf32x3_two_strips_per_item(native, torch_cuda, n, c, h, w, cpg):
    """Groups of 32 and 48 channels on large planes take two strips per item."""
    s = Shape(n=n, cin=c, cout=c, h=h, w=w, groups=c // cpg)
    x, wt = inputs(s, 5)
    y, plan = run(native, torch_cuda, s, x, wt, kernel='tf32x3')
    assert ' sp=2 ' in plan, plan
    assert_matches(s, x, wt, y, label=f'{s} {plan}')


@pytest.mark.parametrize('n,c,h,w,cpg', TF32_SHAPES)
def test_tf32x3_tensor_core_path(native, torch_cuda, n, c, h, w, cpg):
    """The tcgen05 3xTF32 implicit GEMM meets the FP32 acceptance bound."""
    s = Shape(n=n, cin=c, cout=c, h=h, w=w, groups=c // cpg)
    x, wt = inputs(s, 5)
    y, plan = run(native, torch_cuda, s, x, wt, kernel='tf32x3')
    assert plan.startswith('kernel=tf32x3'), plan
    res = assert_matches(s, x, wt, y, label=f'{s} {plan}')
    assert res['max_ratio_to_bound'] < 0.5, res
    assert native.device_status(clear=True) == 0


# Layers with too few output tiles to fill the GPU: the input channels are
# split over several CTAs whose partial sums add into the zeroed output.
SPLIT_SHAPES = [(1, 256, 7, 7, 256), (1, 256, 14, 14, 256), (1, 64, 7, 7, 64), (1, 128, 12, 13, 128),
                (2, 32, 6, 9, 32), (32, 256, 7, 7, 256)]


@pytest.mark.parametrize('n,c,h,w,cpg', SPLIT_SHAPES)
@pytest.mark.parametrize('entry', ['impl3', 'tf32x3'])
def test_tf32x3_input_channel_split(native, torch_cuda, n, c, h, w, cpg, entry):
    s = Shape(n=n, cin=c, cout=c, h=h, w=w, groups=c // cpg)
    x, wt = inputs(s, 5)
    for _ in range(2):  # the output is zeroed by every call, not only the first
        if entry == 'impl3':
            y, plan = run(native, torch_cuda, s, x, wt, impl=3, sentinel=True)
        else:
            y, plan = run(native, torch_cuda, s, x, wt, kernel='tf32x3', sentinel=True)
        assert plan.startswith('kernel=tf32x3'), plan
        assert int(re.search(r'\bks=(\d+)', plan).group(1)) > 1, plan
        res = assert_matches(s, x, wt, y, label=f'{s} {plan}')
        assert res['max_ratio_to_bound'] < 0.5, res
    assert native.device_status(clear=True) == 0


# Depthwise layers outside B geometry: the depthwise engine behind
# implementation 0 (strided, dilated, 5x5 and 7x7 kernels, padding wider than
# the kernel, wide rows whose stage limits the band height).
DW_SHAPES = [
    dict(n=1, cin=96, cout=96, h=112, w=112, groups=96, sh=2, sw=2),  # MobileNetV2 features.2 geometry
    dict(n=2, cin=32, cout=32, h=57, w=61, groups=32, sh=2, sw=2),
    dict(n=1, cin=24, cout=24, h=33, w=35, r=5, s=5, groups=24, ph=2, pw=2),
    dict(n=2, cin=16, cout=16, h=28, w=28, r=7, s=7, groups=16, ph=3, pw=3),  # ConvNeXt geometry, no bias
    dict(n=1, cin=16, cout=16, h=30, w=29, groups=16, dh=2, dw=2, ph=2, pw=2),
    dict(n=1, cin=8, cout=8, h=31, w=40, groups=8, sh=3, sw=2, ph=0, pw=1),
    dict(n=1, cin=4, cout=4, h=6, w=7, groups=4, ph=3, pw=4),
    dict(n=1, cin=8, cout=8, h=300, w=20, r=5, s=5, groups=8, ph=2, pw=2),
    dict(n=1, cin=2, cout=2, h=10, w=2000, groups=2, sh=2, sw=2),
    dict(n=3, cin=5, cout=5, h=9, w=9, r=7, s=7, groups=5, sh=2, sw=2, ph=1, pw=1, dh=1, dw=1),
    # 3x3 stride 2 (the register-blocked stride-2 engine): aligned rows, odd widths, tiny planes
    dict(n=3, cin=8, cout=8, h=20, w=24, groups=8, sh=2, sw=2),
    dict(n=1, cin=4, cout=4, h=1, w=1, groups=4, sh=2, sw=2),
    dict(n=2, cin=3, cout=3, h=2, w=3, groups=3, sh=2, sw=2),
    dict(n=1, cin=6, cout=6, h=15, w=28, groups=6, sh=2, sw=2),
    # 5x5 stride 2 padding 2 (EfficientNet / MobileNetV3 downsampling geometry)
    dict(n=2, cin=16, cout=16, h=28, w=28, r=5, s=5, groups=16, sh=2, sw=2, ph=2, pw=2),
    dict(n=1, cin=8, cout=8, h=19, w=36, r=5, s=5, groups=8, sh=2, sw=2, ph=2, pw=2),
    dict(n=1, cin=4, cout=4, h=3, w=5, r=5, s=5, groups=4, sh=2, sw=2, ph=2, pw=2),
]


@pytest.mark.parametrize('geo', DW_SHAPES, ids=lambda g: '-'.join(f'{k}{v}' for k, v in g.items()))
@pytest.mark.parametrize('entry', ['impl0', 'general'])
def test_depthwise_engine(native, torch_cuda, geo, entry):
    s = Shape(**geo)
    x, w = inputs(s)
    if entry == 'impl0':
        y, plan = run(native, torch_cuda, s, x, w, impl=0)
    else:
        y, plan = run(native, torch_cuda, s, x, w, kernel='general')
    assert plan.startswith('kernel=general engine=depthwise'), plan
    assert_matches(s, x, w, y, label=str(geo))


def test_depthwise_engine_leaves_other_kernel_sizes_to_the_general_kernel(native, torch_cuda):
    s = Shape(n=1, cin=4, cout=4, h=12, w=12, r=9, s=9, groups=4, ph=4, pw=4)
    x, w = inputs(s)
    y, plan = run(native, torch_cuda, s, x, w, impl=0)
    assert plan.startswith('kernel=general grid='), plan
    assert_matches(s, x, w, y, label='9x9 depthwise')


AUTOTUNE_SHAPES = [(4, 64, 56, 56, 1), (8, 64, 28, 28, 2), (16, 128, 56, 56, 4), (8, 256, 56, 56, 8),
                   (4, 64, 28, 28, 16), (2, 32, 30, 44, 4)]


@pytest.mark.parametrize('n,c,h,w,cpg', AUTOTUNE_SHAPES)
def test_autotune_keeps_results_and_caches_a_plan(native, torch_cuda, n, c, h, w, cpg):
    """Benchmark mode times candidate tilings and caches the fastest; every
    candidate sums each output over ci then the 9 taps in order, so the result
    before, during and after tuning is the same bit for bit."""
    torch = torch_cuda
    s = Shape(n=n, cin=c, cout=c, h=h, w=w, groups=c // cpg)
    x, wt = inputs(s, 21)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dx, dw = torch.from_numpy(x).cuda(), torch.from_numpy(wt).cuda()
        before = torch.full(s.output, float('nan'), device='cuda')
        tuned = torch.full(s.output, float('nan'), device='cuda')
        after = torch.full(s.output, float('nan'), device='cuda')
        native.cuda(s, dx, dw, before, 3, stream.cuda_stream)
        native.autotune(s, dx, dw, tuned, stream=stream.cuda_stream)
        native.cuda(s, dx, dw, after, 3, stream.cuda_stream)
        plan = native.last_plan()
        stream.synchronize()
    assert torch.equal(before, tuned) and torch.equal(before, after), plan
    assert_matches(s, x, wt, after.cpu().numpy(), label=f'{s} {plan}')


def test_autotune_refuses_inside_a_capture(native, torch_cuda):
    torch = torch_cuda
    s = Shape(n=2, cin=32, cout=32, h=28, w=28, groups=8)
    x, wt = inputs(s, 22)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dx, dw = torch.from_numpy(x).cuda(), torch.from_numpy(wt).cuda()
        dy = torch.empty(s.output, device='cuda')
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with pytest.raises(NativeError) as err:
        with torch.cuda.graph(graph, stream=stream):
            native.autotune(s, dx, dw, dy, stream=stream.cuda_stream)
    assert err.value.status == GC_UNSUPPORTED
