"""GPU parity at the workloads' real sizes, through the C ABI:

  * the large-batch layer N1024 C256 56x56 (32 groups of 8 channels, and 4
    groups of 64 on the tensor-core path) in ONE call over the whole batch:
    images 0, 511 and 1023 checked in full against the FP64 oracle (image
    1023 starts 3.2 GB into the tensors, so every element offset past 2^31
    is exercised) plus 64 FP64 points over the whole batch;
  * the multi-GPU split run on one GPU: every unit of shard.units_for_rank
    for 8 ranks, each as its own call at pointer offsets into the full
    tensors (batch ranges, and group blocks when N < ranks), against the
    oracle and against the one-call result;
  * the reference's 80-shape Atlas grid and its 8 no-bias model layers at
    their real batch sizes: a one-image slice checked in full (for the
    heaviest dense layers the first rows of that image) plus 64 FP64 points
    of the full batch.
"""
import dataclasses
import math

import numpy as np
import pytest

from groupconv_atlas_b200 import shard, workloads
from groupconv_atlas_b200.api import Shape, inputs
from oracle import oracle as orc
from tests.gpu_helpers import assert_matches, run

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def config5_inputs():
    """The N1024 batch of the large-batch layer (seed 3, U[-1,1); the same
    images for the 32-group and the 4-group variant)."""
    wl = workloads.config5(32, with_x=False)
    return workloads.images(wl.shape, wl.seed, wl.dist)


def _device_run(native, torch, shape, dx, dw, impl=3, sentinel=True):
    dy = torch.full(shape.output, float('nan') if sentinel else 0.0, device='cuda')
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())  # the inputs' copies and the NaN fill come first
    with torch.cuda.stream(stream):
        native.cuda(shape, dx, dw, dy, impl, stream.cuda_stream)
        plan = native.last_plan()
    stream.synchronize()
    return dy, plan


@pytest.mark.parametrize('groups', [32, 4])
def test_config5_full_batch_one_call(native, torch_cuda, config5_inputs, groups):
    torch = torch_cuda
    wl = workloads.config5(groups, with_x=False)
    s = wl.shape
    dx = torch.from_numpy(config5_inputs).cuda()
    dw = torch.from_numpy(wl.w).cuda()
    dy, plan = _device_run(native, torch, s, dx, dw)
    assert native.device_status(clear=True) == 0
    assert not torch.isnan(dy).any().item(), f'unwritten outputs [{plan}]'
    one = dataclasses.replace(s, n=1)
    for img in (0, 511, 1023):
        y = dy[img:img + 1].cpu().numpy()
        assert_matches(one, config5_inputs[img:img + 1], wl.w, y, label=f'config5 g{groups} image {img} [{plan}]')
    p = orc.check_points(s, config5_inputs, wl.w, dy)
    assert p['passed'], f'config5 g{groups} whole-batch points: {p["failed_points"]} [{plan}]'
    del dx, dy
    torch.cuda.empty_cache()


@pytest.mark.parametrize('groups', [32, 4])
def test_config5_units_of_eight_ranks_on_one_gpu(native, torch_cuda, config5_inputs, groups):
    """Every rank's units of an 8-GPU split, run one after another on this GPU
    at pointer offsets into the full tensors, reproduce the one-call result
    (same kernels, same per-element summation order)."""
    torch = torch_cuda
    wl = workloads.config5(groups, with_x=False)
    s = wl.shape
    dx = torch.from_numpy(config5_inputs).cuda()
    dw = torch.from_numpy(wl.w).cuda()
    whole, plan = _device_run(native, torch, s, dx, dw)
    dy = torch.full(s.output, float('nan'), device='cuda')
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    firsts = []
    with torch.cuda.stream(stream):
        for rank in range(8):
            for u in shard.units_for_rank(s, 8, rank):
                sub = u.shape(s)
                ox, ow, oy = u.offsets(s)
                xv = dx.view(-1)[ox:ox + math.prod(sub.input)].view(sub.input)
                wv = dw.view(-1)[ow:ow + math.prod(sub.weight)].view(sub.weight)
                yv = dy.view(-1)[oy:oy + math.prod(sub.output)].view(sub.output)
                native.cuda(sub, xv, wv, yv, 3, stream.cuda_stream)
                firsts.append(u.n0)
    stream.synchronize()
    assert native.device_status(clear=True) == 0
    assert firsts == [128 * r for r in range(8)]
    assert not torch.isnan(dy).any().item()
    one = dataclasses.replace(s, n=1)
    for img in (127, 128, 895, 896):  # both sides of unit boundaries, offsets past 2^31 bytes
        assert_matches(one, config5_inputs[img:img + 1], wl.w, dy[img:img + 1].cpu().numpy(),
                       label=f'config5 g{groups} units image {img}')
    diff = (dy - whole).abs().max().item()
    assert diff == 0.0, f'units differ from the one-call result by {diff} [{plan}]'
    del dx, dy, whole
    torch.cuda.empty_cache()


@pytest.mark.parametrize('n,groups,world', [(3, 32, 8), (1, 32, 8), (2, 4, 8), (5, 32, 8)])
def test_group_block_units_on_one_gpu(native, torch_cuda, n, groups, world):
    """Fewer images than ranks: each image is split into blocks of whole
    groups (x[n, c0:c1], w[c0:c1], y[n, c0:c1] contiguous), one call each."""
    torch = torch_cuda
    s = Shape(n=n, cin=256, cout=256, h=56, w=56, groups=groups)
    x, w = inputs(s, 3)
    dx, dw = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    dy = torch.full(s.output, float('nan'), device='cuda')
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    count = 0
    with torch.cuda.stream(stream):
        for rank in range(world):
            for u in shard.units_for_rank(s, world, rank):
                sub = u.shape(s)
                ox, ow, oy = u.offsets(s)
                native.cuda(sub, dx.view(-1)[ox:ox + math.prod(sub.input)].view(sub.input),
                            dw.view(-1)[ow:ow + math.prod(sub.weight)].view(sub.weight),
                            dy.view(-1)[oy:oy + math.prod(sub.output)].view(sub.output), 3, stream.cuda_stream)
                count += 1
    stream.synchronize()
    assert count >= min(world, n * groups)
    assert_matches(s, x, w, dy.cpu().numpy(), label=f'group-block units {s}')


def _rows_check(s, x_img, w, y_img, rows):
    """The first `rows` output rows of one image against the FP64 oracle: the
    oracle runs on the input's first rows + 1 (zero padding above as in the
    layer; the last computed row, which would need the next input row, is
    dropped)."""
    crop = dataclasses.replace(s, n=1, h=rows + 1)
    xc = np.ascontiguousarray(x_img[:, :, :rows + 1, :])
    y64, bound = orc.conv_f64_bound(crop, xc, w)
    res = orc.bound_check(y_img[:, :, :rows, :], y64[:, :, :rows, :], bound[:, :, :rows, :])
    assert res['passed'], f'{s} first {rows} rows: {res}'


def _slice_and_points(native, torch, s, impl, label):
    x, w = inputs(s)
    dx, dw = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    dy, plan = _device_run(native, torch, s, dx, dw, impl=impl)
    assert native.device_status(clear=True) == 0
    one = dataclasses.replace(s, n=1)
    y0 = dy[0:1].cpu().numpy()
    work = s.cout * s.h * s.w * s.cpg * s.r * s.s
    if work <= 2e9:
        assert_matches(one, x[0:1], w, y0, label=f'{label} {s} image 0 [{plan}]')
    else:
        _rows_check(s, x[0:1], w, y0, rows=8 if s.h >= 8 else s.h)
    p = orc.check_points(s, x, w, dy)
    long_sum = s.cpg * s.r * s.s > 576  # the reference's fixed gates are sized for sums of <= 576 terms
    assert p['passed'] or long_sum, f'{label} {s} points {p["failed_points"]} [{plan}]'
    if long_sum:
        got = np.array([float(dy[q]) for q in p['points']])
        expected = orc.oracle_points(s, x, w, p['points'])
        abs_sum = orc.oracle_points(s, np.abs(x), np.abs(w), p['points'])
        assert np.all(np.abs(got - expected) <= orc.BOUND_FACTOR * abs_sum), f'{label} {s} bound at points'
    del dx, dy
    torch.cuda.empty_cache()


@pytest.mark.parametrize('index', range(80))
def test_atlas_shape(native, torch_cuda, index):
    s = workloads.atlas_shapes()[index]
    _slice_and_points(native, torch_cuda, s, 3, f'atlas[{index}]')


@pytest.mark.parametrize('index', range(8))
def test_model_layer(native, torch_cuda, index):
    layer = [l for l in workloads.model_layers() if not l.bias][index]
    s = layer.shape
    impl = 3 if s.b_geometry else 0
    x, w = inputs(s)
    dx, dw = torch_cuda.from_numpy(x).cuda(), torch_cuda.from_numpy(w).cuda()
    dy, plan = _device_run(native, torch_cuda, s, dx, dw, impl=impl)
    assert_matches(s, x, w, dy.cpu().numpy(), label=f'{layer.model} {layer.module_path} N{s.n} [{plan}]')
