"""The torch.nn front end: module substitution of the MobileNetV2 block's
depthwise 3x3 (config 4), after the reference's bench/module_run.py:215-245."""
import copy

import numpy as np
import pytest
import torch

from groupconv_atlas_b200 import torch_module
from oracle import oracle as orc


def test_rejects_bias_and_string_padding(native):
    with pytest.raises(ValueError):
        torch_module.B200Conv2d(torch.nn.Conv2d(4, 4, 3, padding=1, groups=4, bias=True), native)
    with pytest.raises(ValueError):
        torch_module.B200Conv2d(torch.nn.Conv2d(4, 4, 3, padding='same', groups=4, bias=False), native)
    conv = torch.nn.Conv2d(8, 8, 3, padding=1, groups=8, bias=False)
    assert torch_module.is_depthwise_3x3(conv)
    assert not torch_module.is_depthwise_3x3(torch.nn.Conv2d(8, 8, 3, padding=1, stride=2, groups=8, bias=False))


@pytest.mark.gpu
def test_mobilenet_block_substitution(native, torch_cuda):
    torchvision = pytest.importorskip('torchvision')
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(2)
    block = torchvision.models.mobilenet_v2(weights=None).features[3].eval().cuda()
    cand = copy.deepcopy(block)
    replaced = torch_module.substitute(cand, torch_module.is_depthwise_3x3, native)
    assert replaced == ['conv.1.0']
    x = torch.randn((4, 24, 56, 56), generator=torch.Generator().manual_seed(2)).cuda()
    with torch.inference_mode():
        ref, out = block(x), cand(x)
        # the leaf alone against the FP64 oracle
        conv = block.conv[1][0]
        leaf_in = block.conv[0](x)
        leaf = cand.conv[1][0](leaf_in)
    torch.cuda.synchronize()
    assert orc.error_metrics(out.cpu().numpy(), ref.cpu().numpy())['passed']
    s = torch_module.B200Conv2d(conv, native)._descriptors(leaf_in)[0]
    xi, wi = leaf_in.cpu().numpy(), conv.weight.detach().cpu().numpy()
    y64, bound = orc.conv_f64_bound(s, xi, wi)
    assert orc.bound_check(leaf.cpu().numpy(), y64, bound)['passed']
    # repeated calls reuse cached descriptors and stay correct
    with torch.inference_mode():
        again = cand(x)
    torch.cuda.synchronize()
    assert torch.equal(again, out)


def test_cpp_front_end_reports_status_like_the_c_abi(native):
    """Both host paths of the module turn a rejected call into NativeError with
    the library's status (a CPU tensor is not CUDA device memory: GC_INVALID)."""
    from groupconv_atlas_b200 import api
    conv = torch.nn.Conv2d(4, 4, 3, padding=1, groups=4, bias=False)
    x = torch.randn(1, 4, 6, 6)
    for cpp in (True, False):
        mod = torch_module.B200Conv2d(conv, native, cpp=cpp)
        if cpp:
            assert mod._op is not None, 'C++ front end not built'
        with pytest.raises(api.NativeError) as err:
            mod(x)
        assert err.value.status == 1


@pytest.mark.gpu
@pytest.mark.parametrize('geo', [dict(c=144, h=56, stride=1), dict(c=96, h=112, stride=2), dict(c=64, h=28, stride=1)])
def test_cpp_front_end_matches_ctypes_path(native, torch_cuda, geo):
    """The C++ front end and the ctypes path launch the same kernel: identical outputs."""
    torch.manual_seed(4)
    conv = torch.nn.Conv2d(geo['c'], geo['c'], 3, stride=geo['stride'], padding=1, groups=geo['c'] // 8 if geo['c'] == 64 else geo['c'],
                           bias=False).cuda()
    x = torch.randn(2, geo['c'], geo['h'], geo['h'], device='cuda')
    impl = 3 if geo['stride'] == 1 else 0  # implementations 1-3 take B geometry only
    with torch.inference_mode():
        a = torch_module.B200Conv2d(conv, native, implementation=impl, cpp=True)(x)
        b = torch_module.B200Conv2d(conv, native, implementation=impl, cpp=False)(x)
        ref = torch.nn.functional.conv2d(x, conv.weight, stride=geo['stride'], padding=1, groups=conv.groups)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert orc.error_metrics(a.cpu().numpy(), ref.cpu().numpy())['passed']


def test_ctypes_descriptor_cache_is_keyed_by_dtype(native):
    """A float64 input after a float32 one must not reuse float32 descriptors:
    the call is rejected (GC_INVALID: the CUDA backend computes FP32 only)
    instead of running on stale dtype and byte counts."""
    from groupconv_atlas_b200 import api
    conv = torch.nn.Conv2d(4, 4, 3, padding=1, groups=4, bias=False)
    mod = torch_module.B200Conv2d(conv, native, cpp=False)
    a = mod._descriptors(torch.zeros(1, 4, 6, 6))
    b = mod._descriptors(torch.zeros(1, 4, 6, 6, dtype=torch.float64))
    assert a is not b and b[2][1].dtype == api.tensor(torch.zeros(1, dtype=torch.float64)).dtype
    with pytest.raises(api.NativeError) as err:
        mod(torch.zeros(1, 4, 6, 6, dtype=torch.float64))
    assert err.value.status == 1


@pytest.mark.gpu
def test_input_on_a_device_other_than_the_current_one(native, torch_cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip('needs two CUDA devices')
    conv = torch.nn.Conv2d(16, 16, 3, padding=1, groups=4, bias=False).to('cuda:1')
    x = torch.randn(2, 16, 12, 12, device='cuda:1')
    torch.cuda.set_device(0)
    with torch.inference_mode():
        ref = torch.nn.functional.conv2d(x, conv.weight, padding=1, groups=4)
        for cpp in (True, False):
            y = torch_module.B200Conv2d(conv, native, cpp=cpp)(x)
            assert y.device == x.device
            torch.cuda.synchronize(1)
            assert orc.error_metrics(y.cpu().numpy(), ref.cpu().numpy())['passed']


@pytest.mark.gpu
def test_fused_conv_bn_relu6_block(native, torch_cuda):
    """MobileNetV2 features[3] with its depthwise Conv2dNormActivation fused
    into one gc_b200_conv_ex call (batch norm folded, ReLU6 in the epilogue)
    matches the cuDNN block, with non-trivial batch-norm statistics."""
    torchvision = pytest.importorskip('torchvision')
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(2)
    block = torchvision.models.mobilenet_v2(weights=None).features[3].eval()
    g = torch.Generator().manual_seed(5)
    for m in block.modules():
        if isinstance(m, torch.nn.BatchNorm2d):
            m.running_mean.copy_(torch.randn(m.num_features, generator=g) * 0.2)
            m.running_var.copy_(torch.rand(m.num_features, generator=g) + 0.5)
            m.weight.data.copy_(torch.rand(m.num_features, generator=g) + 0.5)
            m.bias.data.copy_(torch.randn(m.num_features, generator=g) * 0.2)
    block = block.cuda()
    fused = copy.deepcopy(block)
    names = torch_module.fuse_conv_bn_act(fused, torch_module.is_depthwise, native)
    assert names == ['conv.1']
    x = torch.randn((4, 24, 56, 56), generator=torch.Generator().manual_seed(2)).cuda()
    with torch.inference_mode():
        ref, out = block(x), fused(x)
        again = fused(x)
    torch.cuda.synchronize()
    assert orc.error_metrics(out.cpu().numpy(), ref.cpu().numpy())['passed']
    assert torch.equal(out, again)
    for cpp in (True, False):  # the ctypes path gives the same result
        mod = fused.conv[1]
        op = mod._op
        if not cpp:
            mod._op = None
        with torch.inference_mode():
            got = fused(x)
        mod._op = op
        torch.cuda.synchronize()
        assert torch.equal(got, out)
