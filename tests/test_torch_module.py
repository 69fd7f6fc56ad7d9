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
