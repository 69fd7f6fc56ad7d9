"""Seeded synthetic inputs for the five benchmark configurations.

All shapes are 3x3, stride 1, pad 1, dilation 1, FP32 NCHW, no bias,
Cin == Cout.  Inputs are generated per image from ``(seed, image index)`` so
that a batch slice ``[0, b)`` is exactly the first ``b`` images of the full
batch - tests check slices against the oracle, benchmarks run the full batch.

  config1  N1    C32  56x56 groups 8  (cpg 4)   x~U[-1,1), w~U[-1,1)/sqrt(9 cpg), seed 0
  config2  N32   C256 56x56 groups 256 (cpg 1)  x~N(0,1),  w~N(0,1/9),               seed 20260908
  config3  80 shapes drawn (seed 1, no replacement) from N{1,4,16,64} x C{32..512}
           x cpg{1..64} (cpg <= C) x H=W{7,14,28,56,112}; x~U[-1,1), w~U[-1,1)/sqrt(9 cpg)
  config4  MobileNetV2 block, N4, depthwise 3x3 on C144 56x56 (see bench.py)   seed 2
  config5  N1024 C256 56x56 groups 32 (cpg 8) and groups 4 (cpg 64)
           x~U[-1,1), w~U[-1,1)/sqrt(9 cpg),                                      seed 3
  atlas    the reference's 80-shape Atlas: N{1,32} x H=W{7,14,28,56,112}
           x cpg{1,2,4,8,16,32,64,256}, C256; x, w ~U[-1,1) seeded per shape id
"""
from __future__ import annotations

import dataclasses
import itertools
import math

import numpy as np

from .api import Shape


@dataclasses.dataclass
class Workload:
    name: str
    shape: Shape
    x: np.ndarray | None
    w: np.ndarray
    seed: int
    dist: str  # 'uniform' or 'normal'

    @property
    def bytes(self):
        """Algorithmic bytes: x read once, w read once, y written once."""
        n, c, ho, wo = self.shape.output
        return 4 * (math.prod(self.shape.input) + math.prod(self.shape.weight) + n * c * ho * wo)

    @property
    def flops(self):
        """2 * N * Cout * Ho * Wo * cpg * R * S (the reference's convention)."""
        n, c, ho, wo = self.shape.output
        return 2 * n * c * ho * wo * self.shape.cpg * self.shape.r * self.shape.s


def _weights(shape, seed, dist):
    rng = np.random.default_rng([seed, 1 << 31])
    if dist == 'normal':
        return (rng.standard_normal(shape.weight) / 3.0).astype(np.float32)
    scale = 1.0 / math.sqrt(9 * shape.cpg)
    return (rng.uniform(-1.0, 1.0, shape.weight) * scale).astype(np.float32)


def images(shape, seed, dist, first=0, count=None):
    """Images [first, first+count) of the seeded input batch, as float32."""
    count = shape.n - first if count is None else count
    out = np.empty((count,) + shape.input[1:], np.float32)
    for i in range(count):
        rng = np.random.default_rng([seed, first + i])
        if dist == 'normal':
            out[i] = rng.standard_normal(shape.input[1:], dtype=np.float32)
        else:
            out[i] = rng.uniform(-1.0, 1.0, shape.input[1:]).astype(np.float32)
    return out


def _make(name, shape, seed, dist, batch=None, with_x=True):
    full = shape
    if batch is not None:
        shape = dataclasses.replace(shape, n=batch)
    w = _weights(full, seed, dist)
    x = images(shape, seed, dist) if with_x else None
    return Workload(name, shape, x, w, seed, dist)


def config1(batch=None, with_x=True):
    return _make('config1', Shape(n=1, cin=32, cout=32, h=56, w=56, groups=8), 0, 'uniform', batch, with_x)


def config2(batch=None, with_x=True):
    return _make('config2', Shape(n=32, cin=256, cout=256, h=56, w=56, groups=256), 20260908, 'normal',
                 batch, with_x)


def config4_leaf(batch=None, with_x=True):
    return _make('config4_leaf', Shape(n=4, cin=144, cout=144, h=56, w=56, groups=144), 2, 'normal', batch,
                 with_x)


def config5(groups=32, batch=None, with_x=True):
    return _make(f'config5_g{groups}', Shape(n=1024, cin=256, cout=256, h=56, w=56, groups=groups), 3,
                 'uniform', batch, with_x)


def custom(spec, batch=None, with_x=True):
    """'N,C,H,W,CPG' -> a 3x3/s1/p1 shape with uniform inputs (seed from its id)."""
    n, c, h, w, cpg = (int(v) for v in spec.split(','))
    shape = Shape(n=n, cin=c, cout=c, h=h, w=w, groups=c // cpg)
    return _make('custom:' + spec, shape, int(shape.id[3:11], 16), 'uniform', batch, with_x)


def by_name(name, batch=None, with_x=True):
    if name.startswith('custom:'):
        return custom(name.split(':', 1)[1], batch, with_x)
    if name == 'config1':
        return config1(batch, with_x)
    if name == 'config2':
        return config2(batch, with_x)
    if name == 'config4_leaf':
        return config4_leaf(batch, with_x)
    if name == 'config5_g32':
        return config5(32, batch, with_x)
    if name == 'config5_g4':
        return config5(4, batch, with_x)
    raise KeyError(name)


SWEEP_N = (1, 4, 16, 64)
SWEEP_C = (32, 64, 128, 256, 512)
SWEEP_CPG = (1, 2, 4, 8, 16, 32, 64)
SWEEP_HW = (7, 14, 28, 56, 112)


def sweep_shapes(count=80, seed=1):
    """The config-3 sweep: `count` shapes drawn without replacement from the
    grid (cpg > C skipped), in grid order of the drawn indices."""
    grid = [Shape(n=n, cin=c, cout=c, h=hw, w=hw, groups=c // cpg)
            for n, c, cpg, hw in itertools.product(SWEEP_N, SWEEP_C, SWEEP_CPG, SWEEP_HW) if cpg <= c]
    picks = np.random.default_rng(seed).choice(len(grid), size=count, replace=False)
    return [grid[i] for i in sorted(int(i) for i in picks)]


ATLAS_N = (1, 32)
ATLAS_HW = (7, 14, 28, 56, 112)
ATLAS_CPG = (1, 2, 4, 8, 16, 32, 64, 256)
ATLAS_C = 256


def atlas_shapes():
    """The reference's frozen 80-shape Atlas (configs/atlas.json): C256, 3x3,
    stride 1, pad 1, N x H=W x cpg over the grid above, in the file's order
    (N, then H, then cpg ascending); cpg 256 is a dense layer (one group).
    Inputs are the reference's per-shape seeding (``api.inputs``)."""
    return [Shape(n=n, cin=ATLAS_C, cout=ATLAS_C, h=hw, w=hw, groups=ATLAS_C // cpg)
            for n, hw, cpg in itertools.product(ATLAS_N, ATLAS_HW, ATLAS_CPG)]


@dataclasses.dataclass(frozen=True)
class ModelLayer:
    model: str
    module_path: str
    shape: Shape
    bias: bool


def model_layers():
    """The reference's 12 frozen model-layer operations
    (configs/model-shapes-protocol.json: torchvision forward hooks at 224x224,
    batches 1 and 4): MobileNetV2 depthwise 3x3 (stride 1 and 2), ResNeXt50
    grouped 3x3 with 32 groups (stride 1 and 2), and ConvNeXt-tiny depthwise
    7x7, which carry a bias the ABI does not have and are reported as
    unsupported, as the reference does (bench/model_run.py).  Inputs are the
    reference's per-shape seeding (``api.inputs``)."""
    def layer(model, path, bias, **geo):
        return [ModelLayer(model, path, Shape(n=n, **geo), bias) for n in (1, 4)]
    mbv2_s1 = layer('mobilenet_v2', 'features.3.conv.1.0', False, cin=144, cout=144, h=56, w=56, groups=144)
    mbv2_s2 = layer('mobilenet_v2', 'features.2.conv.1.0', False, cin=96, cout=96, h=112, w=112, groups=96, sh=2, sw=2)
    rx_s1 = layer('resnext50_32x4d', 'layer1.0.conv2', False, cin=128, cout=128, h=56, w=56, groups=32)
    rx_s2 = layer('resnext50_32x4d', 'layer2.0.conv2', False, cin=256, cout=256, h=56, w=56, groups=32, sh=2, sw=2)
    cn_1 = layer('convnext_tiny', 'features.1.0.block.0', True, cin=96, cout=96, h=56, w=56, r=7, s=7, groups=96,
                 ph=3, pw=3)
    cn_3 = layer('convnext_tiny', 'features.3.0.block.0', True, cin=192, cout=192, h=28, w=28, r=7, s=7, groups=192,
                 ph=3, pw=3)
    # the protocol's order: per model, batch 1 then batch 4, layers in selection order
    layers = []
    for a, b in ((mbv2_s1, mbv2_s2), (rx_s1, rx_s2), (cn_1, cn_3)):
        layers += [a[0], b[0], a[1], b[1]]
    return layers


def sweep_inputs(shape, first=0, count=None):
    """Seeded uniform inputs of one sweep shape (seed derived from its id)."""
    seed = int(shape.id[3:11], 16)
    return images(shape, seed, 'uniform', first, count), _weights(shape, seed, 'uniform')
