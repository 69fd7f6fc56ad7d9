"""torch.nn front end: run a bias-free grouped Conv2d through gc_cuda_conv, or
a Conv2d -> BatchNorm2d -> ReLU/ReLU6 sequence through one gc_b200_conv_ex call.

Mirrors the reference's module substitution (``NativeDepthwise`` in
bench/module_run.py:215-230): the replacement keeps the convolution's weights,
allocates its output with torch, and calls the C ABI on the current stream.
The difference is the host path: a small C++ front end (torch_ext/conv_op.cpp,
built next to the library) allocates the output and calls the C ABI with no
Python in between, so a substituted layer costs about as much host time as a
cuDNN convolution and the block is competitive in synchronized (API) time, not
just in device time.  Without that front end the module falls back to ctypes
descriptors built once per input geometry (only their data pointers change per
call).  Both paths run the same CUDA kernels; outputs are computed on the GPU
only, and a missing library or an unsupported geometry raises NativeError.
"""
from __future__ import annotations

import ctypes as ct

import torch

from . import api

def _cpp_conv():
    """The C++ front end's entry point (built next to the library by
    build.build_torch_ext), or None when it has not been built."""
    try:
        from . import _gcb_torch
    except ImportError:
        return None
    return _gcb_torch.conv


class B200Conv2d(torch.nn.Module):
    """Forward-only replacement of a bias-free ``torch.nn.Conv2d``."""

    def __init__(self, conv: torch.nn.Conv2d, native: api.Native | None = None, implementation: int = 3,
                 cpp: bool = True):
        super().__init__()
        if conv.bias is not None:
            raise ValueError('gc_cuda_conv has no bias term')
        if isinstance(conv.padding, str):
            raise ValueError('explicit integer padding required')
        self.native = native or api.Native()
        self.implementation = implementation
        self.register_buffer('weight', conv.weight.detach().contiguous().clone())
        self.geometry = dict(cin=conv.in_channels, cout=conv.out_channels, r=conv.kernel_size[0],
                             s=conv.kernel_size[1], groups=conv.groups, sh=conv.stride[0], sw=conv.stride[1],
                             ph=conv.padding[0], pw=conv.padding[1], dh=conv.dilation[0], dw=conv.dilation[1])
        self._cache = {}
        # The C++ front end allocates the output and calls gc_cuda_conv on the
        # current stream without Python in between (about 3 us less host time
        # per call than the ctypes path below, which serves when it is absent).
        self._op = _cpp_conv() if cpp else None
        g = self.geometry
        self._geo = (g['cout'], g['r'], g['s'], g['groups'], g['sh'], g['sw'], g['ph'], g['pw'], g['dh'], g['dw'])
        # gc_cuda_conv through a prototype taking plain addresses: the cached
        # descriptors are passed by address, which costs about half of what
        # ctypes' pointer-argument conversion does
        proto = ct.CFUNCTYPE(ct.c_int, ct.c_void_p, ct.c_void_p, ct.c_void_p, ct.c_void_p, ct.c_int, ct.c_void_p)
        self._fn = proto(ct.cast(self.native.lib.gc_cuda_conv, ct.c_void_p).value)
        # raw handle of the current stream; the public accessor builds a
        # Stream object per call, which costs more than the launch itself
        raw = getattr(torch._C, '_cuda_getCurrentRawStream', None)
        self._stream = (lambda dev: raw(dev)) if raw is not None else \
            (lambda dev: torch.cuda.current_stream(dev).cuda_stream)

    def _descriptors(self, x: torch.Tensor):
        """Per input geometry, device and dtype (input and weight): the
        convolution's Shape, its output size, the ctypes descriptors (only
        their data pointers change per call; their dtype and byte counts are
        part of the key) and their addresses."""
        key = (x.shape, x.get_device(), x.dtype, self.weight.dtype)
        entry = self._cache.get(key)
        if entry is None:
            shape = api.Shape(n=x.shape[0], h=x.shape[2], w=x.shape[3], **self.geometry)
            y = torch.empty(shape.output, device=x.device, dtype=x.dtype)
            descs = (api.cshape(shape), api.tensor(x), api.tensor(self.weight), api.tensor(y))
            entry = (shape, shape.output, descs, tuple(ct.addressof(d) for d in descs))
            self._cache[key] = entry
        return entry

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_contiguous():
            x = x.contiguous()
        if self._op is not None:
            try:
                return self._op(x, self.weight, *self._geo, self.implementation)
            except RuntimeError as e:
                text = str(e)
                if text.startswith('gc_status '):
                    status, _, message = text[len('gc_status '):].partition(': ')
                    raise api.NativeError(int(status), message) from None
                raise
        if x.is_cuda and x.get_device() != torch.cuda.current_device():
            # gc_cuda_conv runs on the current device, which must hold the
            # tensors (nn.Conv2d runs on its input's device)
            with torch.cuda.device(x.device):
                return self.forward(x)
        _, out_shape, (_, xd, wd, yd), (pa, xa, wa, ya) = self._descriptors(x)
        y = x.new_empty(out_shape)
        xd.data = x.data_ptr()
        wd.data = self.weight.data_ptr()
        yd.data = y.data_ptr()
        status = self._fn(pa, xa, wa, ya, self.implementation, (self._stream(xd.device_index) if x.is_cuda else None))
        if status:
            self.native.check(status)
        return y


def _cpp_conv_ex():
    try:
        from . import _gcb_torch
    except ImportError:
        return None
    return getattr(_gcb_torch, 'conv_ex', None)


def _activation_name(act: torch.nn.Module | None) -> str:
    if act is None or isinstance(act, torch.nn.Identity):
        return 'none'
    if isinstance(act, torch.nn.ReLU6) or (isinstance(act, torch.nn.Hardtanh) and act.min_val == 0.0
                                           and act.max_val == 6.0):
        return 'relu6'
    if isinstance(act, torch.nn.ReLU):
        return 'relu'
    raise ValueError(f'activation {type(act).__name__} has no epilogue in gc_b200_conv_ex')


class B200ConvBNAct(torch.nn.Module):
    """Inference replacement of Conv2d -> BatchNorm2d -> ReLU/ReLU6 by ONE
    gc_b200_conv_ex call: the batch normalisation's running statistics are
    folded into the weights and a bias (w' = w * g / sqrt(var + eps),
    b' = beta + (b - mean) * g / sqrt(var + eps)) and the activation runs in
    the kernel's epilogue, so the three framework operations (three launches,
    three host paths) become one.  Eval mode only: the folded statistics are
    those at construction time."""

    def __init__(self, conv: torch.nn.Conv2d, bn: torch.nn.BatchNorm2d | None = None,
                 act: torch.nn.Module | None = None, native: api.Native | None = None):
        super().__init__()
        if isinstance(conv.padding, str):
            raise ValueError('explicit integer padding required')
        self.native = native or api.Native()
        w = conv.weight.detach().double()
        b = conv.bias.detach().double() if conv.bias is not None else torch.zeros(conv.out_channels,
                                                                                  dtype=torch.float64,
                                                                                  device=w.device)
        if bn is not None:
            scale = bn.weight.detach().double() / torch.sqrt(bn.running_var.detach().double() + bn.eps)
            w = w * scale[:, None, None, None]
            b = bn.bias.detach().double() + (b - bn.running_mean.detach().double()) * scale
        self.register_buffer('weight', w.float().contiguous())
        self.register_buffer('bias', b.float().contiguous())
        self.activation = _activation_name(act)
        self._act = api.ACTIVATIONS[self.activation]
        self.geometry = dict(cin=conv.in_channels, cout=conv.out_channels, r=conv.kernel_size[0],
                             s=conv.kernel_size[1], groups=conv.groups, sh=conv.stride[0], sw=conv.stride[1],
                             ph=conv.padding[0], pw=conv.padding[1], dh=conv.dilation[0], dw=conv.dilation[1])
        g = self.geometry
        self._geo = (g['cout'], g['r'], g['s'], g['groups'], g['sh'], g['sw'], g['ph'], g['pw'], g['dh'], g['dw'])
        self._op = _cpp_conv_ex()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        nhwc = x.is_contiguous(memory_format=torch.channels_last) and not x.is_contiguous()
        layout = api.NHWC if nhwc else api.NCHW
        if not nhwc and not x.is_contiguous():
            x = x.contiguous()
        if self._op is not None:
            try:
                return self._op(x, self.weight, self.bias, *self._geo, layout, self._act)
            except RuntimeError as e:
                text = str(e)
                if text.startswith('gc_status '):
                    status, _, message = text[len('gc_status '):].partition(': ')
                    raise api.NativeError(int(status), message) from None
                raise
        shape = api.Shape(n=x.shape[0], h=x.shape[2], w=x.shape[3], **self.geometry)
        y = torch.empty(shape.output, device=x.device, dtype=x.dtype,
                        memory_format=torch.channels_last if nhwc else torch.contiguous_format)
        with torch.cuda.device(x.device):
            self.native.conv_ex(shape, x, self.weight, y, bias=self.bias, layout=layout, activation=self._act,
                                stream=torch.cuda.current_stream(x.device).cuda_stream)
        return y


def fuse_conv_bn_act(module: torch.nn.Module, predicate, native: api.Native | None = None) -> list[str]:
    """Replace every Sequential child whose first three members are Conv2d,
    BatchNorm2d and an activation (torchvision's Conv2dNormActivation, e.g.)
    and whose convolution satisfies predicate(conv) by one B200ConvBNAct;
    returns the dotted names replaced.  For inference (eval) models."""
    native = native or api.Native()
    replaced = []
    for name, child in list(module.named_modules()):
        for attr, sub in list(child._modules.items()):
            if not isinstance(sub, torch.nn.Sequential) or len(sub) < 2:
                continue
            conv, bn = sub[0], sub[1]
            act = sub[2] if len(sub) > 2 else None
            if not (isinstance(conv, torch.nn.Conv2d) and isinstance(bn, torch.nn.BatchNorm2d) and predicate(conv)):
                continue
            if len(sub) > 3:
                continue
            try:
                fused = B200ConvBNAct(conv, bn, act, native)
            except ValueError:
                continue
            child._modules[attr] = fused
            replaced.append(f'{name}.{attr}' if name else attr)
    return replaced


def substitute(module: torch.nn.Module, predicate, native: api.Native | None = None) -> list[str]:
    """Replace every Conv2d child for which predicate(conv) is true; returns
    the dotted names replaced."""
    native = native or api.Native()
    replaced = []
    for name, child in list(module.named_modules()):
        for attr, sub in list(child._modules.items()):
            if isinstance(sub, torch.nn.Conv2d) and predicate(sub):
                child._modules[attr] = B200Conv2d(sub, native)
                replaced.append(f'{name}.{attr}' if name else attr)
    return replaced


def is_depthwise_3x3(conv: torch.nn.Conv2d) -> bool:
    return (conv.groups == conv.in_channels == conv.out_channels and conv.kernel_size == (3, 3)
            and conv.stride == (1, 1) and conv.padding == (1, 1) and conv.dilation == (1, 1)
            and conv.bias is None)


def is_depthwise(conv: torch.nn.Conv2d) -> bool:
    """Any depthwise convolution (groups == Cin == Cout), biased or not."""
    return conv.groups == conv.in_channels == conv.out_channels
