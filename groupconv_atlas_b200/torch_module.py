"""torch.nn front end: run a bias-free grouped Conv2d through gc_cuda_conv.

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
