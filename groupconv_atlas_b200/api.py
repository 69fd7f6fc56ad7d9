"""ctypes binding of the B200 ``libgroupconv.so``, shaped like the reference's.

Mirrors the reference's ``bench/api.py:1-158`` interface - ``Shape``,
``CShape``, ``Tensor``, ``tensor()``, ``cshape()``, ``native_int()``,
``NativeError``, ``Native`` and ``inputs()`` - with the same names, argument
meaning and error behaviour, so callers written against the reference bind
this library unchanged.  ``Native`` additionally binds the ``gc_b200_*``
extensions (kernel-family selection, launch plan, device status word).

Buffers are borrowed: every native call takes raw pointers and sizes from
numpy arrays or torch tensors and never keeps them.  Nothing here computes a
convolution; the CUDA library does, and a missing library is an error.
"""
from __future__ import annotations

import ctypes as ct
import dataclasses
import hashlib
import json
import operator
import os
from pathlib import Path

import numpy as np

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
LIBRARY = PACKAGE / 'libgroupconv.so'
FIELDS = ('n', 'cin', 'cout', 'h', 'w', 'r', 's', 'groups', 'sh', 'sw', 'ph', 'pw', 'dh', 'dw')

# Status codes (include/groupconv.h, reference csrc/common/groupconv.h:10-11).
GC_OK, GC_INVALID, GC_UNSUPPORTED, GC_DEVICE_ERROR, GC_UNAVAILABLE = range(5)
# Kernel families of gc_b200_conv.
AUTO, GENERAL, DIRECT_LDG, DIRECT_TMA, TF32X3, SMALL = range(6)
KERNELS = {'auto': AUTO, 'general': GENERAL, 'direct_ldg': DIRECT_LDG,
           'direct_tma': DIRECT_TMA, 'tf32x3': TF32X3, 'small': SMALL}
# Layouts of gc_b200_conv_ex.
NCHW, NHWC = 0, 1
LAYOUTS = {'nchw': NCHW, 'nhwc': NHWC}
# Activations of gc_b200_conv_ex.
ACT_NONE, ACT_RELU, ACT_RELU6 = 0, 1, 2
ACTIVATIONS = {'none': ACT_NONE, 'relu': ACT_RELU, 'relu6': ACT_RELU6}
STATUS_TMA_TIMEOUT = 0x1
STATUS_MMA_TIMEOUT = 0x2


@dataclasses.dataclass(frozen=True)
class Shape:
    """Convolution geometry; defaults and id hash as reference bench/api.py:15-52."""
    n: int = 1
    cin: int = 16
    cout: int = 16
    h: int = 16
    w: int = 16
    r: int = 3
    s: int = 3
    groups: int = 1
    sh: int = 1
    sw: int = 1
    ph: int = 1
    pw: int = 1
    dh: int = 1
    dw: int = 1

    @property
    def output(self):
        return (self.n, self.cout,
                (self.h + 2 * self.ph - self.dh * (self.r - 1) - 1) // self.sh + 1,
                (self.w + 2 * self.pw - self.dw * (self.s - 1) - 1) // self.sw + 1)

    @property
    def input(self):
        return (self.n, self.cin, self.h, self.w)

    @property
    def weight(self):
        return (self.cout, self.cin // self.groups, self.r, self.s)

    @property
    def cpg(self):
        return self.cin // self.groups

    @property
    def b_geometry(self):
        """3x3, stride 1, pad 1, dilation 1, Cin == Cout: the engine's fast path."""
        return (self.cin == self.cout and self.r == self.s == 3 and self.sh == self.sw == 1
                and self.ph == self.pw == 1 and self.dh == self.dw == 1)

    @property
    def id(self):
        key = {**dataclasses.asdict(self), 'dtype': 'float32', 'layout': 'NCHW', 'bias': False}
        digest = hashlib.sha256(json.dumps(key, sort_keys=True, separators=(',', ':')).encode())
        return 'gc_' + digest.hexdigest()[:16]

    def record(self):
        return {**dataclasses.asdict(self), 'shape_id': self.id, 'input_dims': self.input,
                'weight_dims': self.weight, 'output_dims': self.output, 'dtype': 'float32',
                'layout': 'NCHW', 'bias': False}

    @classmethod
    def from_record(cls, value):
        return cls(**{k: value[k] for k in FIELDS})


class CShape(ct.Structure):
    _fields_ = [(field, ct.c_int64) for field in FIELDS]


class Tensor(ct.Structure):
    _fields_ = [('data', ct.c_void_p), ('bytes', ct.c_uint64), ('dtype', ct.c_int32),
                ('device', ct.c_int32), ('device_index', ct.c_int32), ('rank', ct.c_int32),
                ('dims', ct.c_int64 * 4), ('strides', ct.c_int64 * 4)]


def native_int(value, bits=32):
    """Integral value in signed `bits` range, else ValueError (reference api.py:62-67)."""
    try:
        value = operator.index(value)
    except TypeError as exc:
        raise ValueError('native integers must be integral') from exc
    if not -(1 << (bits - 1)) <= value < (1 << (bits - 1)):
        raise ValueError(f'integer outside signed {bits}-bit range')
    return value


def cshape(shape):
    return CShape(*[native_int(getattr(shape, k), 64) for k in FIELDS])


def tensor(array):
    """Borrowed descriptor of a numpy array or torch tensor (reference api.py:71-83)."""
    if isinstance(array, np.ndarray):
        dtype = {np.dtype('float32'): 0, np.dtype('float64'): 1}.get(array.dtype, -1)
        ptr, size = array.ctypes.data, array.nbytes
        shape, strides = array.shape, tuple(s // array.itemsize for s in array.strides)
        device, index = 0, 0
    else:
        dtype = {'torch.float32': 0, 'torch.float64': 1}.get(str(array.dtype), -1)
        ptr, size = array.data_ptr(), array.numel() * array.element_size()
        shape, strides = tuple(array.shape), tuple(array.stride())
        device, index = (1, array.device.index or 0) if array.device.type == 'cuda' else (0, 0)
        if array.device.type not in ('cpu', 'cuda'):
            device = -1
    dims = (ct.c_int64 * 4)(*shape)
    strd = (ct.c_int64 * 4)(*strides)
    return Tensor(ptr, size, dtype, device, index, len(shape), dims, strd)


class NativeError(RuntimeError):
    def __init__(self, status, message):
        self.status = status
        super().__init__(message)


class Native:
    """Loads ``libgroupconv.so`` and binds every ABI symbol (reference api.py:90-126).

    The default library is the in-tree build next to this file;
    ``$GROUPCONV_LIBRARY`` overrides it as in the reference.
    """

    def __init__(self, path=None):
        if path is None:
            path = os.environ.get('GROUPCONV_LIBRARY') or (str(LIBRARY) if LIBRARY.exists() else '')
        if not path:
            raise FileNotFoundError(
                'libgroupconv.so is not built: run python -m groupconv_atlas_b200.build')
        self.path = str(Path(path).resolve())
        self.lib = ct.CDLL(self.path)
        lib = self.lib
        lib.gc_last_error.restype = ct.c_char_p
        lib.gc_build_info.restype = ct.c_char_p
        lib.gc_abi_version.restype = ct.c_int
        if lib.gc_abi_version() != 1:
            raise RuntimeError('native ABI version mismatch')
        lib.gc_validate_shape.argtypes = [ct.POINTER(CShape), ct.POINTER(ct.c_int64), ct.POINTER(ct.c_int64)]
        lib.gc_validate_tensors.argtypes = [ct.POINTER(CShape)] + [ct.POINTER(Tensor)] * 3 + [ct.c_int, ct.c_int]
        lib.gc_cpu_conv.argtypes = [ct.POINTER(CShape)] + [ct.POINTER(Tensor)] * 3 + [ct.c_int, ct.c_int]
        lib.gc_cuda_conv.argtypes = [ct.POINTER(CShape)] + [ct.POINTER(Tensor)] * 3 + [ct.c_int, ct.c_void_p]
        lib.gc_opencl_create.argtypes = [ct.POINTER(ct.c_void_p)]
        lib.gc_opencl_info.argtypes = [ct.c_void_p]
        lib.gc_opencl_info.restype = ct.c_char_p
        lib.gc_opencl_upload.argtypes = [ct.c_void_p, ct.POINTER(CShape)] + [ct.POINTER(Tensor)] * 3
        lib.gc_opencl_run.argtypes = [ct.c_void_p, ct.c_int, ct.c_int, ct.POINTER(ct.c_double)]
        lib.gc_opencl_download.argtypes = [ct.c_void_p, ct.POINTER(Tensor)]
        lib.gc_opencl_destroy.argtypes = [ct.c_void_p]
        lib.gc_opencl_destroy.restype = None
        # B200 extensions.
        lib.gc_b200_conv.argtypes = [ct.POINTER(CShape)] + [ct.POINTER(Tensor)] * 3 + [ct.c_int, ct.c_void_p]
        lib.gc_b200_last_plan.restype = ct.c_char_p
        lib.gc_b200_device_status.argtypes = [ct.POINTER(ct.c_uint32), ct.c_int]
        lib.gc_b200_selftest_wait_timeout.argtypes = [ct.c_uint32, ct.c_void_p]
        lib.gc_b200_conv_ex.argtypes = [ct.POINTER(CShape)] + [ct.POINTER(Tensor)] * 4 + [ct.c_int, ct.c_int,
                                                                                              ct.c_void_p]
        lib.gc_b200_autotune.argtypes = [ct.POINTER(CShape)] + [ct.POINTER(Tensor)] * 3 + [ct.c_int, ct.c_void_p]
        lib.gc_b200_probe_ffma.argtypes = [ct.c_void_p, ct.c_int, ct.c_int, ct.c_void_p]
        lib.gc_b200_probe_ffma_flops.argtypes = [ct.c_int, ct.c_int]
        lib.gc_b200_probe_ffma_flops.restype = ct.c_longlong
        lib.gc_b200_probe_tf32_mma.argtypes = [ct.c_void_p, ct.c_int, ct.c_int, ct.c_void_p]
        lib.gc_b200_probe_tf32_mma_flops.argtypes = [ct.c_int, ct.c_int]
        lib.gc_b200_probe_tf32_mma_flops.restype = ct.c_longlong
        lib.gc_b200_probe_copy.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_uint64, ct.c_int, ct.c_void_p]

    def check(self, status):
        if status:
            raise NativeError(status, self.lib.gc_last_error().decode())

    def cpu(self, shape, x, w, y, impl=0, threads=1):
        p, xd, wd, yd = cshape(shape), tensor(x), tensor(w), tensor(y)
        self.check(self.lib.gc_cpu_conv(ct.byref(p), ct.byref(xd), ct.byref(wd), ct.byref(yd),
                                        native_int(impl), native_int(threads)))
        return y

    @staticmethod
    def _stream(stream):
        stream = operator.index(stream)
        if not 0 <= stream < (1 << (ct.sizeof(ct.c_void_p) * 8)):
            raise ValueError('stream pointer out of range')
        return stream

    def cuda(self, shape, x, w, y, impl=0, stream=0):
        """gc_cuda_conv on borrowed device tensors; asynchronous on `stream`."""
        p, xd, wd, yd = cshape(shape), tensor(x), tensor(w), tensor(y)
        stream = self._stream(stream)
        self.check(self.lib.gc_cuda_conv(ct.byref(p), ct.byref(xd), ct.byref(wd), ct.byref(yd),
                                         native_int(impl), stream))
        return y

    def b200(self, shape, x, w, y, kernel=AUTO, stream=0):
        """gc_b200_conv: run one named kernel family (see KERNELS)."""
        kernel = KERNELS.get(kernel, kernel) if isinstance(kernel, str) else kernel
        p, xd, wd, yd = cshape(shape), tensor(x), tensor(w), tensor(y)
        stream = self._stream(stream)
        self.check(self.lib.gc_b200_conv(ct.byref(p), ct.byref(xd), ct.byref(wd), ct.byref(yd),
                                         native_int(kernel), stream))
        return y

    def conv_ex(self, shape, x, w, y, bias=None, layout='nchw', activation='none', stream=0):
        """gc_b200_conv_ex: optional bias (rank-1, Cout), activation ('none',
        'relu', 'relu6') and layout 'nchw' or 'nhwc' (x and y channels-last,
        e.g. torch.channels_last tensors)."""
        lay = LAYOUTS.get(layout, layout) if isinstance(layout, str) else layout
        act = ACTIVATIONS.get(activation, activation) if isinstance(activation, str) else activation
        p, xd, wd, yd = cshape(shape), tensor(x), tensor(w), tensor(y)
        bd = tensor(bias) if bias is not None else None
        self.check(self.lib.gc_b200_conv_ex(ct.byref(p), ct.byref(xd), ct.byref(wd),
                                            ct.byref(bd) if bd is not None else None, ct.byref(yd),
                                            native_int(lay), native_int(act), self._stream(stream)))
        return y

    def autotune(self, shape, x, w, y, candidates=8, stream=0):
        """gc_b200_autotune: time the planner's best candidates on these
        buffers once (synchronizing) and cache the fastest plan."""
        p, xd, wd, yd = cshape(shape), tensor(x), tensor(w), tensor(y)
        self.check(self.lib.gc_b200_autotune(ct.byref(p), ct.byref(xd), ct.byref(wd), ct.byref(yd),
                                             native_int(candidates), self._stream(stream)))
        return y

    def last_plan(self):
        return self.lib.gc_b200_last_plan().decode()

    def device_status(self, clear=True):
        """Synchronizes the current device and returns (and clears) its status word."""
        value = ct.c_uint32(0)
        self.check(self.lib.gc_b200_device_status(ct.byref(value), 1 if clear else 0))
        return value.value

    def selftest_wait_timeout(self, limit_us, stream=0):
        self.check(self.lib.gc_b200_selftest_wait_timeout(native_int(limit_us, 33), self._stream(stream)))

    # Peak-rate probes: each launches one kernel into caller-owned device
    # buffers (torch tensors here) and returns the work it does.
    def probe_ffma(self, out, blocks, iters, stream=0):
        """FFMA chains; returns the FLOPs of the launch."""
        self.check(self.lib.gc_b200_probe_ffma(ct.c_void_p(out.data_ptr()), native_int(blocks),
                                               native_int(iters), self._stream(stream)))
        return self.lib.gc_b200_probe_ffma_flops(native_int(blocks), native_int(iters))

    def probe_tf32_mma(self, status, blocks, iters, stream=0):
        """Back-to-back tcgen05 TF32 MMAs; returns the FLOPs of the launch."""
        self.check(self.lib.gc_b200_probe_tf32_mma(ct.c_void_p(status.data_ptr()), native_int(blocks),
                                                   native_int(iters), self._stream(stream)))
        return self.lib.gc_b200_probe_tf32_mma_flops(native_int(blocks), native_int(iters))

    def probe_copy(self, src, dst, blocks, stream=0):
        """Device copy src -> dst; returns the bytes moved (read + write)."""
        nbytes = src.numel() * src.element_size()
        self.check(self.lib.gc_b200_probe_copy(ct.c_void_p(src.data_ptr()), ct.c_void_p(dst.data_ptr()),
                                               nbytes, native_int(blocks), self._stream(stream)))
        return 2 * nbytes


def inputs(shape, seed=20260908):
    """Seeded FP32 inputs exactly as reference bench/api.py:156-158."""
    rng = np.random.default_rng(seed ^ int(shape.id[3:11], 16))
    return (rng.uniform(-1, 1, shape.input).astype(np.float32),
            rng.uniform(-1, 1, shape.weight).astype(np.float32))
