"""The drop-in boundary on the CPU: the library loads, exports every symbol
include/groupconv.h declares, and answers every malformed or unsupported
request with the reference's status codes.  No kernel is launched here."""
import ctypes as ct
import dataclasses
import re
import threading

import numpy as np
import pytest

from groupconv_atlas_b200 import api
from groupconv_atlas_b200.api import (Shape, cshape, tensor, native_int, NativeError, inputs,
                                      GC_OK, GC_INVALID, GC_UNSUPPORTED, GC_DEVICE_ERROR, GC_UNAVAILABLE)

HEADER = api.ROOT / 'include' / 'groupconv.h'


def declared_functions():
    text = re.sub(r'/\*.*?\*/', '', HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r'\b(gc_\w+)\s*\(', text)) - {'gc_error'})


def test_exports_every_declared_symbol(native):
    names = declared_functions()
    assert 'gc_cuda_conv' in names and 'gc_b200_conv' in names and len(names) >= 19
    for name in names:
        assert hasattr(native.lib, name), name


def test_abi_identity(native):
    assert native.lib.gc_abi_version() == 1
    info = native.lib.gc_build_info().decode()
    assert 'ABI=1' in info and 'sm_100a' in info
    assert native.lib.gc_has_openmp() == 0


def test_struct_layout_matches_reference_abi():
    # 14 x int64 shape; tensor descriptor 8 + 8 + 4*4 + 2*4*8 bytes.
    assert ct.sizeof(api.CShape) == 14 * 8
    assert ct.sizeof(api.Tensor) == 96
    assert api.Tensor.dims.offset == 32 and api.Tensor.strides.offset == 64


def contract_cases(native):
    """The reference's contract checks (bench/check.py:115-140) through gc_cpu_conv."""
    shape = Shape(cin=2, cout=2, groups=2, h=2, w=3)
    x, w = inputs(shape)
    y = np.empty(shape.output, np.float32)
    out = {}
    for name, expected in [('dtype', 1), ('rank', 1), ('strides', 2), ('misaligned', 1), ('device', 1),
                           ('buffer_bytes', 1), ('alias', 1), ('groups', 1), ('geometry', 1),
                           ('implementation', 1)]:
        p, xd, wd, yd = cshape(shape), tensor(x), tensor(w), tensor(y)
        impl = 0
        if name == 'dtype': xd.dtype = 99
        elif name == 'rank': xd.rank = 3
        elif name == 'strides': xd.strides[2] += 1
        elif name == 'misaligned': xd.data += 1
        elif name == 'device': xd.device = 1
        elif name == 'buffer_bytes': xd.bytes -= 4
        elif name == 'alias': yd.data = xd.data
        elif name == 'groups': p.groups = 3
        elif name == 'geometry': p.sh = 0
        elif name == 'implementation': impl = 99
        out[name] = (native.lib.gc_cpu_conv(ct.byref(p), ct.byref(xd), ct.byref(wd), ct.byref(yd), impl, 1),
                     expected)
    return out


def test_reference_contract_checks(native):
    for name, (got, expected) in contract_cases(native).items():
        assert got == expected, name


def test_python_binding_range_checks():
    shape = Shape(cin=2, cout=2, groups=2, h=2, w=3)
    with pytest.raises(ValueError):
        cshape(dataclasses.replace(shape, n=2 ** 64 + 1))
    with pytest.raises(ValueError):
        native_int(2 ** 32)
    with pytest.raises(ValueError):
        native_int(1.5)


def desc(a, device=0, index=0):
    t = tensor(a)
    t.device, t.device_index = device, index
    return t


def test_native_cpu_status_cases(native):
    """reference tests/native_cpu.cpp:56-76 status expectations."""
    lib = native.lib
    p = api.CShape(1, 2, 2, 2, 3, 1, 1, 2, 1, 1, 0, 0, 1, 1)
    x = np.arange(12, dtype=np.float32).reshape(1, 2, 2, 3)
    w = np.array([2, 3], np.float32).reshape(2, 1, 1, 1)
    y = np.zeros((1, 2, 2, 3), np.float32)
    a, b, c = tensor(x), tensor(w), tensor(y)
    call = lambda pp, aa, bb, cc, impl=0, threads=1: lib.gc_cpu_conv(
        ct.byref(pp) if pp is not None else None, ct.byref(aa) if aa is not None else None,
        ct.byref(bb) if bb is not None else None, ct.byref(cc) if cc is not None else None, impl, threads)
    bad = tensor(x); bad.strides[2] += 1
    assert call(p, bad, b, c) == GC_UNSUPPORTED
    bad = tensor(x); bad.bytes -= 1
    assert call(p, bad, b, c) == GC_INVALID
    bad = tensor(x); bad.rank = 3
    assert call(p, bad, b, c) == GC_INVALID
    bad = tensor(x); bad.device = 1
    assert call(p, bad, b, c) == GC_INVALID
    bad = tensor(x); bad.dtype = 999
    assert call(p, bad, b, c) == GC_INVALID
    bad = tensor(x); bad.data += 1
    assert call(p, bad, b, c) == GC_INVALID
    bad = tensor(x); bad.data = (1 << 64) - 4
    assert call(p, bad, b, c) == GC_INVALID
    bad = tensor(y); bad.data = a.data
    assert call(p, a, b, bad) == GC_INVALID
    assert call(None, a, b, c) == GC_INVALID
    assert call(p, None, b, c) == GC_INVALID
    assert call(p, a, None, c) == GC_INVALID
    assert call(p, a, b, None) == GC_INVALID
    assert call(p, a, b, c, 0, 0) == GC_INVALID
    assert call(p, a, b, c, 3, 1) == GC_INVALID
    ho, wo = ct.c_int64(), ct.c_int64()
    for field, value in [('groups', 3), ('ph', 2 ** 63 - 1), ('n', 2 ** 63 - 1), ('r', 9)]:
        q = api.CShape(*[getattr(p, f) for f in api.FIELDS])
        setattr(q, field, value)
        assert lib.gc_validate_shape(ct.byref(q), ct.byref(ho), ct.byref(wo)) == GC_INVALID, field
    q = api.CShape(*[getattr(p, f) for f in api.FIELDS]); q.r = 2 ** 63 - 1; q.dh = 2
    assert lib.gc_validate_shape(ct.byref(q), ct.byref(ho), ct.byref(wo)) == GC_INVALID
    assert lib.gc_validate_shape(ct.byref(p), None, ct.byref(wo)) == GC_INVALID
    assert lib.gc_validate_shape(ct.byref(p), ct.byref(ho), ct.byref(wo)) == GC_OK
    assert (ho.value, wo.value) == (2, 3)


def test_cpu_backend_is_not_built(native):
    """Valid CPU requests are answered GC_UNAVAILABLE and the output is not
    touched: this library never computes a convolution on the host."""
    s = Shape(cin=4, cout=4, groups=2, h=5, w=6)
    x, w = inputs(s)
    y = np.full(s.output, np.nan, np.float32)
    with pytest.raises(NativeError) as err:
        native.cpu(s, x, w, y, 2, 4)
    assert err.value.status == GC_UNAVAILABLE
    assert np.isnan(y).all()
    y64 = np.empty(s.output, np.float64)
    with pytest.raises(NativeError) as err:
        native.cpu(s, x.astype(np.float64), w.astype(np.float64), y64, 1, 1)
    assert err.value.status == GC_UNSUPPORTED


def test_thread_local_error(native):
    lib = native.lib
    q = api.CShape(1, 2, 2, 2, 3, 1, 1, 3, 1, 1, 0, 0, 1, 1)
    ho, wo = ct.c_int64(), ct.c_int64()
    assert lib.gc_validate_shape(ct.byref(q), ct.byref(ho), ct.byref(wo)) == GC_INVALID
    main_error = lib.gc_last_error()
    seen = {}

    def other():
        ok = api.CShape(1, 2, 2, 2, 3, 1, 1, 2, 1, 1, 0, 0, 1, 1)
        lib.gc_validate_shape(ct.byref(ok), ct.byref(ct.c_int64()), ct.byref(ct.c_int64()))
        seen['err'] = lib.gc_last_error()

    t = threading.Thread(target=other)
    t.start(); t.join()
    assert seen['err'] == b''
    assert lib.gc_last_error() == main_error and main_error


def cuda_descs(shape):
    """Descriptors that claim CUDA device 0 over host arrays: they pass the
    metadata validation, so the support matrix is tested without a GPU."""
    x, w = inputs(shape)
    y = np.empty(shape.output, np.float32)
    return (x, w, y), (desc(x, 1, 0), desc(w, 1, 0), desc(y, 1, 0))


@pytest.mark.parametrize('shape,impl,expected', [
    (Shape(cin=4, cout=4, groups=2, h=7, w=13), 4, GC_UNSUPPORTED),
    (Shape(cin=4, cout=4, groups=2, h=7, w=13), -1, GC_UNSUPPORTED),
    (Shape(cin=4, cout=4, groups=2, h=9, w=11, sh=2, sw=2, ph=0, pw=0), 1, GC_UNSUPPORTED),
    (Shape(cin=4, cout=4, groups=2, h=9, w=11, dh=2, dw=2), 3, GC_UNSUPPORTED),
    (Shape(cin=4, cout=6, groups=2, h=5, w=5), 2, GC_UNSUPPORTED),
    (Shape(cin=6, cout=6, groups=2, h=7, w=13), 2, GC_UNSUPPORTED),  # cpg 3
    (Shape(cin=16, cout=16, groups=2, h=7, w=13), 2, GC_UNSUPPORTED),  # cpg 8
])
def test_cuda_support_matrix_without_gpu(native, shape, impl, expected):
    """UNSUPPORTED is decided on the host before any CUDA call (reference
    groupconv.cu:164-177 order)."""
    keep, (xd, wd, yd) = cuda_descs(shape)
    p = cshape(shape)
    assert native.lib.gc_cuda_conv(ct.byref(p), ct.byref(xd), ct.byref(wd), ct.byref(yd), impl, None) == expected


def test_cuda_metadata_errors_without_gpu(native):
    s = Shape(cin=4, cout=4, groups=2, h=7, w=13)
    keep, (xd, wd, yd) = cuda_descs(s)
    p = cshape(s)
    cpu_x = tensor(keep[0])  # a CPU descriptor handed to the CUDA entry point
    assert native.lib.gc_cuda_conv(ct.byref(p), ct.byref(cpu_x), ct.byref(wd), ct.byref(yd), 0, None) == GC_INVALID
    other = desc(keep[1], 1, 1)  # device indices differ
    assert native.lib.gc_cuda_conv(ct.byref(p), ct.byref(xd), ct.byref(other), ct.byref(yd), 0, None) == GC_INVALID
    f64 = np.zeros(s.input, np.float64)
    assert native.lib.gc_cuda_conv(ct.byref(p), ct.byref(desc(f64, 1, 0)), ct.byref(wd), ct.byref(yd), 0,
                                   None) == GC_INVALID
    strided = desc(keep[0], 1, 0); strided.strides[3] = 2
    assert native.lib.gc_cuda_conv(ct.byref(p), ct.byref(strided), ct.byref(wd), ct.byref(yd), 0, None) == GC_UNSUPPORTED


def test_b200_extension_refusals_without_gpu(native):
    s = Shape(cin=4, cout=4, groups=2, h=7, w=13)
    keep, (xd, wd, yd) = cuda_descs(s)
    p = cshape(s)
    lib = native.lib
    assert lib.gc_b200_conv(ct.byref(p), ct.byref(xd), ct.byref(wd), ct.byref(yd), 9, None) == GC_UNSUPPORTED
    assert lib.gc_b200_conv(ct.byref(p), ct.byref(xd), ct.byref(wd), ct.byref(yd), api.DIRECT_TMA, None) == GC_UNSUPPORTED
    assert lib.gc_b200_conv(ct.byref(p), ct.byref(xd), ct.byref(wd), ct.byref(yd), api.TF32X3, None) == GC_UNSUPPORTED
    s2 = Shape(cin=4, cout=4, groups=2, h=9, w=12, sh=2, sw=2)
    keep2, (x2, w2, y2) = cuda_descs(s2)
    p2 = cshape(s2)
    assert lib.gc_b200_conv(ct.byref(p2), ct.byref(x2), ct.byref(w2), ct.byref(y2), api.DIRECT_LDG, None) == GC_UNSUPPORTED
    assert lib.gc_b200_selftest_wait_timeout(0, None) == GC_INVALID
    assert lib.gc_b200_device_status(None, 0) == GC_INVALID


def test_opencl_stubs(native):
    ctx = ct.c_void_p(1)
    assert native.lib.gc_opencl_create(ct.byref(ctx)) == GC_UNAVAILABLE
    assert ctx.value is None
    assert native.lib.gc_opencl_run(None, 0, 1, None) == GC_UNAVAILABLE
    assert native.lib.gc_opencl_download(None, None) == GC_UNAVAILABLE
    assert native.lib.gc_opencl_upload(None, None, None, None, None) == GC_UNAVAILABLE
    native.lib.gc_opencl_destroy(None)


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(api, 'LIBRARY', tmp_path / 'libgroupconv.so')
    monkeypatch.delenv('GROUPCONV_LIBRARY', raising=False)
    with pytest.raises(FileNotFoundError):
        api.Native()
