// Metadata validation and the thread-local error slot of the C ABI.
//
// Semantics follow the reference's csrc/common/common.cpp:1-110 exactly
// (same checks, same status for each failure, same precedence: every
// GC_INVALID condition of a descriptor is tested before the GC_UNSUPPORTED
// layout condition), written independently for this library.
#include "groupconv.h"

#include <cstdint>
#include <cstddef>
#include <string>

namespace {

thread_local std::string g_last_error;

constexpr int64_t kMax = INT64_MAX;

// a * b into out; false when either factor is negative or the product would
// exceed INT64_MAX (reference common.cpp:10-13).
bool checked_mul(int64_t a, int64_t b, int64_t &out) {
    if (a < 0 || b < 0) return false;
    if (a != 0 && b > kMax / a) return false;
    out = a * b;
    return true;
}

// Output extent of one spatial axis with every intermediate kept in int64
// range (reference common.cpp:14-26).  The last test bounds the largest
// input coordinate a direct kernel forms: (out-1)*stride + (effective-1).
bool axis_extent(int64_t in, int64_t k, int64_t pad, int64_t dil, int64_t stride,
                 int64_t &out) {
    int64_t both_pads = 0, span = 0;
    if (!checked_mul(pad, 2, both_pads)) return false;
    if (in > kMax - both_pads) return false;
    if (!checked_mul(k - 1, dil, span) || span == kMax) return false;
    span += 1;  // receptive field of one output along this axis
    const int64_t padded = in + both_pads;
    if (padded < span) return false;
    out = (padded - span) / stride + 1;
    int64_t last_start = 0;
    if (!checked_mul(out - 1, stride, last_start)) return false;
    return last_start <= kMax - (span - 1);
}

// One descriptor against the dims the geometry implies (reference
// common.cpp:27-50).
int check_descriptor(const gc_tensor *t, const int64_t want[4], int device, int dtype) {
    if (t == nullptr || t->data == nullptr)
        return gc_error(GC_INVALID, "null tensor descriptor or buffer");
    if (t->rank != 4) return gc_error(GC_INVALID, "tensor rank must be four");
    const bool device_ok = t->device == device && t->device_index >= 0 &&
                           !(device == GC_CPU && t->device_index != 0);
    if (!device_ok) return gc_error(GC_INVALID, "tensor device or device index mismatch");
    if (t->dtype != dtype) return gc_error(GC_INVALID, "tensor dtype mismatch");
    int64_t elements = 1;
    bool contiguous = true;
    for (int axis = 3; axis >= 0; --axis) {
        if (t->dims[axis] != want[axis])
            return gc_error(GC_INVALID, "tensor dimensions do not match convolution");
        if (t->strides[axis] != elements) contiguous = false;
        if (!checked_mul(elements, want[axis], elements))
            return gc_error(GC_INVALID, "tensor element count overflow");
    }
    const uint64_t item = dtype == GC_F32 ? 4u : 8u;
    if (static_cast<uint64_t>(elements) > static_cast<uint64_t>(PTRDIFF_MAX) / item)
        return gc_error(GC_INVALID, "tensor byte count exceeds pointer indexing range");
    const uint64_t need = static_cast<uint64_t>(elements) * item;
    const uintptr_t base = reinterpret_cast<uintptr_t>(t->data);
    if (base % item != 0) return gc_error(GC_INVALID, "tensor data is not element aligned");
    if (t->bytes < need) return gc_error(GC_INVALID, "tensor buffer is too small");
    if (t->bytes > UINTPTR_MAX - base) return gc_error(GC_INVALID, "tensor pointer range overflow");
    if (!contiguous)
        return gc_error(GC_UNSUPPORTED, "only dense contiguous NCHW tensors are supported");
    return GC_OK;
}

// Byte ranges [data, data+bytes) intersect (reference common.cpp:51-54).
bool ranges_overlap(const gc_tensor *a, const gc_tensor *b) {
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(a->data);
    const uintptr_t b0 = reinterpret_cast<uintptr_t>(b->data);
    return a0 < b0 + b->bytes && b0 < a0 + a->bytes;
}

}  // namespace

int gc_error(int status, const char *message) {
    g_last_error = message != nullptr ? message : "";
    return status;
}

extern "C" {

int gc_abi_version(void) { return GC_ABI_VERSION; }

const char *gc_last_error(void) { return g_last_error.c_str(); }

// The B200 library has no OpenMP CPU backend.
int gc_has_openmp(void) { return 0; }

const char *gc_build_info(void) {
    return "groupconv-atlas ABI=1; B200 engine; CUDA=sm_100a; CPU=validation-only; "
           "layout=NCHW; dtype=f32; kernels=general,direct_ldg,direct_tma,tf32x3";
}

int gc_validate_shape(const gc_shape *p, int64_t *ho, int64_t *wo) {
    if (p == nullptr || ho == nullptr || wo == nullptr)
        return gc_error(GC_INVALID, "null shape or output extent pointer");
    const bool positive = p->n > 0 && p->cin > 0 && p->cout > 0 && p->h > 0 && p->w > 0 &&
                          p->r > 0 && p->s > 0 && p->groups > 0 && p->sh > 0 &&
                          p->sw > 0 && p->dh > 0 && p->dw > 0 && p->ph >= 0 && p->pw >= 0;
    if (!positive)
        return gc_error(GC_INVALID,
                        "dimensions, groups, strides and dilation must be positive; padding nonnegative");
    if (p->cin % p->groups != 0 || p->cout % p->groups != 0)
        return gc_error(GC_INVALID, "input and output channels must be divisible by groups");
    int64_t oh = 0, ow = 0;
    if (!axis_extent(p->h, p->r, p->ph, p->dh, p->sh, oh) ||
        !axis_extent(p->w, p->s, p->pw, p->dw, p->sw, ow))
        return gc_error(GC_INVALID, "invalid output geometry or signed index overflow");
    const int64_t shapes[3][4] = {{p->n, p->cin, p->h, p->w},
                                  {p->cout, p->cin / p->groups, p->r, p->s},
                                  {p->n, p->cout, oh, ow}};
    for (const auto &dims : shapes) {
        int64_t count = 1;
        for (int i = 0; i < 4; ++i)
            if (!checked_mul(count, dims[i], count))
                return gc_error(GC_INVALID, "shape element count overflow");
    }
    *ho = oh;
    *wo = ow;
    return gc_error(GC_OK, "");
}

int gc_validate_tensors(const gc_shape *p, const gc_tensor *x, const gc_tensor *w,
                        const gc_tensor *y, int device, int dtype) {
    int64_t oh = 0, ow = 0;
    int status = gc_validate_shape(p, &oh, &ow);
    if (status != GC_OK) return status;
    if ((device != GC_CPU && device != GC_CUDA) || (dtype != GC_F32 && dtype != GC_F64))
        return gc_error(GC_INVALID, "unknown expected device or dtype");
    const int64_t xdims[4] = {p->n, p->cin, p->h, p->w};
    const int64_t wdims[4] = {p->cout, p->cin / p->groups, p->r, p->s};
    const int64_t ydims[4] = {p->n, p->cout, oh, ow};
    if ((status = check_descriptor(x, xdims, device, dtype)) != GC_OK) return status;
    if ((status = check_descriptor(w, wdims, device, dtype)) != GC_OK) return status;
    if ((status = check_descriptor(y, ydims, device, dtype)) != GC_OK) return status;
    if (x->device_index != w->device_index || x->device_index != y->device_index)
        return gc_error(GC_INVALID, "tensor device indices differ");
    if (ranges_overlap(y, x) || ranges_overlap(y, w))
        return gc_error(GC_INVALID, "output must not alias input or weights");
    return gc_error(GC_OK, "");
}

// CPU backend entry (reference csrc/cpu/cpu.cpp:3-24): identical argument and
// descriptor checks, then GC_UNAVAILABLE because this library computes only
// on the GPU.
int gc_cpu_conv(const gc_shape *p, const gc_tensor *x, const gc_tensor *w, gc_tensor *y,
                int implementation, int threads) {
    if (implementation < GC_SERIAL || implementation > GC_BLOCKED || threads <= 0)
        return gc_error(GC_INVALID, "invalid CPU implementation or thread count");
    if (x == nullptr) return gc_error(GC_INVALID, "null input tensor descriptor");
    const int status = gc_validate_tensors(p, x, w, y, GC_CPU, x->dtype);
    if (status != GC_OK) return status;
    if (x->dtype == GC_F64 && implementation != GC_SERIAL)
        return gc_error(GC_UNSUPPORTED, "FP64 oracle supports GC_SERIAL only");
    return gc_error(GC_UNAVAILABLE, "CPU backend is not built into the B200 library");
}

// OpenCL backend: not built (reference csrc/opencl/stub.cpp:1-7 behaviour).
int gc_opencl_create(void **context) {
    if (context != nullptr) *context = nullptr;
    return gc_error(GC_UNAVAILABLE, "OpenCL is not built into the B200 library");
}
const char *gc_opencl_info(void *) { return "OpenCL disabled"; }
int gc_opencl_upload(void *, const gc_shape *, const gc_tensor *, const gc_tensor *,
                     const gc_tensor *) {
    return gc_error(GC_UNAVAILABLE, "OpenCL disabled");
}
int gc_opencl_run(void *, int, int, double *) {
    return gc_error(GC_UNAVAILABLE, "OpenCL disabled");
}
int gc_opencl_download(void *, gc_tensor *) {
    return gc_error(GC_UNAVAILABLE, "OpenCL disabled");
}
void gc_opencl_destroy(void *) {}

}  // extern "C"
