/*
 * groupconv.h - C ABI v1 of the grouped 2-D convolution library, B200 build.
 *
 * The types and the v1 entry points below keep the exact layout, names,
 * argument meaning and status codes of the reference interface
 * (csrc/common/groupconv.h:1-58 of LucisZhang/groupconv-atlas), so that a
 * caller bound to that header (its ctypes binding bench/api.py:90-126) loads
 * this library unchanged.  Everything prefixed gc_b200_ is an extension with
 * no counterpart in the reference; callers of the v1 ABI never need it.
 *
 * Conventions (reference csrc/common/groupconv.h:8, :36-37):
 *   - Buffers are borrowed; no function takes ownership.
 *   - Strides are in elements.  Only dense contiguous NCHW is computed.
 *   - CUDA buffers and the stream belong to the caller.  gc_cuda_conv launches
 *     asynchronously on the given stream, never synchronizes and never
 *     allocates device or pinned host memory, so it may be captured in a CUDA
 *     graph.
 *   - Every entry point returns a gc_status; the message of the last call on
 *     the calling thread is available from gc_last_error() (thread local).
 */
#ifndef GROUPCONV_ATLAS_H
#define GROUPCONV_ATLAS_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#define GC_ABI_VERSION 1

/* Status codes: reference csrc/common/groupconv.h:10-11. */
typedef enum {
    GC_OK = 0,
    GC_INVALID = 1,      /* malformed metadata, pointers or sizes           */
    GC_UNSUPPORTED = 2,  /* valid request outside this implementation's set */
    GC_DEVICE_ERROR = 3, /* a CUDA runtime call failed                       */
    GC_UNAVAILABLE = 4   /* backend not built into this library              */
} gc_status;

/* reference csrc/common/groupconv.h:12-14 */
typedef enum { GC_F32 = 0, GC_F64 = 1 } gc_dtype;
typedef enum { GC_CPU = 0, GC_CUDA = 1 } gc_device;
typedef enum { GC_SERIAL = 0, GC_OPENMP = 1, GC_BLOCKED = 2 } gc_cpu_impl;

/* Convolution geometry: 14 x int64 (reference csrc/common/groupconv.h:15-17).
 * x is [n, cin, h, w], weights [cout, cin/groups, r, s],
 * y is [n, cout, ho, wo] with ho = (h + 2ph - dh(r-1) - 1)/sh + 1. */
typedef struct {
    int64_t n, cin, cout, h, w, r, s, groups, sh, sw, ph, pw, dh, dw;
} gc_shape;

/* Borrowed tensor descriptor (reference csrc/common/groupconv.h:18-23). */
typedef struct {
    void *data;
    uint64_t bytes;
    int32_t dtype, device, device_index, rank;
    int64_t dims[4], strides[4];
} gc_tensor;

/* ---- v1 introspection and validation -------------------------------------
 * replaces reference csrc/common/groupconv.h:25-30 (common.cpp:56-109) */
int gc_abi_version(void);
const char *gc_last_error(void);
const char *gc_build_info(void);
int gc_has_openmp(void);
int gc_validate_shape(const gc_shape *p, int64_t *ho, int64_t *wo);
int gc_validate_tensors(const gc_shape *p, const gc_tensor *x,
                        const gc_tensor *w, const gc_tensor *y,
                        int device, int dtype);

/* ---- v1 CPU backend -------------------------------------------------------
 * replaces reference csrc/common/groupconv.h:33-34 (csrc/cpu/cpu.cpp:3-24).
 * This library validates exactly as the reference does (same status for every
 * malformed call) and then answers GC_UNAVAILABLE: the CPU backend is not part
 * of the B200 build, and nothing in it computes a convolution on the host. */
int gc_cpu_conv(const gc_shape *p, const gc_tensor *x, const gc_tensor *w,
                gc_tensor *y, int implementation, int threads);

/* ---- v1 CUDA backend (the hot path) ---------------------------------------
 * replaces reference csrc/common/groupconv.h:38-40 (csrc/cuda/groupconv.cu:
 * 156-222).  implementation (reference support matrix, bench/check.py:106-112):
 *   0  general direct kernel: any valid geometry, any Cin/Cout/groups;
 *   1  3x3/s1/p1/d1, Cin == Cout ("B geometry"), any channels per group;
 *   2  B geometry, channels per group in {1, 2, 4}, otherwise GC_UNSUPPORTED;
 *   3  B geometry, fastest kernel for the shape (the production choice);
 *   any other value: GC_UNSUPPORTED.
 * Implementations 1-3 answer GC_UNSUPPORTED outside B geometry. */
int gc_cuda_available(void);
int gc_cuda_conv(const gc_shape *p, const gc_tensor *x, const gc_tensor *w,
                 gc_tensor *y, int implementation, void *stream);

/* ---- v1 OpenCL backend ----------------------------------------------------
 * replaces reference csrc/common/groupconv.h:44-51.  Not built for B200:
 * every call answers GC_UNAVAILABLE like the reference's csrc/opencl/stub.cpp. */
int gc_opencl_create(void **context);
const char *gc_opencl_info(void *context);
int gc_opencl_upload(void *context, const gc_shape *p, const gc_tensor *x,
                     const gc_tensor *w, const gc_tensor *y);
int gc_opencl_run(void *context, int implementation, int repeats,
                  double *device_op_us);
int gc_opencl_download(void *context, gc_tensor *y);
void gc_opencl_destroy(void *context);

/* ---- B200 extensions (no counterpart in the reference) ------------------- */

/* Kernel families of the B200 engine, for gc_b200_conv. */
typedef enum {
    GC_B200_AUTO = 0,       /* same choice as gc_cuda_conv implementation 3     */
    GC_B200_GENERAL = 1,    /* any geometry, one output column run per thread   */
    GC_B200_DIRECT_LDG = 2, /* B geometry, smem band staged by cp.async         */
    GC_B200_DIRECT_TMA = 3, /* B geometry, smem band staged by TMA tensor loads */
    GC_B200_TF32X3 = 4,     /* B geometry, a multiple of 8 channels per group (dense
                               layers too): tcgen05 3xTF32 implicit GEMM */
    GC_B200_SMALL = 5       /* B geometry, small images (whole planes per CTA, any width) */
} gc_b200_kernel;

/* Same contract as gc_cuda_conv (validation, stream, no allocation, no sync),
 * but runs the named kernel family or answers GC_UNSUPPORTED when that family
 * cannot serve the request (geometry, channels per group, alignment). */
int gc_b200_conv(const gc_shape *p, const gc_tensor *x, const gc_tensor *w,
                 gc_tensor *y, int kernel, void *stream);

/* Layouts of x and y for gc_b200_conv_ex. */
typedef enum {
    GC_B200_NCHW = 0, /* dense NCHW, as gc_cuda_conv                                  */
    GC_B200_NHWC = 1  /* channels last: element strides (H*W*C, 1, W*C, C) for the
                         descriptor dims (N, C, H, W), PyTorch's channels_last format */
} gc_b200_layout;

/* Activation applied after the bias by gc_b200_conv_ex. */
#define GC_B200_ACT_NONE 0
#define GC_B200_ACT_RELU 1  /* max(y, 0)          */
#define GC_B200_ACT_RELU6 2 /* min(max(y, 0), 6)  */

/* Convolution with an optional bias, an optional activation and a choice of
 * layout.  Same contract as gc_cuda_conv (validation, current device,
 * caller's stream, no allocation, no synchronization); weights are always
 * dense [Cout][Cin/groups][R][S].
 *   bias    NULL for none, else a rank-1 dense FP32 CUDA tensor of Cout
 *           elements on the same device; y = conv(x, w) + bias[c], the bias
 *           added after the FP32 sum.  (The reference has no bias: its model
 *           runner reports biased layers, e.g. ConvNeXt's 7x7 depthwise ones,
 *           as unsupported - bench/model_run.py:46-49.)  With a convolution's
 *           batch normalisation folded into w and bias, conv + BN + ReLU6 of
 *           an inference network is one call.
 *   activation  GC_B200_ACT_NONE, _RELU or _RELU6, applied after the bias.
 *   layout  GC_B200_NCHW: without bias and activation the production choice
 *           of gc_cuda_conv implementation 3 (or the general kernel outside
 *           B geometry); with either, the same kernel when it is one of the
 *           direct engines, else the depthwise engines or the general
 *           kernel, any geometry.
 *           GC_B200_NHWC: x and y channels-last (the reference times this
 *           layout only through cuDNN, bench/cuda_boundaries.py:17, and its
 *           ABI rejects it, csrc/common/common.cpp:48).  3x3/s1/p1 layers
 *           with C % 4 == 0 and 16-byte aligned x and y: groups of 16 or
 *           more channels (a multiple of 8, no bias or activation) on the
 *           tcgen05 3xTF32 path, groups of 1, 2, 4 and 8 on the strip kernel,
 *           others on a vectorized kernel; a scalar kernel for every other
 *           geometry.  Strides that are neither -> GC_UNSUPPORTED. */
int gc_b200_conv_ex(const gc_shape *p, const gc_tensor *x, const gc_tensor *w,
                    const gc_tensor *bias, gc_tensor *y, int layout,
                    int activation, void *stream);

/* Benchmark mode (the counterpart of a framework's "benchmark" convolution
 * search): for a shape that implementation 3 serves with a direct engine,
 * time the planner's `candidates` best-scored tilings (1..64) on these
 * buffers and keep the fastest in the library's plan cache, where every later
 * gc_cuda_conv / gc_b200_conv / gc_b200_conv_ex call with the same device,
 * shape and alignment finds it (for the life of the process).  Other shapes:
 * GC_OK, nothing timed.  Unlike gc_cuda_conv it synchronizes `stream`,
 * creates two CUDA events and must not be called inside a stream capture
 * (GC_UNSUPPORTED); y is overwritten with the convolution's result.  Allocates
 * no device memory. */
int gc_b200_autotune(const gc_shape *p, const gc_tensor *x, const gc_tensor *w,
                     gc_tensor *y, int candidates, void *stream);

/* Launch plan chosen by the last successful gc_cuda_conv / gc_b200_conv call
 * on the calling thread: kernel family name, grid, block, shared memory and
 * work split, as one line of text.  Empty before the first launch. */
const char *gc_b200_last_plan(void);

/* Device-side status word shared by every kernel of this library on the
 * current device.  Kernels set a bit when a bounded wait on the asynchronous
 * copy engine gave up (the kernel then leaves its outputs incomplete and
 * returns instead of hanging).  Synchronizes the current device, stores the
 * word in *status and, when clear != 0, resets it to zero. */
#define GC_B200_STATUS_TMA_TIMEOUT 0x1u
#define GC_B200_STATUS_MMA_TIMEOUT 0x2u
int gc_b200_device_status(uint32_t *status, int clear);

/* Self-test of the bounded wait: launches one block on `stream` that waits on
 * a shared-memory barrier nothing will ever complete, gives up after roughly
 * limit_us microseconds, sets GC_B200_STATUS_TMA_TIMEOUT and returns.  Lets a
 * test check the timeout path without faulting or hanging the GPU. */
int gc_b200_selftest_wait_timeout(uint32_t limit_us, void *stream);

/* Peak-rate probes: the denominators of the roofline fractions, measured on
 * the GPU itself (the reference's equivalent for its RTX 4090 is
 * csrc/cuda/microbench.cu:15-29, a logical copy and eight FMA chains).  Each
 * launches one kernel on `stream` into caller-owned device buffers of the
 * current device and returns at once; the caller times it with events.
 *   gc_b200_probe_ffma      `blocks` x 256 threads, 8 independent FFMA
 *                           chains each; out holds blocks * 256 floats.
 *                           FLOPs = gc_b200_probe_ffma_flops(blocks, iters).
 *   gc_b200_probe_tf32_mma  `blocks` CTAs (one per SM), each issuing `iters`
 *                           back-to-back tcgen05.mma.kind::tf32 of
 *                           M = 128, N = 256, K = 8 into TMEM; status holds
 *                           `blocks` words, 0 = completed, 1 = the bounded
 *                           wait for the commit gave up.
 *                           FLOPs = gc_b200_probe_tf32_mma_flops(blocks, iters).
 *   gc_b200_probe_copy      16-byte grid-stride copy src -> dst of `bytes`
 *                           (a multiple of 16; 16-byte aligned buffers that
 *                           do not overlap); bytes moved = 2 * bytes. */
int gc_b200_probe_ffma(float *out, int blocks, int iters, void *stream);
long long gc_b200_probe_ffma_flops(int blocks, int iters);
int gc_b200_probe_tf32_mma(uint32_t *status, int blocks, int iters, void *stream);
long long gc_b200_probe_tf32_mma_flops(int blocks, int iters);
int gc_b200_probe_copy(const void *src, void *dst, uint64_t bytes, int blocks, void *stream);

#ifdef __cplusplus
}
/* Internal shared error helper; returns the supplied status
 * (reference csrc/common/groupconv.h:55-56). */
int gc_error(int status, const char *message);
#endif
#endif
