// Peak-rate probes of the B200 the engine runs on: the denominators of the
// roofline fractions this library reports, measured on the same GPU instead
// of taken from a data sheet.  The reference ships the same idea for its
// RTX 4090 (csrc/cuda/microbench.cu:15-29: a logical copy and eight
// independent FMA chains); these are written for sm_100a and add the tensor
// core's TF32 rate, which bounds the 3xTF32 path.
//
//   ffma_probe_kernel     8 independent FFMA chains per thread, full
//                         occupancy: the FP32 FMA issue rate (2 FLOP per FMA).
//   tf32_mma_probe_kernel one CTA per SM, one thread issues back-to-back
//                         tcgen05.mma.kind::tf32 (M = 128, N = 256, K = 8,
//                         the shape the 3xTF32 path issues) into one TMEM
//                         accumulator, then waits (bounded) for the commit.
//   copy_probe_kernel     16-byte grid-stride copy: HBM read + write rate.
//
// Each probe writes a result per thread or block so the work cannot be
// optimised away; the host entry points only launch, the caller times them
// with events on its stream.
#pragma once
#include "device_util.cuh"
#include "kernel_tf32x3.cuh"

namespace gcb {

constexpr int kProbeChains = 8;     // independent FMA chains per thread
constexpr int kProbeUnroll = 16;    // FMAs per chain per loop iteration
constexpr int kProbeThreads = 256;  // threads per block of the FFMA and copy probes

__global__ void __launch_bounds__(kProbeThreads) ffma_probe_kernel(float *out, float seed, int iters) {
    float a[kProbeChains];
#pragma unroll
    for (int i = 0; i < kProbeChains; ++i) a[i] = seed + 1e-3f * static_cast<float>(threadIdx.x + i);
    // a <- a * m + c stays bounded (|m| < 1), so no value overflows.
    const float m = 0.9999f, c = 1e-4f * seed;
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int u = 0; u < kProbeUnroll; ++u)
#pragma unroll
            for (int i = 0; i < kProbeChains; ++i) a[i] = fmaf(a[i], m, c);
    }
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kProbeChains; ++i) s += a[i];
    out[static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x] = s;
}

__global__ void __launch_bounds__(kProbeThreads) copy_probe_kernel(const float4 *src, float4 *dst, long long n16) {
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n16; i += stride)
        dst[i] = __ldcs(src + i);
}

// Operand tiles in the K-major no-swizzle canonical layout the 3xTF32 path
// uses (core matrix 8 rows x 16 bytes; the two 4-element halves of K = 8 are
// LBO apart): A 128 x 8, B 256 x 8 TF32 values, filled with small finite
// numbers.  status[blockIdx.x] = 0 when the MMAs completed, 1 when the
// bounded wait for their commit gave up.
constexpr int kProbeM = 128;
constexpr int kProbeN = 256;

__global__ void __launch_bounds__(128, 1) tf32_mma_probe_kernel(unsigned *status, int iters) {
    __shared__ __align__(1024) uint32_t a_tile[2 * kProbeM * 4];
    __shared__ __align__(1024) uint32_t b_tile[2 * kProbeN * 4];
    __shared__ uint64_t done_bar;
    __shared__ uint32_t tmem_slot;
    const int tid = threadIdx.x;
    for (int i = tid; i < 2 * kProbeM * 4; i += blockDim.x)
        a_tile[i] = __float_as_uint(static_cast<float>((i * 7 + 3) % 17) * 0.0625f - 0.5f) & 0xFFFFE000u;
    for (int i = tid; i < 2 * kProbeN * 4; i += blockDim.x)
        b_tile[i] = __float_as_uint(static_cast<float>((i * 5 + 1) % 13) * 0.0625f - 0.375f) & 0xFFFFE000u;
    if (tid == 0) {
        mbar_init(&done_bar, 1);
        fence_barrier_init();
    }
    if (tid < 32) tmem_alloc(&tmem_slot, kProbeN);
    fence_async_smem();  // the operand tiles written above become visible to the tensor core
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    bool ok = true;
    if (tid == 0) {
        constexpr uint32_t idesc = umma_idesc_tf32(kProbeM, kProbeN);
        const uint64_t da = umma_desc(smem_addr(a_tile), kProbeM * 16u, 128);
        const uint64_t db = umma_desc(smem_addr(b_tile), kProbeN * 16u, 128);
        for (int k = 0; k < iters; ++k) umma_tf32(tmem, da, db, idesc, k != 0);
        umma_commit(&done_bar);
        ok = mbar_wait_bounded(&done_bar, 0);
        if (!ok) raise_status(kStatusMmaTimeout);
        status[blockIdx.x] = ok ? 0u : 1u;
    }
    if (tid == 0 && !ok) mbar_wait_bounded(&done_bar, 0);  // a second bounded wait before TMEM is freed
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid < 32) tmem_dealloc(tmem, kProbeN);
}

}  // namespace gcb
