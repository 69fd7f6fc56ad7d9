// Device-side building blocks shared by the kernels: the status word, bounded
// mbarrier waits, TMA tensor/bulk loads and cp.async copies, as inline PTX for
// sm_100a.  Every TMA load here is a plain per-CTA copy: it reads this
// GPU's own global memory into the issuing CTA's shared memory.
#pragma once
#include <cstdint>
#include <cuda.h>

namespace gcb {

// Bits of the device status word (mirrors GC_B200_STATUS_* in groupconv.h).
constexpr unsigned kStatusTmaTimeout = 0x1u;
constexpr unsigned kStatusMmaTimeout = 0x2u;

// Longest a single wait on an asynchronous copy may take before the kernel
// gives up: two seconds of GPU global time.  Normal waits take microseconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Status word of this library on each device (one translation unit holds
// all device code, so the definition lives here).
__device__ unsigned int g_status = 0;

__device__ __forceinline__ void raise_status(unsigned bits) { atomicOr(&g_status, bits); }

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- programmatic dependent launch -------------------------------------------------
// Blocks until the grids this launch depends on have completed and their
// memory is visible (returns at once when launched without the attribute).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next launch in the stream start its prologue on free SMs.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

// Makes barrier initialisation visible to the async proxy (TMA) before use.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar_addr), "r"(parity)
        : "memory");
    return done != 0;
}

// Component k (0..3) of a 16-byte vector (k known at compile time after
// unrolling).
__device__ __forceinline__ float f4(const float4 &v, int k) {
    return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}

// Waits for the phase with the given parity to complete, for at most
// limit_ns of global time.  Returns false when it gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  uint64_t limit_ns = kWaitLimitNs) {
    const uint32_t a = smem_addr(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = global_ns();
    while (true) {
        if (mbar_try_wait(a, parity)) return true;
        if (global_ns() - t0 > limit_ns) return false;
    }
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Bounded wait of one role of a warp-specialized kernel: gives up when the
// phase does not complete within the limit (sets the abort word and a status
// bit) or when another role has already given up (abort word set).
__device__ __forceinline__ bool role_wait(uint64_t *bar, uint32_t parity, volatile int *abort, unsigned status) {
    const uint32_t a = smem_addr(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = global_ns();
    while (true) {
        if (mbar_try_wait(a, parity)) return true;
        if (*abort) return false;
        if (global_ns() - t0 > kWaitLimitNs) {
            *abort = 1;
            raise_status(status);
            return false;
        }
    }
}

// ---- TMA ----------------------------------------------------------------------
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 4-D tiled tensor load into shared memory; completion is signalled on bar as
// transaction bytes.  c0 is the innermost coordinate.
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, int c3, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
        "r"(smem_addr(bar))
        : "memory");
}

// Contiguous bulk copy global -> shared (addresses 16-byte aligned, size a
// multiple of 16), completion signalled on bar.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes,
                                          uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// ---- cp.async (per-thread asynchronous copies) ----------------------------------
// 4-byte copy; when valid is false nothing is read and the destination is
// zero-filled.
__device__ __forceinline__ void cp_async_4(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_addr(dst)), "l"(src),
                 "r"(valid ? 4 : 0)
                 : "memory");
}
// 16-byte asynchronous copy global -> shared (both addresses 16-byte aligned).
__device__ __forceinline__ void cp_async_16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Waits until at most `pending` (0..3) of this thread's newest groups are in flight.
__device__ __forceinline__ void cp_async_wait_dynamic(int pending) {
    if (pending <= 0) cp_async_wait<0>();
    else if (pending == 1) cp_async_wait<1>();
    else if (pending == 2) cp_async_wait<2>();
    else cp_async_wait<3>();
}

// ---- shared-memory loads ------------------------------------------------------------
// Predicated 4-byte shared load: the value at p when pred, else v, as one
// predicated instruction (no branch, so no warp divergence around rare edge
// loads).
__device__ __forceinline__ float lds_over(const float *p, bool pred, float v) {
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q ld.shared.f32 %0, [%1];\n\t}"
        : "+f"(v)
        : "r"(smem_addr(p)), "r"(pred ? 1 : 0));
    return v;
}

// ---- output epilogue -------------------------------------------------------------
// Activations gc_b200_conv_ex can apply after the (optional) bias: the values
// of GC_B200_ACT_* in groupconv.h.
constexpr int kActNone = 0, kActRelu = 1, kActRelu6 = 2;

// y = act(v + b): the bias only when there is one and the activation only
// when one is asked for, so that without either the stored value is the sum
// itself (bit for bit, signed zeros included).
__device__ __forceinline__ float epilogue(float v, bool has_bias, float b, int act) {
    if (has_bias) v += b;
    if (act == kActRelu) v = fmaxf(v, 0.0f);
    if (act == kActRelu6) v = fminf(fmaxf(v, 0.0f), 6.0f);
    return v;
}

// ---- stores -----------------------------------------------------------------------
// Streaming 16-byte store: the output is not re-read by this kernel, so it is
// marked evict-first to keep the input halo rows resident in L2.
__device__ __forceinline__ void st_stream_v4(float *p, float a, float b, float c, float d) {
    asm volatile("st.global.cs.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
                 "f"(d)
                 : "memory");
}
__device__ __forceinline__ void st_stream(float *p, float a) {
    asm volatile("st.global.cs.f32 [%0], %1;" ::"l"(p), "f"(a) : "memory");
}

}  // namespace gcb
