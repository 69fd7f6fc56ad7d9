// Grouped 3x3 convolution (stride 1, pad 1, Cin == Cout) as an implicit GEMM
// on the 5th-generation tensor cores (tcgen05, accumulators in TMEM), with
// 3xTF32 split precision so the result stays within FP32 tolerance.
//
// GEMM view, per (image n, group g):  D[o, co] = sum_tap sum_ci A_tap[o, ci] * B_tap[ci, co]
//   o   : output pixel in "padded" numbering o = h * Wp + w, Wp = W + 2 (the two
//         extra columns per row are computed and discarded);
//   A_tap[o, ci] = Xpad[o + r*Wp + s]  for tap (r, s), where Xpad is the input
//         with one zero row/column on every side, numbered the same way.  Every
//         tap is therefore a pure row shift of one shared-memory tile;
//   B_tap[ci, co] = w[g*cpg + co, ci, r, s].
// tcgen05.mma.kind::tf32, M = 128 pixels, N = cpg output channels, K = 8 input
// channels per instruction.  x = hi + lo with hi = x rounded to TF32 (nearest,
// ties away) and lo = x - hi (exact in FP32; the tensor core reads its top 19
// bits); D += A_hi B_hi + A_hi B_lo + A_lo B_hi.  Per product the dropped terms
// are below 2^-20 of |x*w|, far inside the 1e-5 * sum|x*w| acceptance bound.
//
// Work item = (group, image, strip of T consecutive 128-pixel M-tiles); pipeline
// step = (item, chunk of 8 input channels).  Per step:
//   - the converter warps read the step's input pixels straight from global
//     memory (8 coalesced channel loads per A row, issued one step ahead into
//     registers so their latency hides behind the current step), split them
//     into hi/lo TF32 rows of the K-major no-swizzle canonical layout (core
//     matrix = 8 rows x 16 bytes; rows 16 bytes apart, the two 4-channel halves
//     LBO apart, so a shift by one pixel is +16 bytes of descriptor start
//     address), and split the chunk's weights, which one lane of the weight
//     warp stages by TMA (2-D box of the [C][cpg*9] weight matrix);
//   - one lane of the MMA warp issues 27*T MMAs and commits them to the
//     mbarrier that frees the A/B stage.
// The accumulator of item j lives in TMEM buffer j % 2, so the epilogue of item
// j (tcgen05.ld -> coalesced streaming stores of whole output rows) overlaps
// the MMAs of item j+1.  Every wait is bounded; on timeout the kernel records
// it in the status word, drains what it issued, frees its TMEM and returns.
// Inputs are assumed finite: for an infinite input the split is undefined and
// the outputs it reaches come out NaN.
#pragma once
#include "device_util.cuh"

namespace gcb {

struct Tf32Params {
    const float *x;
    const float *w;
    float *y;
    int n, c, h, wd, cpg, groups;
    int wp;              // padded row pitch W + 2
    int tiles;           // 128-pixel M-tiles per image: ceil(h * wp / 128)
    int T;               // M-tiles per item
    int strips;          // ceil(tiles / T)
    int items;           // groups * n * strips
    int chunks;          // cpg / 8
    int rows_a;          // A rows per step: T*128 + 2*wp + 2, rounded up to 8 (<= kTf32MaxRows)
    unsigned a_bytes;    // bytes of one A tile (hi or lo): rows_a * 32
    unsigned b_bytes;    // bytes of one B tile set (hi or lo): 9 taps * cpg * 32
    unsigned wraw_bytes; // bytes of one staged weight chunk: cpg * 72 * 4
    unsigned tmem_cols;  // allocated TMEM columns (power of two)
};

// ---- tcgen05 helpers -----------------------------------------------------------------
// Shared-memory matrix descriptor, K-major, no swizzle (canonical layout
// ((8,m),2):((1,SBO),LBO) in 16-byte units), sm100 version bit set.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;  // descriptor version (Blackwell)
    return d;         // base offset 0, absolute LBO mode 0, layout SWIZZLE_NONE (0)
}

// Instruction descriptor: D f32, A/B tf32, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t umma_idesc_tf32(int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | (8u << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate ? 1 : 0)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Generic-proxy writes to shared memory become visible to the tensor core.
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(dst_smem)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
                 : "memory");
}

// 16 consecutive accumulator columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
        "[%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float (&v)[4]) {
    uint32_t r[4];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr)
                 : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- warp-specialized kernel -------------------------------------------------------------
// Roles (320 threads): warps 0-7 load and convert the A rows and the weights
// to hi/lo TF32 tiles and run the epilogues; warp 8 (one lane) issues the
// MMAs; warp 9 (one lane) issues the weight TMA loads.  Stages are handed
// over through full/empty mbarriers:
//   w_full   (TMA -> converters)     w_empty  (converters -> TMA)
//   ab_full  (converters -> MMA)     ab_empty (MMA commit -> converters)
//   acc_full (MMA commit -> epilogue)  acc_empty (epilogue -> MMA)
// Step k uses stage k % 2 for the k/2-th time, so every wait is on parity
// (k/2) & 1 of that stage's barrier.  Every wait is bounded and also gives up
// as soon as another role has recorded a failure in the shared abort word.
constexpr int kConvWarps = 8;
constexpr int kConvThreads = kConvWarps * 32;
constexpr int kMmaWarp = 8;
constexpr int kTmaWarp = 9;
constexpr int kTf32Threads = 320;
constexpr int kTf32RowsPerThread = 4;
constexpr int kTf32MaxRows = kTf32RowsPerThread * kConvThreads;

// 2-D tiled load (weights viewed as [C rows][cpg*9 columns]).
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
        : "memory");
}

// Item order: group slowest, so consecutive items of one CTA mostly share the
// group's weights in L2.
__device__ __forceinline__ void tf32_decode(const Tf32Params &P, int item, int &g, int &n, int &strip) {
    const unsigned u = static_cast<unsigned>(item);
    const unsigned t = u / static_cast<unsigned>(P.strips);
    strip = static_cast<int>(u - t * static_cast<unsigned>(P.strips));
    g = static_cast<int>(t / static_cast<unsigned>(P.n));
    n = static_cast<int>(t - static_cast<unsigned>(g) * static_cast<unsigned>(P.n));
}

// x = hi + lo: hi rounded to TF32 (nearest, ties away from zero) by integer
// arithmetic on the bit pattern, lo the exact FP32 remainder.
__device__ __forceinline__ void tf32_split(float x, uint32_t &hi, uint32_t &lo) {
    hi = (__float_as_uint(x) + 0x1000u) & 0xFFFFE000u;
    lo = __float_as_uint(x - __uint_as_float(hi));
}

// Converter thread's A rows of one item: plane offset of each row's input
// pixel and a bit per row that lies inside the image (else the row is zero
// padding or past the strip's rows).
struct RowGeom {
    int off[kTf32RowsPerThread];
    unsigned valid;
};

__device__ __forceinline__ RowGeom tf32_rows(const Tf32Params &P, int strip, int ctid) {
    RowGeom gm;
    gm.valid = 0;
    const int o0 = strip * P.T * 128;
#pragma unroll
    for (int r = 0; r < kTf32RowsPerThread; ++r) {
        const int i = ctid + r * kConvThreads;
        const int o = o0 + i;
        const int hp = o / P.wp;
        const int ih = hp - 1, iw = o - hp * P.wp - 1;
        const bool in = i < P.rows_a && ih >= 0 && ih < P.h && iw >= 0 && iw < P.wd;
        gm.off[r] = in ? ih * P.wd + iw : 0;
        gm.valid |= in ? (1u << r) : 0u;
    }
    return gm;
}

// The 8 channels of the chunk at every A row of this thread (0 outside the image).
__device__ __forceinline__ void tf32_load_rows(const Tf32Params &P, int item, int chunk, const RowGeom &gm,
                                               float (&v)[kTf32RowsPerThread][8]) {
    int g, n, strip;
    tf32_decode(P, item, g, n, strip);
    const long long hw = static_cast<long long>(P.h) * P.wd;
    const float *base = P.x + (static_cast<long long>(n) * P.c + g * P.cpg + chunk * 8) * hw;
#pragma unroll
    for (int r = 0; r < kTf32RowsPerThread; ++r) {
        const bool in = (gm.valid >> r) & 1u;
#pragma unroll
        for (int ci = 0; ci < 8; ++ci) v[r][ci] = in ? __ldg(base + ci * hw + gm.off[r]) : 0.0f;
    }
}

// Converter warps: epilogue of one item.  Warp w reads TMEM lanes
// 32*(w%4).. (32 consecutive pixels of each M-tile) and output channels
// [w/4 * NCO/2, (w/4+1) * NCO/2); one coalesced store per channel.
template <int NCO>
__device__ __forceinline__ void tf32_epilogue(const Tf32Params &P, uint32_t acc, int item, int warp, int lane) {
    constexpr int HALF = NCO / 2;
    int g, n, strip;
    tf32_decode(P, item, g, n, strip);
    const int o0 = strip * P.T * 128;
    const int quad = warp & 3, half = warp >> 2;
    const long long plane_out = static_cast<long long>(P.h) * P.wd;
    float *yg = P.y + (static_cast<long long>(n) * P.c + static_cast<long long>(g) * P.cpg + half * HALF) * plane_out;
    for (int t = 0; t < P.T; ++t) {
        if (strip * P.T + t >= P.tiles) break;
        const int o = o0 + t * 128 + quad * 32 + lane;
        const int oh = o / P.wp, ow = o - oh * P.wp;
        const bool store = oh < P.h && ow < P.wd;
        float *yp = yg + static_cast<long long>(oh) * P.wd + ow;
        const uint32_t taddr = acc + t * NCO + half * HALF + (static_cast<uint32_t>(quad * 32) << 16);
        if (HALF % 16 == 0) {
#pragma unroll
            for (int c = 0; c < HALF; c += 16) {
                float v[16];
                tmem_ld16(taddr + c, v);
                if (store) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) st_stream(yp + (c + i) * plane_out, v[i]);
                }
            }
        } else if (HALF % 8 == 0) {
#pragma unroll
            for (int c = 0; c < HALF; c += 8) {
                float v[8];
                tmem_ld8(taddr + c, v);
                if (store) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) st_stream(yp + (c + i) * plane_out, v[i]);
                }
            }
        } else {
#pragma unroll
            for (int c = 0; c < HALF; c += 4) {
                float v[4];
                tmem_ld4(taddr + c, v);
                if (store) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) st_stream(yp + (c + i) * plane_out, v[i]);
                }
            }
        }
    }
}

template <int NCO>
__global__ void __launch_bounds__(kTf32Threads, 1)
    tf32x3_conv_kernel(const __grid_constant__ Tf32Params P, const __grid_constant__ CUtensorMap wmap) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // layout: wraw[2] | a_hi[2] | a_lo[2] | b_hi[2] | b_lo[2] | barriers | words
    unsigned char *const wraw0 = smem_raw;
    unsigned char *const ahi0 = wraw0 + 2 * P.wraw_bytes;
    unsigned char *const alo0 = ahi0 + 2 * P.a_bytes;
    unsigned char *const bhi0 = alo0 + 2 * P.a_bytes;
    unsigned char *const blo0 = bhi0 + 2 * P.b_bytes;
    uint64_t *const bars = reinterpret_cast<uint64_t *>(blo0 + 2 * P.b_bytes);
    uint64_t *const w_full = bars, *const w_empty = bars + 2, *const ab_full = bars + 4,
                    *const ab_empty = bars + 6, *const acc_full = bars + 8, *const acc_empty = bars + 10;
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(bars + 12);
    volatile int *const abort_word = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int first = blockIdx.x, stride = gridDim.x;
    const int my_items = first < P.items ? (P.items - 1 - first) / stride + 1 : 0;
    const int steps = my_items * P.chunks;

    if (tid == 0) {
        for (int s = 0; s < 2; ++s) {
            mbar_init(&w_full[s], 1);
            mbar_init(&w_empty[s], kConvWarps);
            mbar_init(&ab_full[s], kConvWarps);
            mbar_init(&ab_empty[s], 1);
            mbar_init(&acc_full[s], 1);
            mbar_init(&acc_empty[s], kConvWarps);
        }
        *abort_word = 0;
        fence_barrier_init();
    }
    if (warp == 0) tmem_alloc(tmem_slot, P.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    griddep_wait();  // global memory only after the previous launch completed
    griddep_launch_dependents();

    if (warp == kTmaWarp) {
        if (lane == 0) {
            prefetch_tensormap(&wmap);
            int issued = -1, released = -1;
            for (int k = 0; k < steps; ++k) {
                const int s = k & 1;
                if (k >= 2) {
                    if (!role_wait(&w_empty[s], static_cast<uint32_t>(((k - 2) >> 1) & 1), abort_word,
                                   kStatusTmaTimeout))
                        break;
                    released = k - 2;
                }
                const int item_k = k / P.chunks, chunk = k - item_k * P.chunks;
                int g, n, strip;
                tf32_decode(P, first + item_k * stride, g, n, strip);
                mbar_arrive_expect_tx(&w_full[s], P.wraw_bytes);
                tma_load_2d(wraw0 + s * P.wraw_bytes, &wmap, chunk * 72, g * P.cpg, &w_full[s]);
                issued = k;
            }
            // Loads still in flight must land before the CTA's shared memory
            // is released: wait (bounded) for each issued stage not yet seen
            // released by the converters.
            for (int j = released + 1; j <= issued; ++j)
                mbar_wait_bounded(&w_full[j & 1], static_cast<uint32_t>((j >> 1) & 1), 100000000ull);
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            constexpr uint32_t kIdesc = umma_idesc_tf32(NCO);
            const uint32_t lbo_a = P.rows_a * 16u, lbo_b = NCO * 16u;
            int committed = -1;
            for (int k = 0; k < steps; ++k) {
                const int s = k & 1;
                const int item_k = k / P.chunks, chunk = k - item_k * P.chunks;
                if (!role_wait(&ab_full[s], static_cast<uint32_t>((k >> 1) & 1), abort_word, kStatusMmaTimeout))
                    break;
                if (chunk == 0 && item_k >= 2 &&
                    !role_wait(&acc_empty[item_k & 1], static_cast<uint32_t>(((item_k - 2) >> 1) & 1), abort_word,
                               kStatusMmaTimeout))
                    break;
                tc_fence_after();
                int g, n, strip;
                tf32_decode(P, first + item_k * stride, g, n, strip);
                const uint32_t acc = tmem_base + static_cast<uint32_t>((item_k & 1) * P.T * NCO);
                // Descriptors of the stage's tiles; a shift of the start
                // address is an add on the descriptor's low field (16-byte
                // units; every offset stays inside shared memory, so no carry
                // leaves the field).
                const uint64_t dah0 = umma_desc(smem_addr(ahi0 + s * P.a_bytes), lbo_a, 128);
                const uint64_t dal0 = umma_desc(smem_addr(alo0 + s * P.a_bytes), lbo_a, 128);
                const uint64_t dbh0 = umma_desc(smem_addr(bhi0 + s * P.b_bytes), lbo_b, 128);
                const uint64_t dbl0 = umma_desc(smem_addr(blo0 + s * P.b_bytes), lbo_b, 128);
                const uint32_t wp = static_cast<uint32_t>(P.wp);
                for (int t = 0; t < P.T; ++t) {
                    if (strip * P.T + t >= P.tiles) break;
                    const uint32_t d = acc + t * NCO;
                    const uint32_t a_t = static_cast<uint32_t>(t) * 128u;
#pragma unroll
                    for (int tap = 0; tap < 9; ++tap) {
                        const uint32_t r = tap / 3, sx = tap % 3;
                        const uint64_t aoff = a_t + r * wp + sx;              // rows of 16 bytes
                        const uint64_t boff = static_cast<uint64_t>(tap) * NCO * 2u;  // 32 bytes per co
                        const uint64_t dah = dah0 + aoff, dal = dal0 + aoff;
                        const uint64_t dbh = dbh0 + boff, dbl = dbl0 + boff;
                        if (tap == 0)
                            umma_tf32(d, dah, dbh, kIdesc, chunk != 0);
                        else
                            umma_tf32(d, dah, dbh, kIdesc, true);
                        umma_tf32(d, dah, dbl, kIdesc, true);
                        umma_tf32(d, dal, dbh, kIdesc, true);
                    }
                }
                umma_commit(&ab_empty[s]);
                if (chunk == P.chunks - 1) umma_commit(&acc_full[item_k & 1]);
                committed = k;
            }
            if (committed >= 0)
                mbar_wait_bounded(&ab_empty[committed & 1], static_cast<uint32_t>((committed >> 1) & 1),
                                  100000000ull);
        }
    } else {
        // Converter / epilogue warps.
        const int ctid = tid;  // 0 .. 255
        const uint32_t lbo_a = P.rows_a * 16u;
        constexpr int kBVals = 72 * NCO;  // weight values per chunk (hi and lo each)
        constexpr int kBPerThread = (kBVals + kConvThreads - 1) / kConvThreads;
        int pending = -1;  // per-CTA item index whose epilogue is due
        RowGeom gm{};
        float xv[kTf32RowsPerThread][8];
        if (steps > 0) {
            int g, n, strip;
            tf32_decode(P, first, g, n, strip);
            gm = tf32_rows(P, strip, ctid);
            tf32_load_rows(P, first, 0, gm, xv);
        }
        for (int k = 0; k < steps; ++k) {
            const int s = k & 1;
            const int item_k = k / P.chunks, chunk = k - item_k * P.chunks;
            // Next step's rows, in flight while this step converts.
            RowGeom gn = gm;
            float xn[kTf32RowsPerThread][8];
            if (k + 1 < steps) {
                const int item_n = (k + 1) / P.chunks, chunk_n = (k + 1) - item_n * P.chunks;
                if (chunk_n == 0) {
                    int g, n, strip;
                    tf32_decode(P, first + item_n * stride, g, n, strip);
                    gn = tf32_rows(P, strip, ctid);
                }
                tf32_load_rows(P, first + item_n * stride, chunk_n, gn, xn);
            }
            // Lane 0 polls; the other lanes wait in the shuffle.
            bool ok = true;
            if (lane == 0) {
                ok = role_wait(&w_full[s], static_cast<uint32_t>((k >> 1) & 1), abort_word, kStatusTmaTimeout);
                if (ok && k >= 2)
                    ok = role_wait(&ab_empty[s], static_cast<uint32_t>(((k - 2) >> 1) & 1), abort_word,
                                   kStatusMmaTimeout);
            }
            if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
            // Weights: value v of the B tile set is (tap, half, co, j) with j
            // fastest, i.e. the canonical layout is contiguous in v.
            {
                const float *wr = reinterpret_cast<const float *>(wraw0 + s * P.wraw_bytes);
                uint32_t *const bh = reinterpret_cast<uint32_t *>(bhi0 + s * P.b_bytes);
                uint32_t *const bl = reinterpret_cast<uint32_t *>(blo0 + s * P.b_bytes);
#pragma unroll
                for (int q = 0; q < kBPerThread; ++q) {
                    const int v = ctid + q * kConvThreads;
                    if (kBVals % kConvThreads == 0 || v < kBVals) {
                        const int j = v & 3, co = (v >> 2) & (NCO - 1), kt = v / (4 * NCO);
                        const int kg = kt & 1, tap = kt >> 1;
                        uint32_t hi, lo;
                        tf32_split(wr[co * 72 + (kg * 4 + j) * 9 + tap], hi, lo);
                        bh[v] = hi;
                        bl[v] = lo;
                    }
                }
            }
            // Input rows: A[i] = Xpad[o0 + i] for the 8 channels of this chunk.
            {
                unsigned char *const a_hi = ahi0 + s * P.a_bytes, *const a_lo = alo0 + s * P.a_bytes;
#pragma unroll
                for (int r = 0; r < kTf32RowsPerThread; ++r) {
                    const int i = ctid + r * kConvThreads;
                    if (i < P.rows_a) {
                        uint32_t hi[8], lo[8];
#pragma unroll
                        for (int ci = 0; ci < 8; ++ci) tf32_split(xv[r][ci], hi[ci], lo[ci]);
                        const uint32_t off = i * 16u;
                        *reinterpret_cast<uint4 *>(a_hi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                        *reinterpret_cast<uint4 *>(a_hi + off + lbo_a) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
                        *reinterpret_cast<uint4 *>(a_lo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                        *reinterpret_cast<uint4 *>(a_lo + off + lbo_a) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
                    }
                }
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&ab_full[s]);
                mbar_arrive(&w_empty[s]);
            }
            // Epilogue of the previous item while this step's MMAs run.
            if (chunk == 0 && pending >= 0) {
                bool done = true;
                if (lane == 0)
                    done = role_wait(&acc_full[pending & 1], static_cast<uint32_t>((pending >> 1) & 1), abort_word,
                                     kStatusMmaTimeout);
                if (!__shfl_sync(0xffffffffu, done ? 1 : 0, 0)) break;
                tc_fence_after();
                tf32_epilogue<NCO>(P, tmem_base + static_cast<uint32_t>((pending & 1) * P.T * NCO),
                                   first + pending * stride, warp, lane);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[pending & 1]);
                pending = -1;
            }
            if (chunk == P.chunks - 1) pending = item_k;
            gm = gn;
#pragma unroll
            for (int r = 0; r < kTf32RowsPerThread; ++r)
#pragma unroll
                for (int ci = 0; ci < 8; ++ci) xv[r][ci] = xn[r][ci];
        }
        bool last_ok = pending >= 0;
        if (last_ok && lane == 0)
            last_ok = role_wait(&acc_full[pending & 1], static_cast<uint32_t>((pending >> 1) & 1), abort_word,
                                kStatusMmaTimeout);
        if (__shfl_sync(0xffffffffu, last_ok ? 1 : 0, 0)) {
            tc_fence_after();
            tf32_epilogue<NCO>(P, tmem_base + static_cast<uint32_t>((pending & 1) * P.T * NCO),
                               first + pending * stride, warp, lane);
            tc_fence_before();
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem_base, P.tmem_cols);
}

}  // namespace gcb
