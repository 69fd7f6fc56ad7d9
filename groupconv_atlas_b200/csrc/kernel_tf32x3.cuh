// Grouped 3x3 convolution (stride 1, pad 1, Cin == Cout) as an implicit GEMM
// on the 5th-generation tensor cores (tcgen05, accumulators in TMEM), with
// 3xTF32 split precision so the result stays within FP32 tolerance.
//
// GEMM view, per group g and a block of `nb` images stacked along H:
//   D[m, o] = sum_tap sum_ci A_tap[m, ci] * X[o + r*Wp + s, ci]
//   o   : output pixel of the block in "padded" numbering: image k's padded
//         plane (H+2 rows of Wp = W+2 columns, zero border) occupies rows
//         k*(H+2) .. k*(H+2)+H+1, and o = row*Wp + column.  The zero border
//         separates stacked images, so every tap (r, s) is a pure shift of
//         the pixel tile by r*Wp + s rows, and small images share one tile;
//   X   : the padded input of the block, 8 channels per K step;
//   A_tap = [w_hi; w_lo]: the tap's weights of a block of CO output channels
//         (the whole group up to 64 channels, 64-channel blocks of wider
//         groups and dense layers) split x = hi + lo (hi = x rounded to TF32,
//         ties away; lo the exact FP32 remainder, of which the tensor core
//         reads the top 19 bits), stacked along M so one MMA applies both.
// Two MMAs per tap and 8-channel step: D += A_tap X_hi, D += A_tap X_lo, i.e.
// D_hi + D_lo = (w_hi + w_lo)(x_hi + x_lo) up to the truncation of the lo
// parts (below 2^-20 of |x*w| per product, far inside the 1e-5 * sum|x*w|
// acceptance bound).  tcgen05.mma.kind::tf32 with M = 128 (CO > 32) or 64
// rows of weights and N = 256 pixels: at this shape the tensor core runs at
// its full TF32 rate whatever the per-tap shift of the pixel operand.
//
// Rows of A: the M rows are spread over the four TMEM lane quadrants (M = 128:
// row m -> lane m; M = 64: rows 16q..16q+15 -> lanes 32q..32q+15), and within
// a quadrant the first half holds w_hi of a block of output channels, the
// second half w_lo of the same channels, so the epilogue adds the two parts
// with one warp shuffle.
//
// Work item = (output-channel block, image block, strip of sp * 256 pixels,
// part of the input channels); layers with too few output tiles to fill the
// GPU split the input channels into ksplit parts whose partial sums are added
// into the zeroed output, all other layers have ksplit = 1.  Pipeline step =
// (item, chunk of 8 input channels).  Per step:
//   - the converter warps load the step's pixels from global memory into
//     registers (per thread its own pixel rows, 8 coalesced channel loads
//     each; two register sets alternate between even and odd steps, and each
//     set is refilled for step k+2 as soon as step k is converted, so the
//     loads have a whole step to land), split them
//     into the hi/lo pixel tiles (K-major no-swizzle canonical layout: core
//     matrix = 8 rows x 16 bytes, rows 16 bytes apart, the two 4-channel halves
//     LBO apart, so a shift by one pixel is +16 bytes of descriptor address),
//     and split the chunk's weights, which one lane of the weight warp stages
//     by TMA (2-D box of the [C][cpg*9] weight matrix), into the A tiles;
//   - one lane of the MMA warp issues the 18 * sp MMAs and commits them to the
//     mbarrier that frees the stage.
// TMEM holds 512 accumulator columns: with one strip per item, item j uses
// columns 256*(j % 2) and the epilogue of item j overlaps all MMAs of item
// j+1; with two strips per item (the chunk's weights then serve 512 pixels)
// strip s uses columns 256*s, and the MMAs of item j+1 on strip s start as
// soon as the epilogue of item j has drained strip s.  The epilogue
// (tcgen05.ld -> pair sum -> per-warp transpose in shared memory -> coalesced
// streaming stores, consecutive lanes on consecutive pixels) runs on the
// converter warps between their steps.  Every wait is bounded; on timeout the kernel
// records it in the status word, drains what it issued, frees its TMEM and
// returns.  Inputs are assumed finite: for an infinite input the split is
// undefined and the outputs it reaches come out NaN.
#pragma once
#include "device_util.cuh"

namespace gcb {

constexpr int kTf32N = 256;  // pixels per item: the MMA's N

struct Tf32Params {
    const float *x;
    const float *w;
    float *y;
    int n, c, h, wd, cpg, groups;
    int co_blocks;       // output-channel blocks per group: cpg / CO (CO = the kernel's block width)
    int wp;              // padded row pitch W + 2
    int nb;              // images stacked into one block
    int blocks;          // ceil(n / nb)
    int out_rows;        // padded rows holding the block's outputs: (nb - 1) * (h + 2) + h
    int sp;              // 256-pixel strips per item: 1 (two accumulator sets alternate between
                         // items) or 2 (one set holding both strips)
    int strips;          // items per block: ceil(out_rows * wp / (sp * 256))
    int items;           // groups * co_blocks * blocks * strips * ksplit
    int chunks;          // 8-channel steps per item: cpg / 8 / ksplit
    int ksplit;          // parts the input channels of an output tile are split into: 1, or (layers
                         // with too few tiles to fill the GPU) several items whose partial sums are
                         // added into y, zeroed before the launch
    int m;               // MMA M: 128 when CO > 32, else 64
    int rows_b;          // pixel rows per step: sp*256 + 2*wp + 2, rounded up to 8 (<= kTf32MaxRows)
    unsigned a_bytes;    // one step's weight tiles: 9 taps * m * 32
    unsigned b_bytes;    // one pixel tile (hi or lo): rows_b * 32
    unsigned wraw_bytes; // one staged weight chunk: cpg * 72 * 4
};

constexpr int kTf32EpiFloats = 16 * 33;  // per-warp epilogue transpose buffer (16 channels x 32 pixels, padded)

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

// Instruction descriptor: D f32, A/B tf32, both K-major, M = m (64 or 128), N = n.
__host__ __device__ constexpr uint32_t umma_idesc_tf32(int m, int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
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

// 32 consecutive accumulator columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// tmem_ld32 split in two: the load is issued here and its registers are
// valid only after tmem_wait_ld32 on the same array (which takes them as
// read-write operands, so no use can be scheduled before the wait).
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld32(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
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
// Roles (320 threads): warps 0-7 load and convert the pixel rows and the
// weights and run the epilogues; warp 8 (one lane) issues the MMAs; warp 9
// (one lane) issues the weight TMA loads.  Stages are handed over through
// full/empty mbarriers:
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
constexpr int kTf32MaxRows = 4 * kConvThreads;  // pixel rows per step the converters reach

// 2-D tiled load (weights viewed as [C rows][cpg*9 columns]).
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
        : "memory");
}

// Item order: input-channel split fastest, then strip, then image block,
// then output-channel block of a group, group slowest.  gq = group *
// co_blocks + block: the item's weights and outputs are channels gq*CO ..
// gq*CO+CO-1, its inputs the group's 8-channel chunks split*chunks ..
// (split+1)*chunks-1.
__device__ __forceinline__ void tf32_decode(const Tf32Params &P, int item, int &gq, int &blk, int &strip,
                                            int &split) {
    const unsigned u0 = static_cast<unsigned>(item);
    const unsigned u = u0 / static_cast<unsigned>(P.ksplit);
    split = static_cast<int>(u0 - u * static_cast<unsigned>(P.ksplit));
    const unsigned t = u / static_cast<unsigned>(P.strips);
    strip = static_cast<int>(u - t * static_cast<unsigned>(P.strips));
    gq = static_cast<int>(t / static_cast<unsigned>(P.blocks));
    blk = static_cast<int>(t - static_cast<unsigned>(gq) * static_cast<unsigned>(P.blocks));
}

// x = hi + lo: hi rounded to TF32 (nearest, ties away from zero) by integer
// arithmetic on the bit pattern, lo the exact FP32 remainder.
__device__ __forceinline__ void tf32_split(float x, uint32_t &hi, uint32_t &lo) {
    hi = (__float_as_uint(x) + 0x1000u) & 0xFFFFE000u;
    lo = __float_as_uint(x - __uint_as_float(hi));
}

// Converter thread's pixel rows of one item: element offset (image and
// in-plane position) of each row's input pixel, and a bit per row that lies
// inside an image (else the row is zero border or past the block).
template <int ROWS>
struct RowGeom {
    long long off[ROWS];
    unsigned valid;
};

template <int ROWS, bool NHWC>
__device__ __forceinline__ RowGeom<ROWS> tf32_rows(const Tf32Params &P, int blk, int strip, int ctid) {
    RowGeom<ROWS> gm;
    gm.valid = 0;
    const int o0 = strip * P.sp * kTf32N;
    const int hp2 = P.h + 2;
    const long long image_floats = static_cast<long long>(P.c) * P.h * P.wd;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
        const int i = ctid + r * kConvThreads;
        const int o = o0 + i;
        const int vrow = o / P.wp;
        const int k = vrow / hp2;
        const int ih = vrow - k * hp2 - 1, iw = o - vrow * P.wp - 1;
        const int img = blk * P.nb + k;
        const bool in = i < P.rows_b && k < P.nb && img < P.n && ih >= 0 && ih < P.h && iw >= 0 && iw < P.wd;
        // element offset of the pixel: its plane position (NCHW), or the
        // first channel of the pixel (channels last)
        gm.off[r] = !in ? 0
                    : NHWC ? ((static_cast<long long>(img) * P.h + ih) * P.wd + iw) * P.c
                           : static_cast<long long>(img) * image_floats + ih * P.wd + iw;
        gm.valid |= in ? (1u << r) : 0u;
    }
    return gm;
}

// The 8 channels of the chunk at every pixel row of this thread (0 outside images).
template <int ROWS, bool NHWC>
__device__ __forceinline__ void tf32_load_rows(const Tf32Params &P, int gq, int chunk, const RowGeom<ROWS> &gm,
                                               float (&v)[ROWS][8]) {
    const long long hw = static_cast<long long>(P.h) * P.wd;
    const long long c0 = static_cast<long long>(gq / P.co_blocks) * P.cpg + chunk * 8;
    if (NHWC) {
        // channels last: a pixel's 8 channels of the chunk are 32 contiguous bytes
        const float *base = P.x + c0;
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
            const bool in = (gm.valid >> r) & 1u;
            const float4 a = in ? __ldg(reinterpret_cast<const float4 *>(base + gm.off[r])) : make_float4(0, 0, 0, 0);
            const float4 b =
                in ? __ldg(reinterpret_cast<const float4 *>(base + gm.off[r] + 4)) : make_float4(0, 0, 0, 0);
            v[r][0] = a.x, v[r][1] = a.y, v[r][2] = a.z, v[r][3] = a.w;
            v[r][4] = b.x, v[r][5] = b.y, v[r][6] = b.z, v[r][7] = b.w;
        }
        return;
    }
    const float *base = P.x + c0 * hw;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
        const bool in = (gm.valid >> r) & 1u;
#pragma unroll
        for (int ci = 0; ci < 8; ++ci) v[r][ci] = in ? __ldg(base + gm.off[r] + ci * hw) : 0.0f;
    }
}

// Converter warps: epilogue of strip `sub` of one item (256 accumulator
// columns at acc).  Warp w reads lane quadrant w % 4
// and pixel columns [128*(w/4), 128*(w/4) + 128) in chunks of 32.  In the
// quadrant, lane l (l < HALF) holds the w_hi rows and lane l + HALF the w_lo
// rows of the same output channel: one shuffle adds them (lane l keeps
// pixels 0-15 of the chunk, lane l + HALF pixels 16-31).  The sums go through
// the warp's transpose buffer, so that the stores run with consecutive lanes
// on consecutive pixels of one output channel.
template <int M, int CO, bool NHWC>
__device__ __forceinline__ void tf32_epilogue(const Tf32Params &P, uint32_t acc, int item, int sub, int warp,
                                              int lane, float *ep) {
    constexpr int HALF = M / 8;  // output channels per lane quadrant
    int g, blk, strip, split;
    tf32_decode(P, item, g, blk, strip, split);
    const int quad = warp & 3, colhalf = warp >> 2;
    if (quad * HALF >= CO) return;  // quadrant holds only zero rows (warp-uniform)
    const int nco = min(HALF, CO - quad * HALF);
    const bool low = (lane & HALF) == 0;
    const bool writer = lane < 2 * HALF && (lane & (HALF - 1)) < nco;
    const int hp2 = P.h + 2;
    const long long hw = static_cast<long long>(P.h) * P.wd;
    const long long image_floats = static_cast<long long>(P.c) * hw;
    const int out_px = P.out_rows * P.wp;
    float *const ych = P.y + (static_cast<long long>(g) * CO + quad * HALF) * hw;
    float *const epw = ep + (lane & (HALF - 1)) * 33 + (low ? 0 : 16);
    // the TMEM load of chunk c32 + 1 is in flight while chunk c32 is summed
    // and stored (two register sets, alternating)
    const uint32_t tq = acc + colhalf * 128 + (static_cast<uint32_t>(quad * 32) << 16);
    uint32_t rbuf[2][32];
    tmem_ld32_issue(tq, rbuf[0]);
#pragma unroll
    for (int c32 = 0; c32 < 4; ++c32) {
        const int col0 = colhalf * 128 + c32 * 32;
        tmem_wait_ld32(rbuf[c32 & 1]);
        if (c32 + 1 < 4) tmem_ld32_issue(tq + (c32 + 1) * 32, rbuf[(c32 + 1) & 1]);
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(rbuf[c32 & 1][i]);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float send = low ? v[16 + i] : v[i];
            const float r = __shfl_xor_sync(0xffffffffu, send, HALF);
            if (writer) epw[i] = (low ? v[i] : v[16 + i]) + r;
        }
        __syncwarp();
        // lane -> pixel o of the chunk
        const int o = (strip * P.sp + sub) * kTf32N + col0 + lane;
        const int vrow = o / P.wp, col = o - vrow * P.wp;
        const int k = vrow / hp2, hh = vrow - k * hp2;
        const int img = blk * P.nb + k;
        const bool valid = o < out_px && hh < P.h && col < P.wd && img < P.n;
        if (NHWC) {
            const long long poff =
                valid ? ((static_cast<long long>(img) * P.h + hh) * P.wd + col) * P.c + static_cast<long long>(g) * CO +
                            quad * HALF
                      : -1;
            if (P.ksplit == 1) {
                // channels last: each lane stores 4 consecutive channels of a
                // pixel (16 bytes; the quadrant's HALF channels of 32 / (HALF
                // / 4) pixels per store instruction; y is 16-byte aligned and
                // C, CO and HALF are multiples of 4)
                constexpr int V = HALF / 4, PX = 32 / V;
                const int j0 = 4 * (lane % V), pl = lane / V;
#pragma unroll
                for (int it = 0; it < V; ++it) {
                    const int px = it * PX + pl;
                    const long long off = __shfl_sync(0xffffffffu, poff, px);
                    if (off >= 0 && j0 < nco)
                        st_stream_v4(P.y + off + j0, ep[j0 * 33 + px], ep[(j0 + 1) * 33 + px], ep[(j0 + 2) * 33 + px],
                                     ep[(j0 + 3) * 33 + px]);
                }
            } else {
                // a part of the input channels: add into the zeroed output,
                // two pixels (16 lanes of consecutive channels each) per step
                const int j = lane & 15;
#pragma unroll 4
                for (int it = 0; it < 16; ++it) {
                    const int px = 2 * it + (lane >> 4);
                    const long long off = __shfl_sync(0xffffffffu, poff, px);
                    if (off >= 0 && j < nco) atomicAdd(P.y + off + j, ep[j * 33 + px]);
                }
            }
        } else if (valid) {
            float *yp = ych + img * image_floats + static_cast<long long>(hh) * P.wd + col;
            if (P.ksplit == 1) {
                for (int j = 0; j < nco; ++j) st_stream(yp + j * hw, ep[j * 33 + lane]);
            } else {
                // a part of the input channels: add into the zeroed output
                for (int j = 0; j < nco; ++j) atomicAdd(yp + j * hw, ep[j * 33 + lane]);
            }
        }
        __syncwarp();
    }
}

template <int CO, int ROWS, bool NHWC = false>
__global__ void __launch_bounds__(kTf32Threads, 1)
    tf32x3_conv_kernel(const __grid_constant__ Tf32Params P, const __grid_constant__ CUtensorMap wmap) {
    constexpr int M = CO * 2 > 64 ? 128 : 64;
    constexpr int RQ = M / 4;      // A rows per lane quadrant
    constexpr int HALF = RQ / 2;   // output channels per quadrant
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // layout: wraw[2] | a[2] | x_hi[2] | x_lo[2] | epilogue[8 warps] | barriers | words
    unsigned char *const wraw0 = smem_raw;
    unsigned char *const a0 = wraw0 + 2 * P.wraw_bytes;
    unsigned char *const xhi0 = a0 + 2 * P.a_bytes;
    unsigned char *const xlo0 = xhi0 + 2 * P.b_bytes;
    float *const ep0 = reinterpret_cast<float *>(xlo0 + 2 * P.b_bytes);
    uint64_t *const bars = reinterpret_cast<uint64_t *>(ep0 + kConvWarps * kTf32EpiFloats);
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
    // Rows of A no output channel uses (cpg < M / 2) stay zero for the whole kernel.
    if (CO * 2 < M)
        for (unsigned e = tid; e < 2 * P.a_bytes / 16; e += blockDim.x)
            reinterpret_cast<uint4 *>(a0)[e] = make_uint4(0u, 0u, 0u, 0u);
    if (warp == 0) tmem_alloc(tmem_slot, 2 * kTf32N);
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
                int g, blk, strip, split;
                tf32_decode(P, first + item_k * stride, g, blk, strip, split);
                mbar_arrive_expect_tx(&w_full[s], P.wraw_bytes);
                tma_load_2d(wraw0 + s * P.wraw_bytes, &wmap, (split * P.chunks + chunk) * 72, g * CO, &w_full[s]);
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
            constexpr uint32_t kIdesc = umma_idesc_tf32(M, kTf32N);
            int committed = -1;
            for (int k = 0; k < steps; ++k) {
                const int s = k & 1;
                const int item_k = k / P.chunks, chunk = k - item_k * P.chunks;
                if (!role_wait(&ab_full[s], static_cast<uint32_t>((k >> 1) & 1), abort_word, kStatusMmaTimeout))
                    break;
                // Descriptors of the stage's tiles; a shift of the start
                // address is an add on the descriptor's low field (16-byte
                // units; every offset stays inside shared memory, so no carry
                // leaves the field).
                const uint64_t da0 = umma_desc(smem_addr(a0 + s * P.a_bytes), M * 16u, 128);
                const uint64_t dxh0 = umma_desc(smem_addr(xhi0 + s * P.b_bytes), P.rows_b * 16u, 128);
                const uint64_t dxl0 = umma_desc(smem_addr(xlo0 + s * P.b_bytes), P.rows_b * 16u, 128);
                const uint32_t wp = static_cast<uint32_t>(P.wp);
                bool ok = true;
                for (int sub = 0; sub < P.sp && ok; ++sub) {
                    // accumulator set of (item, strip) and the use count of that set
                    const int buf = P.sp == 1 ? (item_k & 1) : sub;
                    const int use = P.sp == 1 ? (item_k >> 1) : item_k;
                    if (chunk == 0 && use >= 1 &&
                        !role_wait(&acc_empty[buf], static_cast<uint32_t>((use - 1) & 1), abort_word,
                                   kStatusMmaTimeout)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem_base + static_cast<uint32_t>(buf * kTf32N);
                    const uint64_t xs = static_cast<uint64_t>(sub) * kTf32N;  // strip's first pixel row
#pragma unroll
                    for (int tap = 0; tap < 9; ++tap) {
                        const uint32_t r = tap / 3, sx = tap % 3;
                        const uint64_t aoff = static_cast<uint64_t>(tap) * M * 2u;  // M rows of 32 bytes
                        const uint64_t xoff = xs + r * wp + sx;                     // pixel rows of 16 bytes
                        if (tap == 0)
                            umma_tf32(d, da0 + aoff, dxh0 + xoff, kIdesc, chunk != 0);
                        else
                            umma_tf32(d, da0 + aoff, dxh0 + xoff, kIdesc, true);
                        umma_tf32(d, da0 + aoff, dxl0 + xoff, kIdesc, true);
                    }
                }
                if (!ok) break;
                umma_commit(&ab_empty[s]);
                if (chunk == P.chunks - 1) umma_commit(&acc_full[P.sp == 1 ? (item_k & 1) : 0]);
                committed = k;
            }
            if (committed >= 0)
                mbar_wait_bounded(&ab_empty[committed & 1], static_cast<uint32_t>((committed >> 1) & 1),
                                  100000000ull);
        }
    } else {
        // Converter / epilogue warps.
        const int ctid = tid;  // 0 .. 255
        const uint32_t lbo_x = P.rows_b * 16u;
        static_assert(kConvThreads == 256, "weight split: 64 quads of 4 lanes");
        float *const ep = ep0 + warp * kTf32EpiFloats;
        int pending = -1;  // per-CTA item index whose epilogue is due
        bool failed = false;
        // Epilogue of item `it`: wait for its last MMAs, then drain strip by
        // strip, releasing each strip's accumulator set as soon as it is read.
        auto drain = [&](int it) -> bool {
            const int fbuf = P.sp == 1 ? (it & 1) : 0;
            const int fuse = P.sp == 1 ? (it >> 1) : it;
            bool done = true;
            if (lane == 0)
                done = role_wait(&acc_full[fbuf], static_cast<uint32_t>(fuse & 1), abort_word, kStatusMmaTimeout);
            if (!__shfl_sync(0xffffffffu, done ? 1 : 0, 0)) return false;
            tc_fence_after();
            for (int sub = 0; sub < P.sp; ++sub) {
                const int buf = P.sp == 1 ? (it & 1) : sub;
                tf32_epilogue<M, CO, NHWC>(P, tmem_base + static_cast<uint32_t>(buf * kTf32N), first + it * stride, sub, warp,
                                 lane, ep);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[buf]);
            }
            return true;
        };
        // Load side: the item whose row geometry is cached.
        int load_item = -1, load_g = 0, load_split = 0;
        RowGeom<ROWS> lgm{};
        auto load = [&](int j, float (&buf)[ROWS][8]) {  // step j's pixel rows into buf
            if (j >= steps) return;
            const int item_j = j / P.chunks, chunk_j = j - item_j * P.chunks;
            if (item_j != load_item) {
                int blk, strip;
                tf32_decode(P, first + item_j * stride, load_g, blk, strip, load_split);
                lgm = tf32_rows<ROWS, NHWC>(P, blk, strip, ctid);
                load_item = item_j;
            }
            tf32_load_rows<ROWS, NHWC>(P, load_g, load_split * P.chunks + chunk_j, lgm, buf);
        };
        // One pipeline step: wait for the stage, convert the weights and the
        // rows held in buf, publish, refill buf with step k+2, and run a due
        // epilogue.
        auto step = [&](int k, float (&buf)[ROWS][8]) {
            const int s = k & 1;
            const int item_k = k / P.chunks, chunk = k - item_k * P.chunks;
            // Lane 0 polls; the other lanes wait in the shuffle.
            bool ok = true;
            if (lane == 0) {
                ok = role_wait(&w_full[s], static_cast<uint32_t>((k >> 1) & 1), abort_word, kStatusTmaTimeout);
                if (ok && k >= 2)
                    ok = role_wait(&ab_empty[s], static_cast<uint32_t>(((k - 2) >> 1) & 1), abort_word,
                                   kStatusMmaTimeout);
            }
            if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) {
                failed = true;
                return;
            }
            // Weights: the chunk's w[co][half*4 + j][tap] (raw [co][72] as
            // staged) go to A row m_hi(co) (hi) and m_hi(co) + HALF (lo), at
            // byte tap*M*32 + half*M*16 + row*16 + j*4.  The converter threads
            // form 64 quads of 4 lanes (lane j of a quad takes input channel
            // j of each half); kWR quads share an output channel and take
            // every kWR-th (tap, half) pair, so the addresses are a per-thread
            // base plus a constant of the unrolled loop (8 consecutive quads
            // store 128 contiguous bytes).
            {
                constexpr int kWR = 64 / CO;  // quads per output channel (CO <= 64)
                const int j = ctid & 3, cq = ctid >> 2;
                if (cq < kWR * CO) {
                    const int co = cq % CO, t0 = cq / CO;
                    const float *wr = reinterpret_cast<const float *>(wraw0 + s * P.wraw_bytes) + co * 72 + j * 9;
                    unsigned char *const at =
                        a0 + s * P.a_bytes + ((co / HALF) * RQ + (co % HALF)) * 16 + j * 4;
#pragma unroll
                    for (int t = 0; t < (18 + kWR - 1) / kWR; ++t) {
                        const int th = t0 + t * kWR;  // (tap, half) pair: th = tap*2 + half
                        if (th < 18) {
                            const int half = th & 1, tap = th >> 1;
                            uint32_t hi, lo;
                            tf32_split(wr[half * 36 + tap], hi, lo);
                            const uint32_t off = tap * M * 32u + half * M * 16u;
                            *reinterpret_cast<uint32_t *>(at + off) = hi;
                            *reinterpret_cast<uint32_t *>(at + off + HALF * 16u) = lo;
                        }
                    }
                }
            }
            // Pixel rows: X[i] = Xpad[o0 + i] for the 8 channels of this chunk.
            {
                unsigned char *const x_hi = xhi0 + s * P.b_bytes, *const x_lo = xlo0 + s * P.b_bytes;
#pragma unroll
                for (int r = 0; r < ROWS; ++r) {
                    const int i = ctid + r * kConvThreads;
                    if (i < P.rows_b) {
                        uint32_t hi[8], lo[8];
#pragma unroll
                        for (int ci = 0; ci < 8; ++ci) tf32_split(buf[r][ci], hi[ci], lo[ci]);
                        const uint32_t off = i * 16u;
                        *reinterpret_cast<uint4 *>(x_hi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                        *reinterpret_cast<uint4 *>(x_hi + off + lbo_x) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
                        *reinterpret_cast<uint4 *>(x_lo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                        *reinterpret_cast<uint4 *>(x_lo + off + lbo_x) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
                    }
                }
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&ab_full[s]);
                mbar_arrive(&w_empty[s]);
            }
            load(k + 2, buf);
            // Epilogue of the previous item while this step's MMAs run.
            if (chunk == 0 && pending >= 0) {
                if (!drain(pending)) {
                    failed = true;
                    return;
                }
                pending = -1;
            }
            if (chunk == P.chunks - 1) pending = item_k;
        };
        float xa[ROWS][8], xb[ROWS][8];
        load(0, xa);
        load(1, xb);
        for (int k = 0; k < steps && !failed; k += 2) {
            step(k, xa);
            if (k + 1 < steps && !failed) step(k + 1, xb);
        }
        if (!failed && pending >= 0) drain(pending);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem_base, 2 * kTf32N);
}

}  // namespace gcb
