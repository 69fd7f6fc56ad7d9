// Direct FP32 grouped 3x3 convolution (stride 1, pad 1, Cin == Cout) for
// 8-channel groups on rows of 50-56 pixels (the ResNeXt-style N1024 C256
// 56x56 32-group layer and its relatives), FFMA-bound: 72 FMAs per output
// against 8 bytes of HBM traffic.
//
// Why a second direct kernel for this case: the group-width kernels of
// kernel_direct.cuh stage all input channels of an item at once, which caps
// a thread's register cell at 4 output channels x 8 pixels (288 FFMAs per
// 21 shared loads) and leaves 7 compute warps per CTA for 56-pixel rows, so
// the four schedulers of an SM get unequal work.  Here the input channels
// stream through the shared-memory ring one at a time, which frees the room
// for a cell of a whole group: 8 output channels x 2 rows x 7 columns per
// thread (1008 FFMAs per 36 scalar + 6 vector shared loads), and a warp of
// 32 cells covers one group on a band of 8 rows x 56 columns (8 cells of 7
// columns per row, 4 row pairs), so a CTA of 8 compute warps serves 8 groups
// with two warps per scheduler.
//
// Work item = (block of `gi` groups, image n, band of 8 output rows), block
// slowest so that a persistent CTA keeps one block's weights for many items.
// Pipeline step = (item, input channel ci of the group).  Roles:
//   copy warp (one lane)  per step one 5-D TMA box (W, H, ci, group, n) =
//                         (68 columns from -4, 10 rows from h0-1, 1 channel,
//                         gi groups, 1 image) into the next ring stage; the
//                         copy engine zero-fills everything outside the
//                         image, which is the convolution's padding.  When
//                         an item starts a new group block it also bulk-
//                         copies that block's raw weights (two buffers).
//   compute warp g        transposes its group's weights to [ci][tap][co]
//                         when the block changes (warp-local, no CTA
//                         barrier), accumulates the 8 input channels of the
//                         item from the ring, and stores its outputs through
//                         a per-warp shared buffer as coalesced 16-byte
//                         streaming stores.
// Per output the FMAs run over ci, then the 9 taps in order, exactly as the
// other direct kernels do, so the results are bitwise the same.  Every wait
// is bounded; on timeout the kernel sets a status bit, the copy warp waits
// (bounded) for its loads in flight, and the CTA returns.
#pragma once
#include "device_util.cuh"

namespace gcb {

constexpr int kKsCpg = 8;       // channels per group
constexpr int kKsCw = 7;        // columns per cell
constexpr int kKsVr = 2;        // rows per cell
constexpr int kKsQc = 8;        // cells per row: rows of 50-56 pixels
constexpr int kKsBand = 8;      // output rows per item: 4 row pairs x 8 cells = 32 lanes
constexpr int kKsRows = kKsBand + 2;
constexpr int kKsPitch = 68;    // staged row: columns -4 .. 63; 68 = 4 mod 16 keeps the
                                // warp's 32 row-segment loads on 32 different banks
constexpr int kKsEpiPitch = 60; // epilogue buffer row pitch (conflict-free stores)
constexpr int kKsMaxGroups = 8; // compute warps per CTA
constexpr int kKsMaxStages = 8;
constexpr int kKsWFloats = kKsCpg * kKsCpg * 9;  // one group's weights: 576

struct KsParams {
    const float *w;
    float *y;
    int n, c, h, wd;
    int groups;          // c / 8
    int gi;              // groups per item (= compute warps), divides groups, <= 8
    int gblocks;         // groups / gi
    int bands;           // ceil(h / 8)
    int items;           // gblocks * n * bands
    int stages;          // ring depth
    unsigned stage_bytes;  // one stage, rounded up to 128 bytes (the TMA box is gi * 10 * 68 * 4)
    unsigned box_bytes;    // bytes one TMA box delivers
    unsigned wraw_bytes;   // one group block's raw weights: gi * 576 * 4
    int vec_store;       // 16-byte output stores (y 16-byte aligned, width % 4 == 0)
};

__device__ __forceinline__ void ks_decode(const KsParams &P, int item, int &gb, int &n, int &band) {
    const unsigned u = static_cast<unsigned>(item);
    const unsigned t = u / static_cast<unsigned>(P.bands);
    band = static_cast<int>(u - t * static_cast<unsigned>(P.bands));
    gb = static_cast<int>(t / static_cast<unsigned>(P.n));
    n = static_cast<int>(t - static_cast<unsigned>(gb) * static_cast<unsigned>(P.n));
}

__device__ __forceinline__ void tma_load_5d(void *dst, const CUtensorMap *map, int c0, int c1, int c2, int c3,
                                            int c4, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(smem_addr(bar))
        : "memory");
}

// Shared memory: ring stages | raw weights x2 | transposed weights (per warp) |
// epilogue buffers (per warp) | barriers | abort word.
__host__ __device__ inline size_t ks_fixed_bytes(int gi) {
    return static_cast<size_t>(gi) * kKsWFloats * 4 * 3 + static_cast<size_t>(gi) * kKsBand * kKsEpiPitch * 4 +
           (2 * kKsMaxStages + 4) * 8 + 16;
}

__global__ void __launch_bounds__(kKsMaxGroups * 32 + 32, 1)
    kstream_conv_kernel(const __grid_constant__ KsParams P, const __grid_constant__ CUtensorMap xmap) {
    extern __shared__ __align__(128) unsigned char ks_smem[];
    const int S = P.stages;
    unsigned char *const ring = ks_smem;
    float *const wraw = reinterpret_cast<float *>(ring + static_cast<size_t>(S) * P.stage_bytes);
    float *const wt = wraw + 2 * P.gi * kKsWFloats;
    float *const epi = wt + P.gi * kKsWFloats;
    uint64_t *const full = reinterpret_cast<uint64_t *>(epi + P.gi * kKsBand * kKsEpiPitch);
    uint64_t *const empty = full + kKsMaxStages;
    uint64_t *const wfull = empty + kKsMaxStages;
    uint64_t *const wempty = wfull + 2;
    volatile int *const abort_word = reinterpret_cast<volatile int *>(wempty + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int first = blockIdx.x, step = gridDim.x;
    const int count = first < P.items ? (P.items - 1 - first) / step + 1 : 0;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], P.gi);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&wfull[b], 1);
            mbar_init(&wempty[b], P.gi);
        }
        *abort_word = 0;
        fence_barrier_init();
        prefetch_tensormap(&xmap);
    }
    // Everything above touches only shared memory and parameters; global
    // memory is read and written after the previous launch in the stream has
    // completed.
    griddep_wait();
    griddep_launch_dependents();
    __syncthreads();

    if (warp == P.gi) {
        // ---- copy warp: one lane issues every load ----
        if (lane != 0) return;
        int j = 0, wk = 0, last_gb = -1;
        bool ok = true;
        for (int k = 0; k < count && ok; ++k) {
            int gb, n, band;
            ks_decode(P, first + k * step, gb, n, band);
            if (gb != last_gb) {
                const int wb = wk & 1;
                if (wk >= 2 &&
                    !role_wait(&wempty[wb], static_cast<uint32_t>(((wk - 2) >> 1) & 1), abort_word,
                               kStatusTmaTimeout)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&wfull[wb], P.wraw_bytes);
                bulk_load(wraw + wb * P.gi * kKsWFloats, P.w + static_cast<long long>(gb) * P.gi * kKsWFloats,
                          P.wraw_bytes, &wfull[wb]);
                ++wk;
                last_gb = gb;
            }
            for (int ci = 0; ci < kKsCpg; ++ci, ++j) {
                const int s = j % S;
                if (j >= S && !role_wait(&empty[s], static_cast<uint32_t>((j / S - 1) & 1), abort_word,
                                         kStatusTmaTimeout)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&full[s], P.box_bytes);
                tma_load_5d(ring + static_cast<size_t>(s) * P.stage_bytes, &xmap, -4, band * kKsBand - 1, ci,
                            gb * P.gi, n, &full[s]);
            }
        }
        // The loads still in flight must land before the CTA's shared memory
        // is released (all earlier stages were consumed before being
        // refilled).  Always, bounded: other warps may have given up.
        for (int i = max(0, j - S); i < j; ++i)
            mbar_wait_bounded(&full[i % S], static_cast<uint32_t>((i / S) & 1));
        for (int i = max(0, wk - 2); i < wk; ++i)
            mbar_wait_bounded(&wfull[i & 1], static_cast<uint32_t>((i >> 1) & 1));
        return;
    }
    if (warp > P.gi) return;

    // ---- compute warp `warp`: group gb * gi + warp of each item ----
    const int q = lane & 7, rb = lane >> 3;  // cell: rows 2rb, 2rb+1; columns 7q .. 7q+6
    float *const wt_g = wt + warp * kKsWFloats;
    float *const epi_g = epi + warp * kKsBand * kKsEpiPitch;
    const long long plane = static_cast<long long>(P.h) * P.wd;
    int j = 0, wk = 0, last_gb = -1;
    for (int k = 0; k < count; ++k) {
        int gb, n, band;
        ks_decode(P, first + k * step, gb, n, band);
        if (gb != last_gb) {
            const int wb = wk & 1;
            if (!__all_sync(0xffffffffu, role_wait(&wfull[wb], static_cast<uint32_t>((wk >> 1) & 1), abort_word,
                                                   kStatusTmaTimeout)))
                return;
            // raw [co][ci][tap] of this warp's group -> [ci][tap][co]
            const float *src = wraw + wb * P.gi * kKsWFloats + warp * kKsWFloats;
            for (int e = lane; e < kKsWFloats; e += 32) {
                const int co = e / 72, kk = e - co * 72;
                wt_g[kk * 8 + co] = src[e];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&wempty[wb]);
            ++wk;
            last_gb = gb;
        }
        float acc[8][kKsVr][kKsCw];
#pragma unroll
        for (int co = 0; co < 8; ++co)
#pragma unroll
            for (int v = 0; v < kKsVr; ++v)
#pragma unroll
                for (int u = 0; u < kKsCw; ++u) acc[co][v][u] = 0.0f;
#pragma unroll 1
        for (int ci = 0; ci < kKsCpg; ++ci, ++j) {
            const int s = j % S;
            if (!__all_sync(0xffffffffu, role_wait(&full[s], static_cast<uint32_t>((j / S) & 1), abort_word,
                                                   kStatusTmaTimeout)))
                return;
            // this warp's group plane: 10 rows x 68, image column c at index c + 4
            const float *xs = reinterpret_cast<const float *>(ring + static_cast<size_t>(s) * P.stage_bytes) +
                              warp * kKsRows * kKsPitch + (2 * rb) * kKsPitch + 7 * q + 3;
            float xr[kKsVr + 2][kKsCw + 2];
#pragma unroll
            for (int rr = 0; rr < kKsVr + 2; ++rr)
#pragma unroll
                for (int t = 0; t < kKsCw + 2; ++t) xr[rr][t] = xs[rr * kKsPitch + t];
            const float *wp = wt_g + ci * 72;
#pragma unroll
            for (int r = 0; r < 3; ++r) {
                float wv[3][8];
#pragma unroll
                for (int sx = 0; sx < 3; ++sx) {
                    const float4 a = *reinterpret_cast<const float4 *>(wp + (r * 3 + sx) * 8);
                    const float4 b = *reinterpret_cast<const float4 *>(wp + (r * 3 + sx) * 8 + 4);
                    wv[sx][0] = a.x, wv[sx][1] = a.y, wv[sx][2] = a.z, wv[sx][3] = a.w;
                    wv[sx][4] = b.x, wv[sx][5] = b.y, wv[sx][6] = b.z, wv[sx][7] = b.w;
                }
#pragma unroll
                for (int v = 0; v < kKsVr; ++v)
#pragma unroll
                    for (int sx = 0; sx < 3; ++sx)
#pragma unroll
                        for (int co = 0; co < 8; ++co)
#pragma unroll
                            for (int u = 0; u < kKsCw; ++u)
                                acc[co][v][u] = fmaf(xr[v + r][u + sx], wv[sx][co], acc[co][v][u]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // ---- epilogue: per output channel, the warp's 8 x W block through
        // the shared buffer, then contiguous streaming stores (the band's
        // rows of one channel are contiguous in NCHW) ----
        const int h0 = band * kKsBand;
        const int rows_valid = min(kKsBand, P.h - h0);
        const int total = rows_valid * P.wd;
        float *ybase = P.y + (static_cast<long long>(n) * P.c + (gb * P.gi + warp) * kKsCpg) * plane +
                       static_cast<long long>(h0) * P.wd;
#pragma unroll  // (acc stays in registers only with constant indices)
        for (int co = 0; co < 8; ++co) {
#pragma unroll
            for (int v = 0; v < kKsVr; ++v)
#pragma unroll
                for (int u = 0; u < kKsCw; ++u)
                    epi_g[(2 * rb + v) * kKsEpiPitch + 7 * q + u] = acc[co][v][u];
            __syncwarp();
            float *yc = ybase + co * plane;
            if (P.vec_store) {
                for (int e = 4 * lane; e < total; e += 128) {
                    const int row = e / P.wd, col = e - row * P.wd;
                    const float4 val = *reinterpret_cast<const float4 *>(epi_g + row * kKsEpiPitch + col);
                    st_stream_v4(yc + e, val.x, val.y, val.z, val.w);
                }
            } else {
                for (int e = lane; e < total; e += 32) {
                    const int row = e / P.wd, col = e - row * P.wd;
                    st_stream(yc + e, epi_g[row * kKsEpiPitch + col]);
                }
            }
            __syncwarp();
        }
    }
}

}  // namespace gcb
