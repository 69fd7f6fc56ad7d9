// Direct FP32 grouped 3x3 convolution (stride 1, pad 1, dilation 1,
// Cin == Cout), the engine behind implementations 1-3 of gc_cuda_conv.
//
// Work item = (image n, block of `cb` channels made of whole groups, band of
// `bh` output rows).  A persistent CTA walks items blockIdx.x, +gridDim.x, ...
// through a STAGES-deep ring of shared-memory stages.  A stage holds
//   - the input band of every channel of the item, rows h0-1 .. h0+bh
//     (rounded up to the row blocking), `pitch` floats per row with the image
//     columns at [4, 4+W) and zeros around them, so the conv's zero padding
//     needs no branches;
//   - the item's raw weights [cb][cpg][3][3].
// Staging is either one TMA tensor load (box starting at column -4 and row
// h0-1; the copy engine zero-fills every out-of-image element) plus one bulk
// copy of the weights, completion tracked by an mbarrier with a bounded
// wait, or per-thread cp.async copies with zero-fill (any width/alignment).
//
// Compute: thread cell = COB output channels x VR rows x 4 columns.  For each
// input channel the cell reads VR+2 rows of 6 values (one 16-byte and two
// 4-byte shared loads per row) and reuses every loaded value across all
// taps, rows and output channels of the cell; weights are warp-broadcast
// shared loads from a per-item transposed copy [group][ci][tap][co].
// Outputs leave registers as streaming 16-byte stores when rows are aligned.
#pragma once
#include "device_util.cuh"

namespace gcb {

struct DirectParams {
    const float *x;
    const float *w;
    float *y;
    int n, c, h, wd;     // batch, channels, height, width
    int cpg;             // channels per group (input == output)
    int cb;              // channels per work item (whole groups)
    int bh;              // output rows per item
    int bands, cblocks;  // ceil(h / bh), c / cb
    long long items;     // n * cblocks * bands
    int pitch;           // shared row pitch in floats, multiple of 4, >= wd + 8
    int rows;            // tile rows: round_up(bh, VR) + 2
    int x_floats;        // input tile floats per stage (multiple of 32)
    int wraw_floats;     // raw weight floats per stage (multiple of 32)
    int stage_floats;    // x_floats + wraw_floats
    int wt_floats;       // transposed weight floats (0 when cpg == 1)
    int qcols;           // ceil(wd / 4)
    int rblocks;         // ceil(bh / VR)
    int cells;           // (cb / COB) * rblocks * qcols
    int vec_store;       // 16-byte output stores allowed
    int bulk_w;          // TMA staging: weights by bulk copy (else plain loads)
    unsigned x_bytes;    // bytes one TMA box delivers
    unsigned w_bytes;    // raw weight bytes per item
};

template <int CPG, int COB, int VR>
struct DirectCell {
    // Accumulates one cell.  xs: this item's input tile; wsrc: transposed
    // weights (or raw weights when cpg == 1).
    static __device__ __forceinline__ void run(const DirectParams &P, const float *xs,
                                               const float *wraw, const float *wt, int cell,
                                               int n, int c0, int h0) {
        const int cpg = CPG > 0 ? CPG : P.cpg;
        const int q = cell % P.qcols;
        const int t = cell / P.qcols;
        const int rb = t % P.rblocks;
        const int cob = t / P.rblocks;
        const int col0 = q * 4;
        const int row0 = rb * VR;
        const int co_item = cob * COB;  // first output channel of the cell, item-local
        const int g = co_item / cpg;    // item-local group
        const int cog = co_item - g * cpg;

        float acc[COB][VR][4];
#pragma unroll
        for (int j = 0; j < COB; ++j)
#pragma unroll
            for (int v = 0; v < VR; ++v)
#pragma unroll
                for (int u = 0; u < 4; ++u) acc[j][v][u] = 0.0f;

        const int chan_floats = P.rows * P.pitch;
        const float *xg = xs + (g * cpg) * chan_floats + row0 * P.pitch + col0 + 3;
#pragma unroll(CPG > 0 ? CPG : 1)
        for (int ci = 0; ci < cpg; ++ci) {
            const float *xc = xg + ci * chan_floats;
            float xr[VR + 2][6];
#pragma unroll
            for (int rr = 0; rr < VR + 2; ++rr) {
                const float *p = xc + rr * P.pitch;
                xr[rr][0] = p[0];
                const float4 m = *reinterpret_cast<const float4 *>(p + 1);
                xr[rr][1] = m.x;
                xr[rr][2] = m.y;
                xr[rr][3] = m.z;
                xr[rr][4] = m.w;
                xr[rr][5] = p[5];
            }
            const float *wp = CPG == 1 ? wraw + co_item * 9
                                       : wt + ((g * cpg + ci) * 9) * cpg + cog;
#pragma unroll
            for (int tap = 0; tap < 9; ++tap) {
                const int r = tap / 3, s = tap % 3;
                float wv[COB];
                if (CPG == 1) {
                    wv[0] = wp[tap];
                } else if (COB % 4 == 0) {
#pragma unroll
                    for (int j = 0; j < COB; j += 4) {
                        const float4 m = *reinterpret_cast<const float4 *>(wp + tap * cpg + j);
                        wv[j] = m.x;
                        wv[j + 1] = m.y;
                        wv[j + 2] = m.z;
                        wv[j + 3] = m.w;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < COB; ++j) wv[j] = wp[tap * cpg + j];
                }
#pragma unroll
                for (int j = 0; j < COB; ++j)
#pragma unroll
                    for (int v = 0; v < VR; ++v)
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            acc[j][v][u] = fmaf(xr[v + r][u + s], wv[j], acc[j][v][u]);
            }
        }

        const long long plane0 = static_cast<long long>(n) * P.c + c0 + co_item;
#pragma unroll
        for (int j = 0; j < COB; ++j)
#pragma unroll
            for (int v = 0; v < VR; ++v) {
                const int oh = h0 + row0 + v;
                if (row0 + v >= P.bh || oh >= P.h) continue;
                float *yp = P.y + ((plane0 + j) * P.h + oh) * static_cast<long long>(P.wd) + col0;
                if (P.vec_store && col0 + 4 <= P.wd) {
                    st_stream_v4(yp, acc[j][v][0], acc[j][v][1], acc[j][v][2], acc[j][v][3]);
                } else {
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        if (col0 + u < P.wd) st_stream(yp + u, acc[j][v][u]);
                }
            }
    }
};

__device__ __forceinline__ void decode_item(const DirectParams &P, long long item, int &n,
                                            int &c0, int &h0) {
    const int band = static_cast<int>(item % P.bands);
    const long long t = item / P.bands;
    const int cblk = static_cast<int>(t % P.cblocks);
    n = static_cast<int>(t / P.cblocks);
    c0 = cblk * P.cb;
    h0 = band * P.bh;
}

// Per-thread asynchronous staging of one item (any width, any alignment).
__device__ __forceinline__ void stage_with_cp_async(const DirectParams &P, float *xs, float *wr,
                                                    long long item) {
    int n, c0, h0;
    decode_item(P, item, n, c0, h0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    const int tile_rows = P.cb * P.rows;
    for (int rowid = warp; rowid < tile_rows; rowid += nwarps) {
        const int cl = rowid / P.rows;
        const int ih = h0 - 1 + (rowid - cl * P.rows);
        const bool row_ok = ih >= 0 && ih < P.h;
        const float *src =
            P.x + ((static_cast<long long>(n) * P.c + c0 + cl) * P.h + (row_ok ? ih : 0)) *
                      static_cast<long long>(P.wd);
        float *dst = xs + rowid * P.pitch;
        for (int j = lane; j < P.pitch; j += 32) {
            const int iw = j - 4;
            const bool ok = row_ok && iw >= 0 && iw < P.wd;
            cp_async_4(dst + j, ok ? src + iw : P.x, ok);
        }
    }
    const int wcount = P.cb * P.cpg * 9;
    const float *wsrc = P.w + static_cast<long long>(c0) * P.cpg * 9;
    for (int e = threadIdx.x; e < wcount; e += blockDim.x) cp_async_4(wr + e, wsrc + e, true);
}

// One elected thread issues the TMA staging of one item into a stage.
__device__ __forceinline__ void stage_with_tma(const DirectParams &P, const CUtensorMap *xmap,
                                               float *xs, float *wr, uint64_t *bar,
                                               long long item) {
    int n, c0, h0;
    decode_item(P, item, n, c0, h0);
    mbar_arrive_expect_tx(bar, P.x_bytes + (P.bulk_w ? P.w_bytes : 0u));
    tma_load_4d(xs, xmap, -4, h0 - 1, c0, n, bar);
    if (P.bulk_w) bulk_load(wr, P.w + static_cast<long long>(c0) * P.cpg * 9, P.w_bytes, bar);
}

template <int CPG, int COB, int VR, bool TMA, int STAGES>
__global__ void __launch_bounds__(256) direct_conv_kernel(const __grid_constant__ DirectParams P,
                                                          const __grid_constant__ CUtensorMap xmap) {
    extern __shared__ __align__(128) float smem[];
    const int cpg = CPG > 0 ? CPG : P.cpg;
    float *wt = smem + STAGES * P.stage_floats;
    uint64_t *bars = reinterpret_cast<uint64_t *>(wt + P.wt_floats);
    const long long first = blockIdx.x, step = gridDim.x;
    const long long count = first < P.items ? (P.items - 1 - first) / step + 1 : 0;
    const int tid = threadIdx.x;

    if (TMA) {
        if (tid == 0) {
            for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 1);
            fence_barrier_init();
            prefetch_tensormap(&xmap);
        }
        __syncthreads();
        if (tid == 0)
            for (int s = 0; s < STAGES && s < count; ++s)
                stage_with_tma(P, &xmap, smem + s * P.stage_floats,
                               smem + s * P.stage_floats + P.x_floats, &bars[s], first + s * step);
    } else {
        for (int s = 0; s < STAGES - 1; ++s) {
            if (s < count)
                stage_with_cp_async(P, smem + s * P.stage_floats,
                                    smem + s * P.stage_floats + P.x_floats, first + s * step);
            cp_async_commit();
        }
    }

    for (long long k = 0; k < count; ++k) {
        const int s = static_cast<int>(k % STAGES);
        const long long item = first + k * step;
        float *xs = smem + s * P.stage_floats;
        float *wr = xs + P.x_floats;
        if (TMA) {
            const bool ok = mbar_wait_bounded(&bars[s], static_cast<uint32_t>((k / STAGES) & 1));
            if (!__syncthreads_and(ok)) {
                // The copy engine did not deliver in time: record it, let the
                // loads still in flight land (bounded), and leave.
                if (tid == 0) {
                    raise_status(kStatusTmaTimeout);
                    for (long long j = k + 1; j < k + STAGES && j < count; ++j)
                        mbar_wait_bounded(&bars[j % STAGES], static_cast<uint32_t>((j / STAGES) & 1));
                }
                return;
            }
            if (!P.bulk_w) {
                int n, c0, h0;
                decode_item(P, item, n, c0, h0);
                const float *wsrc = P.w + static_cast<long long>(c0) * cpg * 9;
                for (int e = tid; e < P.cb * cpg * 9; e += blockDim.x) wr[e] = __ldg(wsrc + e);
                __syncthreads();
            }
        } else {
            const long long kn = k + STAGES - 1;
            if (kn < count)
                stage_with_cp_async(P, smem + (kn % STAGES) * P.stage_floats,
                                    smem + (kn % STAGES) * P.stage_floats + P.x_floats,
                                    first + kn * step);
            cp_async_commit();
            cp_async_wait<STAGES - 1>();
            __syncthreads();
        }
        if (CPG != 1) {
            // raw [co][ci][tap] -> [group][ci][tap][co-in-group]
            const int per_co = cpg * 9;
            for (int e = tid; e < P.cb * per_co; e += blockDim.x) {
                const int co = e / per_co;
                const int rem = e - co * per_co;
                const int g = co / cpg;
                wt[(g * cpg * 9 + rem) * cpg + (co - g * cpg)] = wr[e];
            }
            __syncthreads();
        }
        int n, c0, h0;
        decode_item(P, item, n, c0, h0);
        for (int cell = tid; cell < P.cells; cell += blockDim.x)
            DirectCell<CPG, COB, VR>::run(P, xs, wr, wt, cell, n, c0, h0);
        __syncthreads();
        if (TMA && tid == 0 && k + STAGES < count)
            stage_with_tma(P, &xmap, xs, wr, &bars[s], first + (k + STAGES) * step);
    }
    if (!TMA) cp_async_wait<0>();
}

}  // namespace gcb
