// Direct FP32 grouped 3x3 convolution for wide groups (16 or more channels
// per group, or any group too large for the full-group tiles of
// kernel_direct.cuh).  Same B geometry and numerics (FP32 FMA), but the
// input channels of a group are streamed through shared memory in chunks of
// `kc` channels while every thread keeps its cell's accumulators in
// registers across the chunks - a K loop, as in a GEMM.
//
// Work item = (image, group, band of `bh` rows, block of `co_item` output
// channels); pipeline step = (item, input-channel chunk).  Item order puts the
// output-channel blocks of one band next to each other so that the CTAs
// re-reading that band find it in L2.  Each thread owns at most one cell
// (COB output channels x VR rows x 4 columns), so cells <= blockDim.
// Weights are read with warp-uniform read-only loads.
#pragma once
#include "device_util.cuh"

namespace gcb {

struct WideParams {
    const float *x;
    const float *w;
    float *y;
    int n, c, h, wd, cpg, groups;
    int kc, chunks;            // input channels per chunk, chunks per item
    int co_item, coblocks;     // output channels per item, ceil(cpg / co_item)
    int bh, bands;             // output rows per item, ceil(h / bh)
    long long items;           // n * groups * bands * coblocks
    int pitch, rows;           // shared row pitch (floats), tile rows
    int x_floats;              // floats per stage (multiple of 32)
    int qcols, rblocks, cells; // cell grid of one item (cells <= blockDim)
    int vec_store;
    unsigned x_bytes;          // bytes one TMA box delivers
};

__device__ __forceinline__ void wide_decode(const WideParams &P, long long item, int &n, int &g,
                                            int &h0, int &co0) {
    const int cob = static_cast<int>(item % P.coblocks);
    long long t = item / P.coblocks;
    const int band = static_cast<int>(t % P.bands);
    t /= P.bands;
    g = static_cast<int>(t % P.groups);
    n = static_cast<int>(t / P.groups);
    h0 = band * P.bh;
    co0 = cob * P.co_item;
}

__device__ __forceinline__ void wide_stage_cp_async(const WideParams &P, float *xs, long long item,
                                                    int chunk) {
    int n, g, h0, co0;
    wide_decode(P, item, n, g, h0, co0);
    const int cfirst = g * P.cpg + chunk * P.kc;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    for (int rowid = warp; rowid < P.kc * P.rows; rowid += nwarps) {
        const int cl = rowid / P.rows;
        const int ih = h0 - 1 + (rowid - cl * P.rows);
        const int ch = cfirst + cl;
        const bool row_ok = ih >= 0 && ih < P.h && ch < P.c;
        const float *src = P.x + ((static_cast<long long>(n) * P.c + (row_ok ? ch : 0)) * P.h +
                                  (row_ok ? ih : 0)) *
                                     static_cast<long long>(P.wd);
        float *dst = xs + rowid * P.pitch;
        for (int j = lane; j < P.pitch; j += 32) {
            const int iw = j - 4;
            const bool ok = row_ok && iw >= 0 && iw < P.wd;
            cp_async_4(dst + j, ok ? src + iw : P.x, ok);
        }
    }
}

__device__ __forceinline__ void wide_stage_tma(const WideParams &P, const CUtensorMap *xmap,
                                               float *xs, uint64_t *bar, long long item, int chunk) {
    int n, g, h0, co0;
    wide_decode(P, item, n, g, h0, co0);
    mbar_arrive_expect_tx(bar, P.x_bytes);
    tma_load_4d(xs, xmap, -4, h0 - 1, g * P.cpg + chunk * P.kc, n, bar);
}

template <int COB, int VR, bool TMA, int STAGES>
__global__ void __launch_bounds__(256) wide_conv_kernel(const __grid_constant__ WideParams P,
                                                        const __grid_constant__ CUtensorMap xmap) {
    extern __shared__ __align__(128) float smem[];
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * P.x_floats);
    const long long first = blockIdx.x, step = gridDim.x;
    const long long my_items = first < P.items ? (P.items - 1 - first) / step + 1 : 0;
    const long long count = my_items * P.chunks;
    const int tid = threadIdx.x;

    // This thread's cell (if any) within every item.
    const bool has_cell = tid < P.cells;
    const int q = tid % P.qcols;
    const int rb = (tid / P.qcols) % P.rblocks;
    const int cob = tid / (P.qcols * P.rblocks);
    const int col0 = q * 4, row0 = rb * VR;

    if (TMA && tid == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 1);
        fence_barrier_init();
        prefetch_tensormap(&xmap);
    }
    griddep_wait();
    griddep_launch_dependents();
    if (TMA) {
        __syncthreads();
        if (tid == 0)
            for (int s = 0; s < STAGES && s < count; ++s)
                wide_stage_tma(P, &xmap, smem + s * P.x_floats, &bars[s],
                               first + (s / P.chunks) * step, s % P.chunks);
    } else {
        for (int s = 0; s < STAGES - 1; ++s) {
            if (s < count)
                wide_stage_cp_async(P, smem + s * P.x_floats, first + (s / P.chunks) * step,
                                    s % P.chunks);
            cp_async_commit();
        }
    }

    float acc[COB][VR][4];
    for (long long k = 0; k < count; ++k) {
        const int s = static_cast<int>(k % STAGES);
        const int chunk = static_cast<int>(k % P.chunks);
        const long long item = first + (k / P.chunks) * step;
        float *xs = smem + s * P.x_floats;
        if (TMA) {
            bool ok = true;
            if (tid == 0) ok = mbar_wait_bounded(&bars[s], static_cast<uint32_t>((k / STAGES) & 1));
            if (!__syncthreads_and(ok)) {
                if (tid == 0) {
                    raise_status(kStatusTmaTimeout);
                    for (long long j = k + 1; j < k + STAGES && j < count; ++j)
                        mbar_wait_bounded(&bars[j % STAGES], static_cast<uint32_t>((j / STAGES) & 1));
                }
                return;
            }
        } else {
            const long long kn = k + STAGES - 1;
            if (kn < count)
                wide_stage_cp_async(P, smem + (kn % STAGES) * P.x_floats,
                                    first + (kn / P.chunks) * step, static_cast<int>(kn % P.chunks));
            cp_async_commit();
            cp_async_wait<STAGES - 1>();
            __syncthreads();
        }
        if (chunk == 0) {
#pragma unroll
            for (int j = 0; j < COB; ++j)
#pragma unroll
                for (int v = 0; v < VR; ++v)
#pragma unroll
                    for (int u = 0; u < 4; ++u) acc[j][v][u] = 0.0f;
        }
        int n, g, h0, co0;
        wide_decode(P, item, n, g, h0, co0);
        const int co_first = co0 + cob * COB;  // group-local output channel of the cell
        if (has_cell && co_first < P.cpg) {
            const int kc_eff = min(P.kc, P.cpg - chunk * P.kc);
            const int chan_floats = P.rows * P.pitch;
            const float *xb = xs + row0 * P.pitch + col0 + 3;
            // weights [co][ci][tap] of this cell, at ci = chunk*kc
            const float *wb = P.w + (static_cast<long long>(g) * P.cpg + co_first) * P.cpg * 9 +
                              static_cast<long long>(chunk) * P.kc * 9;
            const int wco = P.cpg * 9;
            for (int ci = 0; ci < kc_eff; ++ci) {
                const float *xc = xb + ci * chan_floats;
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
                const float *wc = wb + ci * 9;
#pragma unroll
                for (int tap = 0; tap < 9; ++tap) {
                    const int r = tap / 3, sx = tap % 3;
                    float wv[COB];
#pragma unroll
                    for (int j = 0; j < COB; ++j)
                        wv[j] = (co_first + j < P.cpg) ? __ldg(wc + j * wco + tap) : 0.0f;
#pragma unroll
                    for (int j = 0; j < COB; ++j)
#pragma unroll
                        for (int v = 0; v < VR; ++v)
#pragma unroll
                            for (int u = 0; u < 4; ++u)
                                acc[j][v][u] = fmaf(xr[v + r][u + sx], wv[j], acc[j][v][u]);
                }
            }
            if (chunk == P.chunks - 1) {
                const long long plane0 = static_cast<long long>(n) * P.c + g * P.cpg + co_first;
#pragma unroll
                for (int j = 0; j < COB; ++j) {
                    if (co_first + j >= P.cpg) break;
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
            }
        }
        __syncthreads();
        if (TMA && tid == 0 && k + STAGES < count) {
            const long long kn = k + STAGES;
            wide_stage_tma(P, &xmap, xs, &bars[s], first + (kn / P.chunks) * step,
                           static_cast<int>(kn % P.chunks));
        }
    }
    if (!TMA) cp_async_wait<0>();
}

}  // namespace gcb
