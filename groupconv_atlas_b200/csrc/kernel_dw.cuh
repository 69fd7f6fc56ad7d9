// Depthwise 2-D cross-correlation (groups == Cin == Cout) for the layers the
// 3x3/s1/p1 engine does not take: strided, dilated or wider square kernels
// (K = 3, 5 or 7).  Implementation 0 routes such layers here instead of the
// general kernel (reference k0, csrc/cuda/groupconv.cu:17-37, computes the
// same sums).
//
// Work item = (image, channel, band of BH output rows).  A CTA stages the
// input rows the band reaches - (BH-1)*sh + (K-1)*dh + 1 rows, the columns
// from -pw to the last one an output touches, zero outside the image - into
// shared memory with 4-byte asynchronous copies (one warp per row, lanes on
// consecutive columns, zero fill outside the image), then every thread
// computes outputs of the band from shared memory with the channel's K*K
// weights in registers, consecutive threads on consecutive output columns
// (coalesced stores).  Two stages alternate: the copies of a CTA's next item
// are in flight while it computes the current one.  The per-output sum runs
// over (r, s) in row-major order with fused multiply-adds from zero, as the
// reference's k0 does; an optional per-channel bias and activation are
// applied after the sum.
#pragma once
#include <cstdint>

#include "device_util.cuh"

namespace gcb {

struct DwParams {
    const float *x;
    const float *w;
    float *y;
    const float *bias;           // nullable: per-channel bias added after the sum
    int act;                     // kActNone / kActRelu / kActRelu6, applied after the bias
    int n, c, h, wd;             // input
    int sh, sw, ph, pw, dh, dw;  // geometry (kernel size is the template K)
    int ho, wo;                  // output
    int bh;                      // output rows per item
    int bands;                   // ceil(ho / bh)
    int pitch;                   // staged columns from -pw: (wo-1)*sw + (K-1)*dw + 1, or
                                 // ceil(wo/4)*4 + K - 1 for stride 1 and dilation 1
    long long items;             // n * c * bands (below 2^31)
};

template <int K, bool UNIT>
__global__ void __launch_bounds__(256) dw_conv_kernel(const __grid_constant__ DwParams P) {
    extern __shared__ __align__(16) float tile[];  // two stages of stage_floats
    griddep_wait();
    griddep_launch_dependents();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    const int stage_floats = ((P.bh - 1) * P.sh + (K - 1) * P.dh + 1) * P.pitch;
    const int items = static_cast<int>(P.items);
    const long long plane_in = static_cast<long long>(P.h) * P.wd;
    const long long plane_out = static_cast<long long>(P.ho) * P.wo;
    // Issues the copies of one item's input rows into a stage (one commit group).
    auto stage = [&](int item, float *dst) {
        const int plane = item / P.bands;
        const int oh0 = (item - plane * P.bands) * P.bh;
        const int rows_in = (min(P.bh, P.ho - oh0) - 1) * P.sh + (K - 1) * P.dh + 1;
        const int ih0 = oh0 * P.sh - P.ph;
        const float *xp = P.x + plane * plane_in;
        for (int i = warp; i < rows_in; i += nwarps) {
            const int ih = ih0 + i;
            const bool row_in = ih >= 0 && ih < P.h;
            const float *xr = xp + static_cast<long long>(row_in ? ih : 0) * P.wd;
            float *tr = dst + i * P.pitch;
            for (int j = lane; j < P.pitch; j += 32) {
                const int iw = j - P.pw;
                const bool in = row_in && iw >= 0 && iw < P.wd;
                cp_async_4(tr + j, in ? xr + iw : xp, in);  // zero fill outside the image
            }
        }
        cp_async_commit();
    };
    int item = blockIdx.x;
    if (item < items) stage(item, tile);
    for (int k = 0; item < items; ++k, item += gridDim.x) {
        const int next = item + gridDim.x;
        if (next < items) stage(next, tile + ((k + 1) & 1) * stage_floats);
        if (next < items)
            cp_async_wait<1>();  // this item's copies have landed (the next item's may not)
        else
            cp_async_wait<0>();
        __syncthreads();
        const int plane = item / P.bands;
        const int c = plane % P.c;
        const int oh0 = (item - plane * P.bands) * P.bh;
        const int rows_out = min(P.bh, P.ho - oh0);
        float wr[K * K];
#pragma unroll
        for (int q = 0; q < K * K; ++q) wr[q] = __ldg(P.w + static_cast<long long>(c) * (K * K) + q);
        const bool has_bias = P.bias != nullptr;
        const float bv = has_bias ? __ldg(P.bias + c) : 0.0f;
        const float *st = tile + (k & 1) * stage_floats;
        float *yp = P.y + plane * plane_out + static_cast<long long>(oh0) * P.wo;
        if constexpr (UNIT) {
            // stride 1, dilation 1: four consecutive outputs of a row per
            // thread, one register window of 4 + K - 1 staged values per tap
            // row (the stage holds at least ceil(wo / 4) * 4 + K - 1 columns)
            const int quads = (P.wo + 3) >> 2;
            for (int g = tid; g < rows_out * quads; g += blockDim.x) {
                const int orow = g / quads, ow0 = (g - orow * quads) * 4;
                float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int r = 0; r < K; ++r) {
                    const float *row = st + (orow * P.sh + r * P.dh) * P.pitch + ow0;
                    float v[4 + K - 1];
#pragma unroll
                    for (int u = 0; u < 4 + K - 1; ++u) v[u] = row[u];
#pragma unroll
                    for (int j = 0; j < 4; ++j)
#pragma unroll
                        for (int s = 0; s < K; ++s) acc[j] = fmaf(v[j + s], wr[r * K + s], acc[j]);
                }
                float *yr = yp + static_cast<long long>(orow) * P.wo + ow0;
                if (has_bias || P.act != kActNone)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[j] = epilogue(acc[j], has_bias, bv, P.act);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (ow0 + j < P.wo) yr[j] = acc[j];
            }
        } else {
            const int outs = rows_out * P.wo;
            for (int o = tid; o < outs; o += blockDim.x) {
                const int orow = o / P.wo, ow = o - orow * P.wo;
                const float *t0 = st + orow * P.sh * P.pitch + ow * P.sw;
                float acc = 0.0f;
#pragma unroll
                for (int r = 0; r < K; ++r)
#pragma unroll
                    for (int s = 0; s < K; ++s) acc = fmaf(t0[r * P.dh * P.pitch + s * P.dw], wr[r * K + s], acc);
                yp[o] = epilogue(acc, has_bias, bv, P.act);
            }
        }
        __syncthreads();  // every thread is done with this stage before it is refilled
    }
}

}  // namespace gcb

namespace gcb {

// Depthwise KxK (K = 3 or 5), stride S (1 or 2), padding K/2, dilation 1
// (the downsampling layers of MobileNet- and EfficientNet-style networks at
// S = 2; small planes at S = 1): a thread owns a cell of 2 output rows x 4
// output columns of one plane and reads the (S+K) x (3S+K) input values it
// covers straight from global memory - per input row the 4S columns S*ow0 ..
// S*ow0+4S-1 as 16-byte loads when the row is 16-byte aligned and the cell is
// interior, and the columns either side one by one - so every input value is
// read about once and a warp's loads are contiguous.  8*K*K fused
// multiply-adds in (r, s) order per cell, 16-byte stores when the output row
// allows.  Grid-stride over cells, columns fastest.
struct DwS2Params {
    const float *x;
    const float *w;
    float *y;
    const float *bias;  // nullable: per-channel bias added after the sum
    int act;            // kActNone / kActRelu / kActRelu6, applied after the bias
    int n, c, h, wd, ho, wo;
    int qcols;        // ceil(wo / 4)
    int prows;        // ceil(ho / 2)
    long long cells;  // n * c * prows * qcols
    int vec_in;       // input rows 16-byte aligned (wd % 4 == 0, x aligned)
    int vec_out;      // output rows 16-byte aligned (wo % 4 == 0, y aligned)
};

template <int K, int S>
__global__ void __launch_bounds__(256) dw_s2_conv_kernel(const __grid_constant__ DwS2Params P) {
    constexpr int PAD = K / 2;      // padding of the layer
    constexpr int ROWS = S + K;     // input rows of a cell
    constexpr int COLS = 3 * S + K; // input columns of a cell: S*ow0 - PAD .. S*ow0 + 3S + K - 1 - PAD
    constexpr int NV = 4 * S;       // aligned middle columns, loaded 4 at a time
    griddep_wait();
    griddep_launch_dependents();
    const long long plane_in = static_cast<long long>(P.h) * P.wd;
    const long long plane_out = static_cast<long long>(P.ho) * P.wo;
    const long long per_plane = static_cast<long long>(P.prows) * P.qcols;
    for (long long cell = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; cell < P.cells;
         cell += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long plane = cell / per_plane;
        const int rest = static_cast<int>(cell - plane * per_plane);
        const int pr = rest / P.qcols, qc = rest - pr * P.qcols;
        const int oh0 = 2 * pr, ow0 = 4 * qc;
        const int c = static_cast<int>(plane % P.c);
        const float *xp = P.x + plane * plane_in;
        const int iw0 = S * ow0;      // the cell's 16-byte aligned input column
        const int col0 = iw0 - PAD;   // input column of v[.][0]
        float v[ROWS][COLS];
        const bool interior = P.vec_in && col0 >= 0 && col0 + COLS <= P.wd;
#pragma unroll
        for (int t = 0; t < ROWS; ++t) {
            const int ih = S * oh0 - PAD + t;
            const bool row_in = ih >= 0 && ih < P.h;
            const float *xr = xp + static_cast<long long>(row_in ? ih : 0) * P.wd;
            if (interior) {
#pragma unroll
                for (int q4 = 0; q4 < NV / 4; ++q4) {
                    const float4 a =
                        row_in ? __ldg(reinterpret_cast<const float4 *>(xr + iw0 + 4 * q4)) : make_float4(0, 0, 0, 0);
                    v[t][PAD + 4 * q4 + 0] = a.x;
                    v[t][PAD + 4 * q4 + 1] = a.y;
                    v[t][PAD + 4 * q4 + 2] = a.z;
                    v[t][PAD + 4 * q4 + 3] = a.w;
                }
#pragma unroll
                for (int u = 0; u < PAD; ++u) v[t][u] = row_in ? __ldg(xr + col0 + u) : 0.0f;
#pragma unroll
                for (int u = PAD + NV; u < COLS; ++u) v[t][u] = row_in ? __ldg(xr + col0 + u) : 0.0f;
            } else {
#pragma unroll
                for (int u = 0; u < COLS; ++u) {
                    const int iw = col0 + u;
                    v[t][u] = row_in && iw >= 0 && iw < P.wd ? __ldg(xr + iw) : 0.0f;
                }
            }
        }
        float wr[K * K];
#pragma unroll
        for (int q = 0; q < K * K; ++q) wr[q] = __ldg(P.w + static_cast<long long>(c) * (K * K) + q);
        float *yp = P.y + plane * plane_out;
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const int oh = oh0 + rr;
            if (oh >= P.ho) break;
            float o[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float acc = 0.0f;
#pragma unroll
                for (int r = 0; r < K; ++r)
#pragma unroll
                    for (int s = 0; s < K; ++s) acc = fmaf(v[S * rr + r][S * q + s], wr[r * K + s], acc);
                o[q] = acc;
            }
            if (P.bias != nullptr || P.act != kActNone) {
                const bool hb = P.bias != nullptr;
                const float bv = hb ? __ldg(P.bias + c) : 0.0f;
#pragma unroll
                for (int q = 0; q < 4; ++q) o[q] = epilogue(o[q], hb, bv, P.act);
            }
            float *yr = yp + static_cast<long long>(oh) * P.wo + ow0;
            if (P.vec_out && ow0 + 3 < P.wo) {
                *reinterpret_cast<float4 *>(yr) = make_float4(o[0], o[1], o[2], o[3]);
            } else {
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    if (ow0 + q < P.wo) yr[q] = o[q];
            }
        }
    }
}

}  // namespace gcb
