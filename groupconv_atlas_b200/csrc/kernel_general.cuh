// General grouped 2-D cross-correlation (implementation 0): any kernel size,
// stride, padding, dilation and any Cin/Cout divisible by groups.  It serves
// the geometries outside the 3x3/s1/p1 engine (strided and dilated layers,
// Cin != Cout, depthwise multipliers), so it trades peak speed for
// generality: a thread owns a run of RUN consecutive output columns of one
// output row for COB consecutive output channels of one group (COB divides
// the output channels per group), keeps COB x RUN accumulators, and reuses
// each input value across the COB channels and each weight across the run.
// Consecutive threads take consecutive runs of a row, so input loads are
// coalesced (at the layer's stride) and the threads of a warp share weights
// (L1 broadcast).  Grid-stride over runs; index arithmetic in 32 bits when
// every tensor has fewer than 2^31 elements, else 64 bits.  An optional
// per-output-channel bias and activation are applied after the sum.
#pragma once
#include <cstdint>

#include "device_util.cuh"

namespace gcb {

struct GeneralParams {
    const float *xp;
    const float *wp;
    float *yp;
    const float *bias;  // nullable: per-output-channel bias added after the sum
    int act;            // kActNone / kActRelu / kActRelu6, applied after the bias
    long long n, cin, cout, h, w, r, s, groups, sh, sw, ph, pw, dh, dw;
    long long ho, wo;
    long long runs_per_row;  // ceil(wo / RUN)
    long long total_runs;    // n * (cout / COB) * ho * runs_per_row
};

template <int RUN, int COB, typename I>
__global__ void __launch_bounds__(256) general_conv_kernel(const __grid_constant__ GeneralParams P) {
    griddep_wait();
    griddep_launch_dependents();
    const I cpg = static_cast<I>(P.cin / P.groups);
    const I opg = static_cast<I>(P.cout / P.groups);
    const I R = static_cast<I>(P.r), S = static_cast<I>(P.s);
    const I H = static_cast<I>(P.h), W = static_cast<I>(P.w), HO = static_cast<I>(P.ho), WO = static_cast<I>(P.wo);
    const I sh = static_cast<I>(P.sh), sw = static_cast<I>(P.sw), ph = static_cast<I>(P.ph), pw = static_cast<I>(P.pw);
    const I dh = static_cast<I>(P.dh), dw = static_cast<I>(P.dw);
    const I rpr = static_cast<I>(P.runs_per_row), cobs = static_cast<I>(P.cout / COB);
    const I total = static_cast<I>(P.total_runs);
    const I wsize = cpg * R * S;  // weights per output channel
    for (I idx = static_cast<I>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
         idx += static_cast<I>(gridDim.x) * blockDim.x) {
        I t = idx;
        const I ow0 = (t % rpr) * RUN;
        t /= rpr;
        const I oh = t % HO;
        t /= HO;
        const I co0 = (t % cobs) * COB;
        const I n = t / cobs;
        const I ci0 = (co0 / opg) * cpg;
        float acc[COB][RUN];
#pragma unroll
        for (int c = 0; c < COB; ++c)
#pragma unroll
            for (int j = 0; j < RUN; ++j) acc[c][j] = 0.0f;
        const float *wco = P.wp + co0 * wsize;
        const I iw0 = ow0 * sw - pw;
        for (I ci = 0; ci < cpg; ++ci) {
            const float *plane = P.xp + ((n * static_cast<I>(P.cin) + ci0 + ci) * H) * W;
            const float *wci = wco + ci * R * S;
            for (I r = 0; r < R; ++r) {
                const I ih = oh * sh - ph + r * dh;
                if (ih < 0 || ih >= H) continue;
                const float *row = plane + ih * W;
                for (I s = 0; s < S; ++s) {
                    float xv[RUN];
#pragma unroll
                    for (int j = 0; j < RUN; ++j) {
                        const I iw = iw0 + j * sw + s * dw;
                        xv[j] = (iw >= 0 && iw < W) ? __ldg(row + iw) : 0.0f;
                    }
#pragma unroll
                    for (int c = 0; c < COB; ++c) {
                        const float wv = __ldg(wci + c * wsize + r * S + s);
#pragma unroll
                        for (int j = 0; j < RUN; ++j) acc[c][j] = fmaf(xv[j], wv, acc[c][j]);
                    }
                }
            }
        }
        float *out = P.yp + ((n * static_cast<I>(P.cout) + co0) * HO + oh) * WO + ow0;
        if (P.bias != nullptr || P.act != kActNone)
#pragma unroll
            for (int c = 0; c < COB; ++c) {
                const bool hb = P.bias != nullptr;
                const float b = hb ? __ldg(P.bias + co0 + c) : 0.0f;
#pragma unroll
                for (int j = 0; j < RUN; ++j) acc[c][j] = epilogue(acc[c][j], hb, b, P.act);
            }
#pragma unroll
        for (int c = 0; c < COB; ++c)
#pragma unroll
            for (int j = 0; j < RUN; ++j)
                if (ow0 + j < WO) out[c * HO * WO + j] = acc[c][j];
    }
}

}  // namespace gcb
