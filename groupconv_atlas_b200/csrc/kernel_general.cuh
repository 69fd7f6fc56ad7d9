// General grouped 2-D cross-correlation (implementation 0): any kernel size,
// stride, padding, dilation and any Cin/Cout divisible by groups.  It serves
// the geometries outside the 3x3/s1/p1 engine (strided and dilated layers,
// depthwise multipliers), so it trades peak speed for generality: a thread
// owns a run of RUN consecutive output columns of one output row, keeps one
// accumulator per column, and reuses each weight across the run.  Grid-stride
// over runs with 64-bit indices; the grid is sized from the SM count.
#pragma once
#include <cstdint>

#include "device_util.cuh"

namespace gcb {

struct GeneralParams {
    const float *xp;
    const float *wp;
    float *yp;
    long long n, cin, cout, h, w, r, s, groups, sh, sw, ph, pw, dh, dw;
    long long ho, wo;
    long long runs_per_row;  // ceil(wo / RUN)
    long long total_runs;    // n * cout * ho * runs_per_row
};

template <int RUN>
__global__ void __launch_bounds__(256) general_conv_kernel(const __grid_constant__ GeneralParams P) {
    griddep_wait();
    griddep_launch_dependents();
    const long long cpg = P.cin / P.groups;
    const long long opg = P.cout / P.groups;
    for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
         idx < P.total_runs; idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        long long t = idx;
        const long long ow0 = (t % P.runs_per_row) * RUN;
        t /= P.runs_per_row;
        const long long oh = t % P.ho;
        t /= P.ho;
        const long long co = t % P.cout;
        const long long n = t / P.cout;
        const long long ci0 = (co / opg) * cpg;
        float acc[RUN];
#pragma unroll
        for (int j = 0; j < RUN; ++j) acc[j] = 0.0f;
        const float *wco = P.wp + co * cpg * P.r * P.s;
        for (long long ci = 0; ci < cpg; ++ci) {
            const float *plane = P.xp + ((n * P.cin + ci0 + ci) * P.h) * P.w;
            for (long long r = 0; r < P.r; ++r) {
                const long long ih = oh * P.sh - P.ph + r * P.dh;
                if (ih < 0 || ih >= P.h) continue;
                const float *row = plane + ih * P.w;
                for (long long s = 0; s < P.s; ++s) {
                    const float wv = __ldg(wco + (ci * P.r + r) * P.s + s);
#pragma unroll
                    for (int j = 0; j < RUN; ++j) {
                        const long long iw = (ow0 + j) * P.sw - P.pw + s * P.dw;
                        if (iw >= 0 && iw < P.w) acc[j] = fmaf(__ldg(row + iw), wv, acc[j]);
                    }
                }
            }
        }
        float *out = P.yp + ((n * P.cout + co) * P.ho + oh) * P.wo + ow0;
#pragma unroll
        for (int j = 0; j < RUN; ++j)
            if (ow0 + j < P.wo) out[j] = acc[j];
    }
}

}  // namespace gcb
