// Grouped 2-D cross-correlation on channels-last (NHWC) tensors, with an
// optional per-output-channel bias: the layout PyTorch's channels_last memory
// format gives a 4-D tensor [N, C, H, W] (element strides H*W*C, 1, W*C, C).
// The reference times this layout only through cuDNN (its
// bench/cuda_boundaries.py:17 "torch_tuned_channels_last") and its ABI
// rejects it (csrc/common/common.cpp:48); here it is computed directly, with
// no layout conversion on either side.  Weights stay dense [Cout][cpg][R][S].
//
//   nhwc_conv_kernel<CPG>   3x3, stride 1, pad 1, Cin == Cout, C % 4 == 0,
//                           16-byte aligned x and y: a thread owns 4
//                           consecutive output channels x 4 consecutive
//                           pixels of a row; per tap row it loads the 6
//                           input pixels it needs as 16-byte vectors of 4
//                           channels (the group's channels 4 at a time for
//                           groups of 4 or more, the 4 channels of its own
//                           output quad for groups of 1 and 2), so
//                           consecutive threads read consecutive 16-byte
//                           chunks of a pixel.  CPG = 1 or 2 at compile
//                           time, 0 = any multiple of 4 at run time.
//   nhwc_scalar_kernel      any geometry (strides, dilations, kernel sizes,
//                           Cin != Cout), any alignment: one output element
//                           per thread, consecutive threads on consecutive
//                           channels of a pixel.
// Every output sums in FP32 from zero; the bias is added last, as a
// framework's convolution with bias does, then the optional activation.
#pragma once
#include "device_util.cuh"

namespace gcb {

constexpr int kNhwcPx = 4;  // pixels per thread (vector kernel)

struct NhwcParams {
    const float *x;
    const float *w;
    const float *bias;  // nullable
    float *y;
    int act;            // kActNone / kActRelu / kActRelu6, applied after the bias
    int n, c, h, wd, cpg;
    int qcols;         // ceil(wd / kNhwcPx)
    int cquads;        // c / 4
    long long cells;   // n * h * qcols * cquads
};

__device__ __forceinline__ float4 ldg4(const float *p) { return __ldg(reinterpret_cast<const float4 *>(p)); }

__device__ __forceinline__ float f4(const float4 &v, int k) {
    return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}

template <int CPG>
__global__ void __launch_bounds__(256) nhwc_conv_kernel(const __grid_constant__ NhwcParams P) {
    griddep_wait();
    griddep_launch_dependents();
    const int cpg = CPG > 0 ? CPG : P.cpg;
    const long long C = P.c;
    for (long long cell = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; cell < P.cells;
         cell += static_cast<long long>(gridDim.x) * blockDim.x) {
        long long t = cell;
        const int cq = static_cast<int>(t % P.cquads);
        t /= P.cquads;
        const int qc = static_cast<int>(t % P.qcols);
        t /= P.qcols;
        const int h = static_cast<int>(t % P.h);
        const long long n = t / P.h;
        const int c0 = 4 * cq, w0 = kNhwcPx * qc;
        // input channels read per pixel: the output quad's own 4 channels
        // (groups of 1 and 2), or the group's channels 4 at a time
        const int base = CPG == 1 || CPG == 2 ? c0 : c0 - c0 % cpg;
        const int chunks = CPG == 1 || CPG == 2 ? 1 : cpg / 4;
        float acc[4][kNhwcPx];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int p = 0; p < kNhwcPx; ++p) acc[j][p] = 0.0f;
        for (int r = 0; r < 3; ++r) {
            const int ih = h + r - 1;
            if (ih < 0 || ih >= P.h) continue;
            const float *row = P.x + (n * P.h + ih) * P.wd * C;
            for (int cb = 0; cb < chunks; ++cb) {
                float4 xin[kNhwcPx + 2];
#pragma unroll
                for (int p = 0; p < kNhwcPx + 2; ++p) {
                    const int iw = w0 + p - 1;
                    xin[p] = iw >= 0 && iw < P.wd ? ldg4(row + iw * C + base + 4 * cb) : make_float4(0, 0, 0, 0);
                }
#pragma unroll
                for (int s = 0; s < 3; ++s) {
                    if (CPG == 1) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float wv = __ldg(P.w + (c0 + j) * 9 + r * 3 + s);
#pragma unroll
                            for (int p = 0; p < kNhwcPx; ++p) acc[j][p] = fmaf(f4(xin[p + s], j), wv, acc[j][p]);
                        }
                    } else if (CPG == 2) {
#pragma unroll
                        for (int j = 0; j < 4; ++j)
#pragma unroll
                            for (int ci = 0; ci < 2; ++ci) {
                                const float wv = __ldg(P.w + ((c0 + j) * 2 + ci) * 9 + r * 3 + s);
#pragma unroll
                                for (int p = 0; p < kNhwcPx; ++p)
                                    acc[j][p] = fmaf(f4(xin[p + s], (j / 2) * 2 + ci), wv, acc[j][p]);
                            }
                    } else {
#pragma unroll
                        for (int j = 0; j < 4; ++j)
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                const float wv =
                                    __ldg(P.w + (static_cast<long long>(c0 + j) * cpg + 4 * cb + k) * 9 + r * 3 + s);
#pragma unroll
                                for (int p = 0; p < kNhwcPx; ++p) acc[j][p] = fmaf(f4(xin[p + s], k), wv, acc[j][p]);
                            }
                    }
                }
            }
        }
        float b[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (P.bias != nullptr)
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = __ldg(P.bias + c0 + j);
        float *out = P.y + ((n * P.h + h) * P.wd + w0) * C + c0;
#pragma unroll
        for (int p = 0; p < kNhwcPx; ++p) {
            if (w0 + p >= P.wd) break;
            const bool hb = P.bias != nullptr;
            const float4 v = make_float4(epilogue(acc[0][p], hb, b[0], P.act), epilogue(acc[1][p], hb, b[1], P.act),
                                         epilogue(acc[2][p], hb, b[2], P.act), epilogue(acc[3][p], hb, b[3], P.act));
            *reinterpret_cast<float4 *>(out + p * C) = v;
        }
    }
}

struct NhwcScalarParams {
    const float *x;
    const float *wt;    // weights
    const float *bias;  // nullable
    float *y;
    int act;            // kActNone / kActRelu / kActRelu6, applied after the bias
    long long n, cin, cout, h, w, r, s, groups, sh, sw, ph, pw, dh, dw, ho, wo;
    long long total;    // n * ho * wo * cout
};

__global__ void __launch_bounds__(256) nhwc_scalar_kernel(const __grid_constant__ NhwcScalarParams P) {
    griddep_wait();
    griddep_launch_dependents();
    const long long cpg = P.cin / P.groups, opg = P.cout / P.groups;
    for (long long o = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; o < P.total;
         o += static_cast<long long>(gridDim.x) * blockDim.x) {
        long long t = o;
        const long long co = t % P.cout;
        t /= P.cout;
        const long long ow = t % P.wo;
        t /= P.wo;
        const long long oh = t % P.ho;
        const long long n = t / P.ho;
        const long long ci0 = (co / opg) * cpg;
        float acc = 0.0f;
        for (long long ci = 0; ci < cpg; ++ci)
            for (long long r = 0; r < P.r; ++r) {
                const long long ih = oh * P.sh - P.ph + r * P.dh;
                if (ih < 0 || ih >= P.h) continue;
                for (long long s = 0; s < P.s; ++s) {
                    const long long iw = ow * P.sw - P.pw + s * P.dw;
                    if (iw < 0 || iw >= P.w) continue;
                    acc = fmaf(__ldg(P.x + ((n * P.h + ih) * P.w + iw) * P.cin + ci0 + ci),
                               __ldg(P.wt + ((co * cpg + ci) * P.r + r) * P.s + s), acc);
                }
            }
        const bool hb = P.bias != nullptr;
        P.y[o] = epilogue(acc, hb, hb ? __ldg(P.bias + co) : 0.0f, P.act);
    }
}

}  // namespace gcb
