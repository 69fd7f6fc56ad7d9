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
//                           time, 0 = any multiple of 4 at run time.  Runs
//                           the layers the strip kernel does not take.
//   nhwc_strip_kernel<CPG>  groups of 1, 2, 4 or 8 channels (below): a thread
//                           walks down a strip of output rows, each input
//                           row read once.
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

// Groups of 1, 2, 4 or 8 channels (channels last, 3x3/s1/p1, C % 4 == 0): a
// thread owns 4 consecutive output channels x 4 consecutive pixels of a row
// and walks down a strip of HB output rows.  Each input row of the strip is
// read ONCE (six 16-byte vectors of the channels it needs per 4-channel
// chunk) and added into the three output rows it touches, held as a ring of
// three accumulator sets, so HB output rows cost HB + 2 input rows.  Weights
// come from shared memory, staged once per persistent CTA as [tap][ci][C] so
// that a warp's lanes read consecutive 16-byte vectors (no bank conflicts).
// Depthwise layers of few pixels per channel (one-row strips) cannot amortize
// that staging: there (RW) each thread loads its own 36 weights into
// registers per item instead.  Consecutive threads take consecutive
// channel quads of the same pixels, so every load and store of a warp is
// contiguous.
struct NhwcStripParams {
    const float *x;
    const float *w;
    const float *bias;  // nullable
    float *y;
    int act;            // kActNone / kActRelu / kActRelu6, applied after the bias
    int n, c, h, wd;
    int qcols;          // ceil(wd / 4)
    int cquads;         // c / 4
    int hb;             // output rows per strip
    int hstrips;        // ceil(h / hb)
    long long items;    // n * hstrips * qcols * cquads
};

template <int CPG, bool RW>
__global__ void __launch_bounds__(128, CPG == 8 ? 3 : 4) nhwc_strip_kernel(const __grid_constant__ NhwcStripParams P) {
    constexpr int kChunks = CPG <= 2 ? 1 : CPG / 4;
    static_assert(!RW || CPG == 1, "register weights: depthwise layers only");
    extern __shared__ __align__(16) float wsm[];  // [tap][ci][C]
    griddep_wait();
    griddep_launch_dependents();
    const long long C = P.c;
    if (!RW) {
        // coalesced reads of the dense [Cout][CPG][9] weights, 8 in flight
        // per thread, each scattered to its [tap][ci][C] slot
        const int total = 9 * CPG * P.c;
        for (int e0 = threadIdx.x; e0 < total; e0 += 8 * blockDim.x) {
            float v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int e = e0 + k * blockDim.x;
                v[k] = e < total ? __ldg(P.w + e) : 0.0f;
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int e = e0 + k * blockDim.x;
                if (e < total) {
                    const int co = e / (CPG * 9), rem = e - co * (CPG * 9), ci = rem / 9, tap = rem - ci * 9;
                    wsm[(tap * CPG + ci) * P.c + co] = v[k];
                }
            }
        }
        __syncthreads();
    }
    for (long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; t < P.items;
         t += static_cast<long long>(gridDim.x) * blockDim.x) {
        long long u = t;
        const int cq = static_cast<int>(u % P.cquads);
        u /= P.cquads;
        const int qc = static_cast<int>(u % P.qcols);
        u /= P.qcols;
        const int hs = static_cast<int>(u % P.hstrips);
        const long long n = u / P.hstrips;
        const int c0 = 4 * cq, w0 = 4 * qc, h0 = hs * P.hb;
        const int h1 = min(h0 + P.hb, P.h);
        // RW: the 4 output channels' weights [j][tap] are 9 contiguous 16-byte
        // vectors, loaded per item (no staging: layers of few pixels)
        float wr[RW ? 4 * CPG * 9 : 1];
        if (RW) {
            const float4 *src = reinterpret_cast<const float4 *>(P.w + static_cast<long long>(c0) * CPG * 9);
#pragma unroll
            for (int v = 0; v < (RW ? 9 * CPG : 0); ++v) {
                const float4 q = __ldg(src + v);
                wr[4 * v] = q.x, wr[4 * v + 1] = q.y, wr[4 * v + 2] = q.z, wr[4 * v + 3] = q.w;
            }
        }
        const int xc = CPG <= 2 ? c0 : c0 - c0 % CPG;  // first input channel read per pixel
        float acc[3][4][4];  // [slot][j][pixel]; slot of output row oh = (oh - h0 + 1) mod 3
#pragma unroll
        for (int a = 0; a < 3; ++a)
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int p = 0; p < 4; ++p) acc[a][j][p] = 0.0f;
        for (int base = h0 - 1; base <= h1; base += 3) {
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                const int ih = base + k;  // slot(ih) == k
                if (ih > h1) break;
                if (ih >= 0 && ih < P.h) {
                    const float *row = P.x + ((n * P.h + ih) * P.wd) * C + xc;
#pragma unroll
                    for (int cb = 0; cb < kChunks; ++cb) {
                        float4 xin[6];
#pragma unroll
                        for (int p = 0; p < 6; ++p) {
                            const int iw = w0 + p - 1;
                            xin[p] = iw >= 0 && iw < P.wd ? ldg4(row + iw * C + 4 * cb) : make_float4(0, 0, 0, 0);
                        }
#pragma unroll
                        for (int r = 0; r < 3; ++r) {
                            // input row ih is kernel row r of output row ih + 1 - r
                            const int oh = ih + 1 - r;
                            if (oh < h0 || oh >= h1) continue;
                            float(&a)[4][4] = acc[(k + 4 - r) % 3];
#pragma unroll
                            for (int sx = 0; sx < 3; ++sx) {
#pragma unroll
                                for (int ci = 0; ci < (CPG <= 2 ? CPG : 4); ++ci) {
                                    // weights of output channels c0 .. c0+3 for input channel ci
                                    float wj[4];
                                    if (RW) {
#pragma unroll
                                        for (int j = 0; j < 4; ++j) wj[j] = wr[((j * CPG + ci) * 9 + r * 3 + sx) % (RW ? 4 * CPG * 9 : 1)];
                                    } else {
                                        const float4 wv = *reinterpret_cast<const float4 *>(
                                            wsm + ((r * 3 + sx) * CPG + 4 * cb + ci) * C + c0);
                                        wj[0] = wv.x, wj[1] = wv.y, wj[2] = wv.z, wj[3] = wv.w;
                                    }
#pragma unroll
                                    for (int j = 0; j < 4; ++j) {
                                        // element of the pixel vector output channel j reads
                                        const int e = CPG == 1 ? j : CPG == 2 ? (j / 2) * 2 + ci : ci;
#pragma unroll
                                        for (int p = 0; p < 4; ++p) a[j][p] = fmaf(f4(xin[p + sx], e), wj[j], a[j][p]);
                                    }
                                }
                            }
                        }
                    }
                }
                // output row ih - 1 has all three kernel rows now
                const int done = ih - 1;
                if (done >= h0 && done < h1) {
                    float(&a)[4][4] = acc[(k + 2) % 3];
                    const bool hb = P.bias != nullptr;
                    float bv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    if (hb)
#pragma unroll
                        for (int j = 0; j < 4; ++j) bv[j] = __ldg(P.bias + c0 + j);
                    float *out = P.y + ((n * P.h + done) * P.wd + w0) * C + c0;
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        if (w0 + p < P.wd)
                            *reinterpret_cast<float4 *>(out + p * C) =
                                make_float4(epilogue(a[0][p], hb, bv[0], P.act), epilogue(a[1][p], hb, bv[1], P.act),
                                            epilogue(a[2][p], hb, bv[2], P.act), epilogue(a[3][p], hb, bv[3], P.act));
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j)
#pragma unroll
                        for (int p = 0; p < 4; ++p) a[j][p] = 0.0f;
                }
            }
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
