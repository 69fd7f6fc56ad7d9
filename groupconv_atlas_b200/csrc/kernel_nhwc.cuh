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
//                           the 3x3/s1/p1 layers the kernels below do not
//                           take (other group widths, larger weights).
//   nhwc_dw_tma_kernel<CPG> groups of 1 and 2 channels (below): TMA-staged
//                           tiles of 32 channels, double-buffered.
//   nhwc_grp_tma_kernel<CPG,NC> groups of 4 and 8 channels (below): the
//                           same tiles, one output channel x NC columns per
//                           thread.
//   nhwc_strip_kernel<CPG>  groups of 1, 2, 4 or 8 channels whose weights or
//                           bias are not 16-byte aligned (below):
//                           a thread walks down a strip of output rows, each
//                           input row read once.
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
// (Groups of 1 and 2 channels take this kernel only where the TMA-staged one
// below cannot run: unaligned weights or bias.)  Consecutive threads take consecutive
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

template <int CPG>
__global__ void __launch_bounds__(128, CPG == 8 ? 3 : 4) nhwc_strip_kernel(const __grid_constant__ NhwcStripParams P) {
    constexpr int kChunks = CPG <= 2 ? 1 : CPG / 4;
    extern __shared__ __align__(16) float wsm[];  // [tap][ci][C]
    griddep_wait();
    griddep_launch_dependents();
    const long long C = P.c;
    {
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
                                    const float4 wv = *reinterpret_cast<const float4 *>(
                                        wsm + ((r * 3 + sx) * CPG + 4 * cb + ci) * C + c0);
                                    const float wj[4] = {wv.x, wv.y, wv.z, wv.w};
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

// Depthwise (CPG 1) and 2-channel-group (CPG 2) 3x3/s1/p1 layers on
// channels-last tensors with TMA staging: a work item
// is a tile of TH output rows x TW output columns x 32 channels of one image;
// one elected thread loads the tile's input box (32 channels x TW+2 columns x
// TH+2 rows, starting at column and row -1) with one 4-D TMA copy, whose
// out-of-range elements (the zero padding, and channels past C) read as zero.
// Two stages alternate: the box of the CTA's next item is in flight while the
// current one is computed.  Thread t owns channels 4 (t % 8) .. +3 of the
// block and output column t / 8: it walks down the TH rows with a window of
// 3 x 3 16-byte vectors (three new shared loads per row; a warp's loads are 4
// columns x 128 contiguous bytes, no bank conflicts), its 36 CPG weights in
// registers (a quad of channels holds whole groups, so its inputs are its own
// 4 channels), and writes one 16-byte streaming store per row.
struct NhwcDwTmaParams {
    const float *w;
    const float *bias;  // nullable
    float *y;
    int act;
    int n, c, h, wd;
    int tw, th;          // output columns / rows per tile (tw <= 32, th <= 8)
    int wtiles, htiles;  // ceil(wd / tw), ceil(h / th)
    int cblocks;         // ceil(c / 32)
    int items;           // n * htiles * wtiles * cblocks
    unsigned box_bytes;  // 32 * (tw + 2) * (th + 2) * 4
};

constexpr int kDwTmaCB = 32;  // channels per tile
constexpr int kDwTmaMaxTH = 8;

__device__ __forceinline__ void dw_tma_decode(const NhwcDwTmaParams &P, int item, int &n, int &h0, int &w0, int &c0) {
    int t = item;
    const int cb = t % P.cblocks;
    t /= P.cblocks;
    const int wt = t % P.wtiles;
    t /= P.wtiles;
    const int ht = t % P.htiles;
    n = t / P.htiles;
    h0 = ht * P.th;
    w0 = wt * P.tw;
    c0 = cb * kDwTmaCB;
}

template <int CPG>
__global__ void __launch_bounds__(256) nhwc_dw_tma_kernel(const __grid_constant__ NhwcDwTmaParams P,
                                                          const __grid_constant__ CUtensorMap xmap) {
    extern __shared__ __align__(128) unsigned char dsm[];
    float *const stage0 = reinterpret_cast<float *>(dsm);
    uint64_t *const full = reinterpret_cast<uint64_t *>(dsm + 2 * P.box_bytes);
    const int tid = threadIdx.x;
    const int q = tid & 7, col = tid >> 3;  // channel quad, output column of the tile
    const int first = blockIdx.x, stride = gridDim.x;
    if (tid == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        fence_barrier_init();
    }
    __syncthreads();
    griddep_wait();
    griddep_launch_dependents();
    auto issue = [&](int item, int s) {
        int n, h0, w0, c0;
        dw_tma_decode(P, item, n, h0, w0, c0);
        mbar_arrive_expect_tx(&full[s], P.box_bytes);
        tma_load_4d(reinterpret_cast<unsigned char *>(stage0) + s * P.box_bytes, &xmap, c0, w0 - 1, h0 - 1, n,
                    &full[s]);
    };
    if (tid == 0 && first < P.items) {
        prefetch_tensormap(&xmap);
        issue(first, 0);
    }
    const int bw = P.tw + 2;  // box columns
    const long long C = P.c;
    int it = 0;
    for (int item = first; item < P.items; item += stride, ++it) {
        const int s = it & 1;
        // the next item's box goes to the other stage, free since the
        // barrier at the end of the previous iteration
        if (tid == 0 && item + stride < P.items) issue(item + stride, s ^ 1);
        const bool ok = mbar_wait_bounded(&full[s], static_cast<uint32_t>((it >> 1) & 1));
        if (!__syncthreads_and(ok)) {
            if (tid == 0) {
                raise_status(kStatusTmaTimeout);
                // the other stage's copy may still be landing: wait for it
                if (item + stride < P.items)
                    mbar_wait_bounded(&full[s ^ 1], static_cast<uint32_t>(((it + 1) >> 1) & 1));
            }
            return;
        }
        int n, h0, w0, c0;
        dw_tma_decode(P, item, n, h0, w0, c0);
        const int c = c0 + 4 * q;
        const bool active = col < P.tw && w0 + col < P.wd && c < P.c;
        if (active) {
            // weights [j][ci][tap] of output channels c .. c+3: 9 CPG
            // contiguous 16-byte vectors
            float4 wt[9 * CPG];
            const float4 *wsrc = reinterpret_cast<const float4 *>(P.w + static_cast<long long>(c) * CPG * 9);
#pragma unroll
            for (int v = 0; v < 9 * CPG; ++v) wt[v] = __ldg(wsrc + v);
            auto wk = [&](int j, int ci, int k) -> float {
                const int e = (j * CPG + ci) * 9 + k;
                return f4(wt[e >> 2], e & 3);
            };
            float4 b = make_float4(0, 0, 0, 0);
            const bool hb = P.bias != nullptr;
            if (hb) b = __ldg(reinterpret_cast<const float4 *>(P.bias + c));
            const float *st = stage0 + s * (P.box_bytes / 4) + col * kDwTmaCB + 4 * q;
            float4 win[3][3];  // [row of the window][tap column]
#pragma unroll
            for (int rr = 0; rr < 2; ++rr)
#pragma unroll
                for (int sx = 0; sx < 3; ++sx)
                    win[rr][sx] = *reinterpret_cast<const float4 *>(st + (rr * bw + sx) * kDwTmaCB);
            float *yrow = P.y + ((static_cast<long long>(n) * P.h + h0) * P.wd + w0 + col) * C + c;
#pragma unroll
            for (int r = 0; r < kDwTmaMaxTH; ++r) {
                if (r >= P.th || h0 + r >= P.h) break;
#pragma unroll
                for (int sx = 0; sx < 3; ++sx)
                    win[(r + 2) % 3][sx] =
                        *reinterpret_cast<const float4 *>(st + ((r + 2) * bw + sx) * kDwTmaCB);
                float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int ky = 0; ky < 3; ++ky)
#pragma unroll
                    for (int sx = 0; sx < 3; ++sx) {
                        const float4 xv = win[(r + ky) % 3][sx];
#pragma unroll
                        for (int j = 0; j < 4; ++j)
#pragma unroll
                            for (int ci = 0; ci < CPG; ++ci)
                                a[j] = fmaf(f4(xv, (j / CPG) * CPG + ci), wk(j, ci, ky * 3 + sx), a[j]);
                    }
                st_stream_v4(yrow + static_cast<long long>(r) * P.wd * C, epilogue(a[0], hb, b.x, P.act),
                             epilogue(a[1], hb, b.y, P.act), epilogue(a[2], hb, b.z, P.act),
                             epilogue(a[3], hb, b.w, P.act));
            }
        }
        __syncthreads();  // every thread is done with stage s before it is refilled
    }
}

// Groups of 4 and 8 channels (channels last, 3x3/s1/p1, C % 4 == 0) with the
// same TMA-staged tiles and two stages: here a thread owns ONE output channel
// (t % 32 of the tile's 32) and NC consecutive columns (column group t / 32
// of 8; tiles of at most 8 NC columns), its 9 CPG weights in registers.  The
// 4 (or 8) lanes of a group read the same 16-byte input vectors, so a warp's
// shared load is one 128-byte wavefront; the thread streams the tile's input
// rows top to bottom, adds each into the three output rows it touches (a ring
// of three rows of NC sums: 3 NC independent chains) and stores an output row
// (a warp: 32 consecutive channels of one pixel per store) when its last
// input row has been added.
template <int CPG, int NC>
__global__ void __launch_bounds__(256) nhwc_grp_tma_kernel(const __grid_constant__ NhwcDwTmaParams P,
                                                           const __grid_constant__ CUtensorMap xmap) {
    constexpr int V = CPG / 4;  // 16-byte input vectors per pixel of a group
    extern __shared__ __align__(128) unsigned char dsm[];
    float *const stage0 = reinterpret_cast<float *>(dsm);
    uint64_t *const full = reinterpret_cast<uint64_t *>(dsm + 2 * P.box_bytes);
    const int tid = threadIdx.x;
    const int cl = tid & 31, col0 = (tid >> 5) * NC;  // channel of the tile, first column of the thread
    const int first = blockIdx.x, stride = gridDim.x;
    if (tid == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        fence_barrier_init();
    }
    __syncthreads();
    griddep_wait();
    griddep_launch_dependents();
    auto issue = [&](int item, int s) {
        int n, h0, w0, c0;
        dw_tma_decode(P, item, n, h0, w0, c0);
        mbar_arrive_expect_tx(&full[s], P.box_bytes);
        tma_load_4d(reinterpret_cast<unsigned char *>(stage0) + s * P.box_bytes, &xmap, c0, w0 - 1, h0 - 1, n,
                    &full[s]);
    };
    if (tid == 0 && first < P.items) {
        prefetch_tensormap(&xmap);
        issue(first, 0);
    }
    const int bw = P.tw + 2;
    const long long C = P.c;
    int it = 0;
    for (int item = first; item < P.items; item += stride, ++it) {
        const int s = it & 1;
        if (tid == 0 && item + stride < P.items) issue(item + stride, s ^ 1);
        const bool ok = mbar_wait_bounded(&full[s], static_cast<uint32_t>((it >> 1) & 1));
        if (!__syncthreads_and(ok)) {
            if (tid == 0) {
                raise_status(kStatusTmaTimeout);
                if (item + stride < P.items)
                    mbar_wait_bounded(&full[s ^ 1], static_cast<uint32_t>(((it + 1) >> 1) & 1));
            }
            return;
        }
        int n, h0, w0, c0;
        dw_tma_decode(P, item, n, h0, w0, c0);
        const int c = c0 + cl;
        const int ncols = min(NC, min(P.tw, P.wd - w0) - col0);  // columns of this thread in the image
        if (ncols > 0 && c < P.c) {
            float4 wt[9 * V];  // [ci][tap] of output channel c: 9 CPG contiguous floats
            const float4 *wsrc = reinterpret_cast<const float4 *>(P.w + static_cast<long long>(c) * CPG * 9);
#pragma unroll
            for (int v = 0; v < 9 * V; ++v) wt[v] = __ldg(wsrc + v);
            auto wk = [&](int ci, int k) -> float {
                const int e = ci * 9 + k;
                return f4(wt[e >> 2], e & 3);
            };
            const bool hb = P.bias != nullptr;
            const float b = hb ? __ldg(P.bias + c) : 0.0f;
            // the group's first channel in the tile, at the thread's first column
            const float *st = stage0 + s * (P.box_bytes / 4) + col0 * kDwTmaCB + (cl - cl % CPG);
            float *ycol = P.y + ((static_cast<long long>(n) * P.h + h0) * P.wd + w0 + col0) * C + c;
            const int rows = min(P.th, P.h - h0);  // output rows of this tile
            float acc[3][NC];                      // sums of output rows oh, slot oh % 3
#pragma unroll
            for (int a = 0; a < 3; ++a)
#pragma unroll
                for (int u = 0; u < NC; ++u) acc[a][u] = 0.0f;
#pragma unroll
            for (int ir = 0; ir < kDwTmaMaxTH + 2; ++ir) {  // box row = input row h0 - 1 + ir
                if (ir >= rows + 2) break;
                float4 xv[NC + 2][V];
#pragma unroll
                for (int q = 0; q < NC + 2; ++q)
#pragma unroll
                    for (int v = 0; v < V; ++v)
                        xv[q][v] = *reinterpret_cast<const float4 *>(st + (ir * bw + q) * kDwTmaCB + 4 * v);
#pragma unroll
                for (int ky = 0; ky < 3; ++ky) {
                    const int oh = ir - ky;  // output row this input row feeds with kernel row ky
                    if (oh < 0 || oh >= rows) continue;
#pragma unroll
                    for (int sx = 0; sx < 3; ++sx)
#pragma unroll
                        for (int ci = 0; ci < CPG; ++ci) {
                            const float wv = wk(ci, ky * 3 + sx);
#pragma unroll
                            for (int u = 0; u < NC; ++u)
                                acc[oh % 3][u] = fmaf(f4(xv[u + sx][ci >> 2], ci & 3), wv, acc[oh % 3][u]);
                        }
                }
                if (ir >= 2) {  // output row ir - 2 is complete
                    const int oh = ir - 2;
                    float *yr = ycol + static_cast<long long>(oh) * P.wd * C;
#pragma unroll
                    for (int u = 0; u < NC; ++u) {
                        if (u < ncols) st_stream(yr + u * C, epilogue(acc[oh % 3][u], hb, b, P.act));
                        acc[oh % 3][u] = 0.0f;
                    }
                }
            }
        }
        __syncthreads();  // every thread is done with stage s before it is refilled
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
