// Grouped 3x3 convolution (stride 1, pad 1, Cin == Cout) for small images
// (a few hundred pixels per plane, e.g. 7x7 and 14x14), where whole planes
// are the natural unit and the row-band machinery of the direct engine costs
// more than the work.  Any width, any alignment.
//
// Work item = (image n, block of `cb` channels made of whole groups).  The
// item's input planes are one contiguous block of cb*H*W floats in global
// memory (NCHW), and so are its output planes: the CTA copies the input block
// into shared memory with coalesced 16-byte loads (4-byte when unaligned),
// the weights beside it, and every thread then owns one output pixel of COB
// consecutive output channels.  The nine tap offsets and their in-image
// predicates depend only on the pixel, so they are computed once per thread
// and reused for every input channel and output channel; each input value
// read from shared memory feeds COB FMAs; weights are warp-broadcast reads.
// Output stores are coalesced (consecutive threads, consecutive pixels).
#pragma once
#include "device_util.cuh"

namespace gcb {

struct SmallParams {
    const float *x;
    const float *w;
    float *y;
    int n, c, h, wd, cpg;
    int cb;          // channels per item (whole groups)
    int cblocks;     // c / cb
    int items;       // n * cblocks
    int hw;          // h * wd
    int hwp;         // hw rounded up to a whole warp: threads per pixel slot
    int x_floats;    // cb * hw rounded up to 4
    int vec;         // 16-byte loads allowed for the input block
};

// Threads are laid out as blockDim.x / hwp slots of hwp threads; thread
// (slot, p) owns pixel p for the whole kernel (tap offsets and in-image
// predicates computed once) and walks the item's output-channel blocks
// slot, slot + slots, ...
template <int COB>
__global__ void __launch_bounds__(512, 1) small_conv_kernel(const __grid_constant__ SmallParams P) {
    extern __shared__ __align__(128) float smem[];
    float *xs = smem;
    float *ws = smem + P.x_floats;
    const int cpg = P.cpg;
    const int wcount = P.cb * cpg * 9;
    const int slots = blockDim.x / P.hwp;
    const int p = threadIdx.x % P.hwp, slot = threadIdx.x / P.hwp;
    const bool active = p < P.hw && slot < slots;
    const int oh = p / P.wd, ow = p - oh * P.wd;
    // Tap offsets (0 for taps outside the image) and a 9-bit in-image mask.
    int off[9];
    unsigned okmask = 0;
#pragma unroll
    for (int tap = 0; tap < 9; ++tap) {
        const int ih = oh + tap / 3 - 1, iw = ow + tap % 3 - 1;
        const bool in = active && ih >= 0 && ih < P.h && iw >= 0 && iw < P.wd;
        okmask |= in ? (1u << tap) : 0u;
        off[tap] = in ? ih * P.wd + iw : 0;
    }
    const int ncob = P.cb / COB;
    griddep_wait();
    griddep_launch_dependents();
    for (int item = blockIdx.x; item < P.items; item += gridDim.x) {
        const int nn = item / P.cblocks;
        const int c0 = (item - nn * P.cblocks) * P.cb;
        const long long base = (static_cast<long long>(nn) * P.c + c0) * P.hw;
        __syncthreads();  // the previous item's readers are done
        const int total = P.cb * P.hw;
        if (P.vec) {
            const float4 *src = reinterpret_cast<const float4 *>(P.x + base);
            float4 *dst = reinterpret_cast<float4 *>(xs);
            for (int e = threadIdx.x; e < total / 4; e += blockDim.x) dst[e] = __ldg(src + e);
        } else {
            for (int e = threadIdx.x; e < total; e += blockDim.x) xs[e] = __ldg(P.x + base + e);
        }
        const float *wsrc = P.w + static_cast<long long>(c0) * cpg * 9;
        for (int e = threadIdx.x; e < wcount; e += blockDim.x) ws[e] = __ldg(wsrc + e);
        __syncthreads();
        if (!active) continue;
        float *yp0 = P.y + base + p;
        for (int cob = slot; cob < ncob; cob += slots) {
            const int co0 = cob * COB;  // item-local first output channel
            const int g = co0 / cpg;    // item-local group
            float acc[COB];
#pragma unroll
            for (int j = 0; j < COB; ++j) acc[j] = 0.0f;
            const float *xg = xs + g * cpg * P.hw;
            const float *wg = ws + co0 * cpg * 9;
            for (int ci = 0; ci < cpg; ++ci) {
                const float *xc = xg + ci * P.hw;
                const float *wc = wg + ci * 9;
#pragma unroll
                for (int tap = 0; tap < 9; ++tap) {
                    const float xv = (okmask >> tap) & 1u ? xc[off[tap]] : 0.0f;
#pragma unroll
                    for (int j = 0; j < COB; ++j) acc[j] = fmaf(xv, wc[j * cpg * 9 + tap], acc[j]);
                }
            }
#pragma unroll
            for (int j = 0; j < COB; ++j) st_stream(yp0 + static_cast<long long>(co0 + j) * P.hw, acc[j]);
        }
    }
}

}  // namespace gcb
