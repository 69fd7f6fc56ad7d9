// Grouped 3x3 convolution (stride 1, pad 1, Cin == Cout) for small images
// (a few hundred pixels per plane, e.g. 7x7 and 14x14), where whole planes
// are the natural unit and the row-band machinery of the direct engine costs
// more than the work.  Any width, any alignment.
//
// Work item = (image n, block of `cb` channels made of whole groups).  The
// item's input planes are one contiguous block of cb*H*W floats in global
// memory (NCHW), and so are its output planes.  A persistent CTA walks its
// items through a ring of up to four shared-memory stages: while it computes
// item k, the asynchronous copies of the next items (16-byte cp.async when
// aligned, else 4-byte) are in flight, so the load latency - which dominates
// at these sizes - is paid once per CTA, not once per item.  Every thread owns one
// output pixel of COB consecutive output channels: the nine tap offsets and
// their in-image predicates depend only on the pixel, so they are computed
// once per thread and reused for every input and output channel; each input
// value read from shared memory feeds COB FMAs; weights are warp-broadcast
// reads.  Output stores are coalesced (consecutive threads, consecutive
// pixels).
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
    int w_floats;    // cb * cpg * 9 rounded up to 4
    int vec;         // 16-byte copies allowed for the input block
    int stages;      // shared-memory ring depth, 1..4: the copies of the next stages-1 items
                     // are in flight while an item is computed
};

// Issues the copies of one item into a stage (every thread its share).
__device__ __forceinline__ void small_stage(const SmallParams &P, float *xs, float *ws, int item) {
    const int nn = item / P.cblocks;
    const int c0 = (item - nn * P.cblocks) * P.cb;
    const long long base = (static_cast<long long>(nn) * P.c + c0) * P.hw;
    const int total = P.cb * P.hw;
    if (P.vec) {
        for (int e = threadIdx.x; e < total / 4; e += blockDim.x) cp_async_16(xs + 4 * e, P.x + base + 4 * e);
    } else {
        for (int e = threadIdx.x; e < total; e += blockDim.x) cp_async_4(xs + e, P.x + base + e, true);
    }
    const int wcount = P.cb * P.cpg * 9;
    const float *wsrc = P.w + static_cast<long long>(c0) * P.cpg * 9;
    for (int e = threadIdx.x; e < wcount; e += blockDim.x) cp_async_4(ws + e, wsrc + e, true);
}

// Threads are laid out as blockDim.x / hwp slots of hwp threads; thread
// (slot, p) owns pixel p for the whole kernel (tap offsets and in-image
// predicates computed once) and walks the item's output-channel blocks
// slot, slot + slots, ...
template <int COB>
__global__ void __launch_bounds__(512, 1) small_conv_kernel(const __grid_constant__ SmallParams P) {
    extern __shared__ __align__(128) float smem[];
    const int stage_floats = P.x_floats + P.w_floats;
    const int cpg = P.cpg;
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
    const int first = blockIdx.x, step = gridDim.x;
    const int count = first < P.items ? (P.items - 1 - first) / step + 1 : 0;
    griddep_wait();
    griddep_launch_dependents();
    const int S = P.stages;
    for (int s = 0; s < S - 1; ++s) {
        if (s < count) {
            float *xs = smem + s * stage_floats;
            small_stage(P, xs, xs + P.x_floats, first + s * step);
        }
        cp_async_commit();
    }
    for (int k = 0; k < count; ++k) {
        const int item = first + k * step;
        float *xs = smem + (k % S) * stage_floats;
        const float *ws = xs + P.x_floats;
        // stage (k + S - 1) % S was last read at item k - 1 (barrier at its end)
        if (k + S - 1 < count) {
            float *xn = smem + ((k + S - 1) % S) * stage_floats;
            small_stage(P, xn, xn + P.x_floats, item + (S - 1) * step);
        }
        cp_async_commit();
        cp_async_wait_dynamic(S - 1);  // this thread's copies of item k have landed
        __syncthreads();               // and every other thread's
        if (active) {
            const int nn = item / P.cblocks;
            const int c0 = (item - nn * P.cblocks) * P.cb;
            float *yp0 = P.y + (static_cast<long long>(nn) * P.c + c0) * P.hw + p;
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
        __syncthreads();  // item k's stage is free again
    }
    cp_async_wait<0>();
}

}  // namespace gcb
