// Direct FP32 grouped 3x3 convolution (stride 1, pad 1, dilation 1,
// Cin == Cout) for groups of fewer than 16 channels: the engine behind
// implementations 1-3 of gc_cuda_conv for depthwise and small-group layers.
//
// Work item = (image n, block of `cb` channels made of whole groups, band of
// `bh` output rows).  A persistent CTA walks items blockIdx.x, +gridDim.x, ...
// through a STAGES-deep ring of shared-memory stages.  A stage holds
//   - the input band of every channel of the item, rows h0-1 .. h0+bh
//     (rounded up to the row blocking), `pitch` floats per row with the image
//     columns at [4, 4+W) and zeros around them, so the convolution's zero
//     padding needs no branches;
//   - the item's raw weights [cb][cpg][3][3].
// Staging is either one TMA tensor load (box starting at column -4, row
// h0-1; the copy engine zero-fills every element outside the image) plus one
// bulk copy of the weights, completion tracked by an mbarrier with a bounded
// wait, or per-thread cp.async copies with zero-fill (any width/alignment).
//
// Compute: every thread owns one fixed cell for the whole kernel - COB output
// channels x VR rows x 4 columns - decoded once.  Cells are numbered with the
// column quad fastest, so the lanes of a warp hold neighbouring quads of a
// row: each input row segment is one 16-byte shared load, and the two halo
// columns come from the neighbouring lanes by warp shuffle (a shared load
// only for the first/last lane of the warp).  Each loaded value is reused
// across the 3 taps of its row, the VR output rows it touches and the COB
// output channels.  Weights are warp-broadcast shared loads from a per-item
// transposed copy [group][ci][tap][co].  Outputs leave registers as streaming
// 16-byte stores when rows are 16-byte aligned.
#pragma once
#include "device_util.cuh"

namespace gcb {

constexpr int kMaxStages = 4;

struct DirectParams {
    const float *x;
    const float *w;
    float *y;
    int n, c, h, wd;     // batch, channels, height, width
    int cpg;             // channels per group (input == output)
    int cb;              // channels per work item (whole groups)
    int bh;              // output rows per item
    int bands, cblocks;  // ceil(h / bh), c / cb
    int items;           // n * cblocks * bands
    int pitch;           // shared row pitch in floats, multiple of 4, >= 4*qcols + 8
    int rows;            // tile rows: round_up(bh, VR) + 2
    int x_floats;        // input tile floats per stage (multiple of 32)
    int wraw_floats;     // raw weight floats per stage (multiple of 32)
    int stage_floats;    // x_floats + wraw_floats
    int wt_floats;       // transposed weight floats (0 when cpg == 1)
    int qcols;           // ceil(wd / 4)
    int rblocks;         // ceil(bh / VR)
    int cells;           // (cb / COB) * rblocks * qcols  (<= blockDim.x)
    int stages;          // shared-memory ring depth, 2..kMaxStages
    int vec_store;       // 16-byte output stores allowed
    int bulk_w;          // TMA staging: weights by bulk copy (else plain loads)
    unsigned x_bytes;    // bytes one TMA box delivers
    unsigned w_bytes;    // raw weight bytes per item
};

__device__ __forceinline__ void decode_item(const DirectParams &P, int item, int &n, int &c0,
                                            int &h0) {
    const unsigned u = static_cast<unsigned>(item);
    const unsigned t = u / static_cast<unsigned>(P.bands);
    const unsigned band = u - t * static_cast<unsigned>(P.bands);
    const unsigned nn = t / static_cast<unsigned>(P.cblocks);
    const unsigned cblk = t - nn * static_cast<unsigned>(P.cblocks);
    n = static_cast<int>(nn);
    c0 = static_cast<int>(cblk) * P.cb;
    h0 = static_cast<int>(band) * P.bh;
}

// Per-thread asynchronous staging of one item (any width, any alignment).
__device__ __forceinline__ void stage_with_cp_async(const DirectParams &P, float *xs, float *wr,
                                                    int item) {
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
                                               float *xs, float *wr, uint64_t *bar, int item) {
    int n, c0, h0;
    decode_item(P, item, n, c0, h0);
    mbar_arrive_expect_tx(bar, P.x_bytes + (P.bulk_w ? P.w_bytes : 0u));
    tma_load_4d(xs, xmap, -4, h0 - 1, c0, n, bar);
    if (P.bulk_w) bulk_load(wr, P.w + static_cast<long long>(c0) * P.cpg * 9, P.w_bytes, bar);
}

// Six consecutive values x[col0-1 .. col0+4] of one tile row for a thread
// whose 16-byte quad starts at p: the quad itself is one shared load, the two
// halo values come from the neighbouring lanes by shuffle, or (first/last
// lane of the warp) from a predicated shared load, or are the zero padding at
// the image edges.  Branch-free, so the warp never diverges.
// Four outputs of one row: one streaming 16-byte store when the row is
// 16-byte aligned and fully inside the image, else per-column stores.
__device__ __forceinline__ void store_quad(float *yp, const float (&a)[4], bool vec_ok, int col0,
                                           int width) {
    if (vec_ok) {
        st_stream_v4(yp, a[0], a[1], a[2], a[3]);
    } else {
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (col0 + u < width) st_stream(yp + u, a[u]);
    }
}

struct RowEdges {
    bool zero_left, zero_right;  // quad at the left / right image edge
    bool load_left, load_right;  // neighbour quad lives in another warp
};

__device__ __forceinline__ void load_row6(const float *p, const RowEdges &e, float (&x)[6]) {
    const float4 m = *reinterpret_cast<const float4 *>(p);
    const float sl = __shfl_up_sync(0xffffffffu, m.w, 1);
    const float sr = __shfl_down_sync(0xffffffffu, m.x, 1);
    const float ml = lds_if(p - 1, e.load_left);
    const float mr = lds_if(p + 4, e.load_right);
    x[0] = e.zero_left ? 0.0f : (e.load_left ? ml : sl);
    x[1] = m.x;
    x[2] = m.y;
    x[3] = m.z;
    x[4] = m.w;
    x[5] = e.zero_right ? 0.0f : (e.load_right ? mr : sr);
}

template <int CPG, int COB, int VR, bool TMA>
__global__ void __launch_bounds__(256) direct_conv_kernel(const __grid_constant__ DirectParams P,
                                                          const __grid_constant__ CUtensorMap xmap) {
    extern __shared__ __align__(128) float smem[];
    const int cpg = CPG > 0 ? CPG : P.cpg;
    const int STAGES = P.stages;
    float *wt = smem + STAGES * P.stage_floats;
    uint64_t *bars = reinterpret_cast<uint64_t *>(wt + P.wt_floats);
    const int first = blockIdx.x, step = gridDim.x;
    const int count = first < P.items ? (P.items - 1 - first) / step + 1 : 0;
    const int tid = threadIdx.x, lane = tid & 31;

    // This thread's cell, fixed for every item.  Threads past the last cell
    // (in the last warp) mirror the last cell's loads so that every lane takes
    // part in the shuffles, and store nothing.
    const bool has_cell = tid < P.cells;
    const int cell = has_cell ? tid : P.cells - 1;
    const int q = cell % P.qcols;
    const int rbc = cell / P.qcols;
    const int rb = rbc % P.rblocks;
    const int cob = rbc / P.rblocks;
    const int col0 = q * 4, row0 = rb * VR;
    const int co_item = cob * COB;  // first output channel of the cell, item-local
    const int g = co_item / cpg;    // item-local group
    const int cog = co_item - g * cpg;
    const bool first_q = q == 0, last_q = q == P.qcols - 1;
    const RowEdges edges{first_q, last_q, lane == 0 && !first_q, lane == 31 && !last_q};
    const bool vec_ok = P.vec_store && col0 + 4 <= P.wd;
    const int chan_floats = P.rows * P.pitch;
    const int xoff = (g * cpg) * chan_floats + row0 * P.pitch + col0 + 4;

    if (TMA && tid == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 1);
        fence_barrier_init();
        prefetch_tensormap(&xmap);
    }
    // Everything above touches only shared memory and parameters; global
    // memory is read and written after the previous launch in the stream has
    // completed.
    griddep_wait();
    griddep_launch_dependents();
    if (TMA) {
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

    for (int k = 0; k < count; ++k) {
        const int s = k % STAGES;
        const int item = first + k * step;
        float *xs = smem + s * P.stage_floats;
        float *wr = xs + P.x_floats;
        if (TMA) {
            // One thread polls the barrier; the rest wait in the hardware
            // barrier instead of spinning on issue slots.
            bool ok = true;
            if (tid == 0) ok = mbar_wait_bounded(&bars[s], static_cast<uint32_t>((k / STAGES) & 1));
            if (!__syncthreads_and(ok)) {
                // The copy engine did not deliver in time: record it, let the
                // loads still in flight land (bounded), and leave.
                if (tid == 0) {
                    raise_status(kStatusTmaTimeout);
                    for (int j = k + 1; j < k + STAGES && j < count; ++j)
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
            const int kn = k + STAGES - 1;
            if (kn < count)
                stage_with_cp_async(P, smem + (kn % STAGES) * P.stage_floats,
                                    smem + (kn % STAGES) * P.stage_floats + P.x_floats,
                                    first + kn * step);
            cp_async_commit();
            cp_async_wait_dynamic(STAGES - 1);
            __syncthreads();
        }
        if (CPG != 1) {
            // raw [co][ci][tap] -> [group][ci][tap][co-in-group]
            const int per_co = cpg * 9;
            for (int e = tid; e < P.cb * per_co; e += blockDim.x) {
                const int co = e / per_co;
                const int rem = e - co * per_co;
                const int gg = co / cpg;
                wt[(gg * cpg * 9 + rem) * cpg + (co - gg * cpg)] = wr[e];
            }
            __syncthreads();
        }

        int n, c0, h0;
        decode_item(P, item, n, c0, h0);
        const long long plane_floats = static_cast<long long>(P.h) * P.wd;
        float *ybase = P.y + (static_cast<long long>(n) * P.c + c0 + co_item) * plane_floats +
                       static_cast<long long>(h0 + row0) * P.wd + col0;
        // output rows of this cell inside the band and the image
        const int rows_valid = has_cell ? min(VR, min(P.bh - row0, P.h - h0 - row0)) : 0;
        const float *xg = xs + xoff;
        if (CPG == 1) {
            // Depthwise: nine weights in registers; input rows stream top to
            // bottom and each output row leaves as soon as its last input row
            // has been applied, so only three output rows are ever live.
            float wk[9];
#pragma unroll
            for (int t = 0; t < 9; ++t) wk[t] = wr[co_item * 9 + t];
            float acc[3][4];
#pragma unroll
            for (int rr = 0; rr < VR + 2; ++rr) {
                float xrow[6];
                load_row6(xg + rr * P.pitch, edges, xrow);
#pragma unroll
                for (int r = 0; r < 3; ++r) {
                    const int v = rr - r;  // output row this input row feeds with kernel row r
                    if (v < 0 || v >= VR) continue;
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        float a = r == 0 ? 0.0f : acc[v % 3][u];
#pragma unroll
                        for (int sx = 0; sx < 3; ++sx) a = fmaf(xrow[u + sx], wk[r * 3 + sx], a);
                        acc[v % 3][u] = a;
                    }
                }
                if (rr >= 2 && rr - 2 < rows_valid)
                    store_quad(ybase + (rr - 2) * P.wd, acc[(rr - 2) % 3], vec_ok, col0, P.wd);
            }
        } else {
            float acc[COB][VR][4];
#pragma unroll
            for (int j = 0; j < COB; ++j)
#pragma unroll
                for (int v = 0; v < VR; ++v)
#pragma unroll
                    for (int u = 0; u < 4; ++u) acc[j][v][u] = 0.0f;
#pragma unroll(CPG == 2 ? 2 : 1)
            for (int ci = 0; ci < cpg; ++ci) {
                const float *xc = xg + ci * chan_floats;
                float xr[VR + 2][6];
#pragma unroll
                for (int rr = 0; rr < VR + 2; ++rr) load_row6(xc + rr * P.pitch, edges, xr[rr]);
                const float *wp = wt + ((g * cpg + ci) * 9) * cpg + cog;
#pragma unroll
                for (int tap = 0; tap < 9; ++tap) {
                    const int r = tap / 3, sx = tap % 3;
                    float wv[COB];
                    if (COB % 4 == 0) {
#pragma unroll
                        for (int j = 0; j < COB; j += 4) {
                            const float4 m = *reinterpret_cast<const float4 *>(wp + tap * cpg + j);
                            wv[j] = m.x;
                            wv[j + 1] = m.y;
                            wv[j + 2] = m.z;
                            wv[j + 3] = m.w;
                        }
                    } else if (COB % 2 == 0) {
#pragma unroll
                        for (int j = 0; j < COB; j += 2) {
                            const float2 m = *reinterpret_cast<const float2 *>(wp + tap * cpg + j);
                            wv[j] = m.x;
                            wv[j + 1] = m.y;
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
                                acc[j][v][u] = fmaf(xr[v + r][u + sx], wv[j], acc[j][v][u]);
                }
            }
#pragma unroll
            for (int j = 0; j < COB; ++j)
#pragma unroll
                for (int v = 0; v < VR; ++v)
                    if (v < rows_valid)
                        store_quad(ybase + j * plane_floats + v * P.wd, acc[j][v], vec_ok, col0, P.wd);
        }
        __syncthreads();
        if (TMA && tid == 0 && k + STAGES < count)
            stage_with_tma(P, &xmap, xs, wr, &bars[s], first + (k + STAGES) * step);
    }
    if (!TMA) cp_async_wait<0>();
}

}  // namespace gcb
