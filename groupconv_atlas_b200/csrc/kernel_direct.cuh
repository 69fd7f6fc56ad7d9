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
//   - the item's raw weights [cb][cpg][3][3], and (TMA kernel, cpg > 1) their
//     transposed copy [group][ci][tap][co].
//
// Two kernels share the compute core:
//   direct_ws_kernel   TMA staging, warp-specialized.  A copy warp issues
//                      the TMA box of the input band (column -4 start keeps
//                      the box 16-byte aligned; the copy engine zero-fills
//                      everything outside the image) and a bulk copy of the
//                      weights; a weight warp transposes the weights of each
//                      landed stage; the other warps compute.  Stages are
//                      handed over through mbarriers with bounded waits, so
//                      no CTA-wide barrier sits in the item loop and warps
//                      drift freely within the ring.
//   direct_conv_kernel CTA barriers between items; per-thread cp.async
//                      staging with zero fill (any width and alignment), or
//                      TMA staging for depthwise layers.
//
// Compute: every thread owns one fixed cell for the whole kernel - COB output
// channels x VR rows x CW (4 or 8) columns - decoded once.  Cells are
// numbered with the column block fastest, so the lanes of a warp hold
// neighbouring blocks of a row: each input row segment is CW/4 16-byte shared
// loads, and the two halo
// columns come from the neighbouring lanes by warp shuffle, replaced by a
// predicated shared load for the first/last lane of the warp and at the
// image edges (where the tile holds the zero padding).  Each loaded value is
// reused across the 3 taps of its row, the VR output rows it touches and the
// COB output channels.  Weights are warp-broadcast shared loads.  Outputs
// leave registers as streaming 16-byte stores when rows are 16-byte aligned.
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
    int pitch;           // shared row pitch in floats, multiple of 4, >= CW*qcols + 8
                         // (the last block's right neighbour quad lies inside the row)
    int rows;            // tile rows: round_up(bh, VR) + 2
    int x_floats;        // input tile floats per stage (multiple of 32)
    int wraw_floats;     // raw weight floats per stage (multiple of 32)
    int wt_floats;       // transposed weight floats (0 when cpg == 1)
    int stage_floats;    // TMA kernel: x + wraw + wt per stage; cp.async kernel: x + wraw
    int qcols;           // column blocks per row: ceil(wd / CW)
    int rblocks;         // ceil(bh / VR)
    int cells;           // (cb / COB) * rblocks * qcols  (<= compute threads)
    int stages;          // shared-memory ring depth, 2..kMaxStages
    int vec_store;       // 16-byte output stores allowed
    int bulk_w;          // TMA staging: weights by bulk copy (else plain loads)
    unsigned x_bytes;    // bytes one TMA box delivers
    unsigned w_bytes;    // raw weight bytes per item
    const float *bias;   // nullable: per-output-channel bias added after the sum
    int act;             // kActNone / kActRelu / kActRelu6, applied after the bias
};

// The epilogue of a row segment of CW outputs of one channel, in place.
template <int CW>
__device__ __forceinline__ void finish_row(float (&a)[CW], const DirectParams &P, int channel) {
    if (P.bias == nullptr && P.act == kActNone) return;
    const bool hb = P.bias != nullptr;
    const float b = hb ? __ldg(P.bias + channel) : 0.0f;
#pragma unroll
    for (int u = 0; u < CW; ++u) a[u] = epilogue(a[u], hb, b, P.act);
}

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

__device__ __forceinline__ int decode_c0(const DirectParams &P, int item) {
    int n, c0, h0;
    decode_item(P, item, n, c0, h0);
    return c0;
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

// raw [co][ci][tap] -> [group][ci][tap][co-in-group], threads t0, t0+tstride, ...
__device__ __forceinline__ void transpose_weights(const float *wr, float *wt, int cb, int cpg, int t0,
                                                  int tstride) {
    const int per_co = cpg * 9;
    for (int e = t0; e < cb * per_co; e += tstride) {
        const int co = e / per_co;
        const int rem = e - co * per_co;
        const int gg = co / cpg;
        wt[(gg * cpg * 9 + rem) * cpg + (co - gg * cpg)] = wr[e];
    }
}

// Same layout as transpose_weights, read straight from global memory.
__device__ __forceinline__ void transpose_weights_global(const float *w, float *wt, int cb, int cpg,
                                                         int t0, int tstride) {
    const int per_co = cpg * 9;
    for (int e = t0; e < cb * per_co; e += tstride) {
        const int co = e / per_co;
        const int rem = e - co * per_co;
        const int gg = co / cpg;
        wt[(gg * cpg * 9 + rem) * cpg + (co - gg * cpg)] = __ldg(w + e);
    }
}

// Four outputs of one row: one streaming 16-byte store when the row is
// 16-byte aligned and fully inside the image, else per-column stores.
__device__ __forceinline__ void store_quad(float *yp, float a0, float a1, float a2, float a3, bool vec_ok,
                                           int col0, int width) {
    if (vec_ok) {
        st_stream_v4(yp, a0, a1, a2, a3);
    } else {
        if (col0 < width) st_stream(yp, a0);
        if (col0 + 1 < width) st_stream(yp + 1, a1);
        if (col0 + 2 < width) st_stream(yp + 2, a2);
        if (col0 + 3 < width) st_stream(yp + 3, a3);
    }
}

// The CW + 2 consecutive values x[col0-1 .. col0+CW] of one tile row for a
// thread whose CW columns start at p (16-byte aligned): the columns
// themselves are CW/4 16-byte shared loads and the two halo values come from
// the neighbouring lanes by shuffle.  Where the neighbour block is not in the
// neighbouring lane (first/last lane of the warp, or the block sits at an
// image edge and the neighbouring lane holds another row) a predicated shared
// load reads the tile instead: the neighbour column, or the zero padding
// beside the image.  The shuffles and the loads are independent (selected
// afterwards), so their latencies overlap; branch-free, so the warp never
// diverges.
template <int CW>
__device__ __forceinline__ void load_row(const float *p, bool left_smem, bool right_smem, float (&x)[CW + 2]) {
#pragma unroll
    for (int b = 0; b < CW / 4; ++b) {
        const float4 m = *reinterpret_cast<const float4 *>(p + 4 * b);
        x[1 + 4 * b] = m.x;
        x[2 + 4 * b] = m.y;
        x[3 + 4 * b] = m.z;
        x[4 + 4 * b] = m.w;
    }
    const float sl = __shfl_up_sync(0xffffffffu, x[CW], 1);
    const float sr = __shfl_down_sync(0xffffffffu, x[1], 1);
    const float ml = lds_over(p - 1, left_smem, 0.0f);
    const float mr = lds_over(p + CW, right_smem, 0.0f);
    x[0] = left_smem ? ml : sl;
    x[CW + 1] = right_smem ? mr : sr;
}

// The fixed cell of one thread: COB output channels x VR rows x CW columns.
// Threads past the last cell mirror the last cell's loads, so that every
// lane takes part in the shuffles, and store nothing.
struct Cell {
    int col0, row0;
    int co_item;  // first output channel of the cell, item-local
    int g, cog;   // item-local group, channel within the group
    int xoff;     // offset of the cell's first input row segment in a stage
    bool has_cell, left_smem, right_smem;
    unsigned vec_mask;  // bit b: quad b of the cell may use a 16-byte store
};

template <int COB, int VR, int CW>
__device__ __forceinline__ Cell make_cell(const DirectParams &P, int tid, int cpg) {
    Cell c;
    const int lane = tid & 31;
    c.has_cell = tid < P.cells;
    const int cell = c.has_cell ? tid : P.cells - 1;
    // Cell order: quad fastest (depthwise cells take their halo columns from
    // the neighbouring lanes; for groups of 2 and 4 channels, which are
    // bandwidth-bound, this order measured faster); for groups of 8 or more
    // channels (FFMA-bound) the row block fastest, so that with a row pitch
    // of an odd number of 16-byte chunks per row block every 8-lane phase of
    // a 16-byte shared load touches 8 different bank groups.
    int q, rb, cob;
    if (cpg < 8) {
        q = cell % P.qcols;
        const int rbc = cell / P.qcols;
        rb = rbc % P.rblocks;
        cob = rbc / P.rblocks;
    } else {
        rb = cell % P.rblocks;
        const int qc = cell / P.rblocks;
        q = qc % P.qcols;
        cob = qc / P.qcols;
    }
    c.col0 = q * CW;
    c.row0 = rb * VR;
    c.co_item = cob * COB;
    c.g = c.co_item / cpg;
    c.cog = c.co_item - c.g * cpg;
    c.left_smem = q == 0 || lane == 0;
    c.right_smem = q == P.qcols - 1 || lane == 31;
    c.vec_mask = 0;
#pragma unroll
    for (int b = 0; b < CW / 4; ++b)
        if (P.vec_store && c.col0 + 4 * b + 4 <= P.wd) c.vec_mask |= 1u << b;
    c.xoff = (c.g * cpg) * P.rows * P.pitch + c.row0 * P.pitch + c.col0 + 4;
    return c;
}

// Same values by three plain loads per quad row: the quads left and right of
// the thread's own are loaded whole (16 bytes each, conflict-free like the
// centre load) and only their inner columns kept.  Three load instructions
// and no shuffles or selects: fewer issue slots, more shared-memory
// wavefronts - the better trade where FFMA issue is the bound.
template <int CW>
__device__ __forceinline__ void load_row_wide(const float *p, float (&x)[CW + 2]) {
    const float4 l = *reinterpret_cast<const float4 *>(p - 4);
#pragma unroll
    for (int b = 0; b < CW / 4; ++b) {
        const float4 m = *reinterpret_cast<const float4 *>(p + 4 * b);
        x[1 + 4 * b] = m.x;
        x[2 + 4 * b] = m.y;
        x[3 + 4 * b] = m.z;
        x[4 + 4 * b] = m.w;
    }
    const float4 r = *reinterpret_cast<const float4 *>(p + CW);
    x[0] = l.w;
    x[CW + 1] = r.x;
}

// One output row segment of a cell: CW/4 quads.
template <int CW>
__device__ __forceinline__ void store_row(float *yp, const float (&a)[CW], const Cell &c, int width) {
#pragma unroll
    for (int b = 0; b < CW / 4; ++b)
        store_quad(yp + 4 * b, a[4 * b], a[4 * b + 1], a[4 * b + 2], a[4 * b + 3], (c.vec_mask >> b) & 1u,
                   c.col0 + 4 * b, width);
}

// One item of one cell: xs is the stage's input tile, wk the weights (raw
// [co][tap] for depthwise, transposed [group][ci][tap][co] otherwise).
template <int CPG, int COB, int VR, int CW>
__device__ __forceinline__ void compute_item(const DirectParams &P, const Cell &c, const float *xs,
                                             const float *wk_base, int item) {
    const int cpg = CPG > 0 ? CPG : P.cpg;
    int n, c0, h0;
    decode_item(P, item, n, c0, h0);
    const long long plane_floats = static_cast<long long>(P.h) * P.wd;
    float *ybase = P.y + (static_cast<long long>(n) * P.c + c0 + c.co_item) * plane_floats +
                   static_cast<long long>(h0 + c.row0) * P.wd + c.col0;
    // output rows of this cell inside the band and the image
    const int rows_valid = c.has_cell ? min(VR, min(P.bh - c.row0, P.h - h0 - c.row0)) : 0;
    const float *xg = xs + c.xoff;
    if (CPG == 1) {
        // Depthwise: nine weights in registers; input rows stream top to
        // bottom and each output row leaves as soon as its last input row
        // has been applied, so only three output rows are ever live.
        float wk[9];
#pragma unroll
        for (int t = 0; t < 9; ++t) wk[t] = wk_base[c.co_item * 9 + t];
        float acc[3][CW];
#pragma unroll
        for (int rr = 0; rr < VR + 2; ++rr) {
            float xrow[CW + 2];
            load_row<CW>(xg + rr * P.pitch, c.left_smem, c.right_smem, xrow);
#pragma unroll
            for (int r = 0; r < 3; ++r) {
                const int v = rr - r;  // output row this input row feeds with kernel row r
                if (v < 0 || v >= VR) continue;
#pragma unroll
                for (int u = 0; u < CW; ++u) {
                    float a = r == 0 ? 0.0f : acc[v % 3][u];
#pragma unroll
                    for (int sx = 0; sx < 3; ++sx) a = fmaf(xrow[u + sx], wk[r * 3 + sx], a);
                    acc[v % 3][u] = a;
                }
            }
            if (rr >= 2 && rr - 2 < rows_valid) {
                finish_row<CW>(acc[(rr - 2) % 3], P, c0 + c.co_item);
                store_row<CW>(ybase + (rr - 2) * P.wd, acc[(rr - 2) % 3], c, P.wd);
            }
        }
    } else {
        const int chan_floats = P.rows * P.pitch;
        float acc[COB][VR][CW];
#pragma unroll
        for (int j = 0; j < COB; ++j)
#pragma unroll
            for (int v = 0; v < VR; ++v)
#pragma unroll
                for (int u = 0; u < CW; ++u) acc[j][v][u] = 0.0f;
#pragma unroll 1
        for (int ci = 0; ci < cpg; ++ci) {
            const float *xc = xg + ci * chan_floats;
            float xr[VR + 2][CW + 2];
#pragma unroll
            for (int rr = 0; rr < VR + 2; ++rr) load_row_wide<CW>(xc + rr * P.pitch, xr[rr]);
            const float *wp = wk_base + ((c.g * cpg + ci) * 9) * cpg + c.cog;
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
                        for (int u = 0; u < CW; ++u)
                            acc[j][v][u] = fmaf(xr[v + r][u + sx], wv[j], acc[j][v][u]);
            }
        }
#pragma unroll
        for (int j = 0; j < COB; ++j)
#pragma unroll
            for (int v = 0; v < VR; ++v)
                if (v < rows_valid) {
                    finish_row<CW>(acc[j][v], P, c0 + c.co_item + j);
                    store_row<CW>(ybase + j * plane_floats + v * P.wd, acc[j][v], c, P.wd);
                }
    }
}

// ---- TMA staging: copy warp, weight warp, compute warps ----------------------------
// Block = compute warps (cells rounded up to whole warps), then the copy warp
// (one lane issues the TMA box and the weights' bulk copy of each item as
// soon as the compute warps have released the stage), then - when weights
// need work (transpose for cpg > 1, or plain loads when no bulk copy is
// possible) - the weight warp, which prepares each landed stage.  Per stage
// three mbarriers: full (TMA bytes landed), ready (weights prepared; count 1;
// used only with a weight warp), empty (every compute warp is done with the
// stage; count = compute warps).  The copy warp never waits for a landing,
// so each stage is refilled the moment it is free.
constexpr int kWsMaxThreads = 288;

__host__ __device__ inline int direct_ws_producer_warps(int cpg, int bulk_w) {
    return (cpg != 1 || !bulk_w) ? 2 : 1;
}

template <int CPG, int COB, int VR, int CW>
__global__ void __launch_bounds__(kWsMaxThreads) direct_ws_kernel(const __grid_constant__ DirectParams P,
                                                         const __grid_constant__ CUtensorMap xmap) {
    extern __shared__ __align__(128) float smem[];
    const int cpg = CPG > 0 ? CPG : P.cpg;
    const int STAGES = P.stages;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * P.stage_floats);
    uint64_t *ready = full + kMaxStages;
    uint64_t *empty = ready + kMaxStages;
    volatile int *abort_word = reinterpret_cast<volatile int *>(empty + kMaxStages);
    const int first = blockIdx.x, step = gridDim.x;
    const int count = first < P.items ? (P.items - 1 - first) / step + 1 : 0;
    const int tid = threadIdx.x, lane = tid & 31;
    const bool weight_warp = direct_ws_producer_warps(cpg, P.bulk_w) == 2;
    const int compute_threads = blockDim.x - (weight_warp ? 64 : 32);
    const int compute_warps = compute_threads >> 5;
    auto xs_of = [&](int s) { return smem + s * P.stage_floats; };
    auto wr_of = [&](int s) { return smem + s * P.stage_floats + P.x_floats; };

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&ready[s], 1);
            mbar_init(&empty[s], compute_warps);
        }
        *abort_word = 0;
        fence_barrier_init();
        prefetch_tensormap(&xmap);
    }
    // Everything above touches only shared memory and parameters; global
    // memory is read and written after the previous launch in the stream has
    // completed.
    griddep_wait();
    griddep_launch_dependents();
    __syncthreads();

    if (tid >= compute_threads + 32) {
        // ---- weight warp: prepare each landed stage, publish it ----
        float *const wt0 = smem + P.x_floats + P.wraw_floats;
        for (int k = 0; k < count; ++k) {
            const int s = k % STAGES;
            const bool ok = __all_sync(0xffffffffu, role_wait(&full[s], static_cast<uint32_t>((k / STAGES) & 1),
                                                                abort_word, kStatusTmaTimeout));
            if (!ok) return;
            float *wt = wt0 + s * P.stage_floats;
            if (CPG != 1) {
                if (P.bulk_w)
                    transpose_weights(wr_of(s), wt, P.cb, cpg, lane, 32);
                else
                    transpose_weights_global(P.w + static_cast<long long>(decode_c0(P, first + k * step)) * cpg * 9,
                                             wt, P.cb, cpg, lane, 32);
            } else {
                const float *wsrc = P.w + static_cast<long long>(decode_c0(P, first + k * step)) * 9;
                for (int e = lane; e < P.cb * 9; e += 32) wr_of(s)[e] = __ldg(wsrc + e);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&ready[s]);
        }
        return;
    }
    if (tid >= compute_threads) {
        // ---- copy warp: one lane refills each stage as soon as it is free ----
        if (lane != 0) return;
        int issued = 0;
        bool ok = true;
        for (int i = 0; i < count; ++i) {
            const int s = i % STAGES;
            if (i >= STAGES) {
                // item i - STAGES used this stage: wait until every compute warp released it
                ok = role_wait(&empty[s], static_cast<uint32_t>(((i - STAGES) / STAGES) & 1), abort_word,
                               kStatusTmaTimeout);
                if (!ok) break;
            }
            stage_with_tma(P, &xmap, xs_of(s), wr_of(s), &full[s], first + i * step);
            issued = i + 1;
        }
        // Before the CTA's shared memory is released, the copies still in
        // flight must land: the last STAGES items (all earlier ones were
        // consumed before their stage was refilled).  Always, not only when
        // this warp gave up: the compute or weight warps may have given up
        // while its last copies were still arriving.  Bounded.
        (void)ok;
        for (int i = max(0, issued - STAGES); i < issued; ++i)
            mbar_wait_bounded(&full[i % STAGES], static_cast<uint32_t>((i / STAGES) & 1));
        return;
    }

    // ---- compute warps ----
    const Cell c = make_cell<COB, VR, CW>(P, tid, cpg);
    uint64_t *const publish = weight_warp ? ready : full;
    for (int k = 0; k < count; ++k) {
        const int s = k % STAGES;
        const bool ok = __all_sync(0xffffffffu, role_wait(&publish[s], static_cast<uint32_t>((k / STAGES) & 1),
                                                            abort_word, kStatusTmaTimeout));
        if (!ok) return;
        const float *xs = xs_of(s);
        const float *wk = CPG == 1 ? xs + P.x_floats : xs + P.x_floats + P.wraw_floats;
        compute_item<CPG, COB, VR, CW>(P, c, xs, wk, first + k * step);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

// ---- CTA-synchronous kernel: cp.async or TMA staging -------------------------------
// Every thread computes; stages are handed over at CTA barriers.  With TMA
// staging one thread issues the copies and polls the stage's mbarrier while
// the others wait in the hardware barrier (no issue slots spent spinning).
// Used for cp.async staging, and for depthwise layers with TMA staging,
// where a whole CTA moving in lockstep keeps the most bytes in flight.
template <int CPG, int COB, int VR, int CW, bool TMA>
__global__ void __launch_bounds__(256) direct_conv_kernel(const __grid_constant__ DirectParams P,
                                                          const __grid_constant__ CUtensorMap xmap) {
    extern __shared__ __align__(128) float smem[];
    const int cpg = CPG > 0 ? CPG : P.cpg;
    const int STAGES = P.stages;
    float *wt = smem + STAGES * P.stage_floats;
    uint64_t *bars = reinterpret_cast<uint64_t *>(wt + P.wt_floats);
    const int first = blockIdx.x, step = gridDim.x;
    const int count = first < P.items ? (P.items - 1 - first) / step + 1 : 0;
    const int tid = threadIdx.x;
    const Cell c = make_cell<COB, VR, CW>(P, tid, cpg);

    if (TMA && tid == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 1);
        fence_barrier_init();
        prefetch_tensormap(&xmap);
    }
    // Everything above touches only shared memory and parameters.
    griddep_wait();
    griddep_launch_dependents();
    if (TMA) {
        __syncthreads();
        if (tid == 0)
            for (int s = 0; s < STAGES && s < count; ++s)
                stage_with_tma(P, &xmap, smem + s * P.stage_floats, smem + s * P.stage_floats + P.x_floats,
                               &bars[s], first + s * step);
    } else {
        for (int s = 0; s < STAGES - 1; ++s) {
            if (s < count)
                stage_with_cp_async(P, smem + s * P.stage_floats, smem + s * P.stage_floats + P.x_floats,
                                    first + s * step);
            cp_async_commit();
        }
    }
    for (int k = 0; k < count; ++k) {
        const int s = k % STAGES;
        float *xs = smem + s * P.stage_floats;
        float *wr = xs + P.x_floats;
        if (TMA) {
            bool ok = true;
            if (tid == 0) ok = mbar_wait_bounded(&bars[s], static_cast<uint32_t>((k / STAGES) & 1));
            if (!__syncthreads_and(ok)) {
                // The copy engine did not deliver in time: record it, let the
                // copies still in flight land (bounded), and leave.
                if (tid == 0) {
                    raise_status(kStatusTmaTimeout);
                    for (int j = k + 1; j < k + STAGES && j < count; ++j)
                        mbar_wait_bounded(&bars[j % STAGES], static_cast<uint32_t>((j / STAGES) & 1));
                }
                return;
            }
            if (!P.bulk_w) {
                const float *wsrc = P.w + static_cast<long long>(decode_c0(P, first + k * step)) * cpg * 9;
                for (int e = tid; e < P.cb * cpg * 9; e += blockDim.x) wr[e] = __ldg(wsrc + e);
                __syncthreads();
            }
        } else {
            const int kn = k + STAGES - 1;
            if (kn < count)
                stage_with_cp_async(P, smem + (kn % STAGES) * P.stage_floats,
                                    smem + (kn % STAGES) * P.stage_floats + P.x_floats, first + kn * step);
            cp_async_commit();
            cp_async_wait_dynamic(STAGES - 1);
            __syncthreads();
        }
        if (CPG != 1) {
            transpose_weights(wr, wt, P.cb, cpg, tid, blockDim.x);
            __syncthreads();
        }
        compute_item<CPG, COB, VR, CW>(P, c, xs, CPG == 1 ? wr : wt, first + k * step);
        __syncthreads();
        if (TMA && tid == 0 && k + STAGES < count)
            stage_with_tma(P, &xmap, xs, wr, &bars[s], first + (k + STAGES) * step);
    }
    if (!TMA) cp_async_wait<0>();
}

}  // namespace gcb
