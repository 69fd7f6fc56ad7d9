// CUDA backend of the C ABI: gc_cuda_conv (reference csrc/cuda/groupconv.cu:
// 156-222 contract) and the gc_b200_* extensions.
//
// Call path: validate descriptors (common.cpp) -> support matrix of the
// requested implementation -> pointer and stream checks -> plan (cached per
// shape) -> one kernel launch on the caller's stream -> cudaGetLastError.
// Nothing here allocates memory or synchronizes; the TMA descriptor is built
// on the host and passed as a __grid_constant__ kernel parameter, so a call
// can be captured into a CUDA graph.
#include "groupconv.h"

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "device_util.cuh"
#include "kernel_direct.cuh"
#include "kernel_general.cuh"
#include "kernel_dw.cuh"
#include "kernel_wide.cuh"
#include "kernel_tf32x3.cuh"
#include "kernel_small.cuh"
#include "kernel_nhwc.cuh"
#include "kernel_probe.cuh"

namespace {

using gcb::DirectParams;
using gcb::GeneralParams;

constexpr int kStages = 3;

// The last launch's plan on this thread, kept as numbers and formatted only
// when gc_b200_last_plan asks for it (formatting costs about a third of a
// microsecond, a tenth of the host time of a call).
struct PlanRecord {
    enum Kind { kNone, kDirect, kWide, kTf32, kSmall, kGeneral, kDw, kDwS2, kNhwc } kind = kNone;
    const char *name = "";  // variant name, static storage
    bool tma = false;
    long long v[14] = {};
};
thread_local PlanRecord g_last;
thread_local std::string g_plan;

std::string format_plan(const PlanRecord &r) {
    char buf[400];
    const long long *v = r.v;
    switch (r.kind) {
    case PlanRecord::kDirect:
        std::snprintf(buf, sizeof(buf),
                      "kernel=direct_%s engine=group variant=%s grid=%lld block=%lld smem=%lld ctas_per_sm=%lld "
                      "cb=%lld bh=%lld items=%lld cells=%lld stages=%lld pitch=%lld rows=%lld bulk_w=%lld "
                      "vec_store=%lld",
                      r.tma ? "tma" : "ldg", r.name, v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7], v[8], v[9],
                      v[10], v[11], v[12]);
        break;
    case PlanRecord::kWide:
        std::snprintf(buf, sizeof(buf),
                      "kernel=direct_%s engine=wide variant=%s grid=%lld block=%lld smem=%lld ctas_per_sm=%lld "
                      "kc=%lld chunks=%lld co_item=%lld bh=%lld items=%lld cells=%lld pitch=%lld rows=%lld "
                      "vec_store=%lld",
                      r.tma ? "tma" : "ldg", r.name, v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7], v[8], v[9],
                      v[10], v[11], v[12]);
        break;
    case PlanRecord::kTf32:
        std::snprintf(buf, sizeof(buf),
                      "kernel=tf32x3 engine=tcgen05 n_cta=%lld block=320 smem=%lld M=%lld N=%lld nb=%lld sp=%lld "
                      "strips=%lld items=%lld chunks=%lld rows_b=%lld ks=%lld layout=%s",
                      v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7], v[8], v[9], v[10], r.name);
        break;
    case PlanRecord::kSmall:
        std::snprintf(buf, sizeof(buf),
                      "kernel=small grid=%lld block=%lld smem=%lld ctas_per_sm=%lld cob=%lld cb=%lld items=%lld "
                      "vec=%lld stages=%lld",
                      v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7], v[8]);
        break;
    case PlanRecord::kDw:
        std::snprintf(buf, sizeof(buf),
                      "kernel=general engine=depthwise k=%lld grid=%lld block=%lld smem=%lld bh=%lld bands=%lld "
                      "pitch=%lld items=%lld",
                      v[0], v[1], v[7], v[2], v[3], v[4], v[5], v[6]);
        break;
    case PlanRecord::kDwS2:
        std::snprintf(buf, sizeof(buf),
                      "kernel=general engine=depthwise_cells k=%lld stride=%lld grid=%lld block=256 cells=%lld "
                      "vec_in=%lld vec_out=%lld",
                      v[0], v[5], v[1], v[2], v[3], v[4]);
        break;
    case PlanRecord::kNhwc:
        std::snprintf(buf, sizeof(buf), "kernel=nhwc engine=%s grid=%lld block=%lld cpg=%lld bias=%lld rows=%lld",
                      r.name, v[0], v[1], v[2], v[3], v[4]);
        break;
    case PlanRecord::kGeneral:
        std::snprintf(buf, sizeof(buf), "kernel=general grid=%lld block=%lld run=%lld cob=%lld index=%s runs=%lld",
                      v[0], v[1], v[2], v[3], v[4] ? "32" : "64", v[5]);
        break;
    default:
        buf[0] = '\0';
    }
    return buf;
}

template <class... T>
void record_plan(PlanRecord::Kind kind, const char *name, bool tma, T... values) {
    g_last.kind = kind;
    g_last.name = name;
    g_last.tma = tma;
    const long long vals[] = {static_cast<long long>(values)...};
    for (size_t i = 0; i < sizeof...(T); ++i) g_last.v[i] = vals[i];
}

long long round_up(long long v, long long m) { return (v + m - 1) / m * m; }
long long ceil_div(long long a, long long b) { return (a + b - 1) / b; }

// ---- device facts, cached per device -----------------------------------------
struct DeviceFacts {
    int sms = 0;
    int smem_optin = 0;   // max dynamic shared memory per block (opt-in)
    int smem_per_sm = 0;  // shared memory per multiprocessor
};

std::mutex g_mutex;
std::map<int, DeviceFacts> g_facts;
std::map<std::pair<int, const void *>, bool> g_attr_done;
std::map<std::tuple<int, const void *, int, size_t>, int> g_occupancy;

int device_facts(int dev, DeviceFacts &out) {
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_facts.find(dev);
    if (it != g_facts.end()) {
        out = it->second;
        return GC_OK;
    }
    DeviceFacts f;
    cudaError_t e = cudaDeviceGetAttribute(&f.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
        e = cudaDeviceGetAttribute(&f.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e == cudaSuccess)
        e = cudaDeviceGetAttribute(&f.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    g_facts[dev] = f;
    out = f;
    return GC_OK;
}

// Opt a kernel into the device's full dynamic shared memory once, then ask
// the occupancy calculator (cached) how many CTAs fit per SM.
int kernel_occupancy(int dev, const void *fn, int threads, size_t smem, int smem_optin,
                     int &ctas) {
    std::lock_guard<std::mutex> lock(g_mutex);
    auto key = std::make_tuple(dev, fn, threads, smem);
    auto it = g_occupancy.find(key);
    if (it != g_occupancy.end()) {
        ctas = it->second;
        return GC_OK;
    }
    auto akey = std::make_pair(dev, fn);
    if (!g_attr_done[akey]) {
        cudaError_t e =
            cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_optin);
        if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
        g_attr_done[akey] = true;
    }
    int n = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, smem);
    if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    g_occupancy[key] = n;
    ctas = n;
    return GC_OK;
}

// Launch on the caller's stream with programmatic stream serialization: the
// kernel may start its prologue while the previous kernel in the stream
// drains, and waits (griddepcontrol.wait) before touching global memory.
cudaError_t launch_pdl(const void *fn, dim3 grid, dim3 block, void **args, size_t smem, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

// ---- TMA descriptor encoding ---------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_error = cudaSuccess;

int tensor_map_encoder(PFN_cuTensorMapEncodeTiled_v12000 &fn) {
    std::call_once(g_encode_once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        g_encode_error =
            cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q);
        if (g_encode_error == cudaSuccess && q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    if (g_encode == nullptr) {
        const char *why = g_encode_error != cudaSuccess ? cudaGetErrorString(g_encode_error)
                                                        : "cuTensorMapEncodeTiled not found";
        return gc_error(GC_DEVICE_ERROR, why);
    }
    fn = g_encode;
    return GC_OK;
}

// 4-D map over an NCHW float tensor: dims (W, H, C, N), box (bw, bh, bc, 1),
// out-of-range elements read as zero.
int encode_nchw_map(CUtensorMap &map, const float *base, long long n, long long c, long long h,
                    long long w, int bw, int bh, int bc) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    int st = tensor_map_encoder(encode);
    if (st != GC_OK) return st;
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(w), static_cast<cuuint64_t>(h),
                          static_cast<cuuint64_t>(c), static_cast<cuuint64_t>(n)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(w) * 4, static_cast<cuuint64_t>(h * w) * 4,
                             static_cast<cuuint64_t>(c * h * w) * 4};
    cuuint32_t box[4] = {static_cast<cuuint32_t>(bw), static_cast<cuuint32_t>(bh),
                         static_cast<cuuint32_t>(bc), 1u};
    cuuint32_t estride[4] = {1, 1, 1, 1};
    CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float *>(base), dims,
                        strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return gc_error(GC_DEVICE_ERROR, "cuTensorMapEncodeTiled failed");
    return GC_OK;
}

// 4-D map over a channels-last float tensor: dims (C, W, H, N), box (bc, bw,
// bh, 1), out-of-range elements read as zero (C % 4 == 0: every stride is a
// multiple of 16 bytes).
int encode_nhwc_map(CUtensorMap &map, const float *base, long long n, long long c, long long h, long long w,
                    int bc, int bw, int bh) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    int st = tensor_map_encoder(encode);
    if (st != GC_OK) return st;
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(c), static_cast<cuuint64_t>(w), static_cast<cuuint64_t>(h),
                          static_cast<cuuint64_t>(n)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(c) * 4, static_cast<cuuint64_t>(w * c) * 4,
                             static_cast<cuuint64_t>(h * w * c) * 4};
    cuuint32_t box[4] = {static_cast<cuuint32_t>(bc), static_cast<cuuint32_t>(bw), static_cast<cuuint32_t>(bh), 1u};
    cuuint32_t estride[4] = {1, 1, 1, 1};
    CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float *>(base), dims, strides, box,
                        estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return gc_error(GC_DEVICE_ERROR, "cuTensorMapEncodeTiled failed");
    return GC_OK;
}

// 2-D map over a row-major float matrix [rows][cols] (cols * 4 a multiple of
// 16 bytes): box (bw, bh), element (col, row) coordinates.
int encode_rows_map(CUtensorMap &map, const float *base, long long rows, long long cols, int bw, int bh) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    int st = tensor_map_encoder(encode);
    if (st != GC_OK) return st;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 4};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(bw), static_cast<cuuint32_t>(bh)};
    cuuint32_t estride[2] = {1, 1};
    CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box,
                        estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return gc_error(GC_DEVICE_ERROR, "cuTensorMapEncodeTiled failed");
    return GC_OK;
}

// ---- direct engines: variants, planning, launch ----------------------------------
struct Variant {
    const char *name;
    int cob, vr;
    int cw;  // columns per thread (direct kernels)
    const void *fn_tma;
    const void *fn_ldg;
    bool ws;  // TMA staging runs the warp-specialized kernel (else CTA-synchronous)
};

// TMA staging: depthwise layers run the CTA-synchronous kernel (measured
// faster on HBM-bound shapes), grouped layers the warp-specialized one.
// LDG = false: TMA staging only (no cp.async instance; the planner skips the
// variant for shapes TMA cannot stage).
template <int CPG, int COB, int VR, int CW, bool LDG = true>
Variant make_variant(const char *name) {
    const void *tma_fn;
    if constexpr (CPG == 1)
        tma_fn = reinterpret_cast<const void *>(&gcb::direct_conv_kernel<CPG, COB, VR, CW, true>);
    else
        tma_fn = reinterpret_cast<const void *>(&gcb::direct_ws_kernel<CPG, COB, VR, CW>);
    const void *ldg_fn = nullptr;
    if constexpr (LDG) ldg_fn = reinterpret_cast<const void *>(&gcb::direct_conv_kernel<CPG, COB, VR, CW, false>);
    return Variant{name, COB, VR, CW, tma_fn, ldg_fn, CPG != 1};
}

template <int COB, int VR>
Variant make_wide(const char *name) {
    return Variant{name, COB, VR, 4,
                   reinterpret_cast<const void *>(&gcb::wide_conv_kernel<COB, VR, true, kStages>),
                   reinterpret_cast<const void *>(&gcb::wide_conv_kernel<COB, VR, false, kStages>), false};
}

// Full-group kernel variants that can serve a group width (first = preferred).
std::vector<const Variant *> small_variants(long long cpg) {
    // name: d<cpg> + cell shape (out-channels COB x rows VR x columns CW)
    static const Variant d1 = make_variant<1, 1, 4, 4>("d1");
    static const Variant d1r8 = make_variant<1, 1, 8, 4>("d1r8");
    static const Variant d2 = make_variant<2, 2, 4, 4>("d2");
    static const Variant d4 = make_variant<4, 4, 2, 4>("d4");
    static const Variant d4q = make_variant<4, 2, 4, 4>("d4q");
    static const Variant d4o1 = make_variant<4, 4, 1, 8, false>("d4o1");
    static const Variant d8h = make_variant<8, 4, 2, 4>("d8h");
    static const Variant d8v4 = make_variant<8, 4, 4, 4>("d8v4");
    static const Variant d8q = make_variant<8, 2, 4, 4>("d8q");
    static const Variant d8o41 = make_variant<8, 4, 1, 8, false>("d8o41");
    static const Variant d16h = make_variant<16, 4, 2, 4, false>("d16h");
    static const Variant d16q = make_variant<16, 2, 4, 4, false>("d16q");
    static const Variant d16o41 = make_variant<16, 4, 1, 8, false>("d16o41");
    static const Variant gen = make_variant<0, 1, 4, 4>("g1");
    if (cpg == 1) return {&d1r8, &d1};
    if (cpg == 2) return {&d2};
    if (cpg == 4) return {&d4, &d4q, &d4o1};
    if (cpg == 8) return {&d8h, &d8v4, &d8q, &d8o41};
    if (cpg == 16) return {&d16h, &d16q, &d16o41};  // TMA staging only
    return {&gen};
}

// Channel-chunked kernel variant for wide groups.
const Variant &wide_variant(long long cpg) {
    static const Variant w8 = make_wide<8, 2>("w8");
    static const Variant w4 = make_wide<4, 2>("w4");
    static const Variant w1 = make_wide<1, 4>("w1");
    if (cpg % 8 == 0) return w8;
    if (cpg % 4 == 0) return w4;
    return w1;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Whether the TMA staging can serve this shape and this input pointer.
bool tma_eligible(const gc_shape *p, const void *x) {
    return p->w % 4 == 0 && p->w + 8 <= 256 && aligned16(x) && p->h < (1ll << 30) &&
           p->cin < (1ll << 30) && p->n < (1ll << 30);
}

// Everything a launch needs except the three data pointers.
struct EnginePlan {
    bool wide = false;
    const Variant *var = nullptr;
    bool tma = false;
    int threads = 0;
    size_t smem = 0;
    int grid = 0;
    int ctas_per_sm = 0;
    DirectParams D;  // valid when !wide
    gcb::WideParams Wp;  // valid when wide
};

// Fraction of the machine a persistent grid keeps busy: with fewer items than
// CTA slots, the share of SMs that get work; otherwise the fill of the last
// wave.
double grid_balance(long long items, long long slots, int sms) {
    if (items <= slots) {
        const long long per_sm = ceil_div(items, sms);
        return static_cast<double>(items) / (static_cast<double>(per_sm) * sms);
    }
    const long long waves = ceil_div(items, slots);
    return static_cast<double>(items) / (static_cast<double>(waves) * slots);
}

// Shared scoring of a candidate tiling: load balance of the persistent grid,
// thread utilisation, the input re-read factor (halo rows, output-channel
// blocks) and the latency-hiding capacity of the SM.
double score_tiling(long long items, long long slots, long long cells, int threads, double reread,
                    int ctas, double stage_bytes) {
    const long long waves = ceil_div(items, slots);
    const double balance = static_cast<double>(items) / (static_cast<double>(waves) * slots);
    const double cell_eff = static_cast<double>(cells) / (ceil_div(cells, threads) * threads);
    double score = std::min(balance, 1.0) * cell_eff / (1.0 + 0.15 * (reread - 1.0));
    const double warps = ctas * threads / 32.0;
    if (warps < 16) score *= 0.75 + 0.25 * warps / 16.0;
    const double inflight = ctas * (kStages - 1) * stage_bytes;
    if (inflight < 48.0 * 1024) score *= 0.8 + 0.2 * inflight / (48.0 * 1024);
    return score;
}

const std::vector<long long> band_candidates(long long H) {
    return {H, ceil_div(H, 2), ceil_div(H, 3), ceil_div(H, 4), ceil_div(H, 7), 64, 32, 28, 16, 14, 8, 4, 2, 1};
}

// Estimated fraction of a direct-kernel thread's instructions that are FFMA:
// per input channel a cell loads VR+2 row segments (CW/4 16-byte loads, two
// shuffles, two predicated edge loads, two selects each) and its weights, and
// per item it pays a fixed cost (item decode, barriers, output addresses) plus
// its stores.
double issue_efficiency(const Variant &var, long long cpg) {
    const double vr = var.vr, cob = var.cob, cw = var.cw;
    const double ffma = cob * vr * 9.0 * cw * cpg;
    const double rows = (vr + 2) * (6.0 + cw / 4.0) * cpg;
    const double weights = cpg == 1 ? 9.0 : 9.0 * std::ceil(cob / 4.0) * cpg;
    const double fixed = 40.0 + vr * cob * 0.75 * cw;
    return ffma / (ffma + rows + weights + fixed);
}

// Row pitch (floats) of the direct kernel's tile: the smallest multiple of 4
// holding 4*qcols + 8 columns whose warp-wide 16-byte loads need the fewest
// shared-memory wavefronts, found by replaying the lane -> address map of
// the first warps (8 lanes of 16 bytes fill the 32 banks once; distinct
// addresses in the same 16-byte bank group serialize).
int choose_pitch(int W, int qcols, int cw, int rblocks, int vr, int rows, int cells, int cob, int cpg,
                 bool tma) {
    const int base = static_cast<int>(round_up(static_cast<long long>(cw) * qcols + 8, 4));
    int best = base, best_cost = 1 << 30;
    for (int p = base; p <= base + 60; p += 4) {
        if (tma && p > 256) break;
        // exact per-lane addresses: channel block, row block (rb * vr rows),
        // quad, in the kernel's cell order (make_cell: quad fastest below 8
        // channels per group, row block fastest from 8 on)
        const int warps = std::min((cells + 31) / 32, 8);
        int cost = 0;
        for (int wp = 0; wp < warps; ++wp) {
            long long addr[32];
            for (int lane = 0; lane < 32; ++lane) {
                const int cell = std::min(wp * 32 + lane, cells - 1);
                int q, rb, cbk;
                if (cpg < 8) {
                    q = cell % qcols;
                    rb = (cell / qcols) % rblocks;
                    cbk = cell / qcols / rblocks;
                } else {
                    rb = cell % rblocks;
                    q = (cell / rblocks) % qcols;
                    cbk = cell / rblocks / qcols;
                }
                const int g = cbk * cob / cpg;
                addr[lane] = ((static_cast<long long>(g) * cpg * rows + rb * vr) * p + q * cw + 4) * 4;
            }
            // Below 8 channels per group: the warp's distinct addresses per
            // 16-byte bank group (the model these tiles were tuned with).
            // From 8 on (16-byte loads served in four phases of 8 lanes): per
            // phase, the most distinct addresses in one bank group, summed
            // over the phases.
            const int phases = cpg < 8 ? 1 : 4, width = 32 / phases;
            for (int ph = 0; ph < phases; ++ph) {
                int worst = 0;
                for (int bank = 0; bank < 8; ++bank) {
                    long long seen[32];
                    int n = 0;
                    for (int lane = ph * width; lane < (ph + 1) * width; ++lane) {
                        if ((addr[lane] / 16) % 8 != bank) continue;
                        bool dup = false;
                        for (int i = 0; i < n; ++i) dup |= seen[i] == addr[lane];
                        if (!dup) seen[n++] = addr[lane];
                    }
                    worst = std::max(worst, n);
                }
                cost += worst;
            }
        }
        if (cost < best_cost) {
            best_cost = cost;
            best = p;
        }
    }
    (void)W;
    return best;
}

// Full-group tiling (kernel_direct.cuh) for groups of fewer than 16 channels.
// Every CTA thread owns one cell, so a candidate needs cells <= 256; the
// block is the cells rounded up to whole warps.
int plan_small(const gc_shape *p, bool tma, bool w_aligned, bool y_aligned, int dev,
               const DeviceFacts &facts, EnginePlan &out, bool &found,
               std::vector<std::pair<double, EnginePlan>> *cands = nullptr) {
    const long long N = p->n, C = p->cin, H = p->h, W = p->w, cpg = p->cin / p->groups;
    const long long groups = p->groups;
    const bool compute_bound = cpg >= 4;
    double best = -1.0;
    found = false;
    for (const Variant *vp : small_variants(cpg)) {
        const Variant &var = *vp;
        if (!tma && var.fn_ldg == nullptr) continue;
        const int vr = var.vr;
        const long long qcols = ceil_div(W, var.cw);
        for (long long gpi = 1; gpi <= groups; ++gpi) {
            if (groups % gpi != 0) continue;
            const long long cb = gpi * cpg;
            if (cb > std::max<long long>(cpg, 64)) break;
            for (long long bh : band_candidates(H)) {
                if (bh < 1 || bh > H) continue;
                if (bh != H && bh % vr != 0) continue;
                const long long rblocks = ceil_div(bh, vr);
                const long long cells = (cb / var.cob) * rblocks * qcols;
                if (cells > 256) continue;
                const long long rows = rblocks * vr + 2;
                if (tma && (rows > 256 || cb > 256)) continue;
                const long long bands = ceil_div(H, bh);
                const long long items = N * (C / cb) * bands;
                if (items >= (1LL << 31)) continue;
                const int bulk_w = (tma && w_aligned && (cb * cpg) % 4 == 0) ? 1 : 0;
                const bool ws = tma && var.ws;
                // the warp-specialized kernel adds the copy warp and, when
                // weights need work, the weight warp
                const int threads = static_cast<int>(round_up(cells, 32)) +
                                    (ws ? 32 * gcb::direct_ws_producer_warps(static_cast<int>(cpg), bulk_w) : 0);
                if (threads > (ws ? gcb::kWsMaxThreads : 256)) continue;
                const int pitch = choose_pitch(static_cast<int>(W), static_cast<int>(qcols), var.cw,
                                               static_cast<int>(rblocks), vr, static_cast<int>(rows),
                                               static_cast<int>(cells), var.cob, static_cast<int>(cpg), tma);
                if (tma && pitch > 256) continue;
                const long long xf = round_up(cb * rows * pitch, 32);
                const long long wf = round_up(cb * cpg * 9, 32);
                const long long wtf = cpg == 1 ? 0 : wf;  // transposed copy
                // warp-specialized: x, raw and transposed weights per stage,
                // then full / ready / empty barriers and the abort word;
                // CTA-synchronous: x and raw weights per stage, one
                // transposed copy, one barrier per stage.
                const long long stage_floats = ws ? xf + wf + wtf : xf + wf;
                for (int stages = 2; stages <= gcb::kMaxStages; ++stages) {
                    const size_t smem =
                        ws ? static_cast<size_t>(stages * stage_floats * 4 + 3 * 8 * gcb::kMaxStages + 16)
                           : static_cast<size_t>((stages * stage_floats + wtf) * 4 + 8 * gcb::kMaxStages);
                    if (smem > static_cast<size_t>(facts.smem_optin)) break;
                    int ctas = 0;
                    int st = kernel_occupancy(dev, tma ? var.fn_tma : var.fn_ldg, threads, smem,
                                              facts.smem_optin, ctas);
                    if (st != GC_OK) return st;
                    if (ctas < 1) continue;
                    const long long slots = static_cast<long long>(facts.sms) * ctas;
                    const double balance = grid_balance(items, slots, facts.sms);
                    const double cell_eff = static_cast<double>(cells) / round_up(cells, 32);
                    // An SM overlaps the staging of its next items with compute
                    // only when it holds several items (in one CTA or several:
                    // while one CTA waits for its stage, another computes).
                    const double per_cta =
                        static_cast<double>(items) / std::min(items, static_cast<long long>(facts.sms));
                    const double halo = static_cast<double>(rows) / bh;
                    // compute warps per SM (the copy and weight warps of the
                    // warp-specialized kernel do no FFMAs)
                    const double warps = ctas * std::ceil(cells / 32.0);
                    // rows computed past the image in the last band
                    const double band_eff = static_cast<double>(H) / (bands * rblocks * vr);
                    double score = balance * issue_efficiency(var, cpg);
                    if (compute_bound) {
                        score *= cell_eff * band_eff / (1.0 + 0.05 * (halo - 1.0));
                        score *= std::min(1.0, 0.55 + 0.45 * warps / 16.0);
                    } else {
                        score *= cell_eff;
                        score /= 1.0 + 0.15 * (halo - 1.0);
                        score *= std::min(1.0, 0.75 + 0.25 * warps / 16.0);
                        score *= std::min(1.0, 0.6 + 0.4 * (per_cta - 1.0) / 3.0);
                        const double inflight = ctas * (stages - 1) * (xf + wf) * 4.0;
                        score *= std::min(1.0, 0.7 + 0.3 * inflight / (64.0 * 1024));
                    }
                    EnginePlan cand;
                    DirectParams &P = cand.D;
                    std::memset(&P, 0, sizeof(P));
                    P.n = static_cast<int>(N);
                    P.c = static_cast<int>(C);
                    P.h = static_cast<int>(H);
                    P.wd = static_cast<int>(W);
                    P.cpg = static_cast<int>(cpg);
                    P.cb = static_cast<int>(cb);
                    P.bh = static_cast<int>(bh);
                    P.bands = static_cast<int>(bands);
                    P.cblocks = static_cast<int>(C / cb);
                    P.items = static_cast<int>(items);
                    P.pitch = pitch;
                    P.rows = static_cast<int>(rows);
                    P.x_floats = static_cast<int>(xf);
                    P.wraw_floats = static_cast<int>(wf);
                    P.stage_floats = static_cast<int>(stage_floats);
                    P.wt_floats = static_cast<int>(wtf);
                    P.qcols = static_cast<int>(qcols);
                    P.rblocks = static_cast<int>(rblocks);
                    P.cells = static_cast<int>(cells);
                    P.stages = stages;
                    P.vec_store = (W % 4 == 0 && y_aligned) ? 1 : 0;
                    P.bulk_w = bulk_w;
                    P.x_bytes = static_cast<unsigned>(pitch * rows * cb * 4);
                    P.w_bytes = static_cast<unsigned>(cb * cpg * 9 * 4);
                    cand.wide = false;
                    cand.var = &var;
                    cand.tma = tma;
                    cand.threads = threads;
                    cand.smem = smem;
                    cand.ctas_per_sm = ctas;
                    cand.grid = static_cast<int>(std::min<long long>(items, slots));
                    if (cands != nullptr) cands->emplace_back(score, cand);
                    if (score <= best + 1e-9) continue;
                    best = score;
                    found = true;
                    out = cand;
                }
            }
        }
    }
    return GC_OK;
}

// Channel-chunked tiling (kernel_wide.cuh): any group width.
int plan_wide(const gc_shape *p, bool tma, bool y_aligned, int dev, const DeviceFacts &facts,
              EnginePlan &out, bool &found) {
    const long long N = p->n, C = p->cin, H = p->h, W = p->w, cpg = p->cin / p->groups;
    const Variant &var = wide_variant(cpg);
    const int vr = var.vr, cob = var.cob;
    const int pitch = round_up((W) + 8, 4);
    const long long qcols = ceil_div(W, 4);
    const size_t budget = std::min<size_t>(static_cast<size_t>(facts.smem_optin), 112 * 1024);
    double best = -1.0;
    found = false;
    for (int threads : {256, 128}) {
        for (long long co_item = cob; co_item < cpg + cob; co_item += cob) {
            const long long coblocks = ceil_div(cpg, co_item);
            for (long long bh : band_candidates(H)) {
                if (bh < 1 || bh > H) continue;
                if (bh != H && bh % vr != 0) continue;
                const long long cells = (co_item / cob) * ceil_div(bh, vr) * qcols;
                if (cells > threads) continue;
                const long long rows = round_up((bh), vr) + 2;
                if (tma && rows > 256) continue;
                const long long row_floats = rows * pitch;
                // Largest chunk whose stages fit the budget, at most the group.
                long long kc = std::min<long long>(cpg, 256);
                while (kc > 1 && kStages * round_up((kc * row_floats), 32) * 4 + 64 >
                                     static_cast<long long>(budget))
                    --kc;
                const long long xf = round_up((kc * row_floats), 32);
                const size_t smem = static_cast<size_t>(kStages * xf * 4 + 64);
                if (smem > static_cast<size_t>(facts.smem_optin)) continue;
                const long long bands = ceil_div(H, bh);
                const long long items = N * p->groups * bands * coblocks;
                int ctas = 0;
                int st = kernel_occupancy(dev, tma ? var.fn_tma : var.fn_ldg, threads, smem,
                                          facts.smem_optin, ctas);
                if (st != GC_OK) return st;
                if (ctas < 1) continue;
                const long long slots = static_cast<long long>(facts.sms) * ctas;
                const double reread = static_cast<double>(rows) / bh * coblocks;
                const double score = score_tiling(items, slots, cells, threads, reread, ctas, xf * 4.0);
                if (score <= best + 1e-9) continue;
                best = score;
                found = true;
                gcb::WideParams &P = out.Wp;
                std::memset(&P, 0, sizeof(P));
                P.n = static_cast<int>(N);
                P.c = static_cast<int>(C);
                P.h = static_cast<int>(H);
                P.wd = static_cast<int>(W);
                P.cpg = static_cast<int>(cpg);
                P.groups = static_cast<int>(p->groups);
                P.kc = static_cast<int>(kc);
                P.chunks = static_cast<int>(ceil_div(cpg, kc));
                P.co_item = static_cast<int>(co_item);
                P.coblocks = static_cast<int>(coblocks);
                P.bh = static_cast<int>(bh);
                P.bands = static_cast<int>(bands);
                P.items = items;
                P.pitch = pitch;
                P.rows = static_cast<int>(rows);
                P.x_floats = static_cast<int>(xf);
                P.qcols = static_cast<int>(qcols);
                P.rblocks = static_cast<int>(ceil_div(bh, vr));
                P.cells = static_cast<int>(cells);
                P.vec_store = (W % 4 == 0 && y_aligned) ? 1 : 0;
                P.x_bytes = static_cast<unsigned>(pitch * rows * kc * 4);
                out.wide = true;
                out.var = &var;
                out.tma = tma;
                out.threads = threads;
                out.smem = smem;
                out.ctas_per_sm = ctas;
                out.grid = static_cast<int>(std::min<long long>(items, slots));
            }
        }
    }
    return GC_OK;
}

using PlanKey = std::tuple<int, long long, long long, long long, long long, long long, int>;
std::map<PlanKey, EnginePlan> g_plans;

// Plan for the direct engines, cached per (device, shape, staging, alignment).
int plan_engine(const gc_shape *p, const float *w, const float *y, bool tma, int dev,
                EnginePlan &plan) {
    const bool w_al = aligned16(w), y_al = aligned16(y);
    const PlanKey key{dev, p->n, p->cin, p->h, p->w, p->groups,
                      (tma ? 1 : 0) | (w_al ? 2 : 0) | (y_al ? 4 : 0)};
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        auto it = g_plans.find(key);
        if (it != g_plans.end()) {
            plan = it->second;
            return GC_OK;
        }
    }
    const long long N = p->n, C = p->cin, H = p->h, W = p->w;
    if (H > (1 << 30) || W > (1 << 20) || C > (1 << 30) || N > (1 << 30))
        return gc_error(GC_UNSUPPORTED, "direct engine: tensor extent beyond its 32-bit tile indices");
    DeviceFacts facts;
    int st = device_facts(dev, facts);
    if (st != GC_OK) return st;
    bool found = false;
    const long long cpg = p->cin / p->groups;
    if (cpg < 16 || (cpg == 16 && tma)) {
        st = plan_small(p, tma, w_al, y_al, dev, facts, plan, found);
        if (st != GC_OK) return st;
    }
    if (!found) {
        st = plan_wide(p, tma, y_al, dev, facts, plan, found);
        if (st != GC_OK) return st;
    }
    if (!found) return gc_error(GC_UNSUPPORTED, "direct engine: no tile fits in shared memory");
    std::lock_guard<std::mutex> lock(g_mutex);
    g_plans[key] = plan;
    return GC_OK;
}

// Launches one planned direct-engine kernel (the plan is a copy; its data
// pointers and epilogue are filled in here).
int launch_plan(EnginePlan plan, const gc_shape *p, const float *x, const float *w, float *y, bool tma,
                cudaStream_t stream, const float *bias, int act) {
    int st = GC_OK;
    if (plan.wide && (bias != nullptr || act != gcb::kActNone))
        return gc_error(GC_UNSUPPORTED, "channel-chunked kernel: no bias or activation epilogue");
    CUtensorMap map;
    std::memset(&map, 0, sizeof(map));
    void *args[2];
    if (!plan.wide) {
        plan.D.x = x;
        plan.D.w = w;
        plan.D.y = y;
        plan.D.bias = bias;
        plan.D.act = act;
        if (tma) {
            st = encode_nchw_map(map, x, p->n, p->cin, p->h, p->w, plan.D.pitch, plan.D.rows, plan.D.cb);
            if (st != GC_OK) return st;
        }
        args[0] = &plan.D;
    } else {
        plan.Wp.x = x;
        plan.Wp.w = w;
        plan.Wp.y = y;
        if (tma) {
            st = encode_nchw_map(map, x, p->n, p->cin, p->h, p->w, plan.Wp.pitch, plan.Wp.rows, plan.Wp.kc);
            if (st != GC_OK) return st;
        }
        args[0] = &plan.Wp;
    }
    args[1] = &map;
    const void *fn = tma ? plan.var->fn_tma : plan.var->fn_ldg;
    cudaError_t e = launch_pdl(fn, dim3(plan.grid), dim3(plan.threads), args, plan.smem, stream);
    if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    if (!plan.wide)
        record_plan(PlanRecord::kDirect, plan.var->name, tma, plan.grid, plan.threads, plan.smem, plan.ctas_per_sm,
                    plan.D.cb, plan.D.bh, plan.D.items, plan.D.cells, plan.D.stages, plan.D.pitch, plan.D.rows,
                    plan.D.bulk_w, plan.D.vec_store);
    else
        record_plan(PlanRecord::kWide, plan.var->name, tma, plan.grid, plan.threads, plan.smem, plan.ctas_per_sm,
                    plan.Wp.kc, plan.Wp.chunks, plan.Wp.co_item, plan.Wp.bh, plan.Wp.items, plan.Wp.cells,
                    plan.Wp.pitch, plan.Wp.rows, plan.Wp.vec_store);
    return GC_OK;
}

int launch_direct(const gc_shape *p, const float *x, const float *w, float *y, bool tma, int dev,
                  cudaStream_t stream, const float *bias = nullptr, int act = gcb::kActNone) {
    EnginePlan plan;
    int st = plan_engine(p, w, y, tma, dev, plan);
    if (st != GC_OK) return st;
    return launch_plan(plan, p, x, w, y, tma, stream, bias, act);
}

// Benchmark mode for the direct engines: time the planner's best-scored
// candidate tilings (up to `candidates`) on the caller's buffers and store
// the fastest in the plan cache, where every later call of the shape finds
// it.  Synchronizes the stream; y ends with the result of the chosen plan.
int autotune_direct(const gc_shape *p, const float *x, const float *w, float *y, bool tma, int dev,
                    cudaStream_t stream, int candidates) {
    DeviceFacts facts;
    int st = device_facts(dev, facts);
    if (st != GC_OK) return st;
    const long long cpg = p->cin / p->groups;
    if (!(cpg < 16 || (cpg == 16 && tma))) return GC_OK;  // the channel-chunked kernel has no candidates
    std::vector<std::pair<double, EnginePlan>> cands;
    EnginePlan best_plan;
    bool found = false;
    st = plan_small(p, tma, aligned16(w), aligned16(y), dev, facts, best_plan, found, &cands);
    if (st != GC_OK) return st;
    if (!found) return GC_OK;
    std::stable_sort(cands.begin(), cands.end(),
                     [](const auto &a, const auto &b) { return a.first > b.first; });
    if (static_cast<int>(cands.size()) > candidates) cands.resize(candidates);
    cudaEvent_t ev[2];
    cudaError_t e = cudaEventCreate(&ev[0]);
    if (e == cudaSuccess) e = cudaEventCreate(&ev[1]);
    if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    float best_ms = -1.0f;
    size_t best_i = 0;
    for (size_t i = 0; i < cands.size() && st == GC_OK; ++i) {
        st = launch_plan(cands[i].second, p, x, w, y, tma, stream, nullptr, gcb::kActNone);  // warm-up
        if (st != GC_OK) break;
        e = cudaEventRecord(ev[0], stream);
        for (int r = 0; r < 3 && e == cudaSuccess && st == GC_OK; ++r)
            st = launch_plan(cands[i].second, p, x, w, y, tma, stream, nullptr, gcb::kActNone);
        if (e == cudaSuccess) e = cudaEventRecord(ev[1], stream);
        if (e == cudaSuccess) e = cudaEventSynchronize(ev[1]);
        float ms = 0.0f;
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, ev[0], ev[1]);
        if (e != cudaSuccess) st = gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
        if (st == GC_OK && (best_ms < 0.0f || ms < best_ms)) {
            best_ms = ms;
            best_i = i;
        }
    }
    cudaEventDestroy(ev[0]);
    cudaEventDestroy(ev[1]);
    if (st != GC_OK) return st;
    {
        const PlanKey key{dev, p->n, p->cin, p->h, p->w, p->groups,
                          (tma ? 1 : 0) | (aligned16(w) ? 2 : 0) | (aligned16(y) ? 4 : 0)};
        std::lock_guard<std::mutex> lock(g_mutex);
        g_plans[key] = cands[best_i].second;
    }
    return launch_plan(cands[best_i].second, p, x, w, y, tma, stream, nullptr, gcb::kActNone);
}

// ---- tcgen05 3xTF32 implicit GEMM ------------------------------------------------------
// Output channels per tensor-path item (the kernel's CO): the widest
// multiple of 8 up to 64 dividing the group (the whole group up to 64
// channels; blocks of wider groups and of dense layers).  0: not served
// (groups that are not a multiple of 8 channels).
long long tf32_co(long long cpg) {
    for (long long co = 64; co >= 8; co -= 8)
        if (cpg % co == 0) return co;
    return 0;
}
bool tf32_cpg_supported(long long cpg) { return tf32_co(cpg) != 0; }

// Pixel rows per step and shared memory of the tensor-core path for a shape:
// weights staged twice, A tiles of max(64, 2 cpg) rows twice, hi/lo pixel
// tiles twice, the epilogue buffers and the barrier block.
constexpr size_t kTf32SmemLimit = 227 * 1024;  // B200 opt-in shared memory per block
long long tf32_rows_b(long long w, int sp) { return round_up(sp * gcb::kTf32N + 2 * (w + 2) + 2, 8); }
size_t tf32_smem(long long cpg, long long w, int sp) {
    const long long co = tf32_co(cpg);
    const long long m = 2 * co > 64 ? 128 : 64;
    return static_cast<size_t>(2 * co * 72 * 4 + 2 * 9 * m * 32 + 4 * tf32_rows_b(w, sp) * 32 +
                               gcb::kConvWarps * gcb::kTf32EpiFloats * 4 + 128);
}
bool tf32_fits(long long cpg, long long w, int sp, size_t limit) {
    return tf32_rows_b(w, sp) <= gcb::kTf32MaxRows && tf32_smem(cpg, w, sp) <= limit;
}

// Whether the tensor-core path can serve this shape: a supported group width,
// 16-byte aligned weights (TMA-staged), one 256-pixel strip plus its
// 2*(W+2)+2 halo rows within the converters' reach and shared memory, and
// 32-bit pixel indices.  Inputs are read with plain loads: any width, any
// alignment.
bool tf32_eligible(const gc_shape *p, const void *x, const void *w) {
    (void)x;
    const long long cpg = p->cin / p->groups;
    return tf32_cpg_supported(cpg) && aligned16(w) && tf32_fits(cpg, p->w, 1, kTf32SmemLimit) &&
           (p->h + 2) * (p->w + 2) < (1LL << 30) &&
           p->n < (1LL << 30) && p->cin < (1LL << 30);
}

struct Tf32Plan {
    gcb::Tf32Params P;
    const void *fn = nullptr;
    size_t smem = 0;
    int grid = 0;
};

// Kernel instance for an output-channel block width and the pixel rows per
// step (two or four rows per converter thread).
template <int CO>
const void *tf32_instance(bool two, bool nhwc) {
    if (nhwc)
        return two ? reinterpret_cast<const void *>(&gcb::tf32x3_conv_kernel<CO, 2, true>)
                   : reinterpret_cast<const void *>(&gcb::tf32x3_conv_kernel<CO, 4, true>);
    return two ? reinterpret_cast<const void *>(&gcb::tf32x3_conv_kernel<CO, 2>)
               : reinterpret_cast<const void *>(&gcb::tf32x3_conv_kernel<CO, 4>);
}
const void *tf32_kernel_for(long long co, long long rows_b, bool nhwc) {
    const bool two = rows_b <= 2 * gcb::kConvThreads;
    switch (co) {
    case 8: return tf32_instance<8>(two, nhwc);
    case 16: return tf32_instance<16>(two, nhwc);
    case 24: return tf32_instance<24>(two, nhwc);
    case 32: return tf32_instance<32>(two, nhwc);
    case 40: return tf32_instance<40>(two, nhwc);
    case 48: return tf32_instance<48>(two, nhwc);
    case 56: return tf32_instance<56>(two, nhwc);
    case 64: return tf32_instance<64>(two, nhwc);
    default: return nullptr;
    }
}

// Work split of the tensor-core path: images stacked per block, 256-pixel
// strips per item (one, or two for 64-channel groups of large planes), items
// in waves over the SMs.
int plan_tf32(const gc_shape *p, int dev, Tf32Plan &out, bool nhwc = false) {
    DeviceFacts facts;
    int st = device_facts(dev, facts);
    if (st != GC_OK) return st;
    const long long N = p->n, C = p->cin, H = p->h, W = p->w, cpg = C / p->groups;
    const long long co = tf32_co(cpg), co_blocks = cpg / co;
    const long long wp = W + 2, hp2 = H + 2;
    const size_t limit = std::min(kTf32SmemLimit, static_cast<size_t>(facts.smem_optin));
    if (!tf32_fits(cpg, W, 1, limit)) return gc_error(GC_UNSUPPORTED, "3xTF32 path: pixel strip does not fit");
    // Images per block and strips per item.  Every 256-pixel strip costs the
    // same MMA time; two strips per item share the chunk's weights (half the
    // weight work per pixel, fewer halo rows) but finish an item's MMAs
    // before its epilogue, so they must not cost more waves than +15 %, and
    // the item needs at least 4 steps to amortize that epilogue (measured:
    // 16-channel groups, 2 steps per item, lose 16 % with two strips; 32- and
    // 64-channel groups of large planes gain up to 10 %).  Stacked small
    // images keep one strip per item.
    long long best_nb = 1, best_items = 0, best_strips = 0, best_ks = 1;
    int best_sp = 1;
    const long long chunks = cpg / 8;
    double best_cost = -1.0;
    for (int sp = 1; sp <= (chunks >= 4 ? 2 : 1); ++sp) {
        if (!tf32_fits(cpg, W, sp, limit)) continue;
        for (long long nb = 1; nb <= N; ++nb) {
            if (sp == 2 && nb > 1) break;
            const long long out_rows = (nb - 1) * hp2 + H;
            if (nb > 1 && out_rows * wp > 16 * gcb::kTf32N) break;  // stacking only pays for small planes
            if (nb * hp2 * wp >= (1LL << 30)) break;
            const long long strips = ceil_div(out_rows * wp, sp * gcb::kTf32N);
            const long long items = static_cast<long long>(p->groups) * co_blocks * ceil_div(N, nb) * strips;
            if (items >= (1LL << 31)) continue;
            // Too few output tiles for the GPU: split the input channels
            // into parts (a divisor of the chunks) so that the
            // serial chain of steps per CTA shrinks; the split minimizes
            // waves x (steps per item + 1), the +1 for an item's prologue and
            // epilogue (measured: N32 C256 7x7 dense 37.1 -> 34.4 us with 8
            // parts in 3 waves against 2 parts in one wave).
            long long ks = 1;
            if (sp == 1 && 2 * items <= facts.sms) {
                double best_split = -1.0;
                for (long long d = 1; d <= chunks; ++d) {
                    if (chunks % d != 0) continue;
                    const double c = static_cast<double>(ceil_div(items * d, facts.sms)) * (chunks / d + 1);
                    if (best_split < 0.0 || c < best_split - 1e-9) {
                        best_split = c;
                        ks = d;
                    }
                }
            }
            // estimated time: waves of items x steps per item
            const double cost = static_cast<double>(ceil_div(items * ks, facts.sms)) * (chunks / ks) * sp *
                                (sp == 2 ? 0.87 : 1.0);
            if (best_cost < 0.0 || cost < best_cost - 1e-9) {
                best_cost = cost;
                best_nb = nb;
                best_items = items * ks;
                best_strips = strips;
                best_sp = sp;
                best_ks = ks;
            }
        }
    }
    if (best_cost < 0.0) return gc_error(GC_UNSUPPORTED, "3xTF32 path: too many work items");
    const long long rows_b = tf32_rows_b(W, best_sp);
    const size_t smem = tf32_smem(cpg, W, best_sp);
    gcb::Tf32Params P{};
    P.n = static_cast<int>(N);
    P.c = static_cast<int>(C);
    P.h = static_cast<int>(H);
    P.wd = static_cast<int>(W);
    P.cpg = static_cast<int>(cpg);
    P.groups = static_cast<int>(p->groups);
    P.co_blocks = static_cast<int>(co_blocks);
    P.wp = static_cast<int>(wp);
    P.nb = static_cast<int>(best_nb);
    P.blocks = static_cast<int>(ceil_div(N, best_nb));
    P.out_rows = static_cast<int>((best_nb - 1) * hp2 + H);
    P.sp = best_sp;
    P.strips = static_cast<int>(best_strips);
    P.items = static_cast<int>(best_items);
    P.chunks = static_cast<int>(chunks / best_ks);
    P.ksplit = static_cast<int>(best_ks);
    P.m = 2 * co > 64 ? 128 : 64;
    P.rows_b = static_cast<int>(rows_b);
    P.a_bytes = static_cast<unsigned>(9 * P.m * 32);
    P.b_bytes = static_cast<unsigned>(rows_b * 32);
    P.wraw_bytes = static_cast<unsigned>(co * 72 * 4);
    const void *fn = tf32_kernel_for(co, rows_b, nhwc);
    int ctas = 0;
    st = kernel_occupancy(dev, fn, gcb::kTf32Threads, smem, facts.smem_optin, ctas);
    if (st != GC_OK) return st;
    if (ctas < 1) return gc_error(GC_UNSUPPORTED, "3xTF32 path: kernel does not fit on an SM");
    out.P = P;
    out.fn = fn;
    out.smem = smem;
    out.grid = static_cast<int>(std::min<long long>(P.items, static_cast<long long>(facts.sms)));
    return GC_OK;
}

int launch_tf32(const gc_shape *p, const float *x, const float *w, float *y, int dev, cudaStream_t stream,
                bool nhwc = false) {
    Tf32Plan plan;
    int st = plan_tf32(p, dev, plan, nhwc);
    if (st != GC_OK) return st;
    plan.P.x = x;
    plan.P.w = w;
    plan.P.y = y;
    CUtensorMap wmap;
    std::memset(&wmap, 0, sizeof(wmap));
    st = encode_rows_map(wmap, w, p->cout, (p->cin / p->groups) * 9, 72, plan.P.cpg / plan.P.co_blocks);
    if (st != GC_OK) return st;
    void *args[] = {&plan.P, &wmap};
    cudaError_t e;
    if (plan.P.ksplit == 1) {
        e = launch_pdl(plan.fn, dim3(plan.grid), dim3(gcb::kTf32Threads), args, plan.smem, stream);
    } else {
        // The parts of the input channels add into y: zero it first (a plain
        // stream-ordered launch follows the memset).
        e = cudaMemsetAsync(y, 0, static_cast<size_t>(p->n * p->cout * p->h * p->w) * sizeof(float), stream);
        if (e == cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(plan.grid);
            cfg.blockDim = dim3(gcb::kTf32Threads);
            cfg.dynamicSmemBytes = plan.smem;
            cfg.stream = stream;
            e = cudaLaunchKernelExC(&cfg, plan.fn, args);
        }
    }
    if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    record_plan(PlanRecord::kTf32, nhwc ? "nhwc" : "nchw", false, plan.grid, plan.smem, plan.P.m, gcb::kTf32N,
                plan.P.nb, plan.P.sp, plan.P.strips, plan.P.items, plan.P.chunks, plan.P.rows_b, plan.P.ksplit);
    return GC_OK;
}

// ---- small-image kernel ----------------------------------------------------------------------
constexpr long long kSmallMaxPixels = 512;  // one thread per pixel: at most 512 threads

bool small_eligible(const gc_shape *p) {
    return p->h * p->w <= kSmallMaxPixels && p->n < (1LL << 30) && p->cin < (1LL << 20);
}

const void *small_kernel_for(int cob) {
    switch (cob) {
    case 8: return reinterpret_cast<const void *>(&gcb::small_conv_kernel<8>);
    case 4: return reinterpret_cast<const void *>(&gcb::small_conv_kernel<4>);
    case 2: return reinterpret_cast<const void *>(&gcb::small_conv_kernel<2>);
    default: return reinterpret_cast<const void *>(&gcb::small_conv_kernel<1>);
    }
}

// Channels per item: the largest block of whole groups that still leaves at
// least two items per SM and fits 48 KB of shared memory (several CTAs per
// SM), else the smallest (one group).
int launch_small(const gc_shape *p, const float *x, const float *w, float *y, int dev, cudaStream_t stream) {
    DeviceFacts facts;
    int st = device_facts(dev, facts);
    if (st != GC_OK) return st;
    const long long N = p->n, C = p->cin, cpg = C / p->groups, hw = p->h * p->w;
    const int cob = cpg % 8 == 0 ? 8 : cpg % 4 == 0 ? 4 : cpg % 2 == 0 ? 2 : 1;
    // Channels per item: the largest block that still leaves every CTA about
    // two items (at ~3 resident CTAs per SM), so the double-buffered copies
    // of the next item hide the load latency; else the smallest block.
    long long best_cb = 0;
    for (long long gpi = 1; gpi <= p->groups; ++gpi) {
        if (p->groups % gpi) continue;
        const long long cb = gpi * cpg;
        const long long smem = (round_up(cb * hw, 4) + round_up(cb * cpg * 9, 4)) * 4;  // one stage
        if (2 * smem > 48 * 1024 && best_cb != 0) break;
        if (smem > facts.smem_optin) break;
        const long long items = N * (C / cb);
        if (best_cb == 0 || items >= 6LL * facts.sms) best_cb = cb;
        if (items < 6LL * facts.sms) break;
    }
    if (best_cb == 0) return gc_error(GC_UNSUPPORTED, "small-image kernel: one group does not fit in shared memory");
    gcb::SmallParams P{};
    P.x = x;
    P.w = w;
    P.y = y;
    P.n = static_cast<int>(N);
    P.c = static_cast<int>(C);
    P.h = static_cast<int>(p->h);
    P.wd = static_cast<int>(p->w);
    P.cpg = static_cast<int>(cpg);
    P.cb = static_cast<int>(best_cb);
    P.cblocks = static_cast<int>(C / best_cb);
    const long long items = N * P.cblocks;
    if (items >= (1LL << 31)) return gc_error(GC_UNSUPPORTED, "small-image kernel: too many items");
    P.items = static_cast<int>(items);
    P.hw = static_cast<int>(hw);
    P.hwp = static_cast<int>(round_up(hw, 32));
    P.x_floats = static_cast<int>(round_up(best_cb * hw, 4));
    P.w_floats = static_cast<int>(round_up(best_cb * cpg * 9, 4));
    P.vec = (aligned16(x) && (C * hw) % 4 == 0 && (best_cb * hw) % 4 == 0) ? 1 : 0;
    // Ring depth: up to 4 stages within 48 KB (more bytes in flight per CTA),
    // at least one stage.
    const size_t stage_bytes = static_cast<size_t>(P.x_floats + P.w_floats) * 4;
    P.stages = static_cast<int>(std::max<size_t>(1, std::min<size_t>(4, 48 * 1024 / stage_bytes)));
    while (P.stages > 1 && P.stages * stage_bytes > static_cast<size_t>(facts.smem_optin)) --P.stages;
    const size_t smem = P.stages * stage_bytes;
    // pixel slots per CTA: up to 256 threads, never more slots than channel blocks
    const long long slots = std::max<long long>(1, std::min<long long>(256 / P.hwp, best_cb / cob));
    const int threads = static_cast<int>(slots * P.hwp);
    const void *fn = small_kernel_for(cob);
    int ctas = 0;
    st = kernel_occupancy(dev, fn, threads, smem, facts.smem_optin, ctas);
    if (st != GC_OK) return st;
    if (ctas < 1) return gc_error(GC_UNSUPPORTED, "small-image kernel: does not fit on an SM");
    const int grid = static_cast<int>(std::min<long long>(items, static_cast<long long>(facts.sms) * ctas));
    void *args[] = {&P};
    cudaError_t e = launch_pdl(fn, dim3(grid), dim3(threads), args, smem, stream);
    if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    record_plan(PlanRecord::kSmall, "", false, grid, threads, smem, ctas, cob, P.cb, P.items, P.vec, P.stages);
    return GC_OK;
}

// ---- depthwise kernel for strided, dilated and 5x5/7x7 layers ---------------------------
constexpr size_t kDwSmemLimit = 48 * 1024;  // stage per CTA: several CTAs per SM, no opt-in

// Staged columns per input row: every column an output reaches, and for
// stride 1 / dilation 1 (four outputs per thread) whole quads of outputs.
bool dw_unit(const gc_shape *p) { return p->sw == 1 && p->dw == 1; }
long long dw_pitch(const gc_shape *p, int64_t wo) {
    return dw_unit(p) ? round_up(wo, 4) + p->s - 1 : (wo - 1) * p->sw + (p->s - 1) * p->dw + 1;
}

// Two stages of the input rows a band of bh output rows reaches.
size_t dw_smem(const gc_shape *p, int64_t wo, long long bh) {
    const long long rows = (bh - 1) * p->sh + (p->r - 1) * p->dh + 1;
    return static_cast<size_t>(2 * rows * dw_pitch(p, wo) * 4);
}

// Depthwise layers (groups == Cin == Cout) with a square 3x3, 5x5 or 7x7
// kernel whose one-output-row stage fits, and 32-bit in-plane indices.
bool dw_eligible(const gc_shape *p, int64_t ho, int64_t wo) {
    return p->groups == p->cin && p->cin == p->cout && p->r == p->s && (p->r == 3 || p->r == 5 || p->r == 7) &&
           p->h * p->w < (1LL << 31) && ho * wo < (1LL << 31) && p->sh * wo < (1LL << 30) &&
           p->dh * p->r < (1LL << 20) && p->dw * p->s < (1LL << 20) && p->ph < (1LL << 20) &&
           p->pw < (1LL << 20) && p->n * p->cin * ho < (1LL << 31) && dw_smem(p, wo, 1) <= kDwSmemLimit;
}

int launch_dw(const gc_shape *p, int64_t ho, int64_t wo, const float *x, const float *w, float *y, int dev,
              cudaStream_t stream, const float *bias = nullptr, int act = gcb::kActNone) {
    DeviceFacts facts;
    int st = device_facts(dev, facts);
    if (st != GC_OK) return st;
    // Output rows per item: the largest band whose stage fits and that still
    // gives every SM eight items, else the smallest that fits.
    long long bh = 1;
    for (long long cand : {64LL, 32LL, 16LL, 8LL, 4LL, 2LL, 1LL}) {
        if (cand > ho || dw_smem(p, wo, cand) > kDwSmemLimit) continue;
        bh = cand;
        if (p->n * p->cin * ceil_div(ho, cand) >= 8LL * facts.sms) break;
    }
    gcb::DwParams P;
    P.x = x;
    P.w = w;
    P.y = y;
    P.bias = bias;
    P.act = act;
    P.n = static_cast<int>(p->n);
    P.c = static_cast<int>(p->cin);
    P.h = static_cast<int>(p->h);
    P.wd = static_cast<int>(p->w);
    P.sh = static_cast<int>(p->sh);
    P.sw = static_cast<int>(p->sw);
    P.ph = static_cast<int>(p->ph);
    P.pw = static_cast<int>(p->pw);
    P.dh = static_cast<int>(p->dh);
    P.dw = static_cast<int>(p->dw);
    P.ho = static_cast<int>(ho);
    P.wo = static_cast<int>(wo);
    P.bh = static_cast<int>(bh);
    P.bands = static_cast<int>(ceil_div(ho, bh));
    P.pitch = static_cast<int>(dw_pitch(p, wo));
    P.items = p->n * p->cin * P.bands;
    const size_t smem = dw_smem(p, wo, bh);
    const bool unit = dw_unit(p);
    const void *fn = p->r == 3   ? (unit ? reinterpret_cast<const void *>(&gcb::dw_conv_kernel<3, true>)
                                         : reinterpret_cast<const void *>(&gcb::dw_conv_kernel<3, false>))
                     : p->r == 5 ? (unit ? reinterpret_cast<const void *>(&gcb::dw_conv_kernel<5, true>)
                                         : reinterpret_cast<const void *>(&gcb::dw_conv_kernel<5, false>))
                                 : (unit ? reinterpret_cast<const void *>(&gcb::dw_conv_kernel<7, true>)
                                         : reinterpret_cast<const void *>(&gcb::dw_conv_kernel<7, false>));
    // Threads per CTA: an item's outputs (quads of 4 for stride 1 and
    // dilation 1), in whole warps, 64 to 256: small bands of small planes get
    // small CTAs, so that more of them are resident per SM instead of most
    // threads of a 256-thread CTA idling.
    const long long work = bh * (unit ? ceil_div(wo, 4) : wo);
    const int threads = static_cast<int>(std::min<long long>(256, std::max<long long>(64, round_up(work, 32))));
    int ctas = 0;
    st = kernel_occupancy(dev, fn, threads, smem, facts.smem_optin, ctas);
    if (st != GC_OK) return st;
    if (ctas < 1) return gc_error(GC_UNSUPPORTED, "depthwise kernel: does not fit on an SM");
    const int grid = static_cast<int>(std::min<long long>(P.items, static_cast<long long>(facts.sms) * ctas));
    void *args[] = {&P};
    cudaError_t e = launch_pdl(fn, dim3(grid), dim3(threads), args, smem, stream);
    if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    record_plan(PlanRecord::kDw, "", false, p->r, grid, smem, bh, P.bands, P.pitch, P.items, threads);
    return GC_OK;
}

// Depthwise 3x3 or 5x5, stride 2 (or 3x3 stride 1), padding K/2, dilation
// 1 with 32-bit in-plane indices.
bool dw_s2_eligible(const gc_shape *p) {
    const bool s2 = p->sh == 2 && p->sw == 2, s1 = p->sh == 1 && p->sw == 1 && p->r == 3;
    return p->groups == p->cin && p->cin == p->cout && (p->r == 3 || p->r == 5) && p->s == p->r && (s1 || s2) &&
           p->ph == p->r / 2 && p->pw == p->r / 2 && p->dh == 1 && p->dw == 1 &&
           p->h * p->w < (1LL << 31) &&
           p->w < (1LL << 29) && p->h < (1LL << 29) && p->cin < (1LL << 31);
}

int launch_dw_s2(const gc_shape *p, int64_t ho, int64_t wo, const float *x, const float *w, float *y, int dev,
                 cudaStream_t stream, const float *bias = nullptr, int act = gcb::kActNone) {
    DeviceFacts facts;
    int st = device_facts(dev, facts);
    if (st != GC_OK) return st;
    gcb::DwS2Params P;
    P.x = x;
    P.w = w;
    P.y = y;
    P.bias = bias;
    P.act = act;
    P.n = static_cast<int>(p->n);
    P.c = static_cast<int>(p->cin);
    P.h = static_cast<int>(p->h);
    P.wd = static_cast<int>(p->w);
    P.ho = static_cast<int>(ho);
    P.wo = static_cast<int>(wo);
    P.qcols = static_cast<int>(ceil_div(wo, 4));
    P.prows = static_cast<int>(ceil_div(ho, 2));
    const int stride = static_cast<int>(p->sh);
    P.cells = p->n * p->cin * P.prows * P.qcols;
    P.vec_in = p->w % 4 == 0 && aligned16(x);
    P.vec_out = wo % 4 == 0 && aligned16(y);
    const void *fn = stride == 1  ? reinterpret_cast<const void *>(&gcb::dw_s2_conv_kernel<3, 1>)
                     : p->r == 3 ? reinterpret_cast<const void *>(&gcb::dw_s2_conv_kernel<3, 2>)
                                 : reinterpret_cast<const void *>(&gcb::dw_s2_conv_kernel<5, 2>);
    int ctas = 0;
    st = kernel_occupancy(dev, fn, 256, 0, facts.smem_optin, ctas);
    if (st != GC_OK) return st;
    if (ctas < 1) return gc_error(GC_UNSUPPORTED, "stride-2 depthwise kernel: does not fit on an SM");
    const long long blocks = std::min<long long>(ceil_div(P.cells, 256), static_cast<long long>(facts.sms) * ctas);
    void *args[] = {&P};
    cudaError_t e = launch_pdl(fn, dim3(static_cast<unsigned>(blocks)), dim3(256), args, 0, stream);
    if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    record_plan(PlanRecord::kDwS2, "", false, p->r, blocks, P.cells, P.vec_in, P.vec_out, stride);
    return GC_OK;
}

// ---- general kernel ------------------------------------------------------------------
constexpr int kGeneralRun = 4;

template <int COB>
const void *general_kernel_for(bool narrow) {
    return narrow ? reinterpret_cast<const void *>(&gcb::general_conv_kernel<kGeneralRun, COB, int>)
                  : reinterpret_cast<const void *>(&gcb::general_conv_kernel<kGeneralRun, COB, long long>);
}

int launch_general(const gc_shape *p, int64_t ho, int64_t wo, const float *x, const float *w,
                   float *y, int dev, cudaStream_t stream, const float *bias = nullptr, int act = gcb::kActNone) {
    if (dw_s2_eligible(p)) return launch_dw_s2(p, ho, wo, x, w, y, dev, stream, bias, act);
    if (dw_eligible(p, ho, wo)) return launch_dw(p, ho, wo, x, w, y, dev, stream, bias, act);
    DeviceFacts facts;
    int st = device_facts(dev, facts);
    if (st != GC_OK) return st;
    GeneralParams P;
    P.xp = x;
    P.wp = w;
    P.yp = y;
    P.bias = bias;
    P.act = act;
    P.n = p->n;
    P.cin = p->cin;
    P.cout = p->cout;
    P.h = p->h;
    P.w = p->w;
    P.r = p->r;
    P.s = p->s;
    P.groups = p->groups;
    P.sh = p->sh;
    P.sw = p->sw;
    P.ph = p->ph;
    P.pw = p->pw;
    P.dh = p->dh;
    P.dw = p->dw;
    P.ho = ho;
    P.wo = wo;
    // output channels per thread: the largest of 8, 4, 2, 1 dividing the
    // output channels per group
    const long long opg = p->cout / p->groups;
    const int cob = opg % 8 == 0 ? 8 : opg % 4 == 0 ? 4 : opg % 2 == 0 ? 2 : 1;
    P.runs_per_row = ceil_div(wo, kGeneralRun);
    P.total_runs = p->n * (p->cout / cob) * ho * P.runs_per_row;
    // 32-bit indices when every element index (and the run count, and the
    // worst intermediate of the input index) stays below 2^31
    const long long lim = 1LL << 31;
    const long long runs_padded = P.total_runs + static_cast<long long>(facts.sms) * 8 * 256;
    const bool narrow = p->n * p->cin * p->h * p->w < lim && p->n * p->cout * ho * wo + kGeneralRun < lim &&
                        p->cout * (p->cin / p->groups) * p->r * p->s < lim && runs_padded < lim &&
                        p->h + 2 * p->ph + 2 * p->sh + p->r * p->dh < lim &&
                        p->w + 2 * p->pw + (kGeneralRun + 2) * p->sw + p->s * p->dw < lim;
    const int threads = 256;
    const long long blocks = std::min<long long>(ceil_div(P.total_runs, threads),
                                                 static_cast<long long>(facts.sms) * 8);
    const void *fn = cob == 8 ? general_kernel_for<8>(narrow)
                   : cob == 4 ? general_kernel_for<4>(narrow)
                   : cob == 2 ? general_kernel_for<2>(narrow)
                              : general_kernel_for<1>(narrow);
    void *args[] = {&P};
    cudaError_t e = launch_pdl(fn, dim3(static_cast<unsigned>(blocks)), dim3(threads), args, 0, stream);
    if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    record_plan(PlanRecord::kGeneral, "", false, blocks, threads, kGeneralRun, cob, narrow ? 1 : 0, P.total_runs);
    return GC_OK;
}

// ---- channels-last (NHWC) tensors (kernel_nhwc.cuh) --------------------------------------
bool channels_last_strides(const gc_tensor *t) {
    return t->rank == 4 && t->strides[1] == 1 && t->strides[3] == t->dims[1] &&
           t->strides[2] == t->dims[3] * t->dims[1] && t->strides[0] == t->dims[2] * t->dims[3] * t->dims[1];
}

int launch_nhwc(const gc_shape *p, int64_t ho, int64_t wo, const float *x, const float *w, const float *bias,
                int act, float *y, int dev, cudaStream_t stream) {
    DeviceFacts facts;
    int st = device_facts(dev, facts);
    if (st != GC_OK) return st;
    const long long cpg = p->cin / p->groups;
    const bool b = p->cin == p->cout && p->r == 3 && p->s == 3 && p->sh == 1 && p->sw == 1 && p->ph == 1 &&
                   p->pw == 1 && p->dh == 1 && p->dw == 1;
    const bool vec = b && p->cin % 4 == 0 && aligned16(x) && aligned16(y) && (cpg == 1 || cpg == 2 || cpg % 4 == 0) &&
                     p->h < (1LL << 30) && p->w < (1LL << 30) && p->cin < (1LL << 30);
    cudaError_t e;
    // Groups of more than 16 channels (a multiple of 8): the tensor-core
    // path reads channels-last pixels directly (each pixel's 8 channels of a
    // step are 32 contiguous bytes) and stores channels-last outputs.
    if (b && bias == nullptr && act == gcb::kActNone && cpg >= 16 && p->cin % 8 == 0 && aligned16(x) &&
        aligned16(y)) {
        gc_shape q = *p;
        if (tf32_eligible(&q, x, w)) {
            st = launch_tf32(&q, x, w, y, dev, stream, true);
            if (st != GC_UNSUPPORTED) return st;
        }
    }
    // Groups of 1, 2, 4 and 8 channels: TMA-staged tiles of 32 channels x up
    // to 8 rows x up to 32 columns (groups of 1 and 2: a thread per 4 channels
    // of a column; groups of 4: a thread per channel of 4 columns), or 8
    // columns (groups of 8: a thread per channel of 2 columns, 128-thread
    // CTAs, so that their 138 registers still leave 3 CTAs per SM), two
    // stages per persistent CTA.
    if (vec && (cpg == 1 || cpg == 2 || cpg == 4 || cpg == 8) && aligned16(w) &&
        (bias == nullptr || aligned16(bias)) && p->n < (1LL << 31)) {
        const bool quad = cpg <= 2;  // a thread per 4 channels (else per channel)
        const int nc = cpg == 4 ? 4 : 2;  // columns per thread, groups of 4 and 8
        const int max_tw = quad ? 32 : cpg == 4 ? 8 * nc : 8;
        gcb::NhwcDwTmaParams P{};
        P.w = w;
        P.bias = bias;
        P.y = y;
        P.act = act;
        P.n = static_cast<int>(p->n);
        P.c = static_cast<int>(p->cin);
        P.h = static_cast<int>(p->h);
        P.wd = static_cast<int>(p->w);
        P.wtiles = static_cast<int>(ceil_div(p->w, max_tw));
        // groups of 4 and 8: a multiple of the thread's columns, so that every
        // column a thread reads lies inside the box
        P.tw = static_cast<int>(quad ? ceil_div(p->w, P.wtiles) : round_up(ceil_div(p->w, P.wtiles), nc));
        P.htiles = static_cast<int>(ceil_div(p->h, gcb::kDwTmaMaxTH));
        P.th = static_cast<int>(ceil_div(p->h, P.htiles));
        P.cblocks = static_cast<int>(ceil_div(p->cin, gcb::kDwTmaCB));
        const long long items = p->n * P.htiles * P.wtiles * static_cast<long long>(P.cblocks);
        if (items < (1LL << 31)) {
            P.items = static_cast<int>(items);
            P.box_bytes = static_cast<unsigned>(gcb::kDwTmaCB * (P.tw + 2) * (P.th + 2) * 4);
            const size_t smem = 2 * static_cast<size_t>(P.box_bytes) + 16;
            const int threads = quad ? 8 * P.tw : 32 * static_cast<int>(ceil_div(P.tw, nc));
            const void *fn = cpg == 1   ? reinterpret_cast<const void *>(&gcb::nhwc_dw_tma_kernel<1>)
                             : cpg == 2 ? reinterpret_cast<const void *>(&gcb::nhwc_dw_tma_kernel<2>)
                             : cpg == 4 ? reinterpret_cast<const void *>(&gcb::nhwc_grp_tma_kernel<4, 4>)
                                        : reinterpret_cast<const void *>(&gcb::nhwc_grp_tma_kernel<8, 2>);
            int ctas = 0;
            st = kernel_occupancy(dev, fn, threads, smem, facts.smem_optin, ctas);
            if (st != GC_OK) return st;
            if (ctas >= 1) {
                CUtensorMap xmap;
                std::memset(&xmap, 0, sizeof(xmap));
                st = encode_nhwc_map(xmap, x, p->n, p->cin, p->h, p->w, gcb::kDwTmaCB, P.tw + 2, P.th + 2);
                if (st != GC_OK) return st;
                const long long blocks = std::min<long long>(items, static_cast<long long>(facts.sms) * ctas);
                void *args[] = {&P, &xmap};
                e = launch_pdl(fn, dim3(static_cast<unsigned>(blocks)), dim3(threads), args, smem, stream);
                if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
                record_plan(PlanRecord::kNhwc, quad ? "dw_tma" : "grp_tma", false, blocks, threads, cpg,
                            bias != nullptr ? 1 : 0, P.th);
                return GC_OK;
            }
        }
    }
    // Groups of 1, 2, 4 and 8: threads walk down strips of output rows, the
    // layer's weights in shared memory (when they fit in 160 KB).
    const size_t wbytes = static_cast<size_t>(p->cin) * cpg * 9 * 4;
    if (vec && p->n < (1LL << 30) && (cpg == 1 || cpg == 2 || cpg == 4 || cpg == 8) && wbytes <= 160 * 1024) {
        gcb::NhwcStripParams P{};
        P.x = x;
        P.w = w;
        P.bias = bias;
        P.y = y;
        P.act = act;
        P.n = static_cast<int>(p->n);
        P.c = static_cast<int>(p->cin);
        P.h = static_cast<int>(p->h);
        P.wd = static_cast<int>(p->w);
        P.qcols = static_cast<int>(ceil_div(p->w, 4));
        P.cquads = static_cast<int>(p->cin / 4);
        const void *fn = cpg == 1   ? reinterpret_cast<const void *>(&gcb::nhwc_strip_kernel<1>)
                         : cpg == 2 ? reinterpret_cast<const void *>(&gcb::nhwc_strip_kernel<2>)
                         : cpg == 4 ? reinterpret_cast<const void *>(&gcb::nhwc_strip_kernel<4>)
                                    : reinterpret_cast<const void *>(&gcb::nhwc_strip_kernel<8>);
        const size_t smem = wbytes;
        int ctas = 0;
        st = kernel_occupancy(dev, fn, 128, smem, facts.smem_optin, ctas);
        if (st != GC_OK) return st;
        if (ctas >= 1) {
            // longest strips (8, 4, 2 or 1 rows) that still give every
            // resident thread two items
            const long long resident = static_cast<long long>(facts.sms) * ctas * 128;
            const long long cols = p->n * P.qcols * static_cast<long long>(P.cquads);
            int hb = 8;
            while (hb > 1 && cols * ceil_div(p->h, hb) < 2 * resident) hb /= 2;
            P.hb = hb;
            P.hstrips = static_cast<int>(ceil_div(p->h, hb));
            P.items = cols * P.hstrips;
            const long long blocks =
                std::min<long long>(ceil_div(P.items, 128), static_cast<long long>(facts.sms) * ctas);
            void *args[] = {&P};
            e = launch_pdl(fn, dim3(static_cast<unsigned>(blocks)), dim3(128), args, smem, stream);
            if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
            record_plan(PlanRecord::kNhwc, "strip", false, blocks, 128, cpg, bias != nullptr ? 1 : 0, hb);
            return GC_OK;
        }
    }
    if (vec) {
        gcb::NhwcParams P{};
        P.x = x;
        P.w = w;
        P.bias = bias;
        P.y = y;
        P.act = act;
        P.n = static_cast<int>(std::min<long long>(p->n, 1LL << 30));
        P.c = static_cast<int>(p->cin);
        P.h = static_cast<int>(p->h);
        P.wd = static_cast<int>(p->w);
        P.cpg = static_cast<int>(cpg);
        P.qcols = static_cast<int>(ceil_div(p->w, gcb::kNhwcPx));
        P.cquads = static_cast<int>(p->cin / 4);
        P.cells = p->n * p->h * P.qcols * P.cquads;
        const void *fn = cpg == 1   ? reinterpret_cast<const void *>(&gcb::nhwc_conv_kernel<1>)
                         : cpg == 2 ? reinterpret_cast<const void *>(&gcb::nhwc_conv_kernel<2>)
                                    : reinterpret_cast<const void *>(&gcb::nhwc_conv_kernel<0>);
        const long long blocks = std::min<long long>(ceil_div(P.cells, 256), static_cast<long long>(facts.sms) * 8);
        void *args[] = {&P};
        e = launch_pdl(fn, dim3(static_cast<unsigned>(blocks)), dim3(256), args, 0, stream);
        if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
        record_plan(PlanRecord::kNhwc, "vector4x4", false, blocks, 256, cpg, bias != nullptr ? 1 : 0, 1);
        return GC_OK;
    }
    gcb::NhwcScalarParams P{};
    P.x = x;
    P.wt = w;
    P.bias = bias;
    P.y = y;
    P.act = act;
    P.n = p->n;
    P.cin = p->cin;
    P.cout = p->cout;
    P.h = p->h;
    P.w = p->w;
    P.r = p->r;
    P.s = p->s;
    P.groups = p->groups;
    P.sh = p->sh;
    P.sw = p->sw;
    P.ph = p->ph;
    P.pw = p->pw;
    P.dh = p->dh;
    P.dw = p->dw;
    P.ho = ho;
    P.wo = wo;
    P.total = p->n * ho * wo * p->cout;
    const long long blocks = std::min<long long>(ceil_div(P.total, 256), static_cast<long long>(facts.sms) * 8);
    void *args[] = {&P};
    e = launch_pdl(reinterpret_cast<const void *>(&gcb::nhwc_scalar_kernel), dim3(static_cast<unsigned>(blocks)),
                   dim3(256), args, 0, stream);
    if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    record_plan(PlanRecord::kNhwc, "scalar", false, blocks, 256, cpg, bias != nullptr ? 1 : 0, 1);
    return GC_OK;
}

// Structure of an optional bias descriptor: rank 1, Cout dense FP32 elements
// on the CUDA device of the data tensors.
int check_bias_descriptor(const gc_tensor *b, const gc_shape *p, const gc_tensor *x) {
    if (b->data == nullptr) return gc_error(GC_INVALID, "bias data pointer is null");
    if (b->dtype != GC_F32) return gc_error(GC_INVALID, "bias dtype must be F32");
    if (b->device != GC_CUDA || b->device_index != x->device_index)
        return gc_error(GC_INVALID, "bias must be CUDA memory on the tensors' device");
    if (b->rank != 1 || b->dims[0] != p->cout) return gc_error(GC_INVALID, "bias must be a rank-1 tensor of Cout");
    if (b->bytes < static_cast<uint64_t>(p->cout) * 4u) return gc_error(GC_INVALID, "bias buffer too small");
    if ((reinterpret_cast<uintptr_t>(b->data) & 3u) != 0) return gc_error(GC_INVALID, "bias is not 4-byte aligned");
    if (b->strides[0] != 1) return gc_error(GC_UNSUPPORTED, "bias must be dense");
    return GC_OK;
}

// ---- contract checks shared by both entry points ----------------------------------------
bool b_geometry(const gc_shape *p) {
    return p->cin == p->cout && p->r == 3 && p->s == 3 && p->sh == 1 && p->sw == 1 && p->ph == 1 &&
           p->pw == 1 && p->dh == 1 && p->dw == 1;
}

// Device memory on the descriptor's device, which must be the current device
// (reference groupconv.cu:130-139).  Managed and mapped host memory are
// outside the contract.
int check_pointer(const gc_tensor *t, int current) {
    cudaPointerAttributes attr;
    std::memset(&attr, 0, sizeof(attr));
    cudaError_t e = cudaPointerGetAttributes(&attr, t->data);
    if (e != cudaSuccess) {
        cudaGetLastError();  // the failed query must not poison the next launch check
        return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    }
    if (attr.type != cudaMemoryTypeDevice || attr.device != t->device_index || attr.device != current)
        return gc_error(GC_INVALID, "CUDA pointer must be device memory on descriptor/current device");
    return GC_OK;
}

int device_and_stream_checks(const gc_tensor *x, const gc_tensor *w, const gc_tensor *y,
                             void *stream, int &current) {
    cudaError_t e = cudaGetDevice(&current);
    if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    for (const gc_tensor *t : {x, w, y}) {
        int st = check_pointer(t, current);
        if (st != GC_OK) return st;
    }
    // Capture-status lookup validates the handle in eager and captured use
    // alike (stream-flag queries are rejected during capture).
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(reinterpret_cast<cudaStream_t>(stream), &cs);
    if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    return GC_OK;
}

// Launches one kernel family.  With general_when_no_tile, a B-geometry request
// whose image is too wide for any shared-memory tile of the direct engines
// runs on the general kernel instead (the v1 implementations 1-3 support every
// B-geometry shape); gc_b200_conv asks for one family and gets GC_UNSUPPORTED.
int run_kernel(const gc_shape *p, const gc_tensor *x, const gc_tensor *w, gc_tensor *y, int kernel,
               int dev, void *stream, bool general_when_no_tile = false) {
    int64_t ho = 0, wo = 0;
    int st = gc_validate_shape(p, &ho, &wo);
    if (st != GC_OK) return st;
    const float *xp = static_cast<const float *>(x->data);
    const float *wp = static_cast<const float *>(w->data);
    float *yp = static_cast<float *>(y->data);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (kernel) {
    case GC_B200_GENERAL:
        st = launch_general(p, ho, wo, xp, wp, yp, dev, s);
        break;
    case GC_B200_DIRECT_LDG:
        st = launch_direct(p, xp, wp, yp, false, dev, s);
        break;
    case GC_B200_DIRECT_TMA:
        st = launch_direct(p, xp, wp, yp, true, dev, s);
        break;
    case GC_B200_TF32X3:
        st = launch_tf32(p, xp, wp, yp, dev, s);
        break;
    case GC_B200_SMALL:
        st = launch_small(p, xp, wp, yp, dev, s);
        break;
    default:
        return gc_error(GC_UNSUPPORTED, "unknown B200 kernel family");
    }
    if (st == GC_UNSUPPORTED && general_when_no_tile && kernel != GC_B200_GENERAL)
        st = launch_general(p, ho, wo, xp, wp, yp, dev, s);
    if (st != GC_OK) return st;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? gc_error(GC_OK, "") : gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
}

// Production choice for B geometry: the tensor-core path for groups of more
// than 16 channels, else the direct engine with TMA staging where the layout
// allows it.  (Measured per shape against the FFMA engines, 1 x B200: at 8
// channels per group the direct kernel is faster; at 16 the warp-specialized
// direct kernel beats the tensor path by 1-12 % on every measured layer, from
// N1 C256 56x56 to N16 C512 112x112; from 24 on the tensor path wins, at 32
// by 3.5x over the channel-chunked FFMA kernel.)
int auto_kernel(const gc_shape *p, const gc_tensor *x, const gc_tensor *w, int dev) {
    (void)dev;
    const long long cpg = p->cin / p->groups;
    if (cpg == 16 && tma_eligible(p, x->data)) return GC_B200_DIRECT_TMA;
    if (cpg >= 16 && tf32_eligible(p, x->data, w->data)) return GC_B200_TF32X3;
    // Depthwise layers of little work - planes of at most 256 pixels, or at
    // most 256K outputs in all, but not the very smallest (under 32K outputs,
    // where the small-image kernel's launch is cheaper) - run on the
    // register-cell kernel behind the general family (measured: N32 C256 7x7
    // 3.2 vs 6.2 us, 14x14 7.9 vs 13.5 us, N1 C256 28x28 2.3 vs 3.0 us).
    const long long outs = p->n * p->cout * p->h * p->w;
    if (cpg == 1 && dw_s2_eligible(p) && outs >= (32LL << 10) && (p->h * p->w <= 256 || outs <= (256LL << 10)))
        return GC_B200_GENERAL;
    // Small planes that the TMA tiles cannot stage (or that are narrower than
    // a TMA tile's halo) run whole planes per CTA.
    if (small_eligible(p) && (!tma_eligible(p, x->data) || p->w <= 16)) return GC_B200_SMALL;
    return tma_eligible(p, x->data) ? GC_B200_DIRECT_TMA : GC_B200_DIRECT_LDG;
}

__global__ void wait_timeout_selftest_kernel(uint64_t limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        gcb::mbar_init(&bar, 1);
        gcb::fence_barrier_init();
    }
    __syncthreads();
    // Nothing ever arrives on the barrier, so phase 0 never completes.
    if (threadIdx.x == 0 && !gcb::mbar_wait_bounded(&bar, 0, limit_ns))
        gcb::raise_status(gcb::kStatusTmaTimeout);
}

}  // namespace

extern "C" {

int gc_cuda_available(void) {
    int count = 0;
    return cudaGetDeviceCount(&count) == cudaSuccess && count > 0;
}

int gc_cuda_conv(const gc_shape *p, const gc_tensor *x, const gc_tensor *w, gc_tensor *y,
                 int implementation, void *stream) {
    int st = gc_validate_tensors(p, x, w, y, GC_CUDA, GC_F32);
    if (st != GC_OK) return st;
    if (implementation < 0 || implementation > 3)
        return gc_error(GC_UNSUPPORTED, "Unknown CUDA implementation");
    const bool b = b_geometry(p);
    if (implementation != 0 && !b)
        return gc_error(GC_UNSUPPORTED, "Optimized CUDA kernels require B geometry");
    const int64_t cpg = p->cin / p->groups;
    if (implementation == 2 && cpg != 1 && cpg != 2 && cpg != 4)
        return gc_error(GC_UNSUPPORTED, "CUDA shared halo supports cpg 1, 2, or 4");
    int dev = -1;
    st = device_and_stream_checks(x, w, y, stream, dev);
    if (st != GC_OK) return st;
    int kernel = GC_B200_GENERAL;
    if (implementation == 1) kernel = GC_B200_DIRECT_LDG;
    if (implementation == 2) kernel = auto_kernel(p, x, w, dev);  // cpg <= 4: never the tensor-core path
    if (implementation == 3) kernel = auto_kernel(p, x, w, dev);
    return run_kernel(p, x, w, y, kernel, dev, stream, true);
}

int gc_b200_conv(const gc_shape *p, const gc_tensor *x, const gc_tensor *w, gc_tensor *y,
                 int kernel, void *stream) {
    int st = gc_validate_tensors(p, x, w, y, GC_CUDA, GC_F32);
    if (st != GC_OK) return st;
    if (kernel < GC_B200_AUTO || kernel > GC_B200_SMALL)
        return gc_error(GC_UNSUPPORTED, "unknown B200 kernel family");
    const bool b = b_geometry(p);
    if (kernel != GC_B200_GENERAL && kernel != GC_B200_AUTO && !b)
        return gc_error(GC_UNSUPPORTED, "this kernel family requires 3x3/s1/p1/d1 with Cin == Cout");
    if (kernel == GC_B200_DIRECT_TMA && !tma_eligible(p, x->data))
        return gc_error(GC_UNSUPPORTED,
                        "TMA staging needs width % 4 == 0, width <= 248 and a 16-byte aligned input");
    if (kernel == GC_B200_SMALL && !small_eligible(p))
        return gc_error(GC_UNSUPPORTED, "small-image kernel needs at most 512 pixels per plane");
    if (kernel == GC_B200_TF32X3 && !tf32_eligible(p, x->data, w->data))
        return gc_error(GC_UNSUPPORTED,
                        "3xTF32 path needs a multiple of 8 channels per group, 16-byte aligned weights and "
                        "a 256-pixel strip plus halo within 1024 rows and shared memory");
    int dev = -1;
    st = device_and_stream_checks(x, w, y, stream, dev);
    if (st != GC_OK) return st;
    if (kernel == GC_B200_AUTO) kernel = b ? auto_kernel(p, x, w, dev) : GC_B200_GENERAL;
    return run_kernel(p, x, w, y, kernel, dev, stream);
}

int gc_b200_conv_ex(const gc_shape *p, const gc_tensor *x, const gc_tensor *w, const gc_tensor *bias,
                    gc_tensor *y, int layout, int activation, void *stream) {
    if (p == nullptr || x == nullptr || w == nullptr || y == nullptr)
        return gc_error(GC_INVALID, "null shape or tensor descriptor");
    if (layout != GC_B200_NCHW && layout != GC_B200_NHWC) return gc_error(GC_UNSUPPORTED, "unknown layout");
    if (activation != GC_B200_ACT_NONE && activation != GC_B200_ACT_RELU && activation != GC_B200_ACT_RELU6)
        return gc_error(GC_UNSUPPORTED, "unknown activation");
    int st = GC_OK;
    if (layout == GC_B200_NCHW) {
        st = gc_validate_tensors(p, x, w, y, GC_CUDA, GC_F32);
    } else {
        // every GC_INVALID condition first (checked on dense-NCHW views of the
        // same sizes), then the channels-last layout of x and y
        gc_tensor xd = *x, yd = *y;
        for (gc_tensor *t : {&xd, &yd}) {
            t->strides[3] = 1;
            t->strides[2] = t->dims[3];
            t->strides[1] = t->dims[2] * t->dims[3];
            t->strides[0] = t->dims[1] * t->dims[2] * t->dims[3];
        }
        st = gc_validate_tensors(p, &xd, w, &yd, GC_CUDA, GC_F32);
        if (st == GC_OK && (!channels_last_strides(x) || !channels_last_strides(y)))
            st = gc_error(GC_UNSUPPORTED, "NHWC layout needs channels-last strides (H*W*C, 1, W*C, C) for x and y");
    }
    if (st != GC_OK) return st;
    if (bias != nullptr && (st = check_bias_descriptor(bias, p, x)) != GC_OK) return st;
    int dev = -1;
    st = device_and_stream_checks(x, w, y, stream, dev);
    if (st != GC_OK) return st;
    if (bias != nullptr && (st = check_pointer(bias, dev)) != GC_OK) return st;
    const bool b = b_geometry(p);
    const int kernel = b ? auto_kernel(p, x, w, dev) : GC_B200_GENERAL;
    if (layout == GC_B200_NCHW && bias == nullptr && activation == GC_B200_ACT_NONE)
        return run_kernel(p, x, w, y, kernel, dev, stream, true);
    int64_t ho = 0, wo = 0;
    st = gc_validate_shape(p, &ho, &wo);
    if (st != GC_OK) return st;
    const float *xp = static_cast<const float *>(x->data), *wp = static_cast<const float *>(w->data);
    const float *bp = bias != nullptr ? static_cast<const float *>(bias->data) : nullptr;
    float *yp = static_cast<float *>(y->data);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (layout == GC_B200_NHWC) {
        st = launch_nhwc(p, ho, wo, xp, wp, bp, activation, yp, dev, s);
    } else {
        // The production kernel when it has the epilogue (the direct
        // engines), else the depthwise engines or the general kernel.
        st = GC_UNSUPPORTED;
        if (kernel == GC_B200_DIRECT_TMA || kernel == GC_B200_DIRECT_LDG)
            st = launch_direct(p, xp, wp, yp, kernel == GC_B200_DIRECT_TMA, dev, s, bp, activation);
        if (st == GC_UNSUPPORTED) st = launch_general(p, ho, wo, xp, wp, yp, dev, s, bp, activation);
    }
    if (st != GC_OK) return st;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? gc_error(GC_OK, "") : gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
}

int gc_b200_autotune(const gc_shape *p, const gc_tensor *x, const gc_tensor *w, gc_tensor *y, int candidates,
                     void *stream) {
    int st = gc_validate_tensors(p, x, w, y, GC_CUDA, GC_F32);
    if (st != GC_OK) return st;
    if (candidates < 1 || candidates > 64) return gc_error(GC_INVALID, "candidates must be in 1..64");
    int dev = -1;
    st = device_and_stream_checks(x, w, y, stream, dev);
    if (st != GC_OK) return st;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(reinterpret_cast<cudaStream_t>(stream), &cs);
    if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    if (cs != cudaStreamCaptureStatusNone)
        return gc_error(GC_UNSUPPORTED, "autotuning times kernels: not inside a stream capture");
    if (!b_geometry(p)) return gc_error(GC_OK, "");  // the general kernel has one plan
    const int kernel = auto_kernel(p, x, w, dev);
    if (kernel != GC_B200_DIRECT_TMA && kernel != GC_B200_DIRECT_LDG) return gc_error(GC_OK, "");
    st = autotune_direct(p, static_cast<const float *>(x->data), static_cast<const float *>(w->data),
                         static_cast<float *>(y->data), kernel == GC_B200_DIRECT_TMA, dev,
                         reinterpret_cast<cudaStream_t>(stream), candidates);
    if (st != GC_OK) return st;
    e = cudaGetLastError();
    return e == cudaSuccess ? gc_error(GC_OK, "") : gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
}

const char *gc_b200_last_plan(void) {
    g_plan = format_plan(g_last);
    return g_plan.c_str();
}

int gc_b200_device_status(uint32_t *status, int clear) {
    if (status == nullptr) return gc_error(GC_INVALID, "null status pointer");
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(status, gcb::g_status, sizeof(uint32_t));
    if (e == cudaSuccess && clear) {
        const uint32_t zero = 0;
        e = cudaMemcpyToSymbol(gcb::g_status, &zero, sizeof(uint32_t));
    }
    if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    return gc_error(GC_OK, "");
}

int gc_b200_selftest_wait_timeout(uint32_t limit_us, void *stream) {
    if (limit_us == 0 || limit_us > 10000000u)
        return gc_error(GC_INVALID, "limit_us must be in 1..10000000");
    wait_timeout_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<uint64_t>(limit_us) * 1000ull);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    return gc_error(GC_OK, "");
}

// ---- peak-rate probes (the roofline denominators) -------------------------------------
static int probe_launched() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? gc_error(GC_OK, "") : gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
}

static int probe_device_pointer(const void *p) {
    int current = -1;
    cudaError_t e = cudaGetDevice(&current);
    if (e != cudaSuccess) return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    cudaPointerAttributes attr;
    std::memset(&attr, 0, sizeof(attr));
    e = cudaPointerGetAttributes(&attr, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return gc_error(GC_DEVICE_ERROR, cudaGetErrorString(e));
    }
    if (attr.type != cudaMemoryTypeDevice || attr.device != current)
        return gc_error(GC_INVALID, "probe buffers must be device memory of the current device");
    return GC_OK;
}

int gc_b200_probe_ffma(float *out, int blocks, int iters, void *stream) {
    if (out == nullptr || blocks < 1 || blocks > (1 << 20) || iters < 1 || iters > (1 << 24))
        return gc_error(GC_INVALID, "probe_ffma: out must be non-null, blocks in 1..2^20, iters in 1..2^24");
    int st = probe_device_pointer(out);
    if (st != GC_OK) return st;
    gcb::ffma_probe_kernel<<<blocks, gcb::kProbeThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        out, 1.0f, iters);
    return probe_launched();
}

long long gc_b200_probe_ffma_flops(int blocks, int iters) {
    return 2LL * blocks * gcb::kProbeThreads * iters * gcb::kProbeUnroll * gcb::kProbeChains;
}

int gc_b200_probe_tf32_mma(uint32_t *status, int blocks, int iters, void *stream) {
    if (status == nullptr || blocks < 1 || blocks > (1 << 16) || iters < 1 || iters > (1 << 20))
        return gc_error(GC_INVALID, "probe_tf32_mma: status must be non-null, blocks in 1..65536, "
                                    "iters in 1..2^20");
    int st = probe_device_pointer(status);
    if (st != GC_OK) return st;
    gcb::tf32_mma_probe_kernel<<<blocks, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(status, iters);
    return probe_launched();
}

long long gc_b200_probe_tf32_mma_flops(int blocks, int iters) {
    return 2LL * gcb::kProbeM * gcb::kProbeN * 8 * static_cast<long long>(blocks) * iters;
}

int gc_b200_probe_copy(const void *src, void *dst, uint64_t bytes, int blocks, void *stream) {
    if (src == nullptr || dst == nullptr || bytes == 0 || bytes % 16 != 0 || !aligned16(src) || !aligned16(dst) ||
        blocks < 1 || blocks > (1 << 20))
        return gc_error(GC_INVALID, "probe_copy: 16-byte aligned non-null buffers, bytes a non-zero multiple "
                                    "of 16, blocks in 1..2^20");
    const char *s = static_cast<const char *>(src);
    const char *d = static_cast<const char *>(dst);
    if (s < d + bytes && d < s + bytes) return gc_error(GC_INVALID, "probe_copy: buffers overlap");
    int st = probe_device_pointer(src);
    if (st == GC_OK) st = probe_device_pointer(dst);
    if (st != GC_OK) return st;
    gcb::copy_probe_kernel<<<blocks, gcb::kProbeThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const float4 *>(src), static_cast<float4 *>(dst), static_cast<long long>(bytes / 16));
    return probe_launched();
}

}  // extern "C"
