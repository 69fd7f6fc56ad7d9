/*
 * gc_oracle.c - CPU restatement of the reference's grouped 2-D
 * cross-correlation, used ONLY as the checker of the B200 library.
 *
 * TEST INFRASTRUCTURE.  Nothing in the product (groupconv_atlas_b200/) links,
 * loads or calls this file; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py do.
 *
 * Each function restates one function of LucisZhang/groupconv-atlas:
 *   gco_conv_f32_serial   csrc/cpu/cpu_internal.h:7-22 (point) and
 *                         csrc/cpu/reference.cpp:20-26 (serial)
 *   gco_conv_f32_blocked  csrc/cpu/openmp.cpp:5-43 (c2 "blocked" tile, 32 wide)
 *   gco_conv_f64          csrc/cpu/reference.cpp:5-19 (FP64 oracle)
 * The per-output summation order (input channel, kernel row, kernel column,
 * skipping padded taps) and the plain multiply-then-add are the reference's,
 * so with -ffp-contract=off the FP32 results are bit-identical to the
 * reference's own CPU library.  gco_conv_f64_bound adds the quantity the
 * acceptance bound uses: sum over taps of |x*w| per output, in FP64.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

typedef struct {
    int64_t n, cin, cout, h, w, r, s, groups, sh, sw, ph, pw, dh, dw;
} gco_shape;

/* Output extent of a geometry already known to be valid. */
static int64_t extent(int64_t in, int64_t k, int64_t pad, int64_t dil, int64_t stride) {
    return (in + 2 * pad - dil * (k - 1) - 1) / stride + 1;
}

int gco_output(const gco_shape *p, int64_t *ho, int64_t *wo) {
    *ho = extent(p->h, p->r, p->ph, p->dh, p->sh);
    *wo = extent(p->w, p->s, p->pw, p->dw, p->sw);
    return (*ho > 0 && *wo > 0) ? 0 : 1;
}

/* One FP32 output, reference cpu_internal.h:7-22. */
static float point_f32(const gco_shape *p, const float *x, const float *w,
                       int64_t n, int64_t co, int64_t oh, int64_t ow) {
    const int64_t cpg = p->cin / p->groups;
    const int64_t group = co / (p->cout / p->groups);
    float sum = 0.0f;
    for (int64_t ci = 0; ci < cpg; ++ci) {
        for (int64_t r = 0; r < p->r; ++r) {
            const int64_t ih = oh * p->sh - p->ph + r * p->dh;
            if (ih < 0 || ih >= p->h) continue;
            for (int64_t s = 0; s < p->s; ++s) {
                const int64_t iw = ow * p->sw - p->pw + s * p->dw;
                if (iw < 0 || iw >= p->w) continue;
                const float xv = x[((n * p->cin + group * cpg + ci) * p->h + ih) * p->w + iw];
                const float wv = w[((co * cpg + ci) * p->r + r) * p->s + s];
                sum += xv * wv;
            }
        }
    }
    return sum;
}

void gco_conv_f32_serial(const gco_shape *p, const float *x, const float *w, float *y) {
    int64_t ho, wo;
    gco_output(p, &ho, &wo);
    for (int64_t n = 0; n < p->n; ++n)
        for (int64_t co = 0; co < p->cout; ++co)
            for (int64_t oh = 0; oh < ho; ++oh)
                for (int64_t ow = 0; ow < wo; ++ow)
                    y[((n * p->cout + co) * ho + oh) * wo + ow] = point_f32(p, x, w, n, co, oh, ow);
}

/* c2 "blocked": 32-wide output run per task, each weight reused across the
 * run, reference openmp.cpp:5-32 with the task split of openmp.cpp:34-43. */
#define GCO_TILE 32
void gco_conv_f32_blocked(const gco_shape *p, const float *x, const float *w, float *y,
                          int threads) {
    int64_t ho, wo;
    gco_output(p, &ho, &wo);
    const int64_t runs = (wo - 1) / GCO_TILE + 1;
    const int64_t tasks = p->n * p->cout * ho * runs;
    const int64_t cpg = p->cin / p->groups;
    const int64_t opg = p->cout / p->groups;
#pragma omp parallel for schedule(static) num_threads(threads)
    for (int64_t task = 0; task < tasks; ++task) {
        int64_t t = task;
        const int64_t ow0 = (t % runs) * GCO_TILE;
        t /= runs;
        const int64_t oh = t % ho;
        t /= ho;
        const int64_t co = t % p->cout;
        const int64_t n = t / p->cout;
        const int64_t len = wo - ow0 < GCO_TILE ? wo - ow0 : GCO_TILE;
        const int64_t group = co / opg;
        float acc[GCO_TILE];
        for (int64_t j = 0; j < GCO_TILE; ++j) acc[j] = 0.0f;
        for (int64_t ci = 0; ci < cpg; ++ci) {
            const float *plane = x + (n * p->cin + group * cpg + ci) * p->h * p->w;
            for (int64_t r = 0; r < p->r; ++r) {
                const int64_t ih = oh * p->sh - p->ph + r * p->dh;
                if (ih < 0 || ih >= p->h) continue;
                for (int64_t s = 0; s < p->s; ++s) {
                    const float wv = w[((co * cpg + ci) * p->r + r) * p->s + s];
                    for (int64_t j = 0; j < len; ++j) {
                        const int64_t iw = (ow0 + j) * p->sw - p->pw + s * p->dw;
                        if (iw >= 0 && iw < p->w) acc[j] += plane[ih * p->w + iw] * wv;
                    }
                }
            }
        }
        float *out = y + ((n * p->cout + co) * ho + oh) * wo + ow0;
        for (int64_t j = 0; j < len; ++j) out[j] = acc[j];
    }
}

/* FP64 oracle with its own loop nest and addressing, reference
 * reference.cpp:5-19. */
void gco_conv_f64(const gco_shape *p, const double *x, const double *w, double *y) {
    int64_t ho, wo;
    gco_output(p, &ho, &wo);
    const int64_t ic = p->cin / p->groups, oc = p->cout / p->groups;
    for (int64_t b = 0; b < p->n; ++b)
        for (int64_t g = 0; g < p->groups; ++g)
            for (int64_t o = 0; o < oc; ++o)
                for (int64_t row = 0; row < ho; ++row)
                    for (int64_t col = 0; col < wo; ++col) {
                        double v = 0.0;
                        for (int64_t c = 0; c < ic; ++c)
                            for (int64_t kr = 0; kr < p->r; ++kr)
                                for (int64_t ks = 0; ks < p->s; ++ks) {
                                    const int64_t ir = row * p->sh + kr * p->dh - p->ph;
                                    const int64_t is = col * p->sw + ks * p->dw - p->pw;
                                    if (ir < 0 || ir >= p->h || is < 0 || is >= p->w) continue;
                                    v += x[b * (p->cin * p->h * p->w) + (g * ic + c) * (p->h * p->w) +
                                           ir * p->w + is] *
                                         w[(g * oc + o) * (ic * p->r * p->s) + c * (p->r * p->s) +
                                           kr * p->s + ks];
                                }
                        y[((b * p->cout + g * oc + o) * ho + row) * wo + col] = v;
                    }
}

/* FP64 result of FP32 inputs plus, per output, bound[i] = sum |x*w| over the
 * taps that touch the image.  Same loop nest as gco_conv_f64; parallel over
 * (batch, output channel) planes because the checker runs it on large
 * tensors. */
void gco_conv_f64_bound(const gco_shape *p, const float *x, const float *w, double *y,
                        double *bound, int threads) {
    int64_t ho, wo;
    gco_output(p, &ho, &wo);
    const int64_t ic = p->cin / p->groups, oc = p->cout / p->groups;
    const int64_t planes = p->n * p->cout;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
    for (int64_t plane = 0; plane < planes; ++plane) {
        const int64_t b = plane / p->cout, co = plane % p->cout;
        const int64_t g = co / oc;
        for (int64_t row = 0; row < ho; ++row)
            for (int64_t col = 0; col < wo; ++col) {
                double v = 0.0, a = 0.0;
                for (int64_t c = 0; c < ic; ++c)
                    for (int64_t kr = 0; kr < p->r; ++kr) {
                        const int64_t ir = row * p->sh + kr * p->dh - p->ph;
                        if (ir < 0 || ir >= p->h) continue;
                        for (int64_t ks = 0; ks < p->s; ++ks) {
                            const int64_t is = col * p->sw + ks * p->dw - p->pw;
                            if (is < 0 || is >= p->w) continue;
                            const double prod =
                                (double)x[b * (p->cin * p->h * p->w) + (g * ic + c) * (p->h * p->w) +
                                          ir * p->w + is] *
                                (double)w[co * (ic * p->r * p->s) + c * (p->r * p->s) + kr * p->s + ks];
                            v += prod;
                            a += fabs(prod);
                        }
                    }
                const int64_t i = (plane * ho + row) * wo + col;
                y[i] = v;
                bound[i] = a;
            }
    }
}
