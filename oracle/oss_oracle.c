/*
 * oss_oracle.c -- CPU restatement of the reference rasterizer path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library and the CPU baseline of bench.py; nothing on the product path may
 * link or call it.
 *
 * Each function restates the reference algorithm it cites (paths relative to
 * the cashcon57/open-supersampling tree).  Arithmetic follows the reference's
 * operation order in fp32 with no FMA contraction (build with
 * -ffp-contract=off); cos/sin are evaluated in double and rounded once, the
 * same convention as the CUDA preprocess, so conics and tile AABBs agree bit
 * for bit with the GPU.  Gradient sums are accumulated in double.
 *
 * Pinned against the reference's own known-answer tests and golden vectors
 * generated from its PyTorch implementation (tests/golden/).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_TILE 16
#define ORC_MIN_SCALE 1.0e-6f
#define ORC_TAU_TIGHT 9.0f
#define ORC_TAU_EXACT 176.0f
#define ORC_TAU_EXACT56 56.0f

enum { ORC_TIGHT = 0, ORC_EXACT = 1, ORC_FULL = 2, ORC_EXACT56 = 3 };

static float clamp_min_keep_nan(float v, float lo) { return v < lo ? lo : v; }

/* cvt.rzi.s32.f32 semantics: truncate, saturate, NaN -> 0 */
static int sat_f2i(float v) {
    if (!(v == v)) return 0;
    if (v >= 2147483648.0f) return 2147483647;
    if (v <= -2147483648.0f) return -2147483647 - 1;
    return (int)v;
}

static int clamp_i(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

static int num_tiles_1d(int size) { return (size + ORC_TILE - 1) / ORC_TILE; }

/* rasterizer_fwd.cu:52-65 */
static void conic_of(float raw_sx, float raw_sy, float angle, float* a, float* b, float* d) {
    const float sx = clamp_min_keep_nan(raw_sx, ORC_MIN_SCALE);
    const float sy = clamp_min_keep_nan(raw_sy, ORC_MIN_SCALE);
    const float c = (float)cos((double)angle);
    const float s = (float)sin((double)angle);
    const float inv_sx2 = 1.0f / (sx * sx);
    const float inv_sy2 = 1.0f / (sy * sy);
    *a = c * c * inv_sx2 + s * s * inv_sy2;
    *b = c * s * (inv_sx2 - inv_sy2);
    *d = s * s * inv_sx2 + c * c * inv_sy2;
}

/*
 * preprocess_gaussians, rasterizer_fwd.cu:38-109.  mode ORC_TIGHT uses tau = 9
 * and the 3*max(scale) fallback (the reference); ORC_EXACT uses tau = 176
 * (exp(-q/2) below the smallest normal fp32 outside) and sqrt(176)*max(scale);
 * ORC_EXACT56 tau = 56 (weights left out below e^-28) and sqrt(56)*max(scale);
 * ORC_FULL
 * writes the full-frame rectangle for every Gaussian.
 */
void orc_preprocess(int64_t n, int h, int w, int mode, const float* xy, const float* scale, const float* rot,
                    float* conic, int32_t* aabb, int32_t* count) {
    const int ntx = num_tiles_1d(w);
    const int nty = num_tiles_1d(h);
    const float tau = mode == ORC_EXACT ? ORC_TAU_EXACT : (mode == ORC_EXACT56 ? ORC_TAU_EXACT56 : ORC_TAU_TIGHT);
    const float fb = mode == ORC_EXACT ? 13.266499161421599f : (mode == ORC_EXACT56 ? 7.483314773547883f : 3.0f);
#pragma omp parallel for schedule(static)
    for (int64_t g = 0; g < n; ++g) {
        float a, b, d;
        conic_of(scale[2 * g], scale[2 * g + 1], rot[g], &a, &b, &d);
        conic[3 * g + 0] = a;
        conic[3 * g + 1] = b;
        conic[3 * g + 2] = d;
        int32_t* box = aabb + 4 * g;
        if (mode == ORC_FULL) {
            box[0] = 0;
            box[1] = 0;
            box[2] = ntx;
            box[3] = nty;
            count[g] = ntx * nty;
            continue;
        }
        if (!isfinite(a) || !isfinite(b) || !isfinite(d)) {
            box[0] = box[1] = box[2] = box[3] = 0;
            count[g] = 0;
            continue;
        }
        float rx, ry;
        const float det = a * d - b * b;
        if (det > 1e-12f) {
            rx = sqrtf(tau * d / det);
            ry = sqrtf(tau * a / det);
        } else {
            const float r = fb * fmaxf(scale[2 * g], scale[2 * g + 1]);
            rx = r;
            ry = r;
        }
        const float cx = xy[2 * g], cy = xy[2 * g + 1];
        const float ts = (float)ORC_TILE;
        const int tx0 = clamp_i(sat_f2i(floorf((cx - rx) / ts)), 0, ntx);
        const int tx1 = clamp_i(sat_f2i(ceilf((cx + rx) / ts)), 0, ntx);
        const int ty0 = clamp_i(sat_f2i(floorf((cy - ry) / ts)), 0, nty);
        const int ty1 = clamp_i(sat_f2i(ceilf((cy + ry) / ts)), 0, nty);
        const int cnx = tx1 > tx0 ? tx1 - tx0 : 0;
        const int cny = ty1 > ty0 ? ty1 - ty0 : 0;
        box[0] = tx0;
        box[1] = ty0;
        box[2] = tx1;
        box[3] = ty1;
        count[g] = cnx * cny;
    }
}

static int cmp_u64(const void* x, const void* y) {
    const uint64_t a = *(const uint64_t*)x, b = *(const uint64_t*)y;
    return a < b ? -1 : (a > b ? 1 : 0);
}

/*
 * build_tile_pairs + sort + searchsorted, rasterizer_fwd.cu:111-133, 446-475:
 * keys (tile << 32 | gid) in gid-major order, sorted ascending; tile_offsets[t]
 * is the first position whose key is >= t << 32.  gid_sorted needs
 * sum(count) entries; returns that total.
 */
int64_t orc_pair_construction(int64_t n, int h, int w, const int32_t* aabb, const int32_t* count,
                              int32_t* gid_sorted, int32_t* tile_offsets) {
    const int ntx = num_tiles_1d(w);
    const int64_t num_tiles = (int64_t)ntx * num_tiles_1d(h);
    int64_t total = 0;
    for (int64_t g = 0; g < n; ++g) total += count[g];
    uint64_t* keys = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)(total > 0 ? total : 1));
    int64_t k = 0;
    for (int64_t g = 0; g < n; ++g) {
        const int32_t* b = aabb + 4 * g;
        for (int ty = b[1]; ty < b[3]; ++ty) {
            for (int tx = b[0]; tx < b[2]; ++tx) {
                const uint64_t tile = (uint64_t)((int64_t)ty * ntx + tx);
                keys[k++] = (tile << 32) | (uint32_t)g;
            }
        }
    }
    qsort(keys, (size_t)total, sizeof(uint64_t), cmp_u64);
    for (int64_t i = 0; i < total; ++i) gid_sorted[i] = (int32_t)(keys[i] & 0xffffffffu);
    int64_t pos = 0;
    for (int64_t t = 0; t <= num_tiles; ++t) {
        const uint64_t bound = (uint64_t)t << 32;
        while (pos < total && keys[pos] < bound) ++pos;
        tile_offsets[t] = (int32_t)pos;
    }
    free(keys);
    return total;
}

/* build_full_tile_pairs, rasterizer_fwd.cu:135-149 */
void orc_full_pairs(int64_t n, int64_t num_tiles, int32_t* gid_sorted, int32_t* tile_offsets) {
    for (int64_t t = 0; t < num_tiles; ++t)
        for (int64_t i = 0; i < n; ++i) gid_sorted[t * n + i] = (int32_t)i;
    for (int64_t t = 0; t <= num_tiles; ++t) tile_offsets[t] = (int32_t)(t * n);
}

/* q and weight of rasterizer_fwd.cu:242-247 / rasterizer_bwd.cu:82-89 */
static float quad_of(const float* k, float dx, float dy) {
    return k[0] * dx * dx + 2.0f * k[1] * dx * dy + k[2] * dy * dy;
}

/* The same expression with its products folded into fused multiply-adds, as a
 * CUDA build contracts it by default (the reference's op is compiled that way). */
static float quad_of_fma(const float* k, float dx, float dy) {
    return fmaf(k[2] * dy, dy, fmaf(2.0f * k[1] * dx, dy, (k[0] * dx) * dx));
}

/*
 * Additive forward over per-tile lists: out[c][p] = sum over the tile's list,
 * in list order, of feat'[g][c] * exp(-q/2) with q < 0 or non-finite giving 0
 * (rasterizer_fwd.cu:238-247; the sum of rasterizer.py:294-300).
 * feat' = feat * opacity when opacity is non-null.  Only tiles in
 * [tile_lo, tile_hi) are written (the CPU baseline renders a band of tiles).
 */
void orc_render_forward(int64_t n, int f, int h, int w, const float* xy, const float* conic, const float* feat,
                        const float* opacity, const int32_t* gid_sorted, const int32_t* tile_offsets, float* out,
                        int64_t tile_lo, int64_t tile_hi) {
    (void)n;
    const int ntx = num_tiles_1d(w);
    const int64_t plane = (int64_t)h * w;
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t t = tile_lo; t < tile_hi; ++t) {
        const int tx0 = (int)(t % ntx) * ORC_TILE, ty0 = (int)(t / ntx) * ORC_TILE;
        const int beg = tile_offsets[t], end = tile_offsets[t + 1];
        float acc[64];
        for (int ly = 0; ly < ORC_TILE; ++ly) {
            const int py = ty0 + ly;
            if (py >= h) break;
            for (int lx = 0; lx < ORC_TILE; ++lx) {
                const int px = tx0 + lx;
                if (px >= w) break;
                for (int c = 0; c < f; ++c) acc[c] = 0.0f;
                for (int j = beg; j < end; ++j) {
                    const int g = gid_sorted[j];
                    const float dx = (float)px - xy[2 * g];
                    const float dy = (float)py - xy[2 * g + 1];
                    const float q = quad_of(conic + 3 * g, dx, dy);
                    if (!isfinite(q) || q < 0.0f) continue;
                    const float wgt = expf(-0.5f * q);
                    const float op = opacity ? opacity[g] : 1.0f;
                    for (int c = 0; c < f; ++c) acc[c] += wgt * (feat[(int64_t)g * f + c] * op);
                }
                for (int c = 0; c < f; ++c) out[c * plane + (int64_t)py * w + px] = acc[c];
            }
        }
    }
}

/*
 * Backward of orc_render_forward, per pixel and list entry as in
 * rasterizer_bwd.cu:78-109:
 *   dL/dw = sum_c go_c feat'_c;  dL/dq = -0.5 w dL/dw
 *   d_xy -= dL/dq * (2a dx + 2b dy, 2b dx + 2d dy)
 *   d_conic += dL/dq * (dx^2, 2 dx dy, dy^2);  d_feat' += w go
 * Sums run in double: first per list entry over its tile's pixels, then per
 * Gaussian over list entries in list order.  d_feat = opacity * d_feat',
 * d_opacity = sum_c d_feat'_c feat_c.  Gradient outputs are overwritten.
 */
/* Gradients summed in double; written in double (d_*64, any may be null) and/or
 * rounded to fp32 (d_*32, any may be null).  exact_math: 0 = the reference's fp32
 * per-pixel terms, 1 = every per-pixel quantity in double, 2 = fp32 terms with q
 * formed by fused multiply-adds. */
static void render_backward_double(int64_t n, int f, int h, int w, const float* xy, const float* conic,
                                   const float* feat, const float* opacity, const int32_t* gid_sorted,
                                   const int32_t* tile_offsets, const float* grad, float* d_xy, float* d_conic,
                                   float* d_feat, float* d_opacity, double* d_xy64, double* d_conic64,
                                   double* d_feat64, double* d_opacity64, int64_t tile_lo, int64_t tile_hi,
                                   int exact_math);

void orc_render_backward(int64_t n, int f, int h, int w, const float* xy, const float* conic, const float* feat,
                         const float* opacity, const int32_t* gid_sorted, const int32_t* tile_offsets,
                         const float* grad, float* d_xy, float* d_conic, float* d_feat, float* d_opacity,
                         int64_t tile_lo, int64_t tile_hi) {
    render_backward_double(n, f, h, w, xy, conic, feat, opacity, gid_sorted, tile_offsets, grad, d_xy, d_conic,
                           d_feat, d_opacity, NULL, NULL, NULL, NULL, tile_lo, tile_hi, 0);
}

/*
 * The same gradients with every per-pixel quantity in double as well: offsets,
 * q, the weight exp(-q/2) and the terms, from the fp32 inputs (means, conic,
 * features, dL/dimage).  This is the exact value of the reference's formula at
 * its fp32 inputs; orc_render_backward instead sums the terms the reference's
 * fp32 arithmetic forms (its q keeps fp32 rounding, which for a thin Gaussian
 * cancels terms of both signs).  The parity bar is judged against this value,
 * with the reference's fp32 evaluations beside it.
 */
void orc_render_backward_exact(int64_t n, int f, int h, int w, const float* xy, const float* conic, const float* feat,
                               const float* opacity, const int32_t* gid_sorted, const int32_t* tile_offsets,
                               const float* grad, double* d_xy, double* d_conic, double* d_feat, double* d_opacity,
                               int64_t tile_lo, int64_t tile_hi) {
    /* outputs stay in double: a thin Gaussian's d_scale / d_rot cancel d_conic terms */
    render_backward_double(n, f, h, w, xy, conic, feat, opacity, gid_sorted, tile_offsets, grad, NULL, NULL, NULL,
                           NULL, d_xy, d_conic, d_feat, d_opacity, tile_lo, tile_hi, 1);
}

/* Double sums of the per-pixel terms with q formed by fused multiply-adds
 * (quad_of_fma): the terms of the reference's CUDA build, another fp32
 * evaluation of its formula. */
void orc_render_backward_fma(int64_t n, int f, int h, int w, const float* xy, const float* conic, const float* feat,
                             const float* opacity, const int32_t* gid_sorted, const int32_t* tile_offsets,
                             const float* grad, float* d_xy, float* d_conic, float* d_feat, float* d_opacity,
                             int64_t tile_lo, int64_t tile_hi) {
    render_backward_double(n, f, h, w, xy, conic, feat, opacity, gid_sorted, tile_offsets, grad, d_xy, d_conic,
                           d_feat, d_opacity, NULL, NULL, NULL, NULL, tile_lo, tile_hi, 2);
}

static void render_backward_double(int64_t n, int f, int h, int w, const float* xy, const float* conic,
                                   const float* feat, const float* opacity, const int32_t* gid_sorted,
                                   const int32_t* tile_offsets, const float* grad, float* d_xy, float* d_conic,
                                   float* d_feat, float* d_opacity, double* d_xy64, double* d_conic64,
                                   double* d_feat64, double* d_opacity64, int64_t tile_lo, int64_t tile_hi,
                                   int exact_math) {
    const int ntx = num_tiles_1d(w);
    const int64_t plane = (int64_t)h * w;
    const int stride = 5 + f;
    const int64_t p_lo = tile_offsets[tile_lo], p_hi = tile_offsets[tile_hi];
    double* pacc = (double*)calloc((size_t)((p_hi - p_lo) * stride + 1), sizeof(double));
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t t = tile_lo; t < tile_hi; ++t) {
        const int tx0 = (int)(t % ntx) * ORC_TILE, ty0 = (int)(t / ntx) * ORC_TILE;
        const int beg = tile_offsets[t], end = tile_offsets[t + 1];
        for (int j = beg; j < end; ++j) {
            const int g = gid_sorted[j];
            const float* k = conic + 3 * g;
            const float op = opacity ? opacity[g] : 1.0f;
            double* acc = pacc + (int64_t)(j - p_lo) * stride;
            for (int ly = 0; ly < ORC_TILE; ++ly) {
                const int py = ty0 + ly;
                if (py >= h) break;
                for (int lx = 0; lx < ORC_TILE; ++lx) {
                    const int px = tx0 + lx;
                    if (px >= w) break;
                    double dx, dy, wgt;
                    if (exact_math == 1) {
                        dx = (double)px - (double)xy[2 * g];
                        dy = (double)py - (double)xy[2 * g + 1];
                        const double q = (double)k[0] * dx * dx + 2.0 * (double)k[1] * dx * dy + (double)k[2] * dy * dy;
                        if (!isfinite(q) || q < 0.0) continue;
                        wgt = exp(-0.5 * q);
                    } else {
                        const float fdx = (float)px - xy[2 * g];
                        const float fdy = (float)py - xy[2 * g + 1];
                        const float q = exact_math == 2 ? quad_of_fma(k, fdx, fdy) : quad_of(k, fdx, fdy);
                        if (!isfinite(q) || q < 0.0f) continue;
                        dx = fdx;
                        dy = fdy;
                        wgt = (double)expf(-0.5f * q);
                    }
                    double dldw = 0.0;
                    const int64_t pix = (int64_t)py * w + px;
                    for (int c = 0; c < f; ++c) {
                        const double go = grad[c * plane + pix];
                        dldw += go * ((double)feat[(int64_t)g * f + c] * op);
                        acc[5 + c] += wgt * go;
                    }
                    const double dldq = -0.5 * wgt * dldw;
                    acc[0] -= dldq * (2.0 * k[0] * dx + 2.0 * k[1] * dy);
                    acc[1] -= dldq * (2.0 * k[1] * dx + 2.0 * k[2] * dy);
                    acc[2] += dldq * dx * dx;
                    acc[3] += dldq * 2.0 * dx * dy;
                    acc[4] += dldq * dy * dy;
                }
            }
        }
    }
    double* gacc = (double*)calloc((size_t)(n * stride + 1), sizeof(double));
    for (int64_t j = p_lo; j < p_hi; ++j) {
        const int g = gid_sorted[j];
        for (int v = 0; v < stride; ++v) gacc[(int64_t)g * stride + v] += pacc[(j - p_lo) * stride + v];
    }
    for (int64_t g = 0; g < n; ++g) {
        const double* a = gacc + g * stride;
        const double op = opacity ? (double)opacity[g] : 1.0;
        double dop = 0.0;
        for (int c = 0; c < f; ++c) {
            const double v = a[5 + c] * op;
            if (d_feat) d_feat[g * f + c] = (float)v;
            if (d_feat64) d_feat64[g * f + c] = v;
            dop += a[5 + c] * (double)feat[g * f + c];
        }
        for (int i = 0; i < 2; ++i) {
            if (d_xy) d_xy[2 * g + i] = (float)a[i];
            if (d_xy64) d_xy64[2 * g + i] = a[i];
        }
        for (int i = 0; i < 3; ++i) {
            if (d_conic) d_conic[3 * g + i] = (float)a[2 + i];
            if (d_conic64) d_conic64[3 * g + i] = a[2 + i];
        }
        if (d_opacity) d_opacity[g] = (float)dop;
        if (d_opacity64) d_opacity64[g] = dop;
    }
    free(gacc);
    free(pacc);
}

/*
 * The same backward summed the way the reference's kernel sums it: in fp32,
 * one term per pixel and list entry added straight into the Gaussian's
 * accumulator (rasterizer_bwd.cu:95-108 adds them with float atomics; this is
 * one order those atomics may run in: tiles ascending, pixels row-major, list
 * entries in list order; with `reverse` every one of those orders reversed).  The opacity unfold is the fp32 product and dot
 * product the reference's callers get from autograd.  This is not the parity
 * target (orc_render_backward's double sums are): it measures how far the
 * reference's own fp32 evaluation lies from those sums, element by element.
 * Threads own the Gaussians g = tid (mod threads), so every accumulator is
 * added to in the order above.
 */
void orc_render_backward_f32(int64_t n, int f, int h, int w, const float* xy, const float* conic, const float* feat,
                             const float* opacity, const int32_t* gid_sorted, const int32_t* tile_offsets,
                             const float* grad, float* d_xy, float* d_conic, float* d_feat, float* d_opacity,
                             int64_t tile_lo, int64_t tile_hi, int reverse) {
    const int ntx = num_tiles_1d(w);
    const int64_t plane = (int64_t)h * w;
    const int stride = 5 + f;
    float* acc = (float*)calloc((size_t)(n * stride + 1), sizeof(float));
#pragma omp parallel
    {
        int nt = 1, tid = 0;
#ifdef _OPENMP
        nt = omp_get_num_threads();
        tid = omp_get_thread_num();
#endif
        int cap = 0;
        int32_t* mine = NULL;  /* this thread's Gaussians of the tile's list, in list order */
        for (int64_t tt = tile_lo; tt < tile_hi; ++tt) {
            const int64_t t = reverse ? tile_hi - 1 - (tt - tile_lo) : tt;
            const int tx0 = (int)(t % ntx) * ORC_TILE, ty0 = (int)(t / ntx) * ORC_TILE;
            const int beg = tile_offsets[t], end = tile_offsets[t + 1];
            if (end - beg > cap) {
                cap = end - beg;
                mine = (int32_t*)realloc(mine, sizeof(int32_t) * (size_t)cap);
            }
            int m = 0;
            for (int j = beg; j < end; ++j) {
                if (gid_sorted[j] % nt == tid) mine[m++] = gid_sorted[j];
            }
            if (m == 0) continue;
            for (int p = 0; p < ORC_TILE * ORC_TILE; ++p) {
                const int pp = reverse ? ORC_TILE * ORC_TILE - 1 - p : p;
                const int py = ty0 + pp / ORC_TILE, px = tx0 + pp % ORC_TILE;
                if (py >= h || px >= w) continue;
                {
                    const int64_t pix = (int64_t)py * w + px;
                    for (int ii = 0; ii < m; ++ii) {
                        const int g = mine[reverse ? m - 1 - ii : ii];
                        const float* k = conic + 3 * g;
                        const float op = opacity ? opacity[g] : 1.0f;
                        const float dx = (float)px - xy[2 * g];
                        const float dy = (float)py - xy[2 * g + 1];
                        const float q = quad_of(k, dx, dy);
                        if (!isfinite(q) || q < 0.0f) continue;
                        const float wgt = expf(-0.5f * q);
                        float* a = acc + (int64_t)g * stride;
                        float dldw = 0.0f;
                        for (int c = 0; c < f; ++c) {
                            const float go = grad[c * plane + pix];
                            dldw += go * (feat[(int64_t)g * f + c] * op);
                            a[5 + c] += wgt * go;
                        }
                        const float dldq = -0.5f * wgt * dldw;
                        a[0] -= dldq * (2.0f * k[0] * dx + 2.0f * k[1] * dy);
                        a[1] -= dldq * (2.0f * k[1] * dx + 2.0f * k[2] * dy);
                        a[2] += dldq * dx * dx;
                        a[3] += dldq * 2.0f * dx * dy;
                        a[4] += dldq * dy * dy;
                    }
                }
            }
        }
        free(mine);
    }
    for (int64_t g = 0; g < n; ++g) {
        const float* a = acc + g * stride;
        d_xy[2 * g] = a[0];
        d_xy[2 * g + 1] = a[1];
        d_conic[3 * g] = a[2];
        d_conic[3 * g + 1] = a[3];
        d_conic[3 * g + 2] = a[4];
        const float op = opacity ? opacity[g] : 1.0f;
        float dop = 0.0f;
        for (int c = 0; c < f; ++c) {
            d_feat[g * f + c] = a[5 + c] * op;
            dop += a[5 + c] * feat[g * f + c];
        }
        if (d_opacity) d_opacity[g] = dop;
    }
    free(acc);
}

/*
 * Front-to-back alpha compositing over per-tile lists: a build-defined mode (the
 * reference rasterizer is additive only; its design notes name gsplat-style
 * compositing, RESEARCH.md:114, without code).  The standard over operator, per
 * pixel, in list order (lists sorted by (depth, gid)):
 *   G_i = exp(-q_i/2) (0 for q < 0 or non-finite);  a_i = min(0.99, opacity_i G_i)
 *   skip the entry when a_i < 1/255;
 *   stop before the first entry whose T (1 - a_i) would fall below 1e-4;
 *   C += feat_i a_i T;  T *= 1 - a_i;   out = C + T * background.
 * C and T are carried in double.  t_final[p] = T, n_contrib[p] = 1 + the
 * position in the tile list of the last composited entry (0 if none).
 * ambiguous[p] (optional) = 1 when one of the pixel's skip / clamp / stop tests
 * lies within a relative 2e-5 (1e-4 for the transmittance test) of its
 * threshold: there, fp32 rounding of q, of exp or of the running transmittance
 * (a few ulp per entry) may decide it either way.
 */
#define ORC_ALPHA_MAX 0.99
#define ORC_ALPHA_MIN (1.0 / 255.0)
#define ORC_T_MIN 1e-4

static int near_rel(double v, double thr, double rel) { return fabs(v - thr) <= rel * thr; }

void orc_render_alpha_forward(int64_t n, int f, int h, int w, const float* xy, const float* conic, const float* feat,
                              const float* opacity, const float* background, const int32_t* gid_sorted,
                              const int32_t* tile_offsets, float* out, float* t_final, int32_t* n_contrib,
                              uint8_t* ambiguous, int64_t tile_lo, int64_t tile_hi) {
    (void)n;
    const int ntx = num_tiles_1d(w);
    const int64_t plane = (int64_t)h * w;
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t t = tile_lo; t < tile_hi; ++t) {
        const int tx0 = (int)(t % ntx) * ORC_TILE, ty0 = (int)(t / ntx) * ORC_TILE;
        const int beg = tile_offsets[t], end = tile_offsets[t + 1];
        double acc[64];
        for (int ly = 0; ly < ORC_TILE; ++ly) {
            const int py = ty0 + ly;
            if (py >= h) break;
            for (int lx = 0; lx < ORC_TILE; ++lx) {
                const int px = tx0 + lx;
                if (px >= w) break;
                for (int c = 0; c < f; ++c) acc[c] = 0.0;
                double T = 1.0;
                int last = 0;
                int amb = 0;
                for (int j = beg; j < end; ++j) {
                    const int g = gid_sorted[j];
                    const float dx = (float)px - xy[2 * g];
                    const float dy = (float)py - xy[2 * g + 1];
                    const float q = quad_of(conic + 3 * g, dx, dy);
                    if (!isfinite(q) || q < 0.0f) continue;
                    const double og = (double)opacity[g] * (double)expf(-0.5f * q);
                    amb |= near_rel(og, ORC_ALPHA_MAX, 2e-5) | near_rel(og, ORC_ALPHA_MIN, 2e-5);
                    const double a = og < ORC_ALPHA_MAX ? og : ORC_ALPHA_MAX;
                    if (a < ORC_ALPHA_MIN) continue;
                    const double tn = T * (1.0 - a);
                    amb |= near_rel(tn, ORC_T_MIN, 1e-4);
                    if (tn < ORC_T_MIN) break;
                    for (int c = 0; c < f; ++c) acc[c] += (double)feat[(int64_t)g * f + c] * a * T;
                    T = tn;
                    last = j - beg + 1;
                }
                const int64_t pix = (int64_t)py * w + px;
                for (int c = 0; c < f; ++c) {
                    const double bg = background ? (double)background[c] : 0.0;
                    out[c * plane + pix] = (float)(acc[c] + T * bg);
                }
                if (t_final) t_final[pix] = (float)T;
                if (n_contrib) n_contrib[pix] = last;
                if (ambiguous) ambiguous[pix] = (uint8_t)amb;
            }
        }
    }
}

/*
 * Backward of orc_render_alpha_forward.  Per pixel the forward is replayed in
 * double (a_i, T_i, which entries composite), then entries are visited back to
 * front with S = the normalised colour behind entry i (S starts at the
 * background):
 *   dL/da_i = T_i sum_c go_c (feat_ic - S_c);  d feat_ic += a_i T_i go_c;
 *   S_c = feat_ic a_i + S_c (1 - a_i)
 * then, where a_i = opacity_i G_i is not clamped at 0.99,
 *   d opacity_i += G_i dL/da_i;  dL/dq = -0.5 G_i opacity_i dL/da_i
 * and d_xy, d_conic follow from dL/dq exactly as in the additive backward.
 * Per-entry sums in double, then per Gaussian over list entries in list order.
 */
void orc_render_alpha_backward(int64_t n, int f, int h, int w, const float* xy, const float* conic,
                               const float* feat, const float* opacity, const float* background,
                               const int32_t* gid_sorted, const int32_t* tile_offsets, const float* grad,
                               float* d_xy, float* d_conic, float* d_feat, float* d_opacity, int64_t tile_lo,
                               int64_t tile_hi) {
    const int ntx = num_tiles_1d(w);
    const int64_t plane = (int64_t)h * w;
    const int stride = 6 + f;
    const int64_t p_lo = tile_offsets[tile_lo], p_hi = tile_offsets[tile_hi];
    double* pacc = (double*)calloc((size_t)((p_hi - p_lo) * stride + 1), sizeof(double));
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t t = tile_lo; t < tile_hi; ++t) {
        const int tx0 = (int)(t % ntx) * ORC_TILE, ty0 = (int)(t / ntx) * ORC_TILE;
        const int beg = tile_offsets[t], end = tile_offsets[t + 1];
        const int len = end - beg;
        if (len == 0) continue;
        double* av = (double*)malloc(sizeof(double) * (size_t)len * 3);  /* a, T before, G */
        uint8_t* on = (uint8_t*)malloc((size_t)len);
        for (int ly = 0; ly < ORC_TILE; ++ly) {
            const int py = ty0 + ly;
            if (py >= h) break;
            for (int lx = 0; lx < ORC_TILE; ++lx) {
                const int px = tx0 + lx;
                if (px >= w) break;
                const int64_t pix = (int64_t)py * w + px;
                double T = 1.0;
                int last = 0;
                for (int j = 0; j < len; ++j) {
                    on[j] = 0;
                    const int g = gid_sorted[beg + j];
                    const float dx = (float)px - xy[2 * g];
                    const float dy = (float)py - xy[2 * g + 1];
                    const float q = quad_of(conic + 3 * g, dx, dy);
                    if (!isfinite(q) || q < 0.0f) continue;
                    const double G = (double)expf(-0.5f * q);
                    const double og = (double)opacity[g] * G;
                    const double a = og < ORC_ALPHA_MAX ? og : ORC_ALPHA_MAX;
                    if (a < ORC_ALPHA_MIN) continue;
                    const double tn = T * (1.0 - a);
                    if (tn < ORC_T_MIN) break;
                    av[3 * j] = a;
                    av[3 * j + 1] = T;
                    av[3 * j + 2] = G;
                    on[j] = (uint8_t)(og < ORC_ALPHA_MAX ? 1 : 2);
                    T = tn;
                    last = j + 1;
                }
                double S[64];
                for (int c = 0; c < f; ++c) S[c] = background ? (double)background[c] : 0.0;
                for (int j = last - 1; j >= 0; --j) {
                    if (!on[j]) continue;
                    const int g = gid_sorted[beg + j];
                    const double a = av[3 * j], Ti = av[3 * j + 1], G = av[3 * j + 2];
                    double* acc = pacc + (int64_t)(beg + j - p_lo) * stride;
                    double dlda = 0.0;
                    for (int c = 0; c < f; ++c) {
                        const double go = grad[c * plane + pix];
                        const double fc = (double)feat[(int64_t)g * f + c];
                        dlda += go * (fc - S[c]);
                        acc[5 + c] += a * Ti * go;
                        S[c] = fc * a + S[c] * (1.0 - a);
                    }
                    dlda *= Ti;
                    if (on[j] != 1) continue;  /* clamped at 0.99: no gradient through G or opacity */
                    acc[5 + f] += G * dlda;
                    const float* k = conic + 3 * g;
                    const double dx = (double)((float)px - xy[2 * g]);
                    const double dy = (double)((float)py - xy[2 * g + 1]);
                    const double dldq = -0.5 * G * (double)opacity[g] * dlda;
                    acc[0] -= dldq * (2.0 * k[0] * dx + 2.0 * k[1] * dy);
                    acc[1] -= dldq * (2.0 * k[1] * dx + 2.0 * k[2] * dy);
                    acc[2] += dldq * dx * dx;
                    acc[3] += dldq * 2.0 * dx * dy;
                    acc[4] += dldq * dy * dy;
                }
            }
        }
        free(on);
        free(av);
    }
    double* gacc = (double*)calloc((size_t)(n * stride + 1), sizeof(double));
    for (int64_t j = p_lo; j < p_hi; ++j) {
        const int g = gid_sorted[j];
        for (int v = 0; v < stride; ++v) gacc[(int64_t)g * stride + v] += pacc[(j - p_lo) * stride + v];
    }
    for (int64_t g = 0; g < n; ++g) {
        const double* a = gacc + g * stride;
        d_xy[2 * g] = (float)a[0];
        d_xy[2 * g + 1] = (float)a[1];
        d_conic[3 * g] = (float)a[2];
        d_conic[3 * g + 1] = (float)a[3];
        d_conic[3 * g + 2] = (float)a[4];
        for (int c = 0; c < f; ++c) d_feat[g * f + c] = (float)a[5 + c];
        if (d_opacity) d_opacity[g] = (float)a[5 + f];
    }
    free(gacc);
    free(pacc);
}

/* conic_to_scale_rot_grad, rasterizer_bwd.cu:128-153 */
void orc_conic_to_scale_rot_grad(int64_t n, const float* scale, const float* rot, const float* d_conic,
                                 float* d_scale, float* d_rot) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const float rsx = scale[2 * i], rsy = scale[2 * i + 1];
        const float sx = fmaxf(rsx, ORC_MIN_SCALE);
        const float sy = fmaxf(rsy, ORC_MIN_SCALE);
        const float inv_sx2 = 1.0f / (sx * sx);
        const float inv_sy2 = 1.0f / (sy * sy);
        const float diff = inv_sx2 - inv_sy2;
        const float c = (float)cos((double)rot[i]);
        const float s = (float)sin((double)rot[i]);
        const float cc = c * c, ss = s * s, cs = c * s;
        const float dca = d_conic[3 * i], dcb = d_conic[3 * i + 1], dcd = d_conic[3 * i + 2];
        const float d_inv_sx2 = cc * dca + cs * dcb + ss * dcd;
        const float d_inv_sy2 = ss * dca - cs * dcb + cc * dcd;
        d_scale[2 * i] = rsx > ORC_MIN_SCALE ? d_inv_sx2 * (-2.0f / (rsx * rsx * rsx)) : 0.0f;
        d_scale[2 * i + 1] = rsy > ORC_MIN_SCALE ? d_inv_sy2 * (-2.0f / (rsy * rsy * rsy)) : 0.0f;
        d_rot[i] = dca * (-2.0f * cs * diff) + dcb * (diff * (cc - ss)) + dcd * (2.0f * cs * diff);
    }
}

/*
 * tile_bin_counting_sort, tile_bin_counting_sort.cu:24-67, restated as a
 * stable counting sort: per-tile counts of valid ids, exclusive offsets,
 * offsets[T] = n, then entries in input order (valid ones per tile, the
 * out-of-range ones after all valid entries).
 */
void orc_tile_bin_counting_sort(int64_t n, int64_t num_tiles, const int32_t* tile_id, const int32_t* gid,
                                int32_t* sorted_gid, int32_t* tile_offsets) {
    int64_t* cursor = (int64_t*)calloc((size_t)(num_tiles + 1), sizeof(int64_t));
    for (int64_t i = 0; i < n; ++i) {
        const int32_t t = tile_id[i];
        if (t >= 0 && t < num_tiles) cursor[t]++;
    }
    int64_t run = 0;
    for (int64_t t = 0; t < num_tiles; ++t) {
        const int64_t c = cursor[t];
        tile_offsets[t] = (int32_t)run;
        cursor[t] = run;
        run += c;
    }
    tile_offsets[num_tiles] = (int32_t)n;
    int64_t invalid = run;
    for (int64_t i = 0; i < n; ++i) {
        const int32_t t = tile_id[i];
        if (t >= 0 && t < num_tiles) sorted_gid[cursor[t]++] = gid[i];
        else sorted_gid[invalid++] = gid[i];
    }
    free(cursor);
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int t) {
#ifdef _OPENMP
    if (t > 0) omp_set_num_threads(t);
#else
    (void)t;
#endif
}

/* ------------------------------------------------------------------------
 * Canvas warp, oss/sr/v6/canvas_warp.py:177-254 (GS-STVSR), restated per
 * Gaussian without materialising the HR motion field.
 * motion_lr[2][hl][wl] is the first batch item; alpha pre-multiplies it (the
 * extrapolation-alpha composition warp_canvas(canvas, alpha * motion_lr, hw)).
 * ---------------------------------------------------------------------- */
typedef struct {
    const float* m;
    int hl, wl, h, w;
    float alpha, scale_y, scale_x;
    int same;
} orc_field;

static float orc_lr(const orc_field* f, int ch, int y, int x) {
    return f->alpha * f->m[((int64_t)ch * f->hl + y) * f->wl + x];
}

/* F.interpolate(bilinear, align_corners=False) texel of the HR field
 * (aten area_pixel_compute_source_index + linear weights) */
static float orc_hr(const orc_field* f, int ch, int i, int j) {
    if (f->same) return orc_lr(f, ch, i, j);
    float sy = f->scale_y * ((float)i + 0.5f) - 0.5f;
    if (sy < 0.0f) sy = 0.0f;
    float sx = f->scale_x * ((float)j + 0.5f) - 0.5f;
    if (sx < 0.0f) sx = 0.0f;
    const int y0 = (int)sy, x0 = (int)sx;
    const int y1 = y0 + (y0 < f->hl - 1 ? 1 : 0), x1 = x0 + (x0 < f->wl - 1 ? 1 : 0);
    float ly1 = sy - (float)y0;
    if (ly1 > 1.0f) ly1 = 1.0f;
    float lx1 = sx - (float)x0;
    if (lx1 > 1.0f) lx1 = 1.0f;
    const float ly0 = 1.0f - ly1, lx0 = 1.0f - lx1;
    return ly0 * (lx0 * orc_lr(f, ch, y0, x0) + lx1 * orc_lr(f, ch, y0, x1)) +
           ly1 * (lx0 * orc_lr(f, ch, y1, x0) + lx1 * orc_lr(f, ch, y1, x1));
}

/* kind 0: HR motion; 1: d/dx central difference; 2: d/dy (replicate pad) */
static float orc_field_at(const orc_field* f, int kind, int ch, int i, int j) {
    if (kind == 0) return orc_hr(f, ch, i, j);
    if (kind == 1) {
        const int jp = j + 1 < f->w ? j + 1 : f->w - 1, jm = j - 1 >= 0 ? j - 1 : 0;
        return (orc_hr(f, ch, i, jp) - orc_hr(f, ch, i, jm)) * 0.5f;
    }
    const int ip = i + 1 < f->h ? i + 1 : f->h - 1, im = i - 1 >= 0 ? i - 1 : 0;
    return (orc_hr(f, ch, ip, j) - orc_hr(f, ch, im, j)) * 0.5f;
}

/* F.grid_sample(bilinear, align_corners=False) at pixel position (x, y);
 * border != 0 clips the source coordinate (padding_mode="border"), else
 * out-of-range taps read 0 (padding_mode="zeros"). */
static float orc_grid_sample(const orc_field* f, int kind, int ch, float x, float y, int border) {
    const float gx = (x / (float)f->w) * 2.0f - 1.0f;
    const float gy = (y / (float)f->h) * 2.0f - 1.0f;
    float ix = ((gx + 1.0f) * (float)f->w - 1.0f) / 2.0f;
    float iy = ((gy + 1.0f) * (float)f->h - 1.0f) / 2.0f;
    if (border) {
        ix = fminf((float)(f->w - 1), fmaxf(ix, 0.0f));
        iy = fminf((float)(f->h - 1), fmaxf(iy, 0.0f));
    }
    const float x0 = floorf(ix), y0 = floorf(iy);
    const float wx = ix - x0, wy = iy - y0;
    const float ex = 1.0f - wx, sy = 1.0f - wy;
    const float wts[4] = {sy * ex, sy * wx, wy * ex, wy * wx};
    /* every tap out of range (or NaN coordinates): zero padding */
    if (!(x0 > -2.0f && x0 < (float)f->w && y0 > -2.0f && y0 < (float)f->h)) return 0.0f;
    const int xs[4] = {(int)x0, (int)x0 + 1, (int)x0, (int)x0 + 1};
    const int ys[4] = {(int)y0, (int)y0, (int)y0 + 1, (int)y0 + 1};
    float out = 0.0f;
    for (int k = 0; k < 4; ++k) {
        if (xs[k] >= 0 && xs[k] < f->w && ys[k] >= 0 && ys[k] < f->h)
            out += orc_field_at(f, kind, ch, ys[k], xs[k]) * wts[k];
    }
    return out;
}

/*
 * Per Gaussian: new position, in-frame flag, and (for non-identity Jacobians)
 * the resampled covariance J S J^T + recon (+ symmetrise + 1e-7 ridge,
 * covariance_resampling.py:76-116) decomposed largest axis first
 * (canvas_warp.py:148-166).  recon is 2x2 row-major.  Survivors are compacted
 * in input order; returns their count.  colors is [n][f].
 */
int64_t orc_warp_canvas(int64_t n, int f, int hl, int wl, int h, int w, const float* motion, float alpha,
                        const float* recon, const float* pos, const float* scales, const float* rots,
                        const float* ops, const float* colors, float* out_pos, float* out_scales, float* out_rots,
                        float* out_ops, float* out_colors) {
    orc_field fld = {motion, hl, wl, h, w, alpha, (float)hl / (float)h, (float)wl / (float)w,
                     (hl == h && wl == w) ? 1 : 0};
    int64_t k = 0;
    for (int64_t g = 0; g < n; ++g) {
        const float x = pos[2 * g], y = pos[2 * g + 1];
        const float nx = x + orc_grid_sample(&fld, 0, 0, x, y, 0);
        const float ny = y + orc_grid_sample(&fld, 0, 1, x, y, 0);
        const int in_frame = nx >= 0.0f && nx < (float)w && ny >= 0.0f && ny < (float)h;
        const float j00 = 1.0f + orc_grid_sample(&fld, 1, 0, x, y, 1);
        const float j10 = 0.0f + orc_grid_sample(&fld, 1, 1, x, y, 1);
        const float j01 = 0.0f + orc_grid_sample(&fld, 2, 0, x, y, 1);
        const float j11 = 1.0f + orc_grid_sample(&fld, 2, 1, x, y, 1);
        float s0 = scales[2 * g], s1 = scales[2 * g + 1], r = rots[g];
        const float dev = fmaxf(fmaxf(fabsf(j00 - 1.0f), fabsf(j01)), fmaxf(fabsf(j10), fabsf(j11 - 1.0f)));
        if (!(dev < 1.0e-5f)) {
            const float c = (float)cos((double)r), s = (float)sin((double)r);
            const float a0 = fmaxf(s0, 0.0f), a1 = fmaxf(s1, 0.0f);
            const float v0 = a0 * a0, v1 = a1 * a1;
            /* R diag(v) R^T with R = [[c, -s], [s, c]] */
            const float p00 = c * v0, p01 = -s * v1, p10 = s * v0, p11 = c * v1;
            const float q00 = p00 * c + p01 * (-s), q01 = p00 * s + p01 * c;
            const float q10 = p10 * c + p11 * (-s), q11 = p10 * s + p11 * c;
            /* J S J^T */
            const float t00 = j00 * q00 + j01 * q10, t01 = j00 * q01 + j01 * q11;
            const float t10 = j10 * q00 + j11 * q10, t11 = j10 * q01 + j11 * q11;
            float u00 = t00 * j00 + t01 * j01, u01 = t00 * j10 + t01 * j11;
            float u10 = t10 * j00 + t11 * j01, u11 = t10 * j10 + t11 * j11;
            u00 += recon[0];
            u01 += recon[1];
            u10 += recon[2];
            u11 += recon[3];
            /* _ensure_positive_definite: symmetrise + 1e-7 I */
            const float m01 = 0.5f * (u01 + u10);
            float e00 = 0.5f * (u00 + u00) + 1.0e-7f, e11 = 0.5f * (u11 + u11) + 1.0e-7f;
            float e01 = m01 + 0.0f;
            /* _scales_rotations_from_covariance */
            const float a = 0.5f * (e00 + e00), b = 0.5f * (e01 + e01), cc = 0.5f * (e11 + e11);
            const float ht = 0.5f * (a + cc), hd = 0.5f * (a - cc);
            const float rad = sqrtf(hd * hd + b * b + 1.0e-12f);
            float eig0 = ht + rad, eig1 = ht - rad;
            if (eig0 < 1.0e-12f) eig0 = 1.0e-12f;
            if (eig1 < 1.0e-12f) eig1 = 1.0e-12f;
            s0 = sqrtf(eig0);
            s1 = sqrtf(eig1);
            r = 0.5f * atan2f(2.0f * b, a - cc);
        }
        if (in_frame) {
            out_pos[2 * k] = nx;
            out_pos[2 * k + 1] = ny;
            out_scales[2 * k] = s0;
            out_scales[2 * k + 1] = s1;
            out_rots[k] = r;
            out_ops[k] = ops[g];
            for (int c = 0; c < f; ++c) out_colors[k * f + c] = colors[g * f + c];
            ++k;
        }
    }
    return k;
}

/* warp_positions, oss/gaussian/canvas/warp.py:28-91: motion given at the
 * output resolution (hl == h, wl == w), scaled by alpha; no compaction. */
void orc_warp_positions(int64_t n, int h, int w, const float* motion, float alpha, const float* xy, float* out_xy,
                        uint8_t* in_frame) {
    orc_field fld = {motion, h, w, h, w, alpha, 1.0f, 1.0f, 1};
    for (int64_t g = 0; g < n; ++g) {
        const float x = xy[2 * g], y = xy[2 * g + 1];
        const float nx = x + orc_grid_sample(&fld, 0, 0, x, y, 0);
        const float ny = y + orc_grid_sample(&fld, 0, 1, x, y, 0);
        out_xy[2 * g] = nx;
        out_xy[2 * g + 1] = ny;
        in_frame[g] = nx >= 0.0f && nx < (float)w && ny >= 0.0f && ny < (float)h;
    }
}
