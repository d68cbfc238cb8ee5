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
#define ORC_TAU_EXACT 208.0f

enum { ORC_TIGHT = 0, ORC_EXACT = 1, ORC_FULL = 2 };

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
 * and the 3*max(scale) fallback (the reference); ORC_EXACT uses tau = 208
 * (exp(-q/2) == 0 in fp32 outside) and sqrt(208)*max(scale); ORC_FULL
 * writes the full-frame rectangle for every Gaussian.
 */
void orc_preprocess(int64_t n, int h, int w, int mode, const float* xy, const float* scale, const float* rot,
                    float* conic, int32_t* aabb, int32_t* count) {
    const int ntx = num_tiles_1d(w);
    const int nty = num_tiles_1d(h);
    const float tau = mode == ORC_EXACT ? ORC_TAU_EXACT : ORC_TAU_TIGHT;
    const float fb = mode == ORC_EXACT ? 14.422205101855956f : 3.0f;
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
void orc_render_backward(int64_t n, int f, int h, int w, const float* xy, const float* conic, const float* feat,
                         const float* opacity, const int32_t* gid_sorted, const int32_t* tile_offsets,
                         const float* grad, float* d_xy, float* d_conic, float* d_feat, float* d_opacity,
                         int64_t tile_lo, int64_t tile_hi) {
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
                    const float dx = (float)px - xy[2 * g];
                    const float dy = (float)py - xy[2 * g + 1];
                    const float q = quad_of(k, dx, dy);
                    if (!isfinite(q) || q < 0.0f) continue;
                    const double wgt = (double)expf(-0.5f * q);
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
        d_xy[2 * g] = (float)a[0];
        d_xy[2 * g + 1] = (float)a[1];
        d_conic[3 * g] = (float)a[2];
        d_conic[3 * g + 1] = (float)a[3];
        d_conic[3 * g + 2] = (float)a[4];
        const double op = opacity ? (double)opacity[g] : 1.0;
        double dop = 0.0;
        for (int c = 0; c < f; ++c) {
            d_feat[g * f + c] = (float)(a[5 + c] * op);
            dop += a[5 + c] * (double)feat[g * f + c];
        }
        if (d_opacity) d_opacity[g] = (float)dop;
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
