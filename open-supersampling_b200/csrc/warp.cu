// Canvas warp (oss/sr/v6/canvas_warp.py:177-254, GS-STVSR) and the alpha-scaled
// position warp (oss/gaussian/canvas/warp.py:28-91), one thread per Gaussian.
//
// The reference materialises the bilinearly upsampled HR motion field and two
// HR central-difference fields, then grid-samples them.  Here every HR texel a
// Gaussian touches is evaluated on the fly from the LR field (4 LR loads, all
// L1/L2 hits: the LR field is 4 MB at 540x960), so per Gaussian the kernel
// reads 20 B of canvas and writes 20 B + a flag -- HBM-bound, no HR buffers.
// Survivors (new centre inside the frame) are compacted in input order by a
// flag scan and a scatter.  Arithmetic mirrors the reference op order without
// FMA contraction (the same restatement as oracle/oss_oracle.c).
#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

constexpr int kThreads = 256;

struct Field {
    const float* m;  // [2][hl][wl]
    int hl, wl, h, w;
    float alpha, scale_y, scale_x;
    int same;
    double scale_y_d, scale_x_d;  // hl / h and wl / w in double (the backward's exact weights)
};

__device__ __forceinline__ float lr_at(const Field& f, int ch, int y, int x) {
    return __fmul_rn(f.alpha, __ldg(f.m + (static_cast<int64_t>(ch) * f.hl + y) * f.wl + x));
}

// Texel of F.interpolate(motion, (h, w), bilinear, align_corners=False).
__device__ float hr_at(const Field& f, int ch, int i, int j) {
    if (f.same) return lr_at(f, ch, i, j);
    float sy = __fsub_rn(__fmul_rn(f.scale_y, __fadd_rn(static_cast<float>(i), 0.5f)), 0.5f);
    if (sy < 0.0f) sy = 0.0f;
    float sx = __fsub_rn(__fmul_rn(f.scale_x, __fadd_rn(static_cast<float>(j), 0.5f)), 0.5f);
    if (sx < 0.0f) sx = 0.0f;
    const int y0 = static_cast<int>(sy), x0 = static_cast<int>(sx);
    const int y1 = y0 + (y0 < f.hl - 1 ? 1 : 0), x1 = x0 + (x0 < f.wl - 1 ? 1 : 0);
    const float ly1 = fminf(__fsub_rn(sy, static_cast<float>(y0)), 1.0f);
    const float lx1 = fminf(__fsub_rn(sx, static_cast<float>(x0)), 1.0f);
    const float ly0 = __fsub_rn(1.0f, ly1), lx0 = __fsub_rn(1.0f, lx1);
    const float top = __fadd_rn(__fmul_rn(lx0, lr_at(f, ch, y0, x0)), __fmul_rn(lx1, lr_at(f, ch, y0, x1)));
    const float bot = __fadd_rn(__fmul_rn(lx0, lr_at(f, ch, y1, x0)), __fmul_rn(lx1, lr_at(f, ch, y1, x1)));
    return __fadd_rn(__fmul_rn(ly0, top), __fmul_rn(ly1, bot));
}

// kind 0: motion; 1: d/dx, 2: d/dy central differences with replicate padding.
__device__ float field_at(const Field& f, int kind, int ch, int i, int j) {
    if (kind == 0) return hr_at(f, ch, i, j);
    if (kind == 1) {
        const int jp = j + 1 < f.w ? j + 1 : f.w - 1, jm = j - 1 >= 0 ? j - 1 : 0;
        return __fmul_rn(__fsub_rn(hr_at(f, ch, i, jp), hr_at(f, ch, i, jm)), 0.5f);
    }
    const int ip = i + 1 < f.h ? i + 1 : f.h - 1, im = i - 1 >= 0 ? i - 1 : 0;
    return __fmul_rn(__fsub_rn(hr_at(f, ch, ip, j), hr_at(f, ch, im, j)), 0.5f);
}

// F.grid_sample(bilinear, align_corners=False) at pixel position (x, y); border
// clips the source coordinate, otherwise out-of-range taps read zero.
__device__ float grid_sample(const Field& f, int kind, int ch, float x, float y, bool border) {
    const float gx = __fsub_rn(__fmul_rn(__fdiv_rn(x, static_cast<float>(f.w)), 2.0f), 1.0f);
    const float gy = __fsub_rn(__fmul_rn(__fdiv_rn(y, static_cast<float>(f.h)), 2.0f), 1.0f);
    float ix = __fdiv_rn(__fsub_rn(__fmul_rn(__fadd_rn(gx, 1.0f), static_cast<float>(f.w)), 1.0f), 2.0f);
    float iy = __fdiv_rn(__fsub_rn(__fmul_rn(__fadd_rn(gy, 1.0f), static_cast<float>(f.h)), 1.0f), 2.0f);
    if (border) {
        ix = fminf(static_cast<float>(f.w - 1), fmaxf(ix, 0.0f));
        iy = fminf(static_cast<float>(f.h - 1), fmaxf(iy, 0.0f));
    }
    const float x0 = floorf(ix), y0 = floorf(iy);
    const float wx = __fsub_rn(ix, x0), wy = __fsub_rn(iy, y0);
    const float ex = __fsub_rn(1.0f, wx), sy = __fsub_rn(1.0f, wy);
    const float wts[4] = {__fmul_rn(sy, ex), __fmul_rn(sy, wx), __fmul_rn(wy, ex), __fmul_rn(wy, wx)};
    // coordinates beyond int range cannot be in bounds; keep them out without UB
    if (!(x0 > -2.0f && x0 < static_cast<float>(f.w) && y0 > -2.0f && y0 < static_cast<float>(f.h))) return 0.0f;
    const int xi = static_cast<int>(x0), yi = static_cast<int>(y0);
    float out = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int xx = xi + (k & 1), yy = yi + (k >> 1);
        if (xx >= 0 && xx < f.w && yy >= 0 && yy < f.h) out = __fadd_rn(out, __fmul_rn(field_at(f, kind, ch, yy, xx), wts[k]));
    }
    return out;
}

__global__ void __launch_bounds__(kThreads) k_warp_eval(int n, Field fld, float4 recon,
                                                         const float2* __restrict__ pos,
                                                         const float2* __restrict__ scales,
                                                         const float* __restrict__ rots, float4* __restrict__ tmp,
                                                         int32_t* __restrict__ flag) {
    const int g = blockIdx.x * kThreads + threadIdx.x;
    if (g >= n) return;
    const float2 p = pos[g];
    const float nx = __fadd_rn(p.x, grid_sample(fld, 0, 0, p.x, p.y, false));
    const float ny = __fadd_rn(p.y, grid_sample(fld, 0, 1, p.x, p.y, false));
    const bool in_frame = nx >= 0.0f && nx < static_cast<float>(fld.w) && ny >= 0.0f && ny < static_cast<float>(fld.h);
    const float j00 = __fadd_rn(1.0f, grid_sample(fld, 1, 0, p.x, p.y, true));
    const float j10 = __fadd_rn(0.0f, grid_sample(fld, 1, 1, p.x, p.y, true));
    const float j01 = __fadd_rn(0.0f, grid_sample(fld, 2, 0, p.x, p.y, true));
    const float j11 = __fadd_rn(1.0f, grid_sample(fld, 2, 1, p.x, p.y, true));
    const float2 s = scales[g];
    float s0 = s.x, s1 = s.y, r = rots[g];
    const float dev = fmaxf(fmaxf(fabsf(__fsub_rn(j00, 1.0f)), fabsf(j01)), fmaxf(fabsf(j10), fabsf(__fsub_rn(j11, 1.0f))));
    if (!(dev < 1.0e-5f)) {  // _identity_j_mask, canvas_warp.py:169-174
        float c, sn;
        cos_sin_rn(r, c, sn);
        const float a0 = fmaxf(s0, 0.0f), a1 = fmaxf(s1, 0.0f);
        const float v0 = __fmul_rn(a0, a0), v1 = __fmul_rn(a1, a1);
        const float p00 = __fmul_rn(c, v0), p01 = __fmul_rn(-sn, v1), p10 = __fmul_rn(sn, v0), p11 = __fmul_rn(c, v1);
        const float q00 = __fadd_rn(__fmul_rn(p00, c), __fmul_rn(p01, -sn));
        const float q01 = __fadd_rn(__fmul_rn(p00, sn), __fmul_rn(p01, c));
        const float q10 = __fadd_rn(__fmul_rn(p10, c), __fmul_rn(p11, -sn));
        const float q11 = __fadd_rn(__fmul_rn(p10, sn), __fmul_rn(p11, c));
        const float t00 = __fadd_rn(__fmul_rn(j00, q00), __fmul_rn(j01, q10));
        const float t01 = __fadd_rn(__fmul_rn(j00, q01), __fmul_rn(j01, q11));
        const float t10 = __fadd_rn(__fmul_rn(j10, q00), __fmul_rn(j11, q10));
        const float t11 = __fadd_rn(__fmul_rn(j10, q01), __fmul_rn(j11, q11));
        const float u00 = __fadd_rn(__fadd_rn(__fmul_rn(t00, j00), __fmul_rn(t01, j01)), recon.x);
        const float u01 = __fadd_rn(__fadd_rn(__fmul_rn(t00, j10), __fmul_rn(t01, j11)), recon.y);
        const float u10 = __fadd_rn(__fadd_rn(__fmul_rn(t10, j00), __fmul_rn(t11, j01)), recon.z);
        const float u11 = __fadd_rn(__fadd_rn(__fmul_rn(t10, j10), __fmul_rn(t11, j11)), recon.w);
        // symmetrise + 1e-7 ridge (covariance_resampling.py:32-44), then the
        // closed-form eigendecomposition (canvas_warp.py:148-166)
        const float a = __fadd_rn(__fmul_rn(0.5f, __fadd_rn(u00, u00)), 1.0e-7f);
        const float b = __fadd_rn(__fmul_rn(0.5f, __fadd_rn(u01, u10)), 0.0f);
        const float cc = __fadd_rn(__fmul_rn(0.5f, __fadd_rn(u11, u11)), 1.0e-7f);
        const float ht = __fmul_rn(0.5f, __fadd_rn(a, cc)), hd = __fmul_rn(0.5f, __fsub_rn(a, cc));
        const float rad = __fsqrt_rn(__fadd_rn(__fadd_rn(__fmul_rn(hd, hd), __fmul_rn(b, b)), 1.0e-12f));
        const float eig0 = fmaxf(__fadd_rn(ht, rad), 1.0e-12f);
        const float eig1 = fmaxf(__fsub_rn(ht, rad), 1.0e-12f);
        s0 = __fsqrt_rn(eig0);
        s1 = __fsqrt_rn(eig1);
        r = __fmul_rn(0.5f, atan2f(__fmul_rn(2.0f, b), __fsub_rn(a, cc)));
    }
    tmp[2 * g] = make_float4(nx, ny, s0, s1);
    tmp[2 * g + 1] = make_float4(r, 0.0f, 0.0f, 0.0f);
    flag[g] = in_frame ? 1 : 0;
}

// PARKED: no compaction.  Every Gaussian keeps its slot (offs holds the
// in-frame flags); a dropped one is written far outside the frame with zero
// opacity and colours, so it bins into no tile and renders nothing -- the
// survivors' image without the host read of the survivor count.
template <bool PARKED>
__global__ void __launch_bounds__(kThreads) k_warp_scatter(int n, int f, const float4* __restrict__ tmp,
                                                            const int32_t* __restrict__ offs,
                                                            const float* __restrict__ ops,
                                                            const float* __restrict__ colors,
                                                            float2* __restrict__ out_pos,
                                                            float2* __restrict__ out_scales,
                                                            float* __restrict__ out_rots, float* __restrict__ out_ops,
                                                            float* __restrict__ out_colors) {
    const int g = blockIdx.x * kThreads + threadIdx.x;
    if (g >= n) return;
    int k = g;
    if (PARKED) {
        if (offs[g] == 0) {
            out_pos[g] = make_float2(-1.0e7f, -1.0e7f);
            out_scales[g] = make_float2(1.0f, 1.0f);
            out_rots[g] = 0.0f;
            out_ops[g] = 0.0f;
            for (int c = 0; c < f; ++c) out_colors[static_cast<int64_t>(g) * f + c] = 0.0f;
            return;
        }
    } else {
        k = offs[g];
        if (offs[g + 1] == k) return;  // dropped: new centre outside the frame
    }
    const float4 a = tmp[2 * g];
    out_pos[k] = make_float2(a.x, a.y);
    out_scales[k] = make_float2(a.z, a.w);
    out_rots[k] = tmp[2 * g + 1].x;
    out_ops[k] = ops[g];
    for (int c = 0; c < f; ++c) out_colors[static_cast<int64_t>(k) * f + c] = colors[static_cast<int64_t>(g) * f + c];
}

__global__ void __launch_bounds__(kThreads) k_warp_positions(int n, Field fld, const float2* __restrict__ xy,
                                                              float2* __restrict__ out_xy,
                                                              uint8_t* __restrict__ in_frame) {
    const int g = blockIdx.x * kThreads + threadIdx.x;
    if (g >= n) return;
    const float2 p = xy[g];
    const float nx = __fadd_rn(p.x, grid_sample(fld, 0, 0, p.x, p.y, false));
    const float ny = __fadd_rn(p.y, grid_sample(fld, 0, 1, p.x, p.y, false));
    out_xy[g] = make_float2(nx, ny);
    in_frame[g] = (nx >= 0.0f && nx < static_cast<float>(fld.w) && ny >= 0.0f && ny < static_cast<float>(fld.h)) ? 1 : 0;
}

// ---------------------------------------------------------------------------
// Backward of the canvas warp (the gradients PyTorch's autograd takes through
// canvas_warp.py:177-254 and covariance_resampling.py:76-116).
//
// One thread per input Gaussian recomputes its forward values.  A survivor
// (output slot k = offs[g]) receives the upstream gradients of slot k; a dropped
// Gaussian gets zero.  The motion sample and the four Jacobian samples are
// bilinear in the position and linear in their fields: their position
// derivatives add to d_pos, and their field weights are added (fp64 atomics)
// into six HR gradient planes in double (motion x/y, d/dx of motion x/y, d/dy of
// motion x/y).  k_warp_motion_grad then folds the central differences back onto the
// motion planes and k_warp_lr_grad transposes the bilinear upsampling by a
// gather per LR texel, so only the Gaussians' atomics depend on order.
// ---------------------------------------------------------------------------

// The fields in double, for the backward's derivatives: the Jacobian path
// differentiates sampled central differences (second differences of the
// upsampled motion), where fp32 rounding of each texel would dominate.
__device__ double hr_at_f64(const Field& f, int ch, int i, int j) {
    auto lr = [&](int y, int x) {
        return static_cast<double>(f.alpha) * static_cast<double>(__ldg(f.m + (static_cast<int64_t>(ch) * f.hl + y) * f.wl + x));
    };
    if (f.same) return lr(i, j);
    float sy = __fsub_rn(__fmul_rn(f.scale_y, __fadd_rn(static_cast<float>(i), 0.5f)), 0.5f);
    if (sy < 0.0f) sy = 0.0f;
    float sx = __fsub_rn(__fmul_rn(f.scale_x, __fadd_rn(static_cast<float>(j), 0.5f)), 0.5f);
    if (sx < 0.0f) sx = 0.0f;
    // taps as the forward chooses them (fp32), weights exact
    const int y0 = static_cast<int>(sy), x0 = static_cast<int>(sx);
    const int y1 = y0 + (y0 < f.hl - 1 ? 1 : 0), x1 = x0 + (x0 < f.wl - 1 ? 1 : 0);
    const double syd = fmax(f.scale_y_d * (static_cast<double>(i) + 0.5) - 0.5, 0.0);
    const double sxd = fmax(f.scale_x_d * (static_cast<double>(j) + 0.5) - 0.5, 0.0);
    const double ly1 = fmin(syd - y0, 1.0), lx1 = fmin(sxd - x0, 1.0);
    const double ly0 = 1.0 - ly1, lx0 = 1.0 - lx1;
    return ly0 * (lx0 * lr(y0, x0) + lx1 * lr(y0, x1)) + ly1 * (lx0 * lr(y1, x0) + lx1 * lr(y1, x1));
}

__device__ double field_at_f64(const Field& f, int kind, int ch, int i, int j) {
    if (kind == 0) return hr_at_f64(f, ch, i, j);
    if (kind == 1) {
        const int jp = j + 1 < f.w ? j + 1 : f.w - 1, jm = j - 1 >= 0 ? j - 1 : 0;
        return 0.5 * (hr_at_f64(f, ch, i, jp) - hr_at_f64(f, ch, i, jm));
    }
    const int ip = i + 1 < f.h ? i + 1 : f.h - 1, im = i - 1 >= 0 ? i - 1 : 0;
    return 0.5 * (hr_at_f64(f, ch, ip, j) - hr_at_f64(f, ch, im, j));
}

// grid_sample's backward (bilinear, align_corners=False): returns d out / d x and
// d out / d y of the sample at (x, y) and, when `dfield` is non-null, adds
// g * (tap weight) into the tapped texels of dfield (an HR plane).  Border mode
// clips the source coordinate and, as PyTorch does, passes no gradient through a
// clipped coordinate (the borders themselves count as out of range).
__device__ float2 grid_sample_grad(const Field& f, int kind, int ch, float x, float y, bool border, float g,
                                   double* __restrict__ dfield) {
    const float gx = __fsub_rn(__fmul_rn(__fdiv_rn(x, static_cast<float>(f.w)), 2.0f), 1.0f);
    const float gy = __fsub_rn(__fmul_rn(__fdiv_rn(y, static_cast<float>(f.h)), 2.0f), 1.0f);
    float ix = __fdiv_rn(__fsub_rn(__fmul_rn(__fadd_rn(gx, 1.0f), static_cast<float>(f.w)), 1.0f), 2.0f);
    float iy = __fdiv_rn(__fsub_rn(__fmul_rn(__fadd_rn(gy, 1.0f), static_cast<float>(f.h)), 1.0f), 2.0f);
    float mx = 1.0f, my = 1.0f;
    if (border) {
        if (ix <= 0.0f) { ix = 0.0f; mx = 0.0f; }
        else if (ix >= static_cast<float>(f.w - 1)) { ix = static_cast<float>(f.w - 1); mx = 0.0f; }
        if (iy <= 0.0f) { iy = 0.0f; my = 0.0f; }
        else if (iy >= static_cast<float>(f.h - 1)) { iy = static_cast<float>(f.h - 1); my = 0.0f; }
    }
    const float x0 = floorf(ix), y0 = floorf(iy);
    if (!(x0 > -2.0f && x0 < static_cast<float>(f.w) && y0 > -2.0f && y0 < static_cast<float>(f.h))) {
        return make_float2(0.0f, 0.0f);
    }
    const int xi = static_cast<int>(x0), yi = static_cast<int>(y0);
    // the forward's taps with exact weights: the source coordinate is x - 1/2 (or
    // the border it was clipped to)
    const double wx = (mx == 0.0f ? static_cast<double>(ix) : static_cast<double>(x) - 0.5) - x0;
    const double wy = (my == 0.0f ? static_cast<double>(iy) : static_cast<double>(y) - 0.5) - y0;
    const double ex = 1.0 - wx, sy = 1.0 - wy;
    const double wts[4] = {sy * ex, sy * wx, wy * ex, wy * wx};
    // d weight / d ix and d weight / d iy of the four taps
    const double dwx[4] = {-sy, sy, -wy, wy};
    const double dwy[4] = {-ex, -wx, ex, wx};
    double dix = 0.0, diy = 0.0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int xx = xi + (k & 1), yy = yi + (k >> 1);
        if (xx >= 0 && xx < f.w && yy >= 0 && yy < f.h) {
            const double v = field_at_f64(f, kind, ch, yy, xx);
            dix += v * dwx[k];
            diy += v * dwy[k];
            if (dfield != nullptr) {
                atomicAdd(dfield + static_cast<int64_t>(yy) * f.w + xx, static_cast<double>(g) * wts[k]);
            }
        }
    }
    // ix = x - 1/2 and iy = y - 1/2 up to rounding: d ix / d x = 1
    return make_float2(static_cast<float>(g * dix * mx), static_cast<float>(g * diy * my));
}

// grid_sample's value with the field in double (bilinear, align_corners=False).
__device__ double grid_sample_f64(const Field& f, int kind, int ch, float x, float y, bool border) {
    const float gx = __fsub_rn(__fmul_rn(__fdiv_rn(x, static_cast<float>(f.w)), 2.0f), 1.0f);
    const float gy = __fsub_rn(__fmul_rn(__fdiv_rn(y, static_cast<float>(f.h)), 2.0f), 1.0f);
    float ix = __fdiv_rn(__fsub_rn(__fmul_rn(__fadd_rn(gx, 1.0f), static_cast<float>(f.w)), 1.0f), 2.0f);
    float iy = __fdiv_rn(__fsub_rn(__fmul_rn(__fadd_rn(gy, 1.0f), static_cast<float>(f.h)), 1.0f), 2.0f);
    bool cx = false, cy = false;
    if (border) {
        const float bx = fminf(static_cast<float>(f.w - 1), fmaxf(ix, 0.0f));
        const float by = fminf(static_cast<float>(f.h - 1), fmaxf(iy, 0.0f));
        cx = bx != ix;
        cy = by != iy;
        ix = bx;
        iy = by;
    }
    const float x0 = floorf(ix), y0 = floorf(iy);
    if (!(x0 > -2.0f && x0 < static_cast<float>(f.w) && y0 > -2.0f && y0 < static_cast<float>(f.h))) return 0.0;
    // the source coordinate is x - 1/2 exactly (or the border it was clipped to); the
    // taps are the forward's
    const double ixd = cx ? static_cast<double>(ix) : static_cast<double>(x) - 0.5;
    const double iyd = cy ? static_cast<double>(iy) : static_cast<double>(y) - 0.5;
    const double wx = ixd - x0, wy = iyd - y0;
    const double wts[4] = {(1.0 - wy) * (1.0 - wx), (1.0 - wy) * wx, wy * (1.0 - wx), wy * wx};
    const int xi = static_cast<int>(x0), yi = static_cast<int>(y0);
    double out = 0.0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int xx = xi + (k & 1), yy = yi + (k >> 1);
        if (xx >= 0 && xx < f.w && yy >= 0 && yy < f.h) out += field_at_f64(f, kind, ch, yy, xx) * wts[k];
    }
    return out;
}

__global__ void __launch_bounds__(kThreads) k_warp_backward(
    int n, int f, Field fld, float4 recon, const float2* __restrict__ pos, const float2* __restrict__ scales,
    const float* __restrict__ rots, const int32_t* __restrict__ offs, const float2* __restrict__ g_pos,
    const float2* __restrict__ g_scales, const float* __restrict__ g_rots, const float* __restrict__ g_ops,
    const float* __restrict__ g_colors, float2* __restrict__ d_pos, float2* __restrict__ d_scales,
    float* __restrict__ d_rots, float* __restrict__ d_ops, float* __restrict__ d_colors, double* __restrict__ d_hr) {
    const int g = blockIdx.x * kThreads + threadIdx.x;
    if (g >= n) return;
    const int k = offs[g];
    if (offs[g + 1] == k) {  // dropped: the outputs do not depend on it
        d_pos[g] = make_float2(0.0f, 0.0f);
        d_scales[g] = make_float2(0.0f, 0.0f);
        d_rots[g] = 0.0f;
        if (d_ops != nullptr) d_ops[g] = 0.0f;
        for (int c = 0; c < f; ++c) d_colors[static_cast<int64_t>(g) * f + c] = 0.0f;
        return;
    }
    const float2 gp = g_pos != nullptr ? g_pos[k] : make_float2(0.0f, 0.0f);
    const float2 gs = g_scales != nullptr ? g_scales[k] : make_float2(0.0f, 0.0f);
    const float gr = g_rots != nullptr ? g_rots[k] : 0.0f;
    if (d_ops != nullptr) d_ops[g] = g_ops != nullptr ? g_ops[k] : 0.0f;
    for (int c = 0; c < f; ++c) {
        d_colors[static_cast<int64_t>(g) * f + c] = g_colors != nullptr ? g_colors[static_cast<int64_t>(k) * f + c] : 0.0f;
    }
    const int64_t plane = static_cast<int64_t>(fld.h) * fld.w;
    const float2 p = pos[g];
    // new position = p + m(p): d p = g_pos + (d m / d p)^T g_pos
    float2 dp = gp;
    {
        const float2 a = grid_sample_grad(fld, 0, 0, p.x, p.y, false, gp.x, d_hr);
        const float2 b = grid_sample_grad(fld, 0, 1, p.x, p.y, false, gp.y, d_hr + plane);
        dp.x += a.x + b.x;
        dp.y += a.y + b.y;
    }
    const float j00 = __fadd_rn(1.0f, grid_sample(fld, 1, 0, p.x, p.y, true));
    const float j10 = __fadd_rn(0.0f, grid_sample(fld, 1, 1, p.x, p.y, true));
    const float j01 = __fadd_rn(0.0f, grid_sample(fld, 2, 0, p.x, p.y, true));
    const float j11 = __fadd_rn(1.0f, grid_sample(fld, 2, 1, p.x, p.y, true));
    const float2 s = scales[g];
    const float th = rots[g];
    const float dev = fmaxf(fmaxf(fabsf(__fsub_rn(j00, 1.0f)), fabsf(j01)), fmaxf(fabsf(j10), fabsf(__fsub_rn(j11, 1.0f))));
    if (dev < 1.0e-5f) {  // identity Jacobian: scales and rotation pass through
        d_pos[g] = dp;
        d_scales[g] = gs;
        d_rots[g] = gr;
        return;
    }
    // the covariance chain again, in double: the eigendecomposition's derivatives
    // are ill-conditioned where the resampled covariance is nearly isotropic, so
    // fp32 rounding of J, U and the eigenvalues would dominate them
    const double J00 = 1.0 + grid_sample_f64(fld, 1, 0, p.x, p.y, true);
    const double J10 = grid_sample_f64(fld, 1, 1, p.x, p.y, true);
    const double J01 = grid_sample_f64(fld, 2, 0, p.x, p.y, true);
    const double J11 = 1.0 + grid_sample_f64(fld, 2, 1, p.x, p.y, true);
    double sn, c;
    sincos(static_cast<double>(th), &sn, &c);
    const double a0 = fmax(static_cast<double>(s.x), 0.0), a1 = fmax(static_cast<double>(s.y), 0.0);
    const double v0 = a0 * a0, v1 = a1 * a1;
    const double q00 = c * c * v0 + sn * sn * v1, q01 = c * sn * (v0 - v1), q11 = sn * sn * v0 + c * c * v1;
    const double t00 = J00 * q00 + J01 * q01, t01 = J00 * q01 + J01 * q11;
    const double t10 = J10 * q00 + J11 * q01, t11 = J10 * q01 + J11 * q11;
    const double u00 = t00 * J00 + t01 * J01 + recon.x;
    const double u01 = t00 * J10 + t01 * J11 + recon.y;
    const double u10 = t10 * J00 + t11 * J01 + recon.z;
    const double u11 = t10 * J10 + t11 * J11 + recon.w;
    const double a = u00 + 1.0e-7, b = 0.5 * (u01 + u10), cc = u11 + 1.0e-7;
    const double ht = 0.5 * (a + cc), hd = 0.5 * (a - cc);
    const double rad = sqrt(hd * hd + b * b + 1.0e-12);
    const double e0 = ht + rad, e1 = ht - rad;
    // backward of the eigendecomposition: s_i = sqrt(max(e_i, 1e-12)), r = atan2(2b, a - c) / 2
    const double d_e0 = e0 >= 1.0e-12 ? gs.x * 0.5 / sqrt(e0) : 0.0;
    const double d_e1 = e1 >= 1.0e-12 ? gs.y * 0.5 / sqrt(e1) : 0.0;
    const double d_ht = d_e0 + d_e1, d_rad = d_e0 - d_e1;
    const double d_hd = d_rad * hd / rad;
    double d_b = d_rad * b / rad;
    const double ax = a - cc, ay = 2.0 * b, r2 = ax * ax + ay * ay;
    double d_ax = 0.0;
    if (r2 > 0.0) {  // atan2 has no derivative where both arguments vanish (exactly isotropic)
        d_b += 0.5 * gr * 2.0 * ax / r2;
        d_ax = 0.5 * gr * (-ay) / r2;
    }
    const double d_a = 0.5 * d_ht + 0.5 * d_hd + d_ax;
    const double d_c = 0.5 * d_ht - 0.5 * d_hd - d_ax;
    // U = J Q J^T + R, symmetrised: dU = [[d_a, d_b / 2], [d_b / 2, d_c]]
    const double g00 = d_a, g01 = 0.5 * d_b, g11 = d_c;
    // dJ = 2 dU J Q (dU and Q symmetric)
    const double m00 = g00 * J00 + g01 * J10, m01 = g00 * J01 + g01 * J11;
    const double m10 = g01 * J00 + g11 * J10, m11 = g01 * J01 + g11 * J11;
    const float dj00 = static_cast<float>(2.0 * (m00 * q00 + m01 * q01));
    const float dj01 = static_cast<float>(2.0 * (m00 * q01 + m01 * q11));
    const float dj10 = static_cast<float>(2.0 * (m10 * q00 + m11 * q01));
    const float dj11 = static_cast<float>(2.0 * (m10 * q01 + m11 * q11));
    // dQ = J^T dU J
    const double w00 = J00 * g00 + J10 * g01, w01 = J00 * g01 + J10 * g11;
    const double w10 = J01 * g00 + J11 * g01, w11 = J01 * g01 + J11 * g11;
    const double dq00 = w00 * J00 + w01 * J10, dq01 = w00 * J01 + w01 * J11;
    const double dq10 = w10 * J00 + w11 * J10, dq11 = w10 * J01 + w11 * J11;
    // Q = R diag(v) R^T, v = max(s, 0)^2
    const double dqs = dq01 + dq10;
    const double dv0 = c * c * dq00 + c * sn * dqs + sn * sn * dq11;
    const double dv1 = sn * sn * dq00 - c * sn * dqs + c * c * dq11;
    d_scales[g] = make_float2(s.x >= 0.0f ? static_cast<float>(2.0 * a0 * dv0) : 0.0f,
                              s.y >= 0.0f ? static_cast<float>(2.0 * a1 * dv1) : 0.0f);
    d_rots[g] = static_cast<float>((v0 - v1) * (-2.0 * c * sn * dq00 + (c * c - sn * sn) * dqs + 2.0 * c * sn * dq11));
    // J = I + [d/dx m, d/dy m] sampled with border padding
    float2 t;
    t = grid_sample_grad(fld, 1, 0, p.x, p.y, true, dj00, d_hr + 2 * plane);
    dp.x += t.x;
    dp.y += t.y;
    t = grid_sample_grad(fld, 1, 1, p.x, p.y, true, dj10, d_hr + 3 * plane);
    dp.x += t.x;
    dp.y += t.y;
    t = grid_sample_grad(fld, 2, 0, p.x, p.y, true, dj01, d_hr + 4 * plane);
    dp.x += t.x;
    dp.y += t.y;
    t = grid_sample_grad(fld, 2, 1, p.x, p.y, true, dj11, d_hr + 5 * plane);
    dp.x += t.x;
    dp.y += t.y;
    d_pos[g] = dp;
}

// Gradient of the HR motion planes: the motion sample's plane plus the central
// differences (with replicate padding) transposed onto their taps:
// dmdx[i][j] = (m[i][min(j + 1, w - 1)] - m[i][max(j - 1, 0)]) / 2, and dmdy alike.
// Writes planes 0 and 1 of d_hr in place of the sample's.
__global__ void __launch_bounds__(kThreads) k_warp_motion_grad(int h, int w, double* __restrict__ d_hr) {
    const int64_t plane = static_cast<int64_t>(h) * w;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (idx >= 2 * plane) return;
    const int ch = static_cast<int>(idx / plane);
    const int64_t pix = idx - ch * plane;
    const int i = static_cast<int>(pix / w), j = static_cast<int>(pix - static_cast<int64_t>(i) * w);
    const double* gx = d_hr + (2 + ch) * plane + static_cast<int64_t>(i) * w;  // row i of d(dm/dx)
    const double* gy = d_hr + (4 + ch) * plane;                              // d(dm/dy)
    double v = d_hr[idx];
    // texel j is the + tap of column j - 1 (and of w - 1 itself at the right edge) and
    // the - tap of column j + 1 (and of 0 itself at the left edge)
    if (j >= 1) v += 0.5 * gx[j - 1];
    if (j == w - 1) v += 0.5 * gx[w - 1];
    if (j + 1 <= w - 1) v -= 0.5 * gx[j + 1];
    if (j == 0) v -= 0.5 * gx[0];
    if (i >= 1) v += 0.5 * gy[static_cast<int64_t>(i - 1) * w + j];
    if (i == h - 1) v += 0.5 * gy[static_cast<int64_t>(h - 1) * w + j];
    if (i + 1 <= h - 1) v -= 0.5 * gy[static_cast<int64_t>(i + 1) * w + j];
    if (i == 0) v -= 0.5 * gy[j];
    d_hr[idx] = v;
}

// One LR axis of F.interpolate(bilinear, align_corners=False): the two LR taps of
// HR index i and their weights (the forward's hr_at arithmetic).
__device__ __forceinline__ void lr_taps(float scale, int i, int nl, int& t0, int& t1, float& w0, float& w1) {
    float sp = __fsub_rn(__fmul_rn(scale, __fadd_rn(static_cast<float>(i), 0.5f)), 0.5f);
    if (sp < 0.0f) sp = 0.0f;
    t0 = static_cast<int>(sp);
    t1 = t0 + (t0 < nl - 1 ? 1 : 0);
    w1 = fminf(__fsub_rn(sp, static_cast<float>(t0)), 1.0f);
    w0 = __fsub_rn(1.0f, w1);
}

// d motion_lr = alpha * (upsampling)^T d motion_hr, one thread per LR texel
// gathering the HR texels whose taps include it (a window of rows and columns
// around its image under the upsampling), in a fixed order.
__global__ void __launch_bounds__(kThreads) k_warp_lr_grad(Field f, const double* __restrict__ d_hr,
                                                            float* __restrict__ d_motion) {
    const int64_t lplane = static_cast<int64_t>(f.hl) * f.wl;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (idx >= 2 * lplane) return;
    const int ch = static_cast<int>(idx / lplane);
    const int64_t pix = idx - ch * lplane;
    const int y = static_cast<int>(pix / f.wl), x = static_cast<int>(pix - static_cast<int64_t>(y) * f.wl);
    const int64_t plane = static_cast<int64_t>(f.h) * f.w;
    // HR rows whose taps can reach LR row y: sp = s (i + 1/2) - 1/2 in [y - 1, y + 1]
    const int ilo = max(0, static_cast<int>(floorf((static_cast<float>(y) - 0.5f) / f.scale_y - 0.5f)) - 1);
    const int ihi = min(f.h - 1, static_cast<int>(ceilf((static_cast<float>(y) + 1.5f) / f.scale_y - 0.5f)) + 1);
    const int jlo = max(0, static_cast<int>(floorf((static_cast<float>(x) - 0.5f) / f.scale_x - 0.5f)) - 1);
    const int jhi = min(f.w - 1, static_cast<int>(ceilf((static_cast<float>(x) + 1.5f) / f.scale_x - 0.5f)) + 1);
    double acc = 0.0;
    for (int i = ilo; i <= ihi; ++i) {
        int r0, r1;
        float wr0, wr1;
        lr_taps(f.scale_y, i, f.hl, r0, r1, wr0, wr1);
        const double wy = (r0 == y ? wr0 : 0.0f) + (r1 == y ? wr1 : 0.0f);
        if (wy == 0.0) continue;
        double row = 0.0;
        for (int j = jlo; j <= jhi; ++j) {
            int c0, c1;
            float wc0, wc1;
            lr_taps(f.scale_x, j, f.wl, c0, c1, wc0, wc1);
            const double wx = (c0 == x ? wc0 : 0.0f) + (c1 == x ? wc1 : 0.0f);
            if (wx != 0.0) row += wx * d_hr[ch * plane + static_cast<int64_t>(i) * f.w + j];
        }
        acc += wy * row;
    }
    d_motion[idx] = static_cast<float>(static_cast<double>(f.alpha) * acc);
}

Field make_field(const float* m, int hl, int wl, int h, int w, float alpha) {
    Field f;
    f.m = m;
    f.hl = hl;
    f.wl = wl;
    f.h = h;
    f.w = w;
    f.alpha = alpha;
    f.scale_y = static_cast<float>(hl) / static_cast<float>(h);
    f.scale_x = static_cast<float>(wl) / static_cast<float>(w);
    f.same = (hl == h && wl == w) ? 1 : 0;
    f.scale_y_d = static_cast<double>(hl) / static_cast<double>(h);
    f.scale_x_d = static_cast<double>(wl) / static_cast<double>(w);
    return f;
}

}  // namespace

int64_t warp_scratch_bytes(int64_t n) {
    return arena_bytes(n * 2, sizeof(float4)) + arena_bytes(n + 1, sizeof(int32_t)) + scan_scratch_bytes(n);
}

cudaError_t launch_warp_canvas(int n, int f, int hl, int wl, int h, int w, const float* motion, float alpha,
                               const float* recon4, const float* pos, const float* scales, const float* rots,
                               const float* ops, const float* colors, float* out_pos, float* out_scales,
                               float* out_rots, float* out_ops, float* out_colors, int32_t* out_count,
                               void* scratch, cudaStream_t stream) {
    Arena arena{static_cast<char*>(scratch), warp_scratch_bytes(n), 0};
    float4* tmp = arena.take<float4>(static_cast<int64_t>(n) * 2);
    int32_t* flags = arena.take<int32_t>(n + 1);
    void* scan_scratch = arena.base + arena.used;
    const Field fld = make_field(motion, hl, wl, h, w, alpha);
    const float4 recon = make_float4(recon4[0], recon4[1], recon4[2], recon4[3]);
    const unsigned blocks = static_cast<unsigned>(div_up(n > 0 ? n : 1, kThreads));
    if (n > 0) {
        k_warp_eval<<<blocks, kThreads, 0, stream>>>(n, fld, recon, reinterpret_cast<const float2*>(pos),
                                                     reinterpret_cast<const float2*>(scales), rots, tmp, flags);
        cudaError_t err = cudaGetLastError();
        if (err != cudaSuccess) return err;
    }
    cudaError_t err = scan_exclusive_i32(flags, flags, n, true, nullptr, scan_scratch, stream);
    if (err != cudaSuccess) return err;
    if (n > 0) {
        k_warp_scatter<false><<<blocks, kThreads, 0, stream>>>(
            n, f, tmp, flags, ops, colors, reinterpret_cast<float2*>(out_pos), reinterpret_cast<float2*>(out_scales),
            out_rots, out_ops, out_colors);
        err = cudaGetLastError();
        if (err != cudaSuccess) return err;
    }
    return cudaMemcpyAsync(out_count, flags + n, sizeof(int32_t), cudaMemcpyDeviceToDevice, stream);
}

cudaError_t launch_warp_canvas_parked(int n, int f, int hl, int wl, int h, int w, const float* motion, float alpha,
                                      const float* recon4, const float* pos, const float* scales, const float* rots,
                                      const float* ops, const float* colors, float* out_pos, float* out_scales,
                                      float* out_rots, float* out_ops, float* out_colors, void* scratch,
                                      cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    Arena arena{static_cast<char*>(scratch), warp_scratch_bytes(n), 0};
    float4* tmp = arena.take<float4>(static_cast<int64_t>(n) * 2);
    int32_t* flags = arena.take<int32_t>(n + 1);
    const Field fld = make_field(motion, hl, wl, h, w, alpha);
    const float4 recon = make_float4(recon4[0], recon4[1], recon4[2], recon4[3]);
    const unsigned blocks = static_cast<unsigned>(div_up(n, kThreads));
    k_warp_eval<<<blocks, kThreads, 0, stream>>>(n, fld, recon, reinterpret_cast<const float2*>(pos),
                                                 reinterpret_cast<const float2*>(scales), rots, tmp, flags);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    k_warp_scatter<true><<<blocks, kThreads, 0, stream>>>(
        n, f, tmp, flags, ops, colors, reinterpret_cast<float2*>(out_pos), reinterpret_cast<float2*>(out_scales),
        out_rots, out_ops, out_colors);
    return cudaGetLastError();
}

int64_t warp_backward_scratch_bytes(int64_t h, int64_t w) { return arena_bytes(6 * h * w, sizeof(double)); }

cudaError_t launch_warp_canvas_backward(int n, int f, int hl, int wl, int h, int w, const float* motion, float alpha,
                                        const float* recon4, const float* pos, const float* scales, const float* rots,
                                        const void* fwd_scratch, const float* g_pos, const float* g_scales,
                                        const float* g_rots, const float* g_ops, const float* g_colors, float* d_pos,
                                        float* d_scales, float* d_rots, float* d_ops, float* d_colors,
                                        float* d_motion, void* scratch, cudaStream_t stream) {
    // the forward's survivor offsets sit after its per-Gaussian records (launch_warp_canvas)
    Arena fwd{static_cast<char*>(const_cast<void*>(fwd_scratch)), warp_scratch_bytes(n), 0};
    fwd.take<float4>(static_cast<int64_t>(n) * 2);
    const int32_t* offs = fwd.take<int32_t>(n + 1);
    const Field fld = make_field(motion, hl, wl, h, w, alpha);
    const float4 recon = make_float4(recon4[0], recon4[1], recon4[2], recon4[3]);
    const int64_t plane = static_cast<int64_t>(h) * w;
    double* d_hr = static_cast<double*>(scratch);  // six HR gradient planes, accumulated in double
    cudaError_t err = cudaMemsetAsync(d_hr, 0, sizeof(double) * 6 * plane, stream);
    if (err != cudaSuccess) return err;
    if (n > 0) {
        k_warp_backward<<<static_cast<unsigned>(div_up(n, kThreads)), kThreads, 0, stream>>>(
            n, f, fld, recon, reinterpret_cast<const float2*>(pos), reinterpret_cast<const float2*>(scales), rots, offs,
            reinterpret_cast<const float2*>(g_pos), reinterpret_cast<const float2*>(g_scales), g_rots, g_ops, g_colors,
            reinterpret_cast<float2*>(d_pos), reinterpret_cast<float2*>(d_scales), d_rots, d_ops, d_colors, d_hr);
        err = cudaGetLastError();
        if (err != cudaSuccess) return err;
    }
    if (d_motion == nullptr) return cudaSuccess;
    k_warp_motion_grad<<<static_cast<unsigned>(div_up(2 * plane, kThreads)), kThreads, 0, stream>>>(h, w, d_hr);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    const int64_t lplane = static_cast<int64_t>(hl) * wl;
    k_warp_lr_grad<<<static_cast<unsigned>(div_up(2 * lplane, kThreads)), kThreads, 0, stream>>>(fld, d_hr, d_motion);
    return cudaGetLastError();
}

cudaError_t launch_warp_positions(int n, int h, int w, const float* motion, float alpha, const float* xy,
                                  float* out_xy, uint8_t* in_frame, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    const Field fld = make_field(motion, h, w, h, w, alpha);
    k_warp_positions<<<static_cast<unsigned>(div_up(n, kThreads)), kThreads, 0, stream>>>(
        n, fld, reinterpret_cast<const float2*>(xy), reinterpret_cast<float2*>(out_xy), in_frame);
    return cudaGetLastError();
}

}  // namespace oss
