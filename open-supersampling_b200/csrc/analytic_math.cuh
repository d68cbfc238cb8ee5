// Device math of the Analytic-Splatting pixel integral (oss/sr/v6/aa_analytic_splat.py:46-202),
// shared by the elementwise kernels (analytic.cu) and the analytic-weight render
// (raster_analytic.cu): the conditioned logistic CDF and its slope, the per-axis
// integral with its derivatives, the eigen-frame of an inverse covariance, and the
// chain rule from the frame's (sigma_h, sigma_l, theta) back to the covariance entries.
#pragma once

namespace oss {
namespace analytic {

constexpr float kTwoPi = 6.283185307179586f;

__device__ __forceinline__ float logistic(float x) {
    const float z = fmaf(0.07f * x, x * x, 1.6f * x);
    return __frcp_rn(1.0f + expf(-z));  // the correctly rounded 1 / (1 + e^-z)
}

// The render kernels' logistic: e^-z from the hardware base-2 exponential
// (__expf) and 1 / (1 + e) from the approximate reciprocal (__fdividef), a
// fraction of the instructions of the form above.  The absolute error of S stays
// near one ulp of S: __expf's relative error grows with |z| (the rounding of
// z log2 e, about |z| 2^-24), but it reaches S through dS/d(ln e) = -S (1 - S),
// and S (1 - S) |z| 2^-24 stays below 2e-8 for every z; the reciprocal adds at
// most about one ulp.  The elementwise kernels keep the accurate form.
__device__ __forceinline__ float logistic_fast(float x) {
    const float z = fmaf(0.07f * x, x * x, 1.6f * x);
    return __fdividef(1.0f, 1.0f + __expf(-z));
}

template <bool FAST>
__device__ __forceinline__ float logistic_t(float x) {
    return FAST ? logistic_fast(x) : logistic(x);
}

// dS/dx = S (1 - S) (1.6 + 0.21 x^2)
__device__ __forceinline__ float logistic_slope(float x) {
    const float s = logistic(x);
    return s * (1.0f - s) * fmaf(0.21f * x, x, 1.6f);
}

struct AxisTerm {
    float v;        // I(u)
    float du;       // dI / du
    float dsigma;   // dI / dsigma
};

// I(u) and its derivatives from 1 / sigma (FAST: with logistic_fast).
template <bool FAST = false>
__device__ __forceinline__ AxisTerm axis_term_inv(float u, float inv, bool grads) {
    const float xp = (u + 0.5f) * inv, xm = (u - 0.5f) * inv;
    AxisTerm t;
    const float lp = logistic_t<FAST>(xp), lm = logistic_t<FAST>(xm);
    t.v = lp - lm;
    t.du = t.dsigma = 0.0f;
    if (grads) {  // slopes from the values above: S' = S (1 - S) (1.6 + 0.21 x^2)
        const float sp = lp * (1.0f - lp) * fmaf(0.21f * xp, xp, 1.6f);
        const float sm = lm * (1.0f - lm) * fmaf(0.21f * xm, xm, 1.6f);
        t.du = (sp - sm) * inv;
        t.dsigma = -(sp * xp - sm * xm) * inv;
    }
    return t;
}

__device__ __forceinline__ AxisTerm axis_term(float u, float sigma, bool grads) {
    return axis_term_inv(u, 1.0f / sigma, grads);
}

struct Frame {
    float a, b, c, half, t, raw, d, lh, ll, sh, sl;
    bool iso;
    float s;         // isotropic sigma
    float ct, st;    // eigenvector angle
};

__device__ __forceinline__ Frame frame_of(float s00, float s01, float s10, float s11) {
    Frame f;
    f.a = s00 + 1.0e-6f;
    f.b = 0.5f * (s01 + s10);
    f.c = s11 + 1.0e-6f;
    f.half = 0.5f * (f.a - f.c);
    f.t = 0.5f * (f.a + f.c);
    f.raw = f.half * f.half + f.b * f.b;
    f.d = sqrtf(f.raw + 1.0e-6f);
    f.lh = f.t + f.d;
    f.ll = f.t - f.d;
    f.sh = rsqrtf(fmaxf(f.lh, 1.0e-12f));
    f.sl = rsqrtf(fmaxf(f.ll, 1.0e-12f));
    f.iso = 2.0f * sqrtf(f.raw) < 1.0e-5f;
    f.s = rsqrtf(fmaxf(f.t, 1.0e-12f));
    float th = 0.0f;
    if (!f.iso) th = 0.5f * atan2f(2.0f * f.b, f.a - f.c);
    sincosf(th, &f.st, &f.ct);
    return f;
}

// d/d(a, b, c) of the frame from the sums of dL/d(sigma_h, sigma_l, theta) (or, for an
// isotropic frame, dL/dsigma as g_sh + g_sl): the clamps pass gradient at or above the floor.
__device__ __forceinline__ void frame_grad(const Frame& f, float g_sh, float g_sl, float g_theta, float& ga,
                                           float& gb, float& gc) {
    if (f.iso) {
        const float g_s = g_sh + g_sl;
        const float g_t = f.t >= 1.0e-12f ? g_s * (-0.5f * f.s * f.s * f.s) : 0.0f;
        ga = 0.5f * g_t;
        gb = 0.0f;
        gc = 0.5f * g_t;
        return;
    }
    const float g_lh = f.lh >= 1.0e-12f ? g_sh * (-0.5f * f.sh * f.sh * f.sh) : 0.0f;
    const float g_ll = f.ll >= 1.0e-12f ? g_sl * (-0.5f * f.sl * f.sl * f.sl) : 0.0f;
    const float g_t = g_lh + g_ll;
    const float g_raw = (g_lh - g_ll) / (2.0f * f.d);
    const float g_half = g_raw * 2.0f * f.half;
    const float X = f.a - f.c, Y = 2.0f * f.b, r2 = X * X + Y * Y;
    const float g_X = g_theta * (-0.5f * Y / r2), g_Y = g_theta * (0.5f * X / r2);
    gb = g_raw * 2.0f * f.b + 2.0f * g_Y;
    ga = 0.5f * g_t + 0.5f * g_half + g_X;
    gc = 0.5f * g_t - 0.5f * g_half - g_X;
}

}  // namespace analytic
}  // namespace oss
