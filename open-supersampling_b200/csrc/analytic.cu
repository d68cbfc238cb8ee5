// Analytic-Splatting pixel integral (oss/sr/v6/aa_analytic_splat.py:46-202;
// Liang et al., ECCV 2024, Definition 1 and Eq. 15): the integral of an
// un-normalised 2D Gaussian over the unit pixel square around an offset
// (dx, dy), with the 1D normal CDF replaced by the conditioned logistic
// S(x) = 1 / (1 + exp(-1.6 x - 0.07 x^3)).  From the inverse covariance
// [[s00, s01], [s10, s11]]: a = s00 + 1e-6, b = (s01 + s10) / 2, c = s11 + 1e-6,
// eigenvalues t +- d (t = (a + c) / 2, d = sqrt(((a - c) / 2)^2 + b^2 + 1e-6),
// floored at 1e-12), sigma = 1 / sqrt(eigenvalue), the eigenvector angle
// theta = atan2(2b, a - c) / 2 and
//   w = 2 pi sigma_h sigma_l I_h(u_h) I_l(u_l),  I(u) = S((u + 1/2) / sigma) - S((u - 1/2) / sigma),
// with (u_h, u_l) the offset rotated by theta.  Below an eigengap of 1e-5 the
// axes are undefined and the integral is the separable one with a shared
// sigma = 1 / sqrt(max(t, 1e-12)) in screen x and y.
//
// The backward is the chain rule of these steps, branch by branch, with the
// clamps passing gradient where their input is at or above the floor.
#include "analytic_math.cuh"
#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

using namespace analytic;

__global__ void k_analytic_fwd(int64_t n, const float* __restrict__ dx, const float* __restrict__ dy,
                               const float* __restrict__ s00, const float* __restrict__ s01,
                               const float* __restrict__ s10, const float* __restrict__ s11, float* __restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const Frame f = frame_of(s00[i], s01[i], s10[i], s11[i]);
    const float x = dx[i], y = dy[i];
    if (f.iso) {
        const AxisTerm ix = axis_term(x, f.s, false), iy = axis_term(y, f.s, false);
        out[i] = kTwoPi * f.s * f.s * ix.v * iy.v;
    } else {
        const float uh = f.ct * x + f.st * y, ul = -f.st * x + f.ct * y;
        const AxisTerm ih = axis_term(uh, f.sh, false), il = axis_term(ul, f.sl, false);
        out[i] = kTwoPi * f.sh * f.sl * ih.v * il.v;
    }
}

__global__ void k_analytic_bwd(int64_t n, const float* __restrict__ dx, const float* __restrict__ dy,
                               const float* __restrict__ s00, const float* __restrict__ s01,
                               const float* __restrict__ s10, const float* __restrict__ s11,
                               const float* __restrict__ g, float* __restrict__ g_dx, float* __restrict__ g_dy,
                               float* __restrict__ g_s00, float* __restrict__ g_s01, float* __restrict__ g_s10,
                               float* __restrict__ g_s11) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const Frame f = frame_of(s00[i], s01[i], s10[i], s11[i]);
    const float x = dx[i], y = dy[i], gw = g[i];
    float ga = 0.0f, gb = 0.0f, gc = 0.0f, gx, gy;
    if (f.iso) {
        const AxisTerm ix = axis_term(x, f.s, true), iy = axis_term(y, f.s, true);
        const float K = kTwoPi * f.s * f.s;
        gx = gw * K * ix.du * iy.v;
        gy = gw * K * ix.v * iy.du;
        const float w = K * ix.v * iy.v;
        const float g_s = gw * (2.0f * w / f.s + K * (ix.dsigma * iy.v + ix.v * iy.dsigma));
        frame_grad(f, g_s, 0.0f, 0.0f, ga, gb, gc);
    } else {
        const float uh = f.ct * x + f.st * y, ul = -f.st * x + f.ct * y;
        const AxisTerm ih = axis_term(uh, f.sh, true), il = axis_term(ul, f.sl, true);
        const float K = kTwoPi * f.sh * f.sl;
        gx = gw * K * (ih.du * f.ct * il.v - ih.v * il.du * f.st);
        gy = gw * K * (ih.du * f.st * il.v + ih.v * il.du * f.ct);
        const float w = K * ih.v * il.v;
        const float g_theta = gw * K * (ih.du * ul * il.v - ih.v * il.du * uh);
        const float g_sh = gw * (w / f.sh + K * il.v * ih.dsigma);
        const float g_sl = gw * (w / f.sl + K * ih.v * il.dsigma);
        frame_grad(f, g_sh, g_sl, g_theta, ga, gb, gc);
    }
    g_dx[i] = gx;
    g_dy[i] = gy;
    g_s00[i] = ga;
    g_s01[i] = 0.5f * gb;
    g_s10[i] = 0.5f * gb;
    g_s11[i] = gc;
}

__global__ void k_logistic(int64_t n, const float* __restrict__ x, const float* __restrict__ g,
                           float* __restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    out[i] = g == nullptr ? logistic(x[i]) : g[i] * logistic_slope(x[i]);
}

unsigned grid_of(int64_t n) { return static_cast<unsigned>((n + 255) / 256); }

}  // namespace

cudaError_t launch_analytic_forward(int64_t n, const float* dx, const float* dy, const float* s00, const float* s01,
                                    const float* s10, const float* s11, float* out, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    k_analytic_fwd<<<grid_of(n), 256, 0, stream>>>(n, dx, dy, s00, s01, s10, s11, out);
    return cudaGetLastError();
}

cudaError_t launch_analytic_backward(int64_t n, const float* dx, const float* dy, const float* s00, const float* s01,
                                     const float* s10, const float* s11, const float* g, float* g_dx, float* g_dy,
                                     float* g_s00, float* g_s01, float* g_s10, float* g_s11, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    k_analytic_bwd<<<grid_of(n), 256, 0, stream>>>(n, dx, dy, s00, s01, s10, s11, g, g_dx, g_dy, g_s00, g_s01, g_s10,
                                                    g_s11);
    return cudaGetLastError();
}

cudaError_t launch_logistic_cdf(int64_t n, const float* x, const float* g, float* out, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    k_logistic<<<grid_of(n), 256, 0, stream>>>(n, x, g, out);
    return cudaGetLastError();
}

}  // namespace oss
