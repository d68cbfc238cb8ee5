// V6 front end on the device: the sanitisation of V6Rasterizer.forward
// (oss/sr/v6/rasterizer.py:56-157 with _sanitize_active_gaussians :244-291 and
// _token_features :319-327) without its boolean gathers and host reads.
//
// The reference gathers the live, active Gaussians, drops the non-finite ones
// and those whose 3 * max|scale| disc misses the frame, then clamps |scale| to
// [1e-3, max(h, w)], clamps positions into the frame and wraps rotations.
// Compacting needs the survivor count on the host; here every live Gaussian
// keeps its slot: a kept one is written sanitised, a dropped one is parked far
// outside the frame with zero features, so binning gives it no tile and it
// adds nothing to the image or to any gradient.  One thread per Gaussian; the
// features are padded or truncated to the render width, plus an optional
// ones channel (the weight sum).  Per Gaussian a flag word records what the
// backward needs: kept or not, and each clamp's and |.|'s derivative, with
// PyTorch's conventions at ties (clamp passes its bounds, minimum gives half).
#include <math.h>

#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

constexpr int kThreads = 256;
constexpr float kMinPixelScale = 1.0e-3f;
constexpr float kParked = -1.0e7f;  // a centre whose tile box is empty

// flag word: bit 0 kept; two-bit derivative codes (0: 0, 1: +1, 2: -1, 3: +1/2)
// for position x (bits 1-2), position y (3-4), scale x (5-6), scale y (7-8)
__device__ __forceinline__ float code_value(uint32_t code) {
    return code == 1u ? 1.0f : (code == 2u ? -1.0f : (code == 3u ? 0.5f : 0.0f));
}

// |s| clamped to [lo, hi]: d/ds = sign(s) inside the range, bounds included
__device__ __forceinline__ uint32_t scale_code(float s, float lo, float hi) {
    const float a = fabsf(s);
    if (!(a >= lo && a <= hi) || s == 0.0f) return 0u;
    return s > 0.0f ? 1u : 2u;
}

// minimum(max(p, 0), hi): d/dp = [p >= 0] * (1, or 1/2 where max(p, 0) == hi)
__device__ __forceinline__ uint32_t pos_code(float p, float hi) {
    if (!(p >= 0.0f)) return 0u;
    if (p < hi) return 1u;
    return p == hi ? 3u : 0u;
}

__global__ void __launch_bounds__(kThreads) k_v6_sanitize(int n, int h, int w, int f_in, int f_out, int ones,
                                                          const uint8_t* __restrict__ mask,
                                                          const float2* __restrict__ pos,
                                                          const float2* __restrict__ scl,
                                                          const float* __restrict__ rot,
                                                          const float* __restrict__ colors,
                                                          float2* __restrict__ out_xy, float2* __restrict__ out_scale,
                                                          float* __restrict__ out_rot, float* __restrict__ out_feat,
                                                          uint16_t* __restrict__ flags) {
    const int g = blockIdx.x * kThreads + threadIdx.x;
    if (g >= n) return;
    const float2 p = pos[g];
    const float2 s = scl[g];
    const float r = rot[g];
    const float* col = colors + static_cast<int64_t>(g) * f_in;
    const int fc = f_in < f_out ? f_in : f_out;  // channels kept; the rest pad with zeros
    bool finite = isfinite(p.x) && isfinite(p.y) && isfinite(s.x) && isfinite(s.y) && isfinite(r);
    for (int c = 0; c < fc; ++c) finite = finite && isfinite(col[c]);
    const float hi_s = static_cast<float>(h > w ? h : w);
    const float sx = fminf(fmaxf(fabsf(s.x), kMinPixelScale), hi_s);
    const float sy = fminf(fmaxf(fabsf(s.y), kMinPixelScale), hi_s);
    const float rad = 3.0f * fmaxf(sx, sy);
    const bool overlaps = (p.x + rad >= 0.0f) && (p.x - rad < static_cast<float>(w)) && (p.y + rad >= 0.0f) &&
                          (p.y - rad < static_cast<float>(h));
    const bool keep = (mask == nullptr || mask[g] != 0) && finite && overlaps;
    const int fo = f_out + ones;
    float* feat = out_feat + static_cast<int64_t>(g) * fo;
    if (!keep) {
        out_xy[g] = make_float2(kParked, kParked);
        out_scale[g] = make_float2(1.0f, 1.0f);
        out_rot[g] = 0.0f;
        for (int c = 0; c < fo; ++c) feat[c] = 0.0f;
        flags[g] = 0;
        return;
    }
    const float hx = fmaxf(static_cast<float>(w) - 1.0e-4f, 0.0f);
    const float hy = fmaxf(static_cast<float>(h) - 1.0e-4f, 0.0f);
    out_xy[g] = make_float2(fminf(fmaxf(p.x, 0.0f), hx), fminf(fmaxf(p.y, 0.0f), hy));
    out_scale[g] = make_float2(sx, sy);
    out_rot[g] = atan2f(sinf(r), cosf(r));
    for (int c = 0; c < fo; ++c) feat[c] = c < fc ? col[c] : (c == f_out ? 1.0f : 0.0f);
    flags[g] = static_cast<uint16_t>(1u | (pos_code(p.x, hx) << 1) | (pos_code(p.y, hy) << 3) |
                                     (scale_code(s.x, kMinPixelScale, hi_s) << 5) |
                                     (scale_code(s.y, kMinPixelScale, hi_s) << 7));
}

__global__ void __launch_bounds__(kThreads) k_v6_sanitize_backward(int n, int f_in, int f_out, int ones,
                                                                   const uint16_t* __restrict__ flags,
                                                                   const float2* __restrict__ d_xy,
                                                                   const float2* __restrict__ d_scale,
                                                                   const float* __restrict__ d_rot,
                                                                   const float* __restrict__ d_feat,
                                                                   float2* __restrict__ d_pos,
                                                                   float2* __restrict__ d_scl,
                                                                   float* __restrict__ d_rot_in,
                                                                   float* __restrict__ d_colors) {
    const int g = blockIdx.x * kThreads + threadIdx.x;
    if (g >= n) return;
    const uint32_t fl = flags[g];
    const bool keep = (fl & 1u) != 0;
    const float2 dx = d_xy != nullptr ? d_xy[g] : make_float2(0.0f, 0.0f);
    const float2 ds = d_scale != nullptr ? d_scale[g] : make_float2(0.0f, 0.0f);
    d_pos[g] = make_float2(dx.x * code_value((fl >> 1) & 3u), dx.y * code_value((fl >> 3) & 3u));
    d_scl[g] = make_float2(ds.x * code_value((fl >> 5) & 3u), ds.y * code_value((fl >> 7) & 3u));
    d_rot_in[g] = keep && d_rot != nullptr ? d_rot[g] : 0.0f;  // d/dr atan2(sin r, cos r) = 1
    const int fo = f_out + ones;
    const int fc = f_in < f_out ? f_in : f_out;
    float* dc = d_colors + static_cast<int64_t>(g) * f_in;
    for (int c = 0; c < f_in; ++c) {
        dc[c] = keep && c < fc && d_feat != nullptr ? d_feat[static_cast<int64_t>(g) * fo + c] : 0.0f;
    }
}

}  // namespace

cudaError_t launch_v6_sanitize(int n, int h, int w, int f_in, int f_out, int ones, const uint8_t* mask,
                               const float* pos, const float* scl, const float* rot, const float* colors,
                               float* out_xy, float* out_scale, float* out_rot, float* out_feat, uint16_t* flags,
                               cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    k_v6_sanitize<<<static_cast<unsigned>(div_up(n, kThreads)), kThreads, 0, stream>>>(
        n, h, w, f_in, f_out, ones, mask, reinterpret_cast<const float2*>(pos), reinterpret_cast<const float2*>(scl),
        rot, colors, reinterpret_cast<float2*>(out_xy), reinterpret_cast<float2*>(out_scale), out_rot, out_feat, flags);
    return cudaGetLastError();
}

cudaError_t launch_v6_sanitize_backward(int n, int f_in, int f_out, int ones, const uint16_t* flags,
                                        const float* d_xy, const float* d_scale, const float* d_rot,
                                        const float* d_feat, float* d_pos, float* d_scl, float* d_rot_in,
                                        float* d_colors, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    k_v6_sanitize_backward<<<static_cast<unsigned>(div_up(n, kThreads)), kThreads, 0, stream>>>(
        n, f_in, f_out, ones, flags, reinterpret_cast<const float2*>(d_xy), reinterpret_cast<const float2*>(d_scale),
        d_rot, d_feat, reinterpret_cast<float2*>(d_pos), reinterpret_cast<float2*>(d_scl), d_rot_in, d_colors);
    return cudaGetLastError();
}

}  // namespace oss
