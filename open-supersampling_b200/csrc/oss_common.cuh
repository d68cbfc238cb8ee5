// Shared device helpers for the sm_100a rasterizer kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/oss_raster.h"

namespace oss {

constexpr int kTile = OSS_TILE;          // tile edge in pixels
constexpr int kTilePixels = kTile * kTile;
constexpr float kMinScale = 1.0e-6f;     // rasterizer_fwd.cu common.cuh:15
constexpr float kTauTight = 9.0f;        // rasterizer_fwd.cu:92
// Exact-mode cutoff.  For q > 2*126*ln2 = 174.67, 2^(-q/2 log2 e) is below
// 2^-126, the smallest normal fp32: the kernels' ex2.approx.ftz returns exactly
// 0 there (as does any flush-to-zero evaluation, such as the reference CUDA
// op's -ftz=true build), and an evaluation with subnormals gets at most
// 1.2e-38 per Gaussian.  176 keeps a 0.8% margin over fp32 rounding of q and of
// the AABB radius.
constexpr float kTauExact = 176.0f;
// Cutoff of the exact56 lists: every weight left out is below e^-28 = 6.9e-13.
constexpr float kTauExact56 = 56.0f;
// -0.5*log2(e): folds exp(-q/2) = 2^(q * -0.5 log2 e) into the conic.
constexpr float kNegHalfLog2e = -0.72134752044448170368f;

__host__ __device__ inline int64_t div_up(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Asynchronous global -> shared copies (cp.async): they hold no registers while
// in flight.  cp_async4_zfill copies 4 bytes, or writes 0 when !valid (the
// source is then not read).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async4_zfill(void* smem_dst, const void* gmem_src, bool valid) {
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    const int bytes = valid ? 4 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(dst), "l"(gmem_src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_one() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// Saturating float -> int conversion with NaN -> 0 (the semantics of
// cvt.rzi.s32.f32, which the reference's static_cast<int> compiles to).
__device__ __forceinline__ int sat_f2i(float v) {
    if (!(v == v)) return 0;
    if (v >= 2147483648.0f) return 2147483647;
    if (v <= -2147483648.0f) return (-2147483647 - 1);
    return static_cast<int>(v);
}

__device__ __forceinline__ int clamp_i(int v, int lo, int hi) {
    return v < lo ? lo : (v > hi ? hi : v);
}

// 2^x with flush-to-zero; one MUFU op (PTX ex2.approx.ftz.f32).
__device__ __forceinline__ float ex2_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Scaled quadratic form q' = -0.5*log2(e) * (a dx^2 + 2b dx dy + d dy^2) from a
// geo record (A, B, D).  Forward and backward use this one expression so their
// weights are bit-identical.
__device__ __forceinline__ float q_scaled(float A, float B, float D, float dx, float dy) {
    return fmaf(dx, fmaf(A, dx, B * dy), (D * dy) * dy);
}

// Sums of K values across the warp with K - 1 + log2(32 / K) shuffles instead of
// 5 K (K a power of two <= 32): at each of the first log2(K) xor levels a lane
// keeps half of its values and adds its partner's copy of that half, so after
// them lane l holds value (l >> (5 - log2 K)) summed over the K lanes those
// levels joined; the remaining butterfly levels finish the sum.  Returns that
// lane's total; the summation order is fixed, so results are reproducible.
template <int K>
__device__ __forceinline__ float warp_reduce_scatter(float (&x)[K]) {
    static_assert(K >= 1 && K <= 32 && (K & (K - 1)) == 0, "K must be a power of two <= 32");
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int k = K, off = 16; k > 1; k >>= 1, off >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < k / 2; ++i) {
            const float send = upper ? x[i] : x[i + k / 2];
            const float keep = upper ? x[i + k / 2] : x[i];
            x[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
    float v = x[0];
#pragma unroll
    for (int off = 16 / K; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// Inverse covariance (conic) from per-axis scale and rotation, in the
// operation order of rasterizer_fwd.cu:52-65.  Every multiply/add is rounded
// on its own (no FMA contraction) and cos/sin are evaluated in double and
// rounded once, so the CPU oracle (oracle/oss_oracle.c) reproduces these bits.
struct Conic {
    float a, b, d;
};

__device__ __forceinline__ float clamp_min_keep_nan(float v, float lo) { return v < lo ? lo : v; }

__device__ __forceinline__ void cos_sin_rn(float angle, float& c, float& s) {
    double sd, cd;
    sincos(static_cast<double>(angle), &sd, &cd);
    c = __double2float_rn(cd);
    s = __double2float_rn(sd);
}

__device__ __forceinline__ Conic conic_from_scale_rot(float raw_sx, float raw_sy, float angle) {
    const float sx = clamp_min_keep_nan(raw_sx, kMinScale);
    const float sy = clamp_min_keep_nan(raw_sy, kMinScale);
    float c, s;
    cos_sin_rn(angle, c, s);
    const float inv_sx2 = __fdiv_rn(1.0f, __fmul_rn(sx, sx));
    const float inv_sy2 = __fdiv_rn(1.0f, __fmul_rn(sy, sy));
    const float cc = __fmul_rn(c, c);
    const float ss = __fmul_rn(s, s);
    const float cs = __fmul_rn(c, s);
    Conic k;
    k.a = __fadd_rn(__fmul_rn(cc, inv_sx2), __fmul_rn(ss, inv_sy2));
    k.b = __fmul_rn(cs, __fsub_rn(inv_sx2, inv_sy2));
    k.d = __fadd_rn(__fmul_rn(ss, inv_sx2), __fmul_rn(cc, inv_sy2));
    return k;
}

// Tile AABB of the q = tau ellipse (rasterizer_fwd.cu:68-108).  Returns the
// half-open rectangle (tx0, ty0, tx1, ty1) and its tile count.
__device__ __forceinline__ int4 tile_aabb(float cx, float cy, float raw_sx, float raw_sy,
                                          const Conic& k, float tau, float fallback_k,
                                          int ntx, int nty, int& count) {
    if (!isfinite(k.a) || !isfinite(k.b) || !isfinite(k.d)) {
        count = 0;
        return make_int4(0, 0, 0, 0);
    }
    float rx, ry;
    const float det = __fsub_rn(__fmul_rn(k.a, k.d), __fmul_rn(k.b, k.b));
    if (det > 1e-12f) {
        rx = __fsqrt_rn(__fdiv_rn(__fmul_rn(tau, k.d), det));
        ry = __fsqrt_rn(__fdiv_rn(__fmul_rn(tau, k.a), det));
    } else {
        const float r = __fmul_rn(fallback_k, fmaxf(raw_sx, raw_sy));
        rx = r;
        ry = r;
    }
    const float ts = static_cast<float>(kTile);
    const int tx0 = clamp_i(sat_f2i(floorf(__fdiv_rn(__fsub_rn(cx, rx), ts))), 0, ntx);
    const int tx1 = clamp_i(sat_f2i(ceilf(__fdiv_rn(__fadd_rn(cx, rx), ts))), 0, ntx);
    const int ty0 = clamp_i(sat_f2i(floorf(__fdiv_rn(__fsub_rn(cy, ry), ts))), 0, nty);
    const int ty1 = clamp_i(sat_f2i(ceilf(__fdiv_rn(__fadd_rn(cy, ry), ts))), 0, nty);
    const int cnx = tx1 > tx0 ? tx1 - tx0 : 0;
    const int cny = ty1 > ty0 ? ty1 - ty0 : 0;
    count = cnx * cny;
    return make_int4(tx0, ty0, tx1, ty1);
}

// Chain rule d_conic -> (d_scale, d_rot) of rasterizer_bwd.cu:128-153, with the
// same double-evaluated cos/sin as conic_from_scale_rot.
__device__ __forceinline__ void conic_grad_to_scale_rot(float raw_sx, float raw_sy, float theta,
                                                        float dca, float dcb, float dcd,
                                                        float& d_sx, float& d_sy, float& d_rot) {
    const float sx = fmaxf(raw_sx, kMinScale);
    const float sy = fmaxf(raw_sy, kMinScale);
    const float inv_sx2 = __fdiv_rn(1.0f, __fmul_rn(sx, sx));
    const float inv_sy2 = __fdiv_rn(1.0f, __fmul_rn(sy, sy));
    const float diff = __fsub_rn(inv_sx2, inv_sy2);
    float c, s;
    cos_sin_rn(theta, c, s);
    const float cc = __fmul_rn(c, c);
    const float ss = __fmul_rn(s, s);
    const float cs = __fmul_rn(c, s);
    const float d_inv_sx2 = __fadd_rn(__fadd_rn(__fmul_rn(cc, dca), __fmul_rn(cs, dcb)), __fmul_rn(ss, dcd));
    const float d_inv_sy2 = __fadd_rn(__fsub_rn(__fmul_rn(ss, dca), __fmul_rn(cs, dcb)), __fmul_rn(cc, dcd));
    d_sx = raw_sx > kMinScale
               ? __fmul_rn(d_inv_sx2, __fdiv_rn(-2.0f, __fmul_rn(__fmul_rn(raw_sx, raw_sx), raw_sx)))
               : 0.0f;
    d_sy = raw_sy > kMinScale
               ? __fmul_rn(d_inv_sy2, __fdiv_rn(-2.0f, __fmul_rn(__fmul_rn(raw_sy, raw_sy), raw_sy)))
               : 0.0f;
    const float t0 = __fmul_rn(dca, __fmul_rn(__fmul_rn(-2.0f, cs), diff));
    const float t1 = __fmul_rn(dcb, __fmul_rn(diff, __fsub_rn(cc, ss)));
    const float t2 = __fmul_rn(dcd, __fmul_rn(__fmul_rn(2.0f, cs), diff));
    d_rot = __fadd_rn(__fadd_rn(t0, t1), t2);
}

// The same chain rule in double, for gradients summed in double: a thin
// Gaussian's d_scale and d_rot are small differences of d_conic terms, which
// the fp32 form rounds before they cancel.
__device__ __forceinline__ void conic_grad_to_scale_rot_f64(float raw_sx, float raw_sy, float theta, double dca,
                                                            double dcb, double dcd, float& d_sx, float& d_sy,
                                                            float& d_rot) {
    const double sx = fmax(static_cast<double>(raw_sx), static_cast<double>(kMinScale));
    const double sy = fmax(static_cast<double>(raw_sy), static_cast<double>(kMinScale));
    const double inv_sx2 = 1.0 / (sx * sx);
    const double inv_sy2 = 1.0 / (sy * sy);
    const double diff = inv_sx2 - inv_sy2;
    double s, c;
    sincos(static_cast<double>(theta), &s, &c);
    const double cc = c * c, ss = s * s, cs = c * s;
    const double d_inv_sx2 = cc * dca + cs * dcb + ss * dcd;
    const double d_inv_sy2 = ss * dca - cs * dcb + cc * dcd;
    const double rx = raw_sx, ry = raw_sy;
    d_sx = raw_sx > kMinScale ? static_cast<float>(d_inv_sx2 * (-2.0 / (rx * rx * rx))) : 0.0f;
    d_sy = raw_sy > kMinScale ? static_cast<float>(d_inv_sy2 * (-2.0 / (ry * ry * ry))) : 0.0f;
    d_rot = static_cast<float>(dca * (-2.0 * cs * diff) + dcb * diff * (cc - ss) + dcd * (2.0 * cs * diff));
}

// Per-mode AABB parameters.
__host__ __device__ inline float mode_tau(int mode) {
    return mode == OSS_BIN_EXACT ? kTauExact : (mode == OSS_BIN_EXACT56 ? kTauExact56 : kTauTight);
}
// Fallback radius factor for degenerate conics: 3*max(s) for the 3-sigma lists
// (rasterizer_fwd.cu:96), sqrt(tau)*max(s) for the exact lists.
__host__ __device__ inline float mode_fallback(int mode) {
    return mode == OSS_BIN_EXACT ? 13.266499161421599f : (mode == OSS_BIN_EXACT56 ? 7.483314773547883f : 3.0f);
}

}  // namespace oss
