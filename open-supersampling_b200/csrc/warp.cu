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
    const int k = offs[g];
    if (offs[g + 1] == k) return;  // dropped: new centre outside the frame
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
        k_warp_scatter<<<blocks, kThreads, 0, stream>>>(n, f, tmp, flags, ops, colors, reinterpret_cast<float2*>(out_pos),
                                                        reinterpret_cast<float2*>(out_scales), out_rots, out_ops,
                                                        out_colors);
        err = cudaGetLastError();
        if (err != cudaSuccess) return err;
    }
    return cudaMemcpyAsync(out_count, flags + n, sizeof(int32_t), cudaMemcpyDeviceToDevice, stream);
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
