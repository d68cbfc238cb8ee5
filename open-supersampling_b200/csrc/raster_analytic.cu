// The additive tile render with the Analytic-Splatting pixel integral as the
// weight (oss/sr/v6/aa_analytic_splat.py:72-202 in place of exp(-q/2) of
// rasterizer_fwd.cu:151-322): out[c](p) = sum over the tile list of
// feat'[g][c] * w_g(p - xy_g), with w the integral of the un-normalised Gaussian
// of inverse covariance (a, b, d) over the unit pixel square at integer pixel
// centres.  The logistic tails vanish in fp32 before q = 176 (S'(x) ~ exp(-1.6 x
// - 0.07 x^3)), so the exact-mode lists hold every non-zero term.
//
// Per list entry the eigen-frame (rotation, per-axis 1 / sigma, 2 pi sigma_h
// sigma_l; the shared sigma and no rotation below the 1e-5 eigengap) is computed
// once, at staging in the forward and per entry in the backward.  An entry whose
// every pixel of the tile lies 9 sigma or more from its centre along one axis
// adds less than 1e-27 per pixel and is skipped (a zero row in the backward):
// the outer ring of the exact lists, about half of their entries.  The backward
// runs one thread per list entry over the tile's pixels with the tile's
// dL/dimage in shared memory, sums dL/d(dx, dy, sigma_h, sigma_l, theta) and dF,
// and turns them into d_xy and d_conic in the epilogue; the rows feed the
// per-Gaussian reduce of the additive path with rows_dxy set.
#include "analytic_math.cuh"
#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

using namespace analytic;

constexpr int kAnThreads = 256;  // one pixel per thread, one CTA per tile
constexpr int kAnBatch = 64;

template <int FC>
__global__ void __launch_bounds__(kAnThreads) k_render_analytic_fwd(int F, int H, int W, int ntx,
                                                                     const float* __restrict__ geo,
                                                                     const float* __restrict__ feat,
                                                                     const float* __restrict__ opacity,
                                                                     const int32_t* __restrict__ gid_sorted,
                                                                     const int32_t* __restrict__ tile_offsets,
                                                                     float* __restrict__ image) {
    __shared__ float4 s_a[kAnBatch];  // x, y, cos, sin
    __shared__ float4 s_b[kAnBatch];  // 1 / sigma_h, 1 / sigma_l, 2 pi sigma_h sigma_l, far flag
    __shared__ float s_f[kAnBatch][FC];
    const int tile = blockIdx.x;
    const int tx0 = (tile % ntx) * kTile, ty0 = (tile / ntx) * kTile;
    const int px = tx0 + (threadIdx.x & (kTile - 1)), py = ty0 + (threadIdx.x >> 4);
    const float fpx = static_cast<float>(px), fpy = static_cast<float>(py);
    float acc[FC];
#pragma unroll
    for (int c = 0; c < FC; ++c) acc[c] = 0.0f;
    const int beg = tile_offsets[tile], end = tile_offsets[tile + 1];
    for (int b = beg; b < end; b += kAnBatch) {
        const int cnt = min(kAnBatch, end - b);
        __syncthreads();
        if (static_cast<int>(threadIdx.x) < cnt) {
            const int j = threadIdx.x;
            const int g = gid_sorted[b + j];
            const float4* gr = reinterpret_cast<const float4*>(geo + static_cast<int64_t>(g) * 8);
            const float4 g0 = gr[0], g1 = gr[1];  // (x, y, A, B), (D, a, b, d)
            const Frame f = frame_of(g1.y, g1.z, g1.z, g1.w);
            const float sh = f.iso ? f.s : f.sh, sl = f.iso ? f.s : f.sl;
            const float ct = f.iso ? 1.0f : f.ct, st = f.iso ? 0.0f : f.st, ish = 1.0f / sh, isl = 1.0f / sl;
            const float X0 = static_cast<float>(tx0) - g0.x, Y0 = static_cast<float>(ty0) - g0.y;
            const bool far = far_from_tile(ct, st, ish, isl, X0, X0 + static_cast<float>(kTile - 1), Y0,
                                           Y0 + static_cast<float>(kTile - 1));
            s_a[j] = make_float4(g0.x, g0.y, ct, st);
            s_b[j] = make_float4(ish, isl, kTwoPi * sh * sl, far ? 1.0f : 0.0f);
            const float op = opacity != nullptr ? opacity[g] : 1.0f;
#pragma unroll
            for (int c = 0; c < FC; ++c) s_f[j][c] = c < F ? feat[static_cast<int64_t>(g) * F + c] * op : 0.0f;
        }
        __syncthreads();
        for (int j = 0; j < cnt; ++j) {
            const float4 a = s_a[j], q = s_b[j];
            if (q.w != 0.0f) continue;  // below 1e-27 at every pixel of the tile (same for all threads)
            const float dx = fpx - a.x, dy = fpy - a.y;
            const float uh = a.z * dx + a.w * dy, ul = -a.w * dx + a.z * dy;
            const float ih = logistic((uh + 0.5f) * q.x) - logistic((uh - 0.5f) * q.x);
            const float il = logistic((ul + 0.5f) * q.y) - logistic((ul - 0.5f) * q.y);
            const float wgt = q.z * ih * il;
#pragma unroll
            for (int c = 0; c < FC; ++c) acc[c] = fmaf(wgt, s_f[j][c], acc[c]);
        }
    }
    if (px >= W || py >= H) return;
    const int64_t plane = static_cast<int64_t>(H) * W, pix = static_cast<int64_t>(py) * W + px;
#pragma unroll
    for (int c = 0; c < FC; ++c) {
        if (c < F) image[c * plane + pix] = acc[c];
    }
}

template <int FC>
__global__ void __launch_bounds__(kAnThreads) k_render_analytic_bwd(
    int F, int H, int W, int ntx, const float* __restrict__ geo, const float* __restrict__ feat,
    const float* __restrict__ opacity, const int32_t* __restrict__ gid_sorted, const int32_t* __restrict__ tile_offsets,
    const int4* __restrict__ aabb, const int32_t* __restrict__ pair_offset, const float* __restrict__ grad_image,
    float* __restrict__ pairgrad, int pstride) {
    __shared__ float s_go[FC][kTilePixels];
    const int tile = blockIdx.x;
    const int tile_x = tile % ntx, tile_y = tile / ntx;
    const int tx0 = tile_x * kTile, ty0 = tile_y * kTile;
    const int64_t plane = static_cast<int64_t>(H) * W;
    {
        const int px = tx0 + (threadIdx.x & (kTile - 1)), py = ty0 + (threadIdx.x >> 4);
        const bool in = px < W && py < H;
#pragma unroll
        for (int c = 0; c < FC; ++c) {
            s_go[c][threadIdx.x] = in && c < F ? grad_image[c * plane + static_cast<int64_t>(py) * W + px] : 0.0f;
        }
    }
    __syncthreads();
    const int nrow = min(kTile, H - ty0), ncol = min(kTile, W - tx0);
    const int beg = tile_offsets[tile], end = tile_offsets[tile + 1];
    for (int e = beg + static_cast<int>(threadIdx.x); e < end; e += kAnThreads) {
        const int g = gid_sorted[e];
        const float4* gr = reinterpret_cast<const float4*>(geo + static_cast<int64_t>(g) * 8);
        const float4 g0 = gr[0], g1 = gr[1];
        const Frame f = frame_of(g1.y, g1.z, g1.z, g1.w);
        const float sh = f.iso ? f.s : f.sh, sl = f.iso ? f.s : f.sl;
        const float ct = f.iso ? 1.0f : f.ct, st = f.iso ? 0.0f : f.st;
        const float K = kTwoPi * sh * sl;
        const float op = opacity != nullptr ? opacity[g] : 1.0f;
        float fv[FC], dF[FC];
#pragma unroll
        for (int c = 0; c < FC; ++c) {
            fv[c] = c < F ? feat[static_cast<int64_t>(g) * F + c] * op : 0.0f;
            dF[c] = 0.0f;
        }
        float Gx = 0.0f, Gy = 0.0f, Gt = 0.0f, Gh = 0.0f, Gl = 0.0f;
        const float X0 = static_cast<float>(tx0) - g0.x, Y0 = static_cast<float>(ty0) - g0.y;
        const bool far = far_from_tile(ct, st, 1.0f / sh, 1.0f / sl, X0, X0 + static_cast<float>(kTile - 1), Y0,
                                       Y0 + static_cast<float>(kTile - 1));
        for (int ly = 0; ly < (far ? 0 : nrow); ++ly) {
            const float dy = static_cast<float>(ty0 + ly) - g0.y;
            for (int lx = 0; lx < ncol; ++lx) {
                const float dx = static_cast<float>(tx0 + lx) - g0.x;
                const float uh = ct * dx + st * dy, ul = -st * dx + ct * dy;
                const AxisTerm ih = axis_term(uh, sh, true), il = axis_term(ul, sl, true);
                const float wgt = K * ih.v * il.v;
                const int p = ly * kTile + lx;
                float dLdw = 0.0f;
#pragma unroll
                for (int c = 0; c < FC; ++c) {
                    const float go = s_go[c][p];
                    dLdw = fmaf(go, fv[c], dLdw);
                    dF[c] = fmaf(wgt, go, dF[c]);
                }
                const float gk = dLdw * K;
                Gx = fmaf(gk, ih.du * ct * il.v - ih.v * il.du * st, Gx);
                Gy = fmaf(gk, ih.du * st * il.v + ih.v * il.du * ct, Gy);
                Gt = fmaf(gk, ih.du * ul * il.v - ih.v * il.du * uh, Gt);
                Gh = fmaf(dLdw, wgt / sh + K * il.v * ih.dsigma, Gh);
                Gl = fmaf(dLdw, wgt / sl + K * ih.v * il.dsigma, Gl);
            }
        }
        float ga, gb, gc;
        frame_grad(f, Gh, Gl, Gt, ga, gb, gc);
        const int4 tb = aabb[g];
        const int slot = pair_offset[g] + (tile_y - tb.y) * (tb.z - tb.x) + (tile_x - tb.x);
        float* row = pairgrad + static_cast<int64_t>(slot) * pstride;
        row[0] = -Gx;  // d/dx of (p - x)
        row[1] = -Gy;
        row[2] = ga;
        row[3] = gb;
        row[4] = gc;
#pragma unroll
        for (int c = 0; c < FC; ++c) {
            if (c < F) row[5 + c] = dF[c];
        }
    }
}

#define OSS_AN_DISPATCH(f, CALL) \
    ((f) <= 1 ? CALL(1) : (f) <= 3 ? CALL(3) : (f) <= 4 ? CALL(4) : (f) <= 8 ? CALL(8) : (f) <= 16 ? CALL(16) : CALL(32))

}  // namespace

cudaError_t launch_render_analytic_forward(int f, int h, int w, const float* geo, const float* feat,
                                           const float* opacity, const int32_t* gid_sorted,
                                           const int32_t* tile_offsets, float* image, cudaStream_t stream) {
    const int ntx = static_cast<int>(div_up(w, kTile)), nty = static_cast<int>(div_up(h, kTile));
    if (ntx * nty == 0 || f == 0) return cudaSuccess;
#define OSS_AN_FWD(FC)                                                                                         \
    (k_render_analytic_fwd<FC><<<static_cast<unsigned>(ntx * nty), kAnThreads, 0, stream>>>(                 \
         f, h, w, ntx, geo, feat, opacity, gid_sorted, tile_offsets, image),                                   \
     cudaGetLastError())
    return OSS_AN_DISPATCH(f, OSS_AN_FWD);
#undef OSS_AN_FWD
}

cudaError_t launch_render_analytic_backward_pairs(int f, int h, int w, const float* geo, const float* feat,
                                                  const float* opacity, const int32_t* gid_sorted,
                                                  const int32_t* tile_offsets, const int32_t* aabb,
                                                  const int32_t* pair_offset, const float* grad_image,
                                                  float* pairgrad, int pair_stride, cudaStream_t stream) {
    const int ntx = static_cast<int>(div_up(w, kTile)), nty = static_cast<int>(div_up(h, kTile));
    if (ntx * nty == 0 || f == 0) return cudaSuccess;
#define OSS_AN_BWD(FC)                                                                                         \
    (k_render_analytic_bwd<FC><<<static_cast<unsigned>(ntx * nty), kAnThreads, 0, stream>>>(                 \
         f, h, w, ntx, geo, feat, opacity, gid_sorted, tile_offsets, reinterpret_cast<const int4*>(aabb),      \
         pair_offset, grad_image, pairgrad, pair_stride),                                                      \
     cudaGetLastError())
    return OSS_AN_DISPATCH(f, OSS_AN_BWD);
#undef OSS_AN_BWD
}

}  // namespace oss
