// The additive tile render with the Analytic-Splatting pixel integral as the
// weight (oss/sr/v6/aa_analytic_splat.py:72-202 in place of exp(-q/2) of
// rasterizer_fwd.cu:151-322): out[c](p) = sum over the tile list of
// feat'[g][c] * w_g(p - xy_g), with w the integral of the un-normalised Gaussian
// of inverse covariance (a, b, d) over the unit pixel square at integer pixel
// centres.  The logistic tails vanish in fp32 before q = 176 (S'(x) ~ exp(-1.6 x
// - 0.07 x^3)), so the exact-mode lists hold every non-zero term.
//
// Work layout: one CTA of 8 warps per 16x16 tile, warp w owning the 8x4 pixel
// patch (w & 1, w >> 1) of it.  A batch of list entries is staged in shared
// memory, one thread per entry: the eigen-frame (rotation, per-axis 1 / sigma,
// 2 pi sigma_h sigma_l; the shared sigma and no rotation below the 1e-5
// eigengap) and an 8-bit mask of the patches the entry reaches.  A patch is out
// of reach when each of its pixel centres lies 9 sigma or more (less the half
// pixel) from the entry's centre along one frame axis: there each pixel's weight
// is below 1e-27, negligible next to the fp32 sums it joins.  About half of an
// exact list's entries reach no patch of their tile, and a reaching entry
// reaches about half of the tile's patches, so the masks remove three quarters
// of the pixel evaluations.
//
// The logistic is the fast form (logistic_fast: __expf and the approximate
// reciprocal, within about one ulp of S); the elementwise integral keeps the
// accurate one.
//
// Forward: each warp walks the batch's entries that reach its patch (ballots of
// the mask bits, so the walk is warp-uniform) and accumulates its 32 pixels.
// Backward: the tile's dL/dimage sits in shared memory in patch order; warps take
// entries one at a time from a shared counter, each lane evaluating its pixel of
// every patch the entry reaches and summing dL/d(u_h, u_l) (in the entry's
// frame), dL/d(theta), dL/d(sigma_h), dL/d(sigma_l) and dF; one reduce-scatter
// per entry (a plain butterfly above 32 sums) gives the warp's totals, and after the batch one thread
// per entry turns them into d_xy and d_conic (frame_grad) and writes the pair
// row.  The rows feed the per-Gaussian reduce of the additive path with
// rows_dxy set.
#include "analytic_math.cuh"
#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

using namespace analytic;

constexpr int kAnThreads = 256;  // 8 warps, one CTA per tile
constexpr int kPatchW = 8, kPatchH = 4, kPatches = kTilePixels / (kPatchW * kPatchH);
static_assert(kPatches * 32 == kAnThreads, "one warp per patch");

// Entries staged per batch: shared memory stays within the 48 KB static limit for
// every channel count (the backward also holds F x 256 floats of dL/dimage).
template <int FC>
struct AnBatch {
    static constexpr int value = FC <= 4 ? 256 : FC <= 8 ? 128 : FC <= 16 ? 64 : 32;
};

__device__ __forceinline__ int patch_x0(int p) { return (p & 1) * kPatchW; }
__device__ __forceinline__ int patch_y0(int p) { return (p >> 1) * kPatchH; }

struct StagedEntry {
    float4 a;  // x, y, cos theta, sin theta
    float4 b;  // 1 / sigma_h, 1 / sigma_l, 2 pi sigma_h sigma_l, unused
    unsigned mask;
};

// Frame and patch mask of one list entry for the tile at (tx0, ty0).  Along a
// frame axis (c, s) the pixel centres of a patch project onto an interval of
// centre u(patch centre) and half-width |c| * 3.5 + |s| * 1.5; the patch is out of
// reach when that interval stays 9 sigma + 1/2 px clear of 0 on either axis.
__device__ __forceinline__ StagedEntry stage_entry(const float* __restrict__ geo, int g, int tx0, int ty0) {
    const float4* gr = reinterpret_cast<const float4*>(geo + static_cast<int64_t>(g) * 8);
    const float4 g0 = gr[0], g1 = gr[1];  // (x, y, A, B), (D, a, b, d)
    const Frame f = frame_of(g1.y, g1.z, g1.z, g1.w);
    const float sh = f.iso ? f.s : f.sh, sl = f.iso ? f.s : f.sl;
    const float ct = f.iso ? 1.0f : f.ct, st = f.iso ? 0.0f : f.st;
    const float ish = 1.0f / sh, isl = 1.0f / sl;
    const float hx = 0.5f * static_cast<float>(kPatchW - 1), hy = 0.5f * static_cast<float>(kPatchH - 1);
    const float eh = fabsf(ct) * hx + fabsf(st) * hy, el = fabsf(st) * hx + fabsf(ct) * hy;
    unsigned mask = 0;
#pragma unroll
    for (int p = 0; p < kPatches; ++p) {
        const float X = static_cast<float>(tx0 + patch_x0(p)) + hx - g0.x;
        const float Y = static_cast<float>(ty0 + patch_y0(p)) + hy - g0.y;
        const float gh = (fabsf(ct * X + st * Y) - eh - 0.5f) * ish;
        const float gl = (fabsf(-st * X + ct * Y) - el - 0.5f) * isl;
        if (!(gh >= 9.0f || gl >= 9.0f)) mask |= 1u << p;
    }
    StagedEntry e;
    e.a = make_float4(g0.x, g0.y, ct, st);
    e.b = make_float4(ish, isl, kTwoPi * sh * sl, 0.0f);
    e.mask = mask;
    return e;
}

template <int FC>
__global__ void __launch_bounds__(kAnThreads) k_render_analytic_fwd(int F, int H, int W, int ntx,
                                                                     const float* __restrict__ geo,
                                                                     const float* __restrict__ feat,
                                                                     const float* __restrict__ opacity,
                                                                     const int32_t* __restrict__ gid_sorted,
                                                                     const int32_t* __restrict__ tile_offsets,
                                                                     float* __restrict__ image) {
    constexpr int B = AnBatch<FC>::value;
    __shared__ float4 s_a[B];
    __shared__ float4 s_b[B];
    __shared__ float s_f[B][FC];
    __shared__ unsigned char s_m[B];
    const int warp = static_cast<int>(threadIdx.x) >> 5, lane = static_cast<int>(threadIdx.x) & 31;
    const int tile = blockIdx.x;
    const int tx0 = (tile % ntx) * kTile, ty0 = (tile / ntx) * kTile;
    const int px = tx0 + patch_x0(warp) + (lane & (kPatchW - 1)), py = ty0 + patch_y0(warp) + (lane >> 3);
    const float fpx = static_cast<float>(px), fpy = static_cast<float>(py);
    float acc[FC];
#pragma unroll
    for (int c = 0; c < FC; ++c) acc[c] = 0.0f;
    const int beg = tile_offsets[tile], end = tile_offsets[tile + 1];
    for (int b = beg; b < end; b += B) {
        const int cnt = min(B, end - b);
        __syncthreads();
        if (static_cast<int>(threadIdx.x) < cnt) {
            const int j = threadIdx.x;
            const int g = gid_sorted[b + j];
            const StagedEntry e = stage_entry(geo, g, tx0, ty0);
            s_a[j] = e.a;
            s_b[j] = e.b;
            s_m[j] = static_cast<unsigned char>(e.mask);
            const float op = opacity != nullptr ? opacity[g] : 1.0f;
#pragma unroll
            for (int c = 0; c < FC; ++c) s_f[j][c] = c < F ? feat[static_cast<int64_t>(g) * F + c] * op : 0.0f;
        }
        __syncthreads();
        for (int k = 0; k < cnt; k += 32) {
            unsigned mine = __ballot_sync(0xffffffffu, k + lane < cnt && ((s_m[k + lane] >> warp) & 1u));
            while (mine != 0u) {
                const int j = k + __ffs(mine) - 1;
                mine &= mine - 1u;
                const float4 a = s_a[j], q = s_b[j];
                const float dx = fpx - a.x, dy = fpy - a.y;
                const float uh = a.z * dx + a.w * dy, ul = -a.w * dx + a.z * dy;
                const float ih = logistic_fast((uh + 0.5f) * q.x) - logistic_fast((uh - 0.5f) * q.x);
                const float il = logistic_fast((ul + 0.5f) * q.y) - logistic_fast((ul - 0.5f) * q.y);
                const float wgt = q.z * ih * il;
#pragma unroll
                for (int c = 0; c < FC; ++c) acc[c] = fmaf(wgt, s_f[j][c], acc[c]);
            }
        }
    }
    if (px >= W || py >= H) return;
    const int64_t plane = static_cast<int64_t>(H) * W, pix = static_cast<int64_t>(py) * W + px;
#pragma unroll
    for (int c = 0; c < FC; ++c) {
        if (c < F) image[c * plane + pix] = acc[c];
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Power-of-two width holding the 5 + FC per-entry sums; 0 above a warp's 32.
template <int FC>
struct SumWidth {
    static constexpr int n = 5 + FC;
    static constexpr int value = n <= 8 ? 8 : n <= 16 ? 16 : n <= 32 ? 32 : 0;
};

template <int FC>
__global__ void __launch_bounds__(kAnThreads) k_render_analytic_bwd(
    int F, int H, int W, int ntx, const float* __restrict__ geo, const float* __restrict__ feat,
    const float* __restrict__ opacity, const int32_t* __restrict__ gid_sorted, const int32_t* __restrict__ tile_offsets,
    const int4* __restrict__ aabb, const int32_t* __restrict__ pair_offset, const float* __restrict__ grad_image,
    float* __restrict__ pairgrad, int pstride) {
    constexpr int B = AnBatch<FC>::value;
    constexpr int NS = (5 + FC) | 1;  // per-entry sums, padded to an odd stride
    __shared__ float s_go[FC][kTilePixels];  // dL/dimage in patch order: [p * 32 + lane]
    __shared__ float4 s_a[B];
    __shared__ float4 s_b[B];
    __shared__ float s_f[B][FC];
    __shared__ float s_sum[B][NS];  // Sa, Sb, G_theta, G_sigma_h, G_sigma_l, dF[F]
    __shared__ int s_gid[B];
    __shared__ unsigned char s_m[B];
    __shared__ int s_next;
    const int warp = static_cast<int>(threadIdx.x) >> 5, lane = static_cast<int>(threadIdx.x) & 31;
    const int tile = blockIdx.x;
    const int tile_x = tile % ntx, tile_y = tile / ntx;
    const int tx0 = tile_x * kTile, ty0 = tile_y * kTile;
    const int64_t plane = static_cast<int64_t>(H) * W;
    {
        const int px = tx0 + patch_x0(warp) + (lane & (kPatchW - 1)), py = ty0 + patch_y0(warp) + (lane >> 3);
        const bool in = px < W && py < H;
#pragma unroll
        for (int c = 0; c < FC; ++c) {
            s_go[c][threadIdx.x] = in && c < F ? grad_image[c * plane + static_cast<int64_t>(py) * W + px] : 0.0f;
        }
    }
    const int beg = tile_offsets[tile], end = tile_offsets[tile + 1];
    for (int b = beg; b < end; b += B) {
        const int cnt = min(B, end - b);
        __syncthreads();  // dL/dimage staged; the previous batch's epilogue done
        if (static_cast<int>(threadIdx.x) < cnt) {
            const int j = threadIdx.x;
            const int g = gid_sorted[b + j];
            const StagedEntry e = stage_entry(geo, g, tx0, ty0);
            s_a[j] = e.a;
            s_b[j] = e.b;
            s_m[j] = static_cast<unsigned char>(e.mask);
            s_gid[j] = g;
            const float op = opacity != nullptr ? opacity[g] : 1.0f;
#pragma unroll
            for (int c = 0; c < FC; ++c) s_f[j][c] = c < F ? feat[static_cast<int64_t>(g) * F + c] * op : 0.0f;
        }
        if (threadIdx.x == 0) s_next = 0;
        __syncthreads();
        for (;;) {
            int j = 0;
            if (lane == 0) j = atomicAdd(&s_next, 1);
            j = __shfl_sync(0xffffffffu, j, 0);
            if (j >= cnt) break;
            unsigned m = s_m[j];
            if (m == 0u) continue;
            const float4 a = s_a[j], q = s_b[j];
            float fv[FC], dF[FC];
#pragma unroll
            for (int c = 0; c < FC; ++c) {
                fv[c] = s_f[j][c];
                dF[c] = 0.0f;
            }
            float Sa = 0.0f, Sb = 0.0f, Gt = 0.0f, Gh = 0.0f, Gl = 0.0f;
            while (m != 0u) {
                const int p = __ffs(m) - 1;
                m &= m - 1u;
                const float fpx = static_cast<float>(tx0 + patch_x0(p) + (lane & (kPatchW - 1)));
                const float fpy = static_cast<float>(ty0 + patch_y0(p) + (lane >> 3));
                const float dx = fpx - a.x, dy = fpy - a.y;
                const float uh = a.z * dx + a.w * dy, ul = -a.w * dx + a.z * dy;
                const AxisTerm ih = axis_term_inv<true>(uh, q.x, true), il = axis_term_inv<true>(ul, q.y, true);
                const float wgt = q.z * ih.v * il.v;
                float dLdw = 0.0f;
#pragma unroll
                for (int c = 0; c < FC; ++c) {
                    const float go = s_go[c][p * 32 + lane];
                    dLdw = fmaf(go, fv[c], dLdw);
                    dF[c] = fmaf(wgt, go, dF[c]);
                }
                const float gk = dLdw * q.z;
                const float A = ih.du * il.v, Bv = ih.v * il.du;  // dI_h/du_h I_l, I_h dI_l/du_l
                Sa = fmaf(gk, A, Sa);
                Sb = fmaf(gk, Bv, Sb);
                Gt = fmaf(gk, A * ul - Bv * uh, Gt);
                Gh = fmaf(gk, il.v * fmaf(ih.v, q.x, ih.dsigma), Gh);  // d(2 pi s_h s_l I_h I_l)/ds_h
                Gl = fmaf(gk, ih.v * fmaf(il.v, q.y, il.dsigma), Gl);
            }
            constexpr int V = SumWidth<FC>::value;
            if constexpr (V > 0) {
                float v[V];
                v[0] = Sa;
                v[1] = Sb;
                v[2] = Gt;
                v[3] = Gh;
                v[4] = Gl;
#pragma unroll
                for (int i = 5; i < V; ++i) v[i] = i - 5 < FC ? dF[i - 5] : 0.0f;
                const float t = warp_reduce_scatter<V>(v);  // lane l: total of v[l >> kShift]
                constexpr int kShift = V == 8 ? 2 : V == 16 ? 1 : 0;
                const int idx = lane >> kShift;
                if ((lane & ((1 << kShift) - 1)) == 0 && idx < 5 + FC) s_sum[j][idx] = t;
            } else {
                Sa = warp_sum(Sa);
                Sb = warp_sum(Sb);
                Gt = warp_sum(Gt);
                Gh = warp_sum(Gh);
                Gl = warp_sum(Gl);
#pragma unroll
                for (int c = 0; c < FC; ++c) dF[c] = warp_sum(dF[c]);
                if (lane == 0) {
                    s_sum[j][0] = Sa;
                    s_sum[j][1] = Sb;
                    s_sum[j][2] = Gt;
                    s_sum[j][3] = Gh;
                    s_sum[j][4] = Gl;
#pragma unroll
                    for (int c = 0; c < FC; ++c) s_sum[j][5 + c] = dF[c];
                }
            }
        }
        __syncthreads();
        if (static_cast<int>(threadIdx.x) < cnt) {
            const int j = threadIdx.x, g = s_gid[j];
            const int4 tb = aabb[g];
            const int slot = pair_offset[g] + (tile_y - tb.y) * (tb.z - tb.x) + (tile_x - tb.x);
            float* row = pairgrad + static_cast<int64_t>(slot) * pstride;
            float gx = 0.0f, gy = 0.0f, ga = 0.0f, gb = 0.0f, gc = 0.0f;
            const bool reach = s_m[j] != 0;
            if (reach) {
                const float4 g1 = reinterpret_cast<const float4*>(geo + static_cast<int64_t>(g) * 8)[1];
                const Frame f = frame_of(g1.y, g1.z, g1.z, g1.w);
                const float ct = s_a[j].z, st = s_a[j].w, Sa = s_sum[j][0], Sb = s_sum[j][1];
                gx = ct * Sa - st * Sb;  // dL/d(dx, dy) from the frame-axis sums
                gy = st * Sa + ct * Sb;
                frame_grad(f, s_sum[j][3], s_sum[j][4], s_sum[j][2], ga, gb, gc);
            }
            row[0] = -gx;  // d/dx of (p - x)
            row[1] = -gy;
            row[2] = ga;
            row[3] = gb;
            row[4] = gc;
#pragma unroll
            for (int c = 0; c < FC; ++c) {
                if (c < F) row[5 + c] = reach ? s_sum[j][5 + c] : 0.0f;
            }
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
