// Front-to-back alpha compositing: the opt-in blend="alpha" mode.  The
// reference rasterizer is additive only (rasterizer_fwd.cu:238-286); this mode
// follows the standard over operator instead, on the same tile lists ordered by
// (depth, gid):
//   G = exp(-q/2) (0 for q < 0 or non-finite), a = min(0.99, opacity G),
//   entries with a < 1/255 are skipped, compositing stops before the first
//   entry that would take the transmittance T below 1e-4,
//   C += feat a T, T *= 1 - a, out = C + T background.
// The forward keeps, per pixel, the final T and the list position after the
// last composited entry; the backward replays the list back to front from
// there, dividing T back out and carrying the normalised colour behind each
// entry, so it needs no per-entry storage.
//
// Forward: one CTA per tile, PX pixels of one column per thread (the layout of
// the additive forward), list staged in batches in shared memory; a CTA stops
// fetching batches once every one of its pixels has stopped, and a warp skips
// the rest of a batch once all of its pixels have.
//
// Backward: the same pixel layout, entries visited back to front.  Per entry a
// thread sums its pixels' contributions (Sx, Sy, Sxx, Sxy, Syy of the
// dq-weight, d opacity, d feat), the warp reduces them with a fixed xor-shuffle
// tree, and the warps' partials are added in warp order into one row per pair
// at its gid-major slot: gradients are bitwise reproducible.  Entries behind
// every pixel's last composited one get zero rows.
#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

constexpr float kAlphaMax = 0.99f;
constexpr float kAlphaMin = 1.0f / 255.0f;
constexpr float kTransMin = 1.0e-4f;

template <int FC>
struct AlphaCfg {
    static constexpr int PX = FC <= 4 ? 4 : (FC <= 16 ? 2 : 1);  // pixels per thread
    static constexpr int NT = kTilePixels / PX;                   // threads per tile
    static constexpr int NW = NT / 32;                            // warps per tile
    static constexpr int S = ((2 + FC + 3) / 4) * 4;              // [D, opacity, feat...] floats
    static constexpr int BATCH = S <= 8 ? 128 : (S <= 20 ? 64 : (S <= 36 ? 32 : 16));
    static constexpr int NV = 6 + FC;                             // Sx Sy Sxx Sxy Syy dOp dF[FC]
    static_assert((2 + FC) % 4 != 0, "the record's last float must be padding (it holds the alpha cut)");
};

// Stage list entries [b, b + cnt) of a tile: geometry (x, y, A, B) and the
// [D, opacity, feat(F), 0...] record.
template <int FC>
__device__ __forceinline__ void stage_alpha(int b, int cnt, int F, const float* __restrict__ geo,
                                            const float* __restrict__ feat, const float* __restrict__ opacity,
                                            const int32_t* __restrict__ gid_sorted, float4* s_geo, float* s_rec,
                                            int* s_gid) {
    constexpr int S = AlphaCfg<FC>::S;
    for (int j = threadIdx.x; j < cnt; j += AlphaCfg<FC>::NT) {
        const int g = gid_sorted[b + j];
        const float4* rec = reinterpret_cast<const float4*>(geo + static_cast<int64_t>(g) * 8);
        s_geo[j] = rec[0];
        float* r = s_rec + j * S;
        r[0] = rec[1].x;
        r[1] = opacity != nullptr ? opacity[g] : 1.0f;
        const float* fg = feat + static_cast<int64_t>(g) * F;
#pragma unroll
        for (int c = 0; c < S - 2; ++c) r[2 + c] = c < F && c < FC ? fg[c] : 0.0f;
        // r[S - 1] (always padding: 2 + FC is never a multiple of 4) = the q' below which
        // alpha = opacity * 2^q' is clearly under 1/255, with a 1e-3 margin (0.07% in
        // alpha): pixels below it are skipped before the exact test
        r[S - 1] = -log2f(255.0f * r[1]) - 1.0e-3f;
        if (s_gid != nullptr) s_gid[j] = g;
    }
}

template <int FC>
__global__ void __launch_bounds__(AlphaCfg<FC>::NT) k_render_alpha_fwd(
    int F, int H, int W, int ntx, const float* __restrict__ geo, const float* __restrict__ feat,
    const float* __restrict__ opacity, const float* __restrict__ background, const int32_t* __restrict__ gid_sorted,
    const int32_t* __restrict__ tile_offsets, float* __restrict__ image, float* __restrict__ t_final,
    int32_t* __restrict__ n_contrib) {
    constexpr int PX = AlphaCfg<FC>::PX;
    constexpr int S = AlphaCfg<FC>::S;
    constexpr int BATCH = AlphaCfg<FC>::BATCH;
    constexpr int ROWSTEP = kTile / PX;
    __shared__ float4 s_geo[BATCH];
    __shared__ __align__(16) float s_rec[BATCH * S];

    const int tile = blockIdx.x;
    const int tx0 = (tile % ntx) * kTile;
    const int ty0 = (tile / ntx) * kTile;
    const int px = tx0 + (threadIdx.x & (kTile - 1));
    const int ly = threadIdx.x >> 4;
    const float fpx = static_cast<float>(px);
    float fpy[PX], T[PX], C[PX][FC];
    int last[PX];
    bool live[PX];
#pragma unroll
    for (int k = 0; k < PX; ++k) {
        const int py = ty0 + ly + k * ROWSTEP;
        fpy[k] = static_cast<float>(py);
        T[k] = 1.0f;
        last[k] = 0;
        live[k] = px < W && py < H;
#pragma unroll
        for (int c = 0; c < FC; ++c) C[k][c] = 0.0f;
    }
    const int start = tile_offsets[tile];
    const int end = tile_offsets[tile + 1];
    for (int b = start; b < end; b += BATCH) {
        bool any = false;
#pragma unroll
        for (int k = 0; k < PX; ++k) any = any || live[k];
        if (__syncthreads_or(any ? 1 : 0) == 0) break;  // every pixel of the tile has stopped
        const int cnt = min(BATCH, end - b);
        stage_alpha<FC>(b, cnt, F, geo, feat, opacity, gid_sorted, s_geo, s_rec, nullptr);
        __syncthreads();
        for (int j = 0; j < cnt; ++j) {
            if ((j & 31) == 0) {
                bool mine = false;
#pragma unroll
                for (int k = 0; k < PX; ++k) mine = mine || live[k];
                if (!__any_sync(0xffffffffu, mine)) break;  // the warp's pixels have all stopped
            }
            const float4 g0 = s_geo[j];
            const float* r = s_rec + j * S;
            const float D = r[0];
            const float op = r[1];
            const float dx = fpx - g0.x;
            const float bdx = g0.w * dx;
            const float adx2 = (g0.z * dx) * dx;
            const float qmin = r[S - 1];
#pragma unroll
            for (int k = 0; k < PX; ++k) {
                if (!live[k]) continue;
                const float dy = fpy[k] - g0.y;
                const float q = fmaf(dy, fmaf(D, dy, bdx), adx2);
                if (q < qmin) continue;      // alpha clearly below 1/255
                if (!(q <= 0.0f)) continue;  // q' > 0 or NaN: weight 0
                const float a = fminf(op * ex2_ftz(q), kAlphaMax);
                if (a < kAlphaMin) continue;
                const float tn = T[k] * (1.0f - a);
                if (tn < kTransMin) {
                    live[k] = false;
                    continue;
                }
                const float wgt = a * T[k];
#pragma unroll
                for (int c = 0; c < FC; ++c) C[k][c] = fmaf(r[2 + c], wgt, C[k][c]);
                T[k] = tn;
                last[k] = b - start + j + 1;
            }
        }
    }
    if (px >= W) return;
    const int64_t plane = static_cast<int64_t>(H) * W;
#pragma unroll
    for (int k = 0; k < PX; ++k) {
        const int py = ty0 + ly + k * ROWSTEP;
        if (py >= H) continue;
        const int64_t pix = static_cast<int64_t>(py) * W + px;
#pragma unroll
        for (int c = 0; c < FC; ++c) {
            if (c < F) image[c * plane + pix] = fmaf(T[k], background != nullptr ? background[c] : 0.0f, C[k][c]);
        }
        t_final[pix] = T[k];
        n_contrib[pix] = last[k];
    }
}

__host__ __device__ constexpr int pow2_ceil32(int v) { return v <= 1 ? 1 : v <= 2 ? 2 : v <= 4 ? 4 : v <= 8 ? 8 : v <= 16 ? 16 : 32; }
__host__ __device__ constexpr int log2_32(int v) { return v >= 32 ? 5 : v >= 16 ? 4 : v >= 8 ? 3 : v >= 4 ? 2 : v >= 2 ? 1 : 0; }

template <int FC>
__global__ void __launch_bounds__(AlphaCfg<FC>::NT) k_render_alpha_bwd(
    int F, int H, int W, int ntx, const float* __restrict__ geo, const float* __restrict__ feat,
    const float* __restrict__ opacity, const float* __restrict__ background, const int32_t* __restrict__ gid_sorted,
    const int32_t* __restrict__ tile_offsets, const float* __restrict__ t_final, const int32_t* __restrict__ n_contrib,
    const float* __restrict__ grad_image, const int4* __restrict__ aabb, const int32_t* __restrict__ pair_offset,
    float* __restrict__ pairgrad, int pstride) {
    constexpr int PX = AlphaCfg<FC>::PX;
    constexpr int NT = AlphaCfg<FC>::NT;
    constexpr int NW = AlphaCfg<FC>::NW;
    constexpr int S = AlphaCfg<FC>::S;
    constexpr int BATCH = AlphaCfg<FC>::BATCH;
    constexpr int NV = AlphaCfg<FC>::NV;
    constexpr int ROWSTEP = kTile / PX;
    __shared__ float4 s_geo[BATCH];
    __shared__ __align__(16) float s_rec[BATCH * S];
    __shared__ int s_gid[BATCH];
    __shared__ float s_part[NW][BATCH][NV];
    __shared__ int s_jmax;

    const int tile = blockIdx.x;
    const int tile_x = tile % ntx;
    const int tile_y = tile / ntx;
    const int tx0 = tile_x * kTile;
    const int ty0 = tile_y * kTile;
    const int px = tx0 + (threadIdx.x & (kTile - 1));
    const int ly = threadIdx.x >> 4;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const float fpx = static_cast<float>(px);
    const int64_t plane = static_cast<int64_t>(H) * W;
    if (threadIdx.x == 0) s_jmax = 0;
    float fpy[PX], T[PX], go[PX][FC], back[PX][FC];
    int nc[PX];
#pragma unroll
    for (int k = 0; k < PX; ++k) {
        const int py = ty0 + ly + k * ROWSTEP;
        fpy[k] = static_cast<float>(py);
        const bool in = px < W && py < H;
        const int64_t pix = static_cast<int64_t>(py) * W + px;
        T[k] = in ? t_final[pix] : 1.0f;
        nc[k] = in ? n_contrib[pix] : 0;
#pragma unroll
        for (int c = 0; c < FC; ++c) {
            go[k][c] = in && c < F ? grad_image[c * plane + pix] : 0.0f;
            back[k][c] = background != nullptr && c < F ? background[c] : 0.0f;
        }
    }
    __syncthreads();
    int mine = 0;
#pragma unroll
    for (int k = 0; k < PX; ++k) mine = max(mine, nc[k]);
    atomicMax(&s_jmax, mine);
    __syncthreads();
    const int jmax = s_jmax;
    const int start = tile_offsets[tile];

    for (int hi = jmax; hi > 0; hi -= BATCH) {
        const int lo = max(0, hi - BATCH);
        const int cnt = hi - lo;
        __syncthreads();  // the previous batch's rows have been written
        stage_alpha<FC>(start + lo, cnt, F, geo, feat, opacity, gid_sorted, s_geo, s_rec, s_gid);
        __syncthreads();
        for (int jj = cnt - 1; jj >= 0; --jj) {
            const int j = lo + jj;  // position in the tile list
            const float4 g0 = s_geo[jj];
            const float* r = s_rec + jj * S;
            const float D = r[0];
            const float op = r[1];
            const float dx = fpx - g0.x;
            const float bdx = g0.w * dx;
            const float adx2 = (g0.z * dx) * dx;
            float v[NV];
#pragma unroll
            for (int i = 0; i < NV; ++i) v[i] = 0.0f;
#pragma unroll
            for (int k = 0; k < PX; ++k) {
                if (j >= nc[k]) continue;
                const float dy = fpy[k] - g0.y;
                const float q = fmaf(dy, fmaf(D, dy, bdx), adx2);
                if (q < r[S - 1]) continue;  // alpha clearly below 1/255
                if (!(q <= 0.0f)) continue;
                const float G = ex2_ftz(q);
                const float og = op * G;
                const float a = fminf(og, kAlphaMax);
                if (a < kAlphaMin) continue;
                // transmittance in front of this entry; 1 - a lies in [0.01, 1), where the
                // fast division is within 2 ulp (a correctly rounded one cost 4% of the step)
                T[k] = __fdividef(T[k], 1.0f - a);
                const float wgt = a * T[k];
                float dlda = 0.0f;
#pragma unroll
                for (int c = 0; c < FC; ++c) {
                    dlda = fmaf(go[k][c], r[2 + c] - back[k][c], dlda);
                    v[6 + c] = fmaf(wgt, go[k][c], v[6 + c]);
                    back[k][c] = fmaf(r[2 + c], a, back[k][c] * (1.0f - a));
                }
                dlda *= T[k];
                if (og < kAlphaMax) {  // not clamped: gradient reaches G and the opacity
                    v[5] = fmaf(G, dlda, v[5]);
                    const float gw = G * op * dlda;  // dL/dq = -gw / 2
                    const float gdx = gw * dx;
                    v[0] += gdx;
                    v[1] = fmaf(gw, dy, v[1]);
                    v[2] = fmaf(gdx, dx, v[2]);
                    v[3] = fmaf(gdx, dy, v[3]);
                    v[4] = fmaf(gw * dy, dy, v[4]);
                }
            }
            // warp sums of the NV values, 32 (or fewer) at a time, each landing on one lane group
#pragma unroll
            for (int c0 = 0; c0 < NV; c0 += 32) {
                constexpr int KK = pow2_ceil32(NV);
                constexpr int KB = KK > 32 ? 32 : KK;
                float x[KB];
#pragma unroll
                for (int i = 0; i < KB; ++i) x[i] = c0 + i < NV ? v[c0 + i < NV ? c0 + i : 0] : 0.0f;
                const float tot = warp_reduce_scatter<KB>(x);
                const int idx = c0 + (lane >> (5 - log2_32(KB)));
                if ((lane & ((32 / KB) - 1)) == 0 && idx < NV && idx < c0 + KB) s_part[warp][jj][idx] = tot;
            }
        }
        __syncthreads();
        // one row per entry: (Sx, Sy, d_conic(3), dF(F), d_opacity) at its gid-major pair slot
        for (int jj = threadIdx.x; jj < cnt; jj += NT) {
            float t[NV];
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                float acc = s_part[0][jj][i];
#pragma unroll
                for (int wv = 1; wv < NW; ++wv) acc += s_part[wv][jj][i];
                t[i] = acc;
            }
            const int g = s_gid[jj];
            const int4 box = aabb[g];
            const int slot = pair_offset[g] + (tile_y - box.y) * (box.z - box.x) + (tile_x - box.x);
            float* row = pairgrad + static_cast<int64_t>(slot) * pstride;
            row[0] = t[0];
            row[1] = t[1];
            row[2] = -0.5f * t[2];
            row[3] = -t[3];
            row[4] = -0.5f * t[4];
#pragma unroll
            for (int c = 0; c < FC; ++c) {
                if (c < F) row[5 + c] = t[6 + c];
            }
            row[5 + F] = t[5];
        }
    }
    // entries past every pixel's last composited one get nothing: zero their rows
    const int len = tile_offsets[tile + 1] - start;
    for (int jj = jmax + threadIdx.x; jj < len; jj += NT) {
        const int g = gid_sorted[start + jj];
        const int4 box = aabb[g];
        const int slot = pair_offset[g] + (tile_y - box.y) * (box.z - box.x) + (tile_x - box.x);
        float* row = pairgrad + static_cast<int64_t>(slot) * pstride;
        for (int i = 0; i < 6 + F; ++i) row[i] = 0.0f;
    }
}

template <int FC>
__global__ void __launch_bounds__(256) k_reduce_alpha(int n, int F, const float* __restrict__ pairgrad, int pstride,
                                                      const int32_t* __restrict__ pair_offset,
                                                      const float* __restrict__ geo, const float* __restrict__ scale,
                                                      const float* __restrict__ rot, float* __restrict__ d_xy,
                                                      float* __restrict__ d_conic, float* __restrict__ d_feat,
                                                      float* __restrict__ d_opacity, float* __restrict__ d_scale,
                                                      float* __restrict__ d_rot) {
    const int g = blockIdx.x * 256 + threadIdx.x;
    if (g >= n) return;
    const int beg = pair_offset[g];
    const int end = pair_offset[g + 1];
    float s[5] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    float dF[FC];
#pragma unroll
    for (int c = 0; c < FC; ++c) dF[c] = 0.0f;
    float dop = 0.0f;
    for (int p = beg; p < end; ++p) {
        const float* row = pairgrad + static_cast<int64_t>(p) * pstride;
#pragma unroll
        for (int i = 0; i < 5; ++i) s[i] += row[i];
#pragma unroll
        for (int c = 0; c < FC; ++c) {
            if (c < F) dF[c] += row[5 + c];
        }
        dop += row[5 + F];
    }
    const float4 k1 = reinterpret_cast<const float4*>(geo + static_cast<int64_t>(g) * 8)[1];
    d_xy[2 * g + 0] = fmaf(k1.y, s[0], k1.z * s[1]);
    d_xy[2 * g + 1] = fmaf(k1.z, s[0], k1.w * s[1]);
    d_conic[3 * g + 0] = s[2];
    d_conic[3 * g + 1] = s[3];
    d_conic[3 * g + 2] = s[4];
#pragma unroll
    for (int c = 0; c < FC; ++c) {
        if (c < F) d_feat[static_cast<int64_t>(g) * F + c] = dF[c];
    }
    if (d_opacity != nullptr) d_opacity[g] = dop;
    if (d_scale != nullptr) {
        float dsx, dsy, dr;
        conic_grad_to_scale_rot(scale[2 * g], scale[2 * g + 1], rot[g], s[2], s[3], s[4], dsx, dsy, dr);
        d_scale[2 * g + 0] = dsx;
        d_scale[2 * g + 1] = dsy;
        d_rot[g] = dr;
    }
}

}  // namespace

int alpha_pair_stride(int f) { return ((6 + f + 3) / 4) * 4; }

#define OSS_ALPHA_DISPATCH(f, CALL) \
    ((f) <= 1 ? CALL(1) : (f) <= 3 ? CALL(3) : (f) <= 4 ? CALL(4) : (f) <= 8 ? CALL(8) : (f) <= 16 ? CALL(16) : (f) <= 32 ? CALL(32) : CALL(64))

cudaError_t launch_render_alpha_forward(int f, int h, int w, const float* geo, const float* feat, const float* opacity,
                                        const float* background, const int32_t* gid_sorted,
                                        const int32_t* tile_offsets, float* image, float* t_final,
                                        int32_t* n_contrib, cudaStream_t stream) {
    const int ntx = static_cast<int>(div_up(w, kTile));
    const int num_tiles = ntx * static_cast<int>(div_up(h, kTile));
    if (num_tiles == 0) return cudaSuccess;
#define OSS_AF(FC)                                                                                               \
    (k_render_alpha_fwd<FC><<<static_cast<unsigned>(num_tiles), AlphaCfg<FC>::NT, 0, stream>>>(                 \
         f, h, w, ntx, geo, feat, opacity, background, gid_sorted, tile_offsets, image, t_final, n_contrib),    \
     cudaGetLastError())
    return OSS_ALPHA_DISPATCH(f, OSS_AF);
#undef OSS_AF
}

cudaError_t launch_render_alpha_backward(int f, int h, int w, const float* geo, const float* feat,
                                         const float* opacity, const float* background, const int32_t* gid_sorted,
                                         const int32_t* tile_offsets, const float* t_final, const int32_t* n_contrib,
                                         const float* grad_image, const int32_t* aabb, const int32_t* pair_offset,
                                         float* pairgrad, cudaStream_t stream) {
    const int ntx = static_cast<int>(div_up(w, kTile));
    const int num_tiles = ntx * static_cast<int>(div_up(h, kTile));
    if (num_tiles == 0) return cudaSuccess;
    const int ps = alpha_pair_stride(f);
#define OSS_AB(FC)                                                                                               \
    (k_render_alpha_bwd<FC><<<static_cast<unsigned>(num_tiles), AlphaCfg<FC>::NT, 0, stream>>>(                 \
         f, h, w, ntx, geo, feat, opacity, background, gid_sorted, tile_offsets, t_final, n_contrib, grad_image, \
         reinterpret_cast<const int4*>(aabb), pair_offset, pairgrad, ps),                                        \
     cudaGetLastError())
    return OSS_ALPHA_DISPATCH(f, OSS_AB);
#undef OSS_AB
}

cudaError_t launch_reduce_alpha_grads(int n, int f, const float* pairgrad, const int32_t* pair_offset,
                                      const float* geo, const float* scale, const float* rot, float* d_xy,
                                      float* d_conic, float* d_feat, float* d_opacity, float* d_scale, float* d_rot,
                                      cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    const int ps = alpha_pair_stride(f);
    const unsigned blocks = static_cast<unsigned>(div_up(n, 256));
#define OSS_AR(FC)                                                                                               \
    (k_reduce_alpha<FC><<<blocks, 256, 0, stream>>>(n, f, pairgrad, ps, pair_offset, geo, scale, rot, d_xy,     \
                                                   d_conic, d_feat, d_opacity, d_scale, d_rot),                 \
     cudaGetLastError())
    return OSS_ALPHA_DISPATCH(f, OSS_AR);
#undef OSS_AR
}

}  // namespace oss
