// Backward of the additive tile render (the reference's rasterize_backward,
// rasterizer_bwd.cu:32-113), re-organised so that no per-pixel atomics remain.
//
// One CTA (4 warps) per tile.  The tile's dL/dimage block is staged once in
// shared memory.  Each lane owns one list entry (Gaussian) and walks all valid
// pixels of the tile, keeping the per-pair sums in registers:
//   g = w * sum_c go_c f'_c      (w = exp(-q/2), dL/dq = -g/2)
//   Sx = sum g dx, Sy = sum g dy, Sxx = sum g dx^2, Sxy = sum g dx dy,
//   Syy = sum g dy^2, dF_c = sum w go_c
// from which d_xy = (a Sx + b Sy, b Sx + d Sy) and
// d_conic = (-Sxx/2, -Sxy, -Syy/2) -- the reference's per-pixel terms
// (rasterizer_bwd.cu:89-108) summed over the tile.  The dy-dependent factors
// are hoisted per pixel row, so an evaluation costs ~16 FP32 ops + 1 MUFU.
//
// Deterministic mode writes each pair's partial row at its gid-major pair slot
// (pair_offset[g] + local tile index, the order oss_bin_pairs expanded it in);
// k_reduce_gaussian then sums a Gaussian's rows in that fixed order and applies
// the conic -> (scale, rot) chain rule and the opacity unfold.
// Atomic mode (caller-supplied lists) adds the pair partials with fp32 atomics:
// (F+5) atomics per pair instead of the reference's (F+5) per pixel-pair.
#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

constexpr int kBwdWarps = 4;
constexpr int kBwdThreads = kBwdWarps * 32;

template <int FC>
struct BwdCfg {
    static constexpr int SG = ((FC + 3) / 4) * 4;  // staged grad floats per pixel
};

__device__ __forceinline__ bool regular_conic_bwd(float x, float y, float a, float b, float d) {
    const bool finite = isfinite(x) && isfinite(y) && isfinite(a) && isfinite(b) && isfinite(d);
    return finite && a > 0.0f && d > 0.0f && (a * d - b * b) >= 1.0e-3f * (a * d);
}

// Per-pair sums over one full 16x16 tile: the 16 column offsets dx are hoisted
// into registers, each row hoists B*dy and D*dy*dy, and the column loop is
// fully unrolled.  CHECK keeps the reference's q >= 0 test per pixel.
template <int FC, bool CHECK>
__device__ __forceinline__ void bwd_full_tile(const float* __restrict__ s_go, float fx0, float fy0, float gx, float gy,
                                              float A, float B, float D, const float (&fv)[FC], float (&dF)[FC],
                                              float& Sx, float& Sy, float& Sxx, float& Sxy, float& Syy) {
    constexpr int SG = BwdCfg<FC>::SG;
    float dxs[kTile];
#pragma unroll
    for (int c = 0; c < kTile; ++c) dxs[c] = (fx0 + static_cast<float>(c)) - gx;
#pragma unroll 1
    for (int r = 0; r < kTile; ++r) {
        const float dy = (fy0 + static_cast<float>(r)) - gy;
        const float bdy = B * dy;
        const float ddy2 = (D * dy) * dy;
        float rowG = 0.0f, rowGx = 0.0f;
        const float* go_row = s_go + r * kTile * SG;
#pragma unroll
        for (int c = 0; c < kTile; ++c) {
            const float dx = dxs[c];
            const float q = fmaf(dx, fmaf(A, dx, bdy), ddy2);
            const float w = CHECK ? (q <= 0.0f ? ex2_ftz(q) : 0.0f) : ex2_ftz(q);
            const float4* go4 = reinterpret_cast<const float4*>(go_row + c * SG);
            float go[SG];
#pragma unroll
            for (int v = 0; v < SG / 4; ++v) {
                const float4 t = go4[v];
                go[4 * v + 0] = t.x;
                go[4 * v + 1] = t.y;
                go[4 * v + 2] = t.z;
                go[4 * v + 3] = t.w;
            }
            float dLdw = 0.0f;
#pragma unroll
            for (int k = 0; k < FC; ++k) {
                dLdw = fmaf(go[k], fv[k], dLdw);
                dF[k] = fmaf(w, go[k], dF[k]);
            }
            const float gw = w * dLdw;
            const float gdx = gw * dx;
            rowGx += gdx;
            Sxx = fmaf(gdx, dx, Sxx);
            rowG += gw;
        }
        Sx += rowGx;
        Sxy = fmaf(rowGx, dy, Sxy);
        Sy = fmaf(rowG, dy, Sy);
        Syy = fmaf(rowG * dy, dy, Syy);
    }
}

template <int FC, bool DETERMINISTIC>
__global__ void __launch_bounds__(kBwdThreads) k_render_bwd(
    int F, int H, int W, int ntx, const float* __restrict__ geo, const float* __restrict__ feat,
    const float* __restrict__ opacity, const int32_t* __restrict__ gid_sorted,
    const int32_t* __restrict__ tile_offsets, const float* __restrict__ grad_image, const int4* __restrict__ aabb,
    const int32_t* __restrict__ pair_offset, float* __restrict__ pairgrad, int pstride, float* __restrict__ d_xy,
    float* __restrict__ d_conic, float* __restrict__ d_feat) {
    constexpr int SG = BwdCfg<FC>::SG;
    extern __shared__ float4 s_go4[];
    float* s_go = reinterpret_cast<float*>(s_go4);

    const int tile = blockIdx.x;
    const int tile_x = tile % ntx;
    const int tile_y = tile / ntx;
    const int tx0 = tile_x * kTile;
    const int ty0 = tile_y * kTile;
    const int nrow = min(kTile, H - ty0);
    const int ncol = min(kTile, W - tx0);
    const int start = tile_offsets[tile];
    const int end = tile_offsets[tile + 1];
    if (start >= end) return;  // uniform per CTA

    // stage dL/dimage of this tile: s_go[pixel * SG + c]
    const int64_t plane = static_cast<int64_t>(H) * W;
    for (int idx = threadIdx.x; idx < SG * kTilePixels; idx += kBwdThreads) {
        const int c = idx / kTilePixels;
        const int p = idx - c * kTilePixels;
        const int ly = p >> 4;
        const int lx = p & (kTile - 1);
        float v = 0.0f;
        if (c < F && ly < nrow && lx < ncol) {
            v = grad_image[c * plane + static_cast<int64_t>(ty0 + ly) * W + (tx0 + lx)];
        }
        s_go[p * SG + c] = v;
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const bool full = nrow == kTile && ncol == kTile;
    for (int base = start + warp * 32; base < end; base += kBwdThreads) {
        // Only a tile's last batch is partial; its idle lanes run on a neutral
        // entry (zero geometry and features) so the warp stays converged.
        const int j = base + lane;
        const bool active = j < end;
        int g = 0;
        float4 g0 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        float4 g1 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        float fv[FC];
#pragma unroll
        for (int c = 0; c < FC; ++c) fv[c] = 0.0f;
        if (active) {
            g = gid_sorted[j];
            const float4* rec = reinterpret_cast<const float4*>(geo + static_cast<int64_t>(g) * 8);
            g0 = rec[0];
            g1 = rec[1];
            const float op = opacity != nullptr ? opacity[g] : 1.0f;
            const float* fg = feat + static_cast<int64_t>(g) * F;
#pragma unroll
            for (int c = 0; c < FC; ++c) fv[c] = c < F ? fg[c] * op : 0.0f;
        }
        const bool regular = !active || regular_conic_bwd(g0.x, g0.y, g1.y, g1.z, g1.w);
        const bool warp_regular = __all_sync(0xffffffffu, regular);

        float dF[FC];
#pragma unroll
        for (int c = 0; c < FC; ++c) dF[c] = 0.0f;
        float Sx = 0.0f, Sy = 0.0f, Sxx = 0.0f, Sxy = 0.0f, Syy = 0.0f;
        const float A = g0.z, B = g0.w, D = g1.x;

        if (full) {
            const float fx0 = static_cast<float>(tx0), fy0 = static_cast<float>(ty0);
            if (warp_regular) {
                bwd_full_tile<FC, false>(s_go, fx0, fy0, g0.x, g0.y, A, B, D, fv, dF, Sx, Sy, Sxx, Sxy, Syy);
            } else {
                bwd_full_tile<FC, true>(s_go, fx0, fy0, g0.x, g0.y, A, B, D, fv, dF, Sx, Sy, Sxx, Sxy, Syy);
            }
        } else for (int r = 0; r < nrow; ++r) {
            const float dy = static_cast<float>(ty0 + r) - g0.y;
            float rowG = 0.0f, rowGx = 0.0f;
            const float* go_row = s_go + r * kTile * SG;
#pragma unroll 4
            for (int cc = 0; cc < ncol; ++cc) {
                const float dx = static_cast<float>(tx0 + cc) - g0.x;
                const float q = q_scaled(A, B, D, dx, dy);
                const float w = q <= 0.0f ? ex2_ftz(q) : 0.0f;
                const float4* go4 = reinterpret_cast<const float4*>(go_row + cc * SG);
                float go[SG];
#pragma unroll
                for (int v = 0; v < SG / 4; ++v) {
                    const float4 t = go4[v];
                    go[4 * v + 0] = t.x;
                    go[4 * v + 1] = t.y;
                    go[4 * v + 2] = t.z;
                    go[4 * v + 3] = t.w;
                }
                float dLdw = 0.0f;
#pragma unroll
                for (int c = 0; c < FC; ++c) {
                    dLdw = fmaf(go[c], fv[c], dLdw);
                    dF[c] = fmaf(w, go[c], dF[c]);
                }
                const float gw = w * dLdw;
                const float gdx = gw * dx;
                rowGx += gdx;
                Sxx = fmaf(gdx, dx, Sxx);
                rowG += gw;
            }
            Sx += rowGx;
            Sxy = fmaf(rowGx, dy, Sxy);
            Sy = fmaf(rowG, dy, Sy);
            Syy = fmaf(rowG * dy, dy, Syy);
        }
        if (!active) continue;
        // raw conic (a, b, d) sits in g1.yzw
        const float dxy_x = fmaf(g1.y, Sx, g1.z * Sy);
        const float dxy_y = fmaf(g1.z, Sx, g1.w * Sy);
        const float dca = -0.5f * Sxx;
        const float dcb = -Sxy;
        const float dcd = -0.5f * Syy;
        if (DETERMINISTIC) {
            const int4 box = aabb[g];
            const int local = (tile_y - box.y) * (box.z - box.x) + (tile_x - box.x);
            float* row = pairgrad + (static_cast<int64_t>(pair_offset[g]) + local) * pstride;
            if (FC <= 3) {
                float4* row4 = reinterpret_cast<float4*>(row);
                row4[0] = make_float4(dxy_x, dxy_y, dca, dcb);
                row4[1] = make_float4(dcd, dF[0], FC > 1 ? dF[FC > 1 ? 1 : 0] : 0.0f,
                                      FC > 2 ? dF[FC > 2 ? 2 : 0] : 0.0f);
            } else {
                row[0] = dxy_x;
                row[1] = dxy_y;
                row[2] = dca;
                row[3] = dcb;
                row[4] = dcd;
#pragma unroll
                for (int c = 0; c < FC; ++c) {
                    if (c < F) row[5 + c] = dF[c];
                }
            }
        } else {
            atomicAdd(&d_xy[2 * g + 0], dxy_x);
            atomicAdd(&d_xy[2 * g + 1], dxy_y);
            atomicAdd(&d_conic[3 * g + 0], dca);
            atomicAdd(&d_conic[3 * g + 1], dcb);
            atomicAdd(&d_conic[3 * g + 2], dcd);
#pragma unroll
            for (int c = 0; c < FC; ++c) {
                if (c < F) atomicAdd(&d_feat[static_cast<int64_t>(g) * F + c], dF[c]);
            }
        }
    }
}

template <int FC>
__global__ void __launch_bounds__(256) k_reduce_gaussian(int n, int F, const float* __restrict__ pairgrad, int pstride,
                                                         const int32_t* __restrict__ pair_offset,
                                                         const float* __restrict__ feat,
                                                         const float* __restrict__ opacity,
                                                         const float* __restrict__ scale, const float* __restrict__ rot,
                                                         float* __restrict__ d_xy, float* __restrict__ d_conic,
                                                         float* __restrict__ d_feat, float* __restrict__ d_opacity,
                                                         float* __restrict__ d_scale, float* __restrict__ d_rot) {
    const int g = blockIdx.x * 256 + threadIdx.x;
    if (g >= n) return;
    const int beg = pair_offset[g];
    const int end = pair_offset[g + 1];
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f, s4 = 0.0f;
    float dF[FC];
#pragma unroll
    for (int c = 0; c < FC; ++c) dF[c] = 0.0f;
    for (int p = beg; p < end; ++p) {
        const float* row = pairgrad + static_cast<int64_t>(p) * pstride;
        if (FC <= 3) {
            const float4 r0 = reinterpret_cast<const float4*>(row)[0];
            const float4 r1 = reinterpret_cast<const float4*>(row)[1];
            s0 += r0.x;
            s1 += r0.y;
            s2 += r0.z;
            s3 += r0.w;
            s4 += r1.x;
            dF[0] += r1.y;
            if (FC > 1) dF[FC > 1 ? 1 : 0] += r1.z;
            if (FC > 2) dF[FC > 2 ? 2 : 0] += r1.w;
        } else {
            s0 += row[0];
            s1 += row[1];
            s2 += row[2];
            s3 += row[3];
            s4 += row[4];
#pragma unroll
            for (int c = 0; c < FC; ++c) {
                if (c < F) dF[c] += row[5 + c];
            }
        }
    }
    d_xy[2 * g + 0] = s0;
    d_xy[2 * g + 1] = s1;
    d_conic[3 * g + 0] = s2;
    d_conic[3 * g + 1] = s3;
    d_conic[3 * g + 2] = s4;
    const float op = opacity != nullptr ? opacity[g] : 1.0f;
    float dop = 0.0f;
#pragma unroll
    for (int c = 0; c < FC; ++c) {
        if (c < F) {
            const int64_t k = static_cast<int64_t>(g) * F + c;
            d_feat[k] = dF[c] * op;
            dop = fmaf(dF[c], feat[k], dop);
        }
    }
    if (d_opacity != nullptr) d_opacity[g] = dop;
    if (d_scale != nullptr) {
        float dsx, dsy, dr;
        conic_grad_to_scale_rot(scale[2 * g], scale[2 * g + 1], rot[g], s2, s3, s4, dsx, dsy, dr);
        d_scale[2 * g + 0] = dsx;
        d_scale[2 * g + 1] = dsy;
        d_rot[g] = dr;
    }
}

template <int FC>
cudaError_t launch_bwd_fc(int f, int h, int w, int ntx, int num_tiles, const float* geo, const float* feat,
                          const float* opacity, const int32_t* gid_sorted, const int32_t* tile_offsets,
                          const float* grad_image, const int32_t* aabb, const int32_t* pair_offset, float* pairgrad,
                          int pstride, float* d_xy, float* d_conic, float* d_feat, cudaStream_t stream) {
    const int smem = kTilePixels * BwdCfg<FC>::SG * static_cast<int>(sizeof(float));
    if (pairgrad != nullptr) {
        auto kern = k_render_bwd<FC, true>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        kern<<<static_cast<unsigned>(num_tiles), kBwdThreads, smem, stream>>>(
            f, h, w, ntx, geo, feat, opacity, gid_sorted, tile_offsets, grad_image,
            reinterpret_cast<const int4*>(aabb), pair_offset, pairgrad, pstride, d_xy, d_conic, d_feat);
    } else {
        auto kern = k_render_bwd<FC, false>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        kern<<<static_cast<unsigned>(num_tiles), kBwdThreads, smem, stream>>>(
            f, h, w, ntx, geo, feat, opacity, gid_sorted, tile_offsets, grad_image,
            reinterpret_cast<const int4*>(aabb), pair_offset, pairgrad, pstride, d_xy, d_conic, d_feat);
    }
    return cudaGetLastError();
}

template <int FC>
cudaError_t launch_reduce_fc(int n, int f, const float* pairgrad, int pstride, const int32_t* pair_offset,
                             const float* feat, const float* opacity, const float* scale, const float* rot,
                             float* d_xy, float* d_conic, float* d_feat, float* d_opacity, float* d_scale,
                             float* d_rot, cudaStream_t stream) {
    k_reduce_gaussian<FC><<<static_cast<unsigned>(div_up(n, 256)), 256, 0, stream>>>(
        n, f, pairgrad, pstride, pair_offset, feat, opacity, scale, rot, d_xy, d_conic, d_feat, d_opacity, d_scale,
        d_rot);
    return cudaGetLastError();
}

}  // namespace

int backward_pair_stride(int f) { return ((5 + f + 3) / 4) * 4; }

#define OSS_DISPATCH_FC(f, CALL) \
    ((f) <= 1 ? CALL(1) : (f) <= 3 ? CALL(3) : (f) <= 4 ? CALL(4) : (f) <= 8 ? CALL(8) : (f) <= 16 ? CALL(16) : (f) <= 32 ? CALL(32) : CALL(64))

cudaError_t launch_render_backward_tiles(int f, int h, int w, const float* geo, const float* feat,
                                         const float* opacity, const int32_t* gid_sorted,
                                         const int32_t* tile_offsets, const float* grad_image, const int32_t* aabb,
                                         const int32_t* pair_offset, float* pairgrad, int pair_stride, float* d_xy,
                                         float* d_conic, float* d_feat, cudaStream_t stream) {
    const int ntx = static_cast<int>(div_up(w, kTile));
    const int nty = static_cast<int>(div_up(h, kTile));
    const int num_tiles = ntx * nty;
    if (num_tiles == 0) return cudaSuccess;
#define OSS_BWD_CALL(FC)                                                                                     \
    launch_bwd_fc<FC>(f, h, w, ntx, num_tiles, geo, feat, opacity, gid_sorted, tile_offsets, grad_image, aabb, \
                      pair_offset, pairgrad, pair_stride, d_xy, d_conic, d_feat, stream)
    return OSS_DISPATCH_FC(f, OSS_BWD_CALL);
#undef OSS_BWD_CALL
}

cudaError_t launch_reduce_gaussian_grads(int n, int f, const float* pairgrad, int pair_stride,
                                         const int32_t* pair_offset, const float* feat, const float* opacity,
                                         const float* scale, const float* rot, float* d_xy, float* d_conic,
                                         float* d_feat, float* d_opacity, float* d_scale, float* d_rot,
                                         cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
#define OSS_RED_CALL(FC)                                                                                          \
    launch_reduce_fc<FC>(n, f, pairgrad, pair_stride, pair_offset, feat, opacity, scale, rot, d_xy, d_conic, d_feat, \
                         d_opacity, d_scale, d_rot, stream)
    return OSS_DISPATCH_FC(f, OSS_RED_CALL);
#undef OSS_RED_CALL
}

}  // namespace oss
