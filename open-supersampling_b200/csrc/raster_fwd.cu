// Forward additive tile render (the reference's rasterize_sum,
// rasterizer_fwd.cu:151-322, as plain fp32 SIMT -- the weights are dynamic and
// mostly small, so there is no dense contraction for tensor cores to take).
//
// One CTA per 16x16 tile, one thread per pixel.  The tile's list is staged in
// batches into shared memory (geometry float4 + [D, feat'...] record); every
// thread then walks the batch in list order with broadcast shared loads:
//   q' = dx*(A*dx + B*dy) + D*dy*dy   (= -0.5*log2(e) * q)
//   w  = 2^q'  (MUFU ex2), skipped unless q' <= 0   (the reference's
//        isfinite(q) && q >= 0 test, rasterizer_fwd.cu:245)
//   acc[c] += w * feat'[c]
// Per evaluation: 2 LDS.128 (broadcast), ~9 FP32 ops + F FMAs, 1 MUFU.
#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

constexpr int kFwdThreads = kTilePixels;  // 256

template <int FC>
struct FwdCfg {
    static constexpr int S = ((1 + FC + 3) / 4) * 4;  // floats per [D, feat'] record
    static constexpr int BATCH = S <= 20 ? 256 : (S <= 36 ? 128 : 64);
};

template <int FC>
__global__ void __launch_bounds__(kFwdThreads) k_render_fwd(int F, int H, int W, int ntx,
                                                             const float* __restrict__ geo,
                                                             const float* __restrict__ feat,
                                                             const float* __restrict__ opacity,
                                                             const int32_t* __restrict__ gid_sorted,
                                                             const int32_t* __restrict__ tile_offsets,
                                                             float* __restrict__ image) {
    constexpr int S = FwdCfg<FC>::S;
    constexpr int BATCH = FwdCfg<FC>::BATCH;
    __shared__ float4 s_geo[BATCH];
    __shared__ __align__(16) float s_df[BATCH * S];

    const int tile = blockIdx.x;
    const int tx0 = (tile % ntx) * kTile;
    const int ty0 = (tile / ntx) * kTile;
    const int px = tx0 + (threadIdx.x & (kTile - 1));
    const int py = ty0 + (threadIdx.x >> 4);
    const float fpx = static_cast<float>(px);
    const float fpy = static_cast<float>(py);

    float acc[FC];
#pragma unroll
    for (int c = 0; c < FC; ++c) acc[c] = 0.0f;

    const int start = tile_offsets[tile];
    const int end = tile_offsets[tile + 1];
    for (int b = start; b < end; b += BATCH) {
        const int cnt = min(BATCH, end - b);
        __syncthreads();  // the previous batch has been consumed
        for (int j = threadIdx.x; j < cnt; j += kFwdThreads) {
            const int g = gid_sorted[b + j];
            const float4* rec = reinterpret_cast<const float4*>(geo + static_cast<int64_t>(g) * 8);
            s_geo[j] = rec[0];
            const float op = opacity != nullptr ? opacity[g] : 1.0f;
            float* df = s_df + j * S;
            df[0] = rec[1].x;
            const float* fg = feat + static_cast<int64_t>(g) * F;
#pragma unroll
            for (int c = 0; c < FC; ++c) df[1 + c] = c < F ? fg[c] * op : 0.0f;
        }
        __syncthreads();
#pragma unroll 4
        for (int j = 0; j < cnt; ++j) {
            const float4 g0 = s_geo[j];
            const float4* df4 = reinterpret_cast<const float4*>(s_df + j * S);
            float r[S];
#pragma unroll
            for (int v = 0; v < S / 4; ++v) {
                const float4 t = df4[v];
                r[4 * v + 0] = t.x;
                r[4 * v + 1] = t.y;
                r[4 * v + 2] = t.z;
                r[4 * v + 3] = t.w;
            }
            const float dx = fpx - g0.x;
            const float dy = fpy - g0.y;
            const float q = q_scaled(g0.z, g0.w, r[0], dx, dy);
            const float w = q <= 0.0f ? ex2_ftz(q) : 0.0f;
#pragma unroll
            for (int c = 0; c < FC; ++c) acc[c] = fmaf(w, r[1 + c], acc[c]);
        }
    }
    if (px < W && py < H) {
        const int64_t plane = static_cast<int64_t>(H) * W;
        const int64_t pix = static_cast<int64_t>(py) * W + px;
#pragma unroll
        for (int c = 0; c < FC; ++c) {
            if (c < F) image[c * plane + pix] = acc[c];
        }
    }
}

template <int FC>
cudaError_t launch_fwd_fc(int f, int h, int w, int ntx, int num_tiles, const float* geo, const float* feat,
                          const float* opacity, const int32_t* gid_sorted, const int32_t* tile_offsets, float* image,
                          cudaStream_t stream) {
    k_render_fwd<FC><<<static_cast<unsigned>(num_tiles), kFwdThreads, 0, stream>>>(f, h, w, ntx, geo, feat, opacity,
                                                                                  gid_sorted, tile_offsets, image);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_render_forward(int f, int h, int w, const float* geo, const float* feat, const float* opacity,
                                  const int32_t* gid_sorted, const int32_t* tile_offsets, float* image,
                                  cudaStream_t stream) {
    const int ntx = static_cast<int>(div_up(w, kTile));
    const int nty = static_cast<int>(div_up(h, kTile));
    const int num_tiles = ntx * nty;
    if (num_tiles == 0 || f == 0) return cudaSuccess;
    if (f <= 1) return launch_fwd_fc<1>(f, h, w, ntx, num_tiles, geo, feat, opacity, gid_sorted, tile_offsets, image, stream);
    if (f <= 3) return launch_fwd_fc<3>(f, h, w, ntx, num_tiles, geo, feat, opacity, gid_sorted, tile_offsets, image, stream);
    if (f <= 4) return launch_fwd_fc<4>(f, h, w, ntx, num_tiles, geo, feat, opacity, gid_sorted, tile_offsets, image, stream);
    if (f <= 8) return launch_fwd_fc<8>(f, h, w, ntx, num_tiles, geo, feat, opacity, gid_sorted, tile_offsets, image, stream);
    if (f <= 16) return launch_fwd_fc<16>(f, h, w, ntx, num_tiles, geo, feat, opacity, gid_sorted, tile_offsets, image, stream);
    if (f <= 32) return launch_fwd_fc<32>(f, h, w, ntx, num_tiles, geo, feat, opacity, gid_sorted, tile_offsets, image, stream);
    return launch_fwd_fc<64>(f, h, w, ntx, num_tiles, geo, feat, opacity, gid_sorted, tile_offsets, image, stream);
}

}  // namespace oss
