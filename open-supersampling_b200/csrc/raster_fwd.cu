// Forward additive tile render (the reference's rasterize_sum,
// rasterizer_fwd.cu:151-322, as plain fp32 SIMT -- the weights are dynamic and
// mostly small, so there is no dense contraction for tensor cores to take).
//
// One CTA per 16x16 tile; each thread owns PX pixels of one column (rows
// ly, ly + 16/PX, ...).  The tile's list is staged in batches into shared
// memory as a geometry float4 (x, y, A, B) plus a [D, feat'...] record; every
// thread walks the batch in list order with broadcast shared loads.  With
//   q' = dy*(D*dy + B*dx) + A*dx*dx   (= -0.5*log2(e) * q)
// the per-Gaussian terms B*dx and A*dx*dx are shared by the thread's PX
// pixels, so a pixel costs 1 FADD + 2 FFMA for q', one MUFU ex2 and F FFMAs.
// With PX even the pixels are processed in pairs on the packed f32x2 pipe
// (FADD2 / FFMA2: two IEEE round-to-nearest operations per instruction, the
// same results as the scalar form), which halves the FP32 issue slots and
// leaves the ex2 (MUFU, 16 per SM per clock) as the bound.
//
// With `records` non-null the staging pass also writes, for every list entry in
// list order, the record the backward reads instead of gathering it again:
// [x, y, A, B | D, feat'(F) | zero padding] (entry_record_floats(F) floats), and
// the entry's gid-major pair slot pair_offset[g] + (local tile index).
//
// The reference zeroes a weight when q is non-finite or negative
// (rasterizer_fwd.cu:245).  A batch whose conics are all finite and
// well-conditioned (det >= 1e-3 * a * d, i.e. axis ratio below ~60) has
// q' <= 0 at every pixel even after fp32 rounding, so it runs without the
// per-pixel test; other batches keep it.
#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

template <int FC>
struct FwdCfg {
    static constexpr int PX = FC <= 4 ? 4 : (FC <= 16 ? 2 : 1);  // pixels per thread
    static constexpr int NT = kTilePixels / PX;                   // threads per tile
    static constexpr int S = ((1 + FC + 3) / 4) * 4;             // floats per [D, feat'] record
    static constexpr int BATCH = S <= 20 ? 256 : (S <= 36 ? 128 : 64);
};

// Well-conditioned conic test shared by both raster kernels (see file comment).
__device__ __forceinline__ bool regular_conic(float x, float y, float a, float b, float d) {
    const bool finite = isfinite(x) && isfinite(y) && isfinite(a) && isfinite(b) && isfinite(d);
    return finite && a > 0.0f && d > 0.0f && (a * d - b * b) >= 1.0e-3f * (a * d);
}

template <int FC, bool CHECK>
__device__ __forceinline__ void fwd_batch(int cnt, const float4* __restrict__ s_geo, const float* __restrict__ s_df,
                                          float fpx, const float (&fpy)[FwdCfg<FC>::PX],
                                          float (&acc)[FwdCfg<FC>::PX][FC]) {
    constexpr int PX = FwdCfg<FC>::PX;
    constexpr int S = FwdCfg<FC>::S;
#pragma unroll 2
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
        const float bdx = g0.w * dx;
        const float adx2 = (g0.z * dx) * dx;
#pragma unroll
        for (int k = 0; k < PX; ++k) {
            const float dy = fpy[k] - g0.y;
            const float q = fmaf(dy, fmaf(r[0], dy, bdx), adx2);
            const float w = CHECK ? (q <= 0.0f ? ex2_ftz(q) : 0.0f) : ex2_ftz(q);
#pragma unroll
            for (int c = 0; c < FC; ++c) acc[k][c] = fmaf(w, r[1 + c], acc[k][c]);
        }
    }
}

// fwd_batch on pixel pairs: acc2[p][c] holds pixels 2p and 2p+1.
template <int FC, bool CHECK>
__device__ __forceinline__ void fwd_batch_pk(int cnt, const float4* __restrict__ s_geo,
                                             const float* __restrict__ s_df, float fpx,
                                             const float2 (&fpy2)[FwdCfg<FC>::PX / 2],
                                             float2 (&acc2)[FwdCfg<FC>::PX / 2][FC]) {
    constexpr int NP = FwdCfg<FC>::PX / 2;
    constexpr int S = FwdCfg<FC>::S;
#pragma unroll 2
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
        const float bdx = g0.w * dx;
        const float adx2 = (g0.z * dx) * dx;
        const float2 ngy = make_float2(-g0.y, -g0.y);  // fpy + (-gy) == fpy - gy exactly
        const float2 D2 = make_float2(r[0], r[0]);
        const float2 b2 = make_float2(bdx, bdx);
        const float2 a2 = make_float2(adx2, adx2);
#pragma unroll
        for (int p = 0; p < NP; ++p) {
            const float2 dy = __fadd2_rn(fpy2[p], ngy);
            const float2 q = __ffma2_rn(dy, __ffma2_rn(D2, dy, b2), a2);
            float2 w;
            if (CHECK) {
                w.x = q.x <= 0.0f ? ex2_ftz(q.x) : 0.0f;
                w.y = q.y <= 0.0f ? ex2_ftz(q.y) : 0.0f;
            } else {
                w.x = ex2_ftz(q.x);
                w.y = ex2_ftz(q.y);
            }
#pragma unroll
            for (int c = 0; c < FC; ++c) acc2[p][c] = __ffma2_rn(w, make_float2(r[1 + c], r[1 + c]), acc2[p][c]);
        }
    }
}

template <int FC>
__global__ void __launch_bounds__(FwdCfg<FC>::NT) k_render_fwd(int F, int H, int W, int ntx,
                                                                const float* __restrict__ geo,
                                                                const float* __restrict__ feat,
                                                                const float* __restrict__ opacity,
                                                                const int32_t* __restrict__ gid_sorted,
                                                                const int32_t* __restrict__ tile_offsets,
                                                                float* __restrict__ image,
                                                                const int4* __restrict__ aabb,
                                                                const int32_t* __restrict__ pair_offset,
                                                                float* __restrict__ records,
                                                                int32_t* __restrict__ slots) {
    constexpr int PX = FwdCfg<FC>::PX;
    constexpr int NT = FwdCfg<FC>::NT;
    constexpr int S = FwdCfg<FC>::S;
    constexpr int BATCH = FwdCfg<FC>::BATCH;
    constexpr int ROWSTEP = kTile / PX;
    __shared__ float4 s_geo[BATCH];
    __shared__ __align__(16) float s_df[BATCH * S];

    const int tile = blockIdx.x;
    const int tx0 = (tile % ntx) * kTile;
    const int ty0 = (tile / ntx) * kTile;
    const int px = tx0 + (threadIdx.x & (kTile - 1));
    const int ly = threadIdx.x >> 4;  // 0 .. ROWSTEP-1
    const float fpx = static_cast<float>(px);
    float fpy[PX];
#pragma unroll
    for (int k = 0; k < PX; ++k) fpy[k] = static_cast<float>(ty0 + ly + k * ROWSTEP);

    constexpr bool PK = PX % 2 == 0;
    constexpr int NP = PK ? PX / 2 : 1;
    float acc[PX][FC];
    float2 acc2[NP][FC];
    float2 fpy2[NP];
#pragma unroll
    for (int k = 0; k < PX; ++k)
#pragma unroll
        for (int c = 0; c < FC; ++c) acc[k][c] = 0.0f;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        fpy2[p] = PK ? make_float2(fpy[2 * p], fpy[2 * p + 1]) : make_float2(0.0f, 0.0f);
#pragma unroll
        for (int c = 0; c < FC; ++c) acc2[p][c] = make_float2(0.0f, 0.0f);
    }

    const int start = tile_offsets[tile];
    const int end = tile_offsets[tile + 1];
    for (int b = start; b < end; b += BATCH) {
        const int cnt = min(BATCH, end - b);
        __syncthreads();  // the previous batch has been consumed
        bool regular = true;
        for (int j = threadIdx.x; j < cnt; j += NT) {
            const int g = gid_sorted[b + j];
            const float4* rec = reinterpret_cast<const float4*>(geo + static_cast<int64_t>(g) * 8);
            const float4 g0 = rec[0];
            const float4 g1 = rec[1];
            s_geo[j] = g0;
            regular = regular && regular_conic(g0.x, g0.y, g1.y, g1.z, g1.w);
            const float op = opacity != nullptr ? opacity[g] : 1.0f;
            float* df = s_df + j * S;
            df[0] = g1.x;
            const float* fg = feat + static_cast<int64_t>(g) * F;
#pragma unroll
            for (int c = 0; c < FC; ++c) df[1 + c] = c < F ? fg[c] * op : 0.0f;
#pragma unroll
            for (int c = 1 + FC; c < S; ++c) df[c] = 0.0f;
            if (records != nullptr) {
                const int e = b + j;
                float4* rec = reinterpret_cast<float4*>(records + static_cast<int64_t>(e) * (4 + S));
                rec[0] = g0;
                const float4* df4 = reinterpret_cast<const float4*>(df);
#pragma unroll
                for (int v = 0; v < S / 4; ++v) rec[1 + v] = df4[v];
                const int4 box = aabb[g];
                slots[e] = pair_offset[g] + (tile / ntx - box.y) * (box.z - box.x) + (tile % ntx - box.x);
            }
        }
        const bool all_regular = __syncthreads_and(regular ? 1 : 0) != 0;
        if constexpr (PK) {
            if (all_regular) {
                fwd_batch_pk<FC, false>(cnt, s_geo, s_df, fpx, fpy2, acc2);
            } else {
                fwd_batch_pk<FC, true>(cnt, s_geo, s_df, fpx, fpy2, acc2);
            }
        } else {
            if (all_regular) {
                fwd_batch<FC, false>(cnt, s_geo, s_df, fpx, fpy, acc);
            } else {
                fwd_batch<FC, true>(cnt, s_geo, s_df, fpx, fpy, acc);
            }
        }
    }
    if constexpr (PK) {
#pragma unroll
        for (int p = 0; p < NP; ++p)
#pragma unroll
            for (int c = 0; c < FC; ++c) {
                acc[2 * p][c] = acc2[p][c].x;
                acc[2 * p + 1][c] = acc2[p][c].y;
            }
    }
    if (px < W) {
        const int64_t plane = static_cast<int64_t>(H) * W;
#pragma unroll
        for (int k = 0; k < PX; ++k) {
            const int py = ty0 + ly + k * ROWSTEP;
            if (py < H) {
                const int64_t pix = static_cast<int64_t>(py) * W + px;
#pragma unroll
                for (int c = 0; c < FC; ++c) {
                    if (c < F) image[c * plane + pix] = acc[k][c];
                }
            }
        }
    }
}

template <int FC>
cudaError_t launch_fwd_fc(int f, int h, int w, int ntx, int num_tiles, const float* geo, const float* feat,
                          const float* opacity, const int32_t* gid_sorted, const int32_t* tile_offsets, float* image,
                          const int32_t* aabb, const int32_t* pair_offset, float* records, int32_t* slots,
                          cudaStream_t stream) {
    k_render_fwd<FC><<<static_cast<unsigned>(num_tiles), FwdCfg<FC>::NT, 0, stream>>>(
        f, h, w, ntx, geo, feat, opacity, gid_sorted, tile_offsets, image, reinterpret_cast<const int4*>(aabb),
        pair_offset, records, slots);
    return cudaGetLastError();
}

template <int FC>
constexpr int record_floats_fc() {
    return 4 + FwdCfg<FC>::S;
}

}  // namespace

int entry_record_floats(int f) {
    if (f <= 1) return record_floats_fc<1>();
    if (f <= 3) return record_floats_fc<3>();
    if (f <= 4) return record_floats_fc<4>();
    if (f <= 8) return record_floats_fc<8>();
    if (f <= 16) return record_floats_fc<16>();
    if (f <= 32) return record_floats_fc<32>();
    return record_floats_fc<64>();
}

cudaError_t launch_render_forward(int f, int h, int w, const float* geo, const float* feat, const float* opacity,
                                  const int32_t* gid_sorted, const int32_t* tile_offsets, float* image,
                                  const int32_t* aabb, const int32_t* pair_offset, float* records, int32_t* slots,
                                  cudaStream_t stream) {
    const int ntx = static_cast<int>(div_up(w, kTile));
    const int nty = static_cast<int>(div_up(h, kTile));
    const int num_tiles = ntx * nty;
    if (num_tiles == 0 || f == 0) return cudaSuccess;
#define OSS_FWD_CALL(FC)                                                                                           \
    launch_fwd_fc<FC>(f, h, w, ntx, num_tiles, geo, feat, opacity, gid_sorted, tile_offsets, image, aabb,          \
                      pair_offset, records, slots, stream)
    if (f <= 1) return OSS_FWD_CALL(1);
    if (f <= 3) return OSS_FWD_CALL(3);
    if (f <= 4) return OSS_FWD_CALL(4);
    if (f <= 8) return OSS_FWD_CALL(8);
    if (f <= 16) return OSS_FWD_CALL(16);
    if (f <= 32) return OSS_FWD_CALL(32);
    return OSS_FWD_CALL(64);
#undef OSS_FWD_CALL
}

}  // namespace oss
