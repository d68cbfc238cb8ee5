// Per-Gaussian preprocess (conic, tile AABB, pair count, raster record) and the
// per-Gaussian d_conic -> (d_scale, d_rot) chain rule.  One thread per Gaussian,
// fully coalesced SoA loads: these kernels are HBM-bound (20 B in, 32-64 B out).
#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ void write_geo(float* geo, int g, float x, float y, const Conic& k) {
    float4* rec = reinterpret_cast<float4*>(geo + static_cast<int64_t>(g) * 8);
    rec[0] = make_float4(x, y, k.a * kNegHalfLog2e, (2.0f * k.b) * kNegHalfLog2e);
    rec[1] = make_float4(k.d * kNegHalfLog2e, k.a, k.b, k.d);
}

// Packed forward record of Gaussian g: (x, y, A, B | D, feat'[0..F), zeros) in
// prs floats (a multiple of 4), feat' = feat * opacity -- the entry record the
// forward copies into list order, so its staging gathers one record per entry.
__device__ __forceinline__ void write_prec(float* prec, int prs, int g, float x, float y, const Conic& k, int F,
                                           const float* __restrict__ feat, const float* __restrict__ opacity) {
    float4* rec = reinterpret_cast<float4*>(prec + static_cast<int64_t>(g) * prs);
    rec[0] = make_float4(x, y, k.a * kNegHalfLog2e, (2.0f * k.b) * kNegHalfLog2e);
    const float op = opacity != nullptr ? opacity[g] : 1.0f;
    const float* fg = feat + static_cast<int64_t>(g) * F;
    for (int v = 1; v < prs / 4; ++v) {
        float e[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int i = 4 * v + u;  // record float i; feature c = i - 5
            e[u] = i == 4 ? k.d * kNegHalfLog2e : (i - 5 < F ? fg[i - 5] * op : 0.0f);
        }
        rec[v] = make_float4(e[0], e[1], e[2], e[3]);
    }
}

// Frame of Gaussian g: the last b with frame_offsets[b] <= g (offsets non-decreasing).
__device__ __forceinline__ int frame_of(const int32_t* __restrict__ frame_offsets, int frames, int g) {
    int lo = 0, hi = frames - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(frame_offsets + mid) <= g) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// One CTA per kPrepTile Gaussians, one Gaussian per thread.  With block_sums
// non-null the CTA also writes the sum of its pair counts: the reduce half of
// the gid-major pair-offset scan.  With
// tile_count non-null every Gaussian adds one to each tile of its rectangle
// (fire-and-forget reductions into counters kTileCountStride ints apart): the
// per-tile list lengths.  frames > 1: Gaussians [frame_offsets[b],
// frame_offsets[b+1]) are frame b's, whose tiles are rows [b nty, (b+1) nty) of
// the frames stacked; the rectangle moves into those rows.  Two CTAs per SM
// (32 registers): 196 CTAs at config 2 then run as one wave on 148 SMs.
__global__ void __launch_bounds__(kPreprocThreads, 2) k_preprocess(int n, int ntx, int nty, int mode,
                                                              const float2* __restrict__ xy,
                                                              const float2* __restrict__ scale,
                                                              const float* __restrict__ rot,
                                                              float* __restrict__ conic,
                                                              int4* __restrict__ aabb,
                                                              int32_t* __restrict__ count,
                                                              float* __restrict__ geo,
                                                              long long* __restrict__ block_sums,
                                                              int32_t* __restrict__ tile_count, int F, int prs,
                                                              const float* __restrict__ feat,
                                                              const float* __restrict__ opacity,
                                                              float* __restrict__ prec,
                                                              const int32_t* __restrict__ frame_offsets,
                                                              int frames) {
    long long local = 0;
    const int g = blockIdx.x * kPrepTile + threadIdx.x;
    if (g < n) {
        const float2 c = xy[g];
        const float2 s = scale[g];
        const Conic k = conic_from_scale_rot(s.x, s.y, rot[g]);
        conic[3 * g + 0] = k.a;
        conic[3 * g + 1] = k.b;
        conic[3 * g + 2] = k.d;
        int cnt;
        int4 box;
        if (mode == OSS_BIN_FULL) {
            box = make_int4(0, 0, ntx, nty);
            cnt = ntx * nty;
        } else {
            box = tile_aabb(c.x, c.y, s.x, s.y, k, mode_tau(mode), mode_fallback(mode), ntx, nty, cnt);
            if (frames > 1) {
                const int row0 = frame_of(frame_offsets, frames, g) * nty;  // this frame's tile rows
                box.y += row0;
                box.w += row0;
            }
        }
        aabb[g] = box;
        count[g] = cnt;
        local += cnt;
        if (geo != nullptr) write_geo(geo, g, c.x, c.y, k);
        if (prec != nullptr) write_prec(prec, prs, g, c.x, c.y, k, F, feat, opacity);
        if (tile_count != nullptr && cnt > 0) {
            for (int ty = box.y; ty < box.w; ++ty) {
                for (int tx = box.x; tx < box.z; ++tx) {
                    atomicAdd(&tile_count[(static_cast<int64_t>(ty) * ntx + tx) * kTileCountStride], 1);
                }
            }
        }
    }
    if (block_sums != nullptr) {
        __shared__ long long s_part[kPreprocThreads / 32];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) local += __shfl_down_sync(0xffffffffu, local, off);
        if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = local;
        __syncthreads();
        if (threadIdx.x == 0) {
            long long tot = 0;
#pragma unroll
            for (int w = 0; w < kPreprocThreads / 32; ++w) tot += s_part[w];
            block_sums[blockIdx.x] = tot;
        }
    }
}

__global__ void __launch_bounds__(kThreads) k_make_geo(int n, const float2* __restrict__ xy,
                                                        const float* __restrict__ conic, float* __restrict__ geo) {
    const int g = blockIdx.x * kThreads + threadIdx.x;
    if (g >= n) return;
    const float2 c = xy[g];
    Conic k;
    k.a = conic[3 * g + 0];
    k.b = conic[3 * g + 1];
    k.d = conic[3 * g + 2];
    write_geo(geo, g, c.x, c.y, k);
}

__global__ void __launch_bounds__(kThreads) k_conic_to_scale_rot_grad(int n, const float2* __restrict__ scale,
                                                                       const float* __restrict__ rot,
                                                                       const float* __restrict__ d_conic,
                                                                       float2* __restrict__ d_scale,
                                                                       float* __restrict__ d_rot) {
    const int g = blockIdx.x * kThreads + threadIdx.x;
    if (g >= n) return;
    const float2 s = scale[g];
    float dsx, dsy, dr;
    conic_grad_to_scale_rot(s.x, s.y, rot[g], d_conic[3 * g], d_conic[3 * g + 1], d_conic[3 * g + 2], dsx, dsy,
                            dr);
    d_scale[g] = make_float2(dsx, dsy);
    d_rot[g] = dr;
}

}  // namespace

cudaError_t launch_preprocess(int n, int ntx, int nty, int mode, const float* xy, const float* scale,
                              const float* rot, float* conic, int32_t* aabb, int32_t* count, float* geo,
                              long long* block_sums, int32_t* tile_count, int f, const float* feat,
                              const float* opacity, float* prec, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    const int prs = prec != nullptr ? entry_record_floats(f) : 0;
    k_preprocess<<<static_cast<unsigned>(div_up(n, kPrepTile)), kPreprocThreads, 0, stream>>>(
        n, ntx, nty, mode, reinterpret_cast<const float2*>(xy), reinterpret_cast<const float2*>(scale), rot,
        conic, reinterpret_cast<int4*>(aabb), count, geo, block_sums, tile_count, f, prs, feat, opacity, prec,
        nullptr, 1);
    return cudaGetLastError();
}

cudaError_t launch_preprocess_frames(int n, int ntx, int nty, int frames, const int32_t* frame_offsets, int mode,
                                     const float* xy, const float* scale, const float* rot, float* conic,
                                     int32_t* aabb, int32_t* count, float* geo, long long* block_sums,
                                     int32_t* tile_count, int f, const float* feat, const float* opacity,
                                     float* prec, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    const int prs = prec != nullptr ? entry_record_floats(f) : 0;
    k_preprocess<<<static_cast<unsigned>(div_up(n, kPrepTile)), kPreprocThreads, 0, stream>>>(
        n, ntx, nty, mode, reinterpret_cast<const float2*>(xy), reinterpret_cast<const float2*>(scale), rot,
        conic, reinterpret_cast<int4*>(aabb), count, geo, block_sums, tile_count, f, prs, feat, opacity, prec,
        frame_offsets, frames);
    return cudaGetLastError();
}

cudaError_t launch_make_geo(int n, const float* xy, const float* conic, float* geo, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    k_make_geo<<<static_cast<unsigned>(div_up(n, kThreads)), kThreads, 0, stream>>>(
        n, reinterpret_cast<const float2*>(xy), conic, geo);
    return cudaGetLastError();
}

cudaError_t launch_conic_to_scale_rot_grad(int n, const float* scale, const float* rot, const float* d_conic,
                                           float* d_scale, float* d_rot, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    k_conic_to_scale_rot_grad<<<static_cast<unsigned>(div_up(n, kThreads)), kThreads, 0, stream>>>(
        n, reinterpret_cast<const float2*>(scale), rot, d_conic, reinterpret_cast<float2*>(d_scale), d_rot);
    return cudaGetLastError();
}

}  // namespace oss
