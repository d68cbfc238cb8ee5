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

// Exclusive scans of two sequences at once by one CTA of kPreprocThreads
// threads: a[i] = ca[i * sa] (int32 counters, scanned into oa[0..ma)) and
// cb[0..mb) (int64, scanned in place).  Passes of 4 contiguous values per
// thread, all loads of a pass in flight together, read through L2 (other CTAs
// wrote them).  Returns both totals.
__device__ void cta_scan_two(const int32_t* __restrict__ ca, int sa, int64_t ma, int32_t* __restrict__ oa,
                             long long* __restrict__ cb, int64_t mb, long long& tot_a, long long& tot_b) {
    constexpr int NT = kPreprocThreads;
    constexpr int kPer = 4;  // keeps the kernel within 32 registers (two 1024-thread CTAs per SM)
    constexpr int kWarps = NT / 32;
    __shared__ long long s_wa[kWarps];
    __shared__ long long s_wb[kWarps];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    long long carry_a = 0, carry_b = 0;
    const int64_t m = ma > mb ? ma : mb;
    for (int64_t base = 0; base < m; base += static_cast<int64_t>(NT) * kPer) {
        const int64_t lo = base + static_cast<int64_t>(threadIdx.x) * kPer;
        int32_t va[kPer];
        long long vb[kPer];
        long long sum_a = 0, sum_b = 0;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            va[k] = lo + k < ma ? __ldcg(ca + (lo + k) * sa) : 0;
            vb[k] = lo + k < mb ? __ldcg(cb + lo + k) : 0;
        }
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            sum_a += va[k];
            sum_b += vb[k];
        }
        // inclusive warp scans, then the warps' totals
        long long xa = sum_a, xb = sum_b;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const long long ya = __shfl_up_sync(0xffffffffu, xa, off);
            const long long yb = __shfl_up_sync(0xffffffffu, xb, off);
            if (lane >= off) {
                xa += ya;
                xb += yb;
            }
        }
        if (lane == 31) {
            s_wa[warp] = xa;
            s_wb[warp] = xb;
        }
        __syncthreads();
        long long pa = 0, pb = 0, ta = 0, tb = 0;
#pragma unroll 8
        for (int w = 0; w < kWarps; ++w) {
            const long long wa = s_wa[w], wb = s_wb[w];
            pa += w < warp ? wa : 0;
            pb += w < warp ? wb : 0;
            ta += wa;
            tb += wb;
        }
        __syncthreads();  // s_wa / s_wb are rewritten by the next pass
        long long ra = carry_a + pa + xa - sum_a;
        long long rb = carry_b + pb + xb - sum_b;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            if (lo + k < ma) oa[lo + k] = static_cast<int32_t>(ra);
            if (lo + k < mb) cb[lo + k] = rb;
            ra += va[k];
            rb += vb[k];
        }
        carry_a += ta;
        carry_b += tb;
    }
    tot_a = carry_a;
    tot_b = carry_b;
}

// Outputs of the fused preprocess beyond those of the plain one.
struct FusedScan {
    long long* warp_sums;     // [ceil(n / 32)]: pair-count sums, then (last CTA) exclusive bases
    int32_t* tile_offsets;    // [num_tiles + 1]
    int32_t* pair_offset;     // pair_offset[n] = total
    int64_t* total_pairs;
    unsigned int* arrivals;   // CTA arrival counter, zero on entry
};

// One CTA per kPrepTile Gaussians, one Gaussian per thread.  With block_sums
// non-null the CTA also writes the sum of its pair counts: the reduce half of
// the gid-major pair-offset scan.  With
// tile_count non-null every Gaussian adds one to each tile of its rectangle
// (fire-and-forget reductions into counters kTileCountStride ints apart): the
// per-tile list lengths.  FUSED: each warp writes the sum of its 32 pair counts
// instead, and the last CTA to arrive (every CTA fences its writes and
// reductions, then counts itself in) scans the tile counts and the warp sums;
// nothing waits.
template <bool FUSED>
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
                                                              float* __restrict__ prec, FusedScan fs) {
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
        }
        aabb[g] = box;
        if (!FUSED) count[g] = cnt;
        local += cnt;
        if (geo != nullptr) write_geo(geo, g, c.x, c.y, k);
        if (prec != nullptr) write_prec(prec, prs, g, c.x, c.y, k, F, feat, opacity);
        if (tile_count != nullptr && cnt > 0) {
            for (int ty = box.y; ty < box.w; ++ty) {
                for (int tx = box.x; tx < box.z; ++tx) {
                    atomicAdd(&tile_count[static_cast<int64_t>(ty * ntx + tx) * kTileCountStride], 1);
                }
            }
        }
    }
    if (FUSED) {
        __shared__ int s_last;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) local += __shfl_down_sync(0xffffffffu, local, off);
        const int w0 = g & ~31;
        if ((threadIdx.x & 31) == 0 && w0 < n) fs.warp_sums[w0 >> 5] = local;
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) s_last = atomicAdd(fs.arrivals, 1u) == gridDim.x - 1 ? 1 : 0;
        __syncthreads();
        if (s_last == 0) return;
        __threadfence();
        const int64_t num_tiles = static_cast<int64_t>(ntx) * nty;
        long long tot_tiles, tot_pairs;
        cta_scan_two(tile_count, kTileCountStride, num_tiles, fs.tile_offsets, fs.warp_sums, div_up(n, 32),
                     tot_tiles, tot_pairs);
        if (threadIdx.x == 0) {
            fs.tile_offsets[num_tiles] = static_cast<int32_t>(tot_tiles);
            fs.pair_offset[n] = static_cast<int32_t>(tot_pairs);
            *fs.total_pairs = static_cast<int64_t>(tot_pairs);
        }
    } else if (block_sums != nullptr) {
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
    k_preprocess<false><<<static_cast<unsigned>(div_up(n, kPrepTile)), kPreprocThreads, 0, stream>>>(
        n, ntx, nty, mode, reinterpret_cast<const float2*>(xy), reinterpret_cast<const float2*>(scale), rot,
        conic, reinterpret_cast<int4*>(aabb), count, geo, block_sums, tile_count, f, prs, feat, opacity, prec,
        FusedScan{});
    return cudaGetLastError();
}

int64_t preprocess_fused_warps(int64_t n) { return div_up(n, 32); }

cudaError_t launch_preprocess_fused(int n, int ntx, int nty, int mode, const float* xy, const float* scale,
                                    const float* rot, float* conic, int32_t* aabb, int32_t* pair_offset, float* geo,
                                    int32_t* tile_count, int32_t* tile_offsets, long long* warp_sums,
                                    int64_t* total_pairs, int f, const float* feat, const float* opacity,
                                    float* prec, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    const int prs = prec != nullptr ? entry_record_floats(f) : 0;
    const int64_t num_tiles = static_cast<int64_t>(ntx) * nty;
    FusedScan fs{warp_sums, tile_offsets, pair_offset, total_pairs,
                 reinterpret_cast<unsigned int*>(tile_count + num_tiles * kTileCountStride)};
    k_preprocess<true><<<static_cast<unsigned>(div_up(n, kPrepTile)), kPreprocThreads, 0, stream>>>(
        n, ntx, nty, mode, reinterpret_cast<const float2*>(xy), reinterpret_cast<const float2*>(scale), rot,
        conic, reinterpret_cast<int4*>(aabb), nullptr, geo, nullptr, tile_count, f, prs, feat, opacity, prec, fs);
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
