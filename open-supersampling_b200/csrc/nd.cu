// Splat of the v7 N-D time-slice rasterizer (oss/sr/v7/nd_rasterizer.py:107-165,
// _evaluate_2d_gaussian_at_pixels): after the time conditioning, each Gaussian is
// a 2D Gaussian with a mean, an inverse covariance (a, b, d), an amplitude
// (opacity x time weight x Mip factors) and R features, evaluated at pixel
// centres (j + 0.5, i + 0.5) inside its own cull box [x0, x1) x [y0, y1) --
// 3 sqrt(largest eigenvalue) around the mean, the reference's loop bound -- and
// zero outside it.  Its sum is
//   out[c](i, j) = sum_g feat[g][c] * amp[g] * exp(-q_g / 2), (i, j) in box_g.
//
// The lists come from the same tile binning as the additive render: a Gaussian
// covers the tiles its box overlaps.  The preprocess here writes the packed
// record (x - 0.5, y - 0.5, A, B | D, feat * amp) of the additive forward, so
// dx = j - (x - 0.5) equals the reference's (j + 0.5) - x exactly, and q' =
// dx (A dx + B dy) + D dy^2 with (A, B, D) = (a, 2b, d) * (-log2(e) / 2); the
// per-pixel test against the box is the only difference from the additive
// kernels.  The backward writes the additive backward's per-pair rows (Sx, Sy,
// d_conic, dF) over the box's pixels of each tile, so the per-Gaussian reduce of
// the additive path turns them into d_xy, d_conic, d_feat and d_amp.
#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

constexpr int kNdThreads = 256;  // one pixel per thread, one CTA per tile
constexpr int kNdBatch = 64;     // list entries staged per batch

template <int FC>
struct NdCfg {
    static constexpr int S = ((1 + FC + 3) / 4) * 4;  // [D, feat * amp] floats, the additive record's tail
    static constexpr int RS = 4 + S;                  // record floats
};

__global__ void __launch_bounds__(kPreprocThreads) k_nd_preprocess(
    int n, int ntx, int nty, const float2* __restrict__ xy, const float* __restrict__ conic,
    const int4* __restrict__ box, int F, int prs, const float* __restrict__ feat, const float* __restrict__ amp,
    int4* __restrict__ aabb, int32_t* __restrict__ count, float* __restrict__ geo, float* __restrict__ prec,
    long long* __restrict__ block_sums, int32_t* __restrict__ tile_count) {
    long long local = 0;
    const int g = blockIdx.x * kPrepTile + threadIdx.x;
    if (g < n) {
        const float2 c = xy[g];
        const float x = __fsub_rn(c.x, 0.5f), y = __fsub_rn(c.y, 0.5f);
        const float a = conic[3 * g + 0], b = conic[3 * g + 1], d = conic[3 * g + 2];
        const int4 bx = box[g];  // (x0, y0, x1, y1) in pixels
        int4 t = make_int4(0, 0, 0, 0);
        int cnt = 0;
        if (bx.z > bx.x && bx.w > bx.y) {
            t = make_int4(bx.x / kTile, bx.y / kTile, min(ntx, (bx.z + kTile - 1) / kTile),
                          min(nty, (bx.w + kTile - 1) / kTile));
            cnt = (t.z - t.x) * (t.w - t.y);
        }
        aabb[g] = t;
        count[g] = cnt;
        local = cnt;
        const float A = a * kNegHalfLog2e, B = (2.0f * b) * kNegHalfLog2e, D = d * kNegHalfLog2e;
        float4* gr = reinterpret_cast<float4*>(geo + static_cast<int64_t>(g) * 8);
        gr[0] = make_float4(x, y, A, B);
        gr[1] = make_float4(D, a, b, d);
        float4* rec = reinterpret_cast<float4*>(prec + static_cast<int64_t>(g) * prs);
        rec[0] = make_float4(x, y, A, B);
        const float op = amp[g];
        for (int v = 1; v < prs / 4; ++v) {
            float e[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = 4 * v + u;
                e[u] = i == 4 ? D : (i - 5 < F ? feat[static_cast<int64_t>(g) * F + (i - 5)] * op : 0.0f);
            }
            rec[v] = make_float4(e[0], e[1], e[2], e[3]);
        }
        for (int ty = t.y; ty < t.w; ++ty) {
            for (int tx = t.x; tx < t.z; ++tx) {
                atomicAdd(&tile_count[static_cast<int64_t>(ty * ntx + tx) * kTileCountStride], 1);
            }
        }
    }
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

template <int FC>
__global__ void __launch_bounds__(kNdThreads) k_nd_fwd(int F, int H, int W, int ntx, const float* __restrict__ prec,
                                                        const int4* __restrict__ box,
                                                        const int32_t* __restrict__ gid_sorted,
                                                        const int32_t* __restrict__ tile_offsets,
                                                        float* __restrict__ image) {
    constexpr int RS = NdCfg<FC>::RS;
    __shared__ float4 s_rec[kNdBatch][RS / 4];
    __shared__ int4 s_box[kNdBatch];
    const int tile = blockIdx.x;
    const int tx0 = (tile % ntx) * kTile, ty0 = (tile / ntx) * kTile;
    const int px = tx0 + (threadIdx.x & (kTile - 1)), py = ty0 + (threadIdx.x >> 4);
    const float fpx = static_cast<float>(px), fpy = static_cast<float>(py);
    float acc[FC];
#pragma unroll
    for (int c = 0; c < FC; ++c) acc[c] = 0.0f;
    const int beg = tile_offsets[tile], end = tile_offsets[tile + 1];
    for (int b = beg; b < end; b += kNdBatch) {
        const int cnt = min(kNdBatch, end - b);
        __syncthreads();
        for (int e = threadIdx.x; e < cnt * (RS / 4); e += kNdThreads) {
            const int j = e / (RS / 4), v = e - j * (RS / 4);
            const int g = gid_sorted[b + j];
            s_rec[j][v] = reinterpret_cast<const float4*>(prec + static_cast<int64_t>(g) * RS)[v];
            if (v == 0) s_box[j] = box[g];
        }
        __syncthreads();
        for (int j = 0; j < cnt; ++j) {
            const int4 bx = s_box[j];
            if (px < bx.x || px >= bx.z || py < bx.y || py >= bx.w) continue;
            const float4 g0 = s_rec[j][0];
            const float* r = reinterpret_cast<const float*>(&s_rec[j][1]);
            const float dx = fpx - g0.x, dy = fpy - g0.y;
            const float q = fmaf(dx, fmaf(g0.z, dx, g0.w * dy), (r[0] * dy) * dy);
            const float wgt = ex2_ftz(q);
#pragma unroll
            for (int c = 0; c < FC; ++c) acc[c] = fmaf(wgt, r[1 + c], acc[c]);
        }
    }
    if (px >= W || py >= H) return;
    const int64_t plane = static_cast<int64_t>(H) * W, pix = static_cast<int64_t>(py) * W + px;
#pragma unroll
    for (int c = 0; c < FC; ++c) {
        if (c < F) image[c * plane + pix] = acc[c];
    }
}

// Per-pair sums over the pixels of tile t inside the entry's box.  The tile's
// dL/dimage sits in shared memory; the CTA's warps take list entries from a
// shared counter, and a warp's lanes share out the pixels of the entry's box
// clipped to the tile and the image (w x h of them, lane k taking pixels k,
// k + 32, ... in row order), so small boxes keep most lanes busy.  One warp
// reduce-scatter per entry leaves the 5 + F sums in the lanes that write them,
// and a tile with few entries still keeps every warp busy.  Rows (Sx, Sy,
// d_conic, dF) land at the entry's gid-major pair slot, as in the additive backward, so
// k_reduce_gaussian finishes the per-Gaussian gradients.
template <int FC>
struct NdSumWidth {  // power-of-two width holding the 5 + FC sums; 0 above a warp's 32
    static constexpr int n = 5 + FC;
    static constexpr int value = n <= 8 ? 8 : n <= 16 ? 16 : n <= 32 ? 32 : 0;
};

template <int FC>
__global__ void __launch_bounds__(kNdThreads) k_nd_bwd(int F, int H, int W, int ntx, const float* __restrict__ prec,
                                                        const int4* __restrict__ box,
                                                        const int32_t* __restrict__ gid_sorted,
                                                        const int32_t* __restrict__ tile_offsets,
                                                        const int4* __restrict__ aabb,
                                                        const int32_t* __restrict__ pair_offset,
                                                        const float* __restrict__ grad_image,
                                                        float* __restrict__ pairgrad, int pstride) {
    constexpr int RS = NdCfg<FC>::RS;
    static_assert(kNdThreads == kTilePixels, "one thread per pixel for staging");
    // dL/dimage of the tile, row-major with column bit 3 flipped on rows 2 and 3 (mod 4):
    // rows two apart otherwise share banks, and a warp's lanes span several box rows
    __shared__ float s_go[FC][kTilePixels];
    __shared__ int s_next;
    const int lane = static_cast<int>(threadIdx.x) & 31;
    const int tile = blockIdx.x;
    const int tile_x = tile % ntx, tile_y = tile / ntx;
    const int tx0 = tile_x * kTile, ty0 = tile_y * kTile;
    const int64_t plane = static_cast<int64_t>(H) * W;
    {
        const int px = tx0 + (static_cast<int>(threadIdx.x) & (kTile - 1)), py = ty0 + (static_cast<int>(threadIdx.x) >> 4);
        const bool in = px < W && py < H;
        const int ly = static_cast<int>(threadIdx.x) >> 4, lx = static_cast<int>(threadIdx.x) & (kTile - 1);
        const int at = ly * kTile + (lx ^ ((ly & 2) << 2));
#pragma unroll
        for (int c = 0; c < FC; ++c) {
            s_go[c][at] = in && c < F ? grad_image[c * plane + static_cast<int64_t>(py) * W + px] : 0.0f;
        }
    }
    if (threadIdx.x == 0) s_next = 0;
    __syncthreads();
    const int beg = tile_offsets[tile], cnt = tile_offsets[tile + 1] - beg;
    for (;;) {
        int j = 0;
        if (lane == 0) j = atomicAdd(&s_next, 1);
        j = __shfl_sync(0xffffffffu, j, 0);
        if (j >= cnt) break;
        const int g = gid_sorted[beg + j];
        const int4 bx = box[g];
        const int x_lo = max(bx.x, tx0) - tx0, x_hi = min(min(bx.z, tx0 + kTile), W) - tx0;
        const int y_lo = max(bx.y, ty0) - ty0, y_hi = min(min(bx.w, ty0 + kTile), H) - ty0;
        const int bw = x_hi - x_lo, npix = bw > 0 && y_hi > y_lo ? bw * (y_hi - y_lo) : 0;
        float Sx = 0.0f, Sy = 0.0f, Sxx = 0.0f, Sxy = 0.0f, Syy = 0.0f, dF[FC];
#pragma unroll
        for (int c = 0; c < FC; ++c) dF[c] = 0.0f;
        if (npix > 0) {
            const float4* rec = reinterpret_cast<const float4*>(prec + static_cast<int64_t>(g) * RS);
            const float4 g0 = rec[0];
            float r[RS - 4];
#pragma unroll
            for (int v = 0; v < (RS - 4) / 4; ++v) {
                const float4 t = rec[1 + v];
                r[4 * v + 0] = t.x;
                r[4 * v + 1] = t.y;
                r[4 * v + 2] = t.z;
                r[4 * v + 3] = t.w;
            }
            // row of pixel i of the box: floor((i + 1/2) / w) is exact in fp32 here (i < 256,
            // w <= 16: the quotient stays at least 1 / 32 from an integer, the rounding below 1e-4)
            const float inv_w = 1.0f / static_cast<float>(bw);
            for (int i = lane; i < npix; i += 32) {
                const int iy = static_cast<int>((static_cast<float>(i) + 0.5f) * inv_w);
                const int lx = x_lo + (i - iy * bw), ly = y_lo + iy;
                const int p = ly * kTile + (lx ^ ((ly & 2) << 2));
                const float dx = static_cast<float>(tx0 + lx) - g0.x;
                const float dy = static_cast<float>(ty0 + ly) - g0.y;
                const float q = fmaf(dx, fmaf(g0.z, dx, g0.w * dy), (r[0] * dy) * dy);
                const float wgt = ex2_ftz(q);
                float dLdw = 0.0f;
#pragma unroll
                for (int c = 0; c < FC; ++c) {
                    const float go = s_go[c][p];
                    dLdw = fmaf(go, r[1 + c], dLdw);
                    dF[c] = fmaf(wgt, go, dF[c]);
                }
                const float gw = wgt * dLdw;
                Sx = fmaf(gw, dx, Sx);
                Sy = fmaf(gw, dy, Sy);
                Sxx = fmaf(gw * dx, dx, Sxx);
                Sxy = fmaf(gw * dx, dy, Sxy);
                Syy = fmaf(gw * dy, dy, Syy);
            }
        }
        const int4 tb = aabb[g];
        const int slot = pair_offset[g] + (tile_y - tb.y) * (tb.z - tb.x) + (tile_x - tb.x);
        float* row = pairgrad + static_cast<int64_t>(slot) * pstride;
        // row = (Sx, Sy, -Sxx / 2, -Sxy, -Syy / 2, dF): the scalings are exact, so they
        // go in before the sums
        constexpr int V = NdSumWidth<FC>::value;
        if constexpr (V > 0) {
            float v[V];
            v[0] = Sx;
            v[1] = Sy;
            v[2] = -0.5f * Sxx;
            v[3] = -Sxy;
            v[4] = -0.5f * Syy;
#pragma unroll
            for (int i = 5; i < V; ++i) v[i] = i - 5 < FC ? dF[i - 5] : 0.0f;
            const float t = warp_reduce_scatter<V>(v);  // lane l: the total of v[l >> kShift]
            constexpr int kShift = V == 8 ? 2 : V == 16 ? 1 : 0;
            const int idx = lane >> kShift;
            if ((lane & ((1 << kShift) - 1)) == 0 && idx < 5 + F) row[idx] = t;
        } else {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                Sx += __shfl_xor_sync(0xffffffffu, Sx, o);
                Sy += __shfl_xor_sync(0xffffffffu, Sy, o);
                Sxx += __shfl_xor_sync(0xffffffffu, Sxx, o);
                Sxy += __shfl_xor_sync(0xffffffffu, Sxy, o);
                Syy += __shfl_xor_sync(0xffffffffu, Syy, o);
#pragma unroll
                for (int c = 0; c < FC; ++c) dF[c] += __shfl_xor_sync(0xffffffffu, dF[c], o);
            }
            if (lane == 0) {
                row[0] = Sx;
                row[1] = Sy;
                row[2] = -0.5f * Sxx;
                row[3] = -Sxy;
                row[4] = -0.5f * Syy;
#pragma unroll
                for (int c = 0; c < FC; ++c) {
                    if (c < F) row[5 + c] = dF[c];
                }
            }
        }
    }
}

// ---- per-Gaussian time conditioning (nd_rasterizer.py:53-239) -------------
// One thread per Gaussian: Mip 3D smoothing, conditioning on t = t_query (mean
// shift, Schur complement, marginal density of t_query), Mip 2D filter, then the
// splat inputs: mean, inverse covariance (a, b, d), amplitude and the cull box.
// The backward recomputes these steps and applies their chain rule by hand.
struct NdPrep {
    float S[9];              // smoothed 3x3 covariance
    float f3, opf;           // opacity factor, smoothed opacity
    float vtt, k, dt;        // clamped V_tt, dt / V_tt, t_query - mean_t
    float c[4];              // conditional 2x2 covariance
    float wt, W;             // density of t_query, weight before the 2D filter
    float P[4], f2, W2;      // filtered 2x2 covariance, its factor, weight after it
    float D;                 // det P
    float mx, my;            // conditional mean
};

__device__ __forceinline__ float det3(const float* M) {
    const float c0 = __fsub_rn(__fmul_rn(M[4], M[8]), __fmul_rn(M[5], M[7]));
    const float c1 = __fsub_rn(__fmul_rn(M[3], M[8]), __fmul_rn(M[5], M[6]));
    const float c2 = __fsub_rn(__fmul_rn(M[3], M[7]), __fmul_rn(M[4], M[6]));
    return __fadd_rn(__fsub_rn(__fmul_rn(M[0], c0), __fmul_rn(M[1], c1)), __fmul_rn(M[2], c2));
}

// cofactor matrix (d det / d M)
__device__ __forceinline__ void cof3(const float* M, float* out) {
    out[0] = M[4] * M[8] - M[5] * M[7];
    out[1] = -(M[3] * M[8] - M[5] * M[6]);
    out[2] = M[3] * M[7] - M[4] * M[6];
    out[3] = -(M[1] * M[8] - M[2] * M[7]);
    out[4] = M[0] * M[8] - M[2] * M[6];
    out[5] = -(M[0] * M[7] - M[1] * M[6]);
    out[6] = M[1] * M[5] - M[2] * M[4];
    out[7] = -(M[0] * M[5] - M[2] * M[3]);
    out[8] = M[0] * M[4] - M[1] * M[3];
}

__device__ NdPrep nd_prep(const float* m, const float* C, float op, float tq, bool falloff, float v3, float v2) {
    NdPrep p;
#pragma unroll
    for (int i = 0; i < 9; ++i) p.S[i] = C[i];
    p.f3 = 1.0f;
    p.opf = op;
    if (v3 > 0.0f) {
        p.S[0] = __fadd_rn(C[0], v3);
        p.S[4] = __fadd_rn(C[4], v3);
        p.S[8] = __fadd_rn(C[8], v3);
        const float dc = fmaxf(det3(C), 1.0e-12f), ds = fmaxf(det3(p.S), 1.0e-12f);
        p.f3 = __fsqrt_rn(__fdiv_rn(dc, ds));
        p.opf = __fmul_rn(op, p.f3);
    }
    p.vtt = fmaxf(p.S[8], 1.0e-12f);
    p.dt = __fsub_rn(tq, m[2]);
    p.k = __fdiv_rn(p.dt, p.vtt);
    p.mx = __fadd_rn(m[0], __fmul_rn(p.S[2], p.k));
    p.my = __fadd_rn(m[1], __fmul_rn(p.S[5], p.k));
    p.c[0] = __fsub_rn(p.S[0], __fdiv_rn(__fmul_rn(p.S[2], p.S[2]), p.vtt));
    p.c[1] = __fsub_rn(p.S[1], __fdiv_rn(__fmul_rn(p.S[2], p.S[5]), p.vtt));
    p.c[2] = __fsub_rn(p.S[3], __fdiv_rn(__fmul_rn(p.S[5], p.S[2]), p.vtt));
    p.c[3] = __fsub_rn(p.S[4], __fdiv_rn(__fmul_rn(p.S[5], p.S[5]), p.vtt));
    const float lw = __fsub_rn(__fdiv_rn(__fmul_rn(__fmul_rn(-0.5f, p.dt), p.dt), p.vtt),
                               __fmul_rn(0.5f, __fadd_rn(1.8378770664093453f, logf(p.vtt))));
    p.wt = expf(lw);
    p.W = falloff ? p.wt : 1.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) p.P[i] = p.c[i];
    p.f2 = 1.0f;
    p.W2 = p.W;
    if (v2 > 0.0f) {
        p.P[0] = __fadd_rn(p.c[0], v2);
        p.P[3] = __fadd_rn(p.c[3], v2);
        const float dc = fmaxf(__fsub_rn(__fmul_rn(p.c[0], p.c[3]), __fmul_rn(p.c[1], p.c[2])), 1.0e-12f);
        const float dp = fmaxf(__fsub_rn(__fmul_rn(p.P[0], p.P[3]), __fmul_rn(p.P[1], p.P[2])), 1.0e-12f);
        p.f2 = __fsqrt_rn(__fdiv_rn(dc, dp));
        p.W2 = __fmul_rn(p.W, p.f2);
    }
    p.D = __fsub_rn(__fmul_rn(p.P[0], p.P[3]), __fmul_rn(p.P[1], p.P[2]));
    return p;
}

__global__ void __launch_bounds__(256) k_nd_prep_fwd(int n, int H, int W, const float* __restrict__ means,
                                                      const float* __restrict__ covs, const float* __restrict__ opac,
                                                      float tq, int falloff, float v3, float v2,
                                                      float* __restrict__ xy, float* __restrict__ conic,
                                                      float* __restrict__ amp, int4* __restrict__ box) {
    const int g = blockIdx.x * 256 + threadIdx.x;
    if (g >= n) return;
    float m[3], C[9];
#pragma unroll
    for (int i = 0; i < 3; ++i) m[i] = means[3 * static_cast<int64_t>(g) + i];
#pragma unroll
    for (int i = 0; i < 9; ++i) C[i] = covs[9 * static_cast<int64_t>(g) + i];
    const NdPrep p = nd_prep(m, C, opac[g], tq, falloff != 0, v3, v2);
    xy[2 * g + 0] = p.mx;
    xy[2 * g + 1] = p.my;
    conic[3 * g + 0] = __fdiv_rn(p.P[3], p.D);
    conic[3 * g + 1] = __fdiv_rn(-p.P[1], p.D);
    conic[3 * g + 2] = __fdiv_rn(p.P[0], p.D);
    amp[g] = __fmul_rn(p.opf, p.W2);
    // cull box: 3 sqrt(largest eigenvalue, at least 1e-6) around the mean, fp64 floor / ceil
    const float a = p.P[0], d = p.P[3], b = __fmul_rn(0.5f, __fadd_rn(p.P[1], p.P[2]));
    const float half = __fmul_rn(0.5f, __fsub_rn(a, d));
    float lam = __fadd_rn(__fmul_rn(0.5f, __fadd_rn(a, d)), __fsqrt_rn(__fadd_rn(__fmul_rn(half, half), __fmul_rn(b, b))));
    lam = fmaxf(lam, 1.0e-6f);
    const double r = 3.0 * static_cast<double>(__fsqrt_rn(lam));
    const double x0 = fmax(floor(static_cast<double>(p.mx) - r), 0.0);
    const double x1 = fmin(ceil(static_cast<double>(p.mx) + r), static_cast<double>(W));
    const double y0 = fmax(floor(static_cast<double>(p.my) - r), 0.0);
    const double y1 = fmin(ceil(static_cast<double>(p.my) + r), static_cast<double>(H));
    int4 bx = make_int4(0, 0, 0, 0);
    if (isfinite(x0) && isfinite(x1) && isfinite(y0) && isfinite(y1)) {
        bx = make_int4(static_cast<int>(x0), static_cast<int>(y0), static_cast<int>(x1), static_cast<int>(y1));
    }
    box[g] = bx;
}

__global__ void __launch_bounds__(256) k_nd_prep_bwd(int n, const float* __restrict__ means,
                                                      const float* __restrict__ covs, const float* __restrict__ opac,
                                                      float tq, int falloff, float v3, float v2,
                                                      const float* __restrict__ g_xy, const float* __restrict__ g_conic,
                                                      const float* __restrict__ g_amp, float* __restrict__ g_means,
                                                      float* __restrict__ g_covs, float* __restrict__ g_opac) {
    const int g = blockIdx.x * 256 + threadIdx.x;
    if (g >= n) return;
    float m[3], C[9];
#pragma unroll
    for (int i = 0; i < 3; ++i) m[i] = means[3 * static_cast<int64_t>(g) + i];
#pragma unroll
    for (int i = 0; i < 9; ++i) C[i] = covs[9 * static_cast<int64_t>(g) + i];
    const float op = opac[g];
    const NdPrep p = nd_prep(m, C, op, tq, falloff != 0, v3, v2);
    const float gx = g_xy[2 * g], gy = g_xy[2 * g + 1];
    const float ga = g_conic[3 * g], gb = g_conic[3 * g + 1], gd = g_conic[3 * g + 2];
    const float gamp = g_amp[g];
    // amp = opf * W2
    const float g_opf = gamp * p.W2;
    const float g_W2 = gamp * p.opf;
    // conic (a, b, d) = (P11, -P01, P00) / D
    const float a = p.P[3] / p.D, b = -p.P[1] / p.D, d = p.P[0] / p.D;
    const float sd = (ga * a + gb * b + gd * d) / p.D;
    float gP[4];
    gP[0] = gd / p.D - sd * p.P[3];
    gP[3] = ga / p.D - sd * p.P[0];
    gP[1] = -gb / p.D + sd * p.P[2];
    gP[2] = sd * p.P[1];
    // Mip 2D: P = c + v2 I, W2 = W * sqrt(det c / det P)
    float gc[4] = {gP[0], gP[1], gP[2], gP[3]};
    float g_W = g_W2;
    if (v2 > 0.0f) {
        g_W = g_W2 * p.f2;
        const float g_f2 = g_W2 * p.W;
        const float dc = p.c[0] * p.c[3] - p.c[1] * p.c[2];
        const float dp = p.P[0] * p.P[3] - p.P[1] * p.P[2];
        const float g_dc = dc >= 1.0e-12f ? g_f2 * p.f2 / (2.0f * dc) : 0.0f;
        const float g_dp = dp >= 1.0e-12f ? -g_f2 * p.f2 / (2.0f * dp) : 0.0f;
        gc[0] += g_dc * p.c[3] + g_dp * p.P[3];
        gc[3] += g_dc * p.c[0] + g_dp * p.P[0];
        gc[1] += -g_dc * p.c[2] - g_dp * p.P[2];
        gc[2] += -g_dc * p.c[1] - g_dp * p.P[1];
    }
    // W = wt (time falloff) or 1; wt = exp(lw), lw = -dt^2 / (2 vtt) - (log 2 pi + log vtt) / 2
    const float g_lw = falloff ? g_W * p.wt : 0.0f;
    float g_dt = g_lw * (-p.dt / p.vtt);
    float g_vtt = g_lw * (0.5f * p.dt * p.dt / (p.vtt * p.vtt) - 0.5f / p.vtt);
    // conditional mean: m01 + vxt * k, k = dt / vtt
    const float vx0 = p.S[2], vx1 = p.S[5];
    float g_v0 = gx * p.k, g_v1 = gy * p.k;
    const float g_k = gx * vx0 + gy * vx1;
    g_dt += g_k / p.vtt;
    g_vtt += -g_k * p.dt / (p.vtt * p.vtt);
    // Schur complement: c_ij = S_ij - v_i v_j / vtt (i, j in {0, 1})
    float gS[9] = {gc[0], gc[1], 0.0f, gc[2], gc[3], 0.0f, 0.0f, 0.0f, 0.0f};
    g_v0 += -(2.0f * gc[0] * vx0 + (gc[1] + gc[2]) * vx1) / p.vtt;
    g_v1 += -(2.0f * gc[3] * vx1 + (gc[1] + gc[2]) * vx0) / p.vtt;
    g_vtt += (gc[0] * vx0 * vx0 + (gc[1] + gc[2]) * vx0 * vx1 + gc[3] * vx1 * vx1) / (p.vtt * p.vtt);
    gS[2] += g_v0;
    gS[5] += g_v1;
    gS[8] += p.S[8] >= 1.0e-12f ? g_vtt : 0.0f;
    // Mip 3D: S = C + v3 I, opf = op * sqrt(det C / det S)
    float gC[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) gC[i] = gS[i];
    float g_op = g_opf;
    if (v3 > 0.0f) {
        g_op = g_opf * p.f3;
        const float g_f3 = g_opf * op;
        const float dc = det3(C), ds = det3(p.S);
        const float g_dc = dc >= 1.0e-12f ? g_f3 * p.f3 / (2.0f * dc) : 0.0f;
        const float g_ds = ds >= 1.0e-12f ? -g_f3 * p.f3 / (2.0f * ds) : 0.0f;
        float cc[9], cs[9];
        cof3(C, cc);
        cof3(p.S, cs);
#pragma unroll
        for (int i = 0; i < 9; ++i) gC[i] += g_dc * cc[i] + g_ds * cs[i];
    }
    g_means[3 * static_cast<int64_t>(g) + 0] = gx;
    g_means[3 * static_cast<int64_t>(g) + 1] = gy;
    g_means[3 * static_cast<int64_t>(g) + 2] = -g_dt;
#pragma unroll
    for (int i = 0; i < 9; ++i) g_covs[9 * static_cast<int64_t>(g) + i] = gC[i];
    g_opac[g] = g_op;
}

#define OSS_ND_DISPATCH(f, CALL) \
    ((f) <= 1 ? CALL(1) : (f) <= 3 ? CALL(3) : (f) <= 4 ? CALL(4) : (f) <= 8 ? CALL(8) : (f) <= 16 ? CALL(16) : CALL(32))

}  // namespace

cudaError_t launch_nd_prep_forward(int n, int h, int w, const float* means, const float* covs, const float* opac,
                                   float tq, int falloff, float v3, float v2, float* xy, float* conic, float* amp,
                                   int32_t* box, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    k_nd_prep_fwd<<<static_cast<unsigned>(div_up(n, 256)), 256, 0, stream>>>(
        n, h, w, means, covs, opac, tq, falloff, v3, v2, xy, conic, amp, reinterpret_cast<int4*>(box));
    return cudaGetLastError();
}

cudaError_t launch_nd_prep_backward(int n, const float* means, const float* covs, const float* opac, float tq,
                                    int falloff, float v3, float v2, const float* g_xy, const float* g_conic,
                                    const float* g_amp, float* g_means, float* g_covs, float* g_opac,
                                    cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    k_nd_prep_bwd<<<static_cast<unsigned>(div_up(n, 256)), 256, 0, stream>>>(
        n, means, covs, opac, tq, falloff, v3, v2, g_xy, g_conic, g_amp, g_means, g_covs, g_opac);
    return cudaGetLastError();
}

int nd_record_floats(int f) {
#define OSS_ND_RS(FC) NdCfg<FC>::RS
    return OSS_ND_DISPATCH(f, OSS_ND_RS);
#undef OSS_ND_RS
}

cudaError_t launch_nd_preprocess(int n, int ntx, int nty, const float* xy, const float* conic, const int32_t* box,
                                 int f, const float* feat, const float* amp, int32_t* aabb, int32_t* count,
                                 float* geo, float* prec, long long* block_sums, int32_t* tile_count,
                                 cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    k_nd_preprocess<<<static_cast<unsigned>(div_up(n, kPrepTile)), kPreprocThreads, 0, stream>>>(
        n, ntx, nty, reinterpret_cast<const float2*>(xy), conic, reinterpret_cast<const int4*>(box), f,
        nd_record_floats(f), feat, amp, reinterpret_cast<int4*>(aabb), count, geo, prec, block_sums, tile_count);
    return cudaGetLastError();
}

cudaError_t launch_nd_forward(int f, int h, int w, const float* prec, const int32_t* box, const int32_t* gid_sorted,
                              const int32_t* tile_offsets, float* image, cudaStream_t stream) {
    const int ntx = static_cast<int>(div_up(w, kTile)), nty = static_cast<int>(div_up(h, kTile));
    if (ntx * nty == 0 || f == 0) return cudaSuccess;
#define OSS_ND_FWD(FC)                                                                                         \
    (k_nd_fwd<FC><<<static_cast<unsigned>(ntx * nty), kNdThreads, 0, stream>>>(                              \
         f, h, w, ntx, prec, reinterpret_cast<const int4*>(box), gid_sorted, tile_offsets, image),            \
     cudaGetLastError())
    return OSS_ND_DISPATCH(f, OSS_ND_FWD);
#undef OSS_ND_FWD
}

cudaError_t launch_nd_backward_pairs(int f, int h, int w, const float* prec, const int32_t* box,
                                     const int32_t* gid_sorted, const int32_t* tile_offsets, const int32_t* aabb,
                                     const int32_t* pair_offset, const float* grad_image, float* pairgrad,
                                     int pair_stride, cudaStream_t stream) {
    const int ntx = static_cast<int>(div_up(w, kTile)), nty = static_cast<int>(div_up(h, kTile));
    if (ntx * nty == 0 || f == 0) return cudaSuccess;
#define OSS_ND_BWD(FC)                                                                                         \
    (k_nd_bwd<FC><<<static_cast<unsigned>(ntx * nty), kNdThreads, 0, stream>>>(                              \
         f, h, w, ntx, prec, reinterpret_cast<const int4*>(box), gid_sorted, tile_offsets,                     \
         reinterpret_cast<const int4*>(aabb), pair_offset, grad_image, pairgrad, pair_stride),                 \
     cudaGetLastError())
    return OSS_ND_DISPATCH(f, OSS_ND_BWD);
#undef OSS_ND_BWD
}

}  // namespace oss
