// One-pass feathered overlapping-tile render: the reference's
// V6Rasterizer._render_overlapped (oss/sr/v6/rasterizer.py:159-242) without its
// four renders.
//
// The reference renders the means shifted by each of four phase origins
// (0|-o, 0|-o) on crops rounded up to 16, so that each phase's 16-px tile grid
// sits o pixels from the others, and blends the crops with per-phase weights
// m_k = wy_k(row) * wx_k(col) (a cosine ramp over the distance to the nearest
// tile edge of that phase's grid), normalised by their sum W.  Its lists are
// truncated (3-sigma or q = 176 boxes), so which Gaussians a pixel sees depends
// on the phase: a Gaussian contributes to pixel p in phase k exactly when its
// phase-k tile box covers the phase-k tile holding p.  Per axis the weights and
// the box test separate, so the blended image is
//   out(p) = sum_g feat_g w_g(p) Mx_g(col) My_g(row),
//   Mx_g(c) = [box0 covers tile0(c)] nx0(c) + [box1 covers tile1(c)] nx1(c),
//   nx_k = wx_k / (wx_0 + wx_1),   (W = (wx_0 + wx_1)(wy_0 + wy_1))
// one render of every Gaussian with a separable window.  The window is a step
// function of the box, so it carries no gradient: the backward is the ordinary
// one with w * M in place of w.  Both factors enter the exponent: w * M =
// 2^(q' + log2 Mx + log2 My), with log2 of the normalised weights tabulated per
// tile column and phase-bit pattern (FeatherTable).
//
// A phase's shifted mean fl(x + o) is exact for almost every x; where it is not
// (x within o below a power of two, or |x| < o), the reference evaluates that
// phase at a centre one rounding away.  Such a Gaussian is split into variants:
// variant (kx, ky) has the centre (kx ? fl(x + o) - o : x, ky ? ... : y) and
// keeps only the phases whose centre it is.  So the evaluation of every phase
// is the reference's to the bit in dx, dy.  Variant k of Gaussian g is virtual
// Gaussian 4 g + k; absent variants have no tiles.  Lists, forward and backward
// run over the 4N virtual Gaussians; the per-Gaussian reduce sums a Gaussian's
// four variants' rows, which are contiguous in the gid-major pair order.
#include <climits>
#include <math.h>

#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

constexpr int kFeatherThreads = kPrepTile / kFeatherVariants;  // 256 Gaussians, 1024 virtual Gaussians per CTA

__device__ __forceinline__ int4 hull_axis(int a0, int b0, int a1, int b1, int split_shift, int nt) {
    // tiles of the phase-0 grid a variant's window reaches along one axis: its
    // phase-0 range [a0, b0) and the phase-0 tiles its phase-1 range [a1, b1)
    // (already in phase-0 tile units) touches, which start one tile earlier when
    // the grids are offset by a fraction of a tile
    int lo = INT_MAX, hi = INT_MIN;
    if (b0 > a0) {
        lo = a0;
        hi = b0;
    }
    if (b1 > a1) {
        lo = min(lo, a1 - split_shift);
        hi = max(hi, b1);
    }
    lo = max(lo, 0);
    hi = min(hi, nt);
    if (hi <= lo) return make_int4(0, 0, 0, 0);
    return make_int4(lo, hi, 1, 0);
}

__global__ void __launch_bounds__(kFeatherThreads) k_prepare_feathered(
    int n, int ntx0, int nty0, int ntx1, int nty1, int mode, float ov, int qshift, int split_shift,
    const float2* __restrict__ xy, const float2* __restrict__ scale, const float* __restrict__ rot, int F, int prs,
    const float* __restrict__ feat, const float* __restrict__ opacity, float* __restrict__ conic,
    float* __restrict__ geo, int4* __restrict__ vaabb, int32_t* __restrict__ vcount, float* __restrict__ vprec,
    int4* __restrict__ vwin, long long* __restrict__ block_sums, int32_t* __restrict__ tile_count) {
    long long local = 0;
    const int g = blockIdx.x * kFeatherThreads + threadIdx.x;
    if (g < n) {
        const float2 c = xy[g];
        const float2 s = scale[g];
        const Conic k = conic_from_scale_rot(s.x, s.y, rot[g]);
        conic[3 * g + 0] = k.a;
        conic[3 * g + 1] = k.b;
        conic[3 * g + 2] = k.d;
        float4* gr = reinterpret_cast<float4*>(geo + static_cast<int64_t>(g) * 8);
        gr[0] = make_float4(c.x, c.y, k.a * kNegHalfLog2e, (2.0f * k.b) * kNegHalfLog2e);
        gr[1] = make_float4(k.d * kNegHalfLog2e, k.a, k.b, k.d);
        // the shifted phase's means, as the reference forms them (xy - origin in fp32)
        const float x1 = __fadd_rn(c.x, ov);
        const float y1 = __fadd_rn(c.y, ov);
        int4 b0, b1;
        int cnt;
        if (mode == OSS_BIN_FULL) {
            b0 = make_int4(0, 0, ntx0, nty0);
            b1 = make_int4(0, 0, ntx1, nty1);
        } else {
            b0 = tile_aabb(c.x, c.y, s.x, s.y, k, mode_tau(mode), mode_fallback(mode), ntx0, nty0, cnt);
            b1 = tile_aabb(x1, y1, s.x, s.y, k, mode_tau(mode), mode_fallback(mode), ntx1, nty1, cnt);
        }
        // phase-1 tile u holds output columns [16 (u - qshift) - r, ...): in phase-0 tile units
        b1.x -= qshift;
        b1.z -= qshift;
        b1.y -= qshift;
        b1.w -= qshift;
        // centres of the shifted phases in output coordinates; a variant exists where they differ
        const float xs = __fsub_rn(x1, ov);
        const float ys = __fsub_rn(y1, ov);
        const bool sx = isfinite(c.x) && xs != c.x;
        const bool sy = isfinite(c.y) && ys != c.y;
        const float* fg = feat + static_cast<int64_t>(g) * F;
        const float op = opacity != nullptr ? opacity[g] : 1.0f;
#pragma unroll
        for (int v = 0; v < kFeatherVariants; ++v) {
            const int kx = v & 1, ky = v >> 1;
            const int vg = kFeatherVariants * g + v;
            const bool present = (kx == 0 || sx) && (ky == 0 || sy);
            // the phases of this variant: both where the shift is exact, else its own
            const bool x0 = kx == 0, x1p = kx == 1 || !sx;
            const bool y0 = ky == 0, y1p = ky == 1 || !sy;
            const int a0x = x0 ? b0.x : 0, e0x = x0 ? b0.z : 0;
            const int a1x = x1p ? b1.x : 0, e1x = x1p ? b1.z : 0;
            const int a0y = y0 ? b0.y : 0, e0y = y0 ? b0.w : 0;
            const int a1y = y1p ? b1.y : 0, e1y = y1p ? b1.w : 0;
            const int4 hx = hull_axis(a0x, e0x, a1x, e1x, split_shift, ntx0);
            const int4 hy = hull_axis(a0y, e0y, a1y, e1y, split_shift, nty0);
            int vc = 0;
            int4 box = make_int4(0, 0, 0, 0);
            if (present && hx.z && hy.z) {
                box = make_int4(hx.x, hy.x, hx.y, hy.y);
                vc = (hx.y - hx.x) * (hy.y - hy.x);
            }
            vaabb[vg] = box;
            vcount[vg] = vc;
            local += vc;
            if (vc == 0) continue;
            vwin[vg] = make_int4(pack_range(a0x, e0x), pack_range(a1x, e1x), pack_range(a0y, e0y),
                                 pack_range(a1y, e1y));
            float4* rec = reinterpret_cast<float4*>(vprec + static_cast<int64_t>(vg) * prs);
            rec[0] = make_float4(kx ? xs : c.x, ky ? ys : c.y, k.a * kNegHalfLog2e, (2.0f * k.b) * kNegHalfLog2e);
            for (int q = 1; q < prs / 4; ++q) {
                float e[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int i = 4 * q + u;  // record float i; feature i - 5
                    e[u] = i == 4 ? k.d * kNegHalfLog2e : (i - 5 < F ? fg[i - 5] * op : 0.0f);
                }
                rec[q] = make_float4(e[0], e[1], e[2], e[3]);
            }
            for (int ty = box.y; ty < box.w; ++ty) {
                for (int tx = box.x; tx < box.z; ++tx) {
                    atomicAdd(&tile_count[static_cast<int64_t>(ty * ntx0 + tx) * kTileCountStride], 1);
                }
            }
        }
    }
    __shared__ long long s_part[kFeatherThreads / 32];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) local += __shfl_down_sync(0xffffffffu, local, off);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = local;
    __syncthreads();
    if (threadIdx.x == 0) {
        long long tot = 0;
#pragma unroll
        for (int w = 0; w < kFeatherThreads / 32; ++w) tot += s_part[w];
        block_sums[blockIdx.x] = tot;
    }
}

double ramp(double t) { return 0.5 - 0.5 * cos(t * 3.14159265358979323846); }

// Feather weight of one phase at tile column c (the reference's _phase_feather_mask
// per axis): cosine ramp of the distance from the pixel centre to the nearest tile
// edge of the phase whose origin is -shift, over `overlap` pixels.
double phase_weight(int c, int shift, int overlap) {
    double p = fmod(static_cast<double>(c) + 0.5 + static_cast<double>(shift), static_cast<double>(kTile));
    const double d = p < kTile - p ? p : kTile - p;
    double t = d / static_cast<double>(overlap);
    t = t < 0.0 ? 0.0 : (t > 1.0 ? 1.0 : t);
    return ramp(t);
}

}  // namespace

int feather_table(int overlap, FeatherTable* tab) {
    if (overlap <= 0) return 0;
    const int r = overlap % kTile;
    const int split = kTile - r;  // first column whose phase-1 tile is the next one (none when r == 0)
    double min_sum = 1.0e300;
    for (int c = 0; c < kTile; ++c) {
        const double w0 = phase_weight(c, 0, overlap);
        const double w1 = phase_weight(c, overlap, overlap);
        const double sum = w0 + w1;
        min_sum = sum < min_sum ? sum : min_sum;
        const double n0 = w0 / sum, n1 = w1 / sum;
        for (int p = 0; p < 8; ++p) {
            const bool b0 = (p & 1) != 0;
            const bool b1 = r != 0 && c >= split ? (p & 4) != 0 : (p & 2) != 0;
            const double m = (b0 ? n0 : 0.0) + (b1 ? n1 : 0.0);
            // n0 + n1 is 1 up to rounding: an entry both phases include keeps its weight
            const double mm = b0 && b1 ? 1.0 : m;
            tab->lw[p][c] = mm > 0.0 ? static_cast<float>(log2(mm)) : -INFINITY;
        }
    }
    // the separable form needs the reference's clamp of W at 1e-6 to be inactive
    return min_sum * min_sum >= 2.0e-6 ? 1 : 0;
}

cudaError_t launch_prepare_feathered(int n, int h, int w, int mode, int overlap, const float* xy, const float* scale,
                                     const float* rot, int f, const float* feat, const float* opacity, float* conic,
                                     float* geo, int32_t* vaabb, int32_t* vcount, float* vprec, int32_t* vwin,
                                     long long* block_sums, int32_t* tile_count, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    const int ntx0 = static_cast<int>(div_up(w, kTile)), nty0 = static_cast<int>(div_up(h, kTile));
    const int ntx1 = static_cast<int>(div_up(static_cast<int64_t>(w) + overlap, kTile));
    const int nty1 = static_cast<int>(div_up(static_cast<int64_t>(h) + overlap, kTile));
    const int qshift = overlap / kTile;
    const int split_shift = overlap % kTile != 0 ? 1 : 0;
    const int prs = entry_record_floats(f);
    k_prepare_feathered<<<static_cast<unsigned>(div_up(n, kFeatherThreads)), kFeatherThreads, 0, stream>>>(
        n, ntx0, nty0, ntx1, nty1, mode, static_cast<float>(overlap), qshift, split_shift,
        reinterpret_cast<const float2*>(xy), reinterpret_cast<const float2*>(scale), rot, f, prs, feat, opacity, conic,
        geo, reinterpret_cast<int4*>(vaabb), vcount, vprec, reinterpret_cast<int4*>(vwin), block_sums, tile_count);
    return cudaGetLastError();
}

}  // namespace oss
