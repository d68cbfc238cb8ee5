// Backward of the additive tile render (the reference's rasterize_backward,
// rasterizer_bwd.cu:32-113), re-organised so that no per-pixel atomics remain.
//
// Work is cut into items: up to 32 list entries of one tile, listed longest
// first in an item table (tile, first entry, count) built by two small kernels.
// The kernel's warps are persistent and take items one at a time through a
// counter.  For each item a warp stages the tile's dL/dimage block into its own
// shared-memory slot (rows padded so that lanes on different rows hit different
// banks), then each lane owns one list entry and walks the tile's pixels,
// keeping the per-pair sums in registers:
//   g = w * sum_c go_c f'_c      (w = exp(-q/2), dL/dq = -g/2)
//   Sx = sum g dx, Sy = sum g dy, Sxx = sum g dx^2, Sxy = sum g dx dy,
//   Syy = sum g dy^2, dF_c = sum w go_c
// from which d_xy = (a Sx + b Sy, b Sx + d Sy) and
// d_conic = (-Sxx/2, -Sxy, -Syy/2) -- the reference's per-pixel terms
// (rasterizer_bwd.cu:89-108) summed over the tile.  The entry's data comes from
// the forward's entry records (one coalesced load) when the caller kept them,
// else it is gathered through gid_sorted.  The entry's pair slot comes from the
// forward's slots when given, else from gid_sorted, aabb and pair_offset, read
// after the sums so their latency overlaps the arithmetic.
//
// A tile's last item is usually partial.  With r < 32 entries it runs k lanes
// per entry (k = 2, 4, 8 or 16, the largest with r*k <= 32), each lane taking
// 16/k rows, and the k partial sums are combined by a fixed xor-shuffle tree:
// the split depends only on r, so results are bitwise reproducible.
//
// Deterministic mode writes each pair's partial row (Sx, Sy, d_conic, dF) at its
// gid-major pair slot (pair_offset[g] + local tile index, the order of the
// reference's build_tile_pairs); k_reduce_gaussian then sums a Gaussian's rows in
// that fixed order, applies the conic to (Sx, Sy) -- d_xy is linear in them --
// and the conic -> (scale, rot) chain rule and the opacity unfold.  Atomic mode
// (caller-supplied lists) adds each pair's partials with fp32 atomics: (F+5)
// atomics per pair instead of the reference's (F+5) per pixel-pair.
#include <atomic>

#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

constexpr int kItemEntries = 32;

template <int FC>
struct BwdCfg {
    static constexpr int SG = ((FC + 3) / 4) * 4;        // staged grad floats per pixel
    static constexpr int ROW = kTile * SG + 4;            // floats per staged row (+4: bank spread)
    static constexpr int SLOT = kTile * ROW;              // floats per warp slot
    static constexpr int WARPS = SLOT * 4 * 4 <= 200 * 1024 ? 4 : 2;  // warps (slots) per CTA
    static constexpr int THREADS = WARPS * 32;
    static constexpr int MIN_CTAS = FC <= 4 ? 4 : 1;  // 4 x 4 warps per SM (<= 128 registers) for F <= 4
    // F <= 4 runs the packed f32x2 path: the staged block is interleaved by
    // column pairs, [go_k(c), go_k(c+1)] for k = 0..SG-1 per pair of columns.
    static constexpr bool PAIRED = FC <= 4;
};

// Shared-memory index of staged channel k at tile row r, column c.
template <int FC>
__device__ __forceinline__ int go_index(int r, int c, int k) {
    constexpr int SG = BwdCfg<FC>::SG;
    if (BwdCfg<FC>::PAIRED) return r * BwdCfg<FC>::ROW + (c >> 1) * 2 * SG + 2 * k + (c & 1);
    return r * BwdCfg<FC>::ROW + c * SG + k;
}

__device__ __forceinline__ bool regular_conic_bwd(float x, float y, float a, float b, float d) {
    const bool finite = isfinite(x) && isfinite(y) && isfinite(a) && isfinite(b) && isfinite(d);
    return finite && a > 0.0f && d > 0.0f && (a * d - b * b) >= 1.0e-3f * (a * d);
}

// Packed-f32x2 version of the full-row sums for F <= 4: every FP32 operation
// works on two adjacent columns at once (__ffma2_rn / __fmul2_rn / __fadd2_rn),
// halving the FP32 instructions per pixel; exp2 stays one MUFU op per pixel.
// The column offsets dx and their squares are held in registers, so the
// moments take g dx and g dx^2 as one FFMA2 each.
// With WIN (the one-pass feathered render) the entry's log2 window weights by
// column (lwx) and row (lwy) enter the exponent: the column's folded into a
// per-column constant A dx^2 + lwx, the row's into D dy^2.
template <int FC, bool CHECK, bool WIN = false>
__device__ __forceinline__ void bwd_rows_full_pk(const float* __restrict__ s_go, int r0, int r1, float fx0, float fy0,
                                                 float gx, float gy, float A, float B, float D, const float (&fv)[FC],
                                                 float (&dF)[FC], float& Sx, float& Sy, float& Sxx, float& Sxy,
                                                 float& Syy, const float* __restrict__ lwx = nullptr,
                                                 const float* __restrict__ lwy = nullptr) {
    constexpr int SG = BwdCfg<FC>::SG;
    constexpr int ROW = BwdCfg<FC>::ROW;
    float2 dx2[kTile / 2], dxsq2[kTile / 2];
    float2 cx2[WIN ? kTile / 2 : 1];
    const float2 A2 = make_float2(A, A);
#pragma unroll
    for (int j = 0; j < kTile / 2; ++j) {
        dx2[j] = make_float2((fx0 + static_cast<float>(2 * j)) - gx, (fx0 + static_cast<float>(2 * j + 1)) - gx);
        dxsq2[j] = __fmul2_rn(dx2[j], dx2[j]);
        if constexpr (WIN) cx2[j] = __ffma2_rn(A2, dxsq2[j], make_float2(lwx[2 * j], lwx[2 * j + 1]));
    }
    float2 f2[FC], dF2[FC];
#pragma unroll
    for (int k = 0; k < FC; ++k) {
        f2[k] = make_float2(fv[k], fv[k]);
        dF2[k] = make_float2(0.0f, 0.0f);
    }
#pragma unroll 1
    for (int r = r0; r < r1; ++r) {
        const float dy = (fy0 + static_cast<float>(r)) - gy;
        const float bdy = B * dy;
        const float ddy = (D * dy) * dy;
        const float2 bdy2 = make_float2(bdy, bdy);
        const float2 ddy2 = make_float2(ddy, ddy);
        float2 ddyw2 = ddy2;
        if constexpr (WIN) {
            const float t = ddy + lwy[r];
            ddyw2 = make_float2(t, t);
        }
        float2 rowG2 = make_float2(0.0f, 0.0f), rowGx2 = make_float2(0.0f, 0.0f), rowGxx2 = make_float2(0.0f, 0.0f);
        const float* go_row = s_go + r * ROW;
#pragma unroll
        for (int j = 0; j < kTile / 2; ++j) {
            const float2 dx = dx2[j];
            float2 w;
            if constexpr (WIN) {
                const float2 q = __ffma2_rn(dx, bdy2, __fadd2_rn(cx2[j], ddyw2));
                if (CHECK) {
                    const float2 q0 = __ffma2_rn(dx, __ffma2_rn(A2, dx, bdy2), ddy2);  // the q >= 0 test, unwindowed
                    w.x = q0.x <= 0.0f ? ex2_ftz(q.x) : 0.0f;
                    w.y = q0.y <= 0.0f ? ex2_ftz(q.y) : 0.0f;
                } else {
                    w.x = ex2_ftz(q.x);
                    w.y = ex2_ftz(q.y);
                }
            } else {
                const float2 q = __ffma2_rn(dx, __ffma2_rn(A2, dx, bdy2), ddy2);
                w.x = CHECK ? (q.x <= 0.0f ? ex2_ftz(q.x) : 0.0f) : ex2_ftz(q.x);
                w.y = CHECK ? (q.y <= 0.0f ? ex2_ftz(q.y) : 0.0f) : ex2_ftz(q.y);
            }
            const float4* go4 = reinterpret_cast<const float4*>(go_row + j * 2 * SG);
            float2 go2[SG];
#pragma unroll
            for (int v = 0; v < SG / 2; ++v) {
                const float4 t = go4[v];
                go2[2 * v] = make_float2(t.x, t.y);
                go2[2 * v + 1] = make_float2(t.z, t.w);
            }
            float2 dLdw = __fmul2_rn(go2[0], f2[0]);
#pragma unroll
            for (int k = 1; k < FC; ++k) dLdw = __ffma2_rn(go2[k], f2[k], dLdw);
#pragma unroll
            for (int k = 0; k < FC; ++k) dF2[k] = __ffma2_rn(w, go2[k], dF2[k]);
            const float2 gw = __fmul2_rn(w, dLdw);
            rowGx2 = __ffma2_rn(gw, dx, rowGx2);
            rowGxx2 = __ffma2_rn(gw, dxsq2[j], rowGxx2);
            rowG2 = __fadd2_rn(rowG2, gw);
        }
        const float rowGx = rowGx2.x + rowGx2.y;
        const float rowG = rowG2.x + rowG2.y;
        // every moment is summed per row first, then over the rows
        Sxx += rowGxx2.x + rowGxx2.y;
        Sx += rowGx;
        Sxy = fmaf(rowGx, dy, Sxy);
        Sy = fmaf(rowG, dy, Sy);
        Syy = fmaf(rowG * dy, dy, Syy);
    }
#pragma unroll
    for (int k = 0; k < FC; ++k) dF[k] += dF2[k].x + dF2[k].y;
}

// Per-pair sums over rows [r0, r1) of a full 16-wide tile row span: the 16
// column offsets dx are hoisted into registers, each row hoists B*dy and
// D*dy*dy, and the column loop is fully unrolled.  CHECK keeps the reference's
// q >= 0 test per pixel.
template <int FC, bool CHECK, bool WIN = false>
__device__ __forceinline__ void bwd_rows_full(const float* __restrict__ s_go, int r0, int r1, float fx0, float fy0,
                                              float gx, float gy, float A, float B, float D, const float (&fv)[FC],
                                              float (&dF)[FC], float& Sx, float& Sy, float& Sxx, float& Sxy,
                                              float& Syy, const float* __restrict__ lwx = nullptr,
                                              const float* __restrict__ lwy = nullptr) {
    constexpr int SG = BwdCfg<FC>::SG;
    constexpr int ROW = BwdCfg<FC>::ROW;
    float dxs[kTile];
#pragma unroll
    for (int c = 0; c < kTile; ++c) dxs[c] = (fx0 + static_cast<float>(c)) - gx;
    // rows are summed in fp32, the rows' sums in double: five double adds per row
    // against 16 pixels of F + 12 fp32 operations, and a thin Gaussian's moments
    // cancel across rows
    double dSx = 0.0, dSy = 0.0, dSxx = 0.0, dSxy = 0.0, dSyy = 0.0;
#pragma unroll 1
    for (int r = r0; r < r1; ++r) {
        const float dy = (fy0 + static_cast<float>(r)) - gy;
        const float bdy = B * dy;
        const float ddy2 = (D * dy) * dy;
        const float lwr = WIN ? lwy[r] : 0.0f;
        // four interleaved partial sums per moment (columns c mod 4), added pairwise
        float pG[4] = {0.0f, 0.0f, 0.0f, 0.0f}, pGx[4] = {0.0f, 0.0f, 0.0f, 0.0f}, pGxx[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const float* go_row = s_go + r * ROW;
#pragma unroll
        for (int c = 0; c < kTile; ++c) {
            const float dx = dxs[c];
            const float q = fmaf(dx, fmaf(A, dx, bdy), ddy2);
            float w;
            if constexpr (WIN) {
                const float qw = q + (lwx[c] + lwr);
                w = CHECK ? (q <= 0.0f ? ex2_ftz(qw) : 0.0f) : ex2_ftz(qw);
            } else {
                w = CHECK ? (q <= 0.0f ? ex2_ftz(q) : 0.0f) : ex2_ftz(q);
            }
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
            pGx[c & 3] += gdx;
            pGxx[c & 3] = fmaf(gdx, dx, pGxx[c & 3]);
            pG[c & 3] += gw;
        }
        const float rowGx = (pGx[0] + pGx[1]) + (pGx[2] + pGx[3]);
        const float rowGxx = (pGxx[0] + pGxx[1]) + (pGxx[2] + pGxx[3]);
        const float rowG = (pG[0] + pG[1]) + (pG[2] + pG[3]);
        const double ddy = dy;
        dSxx += rowGxx;
        dSx += rowGx;
        dSxy += static_cast<double>(rowGx) * ddy;
        dSy += static_cast<double>(rowG) * ddy;
        dSyy += static_cast<double>(rowG) * ddy * ddy;
    }
    Sx += static_cast<float>(dSx);
    Sy += static_cast<float>(dSy);
    Sxx += static_cast<float>(dSxx);
    Sxy += static_cast<float>(dSxy);
    Syy += static_cast<float>(dSyy);
}

// Same sums for a tile cut by the image border (ncol < 16 or rows beyond H).
template <int FC, bool WIN = false>
__device__ __forceinline__ void bwd_rows_edge(const float* __restrict__ s_go, int r0, int r1, int ncol, int tx0,
                                              int ty0, float gx, float gy, float A, float B, float D,
                                              const float (&fv)[FC], float (&dF)[FC], float& Sx, float& Sy,
                                              float& Sxx, float& Sxy, float& Syy, const float* __restrict__ lwx = nullptr,
                                              const float* __restrict__ lwy = nullptr) {
    constexpr int ROW = BwdCfg<FC>::ROW;
    double dSx = 0.0, dSy = 0.0, dSxx = 0.0, dSxy = 0.0, dSyy = 0.0;  // as bwd_rows_full
    for (int r = r0; r < r1; ++r) {
        const float lwr = WIN ? lwy[r] : 0.0f;
        const float dy = static_cast<float>(ty0 + r) - gy;
        float pG[4] = {0.0f, 0.0f, 0.0f, 0.0f}, pGx[4] = {0.0f, 0.0f, 0.0f, 0.0f}, pGxx[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const float* go_row = s_go + r * ROW;
#pragma unroll
        for (int c = 0; c < kTile; ++c) {  // unrolled, so the partials stay in registers
            if (c >= ncol) break;
            const float dx = static_cast<float>(tx0 + c) - gx;
            const float q = q_scaled(A, B, D, dx, dy);
            const float w = q <= 0.0f ? ex2_ftz(WIN ? q + (lwx[c] + lwr) : q) : 0.0f;
            float go[FC];
#pragma unroll
            for (int k = 0; k < FC; ++k) go[k] = s_go[go_index<FC>(r, c, k)];
            (void)go_row;
            float dLdw = 0.0f;
#pragma unroll
            for (int k = 0; k < FC; ++k) {
                dLdw = fmaf(go[k], fv[k], dLdw);
                dF[k] = fmaf(w, go[k], dF[k]);
            }
            const float gw = w * dLdw;
            const float gdx = gw * dx;
            pGx[c & 3] += gdx;
            pGxx[c & 3] = fmaf(gdx, dx, pGxx[c & 3]);
            pG[c & 3] += gw;
        }
        const float rowGx = (pGx[0] + pGx[1]) + (pGx[2] + pGx[3]);
        const float rowGxx = (pGxx[0] + pGxx[1]) + (pGxx[2] + pGxx[3]);
        const float rowG = (pG[0] + pG[1]) + (pG[2] + pG[3]);
        const double ddy = dy;
        dSxx += rowGxx;
        dSx += rowGx;
        dSxy += static_cast<double>(rowGx) * ddy;
        dSy += static_cast<double>(rowG) * ddy;
        dSyy += static_cast<double>(rowG) * ddy * ddy;
    }
    Sx += static_cast<float>(dSx);
    Sy += static_cast<float>(dSy);
    Sxx += static_cast<float>(dSxx);
    Sxy += static_cast<float>(dSxy);
    Syy += static_cast<float>(dSyy);
}

__device__ __forceinline__ float group_sum(float v, int k) {
    for (int m = 1; m < k; m <<= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}

// Entry sources and pair-gradient sinks of the backward kernel.
enum BwdMode { kAtomicGather = 0, kDetGather = 1, kDetRecords = 2 };

// Persistent warps: warp i of the grid runs item i first, then takes further
// items (from index warps-in-grid on) through a shared counter, so a warp that
// finishes a short item starts the next one at once instead of idling until the
// other warps of its CTA are done, and the table's longest-first order leaves
// only short items for the end of the launch.  A warp whose first item exists
// takes one index past the end before it leaves, so a launch increments the
// counter exactly num_items times, and atomicInc's wrap limit (num_items - 1)
// puts it back to 0 for the next launch.
__device__ __forceinline__ int take_item(uint32_t* work, uint32_t limit, int base, int lane) {
    uint32_t v = 0;
    if (lane == 0) v = atomicInc(work, limit);
    return base + static_cast<int>(__shfl_sync(0xffffffffu, v, 0));
}

// With WIN (the one-pass feathered render, records mode only) each entry's
// phase-bit patterns come from the forward's entry_pat and select its rows of
// the log2 window table, kept in shared memory after the warp slots; the
// window's column terms take 16 more registers (4 CTAs per SM for F <= 4).
// FRAMES: the items' tiles are those of stacked frames (dL/dimage is
// [frames][F][H][W]); a separate instance, so the one-frame kernel carries none of it.
template <int FC, int MODE, bool WIN = false, bool FRAMES = false>
__global__ void __launch_bounds__(BwdCfg<FC>::THREADS, WIN && FC <= 4 ? 4 : BwdCfg<FC>::MIN_CTAS) k_render_bwd(
    int F, int H, int W, int ntx, const float* __restrict__ geo, const float* __restrict__ feat,
    const float* __restrict__ opacity, const int32_t* __restrict__ gid_sorted, const int4* __restrict__ items,
    const int32_t* __restrict__ num_items, uint32_t* __restrict__ work, const float* __restrict__ grad_image,
    const int4* __restrict__ aabb, const int32_t* __restrict__ pair_offset, const float* __restrict__ records,
    const int32_t* __restrict__ slots, float* __restrict__ pairgrad, int pstride, float* __restrict__ d_xy,
    float* __restrict__ d_conic, float* __restrict__ d_feat, const uint16_t* __restrict__ entry_pat,
    const FeatherTable tab) {
    constexpr int SG = BwdCfg<FC>::SG;
    constexpr int RS = 4 + ((1 + FC + 3) / 4) * 4;  // entry record floats (the forward's layout)
    extern __shared__ float4 s_mem4[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    float* s_go = reinterpret_cast<float*>(s_mem4) + warp * BwdCfg<FC>::SLOT;
    float* s_lw = reinterpret_cast<float*>(s_mem4) + BwdCfg<FC>::WARPS * BwdCfg<FC>::SLOT;
    if constexpr (WIN) {
        for (int i = threadIdx.x; i < 8 * kTile; i += BwdCfg<FC>::THREADS) s_lw[i] = tab.lw[i / kTile][i % kTile];
        __syncthreads();
    }
    const int n_items = *num_items;
    const int nty_frame = (H + kTile - 1) / kTile;  // tile rows of one frame (stacked frames)
    const uint32_t limit = static_cast<uint32_t>(n_items) - 1u;
    const int grid_warps = static_cast<int>(gridDim.x) * BwdCfg<FC>::WARPS;
    int item = static_cast<int>(blockIdx.x) * BwdCfg<FC>::WARPS + warp;
    while (item < n_items) {
        __syncwarp();  // the previous item's reads of s_go are done
        const int4 it = items[item];
        const int tile = it.x;
        const int first = it.y;
        const int r = it.z;
        const int tile_x = tile % ntx;
        const int tile_y = tile / ntx;  // row in the stacked frames' grid (the pair slot's coordinates)
        const int frame = FRAMES ? tile_y / nty_frame : 0;
        const int tx0 = tile_x * kTile;
        const int ty0 = (tile_y - frame * nty_frame) * kTile;
        const int nrow = min(kTile, H - ty0);
        const int ncol = min(kTile, W - tx0);

        // stage this tile's dL/dimage (zero outside the image): all of a lane's
        // loads are issued before any store, so staging costs one L2 round trip
        const int64_t plane = static_cast<int64_t>(H) * W;
        {
            constexpr int kPerLane = kTilePixels / 32;  // 8 pixels per lane and channel
            const float* gbase = grad_image + (FRAMES ? static_cast<int64_t>(frame) * F * plane : 0) +
                                 static_cast<int64_t>(ty0) * W + tx0;
#pragma unroll 1
            for (int c0 = 0; c0 < SG; c0 += 4) {  // groups of 4 channels: 32 loads in flight per lane
                float v[4][kPerLane];
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
#pragma unroll
                    for (int i = 0; i < kPerLane; ++i) {
                        const int p = i * 32 + lane;
                        const int ly = p >> 4, lx = p & (kTile - 1);
                        const int c = c0 + cc;
                        v[cc][i] = (c < F && ly < nrow && lx < ncol)
                                       ? __ldg(gbase + c * plane + static_cast<int64_t>(ly) * W + lx)
                                       : 0.0f;
                    }
                }
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
#pragma unroll
                    for (int i = 0; i < kPerLane; ++i) {
                        const int p = i * 32 + lane;
                        s_go[go_index<FC>(p >> 4, p & (kTile - 1), c0 + cc)] = v[cc][i];
                    }
                }
            }
        }
        __syncwarp();

        // lanes per entry (k) and this lane's entry and row band
        const int k = r > 16 ? 1 : (r > 8 ? 2 : (r > 4 ? 4 : (r > 2 ? 8 : 16)));
        const int e = lane / k;
        const int band = lane - e * k;
        const int rows_per = kTile / k;
        const int r0 = band * rows_per;
        const int r1 = min(r0 + rows_per, nrow);
        const bool active = e < r;

        int g = 0;
        int slot = 0;
        float4 g0 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        float4 g1 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        float fv[FC];
#pragma unroll
        for (int c = 0; c < FC; ++c) fv[c] = 0.0f;
        if (active) {  // idle lanes run on a neutral entry so the warp stays converged
            if (MODE == kDetRecords) {
                const float4* rec = reinterpret_cast<const float4*>(records + static_cast<int64_t>(first + e) * RS);
                g0 = rec[0];
                float rv[RS - 4];
#pragma unroll
                for (int v = 0; v < (RS - 4) / 4; ++v) {
                    const float4 t = rec[1 + v];
                    rv[4 * v + 0] = t.x;
                    rv[4 * v + 1] = t.y;
                    rv[4 * v + 2] = t.z;
                    rv[4 * v + 3] = t.w;
                }
                g1.x = rv[0];
#pragma unroll
                for (int c = 0; c < FC; ++c) fv[c] = rv[1 + c];
                if (slots != nullptr) {
                    slot = slots[first + e];
                } else {
                    g = gid_sorted[first + e];  // the slot is derived after the sums
                }
            } else {
                g = gid_sorted[first + e];
                const float4* rec = reinterpret_cast<const float4*>(geo + static_cast<int64_t>(g) * 8);
                g0 = rec[0];
                g1 = rec[1];
                const float op = opacity != nullptr ? opacity[g] : 1.0f;
                const float* fg = feat + static_cast<int64_t>(g) * F;
#pragma unroll
                for (int c = 0; c < FC; ++c) fv[c] = c < F ? fg[c] * op : 0.0f;
            }
        }
        // the same test on (-A, -B/2, -D) = k (a, b, d) with k = 0.5 log2(e) > 0 (records carry no raw conic)
        const bool regular = !active || regular_conic_bwd(g0.x, g0.y, -g0.z, -0.5f * g0.w, -g1.x);
        const bool warp_regular = __all_sync(0xffffffffu, regular);
        const float* lwx = nullptr;
        const float* lwy = nullptr;
        if constexpr (WIN) {
            const int pat = active ? static_cast<int>(entry_pat[first + e]) : 0;  // idle lanes: an all-zero window
            lwx = s_lw + (pat & 0xff) * kTile;
            lwy = s_lw + (pat >> 8) * kTile;
        }

        float dF[FC];
#pragma unroll
        for (int c = 0; c < FC; ++c) dF[c] = 0.0f;
        float Sx = 0.0f, Sy = 0.0f, Sxx = 0.0f, Sxy = 0.0f, Syy = 0.0f;
        const float A = g0.z, B = g0.w, D = g1.x;
        if (ncol == kTile) {
            const float fx0 = static_cast<float>(tx0), fy0 = static_cast<float>(ty0);
            if (warp_regular) {
                if constexpr (BwdCfg<FC>::PAIRED) {
                    bwd_rows_full_pk<FC, false, WIN>(s_go, r0, r1, fx0, fy0, g0.x, g0.y, A, B, D, fv, dF, Sx, Sy, Sxx,
                                                     Sxy, Syy, lwx, lwy);
                } else {
                    bwd_rows_full<FC, false, WIN>(s_go, r0, r1, fx0, fy0, g0.x, g0.y, A, B, D, fv, dF, Sx, Sy, Sxx, Sxy,
                                                  Syy, lwx, lwy);
                }
            } else {
                if constexpr (BwdCfg<FC>::PAIRED) {
                    bwd_rows_full_pk<FC, true, WIN>(s_go, r0, r1, fx0, fy0, g0.x, g0.y, A, B, D, fv, dF, Sx, Sy, Sxx,
                                                    Sxy, Syy, lwx, lwy);
                } else {
                    bwd_rows_full<FC, true, WIN>(s_go, r0, r1, fx0, fy0, g0.x, g0.y, A, B, D, fv, dF, Sx, Sy, Sxx, Sxy,
                                                 Syy, lwx, lwy);
                }
            }
        } else {
            bwd_rows_edge<FC, WIN>(s_go, r0, r1, ncol, tx0, ty0, g0.x, g0.y, A, B, D, fv, dF, Sx, Sy, Sxx, Sxy, Syy,
                                   lwx, lwy);
        }
        if (k > 1) {  // combine the k row bands of each entry (all lanes take part)
            Sx = group_sum(Sx, k);
            Sy = group_sum(Sy, k);
            Sxx = group_sum(Sxx, k);
            Sxy = group_sum(Sxy, k);
            Syy = group_sum(Syy, k);
#pragma unroll
            for (int c = 0; c < FC; ++c) dF[c] = group_sum(dF[c], k);
        }
        // the next item's index; its latency overlaps the epilogue's loads
        const int next = take_item(work, limit, grid_warps, lane);
        if (active && band == 0) {
            const float dca = -0.5f * Sxx;
            const float dcb = -Sxy;
            const float dcd = -0.5f * Syy;
            if (MODE != kAtomicGather) {
                if (MODE == kDetGather || slots == nullptr) {
                    const int4 box = aabb[g];
                    slot = pair_offset[g] + (tile_y - box.y) * (box.z - box.x) + (tile_x - box.x);
                }
                float* row = pairgrad + static_cast<int64_t>(slot) * pstride;
                if (FC <= 3) {
                    float4* row4 = reinterpret_cast<float4*>(row);
                    row4[0] = make_float4(Sx, Sy, dca, dcb);
                    row4[1] = make_float4(dcd, dF[0], FC > 1 ? dF[FC > 1 ? 1 : 0] : 0.0f,
                                          FC > 2 ? dF[FC > 2 ? 2 : 0] : 0.0f);
                } else {
                    row[0] = Sx;
                    row[1] = Sy;
                    row[2] = dca;
                    row[3] = dcb;
                    row[4] = dcd;
#pragma unroll
                    for (int c = 0; c < FC; ++c) {
                        if (c < F) row[5 + c] = dF[c];
                    }
                }
            } else {
                // raw conic (a, b, d) sits in g1.yzw
                atomicAdd(&d_xy[2 * g + 0], fmaf(g1.y, Sx, g1.z * Sy));
                atomicAdd(&d_xy[2 * g + 1], fmaf(g1.z, Sx, g1.w * Sy));
                atomicAdd(&d_conic[3 * g + 0], dca);
                atomicAdd(&d_conic[3 * g + 1], dcb);
                atomicAdd(&d_conic[3 * g + 2], dcd);
#pragma unroll
                for (int c = 0; c < FC; ++c) {
                    if (c < F) atomicAdd(&d_feat[static_cast<int64_t>(g) * F + c], dF[c]);
                }
            }
        }
        item = next;
    }
}

// Work items of the backward: every tile has ceil(L / 32) items of up to 32
// consecutive list entries, item = (tile, first entry, count).  The table lists
// them longest first, in three duration classes: items of 17..32 entries (one
// lane per entry over all 16 rows), of 9..16 (two lanes per entry, 8 rows
// each) and of 1..8 (4 rows or fewer); tile order within a class.  Two parallel
// launches build it: per block of kItemSpan tiles the item count of each class,
// then per block the prefix of the earlier blocks' counts, a block scan and the
// writes.  The last block also stores the item count and clears the backward's
// work counter.
constexpr int kItemThreads = 256;
constexpr int kItemTilesPerThread = 4;
constexpr int kItemSpan = kItemThreads * kItemTilesPerThread;
constexpr int kItemClasses = 3;

__device__ __forceinline__ int item_class(int count) { return count > 16 ? 0 : (count > 8 ? 1 : 2); }

// Items of each class for a list of len entries.
__device__ __forceinline__ void tile_item_counts(int len, int (&cnt)[kItemClasses]) {
    cnt[0] = len / kItemEntries;
    cnt[1] = 0;
    cnt[2] = 0;
    const int rest = len % kItemEntries;
    if (rest > 0) cnt[item_class(rest)] += 1;
}

// Exclusive block scan of one int per thread; `total` receives the block sum.
__device__ __forceinline__ int item_block_scan(int v, int* s_warp, int& total) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    int before = 0;
    total = 0;
#pragma unroll
    for (int w = 0; w < kItemThreads / 32; ++w) {
        const int c = s_warp[w];
        before += w < warp ? c : 0;
        total += c;
    }
    __syncthreads();
    return before + x - v;
}

__global__ void __launch_bounds__(kItemThreads) k_item_block_sums(int num_tiles,
                                                                   const int32_t* __restrict__ tile_offsets,
                                                                   int32_t* __restrict__ block_items) {
    __shared__ int s_warp[kItemThreads / 32];
    const int t0 = blockIdx.x * kItemSpan + threadIdx.x * kItemTilesPerThread;
    int local[kItemClasses] = {0, 0, 0};
#pragma unroll
    for (int k = 0; k < kItemTilesPerThread; ++k) {
        if (t0 + k < num_tiles) {
            int cnt[kItemClasses];
            tile_item_counts(tile_offsets[t0 + k + 1] - tile_offsets[t0 + k], cnt);
#pragma unroll
            for (int c = 0; c < kItemClasses; ++c) local[c] += cnt[c];
        }
    }
#pragma unroll
    for (int c = 0; c < kItemClasses; ++c) {
        int total;
        item_block_scan(local[c], s_warp, total);
        if (threadIdx.x == 0) block_items[blockIdx.x * kItemClasses + c] = total;
    }
}

__global__ void __launch_bounds__(kItemThreads) k_item_table(int num_tiles, const int32_t* __restrict__ tile_offsets,
                                                              const int32_t* __restrict__ block_items,
                                                              int4* __restrict__ items, int32_t* __restrict__ num_items,
                                                              uint32_t* __restrict__ work) {
    __shared__ int s_warp[kItemThreads / 32];
    // start of this block's run in each class: all items of the earlier classes,
    // then the earlier blocks' items of the class
    int before[kItemClasses] = {0, 0, 0}, all[kItemClasses] = {0, 0, 0};
    for (int b = threadIdx.x; b < static_cast<int>(gridDim.x); b += kItemThreads) {
#pragma unroll
        for (int c = 0; c < kItemClasses; ++c) {
            const int v = block_items[b * kItemClasses + c];
            all[c] += v;
            before[c] += b < static_cast<int>(blockIdx.x) ? v : 0;
        }
    }
    int run[kItemClasses];
    int class_base = 0;
#pragma unroll
    for (int c = 0; c < kItemClasses; ++c) {
        int earlier, total;
        item_block_scan(before[c], s_warp, earlier);
        item_block_scan(all[c], s_warp, total);
        run[c] = class_base + earlier;
        class_base += total;
    }
    const int t0 = blockIdx.x * kItemSpan + threadIdx.x * kItemTilesPerThread;
    int beg[kItemTilesPerThread + 1];
#pragma unroll
    for (int k = 0; k <= kItemTilesPerThread; ++k) beg[k] = t0 + k <= num_tiles ? tile_offsets[t0 + k] : 0;
    int local[kItemClasses] = {0, 0, 0};
#pragma unroll
    for (int k = 0; k < kItemTilesPerThread; ++k) {
        if (t0 + k < num_tiles) {
            int cnt[kItemClasses];
            tile_item_counts(beg[k + 1] - beg[k], cnt);
#pragma unroll
            for (int c = 0; c < kItemClasses; ++c) local[c] += cnt[c];
        }
    }
#pragma unroll
    for (int c = 0; c < kItemClasses; ++c) {
        int total;
        run[c] += item_block_scan(local[c], s_warp, total);
    }
#pragma unroll
    for (int k = 0; k < kItemTilesPerThread; ++k) {
        if (t0 + k >= num_tiles) continue;
        const int len = beg[k + 1] - beg[k];
        const int full = len / kItemEntries;
        for (int i = 0; i < full; ++i) items[run[0]++] = make_int4(t0 + k, beg[k] + i * kItemEntries, kItemEntries, 0);
        const int rest = len - full * kItemEntries;
        if (rest > 0) {
            const int c = item_class(rest);
            items[run[c]++] = make_int4(t0 + k, beg[k] + full * kItemEntries, rest, 0);
        }
    }
    if (blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) {
        *num_items = class_base;
        *work = 0u;
    }
}

template <int FC>
__global__ void __launch_bounds__(256) k_reduce_gaussian(int n, int F, const float* __restrict__ pairgrad, int pstride,
                                                         const int32_t* __restrict__ pair_offset,
                                                         const float* __restrict__ geo,
                                                         const float* __restrict__ feat,
                                                         const float* __restrict__ opacity,
                                                         const float* __restrict__ scale, const float* __restrict__ rot,
                                                         float* __restrict__ d_xy, float* __restrict__ d_conic,
                                                         float* __restrict__ d_feat, float* __restrict__ d_opacity,
                                                         float* __restrict__ d_scale, float* __restrict__ d_rot,
                                                         int rows_dxy, int vstride) {
    const int g = blockIdx.x * 256 + threadIdx.x;
    if (g >= n) return;
    // a Gaussian's rows: its vstride virtual Gaussians' rows, contiguous in gid-major order
    const int beg = pair_offset[static_cast<int64_t>(g) * vstride];
    const int end = pair_offset[static_cast<int64_t>(g + 1) * vstride];
    // per-Gaussian inputs of the epilogue, loaded ahead of the row sums so their
    // latency overlaps them
    const float4 k1 = reinterpret_cast<const float4*>(geo + static_cast<int64_t>(g) * 8)[1];
    const float op = opacity != nullptr ? opacity[g] : 1.0f;
    float2 sc = make_float2(0.0f, 0.0f);
    float th = 0.0f;
    if (d_scale != nullptr) {
        sc = make_float2(scale[2 * g], scale[2 * g + 1]);
        th = rot[g];
    }
    // the rows of a Gaussian are summed in double: a handful of adds per Gaussian,
    // and the per-pair partials often cancel
    double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0, s4 = 0.0;
    double dF[FC];
#pragma unroll
    for (int c = 0; c < FC; ++c) dF[c] = 0.0;
    if (FC <= 3) {
        // rows four at a time, all loads issued before the (in-order) sums
        for (int p = beg; p < end; p += 4) {
            float4 r0[4], r1[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (p + u < end) {
                    const float4* row = reinterpret_cast<const float4*>(pairgrad + static_cast<int64_t>(p + u) * pstride);
                    r0[u] = row[0];
                    r1[u] = row[1];
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (p + u < end) {
                    s0 += r0[u].x;
                    s1 += r0[u].y;
                    s2 += r0[u].z;
                    s3 += r0[u].w;
                    s4 += r1[u].x;
                    dF[0] += r1[u].y;
                    if (FC > 1) dF[FC > 1 ? 1 : 0] += r1[u].z;
                    if (FC > 2) dF[FC > 2 ? 2 : 0] += r1[u].w;
                }
            }
        }
    } else {
      for (int p = beg; p < end; ++p) {
        const float* row = pairgrad + static_cast<int64_t>(p) * pstride;
        {
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
    }
    // (s0, s1) = (sum Sx, sum Sy); the raw conic (a, b, d) is geo[g][5..7].  Rows of
    // weights other than exp(-q/2) hold d_xy itself (rows_dxy).
    d_xy[2 * g + 0] = static_cast<float>(rows_dxy ? s0 : static_cast<double>(k1.y) * s0 + static_cast<double>(k1.z) * s1);
    d_xy[2 * g + 1] = static_cast<float>(rows_dxy ? s1 : static_cast<double>(k1.z) * s0 + static_cast<double>(k1.w) * s1);
    const float c2 = static_cast<float>(s2), c3 = static_cast<float>(s3), c4 = static_cast<float>(s4);
    d_conic[3 * g + 0] = c2;
    d_conic[3 * g + 1] = c3;
    d_conic[3 * g + 2] = c4;
    double dop = 0.0;
#pragma unroll
    for (int c = 0; c < FC; ++c) {
        if (c < F) {
            const int64_t kk = static_cast<int64_t>(g) * F + c;
            d_feat[kk] = static_cast<float>(dF[c] * static_cast<double>(op));
            dop += dF[c] * static_cast<double>(feat[kk]);
        }
    }
    if (d_opacity != nullptr) d_opacity[g] = static_cast<float>(dop);
    if (d_scale != nullptr) {
        float dsx, dsy, dr;
        conic_grad_to_scale_rot_f64(sc.x, sc.y, th, s2, s3, s4, dsx, dsy, dr);
        d_scale[2 * g + 0] = dsx;
        d_scale[2 * g + 1] = dsy;
        d_rot[g] = dr;
    }
}

// Persistent grid of the backward: as many CTAs as fit on the device at once
// (cached per device), never more than the table's largest item count needs.
template <int FC, int MODE, bool WIN = false, bool FRAMES = false>
int bwd_grid(int64_t max_items, int smem) {
    static std::atomic<int> cached[64];  // 0 until queried; host threads may race to store the same value
    const int64_t need = div_up(max_items, BwdCfg<FC>::WARPS);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return static_cast<int>(need);
    int grid = cached[dev].load(std::memory_order_relaxed);
    if (grid == 0) {
        int sms = 0, per = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k_render_bwd<FC, MODE, WIN, FRAMES>, BwdCfg<FC>::THREADS,
                                                      smem);
        grid = sms > 0 && per > 0 ? sms * per : 1;
        cached[dev].store(grid, std::memory_order_relaxed);
    }
    return static_cast<int>(need < grid ? need : grid);
}

template <int FC, int MODE, bool FRAMES>
cudaError_t launch_bwd_mode(int f, int h, int w, int ntx, int64_t max_items, const float* geo, const float* feat,
                            const float* opacity, const int32_t* gid_sorted, const int4* items,
                            const int32_t* num_items, uint32_t* work, const float* grad_image, const int32_t* aabb,
                            const int32_t* pair_offset, const float* records, const int32_t* slots, float* pairgrad,
                            int pstride, float* d_xy, float* d_conic, float* d_feat, cudaStream_t stream) {
    const int smem = BwdCfg<FC>::WARPS * BwdCfg<FC>::SLOT * static_cast<int>(sizeof(float));
    auto kern = k_render_bwd<FC, MODE, false, FRAMES>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    const unsigned blocks = static_cast<unsigned>(bwd_grid<FC, MODE, false, FRAMES>(max_items, smem));
    kern<<<blocks, BwdCfg<FC>::THREADS, smem, stream>>>(
        f, h, w, ntx, geo, feat, opacity, gid_sorted, items, num_items, work, grad_image,
        reinterpret_cast<const int4*>(aabb), pair_offset, records, slots, pairgrad, pstride, d_xy, d_conic, d_feat,
        nullptr, FeatherTable{});
    return cudaGetLastError();
}

template <int FC>
cudaError_t launch_bwd_win(int f, int h, int w, int ntx, int64_t max_items, const int32_t* gid_sorted,
                           const int4* items, const int32_t* num_items, uint32_t* work, const float* grad_image,
                           const int32_t* aabb, const int32_t* pair_offset, const float* records,
                           const uint16_t* entry_pat, const FeatherTable& tab, float* pairgrad, int pstride,
                           cudaStream_t stream) {
    const int smem = (BwdCfg<FC>::WARPS * BwdCfg<FC>::SLOT + 8 * kTile) * static_cast<int>(sizeof(float));
    auto kern = k_render_bwd<FC, kDetRecords, true>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    const unsigned blocks = static_cast<unsigned>(bwd_grid<FC, kDetRecords, true>(max_items, smem));
    kern<<<blocks, BwdCfg<FC>::THREADS, smem, stream>>>(
        f, h, w, ntx, nullptr, nullptr, nullptr, gid_sorted, items, num_items, work, grad_image,
        reinterpret_cast<const int4*>(aabb), pair_offset, records, nullptr, pairgrad, pstride, nullptr, nullptr,
        nullptr, entry_pat, tab);
    return cudaGetLastError();
}

template <int FC, bool FRAMES>
cudaError_t launch_bwd_fc(int f, int h, int w, int ntx, int64_t max_items, const float* geo, const float* feat,
                          const float* opacity, const int32_t* gid_sorted, const int4* items, const int32_t* num_items,
                          uint32_t* work,
                          const float* grad_image, const int32_t* aabb, const int32_t* pair_offset,
                          const float* records, const int32_t* slots, float* pairgrad, int pstride, float* d_xy,
                          float* d_conic, float* d_feat, cudaStream_t stream) {
    if (pairgrad == nullptr) {
        return launch_bwd_mode<FC, kAtomicGather, FRAMES>(f, h, w, ntx, max_items, geo, feat, opacity, gid_sorted, items,
                                                  num_items, work, grad_image, aabb, pair_offset, records, slots, pairgrad,
                                                  pstride, d_xy, d_conic, d_feat, stream);
    }
    if (records != nullptr) {
        return launch_bwd_mode<FC, kDetRecords, FRAMES>(f, h, w, ntx, max_items, geo, feat, opacity, gid_sorted, items,
                                                num_items, work, grad_image, aabb, pair_offset, records, slots, pairgrad,
                                                pstride, d_xy, d_conic, d_feat, stream);
    }
    return launch_bwd_mode<FC, kDetGather, FRAMES>(f, h, w, ntx, max_items, geo, feat, opacity, gid_sorted, items, num_items,
                                           work, grad_image, aabb, pair_offset, records, slots, pairgrad, pstride, d_xy,
                                           d_conic, d_feat, stream);
}

template <int FC>
cudaError_t launch_reduce_fc(int n, int f, const float* pairgrad, int pstride, const int32_t* pair_offset,
                             const float* geo, const float* feat, const float* opacity, const float* scale,
                             const float* rot, float* d_xy, float* d_conic, float* d_feat, float* d_opacity,
                             float* d_scale, float* d_rot, bool rows_dxy, int vstride, cudaStream_t stream) {
    k_reduce_gaussian<FC><<<static_cast<unsigned>(div_up(n, 256)), 256, 0, stream>>>(
        n, f, pairgrad, pstride, pair_offset, geo, feat, opacity, scale, rot, d_xy, d_conic, d_feat, d_opacity,
        d_scale, d_rot, rows_dxy ? 1 : 0, vstride);
    return cudaGetLastError();
}

}  // namespace

int backward_pair_stride(int f) { return ((5 + f + 3) / 4) * 4; }

int64_t backward_max_items(int64_t total_pairs, int64_t num_tiles) {
    return num_tiles + (total_pairs + kItemEntries - 1) / kItemEntries;
}

int64_t backward_items_scratch_bytes(int64_t total_pairs, int64_t num_tiles) {
    return arena_bytes(backward_max_items(total_pairs, num_tiles), sizeof(int4)) + arena_bytes(2, sizeof(int32_t)) +
           arena_bytes(div_up(num_tiles, kItemSpan) * kItemClasses, sizeof(int32_t));
}

#define OSS_DISPATCH_FC(f, CALL) \
    ((f) <= 1 ? CALL(1) : (f) <= 3 ? CALL(3) : (f) <= 4 ? CALL(4) : (f) <= 8 ? CALL(8) : (f) <= 16 ? CALL(16) : (f) <= 32 ? CALL(32) : CALL(64))

cudaError_t launch_backward_items(int h, int w, int64_t total_pairs, const int32_t* tile_offsets, void* items_scratch,
                                  cudaStream_t stream, int frames) {
    const int ntx = static_cast<int>(div_up(w, kTile));
    const int nty = static_cast<int>(div_up(h, kTile));
    const int num_tiles = ntx * nty * frames;
    if (num_tiles == 0 || total_pairs == 0) return cudaSuccess;
    const int64_t max_items = backward_max_items(total_pairs, num_tiles);
    Arena arena{static_cast<char*>(items_scratch), backward_items_scratch_bytes(total_pairs, num_tiles), 0};
    int4* items = arena.take<int4>(max_items);
    int32_t* counters = arena.take<int32_t>(2);  // item count, the backward's work counter
    const int item_blocks = static_cast<int>(div_up(num_tiles, kItemSpan));
    int32_t* block_items = arena.take<int32_t>(static_cast<int64_t>(item_blocks) * kItemClasses);
    k_item_block_sums<<<static_cast<unsigned>(item_blocks), kItemThreads, 0, stream>>>(num_tiles, tile_offsets,
                                                                                         block_items);
    k_item_table<<<static_cast<unsigned>(item_blocks), kItemThreads, 0, stream>>>(
        num_tiles, tile_offsets, block_items, items, counters, reinterpret_cast<uint32_t*>(counters + 1));
    return cudaGetLastError();
}

cudaError_t launch_render_backward_items(int f, int h, int w, int64_t total_pairs, const float* geo,
                                         const float* feat, const float* opacity, const int32_t* gid_sorted,
                                         const int32_t* tile_offsets, const float* grad_image, const int32_t* aabb,
                                         const int32_t* pair_offset, const float* records, const int32_t* slots,
                                         float* pairgrad, int pair_stride, float* d_xy, float* d_conic, float* d_feat,
                                         void* items_scratch, cudaStream_t stream, int frames) {
    const int ntx = static_cast<int>(div_up(w, kTile));
    const int nty = static_cast<int>(div_up(h, kTile));
    const int num_tiles = ntx * nty * frames;
    if (num_tiles == 0 || total_pairs == 0) return cudaSuccess;
    const int64_t max_items = backward_max_items(total_pairs, num_tiles);
    Arena arena{static_cast<char*>(items_scratch), backward_items_scratch_bytes(total_pairs, num_tiles), 0};
    const int4* items = arena.take<int4>(max_items);
    int32_t* counters = arena.take<int32_t>(2);
    const int32_t* num_items = counters;
    uint32_t* work = reinterpret_cast<uint32_t*>(counters + 1);
#define OSS_BWD_CALL(FC)                                                                                          \
    (frames > 1 ? launch_bwd_fc<FC, true>(f, h, w, ntx, max_items, geo, feat, opacity, gid_sorted, items, num_items,  \
                                          work, grad_image, aabb, pair_offset, records, slots, pairgrad, pair_stride, \
                                          d_xy, d_conic, d_feat, stream)                                              \
                : launch_bwd_fc<FC, false>(f, h, w, ntx, max_items, geo, feat, opacity, gid_sorted, items,            \
                                           num_items, work, grad_image, aabb, pair_offset, records, slots, pairgrad,  \
                                           pair_stride, d_xy, d_conic, d_feat, stream))
    return OSS_DISPATCH_FC(f, OSS_BWD_CALL);
#undef OSS_BWD_CALL
}

cudaError_t launch_render_backward_feathered(int f, int h, int w, int64_t total_pairs, const FeatherTable& tab,
                                            const int32_t* gid_sorted, const int32_t* tile_offsets,
                                            const float* grad_image, const int32_t* vaabb, const int32_t* vpair_offset,
                                            const float* records, const uint16_t* entry_pat, float* pairgrad,
                                            int pair_stride, void* items_scratch, cudaStream_t stream) {
    (void)tile_offsets;
    const int ntx = static_cast<int>(div_up(w, kTile));
    const int nty = static_cast<int>(div_up(h, kTile));
    const int num_tiles = ntx * nty;
    if (num_tiles == 0 || total_pairs == 0) return cudaSuccess;
    const int64_t max_items = backward_max_items(total_pairs, num_tiles);
    Arena arena{static_cast<char*>(items_scratch), backward_items_scratch_bytes(total_pairs, num_tiles), 0};
    const int4* items = arena.take<int4>(max_items);
    int32_t* counters = arena.take<int32_t>(2);
    const int32_t* num_items = counters;
    uint32_t* work = reinterpret_cast<uint32_t*>(counters + 1);
#define OSS_BWD_WIN(FC)                                                                                           \
    launch_bwd_win<FC>(f, h, w, ntx, max_items, gid_sorted, items, num_items, work, grad_image, vaabb, vpair_offset, \
                       records, entry_pat, tab, pairgrad, pair_stride, stream)
    if (f <= 1) return OSS_BWD_WIN(1);
    if (f <= 3) return OSS_BWD_WIN(3);
    if (f <= 4) return OSS_BWD_WIN(4);
    if (f <= 8) return OSS_BWD_WIN(8);
    if (f <= 16) return OSS_BWD_WIN(16);
    return cudaErrorInvalidValue;
#undef OSS_BWD_WIN
}

cudaError_t launch_render_backward_tiles(int f, int h, int w, int64_t total_pairs, const float* geo, const float* feat,
                                         const float* opacity, const int32_t* gid_sorted,
                                         const int32_t* tile_offsets, const float* grad_image, const int32_t* aabb,
                                         const int32_t* pair_offset, const float* records, const int32_t* slots,
                                         float* pairgrad, int pair_stride, float* d_xy, float* d_conic, float* d_feat,
                                         void* items_scratch, cudaStream_t stream) {
    cudaError_t err = launch_backward_items(h, w, total_pairs, tile_offsets, items_scratch, stream);
    if (err != cudaSuccess) return err;
    return launch_render_backward_items(f, h, w, total_pairs, geo, feat, opacity, gid_sorted, tile_offsets, grad_image,
                                        aabb, pair_offset, records, slots, pairgrad, pair_stride, d_xy, d_conic, d_feat,
                                        items_scratch, stream);
}

cudaError_t launch_reduce_gaussian_grads(int n, int f, const float* pairgrad, int pair_stride,
                                         const int32_t* pair_offset, const float* geo, const float* feat,
                                         const float* opacity, const float* scale, const float* rot, float* d_xy,
                                         float* d_conic, float* d_feat, float* d_opacity, float* d_scale,
                                         float* d_rot, cudaStream_t stream, bool rows_dxy, int vstride) {
    if (n == 0) return cudaSuccess;
#define OSS_RED_CALL(FC)                                                                                          \
    launch_reduce_fc<FC>(n, f, pairgrad, pair_stride, pair_offset, geo, feat, opacity, scale, rot, d_xy, d_conic, \
                         d_feat, d_opacity, d_scale, d_rot, rows_dxy, vstride, stream)
    return OSS_DISPATCH_FC(f, OSS_RED_CALL);
#undef OSS_RED_CALL
}

}  // namespace oss
