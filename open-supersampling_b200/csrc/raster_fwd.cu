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
// [x, y, A, B | D, feat'(F) | zero padding] (entry_record_floats(F) floats), and,
// with `slots` non-null, the entry's gid-major pair slot pair_offset[g] +
// (local tile index).
//
// Staging is a gather through gid_sorted, and scattered loads cost one L1
// wavefront per distinct cache line per instruction: from geo, opacity, feat,
// aabb and pair_offset that is eight per entry, which made the staging, not
// the ex2 math, the larger part of the kernel.  With `prec` (the per-Gaussian
// packed records the preprocess writes, already in the entry-record layout)
// an entry costs one 32-byte line (two 16-byte loads at F <= 3), and the
// backward derives the slots itself.
//
// The reference zeroes a weight when q is non-finite or negative
// (rasterizer_fwd.cu:245).  A batch whose conics are all finite and
// well-conditioned (det >= 1e-3 * a * d, i.e. axis ratio below ~60) has
// q' <= 0 at every pixel even after fp32 rounding, so it runs without the
// per-pixel test; other batches keep it.
#include <atomic>

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

// The same test on the scaled record (A, B, D) = (a, 2b, d) * (-log2(e) / 2):
// the inequality scales by a positive factor, so only rounding (1e-7
// relative, against the 1e-3 margin) separates the two.
__device__ __forceinline__ bool regular_scaled(float x, float y, float A, float B, float D) {
    return regular_conic(x, y, -A, -0.5f * B, -D);
}

// True when the entry's weight is exactly 0 at every pixel of the tile whose
// pixel centres span [tx0, tx0 + 15] x [ty0, ty0 + 15]: the largest q' over
// that rectangle (a concave quadratic for a regular conic, so on a corner or at
// an edge's vertex) lies below -127, and ex2.approx.ftz flushes every 2^q' below
// 2^-126 to 0.  The 1.0 margin covers the fp32 rounding of q'.  Such entries
// add exact zeros, so the forward skips them; this is what the q = 176 lists of
// the exact binning mode carry in their outer tiles.
// Entry skipping pays off on long lists (the outer tiles of exact-mode lists);
// tiles with shorter lists do not test for it.
constexpr int kSkipMinList = 128;

__device__ __forceinline__ bool entry_zero_in_tile(float x, float y, float A, float B, float D, float tx0,
                                                   float ty0) {
    if (!(A < 0.0f && D < 0.0f)) return false;
    const float X0 = tx0 - x, X1 = X0 + static_cast<float>(kTile - 1);
    const float Y0 = ty0 - y, Y1 = Y0 + static_cast<float>(kTile - 1);
    if (X0 <= 0.0f && X1 >= 0.0f && Y0 <= 0.0f && Y1 >= 0.0f) return false;  // the centre is inside
    const float h2d = __fdividef(-0.5f, D), h2a = __fdividef(-0.5f, A);  // only moves the probe points
    float best = -INFINITY;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const float X = e == 0 ? X0 : X1;  // edge dx = X: dy* = -B X / (2 D)
        const float dy = fminf(fmaxf(B * X * h2d, Y0), Y1);
        best = fmaxf(best, fmaf(X, fmaf(A, X, B * dy), D * dy * dy));
        const float Y = e == 0 ? Y0 : Y1;  // edge dy = Y: dx* = -B Y / (2 A)
        const float dx = fminf(fmaxf(B * Y * h2a, X0), X1);
        best = fmaxf(best, fmaf(dx, fmaf(A, dx, B * Y), D * Y * Y));
    }
    return best < -127.0f;
}

template <int FC, bool CHECK, bool SKIP>
__device__ __forceinline__ void fwd_batch(int cnt, const float4* __restrict__ s_geo, const float* __restrict__ s_df,
                                          const unsigned char* __restrict__ s_skip,
                                          float fpx, const float (&fpy)[FwdCfg<FC>::PX],
                                          float (&acc)[FwdCfg<FC>::PX][FC]) {
    constexpr int PX = FwdCfg<FC>::PX;
    constexpr int S = FwdCfg<FC>::S;
#pragma unroll 2
    for (int j = 0; j < cnt; ++j) {
        if (SKIP && s_skip[j]) continue;  // exact zero at every pixel of the tile (same for every thread)
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

// Feather window of the one-pass overlapped render (csrc/feather.cu): per entry
// the phase-bit patterns of its tile column and row ranges (s_pat), and the
// tables of log2 window weights by pattern for this thread's column (s_lwx,
// [pattern][column]) and for its PX rows (s_lwy, [pattern][row step][PX]).
struct FwdWin {
    const uchar2* pat;
    const float* lwx;
    const float* lwy;
    int lx, ly;
};

// fwd_batch on pixel pairs: acc2[p][c] holds pixels 2p and 2p+1.  With WIN the
// log2 window weights of the entry's column and rows are added to q'.
template <int FC, bool CHECK, bool SKIP, bool WIN = false>
__device__ __forceinline__ void fwd_batch_pk(int cnt, const float4* __restrict__ s_geo,
                                             const float* __restrict__ s_df,
                                             const unsigned char* __restrict__ s_skip, float fpx,
                                             const float2 (&fpy2)[FwdCfg<FC>::PX / 2],
                                             float2 (&acc2)[FwdCfg<FC>::PX / 2][FC], FwdWin win = {}) {
    constexpr int PX = FwdCfg<FC>::PX;
    constexpr int NP = PX / 2;
    constexpr int S = FwdCfg<FC>::S;
    constexpr int ROWSTEP = kTile / PX;
#pragma unroll 4
    for (int j = 0; j < cnt; ++j) {
        if (SKIP && s_skip[j]) continue;  // exact zero at every pixel of the tile (same for every thread)
        float lw[PX];
        float lwc = 0.0f;
        if constexpr (WIN) {
            const uchar2 pt = win.pat[j];
            lwc = win.lwx[pt.x * kTile + win.lx];
            const float* ly = win.lwy + (pt.y * ROWSTEP + win.ly) * PX;
            if constexpr (PX == 4) {
                const float4 t = *reinterpret_cast<const float4*>(ly);
                lw[0] = t.x;
                lw[1] = t.y;
                lw[2 % PX] = t.z;
                lw[3 % PX] = t.w;
            } else {
#pragma unroll
                for (int k = 0; k < PX; ++k) lw[k] = ly[k];
            }
        }
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
        const float2 c2 = make_float2(adx2 + lwc, adx2 + lwc);
#pragma unroll
        for (int p = 0; p < NP; ++p) {
            const float2 dy = __fadd2_rn(fpy2[p], ngy);
            float2 w;
            if constexpr (WIN) {
                // q' with the window's log2 weights: the column's folded into the constant
                // term, the row's added per pixel pair
                const float2 t = __ffma2_rn(D2, dy, b2);
                const float2 q = __ffma2_rn(dy, t, __fadd2_rn(c2, make_float2(lw[2 * p], lw[2 * p + 1])));
                if (CHECK) {
                    const float2 q0 = __ffma2_rn(dy, t, a2);  // the reference's q >= 0 test, without the window
                    w.x = q0.x <= 0.0f ? ex2_ftz(q.x) : 0.0f;
                    w.y = q0.y <= 0.0f ? ex2_ftz(q.y) : 0.0f;
                } else {
                    w.x = ex2_ftz(q.x);
                    w.y = ex2_ftz(q.y);
                }
            } else {
                const float2 q = __ffma2_rn(dy, __ffma2_rn(D2, dy, b2), a2);
                if (CHECK) {
                    w.x = q.x <= 0.0f ? ex2_ftz(q.x) : 0.0f;
                    w.y = q.y <= 0.0f ? ex2_ftz(q.y) : 0.0f;
                } else {
                    w.x = ex2_ftz(q.x);
                    w.y = ex2_ftz(q.y);
                }
            }
#pragma unroll
            for (int c = 0; c < FC; ++c) acc2[p][c] = __ffma2_rn(w, make_float2(r[1 + c], r[1 + c]), acc2[p][c]);
        }
    }
}

// Batch loop with its per-pixel sign test only where a conic is irregular and
// its entry skip only where some entry of the batch is zero over the tile.
template <int FC, bool WIN = false>
__device__ __forceinline__ void fwd_batch_pk_sel(bool regular, bool skip, int cnt, const float4* s_geo,
                                                 const float* s_df, const unsigned char* s_skip, float fpx,
                                                 const float2 (&fpy2)[FwdCfg<FC>::PX / 2],
                                                 float2 (&acc2)[FwdCfg<FC>::PX / 2][FC], FwdWin win = {}) {
    if (regular) {
        if (skip) fwd_batch_pk<FC, false, true, WIN>(cnt, s_geo, s_df, s_skip, fpx, fpy2, acc2, win);
        else fwd_batch_pk<FC, false, false, WIN>(cnt, s_geo, s_df, s_skip, fpx, fpy2, acc2, win);
    } else {
        if (skip) fwd_batch_pk<FC, true, true, WIN>(cnt, s_geo, s_df, s_skip, fpx, fpy2, acc2, win);
        else fwd_batch_pk<FC, true, false, WIN>(cnt, s_geo, s_df, s_skip, fpx, fpy2, acc2, win);
    }
}

template <int FC>
__device__ __forceinline__ void fwd_batch_sel(bool regular, bool skip, int cnt, const float4* s_geo,
                                              const float* s_df, const unsigned char* s_skip, float fpx,
                                              const float (&fpy)[FwdCfg<FC>::PX],
                                              float (&acc)[FwdCfg<FC>::PX][FC]) {
    if (regular) {
        if (skip) fwd_batch<FC, false, true>(cnt, s_geo, s_df, s_skip, fpx, fpy, acc);
        else fwd_batch<FC, false, false>(cnt, s_geo, s_df, s_skip, fpx, fpy, acc);
    } else {
        if (skip) fwd_batch<FC, true, true>(cnt, s_geo, s_df, s_skip, fpx, fpy, acc);
        else fwd_batch<FC, true, false>(cnt, s_geo, s_df, s_skip, fpx, fpy, acc);
    }
}

template <int FC, bool FRAMES = false>
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
                                                                int32_t* __restrict__ slots,
                                                                const float* __restrict__ prec) {
    constexpr int PX = FwdCfg<FC>::PX;
    constexpr int NT = FwdCfg<FC>::NT;
    constexpr int S = FwdCfg<FC>::S;
    constexpr int BATCH = FwdCfg<FC>::BATCH;
    constexpr int ROWSTEP = kTile / PX;
    __shared__ float4 s_geo[BATCH];
    __shared__ __align__(16) float s_df[BATCH * S];
    __shared__ unsigned char s_skip[BATCH];

    // stacked frames: tile row trow is row trow - frame * nty of frame `frame`
    const int tile = blockIdx.x;
    const int nty = (H + kTile - 1) / kTile;
    const int trow = tile / ntx;
    const int frame = FRAMES ? trow / nty : 0;
    const int tx0 = (tile % ntx) * kTile;
    const int ty0 = (trow - frame * nty) * kTile;
    if (FRAMES) image += static_cast<int64_t>(frame) * F * H * W;
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
        bool skip_any = false;
        const bool try_skip = end - start > kSkipMinList;  // the same for the whole CTA
        for (int j = threadIdx.x; j < cnt; j += NT) {
            const int g = gid_sorted[b + j];
            const int e = b + j;
            float4* sdf4 = reinterpret_cast<float4*>(s_df + j * S);
            float4* rec = records != nullptr ? reinterpret_cast<float4*>(records + static_cast<int64_t>(e) * (4 + S))
                                             : nullptr;
            if (prec != nullptr) {
                // one packed record per entry: a single gathered cache line
                const float4* pr = reinterpret_cast<const float4*>(prec + static_cast<int64_t>(g) * (4 + S));
                const float4 g0 = pr[0];
                const float4 g1 = pr[1];
                s_geo[j] = g0;
                const bool reg = regular_scaled(g0.x, g0.y, g0.z, g0.w, g1.x);
                regular = regular && reg;
                const bool sk = try_skip && reg &&
                                entry_zero_in_tile(g0.x, g0.y, g0.z, g0.w, g1.x, static_cast<float>(tx0),
                                                   static_cast<float>(ty0));
                s_skip[j] = sk;
                skip_any = skip_any || sk;
                sdf4[0] = g1;
                if (rec != nullptr) {
                    rec[0] = g0;
                    rec[1] = g1;
                }
#pragma unroll
                for (int v = 1; v < S / 4; ++v) {
                    const float4 t = pr[1 + v];
                    sdf4[v] = t;
                    if (rec != nullptr) rec[1 + v] = t;
                }
            } else {
                const float4* gr = reinterpret_cast<const float4*>(geo + static_cast<int64_t>(g) * 8);
                const float4 g0 = gr[0];
                const float4 g1 = gr[1];
                s_geo[j] = g0;
                const bool reg = regular_conic(g0.x, g0.y, g1.y, g1.z, g1.w);
                regular = regular && reg;
                const bool sk = try_skip && reg &&
                                entry_zero_in_tile(g0.x, g0.y, g0.z, g0.w, g1.x, static_cast<float>(tx0),
                                                   static_cast<float>(ty0));
                s_skip[j] = sk;
                skip_any = skip_any || sk;
                const float op = opacity != nullptr ? opacity[g] : 1.0f;
                float* df = s_df + j * S;
                df[0] = g1.x;
                const float* fg = feat + static_cast<int64_t>(g) * F;
#pragma unroll
                for (int c = 0; c < FC; ++c) df[1 + c] = c < F ? fg[c] * op : 0.0f;
#pragma unroll
                for (int c = 1 + FC; c < S; ++c) df[c] = 0.0f;
                if (rec != nullptr) {
                    rec[0] = g0;
#pragma unroll
                    for (int v = 0; v < S / 4; ++v) rec[1 + v] = sdf4[v];
                }
            }
            if (slots != nullptr) {
                const int4 box = aabb[g];
                slots[e] = pair_offset[g] + (tile / ntx - box.y) * (box.z - box.x) + (tile % ntx - box.x);
            }
        }
        const bool all_regular = __syncthreads_and(regular ? 1 : 0) != 0;
        const bool any_skip = try_skip && __syncthreads_or(skip_any ? 1 : 0) != 0;
        if constexpr (PK) {
            fwd_batch_pk_sel<FC>(all_regular, any_skip, cnt, s_geo, s_df, s_skip, fpx, fpy2, acc2);
        } else {
            fwd_batch_sel<FC>(all_regular, any_skip, cnt, s_geo, s_df, s_skip, fpx, fpy, acc);
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

// ---------------------------------------------------------------------------
// Persistent, software-pipelined variant for packed records (F <= 4).
//
// With one CTA per tile, the CTAs an SM holds start together, stage together
// (the MUFU idle) and compute together, wave after wave.  Here a CTA walks the
// tiles blockIdx.x, +gridDim.x, ... and, while it computes tile i, tile i+1's
// records are already on their way into the other shared-memory buffer
// (cp.async, 16-byte global -> shared copies that hold no registers).  The
// gids of tile i+2 and the list offsets of tile i+3 are loaded into registers
// a step earlier still, so no dependent global load waits in front of the
// math.  Lists longer than PBATCH entries stage their later batches in place.
// ---------------------------------------------------------------------------
constexpr int kPipeBatch = 128;


// With WIN (the one-pass feathered render, csrc/feather.cu) every entry also
// carries its virtual Gaussian's packed phase ranges (win, staged beside the
// record), from which the staging pass derives the entry's phase-bit patterns
// for this tile (and stores them for the backward in entry_pat, with the
// records); the math adds the tabulated log2 window weights to q'.
// FRAMES: the tiles are those of stacked frames (a tile row's frame is decoded
// and the image is [frames][F][H][W]); a separate instance, so the one-frame
// kernel carries none of it.
template <int FC, bool WIN, bool FRAMES = false>
__global__ void __launch_bounds__(FwdCfg<FC>::NT) k_render_fwd_pipe(int F, int H, int W, int ntx, int num_tiles,
                                                                     const float* __restrict__ prec,
                                                                     const int32_t* __restrict__ gid_sorted,
                                                                     const int32_t* __restrict__ tile_offsets,
                                                                     float* __restrict__ image,
                                                                     float* __restrict__ records,
                                                                     const int4* __restrict__ win,
                                                                     uint16_t* __restrict__ entry_pat,
                                                                     const FeatherTable tab) {
    constexpr int PX = FwdCfg<FC>::PX;
    static_assert(PX % 2 == 0, "pipelined forward runs the packed pixel-pair path");
    constexpr int NT = FwdCfg<FC>::NT;
    constexpr int S = FwdCfg<FC>::S;
    constexpr int RS = 4 + S;               // record floats
    constexpr int PB = kPipeBatch;
    constexpr int PER = PB / NT;             // entries per thread and batch
    constexpr int ROWSTEP = kTile / PX;
    constexpr int NP = PX / 2;
    constexpr int WB = WIN ? PB : 1;
    __shared__ float4 s_geo[2][PB];
    __shared__ __align__(16) float s_df[2][PB * S];
    __shared__ unsigned char s_skip[2][PB];
    __shared__ int4 s_win[2][WB];
    __shared__ uchar2 s_pat[2][WB];
    __shared__ __align__(16) float s_lwx[WIN ? 8 * kTile : 1];
    __shared__ __align__(16) float s_lwy[WIN ? 8 * kTile : 1];

    const int G = gridDim.x;
    const int lx = threadIdx.x & (kTile - 1);
    const int ly = threadIdx.x >> 4;
    const int nty_frame = (H + kTile - 1) / kTile;
    if constexpr (WIN) {
        // window tables: by column, and by this thread layout's rows (pattern, row step, PX rows)
        for (int i = threadIdx.x; i < 8 * kTile; i += NT) {
            const int p = i / kTile, c = i % kTile;
            s_lwx[i] = tab.lw[p][c];
            const int l = c / PX, k = c % PX;  // s_lwy[(p * ROWSTEP + l) * PX + k] = row l + k * ROWSTEP
            s_lwy[i] = tab.lw[p][l + k * ROWSTEP];
        }
    }

    // register pipeline: offsets of the current, next and next-but-one tile, gids of the next
    int t = blockIdx.x;
    int oc0 = 0, oc1 = 0, on0 = 0, on1 = 0, oq0 = 0, oq1 = 0;
    if (t < num_tiles) { oc0 = tile_offsets[t]; oc1 = tile_offsets[t + 1]; }
    if (t + G < num_tiles) { on0 = tile_offsets[t + G]; on1 = tile_offsets[t + G + 1]; }
    if (t + 2 * G < num_tiles) { oq0 = tile_offsets[t + 2 * G]; oq1 = tile_offsets[t + 2 * G + 1]; }
    int gn[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        const int j = threadIdx.x + k * NT;
        gn[k] = j < min(PB, on1 - on0) ? gid_sorted[on0 + j] : 0;
    }
    // prologue: the first tile's first batch into buffer 0
    {
        const int cnt = min(PB, oc1 - oc0);
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            const int j = threadIdx.x + k * NT;
            if (j < cnt) {
                const int g = gid_sorted[oc0 + j];
                const float4* pr = reinterpret_cast<const float4*>(prec + static_cast<int64_t>(g) * RS);
                cp_async16(&s_geo[0][j], pr);
#pragma unroll
                for (int v = 0; v < S / 4; ++v) cp_async16(&s_df[0][j * S + 4 * v], pr + 1 + v);
                if constexpr (WIN) cp_async16(&s_win[0][j], win + g);
            }
        }
        cp_async_commit();
    }

    for (int it = 0; t < num_tiles; t += G, ++it) {
        const int buf = it & 1;
        // 1. next tile's first batch into the other buffer (its readers finished at the last barrier)
        {
            const int cnt = min(PB, on1 - on0);
#pragma unroll
            for (int k = 0; k < PER; ++k) {
                const int j = threadIdx.x + k * NT;
                if (t + G < num_tiles && j < cnt) {
                    const float4* pr = reinterpret_cast<const float4*>(prec + static_cast<int64_t>(gn[k]) * RS);
                    cp_async16(&s_geo[buf ^ 1][j], pr);
#pragma unroll
                    for (int v = 0; v < S / 4; ++v) cp_async16(&s_df[buf ^ 1][j * S + 4 * v], pr + 1 + v);
                    if constexpr (WIN) cp_async16(&s_win[buf ^ 1][j], win + gn[k]);
                }
            }
            cp_async_commit();
        }
        // 2. gids of the tile after next, offsets of the one after that
        {
            const int cnt = min(PB, oq1 - oq0);
#pragma unroll
            for (int k = 0; k < PER; ++k) {
                const int j = threadIdx.x + k * NT;
                gn[k] = (t + 2 * G < num_tiles && j < cnt) ? gid_sorted[oq0 + j] : 0;
            }
        }
        const int cur0 = oc0, cur1 = oc1;
        oc0 = on0; oc1 = on1; on0 = oq0; on1 = oq1;
        if (t + 3 * G < num_tiles) {
            oq0 = tile_offsets[t + 3 * G];
            oq1 = tile_offsets[t + 3 * G + 1];
        } else {
            oq0 = 0;
            oq1 = 0;
        }

        // stacked frames: tile row trow is row trow - frame * nty of frame `frame`
        const int trow = t / ntx;
        const int frame = FRAMES ? trow / nty_frame : 0;
        const int tx0 = (t % ntx) * kTile;
        const int ty0 = (trow - frame * nty_frame) * kTile;
        const float fpx = static_cast<float>(tx0 + lx);
        float2 fpy2[NP];
#pragma unroll
        for (int q = 0; q < NP; ++q) {
            fpy2[q] = make_float2(static_cast<float>(ty0 + ly + 2 * q * ROWSTEP),
                                  static_cast<float>(ty0 + ly + (2 * q + 1) * ROWSTEP));
        }
        float2 acc2[NP][FC];
#pragma unroll
        for (int q = 0; q < NP; ++q)
#pragma unroll
            for (int c = 0; c < FC; ++c) acc2[q][c] = make_float2(0.0f, 0.0f);

        // 3. this tile's first batch: own copies done, entry records out, then everyone's visible
        cp_async_wait_one();
        const int n0 = min(PB, cur1 - cur0);
        bool regular = true;
        bool skip_any = false;
        const bool try_skip = cur1 - cur0 > kSkipMinList;  // the same for the whole CTA
        const int tile_x = t % ntx, tile_y = trow - frame * nty_frame;
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            const int j = threadIdx.x + k * NT;
            if (j < n0) {
                const float4 g0 = s_geo[buf][j];
                const float4* d4 = reinterpret_cast<const float4*>(&s_df[buf][j * S]);
                const bool reg = regular_scaled(g0.x, g0.y, g0.z, g0.w, d4[0].x);
                regular = regular && reg;
                bool sk = try_skip && reg &&
                          entry_zero_in_tile(g0.x, g0.y, g0.z, g0.w, d4[0].x, static_cast<float>(tx0),
                                             static_cast<float>(ty0));
                if constexpr (WIN) {
                    const int4 wv = s_win[buf][j];
                    const int px_ = feather_pattern(wv.x, wv.y, tile_x), py_ = feather_pattern(wv.z, wv.w, tile_y);
                    s_pat[buf][j] = make_uchar2(static_cast<unsigned char>(px_), static_cast<unsigned char>(py_));
                    sk = sk || px_ == 0 || py_ == 0;  // the window is zero over the whole tile
                    if (entry_pat != nullptr) entry_pat[cur0 + j] = static_cast<uint16_t>(px_ | (py_ << 8));
                }
                s_skip[buf][j] = sk;
                skip_any = skip_any || sk;
                if (records != nullptr) {
                    float4* rec = reinterpret_cast<float4*>(records + static_cast<int64_t>(cur0 + j) * RS);
                    rec[0] = g0;
#pragma unroll
                    for (int v = 0; v < S / 4; ++v) rec[1 + v] = d4[v];
                }
            }
        }
        const bool gate = WIN || try_skip;
        bool all_regular = __syncthreads_and(regular ? 1 : 0) != 0;
        bool any_skip = gate && __syncthreads_or(skip_any ? 1 : 0) != 0;
        const FwdWin fw{s_pat[buf], s_lwx, s_lwy, lx, ly};
        fwd_batch_pk_sel<FC, WIN>(all_regular, any_skip, n0, s_geo[buf], s_df[buf], s_skip[buf], fpx, fpy2, acc2, fw);
        // 4. later batches of a long list, staged in place
        for (int b = cur0 + PB; b < cur1; b += PB) {
            const int cnt = min(PB, cur1 - b);
            __syncthreads();  // the previous batch has been consumed
            bool reg = true;
            bool skp = false;
            for (int j = threadIdx.x; j < cnt; j += NT) {
                const int e = b + j;
                const float4* pr = reinterpret_cast<const float4*>(prec + static_cast<int64_t>(gid_sorted[e]) * RS);
                const float4 g0 = pr[0];
                s_geo[buf][j] = g0;
                float4* d4 = reinterpret_cast<float4*>(&s_df[buf][j * S]);
#pragma unroll
                for (int v = 0; v < S / 4; ++v) d4[v] = pr[1 + v];
                const bool rg = regular_scaled(g0.x, g0.y, g0.z, g0.w, d4[0].x);
                reg = reg && rg;
                bool sk = try_skip && rg &&
                          entry_zero_in_tile(g0.x, g0.y, g0.z, g0.w, d4[0].x, static_cast<float>(tx0),
                                             static_cast<float>(ty0));
                if constexpr (WIN) {
                    const int4 wv = win[gid_sorted[e]];
                    const int px_ = feather_pattern(wv.x, wv.y, tile_x), py_ = feather_pattern(wv.z, wv.w, tile_y);
                    s_pat[buf][j] = make_uchar2(static_cast<unsigned char>(px_), static_cast<unsigned char>(py_));
                    sk = sk || px_ == 0 || py_ == 0;
                    if (entry_pat != nullptr) entry_pat[e] = static_cast<uint16_t>(px_ | (py_ << 8));
                }
                s_skip[buf][j] = sk;
                skp = skp || sk;
                if (records != nullptr) {
                    float4* rec = reinterpret_cast<float4*>(records + static_cast<int64_t>(e) * RS);
                    rec[0] = g0;
#pragma unroll
                    for (int v = 0; v < S / 4; ++v) rec[1 + v] = d4[v];
                }
            }
            all_regular = __syncthreads_and(reg ? 1 : 0) != 0;
            any_skip = gate && __syncthreads_or(skp ? 1 : 0) != 0;
            fwd_batch_pk_sel<FC, WIN>(all_regular, any_skip, cnt, s_geo[buf], s_df[buf], s_skip[buf], fpx, fpy2, acc2,
                                      fw);
        }
        // 5. image
        const int px = tx0 + lx;
        if (px < W) {
            const int64_t plane = static_cast<int64_t>(H) * W;
            // the frame again from t: keeping it live across the sums costs a register
            float* __restrict__ img = FRAMES ? image + static_cast<int64_t>((t / ntx) / nty_frame) * F * plane : image;
#pragma unroll
            for (int q = 0; q < NP; ++q) {
#pragma unroll
                for (int h2 = 0; h2 < 2; ++h2) {
                    const int py = ty0 + ly + (2 * q + h2) * ROWSTEP;
                    if (py < H) {
                        const int64_t pix = static_cast<int64_t>(py) * W + px;
#pragma unroll
                        for (int c = 0; c < FC; ++c) {
                            if (c < F) img[c * plane + pix] = h2 == 0 ? acc2[q][c].x : acc2[q][c].y;
                        }
                    }
                }
            }
        }
        __syncthreads();  // buffer `buf` is free for the prefetch two tiles on
    }
}

// CTAs per SM the pipelined forward runs with (queried once per device).
template <int FC, bool WIN = false, bool FRAMES = false>
int pipe_grid(int num_tiles) {
    static std::atomic<int> cached[64];  // 0 until queried; host threads may race to store the same value
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return num_tiles;
    int grid = cached[dev].load(std::memory_order_relaxed);
    if (grid == 0) {
        int sms = 0, per = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k_render_fwd_pipe<FC, WIN, FRAMES>, FwdCfg<FC>::NT, 0);
        grid = sms > 0 && per > 0 ? sms * per : 1;
        cached[dev].store(grid, std::memory_order_relaxed);
    }
    return num_tiles < grid ? num_tiles : grid;
}

template <int FC, bool FRAMES>
cudaError_t launch_fwd_fc(int f, int h, int w, int ntx, int num_tiles, const float* geo, const float* feat,
                          const float* opacity, const int32_t* gid_sorted, const int32_t* tile_offsets, float* image,
                          const int32_t* aabb, const int32_t* pair_offset, float* records, int32_t* slots,
                          const float* prec, cudaStream_t stream) {
    if constexpr (FwdCfg<FC>::PX % 2 == 0) {
        if (prec != nullptr && slots == nullptr) {
            k_render_fwd_pipe<FC, false, FRAMES>
                <<<static_cast<unsigned>(pipe_grid<FC, false, FRAMES>(num_tiles)), FwdCfg<FC>::NT, 0, stream>>>(
                    f, h, w, ntx, num_tiles, prec, gid_sorted, tile_offsets, image, records, nullptr, nullptr,
                    FeatherTable{});
            return cudaGetLastError();
        }
    }
    k_render_fwd<FC, FRAMES><<<static_cast<unsigned>(num_tiles), FwdCfg<FC>::NT, 0, stream>>>(
        f, h, w, ntx, geo, feat, opacity, gid_sorted, tile_offsets, image, reinterpret_cast<const int4*>(aabb),
        pair_offset, records, slots, prec);
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

cudaError_t launch_render_forward_feathered(int f, int h, int w, const FeatherTable& tab, const float* vprec,
                                           const int32_t* vwin, const int32_t* gid_sorted, const int32_t* tile_offsets,
                                           float* image, float* records, uint16_t* entry_pat, cudaStream_t stream) {
    const int ntx = static_cast<int>(div_up(w, kTile));
    const int nty = static_cast<int>(div_up(h, kTile));
    const int num_tiles = ntx * nty;
    if (num_tiles == 0 || f == 0) return cudaSuccess;
    const int4* win = reinterpret_cast<const int4*>(vwin);
#define OSS_FWD_WIN(FC)                                                                                            \
    (k_render_fwd_pipe<FC, true><<<static_cast<unsigned>(pipe_grid<FC, true>(num_tiles)), FwdCfg<FC>::NT, 0,      \
                                   stream>>>(f, h, w, ntx, num_tiles, vprec, gid_sorted, tile_offsets, image,      \
                                             records, win, entry_pat, tab),                                        \
     cudaGetLastError())
    if (f <= 1) return OSS_FWD_WIN(1);
    if (f <= 3) return OSS_FWD_WIN(3);
    if (f <= 4) return OSS_FWD_WIN(4);
    if (f <= 8) return OSS_FWD_WIN(8);
    if (f <= 16) return OSS_FWD_WIN(16);
    return cudaErrorInvalidValue;  // the feathered render takes at most 16 channels per call
#undef OSS_FWD_WIN
}

cudaError_t launch_render_forward(int f, int h, int w, const float* geo, const float* feat, const float* opacity,
                                  const int32_t* gid_sorted, const int32_t* tile_offsets, float* image,
                                  const int32_t* aabb, const int32_t* pair_offset, float* records, int32_t* slots,
                                  const float* prec, cudaStream_t stream, int frames) {
    const int ntx = static_cast<int>(div_up(w, kTile));
    const int nty = static_cast<int>(div_up(h, kTile));
    const int num_tiles = ntx * nty * frames;
    if (num_tiles == 0 || f == 0) return cudaSuccess;
#define OSS_FWD_CALL(FC)                                                                                           \
    (frames > 1 ? launch_fwd_fc<FC, true>(f, h, w, ntx, num_tiles, geo, feat, opacity, gid_sorted, tile_offsets,    \
                                          image, aabb, pair_offset, records, slots, prec, stream)                   \
                : launch_fwd_fc<FC, false>(f, h, w, ntx, num_tiles, geo, feat, opacity, gid_sorted, tile_offsets,   \
                                           image, aabb, pair_offset, records, slots, prec, stream))
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
