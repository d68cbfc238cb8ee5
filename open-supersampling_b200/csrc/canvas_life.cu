// The persistent canvas's per-frame lifecycle around the render
// (oss/gaussian/canvas/canvas.py:191-295): per-tile error of the render against
// the upsampled LR frame (error_detection.py:26-63), per-Gaussian error and age
// (error_detection.py:66-113, canvas.py:246-270), the prune decision tree with
// its error quantiles and per-frame budget (prune_spawn.py:72-157), the
// spawn-tile ranking (prune_spawn.py:165-208) and the prune/spawn slot update
// (prune_spawn.py:216-255).
//
// Everything stays on the device: quantiles, compaction and ranking come from
// the stable radix sort and the scan of this library, so a frame's update needs
// no host round trip until its statistics are read.
//
// * Tile error: one CTA per tile; the LR frame is upsampled on the fly
//   (F.interpolate bilinear, align_corners=False), so the HR target is never
//   materialised.  Per pixel the channel mean, then the tile mean, as the
//   reference's mean(dim=0) and avg_pool2d.
// * Quantiles follow torch.quantile (linear): rank = q * (m - 1) in fp32, the
//   two neighbours of the ascending sort, and torch's lerp (fused
//   multiply-adds; the weight picks the end it starts from); NaN if any value
//   is NaN.
// * The prune cap orders the selected slots by priority * 1e6 + error
//   (non-finite errors as 1e30) descending, ties in slot order -- a stable sort;
//   under the cap the selection is in slot order, as nonzero() gives it.
// * Spawn tiles: the largest tile errors first (ties in tile order), as many
//   as there are finite eligible tiles, at most n_tiles.
#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

constexpr int kThreads = 256;

// The LR frame and its bilinear map onto the HR grid.
struct LrFrame {
    const float* p;  // [f][hl][wl]
    int hl, wl, h, w;
    float sy, sx;  // hl / h, wl / w
    int same;      // already at the HR size: read it directly
};

// Bilinear taps of HR texel (i, j) in F.interpolate(frame, (h, w), bilinear,
// align_corners=False): LR offsets of the four neighbours and their weights.
struct Taps {
    int o00, o01, o10, o11;
    float lx0, lx1, ly0, ly1;
};

__device__ __forceinline__ Taps taps_at(const LrFrame& f, int i, int j) {
    Taps t;
    if (f.same) {
        t.o00 = t.o01 = t.o10 = t.o11 = i * f.wl + j;
        t.lx0 = t.ly0 = 1.0f;
        t.lx1 = t.ly1 = 0.0f;
        return t;
    }
    float sy = __fsub_rn(__fmul_rn(f.sy, __fadd_rn(static_cast<float>(i), 0.5f)), 0.5f);
    if (sy < 0.0f) sy = 0.0f;
    float sx = __fsub_rn(__fmul_rn(f.sx, __fadd_rn(static_cast<float>(j), 0.5f)), 0.5f);
    if (sx < 0.0f) sx = 0.0f;
    const int y0 = static_cast<int>(sy), x0 = static_cast<int>(sx);
    const int y1 = y0 + (y0 < f.hl - 1 ? 1 : 0), x1 = x0 + (x0 < f.wl - 1 ? 1 : 0);
    t.ly1 = __fsub_rn(sy, static_cast<float>(y0));
    t.lx1 = __fsub_rn(sx, static_cast<float>(x0));
    t.ly0 = __fsub_rn(1.0f, t.ly1);
    t.lx0 = __fsub_rn(1.0f, t.lx1);
    t.o00 = y0 * f.wl + x0;
    t.o01 = y0 * f.wl + x1;
    t.o10 = y1 * f.wl + x0;
    t.o11 = y1 * f.wl + x1;
    return t;
}

__device__ __forceinline__ float bilerp(const Taps& t, float v00, float v01, float v10, float v11) {
    const float top = __fadd_rn(__fmul_rn(t.lx0, v00), __fmul_rn(t.lx1, v01));
    const float bot = __fadd_rn(__fmul_rn(t.lx0, v10), __fmul_rn(t.lx1, v11));
    return __fadd_rn(__fmul_rn(t.ly0, top), __fmul_rn(t.ly1, bot));
}

// Fixed-order block sum (warp trees, then the warp totals in warp order).
__device__ float block_sum(float v, float* s_warp) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) s_warp[warp] = v;
    __syncthreads();
    float t = 0.0f;
    for (int k = 0; k < static_cast<int>(blockDim.x >> 5); ++k) t += s_warp[k];
    return t;
}

// Squared difference of pixel (y, x) summed over channels [c0, c0 + NC): every
// load of the NC channels is issued before the first is used.
template <int NC>
__device__ __forceinline__ float pixel_sq(const float* __restrict__ rendered, int64_t plane, int64_t pix,
                                          const LrFrame& f, const Taps& t, int c0, int F, float s) {
    const int64_t lplane = static_cast<int64_t>(f.hl) * f.wl;
    float r[NC], v[NC][4];
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        const int c = c0 + k < F ? c0 + k : F - 1;
        const float* lp = f.p + c * lplane;
        r[k] = __ldg(rendered + c * plane + pix);
        v[k][0] = __ldg(lp + t.o00);
        v[k][1] = __ldg(lp + t.o01);
        v[k][2] = __ldg(lp + t.o10);
        v[k][3] = __ldg(lp + t.o11);
    }
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        if (c0 + k < F) {
            const float d = __fsub_rn(r[k], f.same ? v[k][0] : bilerp(t, v[k][0], v[k][1], v[k][2], v[k][3]));
            s = __fadd_rn(s, __fmul_rn(d, d));
        }
    }
    return s;
}

// One CTA per tile.  Per pixel the channel mean of the squared difference to the
// target texel, then the tile mean; channels run in groups of NC (F itself up to
// 4) whose loads are all in flight together.
template <int NC>
__global__ void __launch_bounds__(kThreads) k_tile_mse(int F, int H, int W, int ts, int ntx,
                                                       const float* __restrict__ rendered, LrFrame tgt,
                                                       float* __restrict__ tile_err) {
    __shared__ float s_warp[kThreads / 32];
    const int tile = blockIdx.x;
    const int ty = tile / ntx, tx = tile - (tile / ntx) * ntx;
    const int64_t plane = static_cast<int64_t>(H) * W;
    const float ff = static_cast<float>(F);
    float acc = 0.0f;
    for (int p = threadIdx.x; p < ts * ts; p += kThreads) {
        const int y = ty * ts + p / ts, x = tx * ts + p % ts;
        const int64_t pix = static_cast<int64_t>(y) * W + x;
        const Taps t = taps_at(tgt, y, x);
        float s = 0.0f;
        for (int c0 = 0; c0 < F; c0 += NC) s = pixel_sq<NC>(rendered, plane, pix, tgt, t, c0, F, s);
        acc += __fdiv_rn(s, ff);
    }
    const float total = block_sum(acc, s_warp);
    if (threadIdx.x == 0) tile_err[tile] = __fdiv_rn(total, static_cast<float>(ts * ts));
}

// The 16x16-tile path for an LR frame at most the render's size (or the same
// size): a CTA of 64 threads per tile, each thread four adjacent pixels of one
// row read as a float4 per channel, and the LR texels the tile's taps touch
// (at most 18 x 18 per channel when upsampling) staged in shared memory once.
constexpr int kMseThreads = 64;
constexpr int kPatch = 18;

__device__ __forceinline__ float src_coord(float scale, int i) {
    const float v = __fsub_rn(__fmul_rn(scale, __fadd_rn(static_cast<float>(i), 0.5f)), 0.5f);
    return v < 0.0f ? 0.0f : v;
}

template <int NC, bool SAME>
__global__ void __launch_bounds__(kMseThreads) k_tile_mse16(int F, int H, int W, int ntx,
                                                            const float* __restrict__ rendered, LrFrame tgt,
                                                            float* __restrict__ tile_err) {
    __shared__ float s_lr[NC][kPatch][kPatch];
    __shared__ float s_warp[kMseThreads / 32];
    const int tile = blockIdx.x;
    const int ty = tile / ntx, tx = tile - (tile / ntx) * ntx;
    const int y = ty * 16 + (threadIdx.x >> 2);
    const int xq = tx * 16 + (threadIdx.x & 3) * 4;
    const int64_t plane = static_cast<int64_t>(H) * W;
    const int64_t pix = static_cast<int64_t>(y) * W + xq;
    // this thread's row taps and the patch origin (the tile's first source texel)
    int py0 = 0, py1 = 0;
    float wy0 = 1.0f, wy1 = 0.0f;
    int oy = 0, ox = 0;
    if (!SAME) {
        oy = static_cast<int>(src_coord(tgt.sy, ty * 16));
        ox = static_cast<int>(src_coord(tgt.sx, tx * 16));
        const float sy = src_coord(tgt.sy, y);
        const int y0 = static_cast<int>(sy);
        const int y1 = y0 + (y0 < tgt.hl - 1 ? 1 : 0);
        wy1 = __fsub_rn(sy, static_cast<float>(y0));
        wy0 = __fsub_rn(1.0f, wy1);
        py0 = y0 - oy;
        py1 = y1 - oy;
    }
    const int64_t lplane = static_cast<int64_t>(tgt.hl) * tgt.wl;
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int c0 = 0; c0 < F; c0 += NC) {
        float4 r[NC], t4[NC];
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            const int c = c0 + k < F ? c0 + k : F - 1;
            r[k] = __ldg(reinterpret_cast<const float4*>(rendered + c * plane + pix));
            if (SAME) t4[k] = __ldg(reinterpret_cast<const float4*>(tgt.p + c * plane + pix));
        }
        if (!SAME) {
            __syncthreads();  // the previous group's patch is no longer read
            for (int e = threadIdx.x; e < NC * kPatch * kPatch; e += kMseThreads) {
                const int k = e / (kPatch * kPatch), rem = e - k * kPatch * kPatch;
                const int i = rem / kPatch, j = rem - (rem / kPatch) * kPatch;
                const int c = c0 + k < F ? c0 + k : F - 1;
                const int yy = min(oy + i, tgt.hl - 1), xx = min(ox + j, tgt.wl - 1);
                s_lr[k][i][j] = __ldg(tgt.p + c * lplane + static_cast<int64_t>(yy) * tgt.wl + xx);
            }
            __syncthreads();
#pragma unroll 1
            for (int k = 0; k < NC; ++k) {
                if (c0 + k >= F) continue;
                float4 rk = r[0];  // r[k] by selects, so r stays in registers in the rolled loop
#pragma unroll
                for (int u = 1; u < NC; ++u) rk = k == u ? r[u] : rk;
                const float rv[4] = {rk.x, rk.y, rk.z, rk.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float sx = src_coord(tgt.sx, xq + q);
                    const int x0 = static_cast<int>(sx);
                    const int x1 = x0 + (x0 < tgt.wl - 1 ? 1 : 0);
                    const float wx1 = __fsub_rn(sx, static_cast<float>(x0));
                    const float wx0 = __fsub_rn(1.0f, wx1);
                    const int j0 = x0 - ox, j1 = x1 - ox;
                    const float top = __fadd_rn(__fmul_rn(wx0, s_lr[k][py0][j0]), __fmul_rn(wx1, s_lr[k][py0][j1]));
                    const float bot = __fadd_rn(__fmul_rn(wx0, s_lr[k][py1][j0]), __fmul_rn(wx1, s_lr[k][py1][j1]));
                    const float d = __fsub_rn(rv[q], __fadd_rn(__fmul_rn(wy0, top), __fmul_rn(wy1, bot)));
                    s[q] = __fadd_rn(s[q], __fmul_rn(d, d));
                }
            }
        } else {
#pragma unroll
            for (int k = 0; k < NC; ++k) {
                if (c0 + k >= F) continue;
                const float d0 = __fsub_rn(r[k].x, t4[k].x), d1 = __fsub_rn(r[k].y, t4[k].y);
                const float d2 = __fsub_rn(r[k].z, t4[k].z), d3 = __fsub_rn(r[k].w, t4[k].w);
                s[0] = __fadd_rn(s[0], __fmul_rn(d0, d0));
                s[1] = __fadd_rn(s[1], __fmul_rn(d1, d1));
                s[2] = __fadd_rn(s[2], __fmul_rn(d2, d2));
                s[3] = __fadd_rn(s[3], __fmul_rn(d3, d3));
            }
        }
    }
    const float ff = static_cast<float>(F);
    float acc = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) acc += __fdiv_rn(s[q], ff);
    const float total = block_sum(acc, s_warp);
    if (threadIdx.x == 0) tile_err[tile] = __fdiv_rn(total, 256.0f);
}

// Per slot: the error of the tile holding its centre (+inf outside the frame or
// where in_frame says so), the alive-masked copy and the age bump.
__global__ void __launch_bounds__(kThreads) k_canvas_error(int n, int H, int W, int ts, int ntx, int nty,
                                                           const float2* __restrict__ xy,
                                                           const uint8_t* __restrict__ in_frame,
                                                           const float* __restrict__ tile_err,
                                                           const uint8_t* __restrict__ alive,
                                                           int64_t* __restrict__ age, float* __restrict__ g_error,
                                                           float* __restrict__ error) {
    const int g = blockIdx.x * kThreads + threadIdx.x;
    if (g >= n) return;
    const float2 p = xy[g];
    const bool inside = p.x >= 0.0f && p.x < static_cast<float>(W) && p.y >= 0.0f && p.y < static_cast<float>(H);
    float e = INFINITY;
    if (inside) {
        long long tx = __float2ll_rz(__fdiv_rn(p.x, static_cast<float>(ts)));
        long long ty = __float2ll_rz(__fdiv_rn(p.y, static_cast<float>(ts)));
        tx = tx < 0 ? 0 : (tx > ntx - 1 ? ntx - 1 : tx);
        ty = ty < 0 ? 0 : (ty > nty - 1 ? nty - 1 : ty);
        e = tile_err[ty * ntx + tx];
    }
    if (in_frame != nullptr && in_frame[g] == 0) e = INFINITY;
    if (g_error != nullptr) g_error[g] = e;
    if (alive != nullptr) {
        const bool a = alive[g] != 0;
        if (error != nullptr) error[g] = a ? e : 0.0f;
        if (age != nullptr) age[g] = a ? age[g] + 1 : 0;
    }
}

// Order-preserving map of a float onto uint32 (NaN of either sign above +inf).
__device__ __forceinline__ uint32_t ordered_bits(float v) {
    if (isnan(v)) return 0xfffffffeu;
    const uint32_t u = __float_as_uint(v + 0.0f);
    return (u & 0x80000000u) != 0u ? ~u : (u | 0x80000000u);
}

// Alive errors as ascending sort keys (dead slots last) and the alive count.
__global__ void __launch_bounds__(kThreads) k_error_keys(int n, const uint8_t* __restrict__ alive,
                                                         const float* __restrict__ err, uint32_t* __restrict__ keys,
                                                         int32_t* __restrict__ vals, int32_t* __restrict__ count) {
    const int g = blockIdx.x * kThreads + threadIdx.x;
    const bool a = g < n && alive[g] != 0;
    if (g < n) {
        keys[g] = a ? ordered_bits(err[g]) : 0xffffffffu;
        vals[g] = g;
    }
    const unsigned live = __ballot_sync(0xffffffffu, a);
    if ((threadIdx.x & 31) == 0 && live != 0u) atomicAdd(count, __popc(live));
}

// torch.lerp on float: the end nearer the weight is the base of a fused multiply-add.
__device__ __forceinline__ float torch_lerp(float a, float b, float w) {
    const float d = __fsub_rn(b, a);
    return w < 0.5f ? fmaf(w, d, a) : fmaf(-d, __fsub_rn(1.0f, w), b);
}

__device__ float torch_quantile(const float* __restrict__ err, const int32_t* __restrict__ sorted, int m, float q) {
    const float last = err[sorted[m - 1]];
    if (isnan(last)) return last;
    const float rank = __fmul_rn(q, static_cast<float>(m - 1));
    const int lo = static_cast<int>(rank);
    const int hi = static_cast<int>(ceilf(rank));
    const float w = __fsub_rn(rank, static_cast<float>(lo));
    return torch_lerp(err[sorted[lo]], err[sorted[hi]], w);
}

// The two thresholds of the decision tree: quant[0] = the R2 (age) quantile,
// quant[1] = the R3 (tile-error) quantile; 0 and +inf without alive slots.
__global__ void k_quantiles(const int32_t* __restrict__ count, const int32_t* __restrict__ sorted,
                            const float* __restrict__ err, float q_age, float q_tile, float* __restrict__ quant) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const int m = *count;
    if (m == 0) {
        quant[0] = 0.0f;
        quant[1] = INFINITY;
        return;
    }
    quant[0] = torch_quantile(err, sorted, m, q_age);
    quant[1] = torch_quantile(err, sorted, m, q_tile);
}

// R1 | R2 | R3 per slot, and the descending key of its cap priority.
__global__ void __launch_bounds__(kThreads) k_prune_flags(int n, const uint8_t* __restrict__ alive,
                                                          const uint8_t* __restrict__ in_frame,
                                                          const int64_t* __restrict__ age,
                                                          const float* __restrict__ err,
                                                          const float* __restrict__ quant, long long age_max,
                                                          long long min_age, int32_t* __restrict__ flag,
                                                          uint32_t* __restrict__ keys, int32_t* __restrict__ vals) {
    const int g = blockIdx.x * kThreads + threadIdx.x;
    if (g >= n) return;
    const bool a = alive[g] != 0;
    const float e = err[g];
    const long long ag = age[g];
    const bool r1 = a && in_frame[g] == 0;
    const bool r2 = a && ag > age_max && e <= quant[0];
    const bool r3 = a && ag >= min_age && e >= quant[1];
    const bool sel = r1 || r2 || r3;
    flag[g] = sel ? 1 : 0;
    const float prio = r1 ? 3.0f : (r2 ? 2.0f : (r3 ? 1.0f : 0.0f));
    const float clipped = isfinite(e) ? e : 1.0e30f;
    const float score = __fadd_rn(__fmul_rn(prio, 1.0e6f), clipped);
    keys[g] = sel ? ~ordered_bits(score) : 0xffffffffu;
    vals[g] = g;
}

// The prune list: in slot order when the selection fits the cap, else the cap's
// worth of the score order.
__global__ void __launch_bounds__(kThreads) k_prune_out(int n, const int32_t* __restrict__ flag,
                                                        const int32_t* __restrict__ pos,
                                                        const int32_t* __restrict__ by_score, long long cap,
                                                        int64_t* __restrict__ prune_idx,
                                                        int64_t* __restrict__ prune_count) {
    const int g = blockIdx.x * kThreads + threadIdx.x;
    const long long c = pos[n];
    if (g == 0) *prune_count = c < cap ? c : cap;
    if (g >= n) return;
    if (c <= cap) {
        if (flag[g]) prune_idx[pos[g]] = g;
    } else if (g < cap) {
        prune_idx[g] = by_score[g];
    }
}

// Tile errors (classifier-masked to -inf) as descending keys; the count of
// finite eligible tiles.
__global__ void __launch_bounds__(kThreads) k_spawn_keys(int T, const float* __restrict__ tile_err,
                                                         const uint8_t* __restrict__ cls, uint32_t* __restrict__ keys,
                                                         int32_t* __restrict__ vals, int32_t* __restrict__ eligible) {
    const int t = blockIdx.x * kThreads + threadIdx.x;
    bool ok = false;
    if (t < T) {
        const float v = (cls == nullptr || cls[t] != 0) ? tile_err[t] : -INFINITY;
        ok = isfinite(v);
        keys[t] = ~ordered_bits(v);
        vals[t] = t;
    }
    const unsigned any = __ballot_sync(0xffffffffu, ok);
    if ((threadIdx.x & 31) == 0 && any != 0u) atomicAdd(eligible, __popc(any));
}

__global__ void __launch_bounds__(kThreads) k_spawn_out(int T, int tw, const int32_t* __restrict__ order,
                                                        const int32_t* __restrict__ eligible, long long n_tiles,
                                                        int64_t* __restrict__ tiles_yx, int64_t* __restrict__ take) {
    const int i = blockIdx.x * kThreads + threadIdx.x;
    const long long e = *eligible;
    const long long k = n_tiles < e ? n_tiles : e;
    if (i == 0) *take = k > 0 ? k : 0;
    if (i < T && i < k) {
        const int t = order[i];
        tiles_yx[2 * i + 0] = t / tw;
        tiles_yx[2 * i + 1] = t - (t / tw) * tw;
    }
}

// Pruned slots die with age and error reset; indices outside [0, n) are skipped.
__global__ void __launch_bounds__(kThreads) k_prune_apply(int n, const int64_t* __restrict__ idx,
                                                          const int64_t* __restrict__ count, uint8_t* __restrict__ alive,
                                                          int64_t* __restrict__ age, float* __restrict__ error) {
    const long long i = static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x;
    if (i >= *count) return;
    const long long g = idx[i];
    if (g < 0 || g >= n) return;
    alive[g] = 0;
    age[g] = 0;
    error[g] = 0.0f;
}

__global__ void __launch_bounds__(kThreads) k_dead_flags(int n, const uint8_t* __restrict__ alive,
                                                         int32_t* __restrict__ flag) {
    const int g = blockIdx.x * kThreads + threadIdx.x;
    if (g < n) flag[g] = alive[g] == 0 ? 1 : 0;
}

// The r-th dead slot (slot order) takes new Gaussian r, for r < num_new.
__global__ void __launch_bounds__(kThreads) k_spawn_write(int n, int F, int num_new, int f_new, int f_copy,
                                                          const int32_t* __restrict__ rank,
                                                          const float* __restrict__ nxy, const float* __restrict__ nscale,
                                                          const float* __restrict__ nrot, const float* __restrict__ nfeat,
                                                          float* __restrict__ positions, float* __restrict__ scales,
                                                          float* __restrict__ rotations, float* __restrict__ colors,
                                                          uint8_t* __restrict__ alive, int64_t* __restrict__ age,
                                                          float* __restrict__ error, int64_t* __restrict__ n_spawned) {
    const int g = blockIdx.x * kThreads + threadIdx.x;
    if (g == 0) {
        const int nfree = rank[n];
        *n_spawned = nfree < num_new ? nfree : num_new;
    }
    if (g >= n || alive[g] != 0) return;
    const int r = rank[g];
    if (r >= num_new) return;
    positions[2 * g + 0] = nxy[2 * r + 0];
    positions[2 * g + 1] = nxy[2 * r + 1];
    scales[2 * g + 0] = nscale[2 * r + 0];
    scales[2 * g + 1] = nscale[2 * r + 1];
    rotations[g] = nrot[r];
    for (int c = 0; c < f_copy; ++c) colors[static_cast<int64_t>(g) * F + c] = nfeat[static_cast<int64_t>(r) * f_new + c];
    alive[g] = 1;
    age[g] = 0;
    error[g] = 0.0f;
}

unsigned blocks_for(int64_t n) { return static_cast<unsigned>(div_up(n > 0 ? n : 1, kThreads)); }

}  // namespace

cudaError_t launch_tile_mse(int f, int h, int w, int ts, const float* rendered, int hl, int wl, const float* target,
                            float* tile_err, cudaStream_t stream) {
    const int ntx = w / ts, nty = h / ts;
    if (ntx == 0 || nty == 0) return cudaSuccess;
    LrFrame t{target, hl, wl, h, w, static_cast<float>(hl) / static_cast<float>(h),
              static_cast<float>(wl) / static_cast<float>(w), hl == h && wl == w ? 1 : 0};
    const unsigned grid = static_cast<unsigned>(ntx * nty);
    // 16-px tiles over float4-aligned rows, with an LR frame no larger than the render
    const bool vec = ts == 16 && w % 4 == 0 && (reinterpret_cast<uintptr_t>(rendered) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(target) & 15) == 0 && hl <= h && wl <= w;
    if (vec) {
#define OSS_MSE16(NC)                                                                                 \
    (t.same ? k_tile_mse16<NC, true><<<grid, kMseThreads, 0, stream>>>(f, h, w, ntx, rendered, t, tile_err) \
            : k_tile_mse16<NC, false><<<grid, kMseThreads, 0, stream>>>(f, h, w, ntx, rendered, t, tile_err))
        if (f == 1) OSS_MSE16(1);
        else if (f == 2) OSS_MSE16(2);
        else if (f == 3) OSS_MSE16(3);
        else OSS_MSE16(4);
#undef OSS_MSE16
        return cudaGetLastError();
    }
    if (f == 1) k_tile_mse<1><<<grid, kThreads, 0, stream>>>(f, h, w, ts, ntx, rendered, t, tile_err);
    else if (f == 2) k_tile_mse<2><<<grid, kThreads, 0, stream>>>(f, h, w, ts, ntx, rendered, t, tile_err);
    else if (f == 3) k_tile_mse<3><<<grid, kThreads, 0, stream>>>(f, h, w, ts, ntx, rendered, t, tile_err);
    else k_tile_mse<4><<<grid, kThreads, 0, stream>>>(f, h, w, ts, ntx, rendered, t, tile_err);
    return cudaGetLastError();
}

cudaError_t launch_canvas_error(int n, int h, int w, int ts, const float* xy, const uint8_t* in_frame,
                                const float* tile_err, const uint8_t* alive, int64_t* age, float* g_error,
                                float* error, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    k_canvas_error<<<blocks_for(n), kThreads, 0, stream>>>(n, h, w, ts, w / ts, h / ts,
                                                           reinterpret_cast<const float2*>(xy), in_frame, tile_err,
                                                           alive, age, g_error, error);
    return cudaGetLastError();
}

int64_t prune_scratch_bytes(int64_t n) {
    return arena_bytes(n, 4) * 3 + arena_bytes(n + 1, 4) * 2 + arena_bytes(1, 4) + scan_scratch_bytes(n + 1) +
           radix_scratch_bytes(n, 0xffffffffu);
}

cudaError_t launch_select_for_pruning(int n, const uint8_t* alive, const uint8_t* in_frame, const int64_t* age,
                                      const float* err, long long cap, long long age_max, float q_age, float q_tile,
                                      long long min_age, int64_t* prune_idx, int64_t* prune_count, float* quant,
                                      void* scratch, cudaStream_t stream) {
    Arena arena{static_cast<char*>(scratch), prune_scratch_bytes(n), 0};
    uint32_t* keys = arena.take<uint32_t>(n);
    int32_t* vals = arena.take<int32_t>(n);
    int32_t* sorted = arena.take<int32_t>(n);
    int32_t* flag = arena.take<int32_t>(n + 1);
    int32_t* pos = arena.take<int32_t>(n + 1);
    int32_t* count = arena.take<int32_t>(1);
    void* scan_scratch = arena.base + arena.used;
    void* radix_scratch = static_cast<char*>(scan_scratch) + scan_scratch_bytes(n + 1);
    cudaError_t err_ = cudaMemsetAsync(count, 0, sizeof(int32_t), stream);
    if (err_ != cudaSuccess) return err_;
    if (n == 0) {
        k_quantiles<<<1, 32, 0, stream>>>(count, sorted, err, q_age, q_tile, quant);
        err_ = cudaMemsetAsync(prune_count, 0, sizeof(int64_t), stream);
        return err_ != cudaSuccess ? err_ : cudaGetLastError();
    }
    k_error_keys<<<blocks_for(n), kThreads, 0, stream>>>(n, alive, err, keys, vals, count);
    if ((err_ = radix_sort_pairs(keys, vals, n, 0xffffffffu, sorted, radix_scratch, stream)) != cudaSuccess) return err_;
    k_quantiles<<<1, 32, 0, stream>>>(count, sorted, err, q_age, q_tile, quant);
    k_prune_flags<<<blocks_for(n), kThreads, 0, stream>>>(n, alive, in_frame, age, err, quant, age_max, min_age, flag,
                                                          keys, vals);
    if ((err_ = cudaMemsetAsync(flag + n, 0, sizeof(int32_t), stream)) != cudaSuccess) return err_;
    if ((err_ = scan_exclusive_i32(flag, pos, n + 1, false, nullptr, scan_scratch, stream)) != cudaSuccess) return err_;
    if ((err_ = radix_sort_pairs(keys, vals, n, 0xffffffffu, sorted, radix_scratch, stream)) != cudaSuccess) return err_;
    k_prune_out<<<blocks_for(n), kThreads, 0, stream>>>(n, flag, pos, sorted, cap, prune_idx, prune_count);
    return cudaGetLastError();
}

int64_t spawn_tiles_scratch_bytes(int64_t num_tiles) {
    return arena_bytes(num_tiles, 4) * 3 + arena_bytes(1, 4) + radix_scratch_bytes(num_tiles, 0xffffffffu);
}

cudaError_t launch_select_spawn_tiles(int th, int tw, const float* tile_err, const uint8_t* cls, long long n_tiles,
                                      int64_t* tiles_yx, int64_t* take, void* scratch, cudaStream_t stream) {
    const int T = th * tw;
    Arena arena{static_cast<char*>(scratch), spawn_tiles_scratch_bytes(T), 0};
    uint32_t* keys = arena.take<uint32_t>(T);
    int32_t* vals = arena.take<int32_t>(T);
    int32_t* order = arena.take<int32_t>(T);
    int32_t* eligible = arena.take<int32_t>(1);
    void* radix_scratch = arena.base + arena.used;
    cudaError_t err_ = cudaMemsetAsync(eligible, 0, sizeof(int32_t), stream);
    if (err_ != cudaSuccess) return err_;
    if (T == 0) return cudaMemsetAsync(take, 0, sizeof(int64_t), stream);
    k_spawn_keys<<<blocks_for(T), kThreads, 0, stream>>>(T, tile_err, cls, keys, vals, eligible);
    if ((err_ = radix_sort_pairs(keys, vals, T, 0xffffffffu, order, radix_scratch, stream)) != cudaSuccess) return err_;
    k_spawn_out<<<blocks_for(T), kThreads, 0, stream>>>(T, tw, order, eligible, n_tiles, tiles_yx, take);
    return cudaGetLastError();
}

int64_t prune_spawn_scratch_bytes(int64_t n) { return arena_bytes(n + 1, 4) * 2 + scan_scratch_bytes(n + 1); }

cudaError_t launch_apply_prune_spawn(int n, int f, const int64_t* prune_idx, const int64_t* prune_count,
                                     int64_t max_prune, int num_new, int f_new, const float* nxy,
                                     const float* nscale, const float* nrot, const float* nfeat, float* positions,
                                     float* scales, float* rotations, float* colors, uint8_t* alive, int64_t* age,
                                     float* error, int64_t* n_spawned, void* scratch, cudaStream_t stream) {
    if (n == 0) return cudaMemsetAsync(n_spawned, 0, sizeof(int64_t), stream);
    if (max_prune > 0) {
        k_prune_apply<<<blocks_for(max_prune), kThreads, 0, stream>>>(n, prune_idx, prune_count, alive, age, error);
    }
    Arena arena{static_cast<char*>(scratch), prune_spawn_scratch_bytes(n), 0};
    int32_t* flag = arena.take<int32_t>(n + 1);
    int32_t* rank = arena.take<int32_t>(n + 1);
    void* scan_scratch = arena.base + arena.used;
    k_dead_flags<<<blocks_for(n), kThreads, 0, stream>>>(n, alive, flag);
    cudaError_t err_ = cudaMemsetAsync(flag + n, 0, sizeof(int32_t), stream);
    if (err_ != cudaSuccess) return err_;
    if ((err_ = scan_exclusive_i32(flag, rank, n + 1, false, nullptr, scan_scratch, stream)) != cudaSuccess) return err_;
    const int f_copy = f < f_new ? f : f_new;
    k_spawn_write<<<blocks_for(n), kThreads, 0, stream>>>(n, f, num_new, f_new, f_copy, rank, nxy, nscale, nrot, nfeat,
                                                          positions, scales, rotations, colors, alive, age, error,
                                                          n_spawned);
    return cudaGetLastError();
}

}  // namespace oss
