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

__device__ __forceinline__ float lr_tap(const LrFrame& f, int c, int y, int x) {
    return __ldg(f.p + (static_cast<int64_t>(c) * f.hl + y) * f.wl + x);
}

// Texel (i, j) of F.interpolate(frame, (h, w), bilinear, align_corners=False).
__device__ float target_at(const LrFrame& f, int c, int i, int j) {
    if (f.same) return lr_tap(f, c, i, j);
    float sy = __fsub_rn(__fmul_rn(f.sy, __fadd_rn(static_cast<float>(i), 0.5f)), 0.5f);
    if (sy < 0.0f) sy = 0.0f;
    float sx = __fsub_rn(__fmul_rn(f.sx, __fadd_rn(static_cast<float>(j), 0.5f)), 0.5f);
    if (sx < 0.0f) sx = 0.0f;
    const int y0 = static_cast<int>(sy), x0 = static_cast<int>(sx);
    const int y1 = y0 + (y0 < f.hl - 1 ? 1 : 0), x1 = x0 + (x0 < f.wl - 1 ? 1 : 0);
    const float ly1 = __fsub_rn(sy, static_cast<float>(y0));
    const float lx1 = __fsub_rn(sx, static_cast<float>(x0));
    const float ly0 = __fsub_rn(1.0f, ly1), lx0 = __fsub_rn(1.0f, lx1);
    const float top = __fadd_rn(__fmul_rn(lx0, lr_tap(f, c, y0, x0)), __fmul_rn(lx1, lr_tap(f, c, y0, x1)));
    const float bot = __fadd_rn(__fmul_rn(lx0, lr_tap(f, c, y1, x0)), __fmul_rn(lx1, lr_tap(f, c, y1, x1)));
    return __fadd_rn(__fmul_rn(ly0, top), __fmul_rn(ly1, bot));
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
        float s = 0.0f;
        for (int c = 0; c < F; ++c) {
            const float d = __fsub_rn(__ldg(rendered + c * plane + pix), target_at(tgt, c, y, x));
            s = __fadd_rn(s, __fmul_rn(d, d));
        }
        acc += __fdiv_rn(s, ff);
    }
    const float total = block_sum(acc, s_warp);
    if (threadIdx.x == 0) tile_err[tile] = __fdiv_rn(total, static_cast<float>(ts * ts));
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
    k_tile_mse<<<static_cast<unsigned>(ntx * nty), kThreads, 0, stream>>>(f, h, w, ts, ntx, rendered, t, tile_err);
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
