// Per-tile Gaussian lists by scatter + per-tile sort.
//
// The reference builds its tile lists by sorting (tile << 32 | gid) keys
// (rasterizer_fwd.cu:461-468): each tile's list holds, ascending, the gids of
// the Gaussians whose tile rectangle covers the tile.  Here the per-tile counts
// and their exclusive scan (the list offsets) come from render prepare, each
// (Gaussian, tile) pair claims a slot of its tile with an atomic (in no
// particular order), and every tile's list is then sorted.  A Gaussian covers a
// tile at most once, so a sorted list is unique: the output is the reference's
// list whatever order the atomics ran in.
//
// With a sort key (a permutation of [0, n), e.g. a Gaussian's rank by depth)
// the lists hold keys while they are sorted and are mapped back to gids through
// key_order on output: the lists come out ordered by key instead of gid.
//
// The pair total is read on the device and checked against the caller's
// capacity; on overflow every list and every Gaussian's pair range is emptied
// and a flag is raised, so nothing downstream reads or writes past capacity and
// the host need not wait for the total before launching.
#include <limits.h>

#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

constexpr int kScatterThreads = 256;
constexpr int kScatterWarps = kScatterThreads / 32;
constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortBuf = 8192;                    // ints of shared memory per CTA (32 KB)
constexpr int kWarpCap = 1024;                    // lists up to 1024 sorted by one warp in registers
constexpr int kCtaCap = kSortBuf;                 // lists up to 8192 sorted by the CTA in shared memory
constexpr int kWindowBits = kSortBuf * 32;        // gid window of the bitmap path

// One warp per 32 consecutive Gaussians.  The warp's pairs are dealt round-robin
// to its lanes (lane j of round r takes the warp's pair 32 r + j); the owning
// Gaussian is found by a binary search over the lanes' pair prefix.
__global__ void __launch_bounds__(kScatterThreads) k_scatter_pairs(
    int n, int ntx, int num_tiles, const int4* __restrict__ aabb, int32_t* __restrict__ pair_offset,
    int32_t* __restrict__ tile_count, int32_t* __restrict__ tile_offsets, const int64_t* __restrict__ total_pairs,
    int64_t capacity, const int32_t* __restrict__ sort_key, int32_t* __restrict__ unsorted,
    int32_t* __restrict__ overflow) {
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * kScatterThreads + threadIdx.x;
    const int64_t nthreads = static_cast<int64_t>(gridDim.x) * kScatterThreads;
    if (*total_pairs > capacity) {
        // empty every list and every pair range; the image and gradients come out zero
        for (int64_t i = tid; i <= num_tiles; i += nthreads) tile_offsets[i] = 0;
        for (int64_t i = tid; i <= n; i += nthreads) pair_offset[i] = 0;
        if (tid == 0) *overflow = 1;
        return;
    }
    if (tid == 0) *overflow = 0;
    const int lane = threadIdx.x & 31;
    const int g0 = (blockIdx.x * kScatterWarps + (threadIdx.x >> 5)) * 32;
    const int g = g0 + lane;
    int4 box = make_int4(0, 0, 0, 0);
    int key = g;
    if (g < n) {
        box = aabb[g];
        if (sort_key != nullptr) key = sort_key[g];
    }
    const int bw = box.z > box.x ? box.z - box.x : 0;
    const int bh = box.w > box.y ? box.w - box.y : 0;
    const int cnt = bw * bh;
    // inclusive then exclusive warp prefix of the pair counts
    int incl = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
    }
    const int start = incl - cnt;
    const int warp_total = __shfl_sync(0xffffffffu, incl, 31);
    for (int base = 0; base < warp_total; base += 32) {
        const int j = base + lane;
        int owner = 0;
#pragma unroll
        for (int step = 16; step > 0; step >>= 1) {
            const int cand = owner + step;
            const int s = __shfl_sync(0xffffffffu, start, cand);
            if (s <= j) owner = cand;
        }
        const int o_start = __shfl_sync(0xffffffffu, start, owner);
        const int o_x = __shfl_sync(0xffffffffu, box.x, owner);
        const int o_y = __shfl_sync(0xffffffffu, box.y, owner);
        const int o_w = __shfl_sync(0xffffffffu, bw, owner);
        const int o_key = __shfl_sync(0xffffffffu, key, owner);
        if (j < warp_total) {
            const int k = j - o_start;
            const int dy = k / o_w;
            const int t = (o_y + dy) * ntx + o_x + (k - dy * o_w);
            const int slot = atomicSub(&tile_count[static_cast<int64_t>(t) * kTileCountStride], 1) - 1;
            unsorted[tile_offsets[t] + slot] = o_key;
        }
    }
}

__device__ __forceinline__ int next_pow2(int v) {
    int p = 1;
    while (p < v) p <<= 1;
    return p;
}

// Ascending bitonic sort of s[0..lp) in shared memory, lp a power of two, by the
// CTA's threads.
__device__ __forceinline__ void cta_bitonic_sort(int32_t* s, int lp) {
    const int tid = threadIdx.x;
    constexpr int nt = kSortThreads;
    for (int k = 2; k <= lp; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < (lp >> 1); i += nt) {
                const int a = (i << 1) - (i & (j - 1));
                const int b = a + j;
                const int32_t x = s[a];
                const int32_t y = s[b];
                const bool ascending = (a & k) == 0;
                if ((x > y) == ascending) {
                    s[a] = y;
                    s[b] = x;
                }
            }
            __syncthreads();
        }
    }
}

// Ascending bitonic sort of the 32 * R values a warp holds, element r * 32 + lane
// in v[r] of that lane: distances below 32 pair lanes through shuffles,
// distances of 32 and more pair registers of the same lane.
template <int R>
__device__ __forceinline__ void warp_bitonic(int32_t (&v)[R], int lane) {
#pragma unroll
    for (int k = 2; k <= 32 * R; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j >= 32) {
                const int jr = j >> 5;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    if ((r & jr) == 0) {
                        const bool asc = ((r * 32) & k) == 0;  // k >= 64 here: lane bits do not reach it
                        const int32_t a = v[r];
                        const int32_t b = v[r | jr];
                        v[r] = asc ? min(a, b) : max(a, b);
                        v[r | jr] = asc ? max(a, b) : min(a, b);
                    }
                }
            } else {
                const bool lower = (lane & j) == 0;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int32_t p = __shfl_xor_sync(0xffffffffu, v[r], j);
                    const bool asc = ((r * 32 + lane) & k) == 0;
                    v[r] = lower == asc ? min(v[r], p) : max(v[r], p);
                }
            }
        }
    }
}

template <int R>
__device__ __forceinline__ void warp_sort_list(const int32_t* __restrict__ src, int32_t* __restrict__ dst, int len,
                                               int lane, const int32_t* __restrict__ key_order) {
    int32_t v[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int e = r * 32 + lane;
        v[r] = e < len ? src[e] : INT_MAX;
    }
    warp_bitonic<R>(v, lane);
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int e = r * 32 + lane;
        if (e < len) dst[e] = key_order != nullptr ? key_order[v[r]] : v[r];
    }
}

__device__ __forceinline__ int block_exclusive_sum(int v, int* s_warp, int& total) {
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
    for (int w = 0; w < kSortWarps; ++w) {
        const int c = s_warp[w];
        before += w < warp ? c : 0;
        total += c;
    }
    __syncthreads();
    return before + x - v;
}

// Lists longer than kCtaCap: the CTA marks the gids of one window of the gid
// range in a shared bitmap and writes the set bits out in order, window by
// window.  Cost per window: one pass over the list plus the bitmap.
__device__ void bitmap_sort(const int32_t* __restrict__ in, int32_t* __restrict__ out, int len, int n,
                            int32_t* s_buf, int* s_warp, const int32_t* __restrict__ key_order) {
    uint32_t* bm = reinterpret_cast<uint32_t*>(s_buf);
    constexpr int kWordsPerThread = kSortBuf / kSortThreads;
    int written = 0;
    for (int64_t base = 0; base < n; base += kWindowBits) {
        for (int i = threadIdx.x; i < kSortBuf; i += kSortThreads) bm[i] = 0u;
        __syncthreads();
        for (int i = threadIdx.x; i < len; i += kSortThreads) {
            const int64_t r = static_cast<int64_t>(in[i]) - base;
            if (r >= 0 && r < kWindowBits) atomicOr(&bm[r >> 5], 1u << (r & 31));
        }
        __syncthreads();
        const int w0 = threadIdx.x * kWordsPerThread;
        int cnt = 0;
#pragma unroll 8
        for (int w = 0; w < kWordsPerThread; ++w) cnt += __popc(bm[w0 + w]);
        int total;
        int pos = written + block_exclusive_sum(cnt, s_warp, total);
        for (int w = 0; w < kWordsPerThread; ++w) {
            uint32_t bits = bm[w0 + w];
            while (bits != 0u) {
                const int b = __ffs(static_cast<int>(bits)) - 1;
                bits &= bits - 1u;
                const int32_t v = static_cast<int32_t>(base + (w0 + w) * 32 + b);
                out[pos++] = key_order != nullptr ? key_order[v] : v;
            }
        }
        written += total;
        __syncthreads();
    }
}

// One warp per tile; lists above kWarpCap are sorted afterwards by the whole CTA.
__global__ void __launch_bounds__(kSortThreads) k_sort_tiles(int n, int num_tiles,
                                                              const int32_t* __restrict__ tile_offsets,
                                                              const int32_t* __restrict__ unsorted,
                                                              const int32_t* __restrict__ key_order,
                                                              int32_t* __restrict__ gid_sorted) {
    __shared__ int32_t s_buf[kSortBuf];
    __shared__ int s_warp[kSortWarps];
    __shared__ int s_big;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) s_big = 0;
    __syncthreads();
    const int t = blockIdx.x * kSortWarps + warp;
    int off = 0;
    int len = 0;
    if (t < num_tiles) {
        off = tile_offsets[t];
        len = tile_offsets[t + 1] - off;
    }
    const int32_t* src = unsorted + off;
    int32_t* dst = gid_sorted + off;
    if (len <= 32) {
        // rank of each value among the (distinct) values of the warp
        const int32_t v = lane < len ? src[lane] : INT_MAX;
        int rank = 0;
#pragma unroll
        for (int j = 0; j < 32; ++j) rank += __shfl_sync(0xffffffffu, v, j) < v ? 1 : 0;
        if (lane < len) dst[rank] = key_order != nullptr ? key_order[v] : v;
    } else if (len <= 64) {
        warp_sort_list<2>(src, dst, len, lane, key_order);
    } else if (len <= 128) {
        warp_sort_list<4>(src, dst, len, lane, key_order);
    } else if (len <= 256) {
        warp_sort_list<8>(src, dst, len, lane, key_order);
    } else if (len <= 512) {
        warp_sort_list<16>(src, dst, len, lane, key_order);
    } else if (len <= kWarpCap) {
        warp_sort_list<32>(src, dst, len, lane, key_order);
    } else if (lane == 0) {
        atomicOr(&s_big, 1 << warp);
    }
    __syncthreads();
    const int big = s_big;
    for (int wv = 0; wv < kSortWarps; ++wv) {
        if ((big >> wv & 1) == 0) continue;
        const int bt = blockIdx.x * kSortWarps + wv;
        const int boff = tile_offsets[bt];
        const int blen = tile_offsets[bt + 1] - boff;
        if (blen <= kCtaCap) {
            const int lp = next_pow2(blen);
            for (int i = threadIdx.x; i < lp; i += kSortThreads) s_buf[i] = i < blen ? unsorted[boff + i] : INT_MAX;
            __syncthreads();
            cta_bitonic_sort(s_buf, lp);
            for (int i = threadIdx.x; i < blen; i += kSortThreads) {
                gid_sorted[boff + i] = key_order != nullptr ? key_order[s_buf[i]] : s_buf[i];
            }
            __syncthreads();
        } else {
            bitmap_sort(unsorted + boff, gid_sorted + boff, blen, n, s_buf, s_warp, key_order);
        }
    }
}

// Monotone map of a float to uint32 (-0.0 first made +0.0): ordering the keys as
// unsigned integers orders the floats, -inf first and +inf last.
__global__ void k_depth_keys(int n, const float* __restrict__ depth, uint32_t* __restrict__ keys,
                             int32_t* __restrict__ vals) {
    const int g = blockIdx.x * 256 + threadIdx.x;
    if (g >= n) return;
    const uint32_t u = __float_as_uint(depth[g] + 0.0f);
    keys[g] = (u & 0x80000000u) != 0u ? ~u : (u | 0x80000000u);
    vals[g] = g;
}

__global__ void k_rank_of(int n, const int32_t* __restrict__ order, int32_t* __restrict__ rank) {
    const int i = blockIdx.x * 256 + threadIdx.x;
    if (i < n) rank[order[i]] = i;
}

__global__ void k_empty_lists(int num_tiles, int32_t* __restrict__ tile_offsets, int32_t* __restrict__ overflow) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i <= num_tiles) tile_offsets[i] = 0;
    if (i == 0 && overflow != nullptr) *overflow = 0;
}

}  // namespace

int64_t tile_lists_scratch_bytes(int64_t capacity) { return arena_bytes(capacity, sizeof(int32_t)); }

int64_t depth_order_scratch_bytes(int64_t n) {
    return arena_bytes(n, sizeof(uint32_t)) + arena_bytes(n, sizeof(int32_t)) + radix_scratch_bytes(n, 0xffffffffu);
}

cudaError_t depth_order(int n, const float* depth, int32_t* order, int32_t* rank, void* scratch, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    Arena arena{static_cast<char*>(scratch), depth_order_scratch_bytes(n), 0};
    uint32_t* keys = arena.take<uint32_t>(n);
    int32_t* vals = arena.take<int32_t>(n);
    void* radix_scratch = arena.base + arena.used;
    const unsigned blocks = static_cast<unsigned>(div_up(n, 256));
    k_depth_keys<<<blocks, 256, 0, stream>>>(n, depth, keys, vals);
    cudaError_t err = radix_sort_pairs(keys, vals, n, 0xffffffffu, order, radix_scratch, stream);
    if (err != cudaSuccess) return err;
    k_rank_of<<<blocks, 256, 0, stream>>>(n, order, rank);
    return cudaGetLastError();
}

cudaError_t build_tile_lists(int n, int ntx, int num_tiles, const int32_t* aabb, int32_t* pair_offset,
                             int32_t* tile_count, const int64_t* total_pairs, int64_t capacity,
                             const int32_t* sort_key, const int32_t* key_order, int32_t* gid_sorted,
                             int32_t* tile_offsets, int32_t* overflow, void* scratch, cudaStream_t stream) {
    if (n == 0 || num_tiles == 0) {
        k_empty_lists<<<static_cast<unsigned>(div_up(static_cast<int64_t>(num_tiles) + 1, 256)), 256, 0, stream>>>(
            num_tiles, tile_offsets, overflow);
        return cudaGetLastError();
    }
    int32_t* unsorted = static_cast<int32_t*>(scratch);
    k_scatter_pairs<<<static_cast<unsigned>(div_up(n, kScatterThreads)), kScatterThreads, 0, stream>>>(
        n, ntx, num_tiles, reinterpret_cast<const int4*>(aabb), pair_offset, tile_count, tile_offsets, total_pairs,
        capacity, sort_key, unsorted, overflow);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    k_sort_tiles<<<static_cast<unsigned>(div_up(num_tiles, kSortWarps)), kSortThreads, 0, stream>>>(
        n, num_tiles, tile_offsets, unsorted, key_order, gid_sorted);
    return cudaGetLastError();
}

}  // namespace oss
