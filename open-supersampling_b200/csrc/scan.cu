// Device-wide exclusive scan of int32 counts.
//
// Three shapes, picked by size:
//  * n <= 8192: one CTA of 1024 threads (a single launch);
//  * up to 2048 blocks of 2048 values: per-block reduce, then an apply kernel in
//    which every CTA sums the block totals before it (each CTA re-reads at most
//    2048 int64 from L2) and scans its own block -- two launches, no waiting;
//  * larger: reduce, scan of the block totals by one CTA, apply.
// Sums are carried in int64 so an int32 overflow of the total is detected by
// the caller instead of wrapping silently.  The same apply kernel finishes the
// gid-major pair-offset scan whose per-block reduce is fused into the
// preprocess kernel (scan_apply_with_block_sums).
#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;  // 2048 values per block
constexpr int kScanBlocksThreads = 1024;
constexpr int kSingleItems = 8;
constexpr int64_t kSingleMax = kScanBlocksThreads * kSingleItems;  // 8192 (32 KB of static shared memory)
constexpr int64_t kRedundantMaxBlocks = 2048;
// Tile blocks up to which each block sums the counts before it itself (one frame
// of 4K has 32 blocks of 1024 tiles).
constexpr int64_t kTileBlocksRedundant = 16;

// Exclusive block scan of one int64 per thread; returns the block total in `total`.
template <int NT>
__device__ __forceinline__ long long block_exclusive_scan(long long v, long long* s_warp, long long& total) {
    constexpr int kWarps = NT / 32;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    long long x = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const long long y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        long long wv = lane < kWarps ? s_warp[lane] : 0;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const long long y = __shfl_up_sync(0xffffffffu, wv, off);
            if (lane >= off) wv += y;
        }
        if (lane < kWarps) s_warp[lane] = wv;
    }
    __syncthreads();
    const long long warp_prefix = warp > 0 ? s_warp[warp - 1] : 0;
    total = s_warp[kWarps - 1];
    __syncthreads();  // s_warp may be reused by the caller
    return warp_prefix + x - v;
}

__global__ void __launch_bounds__(kScanThreads) k_scan_reduce(const int32_t* __restrict__ in, int64_t n,
                                                               long long* __restrict__ block_sums) {
    __shared__ long long s_warp[32];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile;
    long long sum = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t i = base + k * kScanThreads + threadIdx.x;
        if (i < n) sum += in[i];
    }
    long long total;
    block_exclusive_scan<kScanThreads>(sum, s_warp, total);
    if (threadIdx.x == 0) block_sums[blockIdx.x] = total;
}

// Exclusive scan of the block sums in place by one CTA; writes the grand total.
__global__ void __launch_bounds__(kScanBlocksThreads) k_scan_blocks(long long* __restrict__ block_sums,
                                                                     int64_t nb, long long* __restrict__ total_ll,
                                                                     int64_t* __restrict__ total_out) {
    __shared__ long long s_warp[32];
    const int64_t per = div_up(nb, kScanBlocksThreads);
    const int64_t lo = static_cast<int64_t>(threadIdx.x) * per;
    const int64_t hi = lo + per < nb ? lo + per : nb;
    long long sum = 0;
    for (int64_t i = lo; i < hi; ++i) sum += block_sums[i];
    long long total;
    long long run = block_exclusive_scan<kScanBlocksThreads>(sum, s_warp, total);
    for (int64_t i = lo; i < hi; ++i) {
        const long long v = block_sums[i];
        block_sums[i] = run;
        run += v;
    }
    if (threadIdx.x == 0) {
        *total_ll = total;
        if (total_out != nullptr) *total_out = static_cast<int64_t>(total);
    }
}

// Scan of block `blk` of TILE = NT * ITEMS values.  prefix_mode 0: the block's
// exclusive offset is block_sums[blk] (already scanned); prefix_mode 1:
// block_sums holds raw per-block totals and the CTA sums those before it.
// The last block writes the grand total (out[n] if write_tail, total_out).
template <int NT, int ITEMS>
__device__ __forceinline__ void scan_apply_block(const int32_t* in, int32_t* out, int64_t n,
                                                 const long long* __restrict__ block_sums, int prefix_mode,
                                                 int64_t nb, int write_tail, int64_t* __restrict__ total_out,
                                                 int64_t blk) {
    constexpr int TILE = NT * ITEMS;
    __shared__ int32_t s_val[TILE];
    __shared__ long long s_warp[32];
    __shared__ long long s_prefix;
    const int64_t base = blk * TILE;
#pragma unroll
    for (int k = 0; k < ITEMS; ++k) {
        const int64_t i = base + k * NT + threadIdx.x;
        s_val[k * NT + threadIdx.x] = i < n ? in[i] : 0;
    }
    long long prefix;
    if (prefix_mode == 1) {
        long long part = 0;
        for (int64_t i = threadIdx.x; i < blk; i += NT) part += block_sums[i];
        long long tot;
        block_exclusive_scan<NT>(part, s_warp, tot);
        prefix = tot;
    } else {
        prefix = block_sums[blk];
    }
    __syncthreads();
    int32_t v[ITEMS];
    long long local = 0;
#pragma unroll
    for (int k = 0; k < ITEMS; ++k) {
        v[k] = s_val[threadIdx.x * ITEMS + k];
        local += v[k];
    }
    long long block_total;
    long long run = block_exclusive_scan<NT>(local, s_warp, block_total) + prefix;
#pragma unroll
    for (int k = 0; k < ITEMS; ++k) {
        s_val[threadIdx.x * ITEMS + k] = static_cast<int32_t>(run);
        run += v[k];
    }
    if (threadIdx.x == 0) s_prefix = prefix + block_total;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < ITEMS; ++k) {
        const int64_t i = base + k * NT + threadIdx.x;
        if (i < n) out[i] = s_val[k * NT + threadIdx.x];
    }
    if (blk == nb - 1 && threadIdx.x == 0) {
        const long long total = s_prefix;
        if (write_tail) out[n] = static_cast<int32_t>(total);
        if (total_out != nullptr) *total_out = static_cast<int64_t>(total);
    }
}

template <int NT, int ITEMS>
__global__ void __launch_bounds__(NT) k_scan_apply(const int32_t* in, int32_t* out, int64_t n,
                                                   const long long* __restrict__ block_sums, int prefix_mode,
                                                   int64_t nb, int write_tail, int64_t* __restrict__ total_out) {
    scan_apply_block<NT, ITEMS>(in, out, n, block_sums, prefix_mode, nb, write_tail, total_out, blockIdx.x);
}

// Block `blk` of the tile-offset scan over counters spaced `stride` ints apart:
// offsets[t] = sum of the counts before t, offsets[num_tiles] = the total.  The
// block sums every count before its own range itself (at most num_tiles reads),
// so the blocks need no second pass.
// With block_counts (one int per block of TILE tiles, written by k_tile_block_counts)
// the block sums those instead of every count before its range: linear in the tile
// count, for the grids of many stacked frames.
template <int NT, int ITEMS>
__device__ __forceinline__ void strided_scan_block(const int32_t* __restrict__ count, int stride,
                                                   int64_t num_tiles, int32_t* __restrict__ offsets, int64_t blk,
                                                   int64_t nblk, const int32_t* __restrict__ block_counts) {
    constexpr int TILE = NT * ITEMS;
    __shared__ long long s_warp[32];
    const int64_t base = blk * TILE;
    long long part = 0;
    if (block_counts != nullptr) {
        for (int64_t b = threadIdx.x; b < blk; b += NT) part += block_counts[b * TILE * stride];
    } else {
        // every count before this block; unrolled so the strided loads overlap
        int64_t t = threadIdx.x;
        for (; t + 7 * NT < base; t += 8 * NT) {
            int32_t c[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) c[u] = count[(t + u * NT) * stride];
#pragma unroll
            for (int u = 0; u < 8; ++u) part += c[u];
        }
        for (; t < base; t += NT) part += count[t * stride];
    }
    long long prefix;
    block_exclusive_scan<NT>(part, s_warp, prefix);
    int32_t v[ITEMS];
    long long local = 0;
#pragma unroll
    for (int k = 0; k < ITEMS; ++k) {
        const int64_t t = base + static_cast<int64_t>(threadIdx.x) * ITEMS + k;
        v[k] = t < num_tiles ? count[t * stride] : 0;
        local += v[k];
    }
    long long block_total;
    long long run = block_exclusive_scan<NT>(local, s_warp, block_total) + prefix;
#pragma unroll
    for (int k = 0; k < ITEMS; ++k) {
        const int64_t t = base + static_cast<int64_t>(threadIdx.x) * ITEMS + k;
        if (t < num_tiles) offsets[t] = static_cast<int32_t>(run);
        run += v[k];
    }
    if (blk == nblk - 1 && threadIdx.x == 0) offsets[num_tiles] = static_cast<int32_t>(prefix + block_total);
}

// The scan launch of render prepare: blocks [0, nb) finish the gid-major
// pair-offset scan (block sums from the preprocess kernel), blocks [nb, nb +
// ntb) scan the per-tile pair counts into the tile list offsets.
template <int NT, int ITEMS>
__global__ void __launch_bounds__(NT) k_prepare_scan(const int32_t* in, int32_t* out, int64_t n,
                                                     const long long* __restrict__ block_sums, int64_t nb,
                                                     int64_t* __restrict__ total_out,
                                                     const int32_t* __restrict__ tile_count, int count_stride,
                                                     int64_t num_tiles, int32_t* __restrict__ tile_offsets,
                                                     int64_t ntb, const int32_t* __restrict__ block_counts) {
    if (blockIdx.x < nb) {
        scan_apply_block<NT, ITEMS>(in, out, n, block_sums, 1, nb, 1, total_out, blockIdx.x);
    } else {
        strided_scan_block<NT, ITEMS>(tile_count, count_stride, num_tiles, tile_offsets, blockIdx.x - nb, ntb,
                                      block_counts);
    }
}

// Sum of the counts of each block of kPrepTile tiles, stored in the block's
// first counter line at int 1 (the lines are kTileCountStride ints wide and only
// int 0 holds a count), for strided_scan_block.
__global__ void __launch_bounds__(kPrepThreads) k_tile_block_counts(int32_t* __restrict__ tile_count, int stride,
                                                                     int64_t num_tiles) {
    __shared__ long long s_warp[32];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kPrepTile;
    long long sum = 0;
#pragma unroll
    for (int k = 0; k < kPrepTile / kPrepThreads; ++k) {
        const int64_t t = base + k * kPrepThreads + threadIdx.x;
        if (t < num_tiles) sum += tile_count[t * stride];
    }
    long long total;
    block_exclusive_scan<kPrepThreads>(sum, s_warp, total);
    if (threadIdx.x == 0) tile_count[base * stride + 1] = static_cast<int32_t>(total);
}

// Whole scan in one CTA for n <= kSingleMax.
__global__ void __launch_bounds__(kScanBlocksThreads) k_scan_single(const int32_t* in, int32_t* out, int64_t n,
                                                                     int write_tail, int64_t* __restrict__ total_out) {
    __shared__ int32_t s_val[kSingleMax];
    __shared__ long long s_warp[32];
    for (int k = 0; k < kSingleItems; ++k) {
        const int64_t i = k * kScanBlocksThreads + threadIdx.x;
        s_val[i] = i < n ? in[i] : 0;
    }
    __syncthreads();
    int32_t v[kSingleItems];
    long long local = 0;
#pragma unroll
    for (int k = 0; k < kSingleItems; ++k) {
        v[k] = s_val[threadIdx.x * kSingleItems + k];
        local += v[k];
    }
    long long total;
    long long run = block_exclusive_scan<kScanBlocksThreads>(local, s_warp, total);
#pragma unroll
    for (int k = 0; k < kSingleItems; ++k) {
        s_val[threadIdx.x * kSingleItems + k] = static_cast<int32_t>(run);
        run += v[k];
    }
    __syncthreads();
    for (int k = 0; k < kSingleItems; ++k) {
        const int64_t i = k * kScanBlocksThreads + threadIdx.x;
        if (i < n) out[i] = s_val[i];
    }
    if (threadIdx.x == 0) {
        if (write_tail) out[n] = static_cast<int32_t>(total);
        if (total_out != nullptr) *total_out = static_cast<int64_t>(total);
    }
}

__global__ void k_scan_empty(int32_t* out, int write_tail, int64_t* total_out) {
    if (write_tail) out[0] = 0;
    if (total_out != nullptr) *total_out = 0;
}

}  // namespace

int64_t scan_scratch_bytes(int64_t n) {
    const int64_t nb = div_up(n, kScanTile);
    return arena_bytes(nb + 1, sizeof(long long)) + arena_bytes(1, sizeof(long long));
}

cudaError_t scan_exclusive_i32(const int32_t* in, int32_t* out, int64_t n, bool write_tail, int64_t* total_out,
                               void* scratch, cudaStream_t stream) {
    if (n == 0) {
        k_scan_empty<<<1, 1, 0, stream>>>(out, write_tail ? 1 : 0, total_out);
        return cudaGetLastError();
    }
    if (n <= kSingleMax) {
        k_scan_single<<<1, kScanBlocksThreads, 0, stream>>>(in, out, n, write_tail ? 1 : 0, total_out);
        return cudaGetLastError();
    }
    const int64_t nb = div_up(n, kScanTile);
    Arena arena{static_cast<char*>(scratch), scan_scratch_bytes(n), 0};
    long long* block_sums = arena.take<long long>(nb + 1);
    long long* total_ll = arena.take<long long>(1);
    k_scan_reduce<<<static_cast<unsigned>(nb), kScanThreads, 0, stream>>>(in, n, block_sums);
    if (nb <= kRedundantMaxBlocks) {
        k_scan_apply<kScanThreads, kScanItems><<<static_cast<unsigned>(nb), kScanThreads, 0, stream>>>(
            in, out, n, block_sums, 1, nb, write_tail ? 1 : 0, total_out);
        return cudaGetLastError();
    }
    k_scan_blocks<<<1, kScanBlocksThreads, 0, stream>>>(block_sums, nb, total_ll, nullptr);
    k_scan_apply<kScanThreads, kScanItems><<<static_cast<unsigned>(nb), kScanThreads, 0, stream>>>(
        in, out, n, block_sums, 0, nb, write_tail ? 1 : 0, total_out);
    return cudaGetLastError();
}

int64_t scan_fused_scratch_bytes(int64_t n) { return arena_bytes(div_up(n, kPrepTile) + 1, sizeof(long long)); }

cudaError_t scan_apply_with_block_sums(const int32_t* in, int32_t* out, int64_t n, const long long* block_sums,
                                       int64_t* total_out, const int32_t* tile_count, int count_stride,
                                       int64_t num_tiles, int32_t* tile_offsets, cudaStream_t stream) {
    constexpr int kItems = kPrepTile / kPrepThreads;
    const int64_t ntb = tile_count != nullptr ? div_up(num_tiles, kPrepTile) : 0;
    if (n == 0) {
        k_scan_empty<<<1, 1, 0, stream>>>(out, 1, total_out);
        if (ntb == 0) return cudaGetLastError();
    }
    const int64_t nb = div_up(n, kPrepTile);
    if (nb + ntb == 0) return cudaGetLastError();
    // many tile blocks (stacked frames): per-block tile sums first, so that no block
    // sums every count before its range
    const int32_t* block_counts = nullptr;
    if (ntb > kTileBlocksRedundant) {
        k_tile_block_counts<<<static_cast<unsigned>(ntb), kPrepThreads, 0, stream>>>(
            const_cast<int32_t*>(tile_count), count_stride, num_tiles);
        block_counts = tile_count + 1;
    }
    k_prepare_scan<kPrepThreads, kItems><<<static_cast<unsigned>(nb + ntb), kPrepThreads, 0, stream>>>(
        in, out, n, block_sums, nb, total_out, tile_count, count_stride, num_tiles, tile_offsets, ntb, block_counts);
    return cudaGetLastError();
}

}  // namespace oss
