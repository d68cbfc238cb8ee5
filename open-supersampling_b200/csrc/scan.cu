// Device-wide exclusive scan of int32 counts (reduce -> scan block sums -> apply).
// Used for the gid-major pair offsets, the per-tile list offsets and the radix
// digit offsets.  Sums are carried in int64 so an int32 overflow of the total is
// detected by the caller instead of wrapping silently.
#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;  // 2048 values per block
constexpr int kScanBlocksThreads = 1024;

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

__global__ void __launch_bounds__(kScanThreads) k_scan_apply(const int32_t* in, int32_t* out, int64_t n,
                                                              const long long* __restrict__ block_sums,
                                                              const long long* __restrict__ total_ll,
                                                              int write_tail) {
    __shared__ int32_t s_val[kScanTile];
    __shared__ long long s_warp[32];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t i = base + k * kScanThreads + threadIdx.x;
        s_val[k * kScanThreads + threadIdx.x] = i < n ? in[i] : 0;
    }
    __syncthreads();
    int32_t v[kScanItems];
    long long local = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        v[k] = s_val[threadIdx.x * kScanItems + k];
        local += v[k];
    }
    long long total;
    long long run = block_exclusive_scan<kScanThreads>(local, s_warp, total) + block_sums[blockIdx.x];
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        s_val[threadIdx.x * kScanItems + k] = static_cast<int32_t>(run);
        run += v[k];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const int64_t i = base + k * kScanThreads + threadIdx.x;
        if (i < n) out[i] = s_val[k * kScanThreads + threadIdx.x];
    }
    if (write_tail && blockIdx.x == 0 && threadIdx.x == 0) out[n] = static_cast<int32_t>(*total_ll);
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

cudaError_t scan_exclusive_i32(const int32_t* in, int32_t* out, int64_t n, bool write_tail,
                               int64_t* total_out, void* scratch, cudaStream_t stream) {
    if (n == 0) {
        k_scan_empty<<<1, 1, 0, stream>>>(out, write_tail ? 1 : 0, total_out);
        return cudaGetLastError();
    }
    const int64_t nb = div_up(n, kScanTile);
    Arena arena{static_cast<char*>(scratch), scan_scratch_bytes(n), 0};
    long long* block_sums = arena.take<long long>(nb + 1);
    long long* total_ll = arena.take<long long>(1);
    k_scan_reduce<<<static_cast<unsigned>(nb), kScanThreads, 0, stream>>>(in, n, block_sums);
    k_scan_blocks<<<1, kScanBlocksThreads, 0, stream>>>(block_sums, nb, total_ll, total_out);
    k_scan_apply<<<static_cast<unsigned>(nb), kScanThreads, 0, stream>>>(in, out, n, block_sums, total_ll,
                                                                         write_tail ? 1 : 0);
    return cudaGetLastError();
}

}  // namespace oss
