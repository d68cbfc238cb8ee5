// List layouts for tile binning: the full-frame lists of the reference forward
// (build_full_tile_pairs, rasterizer_fwd.cu:135-149) and the (tile, gid) key
// preparation of the generic counting sort (tile_bin_counting_sort.cu:71-128).
#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) k_full_tile_pairs(int n, int num_tiles, int32_t* __restrict__ gid_sorted,
                                                               int32_t* __restrict__ tile_offsets) {
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    const int64_t total = static_cast<int64_t>(n) * num_tiles;
    if (n > 0 && idx < total) gid_sorted[idx] = static_cast<int32_t>(idx % n);
    if (idx <= num_tiles) tile_offsets[idx] = static_cast<int32_t>(idx * n);
}

__global__ void __launch_bounds__(kThreads) k_tile_keys(int n, int num_tiles, const int32_t* __restrict__ tile_id,
                                                         const int32_t* __restrict__ gid, uint32_t* __restrict__ keys,
                                                         int32_t* __restrict__ vals, int32_t* __restrict__ tile_count) {
    const int i = blockIdx.x * kThreads + threadIdx.x;
    if (i >= n) return;
    const int32_t t = tile_id[i];
    const bool valid = t >= 0 && t < num_tiles;
    keys[i] = valid ? static_cast<uint32_t>(t) : static_cast<uint32_t>(num_tiles);
    vals[i] = gid[i];
    if (valid) atomicAdd(&tile_count[t], 1);
}

__global__ void k_set_i32(int32_t* p, int32_t v) { *p = v; }

__global__ void k_copy_i64(const int64_t* __restrict__ src, int64_t* dst) { *dst = *src; }

}  // namespace

cudaError_t launch_full_tile_pairs(int n, int num_tiles, int32_t* gid_sorted, int32_t* tile_offsets,
                                   cudaStream_t stream) {
    const int64_t total = static_cast<int64_t>(n) * num_tiles;
    const int64_t threads = total > num_tiles + 1 ? total : num_tiles + 1;
    k_full_tile_pairs<<<static_cast<unsigned>(div_up(threads, kThreads)), kThreads, 0, stream>>>(
        n, num_tiles, gid_sorted, tile_offsets);
    return cudaGetLastError();
}

cudaError_t launch_tile_keys(int n, int num_tiles, const int32_t* tile_id, const int32_t* gid, uint32_t* keys,
                             int32_t* vals, int32_t* tile_count, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    k_tile_keys<<<static_cast<unsigned>(div_up(n, kThreads)), kThreads, 0, stream>>>(n, num_tiles, tile_id, gid,
                                                                                     keys, vals, tile_count);
    return cudaGetLastError();
}

cudaError_t launch_copy_i64(const int64_t* src, int64_t* dst, cudaStream_t stream) {
    k_copy_i64<<<1, 1, 0, stream>>>(src, dst);
    return cudaGetLastError();
}

cudaError_t launch_set_i32(int32_t* p, int32_t value, cudaStream_t stream) {
    k_set_i32<<<1, 1, 0, stream>>>(p, value);
    return cudaGetLastError();
}

}  // namespace oss
