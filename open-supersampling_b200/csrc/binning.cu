// Pair expansion and list layouts for tile binning.
//
// expand: each Gaussian writes its tile rectangle, row-major, at its gid-major
// pair offset -- the order of the reference's build_tile_pairs
// (rasterizer_fwd.cu:111-133) -- and counts pairs per tile.  A stable sort of
// that array by tile id then yields, per tile, ascending gids: exactly the
// order of sorting (tile << 32 | gid) keys (rasterizer_fwd.cu:461-468).
#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) k_expand_pairs(int n, int ntx, const int4* __restrict__ aabb,
                                                            const int32_t* __restrict__ pair_offset,
                                                            uint32_t* __restrict__ keys, int32_t* __restrict__ vals,
                                                            int32_t* __restrict__ tile_count) {
    const int g = blockIdx.x * kThreads + threadIdx.x;
    if (g >= n) return;
    const int4 b = aabb[g];
    int out = pair_offset[g];
    for (int ty = b.y; ty < b.w; ++ty) {
        for (int tx = b.x; tx < b.z; ++tx) {
            const uint32_t t = static_cast<uint32_t>(ty * ntx + tx);
            keys[out] = t;
            vals[out] = g;
            atomicAdd(&tile_count[t], 1);
            ++out;
        }
    }
}

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

}  // namespace

cudaError_t launch_expand_pairs(int n, int ntx, const int32_t* aabb, const int32_t* pair_offset, uint32_t* keys,
                                int32_t* vals, int32_t* tile_count, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    k_expand_pairs<<<static_cast<unsigned>(div_up(n, kThreads)), kThreads, 0, stream>>>(
        n, ntx, reinterpret_cast<const int4*>(aabb), pair_offset, keys, vals, tile_count);
    return cudaGetLastError();
}

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

cudaError_t launch_set_i32(int32_t* p, int32_t value, cudaStream_t stream) {
    k_set_i32<<<1, 1, 0, stream>>>(p, value);
    return cudaGetLastError();
}

}  // namespace oss
