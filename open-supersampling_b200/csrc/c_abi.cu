// extern "C" entry points of liboss_b200.so (declared in include/oss_raster.h).
// Argument checks mirror the reference's TORCH_CHECKs (rasterizer_fwd.cu:489-522,
// rasterizer_bwd.cu:170-213, tile_bin_counting_sort.cu:76-81) and come back as
// status codes plus oss_last_error() text.
#include <climits>
#include <cstdint>
#include <mutex>
#include <string>

#include "internal.h"
#include "oss_common.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

#define OSS_CUDA_TRY(expr)                                                                       \
    do {                                                                                         \
        cudaError_t oss_err_ = (expr);                                                           \
        if (oss_err_ != cudaSuccess) {                                                           \
            return fail(OSS_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(oss_err_)); \
        }                                                                                        \
    } while (0)

#define OSS_CHECK(cond, code, msg)          \
    do {                                            \
        if (!(cond)) return fail((code), (msg));    \
    } while (0)

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

struct Grid {
    int n, h, w, ntx, nty, tiles;
};

// Shared size checks: n, h, w non-negative and within int32; tile count within int32.
int check_grid(int64_t n, int64_t h, int64_t w, Grid& g) {
    OSS_CHECK(n >= 0, OSS_ERR_INVALID, "N must be non-negative");
    OSS_CHECK(h >= 0 && w >= 0, OSS_ERR_INVALID, "H and W must be non-negative");
    OSS_CHECK(n <= INT_MAX, OSS_ERR_RANGE, "N exceeds int32 range");
    OSS_CHECK(h <= INT_MAX, OSS_ERR_RANGE, "H exceeds int32 range");
    OSS_CHECK(w <= INT_MAX, OSS_ERR_RANGE, "W exceeds int32 range");
    const int64_t ntx = (w + oss::kTile - 1) / oss::kTile;
    const int64_t nty = (h + oss::kTile - 1) / oss::kTile;
    OSS_CHECK(ntx * nty <= INT_MAX, OSS_ERR_RANGE, "number of tiles exceeds int32 range");
    g.n = static_cast<int>(n);
    g.h = static_cast<int>(h);
    g.w = static_cast<int>(w);
    g.ntx = static_cast<int>(ntx);
    g.nty = static_cast<int>(nty);
    g.tiles = static_cast<int>(ntx * nty);
    return OSS_OK;
}

// frames >= 1 stacked frames of g's tile grid, the stacked tile count within int32.
int check_frames(int64_t frames, const Grid& g) {
    OSS_CHECK(frames >= 1, OSS_ERR_INVALID, "frames must be positive");
    OSS_CHECK(frames <= INT_MAX && static_cast<int64_t>(g.tiles) * frames <= INT_MAX, OSS_ERR_RANGE,
              "number of tiles of all frames exceeds int32 range");
    return OSS_OK;
}

int check_mode(int32_t mode) {
    OSS_CHECK(mode == OSS_BIN_TIGHT3SIGMA || mode == OSS_BIN_EXACT || mode == OSS_BIN_FULL ||
                  mode == OSS_BIN_EXACT56,
              OSS_ERR_INVALID, "binning mode must be 0 (tight3sigma), 1 (exact), 2 (full) or 3 (exact56)");
    return OSS_OK;
}

int check_gaussian_inputs(int n, const float* xy, const float* scale, const float* rot) {
    if (n == 0) return OSS_OK;
    OSS_CHECK(xy != nullptr && scale != nullptr && rot != nullptr, OSS_ERR_INVALID, "xy, scale and rot must be non-null");
    OSS_CHECK(aligned(xy, 8) && aligned(scale, 8), OSS_ERR_INVALID, "xy and scale must be 8-byte aligned");
    return OSS_OK;
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

}  // namespace

extern "C" {

const char* oss_last_error(void) { return g_last_error.c_str(); }

int oss_abi_version(void) { return 9; }

int oss_preprocess(int64_t n, int64_t h, int64_t w, int64_t tile_size, int32_t mode, const float* xy,
                   const float* scale, const float* rot, float* conic, int32_t* aabb, int32_t* pair_count,
                   void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    OSS_CHECK(tile_size == oss::kTile, OSS_ERR_INVALID, "tile_size must be 16");
    if ((rc = check_mode(mode)) != OSS_OK) return rc;
    if ((rc = check_gaussian_inputs(g.n, xy, scale, rot)) != OSS_OK) return rc;
    if (g.n == 0) return OSS_OK;
    OSS_CHECK(conic != nullptr && aabb != nullptr && pair_count != nullptr, OSS_ERR_INVALID, "outputs must be non-null");
    OSS_CHECK(aligned(aabb, 16), OSS_ERR_INVALID, "aabb must be 16-byte aligned");
    OSS_CUDA_TRY(oss::launch_preprocess(g.n, g.ntx, g.nty, mode, xy, scale, rot, conic, aabb, pair_count, nullptr,
                                        nullptr, nullptr, 0, nullptr, nullptr, nullptr, as_stream(stream)));
    return OSS_OK;
}

int64_t oss_render_prepare_scratch_bytes(int64_t n) { return oss::scan_fused_scratch_bytes(n < 0 ? 0 : n); }

int64_t oss_tile_count_elems(int64_t num_tiles) {
    return (num_tiles < 0 ? 0 : num_tiles) * oss::kTileCountStride;
}

int oss_render_prepare(int64_t n, int64_t h, int64_t w, int32_t mode, const float* xy, const float* scale,
                       const float* rot, int64_t f, const float* feat, const float* opacity, float* conic,
                       int32_t* aabb, int32_t* pair_offset, float* geo, float* prec, int64_t* total_pairs,
                       int32_t* tile_count, int32_t* tile_offsets, void* scratch, int64_t scratch_bytes,
                       void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    if ((rc = check_mode(mode)) != OSS_OK) return rc;
    if ((rc = check_gaussian_inputs(g.n, xy, scale, rot)) != OSS_OK) return rc;
    OSS_CHECK(pair_offset != nullptr && total_pairs != nullptr, OSS_ERR_INVALID, "pair_offset and total_pairs must be non-null");
    const bool lists = mode != OSS_BIN_FULL && g.tiles > 0;
    OSS_CHECK(!lists || (tile_count != nullptr && tile_offsets != nullptr), OSS_ERR_INVALID,
              "tile_count and tile_offsets must be non-null");
    OSS_CHECK(scratch_bytes >= oss_render_prepare_scratch_bytes(n), OSS_ERR_SCRATCH, "render_prepare scratch too small");
    if (g.n > 0) {
        OSS_CHECK(conic != nullptr && aabb != nullptr && geo != nullptr, OSS_ERR_INVALID, "outputs must be non-null");
        OSS_CHECK(aligned(aabb, 16) && aligned(geo, 16), OSS_ERR_INVALID, "aabb and geo must be 16-byte aligned");
        OSS_CHECK(prec == nullptr || (aligned(prec, 16) && f >= 0 && f <= OSS_MAX_CHANNELS &&
                                      (f == 0 || feat != nullptr)),
                  OSS_ERR_INVALID, "prec (16-byte aligned) needs F in [0, 64] and feat");
    }
    cudaStream_t s = as_stream(stream);
    long long* block_sums = static_cast<long long*>(scratch);
    OSS_CHECK(g.n == 0 || (block_sums != nullptr && aligned(block_sums, 8)), OSS_ERR_INVALID,
              "scratch must be 8-byte aligned");
    int32_t* counts = lists ? tile_count : nullptr;
    if (counts != nullptr) {
        OSS_CUDA_TRY(cudaMemsetAsync(counts, 0, sizeof(int32_t) * oss_tile_count_elems(g.tiles), s));
    }
    OSS_CUDA_TRY(oss::launch_preprocess(g.n, g.ntx, g.nty, mode, xy, scale, rot, conic, aabb, pair_offset, geo,
                                        block_sums, counts, static_cast<int>(prec != nullptr ? f : 0), feat, opacity,
                                        prec, s));
    OSS_CUDA_TRY(oss::scan_apply_with_block_sums(pair_offset, pair_offset, g.n, block_sums, total_pairs, counts,
                                                 oss::kTileCountStride, g.tiles, lists ? tile_offsets : nullptr, s));
    return OSS_OK;
}

int64_t oss_bin_pairs_scratch_bytes(int64_t n, int64_t capacity, int64_t num_tiles) {
    (void)n;
    (void)num_tiles;
    return oss::tile_lists_scratch_bytes(capacity < 0 ? 0 : capacity);
}

int oss_bin_pairs(int64_t n, int64_t h, int64_t w, int32_t mode, const int32_t* aabb, int32_t* pair_offset,
                  int32_t* tile_count, const int64_t* total_pairs, int64_t capacity, const int32_t* sort_key,
                  const int32_t* key_order, int32_t* gid_sorted, int32_t* tile_offsets, int32_t* overflow,
                  void* scratch, int64_t scratch_bytes, void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    if ((rc = check_mode(mode)) != OSS_OK) return rc;
    OSS_CHECK(capacity >= 0, OSS_ERR_INVALID, "capacity must be non-negative");
    OSS_CHECK(capacity <= INT_MAX, OSS_ERR_RANGE, "capacity exceeds int32 range");
    OSS_CHECK(tile_offsets != nullptr && overflow != nullptr, OSS_ERR_INVALID,
              "tile_offsets and overflow must be non-null");
    OSS_CHECK(capacity == 0 || gid_sorted != nullptr, OSS_ERR_INVALID, "gid_sorted must be non-null");
    cudaStream_t s = as_stream(stream);
    if (mode == OSS_BIN_FULL) {
        OSS_CHECK(static_cast<int64_t>(g.n) * g.tiles <= capacity, OSS_ERR_RANGE,
                  "full-frame binning needs capacity >= N * num_tiles");
        OSS_CUDA_TRY(cudaMemsetAsync(overflow, 0, sizeof(int32_t), s));
        if (g.tiles == 0) {
            OSS_CUDA_TRY(cudaMemsetAsync(tile_offsets, 0, sizeof(int32_t), s));
            return OSS_OK;
        }
        OSS_CUDA_TRY(oss::launch_full_tile_pairs(g.n, g.tiles, gid_sorted, tile_offsets, s));
        return OSS_OK;
    }
    OSS_CHECK(scratch_bytes >= oss_bin_pairs_scratch_bytes(n, capacity, g.tiles), OSS_ERR_SCRATCH,
              "bin_pairs scratch too small");
    OSS_CHECK(g.n == 0 || g.tiles == 0 ||
                  (aabb != nullptr && aligned(aabb, 16) && pair_offset != nullptr && tile_count != nullptr &&
                   total_pairs != nullptr && (capacity == 0 || scratch != nullptr)),
              OSS_ERR_INVALID, "aabb (16-byte aligned), pair_offset, tile_count, total_pairs and scratch must be non-null");
    OSS_CHECK((sort_key == nullptr) == (key_order == nullptr), OSS_ERR_INVALID,
              "sort_key and key_order go together");
    OSS_CHECK(mode != OSS_BIN_FULL || sort_key == nullptr, OSS_ERR_INVALID, "full-frame lists take no sort key");
    OSS_CUDA_TRY(oss::build_tile_lists(g.n, g.ntx, g.tiles, aabb, pair_offset, tile_count, total_pairs, capacity,
                                       sort_key, key_order, gid_sorted, tile_offsets, overflow, scratch, s));
    return OSS_OK;
}

int64_t oss_render_bin_scratch_bytes(int64_t n, int64_t capacity, int64_t num_tiles) {
    (void)num_tiles;
    return oss::scan_fused_scratch_bytes(n < 0 ? 0 : n) + oss::tile_lists_scratch_bytes(capacity < 0 ? 0 : capacity);
}

int oss_render_bin(int64_t n, int64_t h, int64_t w, int64_t frames, const int32_t* frame_offsets, int32_t mode,
                   const float* xy, const float* scale, const float* rot, int64_t f, const float* feat,
                   const float* opacity, float* conic, int32_t* aabb, int32_t* pair_offset, float* geo, float* prec,
                   int64_t* total_pairs, int32_t* tile_count, int32_t* tile_offsets, int64_t capacity,
                   int32_t* gid_sorted, int32_t* overflow, void* scratch, int64_t scratch_bytes, void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    if ((rc = check_frames(frames, g)) != OSS_OK) return rc;
    OSS_CHECK(frames == 1 || frame_offsets != nullptr, OSS_ERR_INVALID, "frame_offsets must be non-null");
    const int tiles = g.tiles * static_cast<int>(frames);
    if ((rc = check_mode(mode)) != OSS_OK) return rc;
    OSS_CHECK(mode != OSS_BIN_FULL, OSS_ERR_INVALID,
              "render_bin builds culled lists; use render_prepare + bin_pairs for full-frame lists");
    if ((rc = check_gaussian_inputs(g.n, xy, scale, rot)) != OSS_OK) return rc;
    OSS_CHECK(capacity >= 0, OSS_ERR_INVALID, "capacity must be non-negative");
    OSS_CHECK(capacity <= INT_MAX, OSS_ERR_RANGE, "capacity exceeds int32 range");
    OSS_CHECK(pair_offset != nullptr && total_pairs != nullptr && tile_count != nullptr && tile_offsets != nullptr &&
                  overflow != nullptr,
              OSS_ERR_INVALID, "pair_offset, total_pairs, tile_count, tile_offsets and overflow must be non-null");
    OSS_CHECK(capacity == 0 || gid_sorted != nullptr, OSS_ERR_INVALID, "gid_sorted must be non-null");
    OSS_CHECK(scratch_bytes >= oss_render_bin_scratch_bytes(n, capacity, tiles), OSS_ERR_SCRATCH,
              "render_bin scratch too small");
    if (g.n > 0) {
        OSS_CHECK(conic != nullptr && aabb != nullptr && geo != nullptr, OSS_ERR_INVALID, "outputs must be non-null");
        OSS_CHECK(aligned(aabb, 16) && aligned(geo, 16), OSS_ERR_INVALID, "aabb and geo must be 16-byte aligned");
        OSS_CHECK(prec == nullptr || (aligned(prec, 16) && f >= 0 && f <= OSS_MAX_CHANNELS &&
                                      (f == 0 || feat != nullptr)),
                  OSS_ERR_INVALID, "prec (16-byte aligned) needs F in [0, 64] and feat");
        OSS_CHECK(scratch != nullptr && aligned(scratch, 8), OSS_ERR_INVALID, "scratch must be 8-byte aligned");
    }
    cudaStream_t s = as_stream(stream);
    oss::Arena arena{static_cast<char*>(scratch), scratch_bytes, 0};
    long long* block_sums = arena.take<long long>(oss::scan_fused_scratch_bytes(g.n) / sizeof(long long));
    void* list_scratch = arena.base + arena.used;
    int32_t* counts = tiles > 0 ? tile_count : nullptr;
    if (counts != nullptr) OSS_CUDA_TRY(cudaMemsetAsync(counts, 0, sizeof(int32_t) * oss_tile_count_elems(tiles), s));
    OSS_CUDA_TRY(oss::launch_preprocess_frames(g.n, g.ntx, g.nty, static_cast<int>(frames), frame_offsets, mode, xy,
                                               scale, rot, conic, aabb, pair_offset, geo, block_sums, counts,
                                               static_cast<int>(prec != nullptr ? f : 0), feat, opacity, prec, s));
    OSS_CUDA_TRY(oss::scan_apply_with_block_sums(pair_offset, pair_offset, g.n, block_sums, total_pairs, counts,
                                                 oss::kTileCountStride, tiles, counts != nullptr ? tile_offsets : nullptr,
                                                 s));
    OSS_CUDA_TRY(oss::build_tile_lists(g.n, g.ntx, tiles, aabb, pair_offset, tile_count, total_pairs, capacity,
                                       nullptr, nullptr, gid_sorted, tile_offsets, overflow, list_scratch, s));
    return OSS_OK;
}

int oss_publish_total(const int64_t* total_pairs, int64_t* host_total, void* stream) {
    OSS_CHECK(total_pairs != nullptr && host_total != nullptr, OSS_ERR_INVALID, "pointers must be non-null");
    void* mapped = nullptr;
    if (cudaHostGetDevicePointer(&mapped, host_total, 0) != cudaSuccess || mapped == nullptr) {
        cudaGetLastError();  // clear the sticky-free error of the failed query
        OSS_CHECK(false, OSS_ERR_INVALID, "host_total must be pinned host memory");
    }
    OSS_CUDA_TRY(oss::launch_copy_i64(total_pairs, static_cast<int64_t*>(mapped), as_stream(stream)));
    return OSS_OK;
}

int64_t oss_depth_order_scratch_bytes(int64_t n) { return oss::depth_order_scratch_bytes(n < 0 ? 0 : n); }

int oss_depth_order(int64_t n, const float* depth, int32_t* order, int32_t* rank, void* scratch,
                    int64_t scratch_bytes, void* stream) {
    OSS_CHECK(n >= 0, OSS_ERR_INVALID, "N must be non-negative");
    OSS_CHECK(n <= INT_MAX, OSS_ERR_RANGE, "N exceeds int32 range");
    OSS_CHECK(scratch_bytes >= oss_depth_order_scratch_bytes(n), OSS_ERR_SCRATCH, "depth_order scratch too small");
    if (n == 0) return OSS_OK;
    OSS_CHECK(depth != nullptr && order != nullptr && rank != nullptr && scratch != nullptr, OSS_ERR_INVALID,
              "depth, order, rank and scratch must be non-null");
    OSS_CUDA_TRY(oss::depth_order(static_cast<int>(n), depth, order, rank, scratch, as_stream(stream)));
    return OSS_OK;
}

int oss_render_alpha_forward(int64_t n, int64_t f, int64_t h, int64_t w, const float* geo, const float* feat,
                             const float* opacity, const float* background, const int32_t* gid_sorted,
                             const int32_t* tile_offsets, float* image, float* t_final, int32_t* n_contrib,
                             void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    OSS_CHECK(f >= 0 && f <= OSS_MAX_CHANNELS, OSS_ERR_INVALID, "F must be in [0, 64]");
    if (g.tiles == 0) return OSS_OK;
    OSS_CHECK(tile_offsets != nullptr && t_final != nullptr && n_contrib != nullptr && (f == 0 || image != nullptr),
              OSS_ERR_INVALID, "tile_offsets, image, t_final and n_contrib must be non-null");
    OSS_CHECK(g.n == 0 || (geo != nullptr && aligned(geo, 16) && (f == 0 || feat != nullptr)), OSS_ERR_INVALID,
              "geo (16-byte aligned) and feat must be non-null");
    OSS_CUDA_TRY(oss::launch_render_alpha_forward(static_cast<int>(f), g.h, g.w, geo, feat, opacity, background,
                                                  gid_sorted, tile_offsets, image, t_final, n_contrib,
                                                  as_stream(stream)));
    return OSS_OK;
}

int oss_alpha_pair_grad_stride(int64_t f) {
    return oss::alpha_pair_stride(static_cast<int>(f < 0 ? 0 : (f > OSS_MAX_CHANNELS ? OSS_MAX_CHANNELS : f)));
}

int64_t oss_render_alpha_backward_scratch_bytes(int64_t total_pairs, int64_t f) {
    if (total_pairs < 0) total_pairs = 0;
    return oss::arena_bytes(total_pairs * oss_alpha_pair_grad_stride(f), 4);
}

int oss_render_alpha_backward(int64_t n, int64_t f, int64_t h, int64_t w, const float* geo, const float* feat,
                              const float* opacity, const float* background, const float* scale, const float* rot,
                              const int32_t* aabb, const int32_t* pair_offset, int64_t total_pairs,
                              const int32_t* gid_sorted, const int32_t* tile_offsets, const float* t_final,
                              const int32_t* n_contrib, const float* grad_image, float* d_xy, float* d_conic,
                              float* d_feat, float* d_opacity, float* d_scale, float* d_rot, void* scratch,
                              int64_t scratch_bytes, void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    OSS_CHECK(f >= 0 && f <= OSS_MAX_CHANNELS, OSS_ERR_INVALID, "F must be in [0, 64]");
    OSS_CHECK(total_pairs >= 0 && total_pairs <= INT_MAX, OSS_ERR_RANGE, "total pair count exceeds int32 range");
    OSS_CHECK(scratch_bytes >= oss_render_alpha_backward_scratch_bytes(total_pairs, f), OSS_ERR_SCRATCH,
              "render_alpha_backward scratch too small");
    if (g.n == 0) return OSS_OK;
    OSS_CHECK(geo != nullptr && aligned(geo, 16) && aabb != nullptr && aligned(aabb, 16) && pair_offset != nullptr,
              OSS_ERR_INVALID, "geo, aabb (16-byte aligned) and pair_offset must be non-null");
    OSS_CHECK(d_xy != nullptr && d_conic != nullptr && (f == 0 || (feat != nullptr && d_feat != nullptr)),
              OSS_ERR_INVALID, "gradient outputs must be non-null");
    OSS_CHECK(d_scale == nullptr || (scale != nullptr && rot != nullptr && d_rot != nullptr), OSS_ERR_INVALID,
              "d_scale needs scale, rot and d_rot");
    cudaStream_t s = as_stream(stream);
    float* pairgrad = static_cast<float*>(scratch);
    if (g.tiles > 0 && total_pairs > 0) {
        OSS_CHECK(scratch != nullptr && aligned(scratch, 16), OSS_ERR_INVALID, "scratch must be 16-byte aligned");
        OSS_CHECK(gid_sorted != nullptr && tile_offsets != nullptr && t_final != nullptr && n_contrib != nullptr &&
                      grad_image != nullptr,
                  OSS_ERR_INVALID, "lists, t_final, n_contrib and grad_image must be non-null");
        OSS_CUDA_TRY(oss::launch_render_alpha_backward(static_cast<int>(f), g.h, g.w, geo, feat, opacity, background,
                                                       gid_sorted, tile_offsets, t_final, n_contrib, grad_image, aabb,
                                                       pair_offset, pairgrad, s));
    }
    OSS_CUDA_TRY(oss::launch_reduce_alpha_grads(g.n, static_cast<int>(f), pairgrad, pair_offset, geo, scale, rot, d_xy,
                                                d_conic, d_feat, d_opacity, d_scale, d_rot, s));
    return OSS_OK;
}

int oss_entry_record_floats(int64_t f) {
    return oss::entry_record_floats(static_cast<int>(f < 1 ? 1 : (f > OSS_MAX_CHANNELS ? OSS_MAX_CHANNELS : f)));
}

int oss_render_forward(int64_t n, int64_t f, int64_t h, int64_t w, const float* geo, const float* feat,
                       const float* opacity, const float* prec, const int32_t* gid_sorted,
                       const int32_t* tile_offsets, float* image, const int32_t* aabb, const int32_t* pair_offset,
                       float* records, int32_t* slots, void* stream) {
    return oss_render_forward_frames(n, f, h, w, 1, geo, feat, opacity, prec, gid_sorted, tile_offsets, image, aabb,
                                     pair_offset, records, slots, stream);
}

int oss_render_forward_frames(int64_t n, int64_t f, int64_t h, int64_t w, int64_t frames, const float* geo,
                              const float* feat, const float* opacity, const float* prec, const int32_t* gid_sorted,
                              const int32_t* tile_offsets, float* image, const int32_t* aabb,
                              const int32_t* pair_offset, float* records, int32_t* slots, void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    if ((rc = check_frames(frames, g)) != OSS_OK) return rc;
    OSS_CHECK(f >= 0, OSS_ERR_INVALID, "F must be non-negative");
    OSS_CHECK(f <= OSS_MAX_CHANNELS, OSS_ERR_INVALID, "F must be <= 64");
    if (g.tiles == 0 || f == 0) return OSS_OK;
    OSS_CHECK(tile_offsets != nullptr && image != nullptr, OSS_ERR_INVALID, "tile_offsets and image must be non-null");
    OSS_CHECK(g.n == 0 || (prec != nullptr ? aligned(prec, 16)
                                            : (geo != nullptr && feat != nullptr && aligned(geo, 16))),
              OSS_ERR_INVALID, "prec (16-byte aligned), or geo (16-byte aligned) and feat, must be non-null");
    OSS_CHECK(slots == nullptr || records != nullptr, OSS_ERR_INVALID, "slots are written with records");
    OSS_CHECK(records == nullptr || aligned(records, 16), OSS_ERR_INVALID, "records must be 16-byte aligned");
    OSS_CHECK(slots == nullptr || (aabb != nullptr && aligned(aabb, 16) && pair_offset != nullptr), OSS_ERR_INVALID,
              "slots need aabb (16-byte aligned) and pair_offset");
    OSS_CUDA_TRY(oss::launch_render_forward(static_cast<int>(f), g.h, g.w, geo, feat, opacity, gid_sorted,
                                            tile_offsets, image, aabb, pair_offset, records, slots, prec,
                                            as_stream(stream), static_cast<int>(frames)));
    return OSS_OK;
}

int64_t oss_render_backward_pairs_scratch_bytes(int64_t total_pairs, int64_t num_tiles) {
    if (total_pairs < 0) total_pairs = 0;
    if (num_tiles < 0) num_tiles = 0;
    return oss::backward_items_scratch_bytes(total_pairs, num_tiles);
}

int64_t oss_render_backward_scratch_bytes(int64_t total_pairs, int64_t f, int64_t num_tiles) {
    if (total_pairs < 0) total_pairs = 0;
    if (f < 0) f = 0;
    return oss::arena_bytes(total_pairs * oss::backward_pair_stride(static_cast<int>(f)), 4) +
           oss_render_backward_pairs_scratch_bytes(total_pairs, num_tiles);
}

int oss_render_backward(int64_t n, int64_t f, int64_t h, int64_t w, const float* geo, const float* feat,
                        const float* opacity, const float* scale, const float* rot, const int32_t* aabb,
                        const int32_t* pair_offset, int64_t total_pairs, const int32_t* gid_sorted,
                        const int32_t* tile_offsets, const float* records, const int32_t* slots,
                        const float* grad_image, float* d_xy, float* d_conic, float* d_feat, float* d_opacity,
                        float* d_scale, float* d_rot, void* scratch, int64_t scratch_bytes, void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    OSS_CHECK(f >= 0 && f <= OSS_MAX_CHANNELS, OSS_ERR_INVALID, "F must be in [0, 64]");
    OSS_CHECK(total_pairs >= 0 && total_pairs <= INT_MAX, OSS_ERR_RANGE, "total pair count exceeds int32 range");
    OSS_CHECK(scratch_bytes >= oss_render_backward_scratch_bytes(total_pairs, f, g.tiles), OSS_ERR_SCRATCH,
              "render_backward scratch too small");
    if (g.n == 0) return OSS_OK;
    OSS_CHECK(geo != nullptr && aligned(geo, 16) && aabb != nullptr && aligned(aabb, 16) && pair_offset != nullptr,
              OSS_ERR_INVALID, "geo, aabb (16-byte aligned) and pair_offset must be non-null");
    OSS_CHECK(d_xy != nullptr && d_conic != nullptr, OSS_ERR_INVALID, "d_xy and d_conic must be non-null");
    OSS_CHECK(f == 0 || (feat != nullptr && d_feat != nullptr), OSS_ERR_INVALID, "feat and d_feat must be non-null");
    OSS_CHECK(d_scale == nullptr || (scale != nullptr && rot != nullptr && d_rot != nullptr), OSS_ERR_INVALID,
              "d_scale needs scale, rot and d_rot");
    float* pairgrad = static_cast<float*>(scratch);
    const int64_t pg_bytes = oss::arena_bytes(total_pairs * oss::backward_pair_stride(static_cast<int>(f)), 4);
    void* items = static_cast<char*>(scratch) + pg_bytes;
    rc = oss_render_backward_pairs(n, f, h, w, geo, feat, opacity, aabb, pair_offset, total_pairs, gid_sorted,
                                   tile_offsets, records, slots, grad_image, pairgrad, items, scratch_bytes - pg_bytes,
                                   stream);
    if (rc != OSS_OK) return rc;
    return oss_reduce_pair_grads(n, f, pairgrad, pair_offset, geo, feat, opacity, scale, rot, d_xy, d_conic, d_feat,
                                 d_opacity, d_scale, d_rot, stream);
}

int oss_pair_grad_stride(int64_t f) {
    return oss::backward_pair_stride(static_cast<int>(f < 0 ? 0 : (f > OSS_MAX_CHANNELS ? OSS_MAX_CHANNELS : f)));
}

int oss_render_backward_pairs(int64_t n, int64_t f, int64_t h, int64_t w, const float* geo, const float* feat,
                              const float* opacity, const int32_t* aabb, const int32_t* pair_offset,
                              int64_t total_pairs, const int32_t* gid_sorted, const int32_t* tile_offsets,
                              const float* records, const int32_t* slots, const float* grad_image, float* pairgrad,
                              void* scratch, int64_t scratch_bytes, void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    OSS_CHECK(f >= 0 && f <= OSS_MAX_CHANNELS, OSS_ERR_INVALID, "F must be in [0, 64]");
    OSS_CHECK(total_pairs >= 0 && total_pairs <= INT_MAX, OSS_ERR_RANGE, "total pair count exceeds int32 range");
    OSS_CHECK(scratch_bytes >= oss_render_backward_pairs_scratch_bytes(total_pairs, g.tiles), OSS_ERR_SCRATCH,
              "render_backward_pairs scratch too small");
    if (g.n == 0 || total_pairs == 0 || g.tiles == 0) return OSS_OK;
    OSS_CHECK(geo != nullptr && aligned(geo, 16) && aabb != nullptr && aligned(aabb, 16) && pair_offset != nullptr,
              OSS_ERR_INVALID, "geo, aabb (16-byte aligned) and pair_offset must be non-null");
    OSS_CHECK(f == 0 || feat != nullptr, OSS_ERR_INVALID, "feat must be non-null");
    OSS_CHECK(pairgrad != nullptr && aligned(pairgrad, 16), OSS_ERR_INVALID, "pairgrad must be 16-byte aligned");
    OSS_CHECK(scratch != nullptr && aligned(scratch, 16), OSS_ERR_INVALID, "scratch must be 16-byte aligned");
    OSS_CHECK(gid_sorted != nullptr && tile_offsets != nullptr && grad_image != nullptr, OSS_ERR_INVALID,
              "lists and grad_image must be non-null");
    OSS_CHECK(slots == nullptr || records != nullptr, OSS_ERR_INVALID, "slots come with records");
    OSS_CHECK(records == nullptr || aligned(records, 16), OSS_ERR_INVALID, "records must be 16-byte aligned");
    OSS_CUDA_TRY(oss::launch_render_backward_tiles(static_cast<int>(f), g.h, g.w, total_pairs, geo, feat, opacity,
                                                   gid_sorted, tile_offsets, grad_image, aabb, pair_offset, records,
                                                   slots, pairgrad, oss_pair_grad_stride(f), nullptr, nullptr, nullptr,
                                                   scratch, as_stream(stream)));
    return OSS_OK;
}

int oss_backward_items(int64_t h, int64_t w, int64_t total_pairs, const int32_t* tile_offsets, void* items,
                       int64_t items_bytes, void* stream) {
    return oss_backward_items_frames(h, w, 1, total_pairs, tile_offsets, items, items_bytes, stream);
}

int oss_backward_items_frames(int64_t h, int64_t w, int64_t frames, int64_t total_pairs, const int32_t* tile_offsets,
                              void* items, int64_t items_bytes, void* stream) {
    Grid g;
    int rc = check_grid(0, h, w, g);
    if (rc != OSS_OK) return rc;
    if ((rc = check_frames(frames, g)) != OSS_OK) return rc;
    const int64_t tiles = static_cast<int64_t>(g.tiles) * frames;
    OSS_CHECK(total_pairs >= 0 && total_pairs <= INT_MAX, OSS_ERR_RANGE, "total pair count exceeds int32 range");
    OSS_CHECK(items_bytes >= oss_render_backward_pairs_scratch_bytes(total_pairs, tiles), OSS_ERR_SCRATCH,
              "backward item table too small");
    if (total_pairs == 0 || tiles == 0) return OSS_OK;
    OSS_CHECK(tile_offsets != nullptr && items != nullptr && aligned(items, 16), OSS_ERR_INVALID,
              "tile_offsets and items (16-byte aligned) must be non-null");
    OSS_CUDA_TRY(oss::launch_backward_items(g.h, g.w, total_pairs, tile_offsets, items, as_stream(stream),
                                            static_cast<int>(frames)));
    return OSS_OK;
}

int oss_render_backward_items(int64_t n, int64_t f, int64_t h, int64_t w, const float* geo, const float* feat,
                              const float* opacity, const int32_t* aabb, const int32_t* pair_offset,
                              int64_t total_pairs, const int32_t* gid_sorted, const int32_t* tile_offsets,
                              const float* records, const int32_t* slots, const float* grad_image, float* pairgrad,
                              void* items, int64_t items_bytes, void* stream) {
    return oss_render_backward_items_frames(n, f, h, w, 1, geo, feat, opacity, aabb, pair_offset, total_pairs,
                                            gid_sorted, tile_offsets, records, slots, grad_image, pairgrad, items,
                                            items_bytes, stream);
}

int oss_render_backward_items_frames(int64_t n, int64_t f, int64_t h, int64_t w, int64_t frames, const float* geo,
                                     const float* feat, const float* opacity, const int32_t* aabb,
                                     const int32_t* pair_offset, int64_t total_pairs, const int32_t* gid_sorted,
                                     const int32_t* tile_offsets, const float* records, const int32_t* slots,
                                     const float* grad_image, float* pairgrad, void* items, int64_t items_bytes,
                                     void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    if ((rc = check_frames(frames, g)) != OSS_OK) return rc;
    const int64_t tiles = static_cast<int64_t>(g.tiles) * frames;
    OSS_CHECK(f >= 0 && f <= OSS_MAX_CHANNELS, OSS_ERR_INVALID, "F must be in [0, 64]");
    OSS_CHECK(total_pairs >= 0 && total_pairs <= INT_MAX, OSS_ERR_RANGE, "total pair count exceeds int32 range");
    OSS_CHECK(items_bytes >= oss_render_backward_pairs_scratch_bytes(total_pairs, tiles), OSS_ERR_SCRATCH,
              "backward item table too small");
    if (g.n == 0 || total_pairs == 0 || tiles == 0) return OSS_OK;
    OSS_CHECK(geo != nullptr && aligned(geo, 16) && aabb != nullptr && aligned(aabb, 16) && pair_offset != nullptr,
              OSS_ERR_INVALID, "geo, aabb (16-byte aligned) and pair_offset must be non-null");
    OSS_CHECK(f == 0 || feat != nullptr, OSS_ERR_INVALID, "feat must be non-null");
    OSS_CHECK(pairgrad != nullptr && aligned(pairgrad, 16), OSS_ERR_INVALID, "pairgrad must be 16-byte aligned");
    OSS_CHECK(items != nullptr && aligned(items, 16), OSS_ERR_INVALID, "items must be 16-byte aligned");
    OSS_CHECK(gid_sorted != nullptr && tile_offsets != nullptr && grad_image != nullptr, OSS_ERR_INVALID,
              "lists and grad_image must be non-null");
    OSS_CHECK(slots == nullptr || records != nullptr, OSS_ERR_INVALID, "slots come with records");
    OSS_CHECK(records == nullptr || aligned(records, 16), OSS_ERR_INVALID, "records must be 16-byte aligned");
    OSS_CUDA_TRY(oss::launch_render_backward_items(static_cast<int>(f), g.h, g.w, total_pairs, geo, feat, opacity,
                                                   gid_sorted, tile_offsets, grad_image, aabb, pair_offset, records,
                                                   slots, pairgrad, oss_pair_grad_stride(f), nullptr, nullptr, nullptr,
                                                   items, as_stream(stream), static_cast<int>(frames)));
    return OSS_OK;
}

int oss_reduce_pair_grads(int64_t n, int64_t f, const float* pairgrad, const int32_t* pair_offset, const float* geo,
                          const float* feat, const float* opacity, const float* scale, const float* rot, float* d_xy,
                          float* d_conic, float* d_feat, float* d_opacity, float* d_scale, float* d_rot,
                          void* stream) {
    OSS_CHECK(n >= 0 && n <= INT_MAX, OSS_ERR_RANGE, "N exceeds int32 range");
    OSS_CHECK(f >= 0 && f <= OSS_MAX_CHANNELS, OSS_ERR_INVALID, "F must be in [0, 64]");
    if (n == 0) return OSS_OK;
    OSS_CHECK(pair_offset != nullptr && d_xy != nullptr && d_conic != nullptr, OSS_ERR_INVALID,
              "pair_offset, d_xy and d_conic must be non-null");
    OSS_CHECK(geo != nullptr && aligned(geo, 16), OSS_ERR_INVALID, "geo must be 16-byte aligned");
    OSS_CHECK(f == 0 || (feat != nullptr && d_feat != nullptr), OSS_ERR_INVALID, "feat and d_feat must be non-null");
    OSS_CHECK(d_scale == nullptr || (scale != nullptr && rot != nullptr && d_rot != nullptr), OSS_ERR_INVALID,
              "d_scale needs scale, rot and d_rot");
    OSS_CHECK(pairgrad == nullptr || aligned(pairgrad, 16), OSS_ERR_INVALID, "pairgrad must be 16-byte aligned");
    OSS_CUDA_TRY(oss::launch_reduce_gaussian_grads(static_cast<int>(n), static_cast<int>(f), pairgrad,
                                                   oss_pair_grad_stride(f), pair_offset, geo, feat, opacity, scale, rot,
                                                   d_xy, d_conic, d_feat, d_opacity, d_scale, d_rot,
                                                   as_stream(stream)));
    return OSS_OK;
}

// ---- one-pass feathered overlapping-tile render -------------------------------

namespace {

int check_feather(int32_t overlap, int64_t f, const Grid& g, oss::FeatherTable* tab) {
    OSS_CHECK(overlap > 0, OSS_ERR_INVALID, "overlap must be positive");
    OSS_CHECK(f >= 0 && f <= 16, OSS_ERR_INVALID, "the feathered render takes F in [0, 16]");
    OSS_CHECK((static_cast<int64_t>(g.w) + overlap + oss::kTile - 1) / oss::kTile <= oss::kFeatherMaxTiles &&
                  (static_cast<int64_t>(g.h) + overlap + oss::kTile - 1) / oss::kTile <= oss::kFeatherMaxTiles,
              OSS_ERR_RANGE, "the feathered render takes at most 32767 tiles per axis");
    OSS_CHECK(oss::feather_table(overlap, tab) != 0, OSS_ERR_RANGE,
              "overlap too wide for the one-pass feathered render (its weight sum could reach the 1e-6 clamp)");
    return OSS_OK;
}

}  // namespace

int oss_feather_supported(int32_t overlap, int64_t f, int64_t h, int64_t w) {
    Grid g;
    if (check_grid(0, h, w, g) != OSS_OK) return 0;
    oss::FeatherTable tab;
    return check_feather(overlap, f, g, &tab) == OSS_OK ? 1 : 0;
}

int64_t oss_feather_virtual_count(int64_t n) { return (n < 0 ? 0 : n) * oss::kFeatherVariants; }

int64_t oss_render_prepare_feathered_scratch_bytes(int64_t n) {
    return oss::scan_fused_scratch_bytes(oss_feather_virtual_count(n));
}

int oss_render_prepare_feathered(int64_t n, int64_t h, int64_t w, int32_t mode, int32_t overlap, const float* xy,
                                 const float* scale, const float* rot, int64_t f, const float* feat,
                                 const float* opacity, float* conic, float* geo, int32_t* vaabb, int32_t* vpair_offset,
                                 float* vprec, int32_t* vwin, int64_t* total_pairs, int32_t* tile_count,
                                 int32_t* tile_offsets, void* scratch, int64_t scratch_bytes, void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    if ((rc = check_mode(mode)) != OSS_OK) return rc;
    if ((rc = check_gaussian_inputs(g.n, xy, scale, rot)) != OSS_OK) return rc;
    oss::FeatherTable tab;
    if ((rc = check_feather(overlap, f, g, &tab)) != OSS_OK) return rc;
    const int64_t nv = oss_feather_virtual_count(n);
    OSS_CHECK(nv <= INT_MAX, OSS_ERR_RANGE, "4 N exceeds int32 range");
    OSS_CHECK(vpair_offset != nullptr && total_pairs != nullptr, OSS_ERR_INVALID,
              "vpair_offset and total_pairs must be non-null");
    OSS_CHECK(g.tiles == 0 || (tile_count != nullptr && tile_offsets != nullptr), OSS_ERR_INVALID,
              "tile_count and tile_offsets must be non-null");
    OSS_CHECK(scratch_bytes >= oss_render_prepare_feathered_scratch_bytes(n), OSS_ERR_SCRATCH,
              "render_prepare_feathered scratch too small");
    if (g.n > 0) {
        OSS_CHECK(conic != nullptr && geo != nullptr && vaabb != nullptr && vprec != nullptr && vwin != nullptr,
                  OSS_ERR_INVALID, "outputs must be non-null");
        OSS_CHECK(aligned(geo, 16) && aligned(vaabb, 16) && aligned(vprec, 16) && aligned(vwin, 16), OSS_ERR_INVALID,
                  "geo, vaabb, vprec and vwin must be 16-byte aligned");
        OSS_CHECK(f == 0 || feat != nullptr, OSS_ERR_INVALID, "feat must be non-null");
        OSS_CHECK(scratch != nullptr && aligned(scratch, 8), OSS_ERR_INVALID, "scratch must be 8-byte aligned");
    }
    cudaStream_t s = as_stream(stream);
    if (g.tiles > 0) OSS_CUDA_TRY(cudaMemsetAsync(tile_count, 0, sizeof(int32_t) * oss_tile_count_elems(g.tiles), s));
    long long* block_sums = static_cast<long long*>(scratch);
    OSS_CUDA_TRY(oss::launch_prepare_feathered(g.n, g.h, g.w, mode, overlap, xy, scale, rot, static_cast<int>(f), feat,
                                               opacity, conic, geo, vaabb, vpair_offset, vprec, vwin, block_sums,
                                               g.tiles > 0 ? tile_count : nullptr, s));
    OSS_CUDA_TRY(oss::scan_apply_with_block_sums(vpair_offset, vpair_offset, nv, block_sums, total_pairs,
                                                 g.tiles > 0 ? tile_count : nullptr, oss::kTileCountStride, g.tiles,
                                                 g.tiles > 0 ? tile_offsets : nullptr, s));
    return OSS_OK;
}

int oss_render_forward_feathered(int64_t n, int64_t f, int64_t h, int64_t w, int32_t overlap, const float* vprec,
                                 const int32_t* vwin, const int32_t* gid_sorted, const int32_t* tile_offsets,
                                 float* image, float* records, uint16_t* entry_pat, void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    oss::FeatherTable tab;
    if ((rc = check_feather(overlap, f, g, &tab)) != OSS_OK) return rc;
    if (g.tiles == 0 || f == 0) return OSS_OK;
    OSS_CHECK(tile_offsets != nullptr && image != nullptr, OSS_ERR_INVALID, "tile_offsets and image must be non-null");
    OSS_CHECK(g.n == 0 || (vprec != nullptr && aligned(vprec, 16) && vwin != nullptr && aligned(vwin, 16)),
              OSS_ERR_INVALID, "vprec and vwin (16-byte aligned) must be non-null");
    OSS_CHECK((records == nullptr) == (entry_pat == nullptr), OSS_ERR_INVALID, "records and entry_pat go together");
    OSS_CHECK(records == nullptr || aligned(records, 16), OSS_ERR_INVALID, "records must be 16-byte aligned");
    OSS_CUDA_TRY(oss::launch_render_forward_feathered(static_cast<int>(f), g.h, g.w, tab, vprec, vwin, gid_sorted,
                                                      tile_offsets, image, records, entry_pat, as_stream(stream)));
    return OSS_OK;
}

int oss_render_backward_feathered(int64_t n, int64_t f, int64_t h, int64_t w, int32_t overlap, const int32_t* vaabb,
                                  const int32_t* vpair_offset, int64_t total_pairs, const int32_t* gid_sorted,
                                  const int32_t* tile_offsets, const float* records, const uint16_t* entry_pat,
                                  const float* grad_image, float* pairgrad, void* items, int64_t items_bytes,
                                  void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    oss::FeatherTable tab;
    if ((rc = check_feather(overlap, f, g, &tab)) != OSS_OK) return rc;
    OSS_CHECK(total_pairs >= 0 && total_pairs <= INT_MAX, OSS_ERR_RANGE, "total pair count exceeds int32 range");
    OSS_CHECK(items_bytes >= oss_render_backward_pairs_scratch_bytes(total_pairs, g.tiles), OSS_ERR_SCRATCH,
              "backward item table too small");
    if (g.n == 0 || total_pairs == 0 || g.tiles == 0) return OSS_OK;
    OSS_CHECK(vaabb != nullptr && aligned(vaabb, 16) && vpair_offset != nullptr, OSS_ERR_INVALID,
              "vaabb (16-byte aligned) and vpair_offset must be non-null");
    OSS_CHECK(records != nullptr && aligned(records, 16) && entry_pat != nullptr, OSS_ERR_INVALID,
              "the forward's records (16-byte aligned) and entry_pat must be non-null");
    OSS_CHECK(pairgrad != nullptr && aligned(pairgrad, 16), OSS_ERR_INVALID, "pairgrad must be 16-byte aligned");
    OSS_CHECK(items != nullptr && aligned(items, 16), OSS_ERR_INVALID, "items must be 16-byte aligned");
    OSS_CHECK(gid_sorted != nullptr && tile_offsets != nullptr && grad_image != nullptr, OSS_ERR_INVALID,
              "lists and grad_image must be non-null");
    OSS_CUDA_TRY(oss::launch_render_backward_feathered(static_cast<int>(f), g.h, g.w, total_pairs, tab, gid_sorted,
                                                       tile_offsets, grad_image, vaabb, vpair_offset, records,
                                                       entry_pat, pairgrad, oss_pair_grad_stride(f), items,
                                                       as_stream(stream)));
    return OSS_OK;
}

int oss_reduce_pair_grads_feathered(int64_t n, int64_t f, const float* pairgrad, const int32_t* vpair_offset,
                                    const float* geo, const float* feat, const float* opacity, const float* scale,
                                    const float* rot, float* d_xy, float* d_conic, float* d_feat, float* d_opacity,
                                    float* d_scale, float* d_rot, void* stream) {
    OSS_CHECK(n >= 0 && oss_feather_virtual_count(n) <= INT_MAX, OSS_ERR_RANGE, "4 N exceeds int32 range");
    OSS_CHECK(f >= 0 && f <= OSS_MAX_CHANNELS, OSS_ERR_INVALID, "F must be in [0, 64]");
    if (n == 0) return OSS_OK;
    OSS_CHECK(vpair_offset != nullptr && d_xy != nullptr && d_conic != nullptr, OSS_ERR_INVALID,
              "vpair_offset, d_xy and d_conic must be non-null");
    OSS_CHECK(geo != nullptr && aligned(geo, 16), OSS_ERR_INVALID, "geo must be 16-byte aligned");
    OSS_CHECK(f == 0 || (feat != nullptr && d_feat != nullptr), OSS_ERR_INVALID, "feat and d_feat must be non-null");
    OSS_CHECK(d_scale == nullptr || (scale != nullptr && rot != nullptr && d_rot != nullptr), OSS_ERR_INVALID,
              "d_scale needs scale, rot and d_rot");
    OSS_CHECK(pairgrad == nullptr || aligned(pairgrad, 16), OSS_ERR_INVALID, "pairgrad must be 16-byte aligned");
    OSS_CUDA_TRY(oss::launch_reduce_gaussian_grads(static_cast<int>(n), static_cast<int>(f), pairgrad,
                                                   oss_pair_grad_stride(f), vpair_offset, geo, feat, opacity, scale,
                                                   rot, d_xy, d_conic, d_feat, d_opacity, d_scale, d_rot,
                                                   as_stream(stream), false, oss::kFeatherVariants));
    return OSS_OK;
}

int64_t oss_rasterize_backward_lists_scratch_bytes(int64_t n, int64_t total_pairs, int64_t num_tiles) {
    if (n < 0) n = 0;
    return oss::arena_bytes(n * 8, 4) + oss_render_backward_pairs_scratch_bytes(total_pairs, num_tiles);
}

int oss_rasterize_backward_lists(int64_t n, int64_t f, int64_t h, int64_t w, const float* xy, const float* conic,
                                 const float* feat, const int32_t* gid_sorted, int64_t total_pairs,
                                 const int32_t* tile_offsets, const float* grad_image, float* d_xy, float* d_conic,
                                 float* d_feat, void* scratch, int64_t scratch_bytes, void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    OSS_CHECK(f >= 0 && f <= OSS_MAX_CHANNELS, OSS_ERR_INVALID, "F must be in [0, 64]");
    OSS_CHECK(total_pairs >= 0 && total_pairs <= INT_MAX, OSS_ERR_RANGE, "total pair count exceeds int32 range");
    OSS_CHECK(scratch_bytes >= oss_rasterize_backward_lists_scratch_bytes(n, total_pairs, g.tiles), OSS_ERR_SCRATCH,
              "rasterize_backward_lists scratch too small");
    if (g.n == 0) return OSS_OK;
    OSS_CHECK(xy != nullptr && aligned(xy, 8) && conic != nullptr, OSS_ERR_INVALID, "xy (8-byte aligned) and conic must be non-null");
    OSS_CHECK(d_xy != nullptr && d_conic != nullptr && (f == 0 || (d_feat != nullptr && feat != nullptr)),
              OSS_ERR_INVALID, "gradient outputs must be non-null");
    OSS_CHECK(scratch != nullptr && aligned(scratch, 16), OSS_ERR_INVALID, "scratch must be 16-byte aligned");
    cudaStream_t s = as_stream(stream);
    OSS_CUDA_TRY(cudaMemsetAsync(d_xy, 0, sizeof(float) * 2 * g.n, s));
    OSS_CUDA_TRY(cudaMemsetAsync(d_conic, 0, sizeof(float) * 3 * g.n, s));
    if (f > 0) OSS_CUDA_TRY(cudaMemsetAsync(d_feat, 0, sizeof(float) * f * g.n, s));
    if (f == 0 || g.tiles == 0 || total_pairs == 0) return OSS_OK;
    OSS_CHECK(gid_sorted != nullptr && tile_offsets != nullptr && grad_image != nullptr, OSS_ERR_INVALID,
              "lists and grad_image must be non-null");
    float* geo = static_cast<float*>(scratch);
    void* items = static_cast<char*>(scratch) + oss::arena_bytes(static_cast<int64_t>(g.n) * 8, 4);
    OSS_CUDA_TRY(oss::launch_make_geo(g.n, xy, conic, geo, s));
    OSS_CUDA_TRY(oss::launch_render_backward_tiles(static_cast<int>(f), g.h, g.w, total_pairs, geo, feat, nullptr,
                                                   gid_sorted, tile_offsets, grad_image, nullptr, nullptr, nullptr,
                                                   nullptr, nullptr, 0, d_xy, d_conic, d_feat, items, s));
    return OSS_OK;
}

int oss_make_geo(int64_t n, const float* xy, const float* conic, float* geo, void* stream) {
    OSS_CHECK(n >= 0 && n <= INT_MAX, OSS_ERR_RANGE, "N exceeds int32 range");
    if (n == 0) return OSS_OK;
    OSS_CHECK(xy != nullptr && aligned(xy, 8) && conic != nullptr && geo != nullptr && aligned(geo, 16),
              OSS_ERR_INVALID, "xy (8-byte aligned), conic and geo (16-byte aligned) must be non-null");
    OSS_CUDA_TRY(oss::launch_make_geo(static_cast<int>(n), xy, conic, geo, as_stream(stream)));
    return OSS_OK;
}

int oss_conic_to_scale_rot_grad(int64_t n, const float* scale, const float* rot, const float* d_conic, float* d_scale,
                                float* d_rot, void* stream) {
    OSS_CHECK(n >= 0, OSS_ERR_INVALID, "N must be non-negative");
    OSS_CHECK(n <= INT_MAX, OSS_ERR_RANGE, "N exceeds int32 range");
    if (n == 0) return OSS_OK;
    OSS_CHECK(scale != nullptr && aligned(scale, 8) && rot != nullptr && d_conic != nullptr && d_scale != nullptr &&
                  aligned(d_scale, 8) && d_rot != nullptr,
              OSS_ERR_INVALID, "pointers must be non-null (scale, d_scale 8-byte aligned)");
    OSS_CUDA_TRY(oss::launch_conic_to_scale_rot_grad(static_cast<int>(n), scale, rot, d_conic, d_scale, d_rot,
                                                     as_stream(stream)));
    return OSS_OK;
}

int oss_full_tile_pairs(int64_t n, int64_t num_tiles, int32_t* gid_sorted, int32_t* tile_offsets, void* stream) {
    OSS_CHECK(n >= 0 && num_tiles >= 0, OSS_ERR_INVALID, "N and num_tiles must be non-negative");
    OSS_CHECK(num_tiles <= INT_MAX, OSS_ERR_RANGE, "number of tiles exceeds int32 range");
    OSS_CHECK(n == 0 || num_tiles <= INT_MAX / n, OSS_ERR_RANGE, "full-frame raster pair count exceeds int32 range");
    OSS_CHECK(tile_offsets != nullptr, OSS_ERR_INVALID, "tile_offsets must be non-null");
    cudaStream_t s = as_stream(stream);
    if (num_tiles == 0) {
        OSS_CUDA_TRY(cudaMemsetAsync(tile_offsets, 0, sizeof(int32_t), s));
        return OSS_OK;
    }
    OSS_CHECK(n == 0 || gid_sorted != nullptr, OSS_ERR_INVALID, "gid_sorted must be non-null");
    OSS_CUDA_TRY(oss::launch_full_tile_pairs(static_cast<int>(n), static_cast<int>(num_tiles), gid_sorted,
                                             tile_offsets, s));
    return OSS_OK;
}

int64_t oss_warp_canvas_scratch_bytes(int64_t n) { return oss::warp_scratch_bytes(n < 0 ? 0 : n); }

int oss_warp_canvas(int64_t n, int64_t f, int64_t h_lr, int64_t w_lr, int64_t h, int64_t w, const float* motion_lr,
                    float alpha, const float* recon, const float* positions, const float* scales,
                    const float* rotations, const float* opacities, const float* colors, float* out_positions,
                    float* out_scales, float* out_rotations, float* out_opacities, float* out_colors,
                    int32_t* out_count, void* scratch, int64_t scratch_bytes, void* stream) {
    OSS_CHECK(n >= 0 && f >= 0, OSS_ERR_INVALID, "canvas.count must be non-negative");
    OSS_CHECK(n <= INT_MAX && f <= INT_MAX / (n > 0 ? n : 1), OSS_ERR_RANGE, "canvas size exceeds int32 range");
    OSS_CHECK(h > 0 && w > 0, OSS_ERR_INVALID, "output_hw must be positive");
    OSS_CHECK(h_lr > 0 && w_lr > 0, OSS_ERR_INVALID, "motion_lr must be (B, 2, H, W) with H, W > 0");
    OSS_CHECK(h <= INT_MAX && w <= INT_MAX && h_lr <= INT_MAX && w_lr <= INT_MAX &&
                  2 * h_lr * w_lr <= (int64_t)1 << 40,
              OSS_ERR_RANGE, "motion or output size exceeds int32 range");
    OSS_CHECK(recon != nullptr, OSS_ERR_INVALID, "recon must point to 4 host floats");
    OSS_CHECK(out_count != nullptr, OSS_ERR_INVALID, "out_count must be non-null");
    OSS_CHECK(scratch_bytes >= oss_warp_canvas_scratch_bytes(n), OSS_ERR_SCRATCH, "warp_canvas scratch too small");
    if (n > 0) {
        OSS_CHECK(motion_lr != nullptr && positions != nullptr && scales != nullptr && rotations != nullptr &&
                      opacities != nullptr && (f == 0 || colors != nullptr),
                  OSS_ERR_INVALID, "canvas inputs must be non-null");
        OSS_CHECK(out_positions != nullptr && out_scales != nullptr && out_rotations != nullptr &&
                      out_opacities != nullptr && (f == 0 || out_colors != nullptr),
                  OSS_ERR_INVALID, "canvas outputs must be non-null");
        OSS_CHECK(aligned(positions, 8) && aligned(scales, 8) && aligned(out_positions, 8) && aligned(out_scales, 8),
                  OSS_ERR_INVALID, "positions and scales must be 8-byte aligned");
        OSS_CHECK(scratch != nullptr && aligned(scratch, 16), OSS_ERR_INVALID, "scratch must be 16-byte aligned");
    }
    OSS_CUDA_TRY(oss::launch_warp_canvas(static_cast<int>(n), static_cast<int>(f), static_cast<int>(h_lr),
                                         static_cast<int>(w_lr), static_cast<int>(h), static_cast<int>(w), motion_lr,
                                         alpha, recon, positions, scales, rotations, opacities, colors, out_positions,
                                         out_scales, out_rotations, out_opacities, out_colors, out_count, scratch,
                                         as_stream(stream)));
    return OSS_OK;
}

int oss_warp_canvas_parked(int64_t n, int64_t f, int64_t h_lr, int64_t w_lr, int64_t h, int64_t w,
                           const float* motion_lr, float alpha, const float* recon, const float* positions,
                           const float* scales, const float* rotations, const float* opacities, const float* colors,
                           float* out_positions, float* out_scales, float* out_rotations, float* out_opacities,
                           float* out_colors, void* scratch, int64_t scratch_bytes, void* stream) {
    OSS_CHECK(n >= 0 && f >= 0, OSS_ERR_INVALID, "canvas.count must be non-negative");
    OSS_CHECK(n <= INT_MAX && f <= INT_MAX / (n > 0 ? n : 1), OSS_ERR_RANGE, "canvas size exceeds int32 range");
    OSS_CHECK(h > 0 && w > 0, OSS_ERR_INVALID, "output_hw must be positive");
    OSS_CHECK(h_lr > 0 && w_lr > 0, OSS_ERR_INVALID, "motion_lr must be (B, 2, H, W) with H, W > 0");
    OSS_CHECK(h <= INT_MAX && w <= INT_MAX && h_lr <= INT_MAX && w_lr <= INT_MAX &&
                  2 * h_lr * w_lr <= (int64_t)1 << 40,
              OSS_ERR_RANGE, "motion or output size exceeds int32 range");
    OSS_CHECK(recon != nullptr, OSS_ERR_INVALID, "recon must point to 4 host floats");
    OSS_CHECK(scratch_bytes >= oss_warp_canvas_scratch_bytes(n), OSS_ERR_SCRATCH, "warp_canvas scratch too small");
    if (n > 0) {
        OSS_CHECK(motion_lr != nullptr && positions != nullptr && scales != nullptr && rotations != nullptr &&
                      opacities != nullptr && (f == 0 || colors != nullptr),
                  OSS_ERR_INVALID, "canvas inputs must be non-null");
        OSS_CHECK(out_positions != nullptr && out_scales != nullptr && out_rotations != nullptr &&
                      out_opacities != nullptr && (f == 0 || out_colors != nullptr),
                  OSS_ERR_INVALID, "canvas outputs must be non-null");
        OSS_CHECK(aligned(positions, 8) && aligned(scales, 8) && aligned(out_positions, 8) && aligned(out_scales, 8),
                  OSS_ERR_INVALID, "positions and scales must be 8-byte aligned");
        OSS_CHECK(scratch != nullptr && aligned(scratch, 16), OSS_ERR_INVALID, "scratch must be 16-byte aligned");
    }
    OSS_CUDA_TRY(oss::launch_warp_canvas_parked(static_cast<int>(n), static_cast<int>(f), static_cast<int>(h_lr),
                                                static_cast<int>(w_lr), static_cast<int>(h), static_cast<int>(w),
                                                motion_lr, alpha, recon, positions, scales, rotations, opacities,
                                                colors, out_positions, out_scales, out_rotations, out_opacities,
                                                out_colors, scratch, as_stream(stream)));
    return OSS_OK;
}

int oss_v6_sanitize(int64_t n, int64_t h, int64_t w, int64_t f_in, int64_t f_out, int32_t ones_channel,
                    const uint8_t* active_mask, const float* positions, const float* scales, const float* rotations,
                    const float* colors, float* out_xy, float* out_scale, float* out_rot, float* out_feat,
                    uint16_t* flags, void* stream) {
    OSS_CHECK(n >= 0 && n <= INT_MAX, OSS_ERR_RANGE, "N must be in [0, 2^31)");
    OSS_CHECK(h > 0 && w > 0 && h <= INT_MAX && w <= INT_MAX, OSS_ERR_INVALID, "output_hw must be positive");
    OSS_CHECK(f_in >= 0 && f_out > 0 && f_out + (ones_channel ? 1 : 0) <= OSS_MAX_CHANNELS, OSS_ERR_INVALID,
              "feature widths out of range");
    if (n == 0) return OSS_OK;
    OSS_CHECK(positions != nullptr && scales != nullptr && rotations != nullptr && (f_in == 0 || colors != nullptr),
              OSS_ERR_INVALID, "canvas inputs must be non-null");
    OSS_CHECK(out_xy != nullptr && out_scale != nullptr && out_rot != nullptr && out_feat != nullptr &&
                  flags != nullptr,
              OSS_ERR_INVALID, "outputs must be non-null");
    OSS_CHECK(aligned(positions, 8) && aligned(scales, 8) && aligned(out_xy, 8) && aligned(out_scale, 8),
              OSS_ERR_INVALID, "positions and scales must be 8-byte aligned");
    OSS_CUDA_TRY(oss::launch_v6_sanitize(static_cast<int>(n), static_cast<int>(h), static_cast<int>(w),
                                         static_cast<int>(f_in), static_cast<int>(f_out), ones_channel ? 1 : 0,
                                         active_mask, positions, scales, rotations, colors, out_xy, out_scale,
                                         out_rot, out_feat, flags, as_stream(stream)));
    return OSS_OK;
}

int oss_v6_sanitize_backward(int64_t n, int64_t f_in, int64_t f_out, int32_t ones_channel, const uint16_t* flags,
                             const float* d_xy, const float* d_scale, const float* d_rot, const float* d_feat,
                             float* d_positions, float* d_scales, float* d_rotations, float* d_colors,
                             void* stream) {
    OSS_CHECK(n >= 0 && n <= INT_MAX, OSS_ERR_RANGE, "N must be in [0, 2^31)");
    OSS_CHECK(f_in >= 0 && f_out > 0 && f_out + (ones_channel ? 1 : 0) <= OSS_MAX_CHANNELS, OSS_ERR_INVALID,
              "feature widths out of range");
    if (n == 0) return OSS_OK;
    OSS_CHECK(flags != nullptr && d_positions != nullptr && d_scales != nullptr && d_rotations != nullptr &&
                  (f_in == 0 || d_colors != nullptr),
              OSS_ERR_INVALID, "flags and gradient outputs must be non-null");
    OSS_CHECK(aligned(d_positions, 8) && aligned(d_scales, 8) && (d_xy == nullptr || aligned(d_xy, 8)) &&
                  (d_scale == nullptr || aligned(d_scale, 8)),
              OSS_ERR_INVALID, "position and scale gradients must be 8-byte aligned");
    OSS_CUDA_TRY(oss::launch_v6_sanitize_backward(static_cast<int>(n), static_cast<int>(f_in), static_cast<int>(f_out),
                                                  ones_channel ? 1 : 0, flags, d_xy, d_scale, d_rot, d_feat,
                                                  d_positions, d_scales, d_rotations, d_colors, as_stream(stream)));
    return OSS_OK;
}

int64_t oss_warp_canvas_backward_scratch_bytes(int64_t h, int64_t w) {
    return oss::warp_backward_scratch_bytes(h < 0 ? 0 : h, w < 0 ? 0 : w);
}

int oss_warp_canvas_backward(int64_t n, int64_t f, int64_t h_lr, int64_t w_lr, int64_t h, int64_t w,
                             const float* motion_lr, float alpha, const float* recon, const float* positions,
                             const float* scales, const float* rotations, const void* forward_scratch,
                             const float* g_positions, const float* g_scales, const float* g_rotations,
                             const float* g_opacities, const float* g_colors, float* d_positions, float* d_scales,
                             float* d_rotations, float* d_opacities, float* d_colors, float* d_motion_lr,
                             void* scratch, int64_t scratch_bytes, void* stream) {
    OSS_CHECK(n >= 0 && f >= 0, OSS_ERR_INVALID, "canvas.count must be non-negative");
    OSS_CHECK(n <= INT_MAX && f <= INT_MAX / (n > 0 ? n : 1), OSS_ERR_RANGE, "canvas size exceeds int32 range");
    OSS_CHECK(h > 0 && w > 0, OSS_ERR_INVALID, "output_hw must be positive");
    OSS_CHECK(h_lr > 0 && w_lr > 0, OSS_ERR_INVALID, "motion_lr must be (B, 2, H, W) with H, W > 0");
    OSS_CHECK(h <= INT_MAX && w <= INT_MAX && h_lr <= INT_MAX && w_lr <= INT_MAX && 6 * h * w <= INT64_MAX / 8,
              OSS_ERR_RANGE, "motion or output size exceeds int32 range");
    OSS_CHECK(recon != nullptr, OSS_ERR_INVALID, "recon must point to 4 host floats");
    OSS_CHECK(scratch_bytes >= oss_warp_canvas_backward_scratch_bytes(h, w), OSS_ERR_SCRATCH,
              "warp_canvas_backward scratch too small");
    OSS_CHECK(scratch != nullptr && aligned(scratch, 16), OSS_ERR_INVALID, "scratch must be 16-byte aligned");
    if (n > 0) {
        OSS_CHECK(motion_lr != nullptr && positions != nullptr && scales != nullptr && rotations != nullptr &&
                      forward_scratch != nullptr,
                  OSS_ERR_INVALID, "canvas inputs and the forward's scratch must be non-null");
        OSS_CHECK(d_positions != nullptr && d_scales != nullptr && d_rotations != nullptr &&
                      (f == 0 || d_colors != nullptr),
                  OSS_ERR_INVALID, "gradient outputs must be non-null");
        OSS_CHECK(aligned(positions, 8) && aligned(scales, 8) && aligned(d_positions, 8) && aligned(d_scales, 8) &&
                      (g_positions == nullptr || aligned(g_positions, 8)) &&
                      (g_scales == nullptr || aligned(g_scales, 8)) && aligned(forward_scratch, 16),
                  OSS_ERR_INVALID, "positions, scales, their gradients and the forward scratch must be aligned");
    }
    OSS_CUDA_TRY(oss::launch_warp_canvas_backward(
        static_cast<int>(n), static_cast<int>(f), static_cast<int>(h_lr), static_cast<int>(w_lr), static_cast<int>(h),
        static_cast<int>(w), motion_lr, alpha, recon, positions, scales, rotations, forward_scratch, g_positions,
        g_scales, g_rotations, g_opacities, g_colors, d_positions, d_scales, d_rotations, d_opacities, d_colors,
        d_motion_lr, scratch, as_stream(stream)));
    return OSS_OK;
}

int oss_warp_positions(int64_t n, int64_t h, int64_t w, const float* motion, float alpha, const float* xy,
                       float* out_xy, uint8_t* in_frame, void* stream) {
    OSS_CHECK(n >= 0, OSS_ERR_INVALID, "N must be non-negative");
    OSS_CHECK(n <= INT_MAX, OSS_ERR_RANGE, "N exceeds int32 range");
    OSS_CHECK(h > 0 && w > 0 && h <= INT_MAX && w <= INT_MAX, OSS_ERR_INVALID, "hw must be positive");
    if (n == 0) return OSS_OK;
    OSS_CHECK(motion != nullptr && xy != nullptr && out_xy != nullptr && in_frame != nullptr, OSS_ERR_INVALID,
              "pointers must be non-null");
    OSS_CHECK(aligned(xy, 8) && aligned(out_xy, 8), OSS_ERR_INVALID, "xy must be 8-byte aligned");
    OSS_CUDA_TRY(oss::launch_warp_positions(static_cast<int>(n), static_cast<int>(h), static_cast<int>(w), motion,
                                            alpha, xy, out_xy, in_frame, as_stream(stream)));
    return OSS_OK;
}

int oss_analytic_pixel_integral(int64_t n, const float* dx, const float* dy, const float* s00, const float* s01,
                                const float* s10, const float* s11, float* out, void* stream) {
    OSS_CHECK(n >= 0, OSS_ERR_INVALID, "n must be non-negative");
    if (n == 0) return OSS_OK;
    OSS_CHECK(dx != nullptr && dy != nullptr && s00 != nullptr && s01 != nullptr && s10 != nullptr &&
                  s11 != nullptr && out != nullptr,
              OSS_ERR_INVALID, "pointers must be non-null");
    OSS_CUDA_TRY(oss::launch_analytic_forward(n, dx, dy, s00, s01, s10, s11, out, as_stream(stream)));
    return OSS_OK;
}

int oss_analytic_pixel_integral_backward(int64_t n, const float* dx, const float* dy, const float* s00,
                                         const float* s01, const float* s10, const float* s11, const float* g,
                                         float* g_dx, float* g_dy, float* g_s00, float* g_s01, float* g_s10,
                                         float* g_s11, void* stream) {
    OSS_CHECK(n >= 0, OSS_ERR_INVALID, "n must be non-negative");
    if (n == 0) return OSS_OK;
    OSS_CHECK(dx != nullptr && dy != nullptr && s00 != nullptr && s01 != nullptr && s10 != nullptr &&
                  s11 != nullptr && g != nullptr && g_dx != nullptr && g_dy != nullptr && g_s00 != nullptr &&
                  g_s01 != nullptr && g_s10 != nullptr && g_s11 != nullptr,
              OSS_ERR_INVALID, "pointers must be non-null");
    OSS_CUDA_TRY(oss::launch_analytic_backward(n, dx, dy, s00, s01, s10, s11, g, g_dx, g_dy, g_s00, g_s01, g_s10,
                                               g_s11, as_stream(stream)));
    return OSS_OK;
}

int oss_logistic_cdf(int64_t n, const float* x, const float* g, float* out, void* stream) {
    OSS_CHECK(n >= 0, OSS_ERR_INVALID, "n must be non-negative");
    if (n == 0) return OSS_OK;
    OSS_CHECK(x != nullptr && out != nullptr, OSS_ERR_INVALID, "x and out must be non-null");
    OSS_CUDA_TRY(oss::launch_logistic_cdf(n, x, g, out, as_stream(stream)));
    return OSS_OK;
}

int oss_render_analytic_forward(int64_t n, int64_t f, int64_t h, int64_t w, const float* geo, const float* feat,
                                const float* opacity, const int32_t* gid_sorted, const int32_t* tile_offsets,
                                float* image, void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    OSS_CHECK(f >= 1 && f <= 32, OSS_ERR_INVALID, "F must be in [1, 32]");
    if (g.tiles == 0) return OSS_OK;
    OSS_CHECK(tile_offsets != nullptr && image != nullptr, OSS_ERR_INVALID, "tile_offsets and image must be non-null");
    OSS_CHECK(g.n == 0 || (geo != nullptr && aligned(geo, 16) && feat != nullptr && gid_sorted != nullptr),
              OSS_ERR_INVALID, "geo (16-byte aligned), feat and gid_sorted must be non-null");
    OSS_CUDA_TRY(oss::launch_render_analytic_forward(static_cast<int>(f), g.h, g.w, geo, feat, opacity, gid_sorted,
                                                     tile_offsets, image, as_stream(stream)));
    return OSS_OK;
}

int64_t oss_render_analytic_backward_scratch_bytes(int64_t total_pairs, int64_t f) {
    if (total_pairs < 0) total_pairs = 0;
    return oss::arena_bytes(total_pairs, sizeof(float) * oss::backward_pair_stride(static_cast<int>(f < 1 ? 1 : f)));
}

int oss_render_analytic_backward(int64_t n, int64_t f, int64_t h, int64_t w, const float* geo, const float* feat,
                                 const float* opacity, const float* scale, const float* rot, const int32_t* aabb,
                                 const int32_t* pair_offset, int64_t total_pairs, const int32_t* gid_sorted,
                                 const int32_t* tile_offsets, const float* grad_image, float* d_xy, float* d_conic,
                                 float* d_feat, float* d_opacity, float* d_scale, float* d_rot, void* scratch,
                                 int64_t scratch_bytes, void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    OSS_CHECK(f >= 1 && f <= 32, OSS_ERR_INVALID, "F must be in [1, 32]");
    OSS_CHECK(total_pairs >= 0 && total_pairs <= INT_MAX, OSS_ERR_RANGE, "total pair count exceeds int32 range");
    OSS_CHECK(scratch_bytes >= oss_render_analytic_backward_scratch_bytes(total_pairs, f), OSS_ERR_SCRATCH,
              "render_analytic_backward scratch too small");
    if (g.n == 0) return OSS_OK;
    OSS_CHECK(geo != nullptr && aligned(geo, 16) && feat != nullptr && aabb != nullptr && aligned(aabb, 16) &&
                  pair_offset != nullptr && tile_offsets != nullptr && grad_image != nullptr && d_xy != nullptr &&
                  d_conic != nullptr && d_feat != nullptr && (total_pairs == 0 || gid_sorted != nullptr),
              OSS_ERR_INVALID, "pointers must be non-null (geo and aabb 16-byte aligned)");
    OSS_CHECK(d_scale == nullptr || (scale != nullptr && rot != nullptr && d_rot != nullptr), OSS_ERR_INVALID,
              "d_scale needs scale, rot and d_rot");
    cudaStream_t s = as_stream(stream);
    float* pairgrad = static_cast<float*>(scratch);
    const int stride = oss::backward_pair_stride(static_cast<int>(f));
    if (total_pairs > 0 && g.tiles > 0) {
        OSS_CUDA_TRY(oss::launch_render_analytic_backward_pairs(static_cast<int>(f), g.h, g.w, geo, feat, opacity,
                                                                gid_sorted, tile_offsets, aabb, pair_offset, grad_image,
                                                                pairgrad, stride, s));
    }
    OSS_CUDA_TRY(oss::launch_reduce_gaussian_grads(g.n, static_cast<int>(f), pairgrad, stride, pair_offset, geo, feat,
                                                   opacity, scale, rot, d_xy, d_conic, d_feat, d_opacity, d_scale,
                                                   d_rot, s, true));
    return OSS_OK;
}

int64_t oss_nd_record_floats(int64_t f) { return f < 1 || f > 32 ? 0 : oss::nd_record_floats(static_cast<int>(f)); }

int oss_nd_condition(int64_t n, int64_t h, int64_t w, const float* means, const float* covs, const float* opac,
                     float t_query, int32_t time_falloff, float mip3, float mip2, float* xy, float* conic, float* amp,
                     int32_t* box, void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    if (g.n == 0) return OSS_OK;
    OSS_CHECK(means != nullptr && covs != nullptr && opac != nullptr && xy != nullptr && conic != nullptr &&
                  amp != nullptr && box != nullptr && aligned(box, 16),
              OSS_ERR_INVALID, "pointers must be non-null (box 16-byte aligned)");
    OSS_CUDA_TRY(oss::launch_nd_prep_forward(g.n, g.h, g.w, means, covs, opac, t_query, time_falloff, mip3, mip2, xy,
                                             conic, amp, box, as_stream(stream)));
    return OSS_OK;
}

int oss_nd_condition_backward(int64_t n, const float* means, const float* covs, const float* opac, float t_query,
                              int32_t time_falloff, float mip3, float mip2, const float* d_xy, const float* d_conic,
                              const float* d_amp, float* d_means, float* d_covs, float* d_opac, void* stream) {
    OSS_CHECK(n >= 0 && n <= INT_MAX, OSS_ERR_RANGE, "N must be in [0, INT_MAX]");
    if (n == 0) return OSS_OK;
    OSS_CHECK(means != nullptr && covs != nullptr && opac != nullptr && d_xy != nullptr && d_conic != nullptr &&
                  d_amp != nullptr && d_means != nullptr && d_covs != nullptr && d_opac != nullptr,
              OSS_ERR_INVALID, "pointers must be non-null");
    OSS_CUDA_TRY(oss::launch_nd_prep_backward(static_cast<int>(n), means, covs, opac, t_query, time_falloff, mip3, mip2,
                                              d_xy, d_conic, d_amp, d_means, d_covs, d_opac, as_stream(stream)));
    return OSS_OK;
}

int oss_nd_prepare(int64_t n, int64_t h, int64_t w, const float* xy, const float* conic, const int32_t* box,
                   int64_t f, const float* feat, const float* amp, int32_t* aabb, int32_t* pair_offset, float* geo,
                   float* prec, int64_t* total_pairs, int32_t* tile_count, int32_t* tile_offsets, void* scratch,
                   int64_t scratch_bytes, void* stream) {
    Grid g;
    int rc = check_grid(n, h, w, g);
    if (rc != OSS_OK) return rc;
    OSS_CHECK(f >= 1 && f <= 32, OSS_ERR_INVALID, "F must be in [1, 32]");
    OSS_CHECK(pair_offset != nullptr && total_pairs != nullptr, OSS_ERR_INVALID,
              "pair_offset and total_pairs must be non-null");
    OSS_CHECK(g.tiles == 0 || (tile_count != nullptr && tile_offsets != nullptr), OSS_ERR_INVALID,
              "tile_count and tile_offsets must be non-null");
    OSS_CHECK(scratch_bytes >= oss_render_prepare_scratch_bytes(n), OSS_ERR_SCRATCH, "nd_prepare scratch too small");
    if (g.n > 0) {
        OSS_CHECK(xy != nullptr && conic != nullptr && box != nullptr && feat != nullptr && amp != nullptr &&
                      aabb != nullptr && geo != nullptr && prec != nullptr,
                  OSS_ERR_INVALID, "inputs and outputs must be non-null");
        OSS_CHECK(aligned(xy, 8) && aligned(box, 16) && aligned(aabb, 16) && aligned(geo, 16) && aligned(prec, 16),
                  OSS_ERR_INVALID, "xy (8), box, aabb, geo and prec (16) must be aligned");
    }
    cudaStream_t s = as_stream(stream);
    long long* block_sums = static_cast<long long*>(scratch);
    OSS_CHECK(g.n == 0 || (block_sums != nullptr && aligned(block_sums, 8)), OSS_ERR_INVALID,
              "scratch must be 8-byte aligned");
    int32_t* counts = g.tiles > 0 ? tile_count : nullptr;
    if (counts != nullptr) {
        OSS_CUDA_TRY(cudaMemsetAsync(counts, 0, sizeof(int32_t) * oss_tile_count_elems(g.tiles), s));
    }
    if (g.n > 0) {
        OSS_CUDA_TRY(oss::launch_nd_preprocess(g.n, g.ntx, g.nty, xy, conic, box, static_cast<int>(f), feat, amp,
                                               aabb, pair_offset, geo, prec, block_sums, counts, s));
    }
    OSS_CUDA_TRY(oss::scan_apply_with_block_sums(pair_offset, pair_offset, g.n, block_sums, total_pairs, counts,
                                                 oss::kTileCountStride, g.tiles, counts != nullptr ? tile_offsets : nullptr,
                                                 s));
    return OSS_OK;
}

int oss_nd_forward(int64_t f, int64_t h, int64_t w, const float* prec, const int32_t* box, const int32_t* gid_sorted,
                   const int32_t* tile_offsets, float* image, void* stream) {
    Grid g;
    int rc = check_grid(0, h, w, g);
    if (rc != OSS_OK) return rc;
    OSS_CHECK(f >= 1 && f <= 32, OSS_ERR_INVALID, "F must be in [1, 32]");
    if (g.tiles == 0) return OSS_OK;
    OSS_CHECK(prec != nullptr && box != nullptr && gid_sorted != nullptr && tile_offsets != nullptr &&
                  image != nullptr && aligned(prec, 16) && aligned(box, 16),
              OSS_ERR_INVALID, "pointers must be non-null (prec and box 16-byte aligned)");
    OSS_CUDA_TRY(oss::launch_nd_forward(static_cast<int>(f), g.h, g.w, prec, box, gid_sorted, tile_offsets, image,
                                        as_stream(stream)));
    return OSS_OK;
}

int oss_nd_backward_pairs(int64_t f, int64_t h, int64_t w, const float* prec, const int32_t* box,
                          const int32_t* gid_sorted, const int32_t* tile_offsets, const int32_t* aabb,
                          const int32_t* pair_offset, const float* grad_image, float* pairgrad, void* stream) {
    Grid g;
    int rc = check_grid(0, h, w, g);
    if (rc != OSS_OK) return rc;
    OSS_CHECK(f >= 1 && f <= 32, OSS_ERR_INVALID, "F must be in [1, 32]");
    if (g.tiles == 0) return OSS_OK;
    OSS_CHECK(prec != nullptr && box != nullptr && gid_sorted != nullptr && tile_offsets != nullptr && aabb != nullptr &&
                  pair_offset != nullptr && grad_image != nullptr && pairgrad != nullptr && aligned(prec, 16) &&
                  aligned(box, 16) && aligned(aabb, 16),
              OSS_ERR_INVALID, "pointers must be non-null (prec, box and aabb 16-byte aligned)");
    OSS_CUDA_TRY(oss::launch_nd_backward_pairs(static_cast<int>(f), g.h, g.w, prec, box, gid_sorted, tile_offsets,
                                               aabb, pair_offset, grad_image, pairgrad,
                                               oss::backward_pair_stride(static_cast<int>(f)), as_stream(stream)));
    return OSS_OK;
}

int oss_tile_mse(int64_t f, int64_t h, int64_t w, int64_t ts, const float* rendered, int64_t target_h,
                 int64_t target_w, const float* target, float* tile_err, void* stream) {
    OSS_CHECK(f > 0 && f <= INT_MAX, OSS_ERR_INVALID, "F must be positive");
    OSS_CHECK(ts > 0 && ts <= 1024, OSS_ERR_INVALID, "tile_size must be in [1, 1024]");
    OSS_CHECK(h > 0 && w > 0 && h <= INT_MAX && w <= INT_MAX, OSS_ERR_INVALID, "H and W must be positive");
    OSS_CHECK(h % ts == 0 && w % ts == 0, OSS_ERR_INVALID, "H and W must both be multiples of tile_size");
    OSS_CHECK(target_h > 0 && target_w > 0 && target_h <= INT_MAX && target_w <= INT_MAX, OSS_ERR_INVALID,
              "target H and W must be positive");
    OSS_CHECK(f * h * w <= INT64_MAX / 4, OSS_ERR_RANGE, "rendered is too large");
    OSS_CHECK(rendered != nullptr && target != nullptr && tile_err != nullptr, OSS_ERR_INVALID,
              "pointers must be non-null");
    OSS_CUDA_TRY(oss::launch_tile_mse(static_cast<int>(f), static_cast<int>(h), static_cast<int>(w),
                                      static_cast<int>(ts), rendered, static_cast<int>(target_h),
                                      static_cast<int>(target_w), target, tile_err, as_stream(stream)));
    return OSS_OK;
}

int oss_canvas_error(int64_t n, int64_t h, int64_t w, int64_t ts, const float* xy, const uint8_t* in_frame,
                     const float* tile_err, const uint8_t* alive, int64_t* age, float* g_error, float* error,
                     void* stream) {
    OSS_CHECK(n >= 0 && n <= INT_MAX, OSS_ERR_RANGE, "N must be in [0, INT_MAX]");
    OSS_CHECK(ts > 0 && ts <= 1024, OSS_ERR_INVALID, "tile_size must be in [1, 1024]");
    OSS_CHECK(h > 0 && w > 0 && h <= INT_MAX && w <= INT_MAX, OSS_ERR_INVALID, "H and W must be positive");
    OSS_CHECK(h % ts == 0 && w % ts == 0, OSS_ERR_INVALID, "H and W must both be multiples of tile_size");
    if (n == 0) return OSS_OK;
    OSS_CHECK(xy != nullptr && tile_err != nullptr && aligned(xy, 8), OSS_ERR_INVALID,
              "xy (8-byte aligned) and tile_err must be non-null");
    OSS_CUDA_TRY(oss::launch_canvas_error(static_cast<int>(n), static_cast<int>(h), static_cast<int>(w),
                                          static_cast<int>(ts), xy, in_frame, tile_err, alive, age, g_error, error,
                                          as_stream(stream)));
    return OSS_OK;
}

int64_t oss_prune_scratch_bytes(int64_t n) { return oss::prune_scratch_bytes(n < 0 ? 0 : n); }

int oss_select_for_pruning(int64_t n, const uint8_t* alive, const uint8_t* in_frame, const int64_t* age,
                           const float* g_error, int64_t capacity, int64_t age_max, double age_low_error_pct,
                           double tile_error_pct, int64_t min_age_before_prune, double max_prune_frac,
                           int64_t* prune_idx, int64_t* prune_count, float* quantiles, void* scratch,
                           int64_t scratch_bytes, void* stream) {
    OSS_CHECK(n >= 0 && n < INT_MAX, OSS_ERR_RANGE, "N must be in [0, INT_MAX)");
    OSS_CHECK(prune_count != nullptr && quantiles != nullptr && scratch != nullptr, OSS_ERR_INVALID,
              "prune_count, quantiles and scratch must be non-null");
    OSS_CHECK(scratch_bytes >= oss::prune_scratch_bytes(n), OSS_ERR_SCRATCH, "scratch too small");
    OSS_CHECK(n == 0 || (alive != nullptr && in_frame != nullptr && age != nullptr && g_error != nullptr &&
                         prune_idx != nullptr),
              OSS_ERR_INVALID, "alive, in_frame, age, g_error and prune_idx must be non-null");
    // max(1, int(frac * capacity)) in double, as the policy's Python arithmetic
    const double prod = max_prune_frac * static_cast<double>(capacity);
    long long cap = prod >= 9.0e18 ? static_cast<long long>(9e18) : static_cast<long long>(prod);
    if (cap < 1) cap = 1;
    OSS_CUDA_TRY(oss::launch_select_for_pruning(static_cast<int>(n), alive, in_frame, age, g_error, cap, age_max,
                                                static_cast<float>(age_low_error_pct),
                                                static_cast<float>(tile_error_pct), min_age_before_prune, prune_idx,
                                                prune_count, quantiles, scratch, as_stream(stream)));
    return OSS_OK;
}

int64_t oss_spawn_tiles_scratch_bytes(int64_t num_tiles) {
    return oss::spawn_tiles_scratch_bytes(num_tiles < 0 ? 0 : num_tiles);
}

int oss_select_spawn_tiles(int64_t th, int64_t tw, const float* tile_err, const uint8_t* classifier_mask,
                           int64_t n_tiles, int64_t* tiles_yx, int64_t* take, void* scratch, int64_t scratch_bytes,
                           void* stream) {
    OSS_CHECK(th >= 0 && tw >= 0 && th * tw <= INT_MAX, OSS_ERR_RANGE, "tile grid must be in int32 range");
    OSS_CHECK(take != nullptr && scratch != nullptr, OSS_ERR_INVALID, "take and scratch must be non-null");
    OSS_CHECK(scratch_bytes >= oss::spawn_tiles_scratch_bytes(th * tw), OSS_ERR_SCRATCH, "scratch too small");
    OSS_CHECK(th * tw == 0 || (tile_err != nullptr && tiles_yx != nullptr), OSS_ERR_INVALID,
              "tile_err and tiles_yx must be non-null");
    OSS_CUDA_TRY(oss::launch_select_spawn_tiles(static_cast<int>(th), static_cast<int>(tw), tile_err,
                                                classifier_mask, n_tiles, tiles_yx, take, scratch,
                                                as_stream(stream)));
    return OSS_OK;
}

int64_t oss_prune_spawn_scratch_bytes(int64_t n) { return oss::prune_spawn_scratch_bytes(n < 0 ? 0 : n); }

int oss_apply_prune_spawn(int64_t n, int64_t f, const int64_t* prune_idx, const int64_t* prune_count,
                          int64_t max_prune, int64_t num_new, int64_t f_new, const float* new_xy,
                          const float* new_scale, const float* new_rot, const float* new_feat, float* positions,
                          float* scales, float* rotations, float* colors, uint8_t* alive, int64_t* age,
                          float* error, int64_t* n_spawned, void* scratch, int64_t scratch_bytes, void* stream) {
    OSS_CHECK(n >= 0 && n < INT_MAX, OSS_ERR_RANGE, "N must be in [0, INT_MAX)");
    OSS_CHECK(f > 0 && f <= INT_MAX && f_new >= 0 && f_new <= INT_MAX, OSS_ERR_INVALID,
              "F must be positive and F_new non-negative");
    OSS_CHECK(num_new >= 0 && num_new <= INT_MAX && max_prune >= 0, OSS_ERR_INVALID,
              "num_new and max_prune must be non-negative");
    OSS_CHECK(n_spawned != nullptr && scratch != nullptr, OSS_ERR_INVALID, "n_spawned and scratch must be non-null");
    OSS_CHECK(scratch_bytes >= oss::prune_spawn_scratch_bytes(n), OSS_ERR_SCRATCH, "scratch too small");
    OSS_CHECK(max_prune == 0 || (prune_idx != nullptr && prune_count != nullptr), OSS_ERR_INVALID,
              "prune_idx and prune_count must be non-null");
    OSS_CHECK(n == 0 || (positions != nullptr && scales != nullptr && rotations != nullptr && colors != nullptr &&
                         alive != nullptr && age != nullptr && error != nullptr),
              OSS_ERR_INVALID, "canvas arrays must be non-null");
    OSS_CHECK(num_new == 0 || (new_xy != nullptr && new_scale != nullptr && new_rot != nullptr &&
                               (f_new == 0 || new_feat != nullptr)),
              OSS_ERR_INVALID, "new Gaussian arrays must be non-null");
    OSS_CUDA_TRY(oss::launch_apply_prune_spawn(static_cast<int>(n), static_cast<int>(f), prune_idx, prune_count,
                                               max_prune, static_cast<int>(num_new), static_cast<int>(f_new), new_xy,
                                               new_scale, new_rot, new_feat, positions, scales, rotations, colors,
                                               alive, age, error, n_spawned, scratch, as_stream(stream)));
    return OSS_OK;
}

int64_t oss_tile_bin_counting_sort_scratch_bytes(int64_t n, int64_t num_tiles) {
    if (n < 0) n = 0;
    if (num_tiles < 0) num_tiles = 0;
    const uint32_t key_limit = static_cast<uint32_t>(num_tiles > INT_MAX ? INT_MAX : num_tiles);
    return oss::arena_bytes(n, 4) * 2 + oss::arena_bytes(num_tiles, 4) + oss::scan_scratch_bytes(num_tiles) +
           oss::radix_scratch_bytes(n, key_limit);
}

int oss_tile_bin_counting_sort(int64_t n, int64_t num_tiles, const int32_t* tile_id, const int32_t* gid,
                               int32_t* sorted_gid, int32_t* tile_offsets, void* scratch, int64_t scratch_bytes,
                               void* stream) {
    OSS_CHECK(num_tiles > 0, OSS_ERR_INVALID, "num_tiles must be positive");
    OSS_CHECK(num_tiles <= INT_MAX, OSS_ERR_RANGE, "num_tiles exceeds int32 range");
    OSS_CHECK(n >= 0, OSS_ERR_INVALID, "N must be non-negative");
    OSS_CHECK(n <= INT_MAX, OSS_ERR_RANGE, "N exceeds int32 range");
    OSS_CHECK(tile_offsets != nullptr, OSS_ERR_INVALID, "tile_offsets must be non-null");
    OSS_CHECK(n == 0 || (tile_id != nullptr && gid != nullptr && sorted_gid != nullptr), OSS_ERR_INVALID,
              "tile_id, gid and sorted_gid must be non-null");
    OSS_CHECK(scratch_bytes >= oss_tile_bin_counting_sort_scratch_bytes(n, num_tiles), OSS_ERR_SCRATCH,
              "tile_bin_counting_sort scratch too small");
    const int tiles = static_cast<int>(num_tiles);
    cudaStream_t s = as_stream(stream);
    oss::Arena arena{static_cast<char*>(scratch), scratch_bytes, 0};
    uint32_t* keys = arena.take<uint32_t>(n);
    int32_t* vals = arena.take<int32_t>(n);
    int32_t* tile_count = arena.take<int32_t>(tiles);
    void* scan_scratch = arena.base + arena.used;
    arena.used += oss::scan_scratch_bytes(tiles);
    void* radix_scratch = arena.base + arena.used;
    OSS_CUDA_TRY(cudaMemsetAsync(tile_count, 0, sizeof(int32_t) * tiles, s));
    OSS_CUDA_TRY(oss::launch_tile_keys(static_cast<int>(n), tiles, tile_id, gid, keys, vals, tile_count, s));
    OSS_CUDA_TRY(oss::scan_exclusive_i32(tile_count, tile_offsets, tiles, false, nullptr, scan_scratch, s));
    OSS_CUDA_TRY(oss::launch_set_i32(tile_offsets + tiles, static_cast<int32_t>(n), s));
    OSS_CUDA_TRY(oss::radix_sort_pairs(keys, vals, n, static_cast<uint32_t>(tiles), sorted_gid, radix_scratch, s));
    return OSS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free tile binning.
//
// Some callers cannot call cudaMalloc: a hook that runs inside a host
// application's per-frame loop (a game or capture plugin with a fixed device
// memory budget, where the allocator's implicit device synchronisation would
// stall the frame), or an embedding host that owns every device allocation
// itself.  They still need tile binning, whose counting sort wants scratch
// memory (key/value ping-pong buffers, per-tile counts, digit histograms).
// oss_tile_bin_counting_sort_noalloc takes that scratch from the fixed array
// below, which is part of the library's device image: every GPU that loads
// the library holds these 5 MiB until the process exits, and nothing is
// allocated per call.  The caller still passes inputs and outputs.
namespace {

constexpr int64_t kNoAllocMaxN = 262144;       // entries per call
constexpr int64_t kNoAllocMaxTiles = 65536;    // tiles per call
constexpr int64_t kNoAllocScratchBytes = 5242880;  // 5 MiB >= scratch need at both maxima (4.51 MiB)

static __device__ __align__(256) unsigned char g_tile_bin_scratch[kNoAllocScratchBytes];

// Device address of g_tile_bin_scratch in the calling thread's current
// context.  In host code the array's name only stands in for the symbol, so
// its address has to be looked up with the device current.  The lookup runs
// on every call rather than once per device index: a cached address would go
// stale after cudaDeviceReset, or when an embedding host makes a context of
// its own current, and a kernel handed that address faults.  Once the
// library's device code is loaded in a context the lookup is a table read;
// the first call in a context loads that code (the set-up step).
int noalloc_scratch(void** out) {
    void* p = nullptr;
    OSS_CUDA_TRY(cudaGetSymbolAddress(&p, g_tile_bin_scratch));
    OSS_CHECK(p != nullptr, OSS_ERR_CUDA, "cudaGetSymbolAddress returned no address for the no-alloc scratch");
    *out = p;
    return OSS_OK;
}

}  // namespace

extern "C" int oss_tile_bin_counting_sort_noalloc(int64_t n, int64_t num_tiles, const int32_t* tile_id,
                                                  const int32_t* gid, int32_t* sorted_gid, int32_t* tile_offsets,
                                                  void* stream) {
    OSS_CHECK(n >= 0, OSS_ERR_INVALID, "N must be non-negative");
    OSS_CHECK(num_tiles > 0, OSS_ERR_INVALID, "num_tiles must be positive");
    OSS_CHECK(n <= kNoAllocMaxN, OSS_ERR_RANGE,
              "N exceeds the no-alloc maximum of 262144 entries; use oss_tile_bin_counting_sort with caller scratch");
    OSS_CHECK(num_tiles <= kNoAllocMaxTiles, OSS_ERR_RANGE,
              "num_tiles exceeds the no-alloc maximum of 65536; use oss_tile_bin_counting_sort with caller scratch");
    OSS_CHECK(oss_tile_bin_counting_sort_scratch_bytes(n, num_tiles) <= kNoAllocScratchBytes, OSS_ERR_RANGE,
              "scratch need exceeds the no-alloc array");
    void* scratch = nullptr;
    const int rc = noalloc_scratch(&scratch);
    if (rc != OSS_OK) return rc;
    return oss_tile_bin_counting_sort(n, num_tiles, tile_id, gid, sorted_gid, tile_offsets, scratch,
                                      kNoAllocScratchBytes, stream);
}
