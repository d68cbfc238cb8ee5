// Host-side launchers shared between the kernel translation units and the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace oss {

// Scratch carving: 256-byte aligned sub-buffers of one caller buffer.
struct Arena {
    char* base;
    int64_t size;
    int64_t used;
    template <typename T>
    T* take(int64_t count) {
        const int64_t bytes = ((count * static_cast<int64_t>(sizeof(T)) + 255) / 256) * 256;
        T* p = reinterpret_cast<T*>(base + used);
        used += bytes;
        return p;
    }
};

inline int64_t arena_bytes(int64_t count, int64_t elem) { return ((count * elem + 255) / 256) * 256; }

// ---- scan.cu ---------------------------------------------------------------
// Exclusive scan of n int32 values (in may alias out).  The int64 total goes to
// total_out (device, may be null); out[n] = (int32)total if write_tail.
int64_t scan_scratch_bytes(int64_t n);
cudaError_t scan_exclusive_i32(const int32_t* in, int32_t* out, int64_t n, bool write_tail,
                               int64_t* total_out, void* scratch, cudaStream_t stream);

// Preprocess tiling shared with the fused pair-count scan: each preprocess CTA
// handles kPrepTile Gaussians and writes their count sum to block_sums.  The
// preprocess runs one Gaussian per thread (kPreprocThreads = kPrepTile: its
// per-thread chain of loads, double cos/sin, divisions and counter reductions
// is latency-bound, so it wants every Gaussian in flight at once); the scan
// apply runs kPrepThreads threads of kPrepTile / kPrepThreads values.
constexpr int kPrepThreads = 256;
constexpr int kPrepTile = 1024;
constexpr int kPreprocThreads = kPrepTile;
int64_t scan_fused_scratch_bytes(int64_t n);
// Second half of the fused scan: out[0..n) = exclusive scan, out[n] = total.
// With tile_count non-null the same launch also scans the per-tile pair counts
// (spaced count_stride ints apart) into tile_offsets[0..num_tiles].
cudaError_t scan_apply_with_block_sums(const int32_t* in, int32_t* out, int64_t n, const long long* block_sums,
                                       int64_t* total_out, const int32_t* tile_count, int count_stride,
                                       int64_t num_tiles, int32_t* tile_offsets, cudaStream_t stream);

// Per-tile pair counters are spaced one 128-byte line apart: the preprocess and
// scatter atomics then spread over num_tiles lines instead of num_tiles / 32.
constexpr int kTileCountStride = 32;

// ---- radix.cu --------------------------------------------------------------
// Stable LSD sort of (key, val) pairs by key in [0, key_limit].  The sorted vals
// land in vals_out; keys are not kept.  key scratch is consumed.
int64_t radix_scratch_bytes(int64_t n, uint32_t key_limit);
cudaError_t radix_sort_pairs(uint32_t* keys, int32_t* vals, int64_t n, uint32_t key_limit,
                             int32_t* vals_out, void* scratch, cudaStream_t stream);

// ---- preprocess.cu ---------------------------------------------------------
// With prec non-null also the packed forward records (entry_record_floats(f)
// floats per Gaussian: x, y, A, B, D, feat * opacity, zero padding).
cudaError_t launch_preprocess(int n, int ntx, int nty, int mode, const float* xy, const float* scale,
                              const float* rot, float* conic, int32_t* aabb, int32_t* count,
                              float* geo, long long* block_sums, int32_t* tile_count, int f, const float* feat,
                              const float* opacity, float* prec, cudaStream_t stream);
// frames > 1: Gaussians [frame_offsets[b], frame_offsets[b+1]) are frame b's,
// binned into tile rows [b nty, (b+1) nty) of `frames` stacked frames (aabb
// rows are in that stacked grid; nty is one frame's tile rows).
cudaError_t launch_preprocess_frames(int n, int ntx, int nty, int frames, const int32_t* frame_offsets, int mode,
                                     const float* xy, const float* scale, const float* rot, float* conic,
                                     int32_t* aabb, int32_t* count, float* geo, long long* block_sums,
                                     int32_t* tile_count, int f, const float* feat, const float* opacity,
                                     float* prec, cudaStream_t stream);
cudaError_t launch_make_geo(int n, const float* xy, const float* conic, float* geo, cudaStream_t stream);
cudaError_t launch_conic_to_scale_rot_grad(int n, const float* scale, const float* rot,
                                           const float* d_conic, float* d_scale, float* d_rot,
                                           cudaStream_t stream);

// ---- binning.cu ------------------------------------------------------------
cudaError_t launch_full_tile_pairs(int n, int num_tiles, int32_t* gid_sorted, int32_t* tile_offsets,
                                   cudaStream_t stream);
cudaError_t launch_tile_keys(int n, int num_tiles, const int32_t* tile_id, const int32_t* gid,
                             uint32_t* keys, int32_t* vals, int32_t* tile_count, cudaStream_t stream);
cudaError_t launch_set_i32(int32_t* p, int32_t value, cudaStream_t stream);
// One-thread copy of an int64 (dst may be mapped pinned host memory).
cudaError_t launch_copy_i64(const int64_t* src, int64_t* dst, cudaStream_t stream);

// ---- tile_lists.cu --------------------------------------------------------
// Per-tile lists from the tile counts and offsets of render prepare (the
// counts are consumed): atomic scatter, then a per-tile sort.  The pair total
// is read from *total_pairs on the device; above capacity every list and pair
// range is emptied and *overflow = 1.
// With sort_key (a permutation of [0, n)) the lists are ordered by key and
// mapped back to gids through key_order (key -> gid).
int64_t tile_lists_scratch_bytes(int64_t capacity);
cudaError_t build_tile_lists(int n, int ntx, int num_tiles, const int32_t* aabb, int32_t* pair_offset,
                             int32_t* tile_count, const int64_t* total_pairs, int64_t capacity,
                             const int32_t* sort_key, const int32_t* key_order, int32_t* gid_sorted,
                             int32_t* tile_offsets, int32_t* overflow, void* scratch, cudaStream_t stream);
// Stable order of the Gaussians by depth (ties by gid): order[i] = gid of rank i,
// rank[gid] = its position.
int64_t depth_order_scratch_bytes(int64_t n);
cudaError_t depth_order(int n, const float* depth, int32_t* order, int32_t* rank, void* scratch,
                        cudaStream_t stream);

// ---- canvas_life.cu -----------------------------------------------------------
// Persistent-canvas lifecycle: tile error against the (upsampled) LR frame,
// per-slot error and age, the prune decision tree, spawn-tile ranking and the
// prune/spawn slot update.  Counts and lists stay on the device.
cudaError_t launch_tile_mse(int f, int h, int w, int ts, const float* rendered, int hl, int wl, const float* target,
                            float* tile_err, cudaStream_t stream);
cudaError_t launch_canvas_error(int n, int h, int w, int ts, const float* xy, const uint8_t* in_frame,
                                const float* tile_err, const uint8_t* alive, int64_t* age, float* g_error,
                                float* error, cudaStream_t stream);
int64_t prune_scratch_bytes(int64_t n);
cudaError_t launch_select_for_pruning(int n, const uint8_t* alive, const uint8_t* in_frame, const int64_t* age,
                                      const float* err, long long cap, long long age_max, float q_age, float q_tile,
                                      long long min_age, int64_t* prune_idx, int64_t* prune_count, float* quant,
                                      void* scratch, cudaStream_t stream);
int64_t spawn_tiles_scratch_bytes(int64_t num_tiles);
cudaError_t launch_select_spawn_tiles(int th, int tw, const float* tile_err, const uint8_t* cls, long long n_tiles,
                                      int64_t* tiles_yx, int64_t* take, void* scratch, cudaStream_t stream);
int64_t prune_spawn_scratch_bytes(int64_t n);
cudaError_t launch_apply_prune_spawn(int n, int f, const int64_t* prune_idx, const int64_t* prune_count,
                                     int64_t max_prune, int num_new, int f_new, const float* nxy,
                                     const float* nscale, const float* nrot, const float* nfeat, float* positions,
                                     float* scales, float* rotations, float* colors, uint8_t* alive, int64_t* age,
                                     float* error, int64_t* n_spawned, void* scratch, cudaStream_t stream);

// ---- nd.cu -------------------------------------------------------------------
// Splat of the v7 time-slice rasterizer: 2D Gaussians given by mean, inverse
// covariance (a, b, d), amplitude, features and a pixel cull box, evaluated at
// pixel centres inside the box.  The preprocess feeds the additive path's scan
// and binning; the backward writes its per-pair rows (reduced by
// launch_reduce_gaussian_grads with the amplitude as opacity).
int nd_record_floats(int f);
// Per-Gaussian time conditioning: (x, y, t) means, 3x3 covariances and
// opacities -> conditional mean, inverse covariance (a, b, d), amplitude and cull
// box; the backward maps their gradients onto means, covariances and opacities.
cudaError_t launch_nd_prep_forward(int n, int h, int w, const float* means, const float* covs, const float* opac,
                                   float tq, int falloff, float v3, float v2, float* xy, float* conic, float* amp,
                                   int32_t* box, cudaStream_t stream);
cudaError_t launch_nd_prep_backward(int n, const float* means, const float* covs, const float* opac, float tq,
                                    int falloff, float v3, float v2, const float* g_xy, const float* g_conic,
                                    const float* g_amp, float* g_means, float* g_covs, float* g_opac,
                                    cudaStream_t stream);
cudaError_t launch_nd_preprocess(int n, int ntx, int nty, const float* xy, const float* conic, const int32_t* box,
                                 int f, const float* feat, const float* amp, int32_t* aabb, int32_t* count,
                                 float* geo, float* prec, long long* block_sums, int32_t* tile_count,
                                 cudaStream_t stream);
cudaError_t launch_nd_forward(int f, int h, int w, const float* prec, const int32_t* box, const int32_t* gid_sorted,
                              const int32_t* tile_offsets, float* image, cudaStream_t stream);
cudaError_t launch_nd_backward_pairs(int f, int h, int w, const float* prec, const int32_t* box,
                                     const int32_t* gid_sorted, const int32_t* tile_offsets, const int32_t* aabb,
                                     const int32_t* pair_offset, const float* grad_image, float* pairgrad,
                                     int pair_stride, cudaStream_t stream);

// ---- analytic.cu -------------------------------------------------------------
// Analytic-Splatting pixel integral per element (offset dx, dy and inverse
// covariance s00, s01, s10, s11, all of n elements), its backward, and the
// conditioned logistic CDF (g null: values; else g * slope).
cudaError_t launch_analytic_forward(int64_t n, const float* dx, const float* dy, const float* s00, const float* s01,
                                    const float* s10, const float* s11, float* out, cudaStream_t stream);
cudaError_t launch_analytic_backward(int64_t n, const float* dx, const float* dy, const float* s00, const float* s01,
                                     const float* s10, const float* s11, const float* g, float* g_dx, float* g_dy,
                                     float* g_s00, float* g_s01, float* g_s10, float* g_s11, cudaStream_t stream);
cudaError_t launch_logistic_cdf(int64_t n, const float* x, const float* g, float* out, cudaStream_t stream);

// ---- raster_analytic.cu ------------------------------------------------------
// The additive render with the Analytic-Splatting pixel integral as weight (raw
// conic from geo[5..7]) and its per-pair backward rows, which hold d_xy itself
// (reduce with rows_dxy = true).
cudaError_t launch_render_analytic_forward(int f, int h, int w, const float* geo, const float* feat,
                                           const float* opacity, const int32_t* gid_sorted,
                                           const int32_t* tile_offsets, float* image, cudaStream_t stream);
cudaError_t launch_render_analytic_backward_pairs(int f, int h, int w, const float* geo, const float* feat,
                                                  const float* opacity, const int32_t* gid_sorted,
                                                  const int32_t* tile_offsets, const int32_t* aabb,
                                                  const int32_t* pair_offset, const float* grad_image,
                                                  float* pairgrad, int pair_stride, cudaStream_t stream);

// ---- warp.cu ---------------------------------------------------------------
int64_t warp_scratch_bytes(int64_t n);
cudaError_t launch_warp_canvas(int n, int f, int hl, int wl, int h, int w, const float* motion, float alpha,
                               const float* recon4, const float* pos, const float* scales, const float* rots,
                               const float* ops, const float* colors, float* out_pos, float* out_scales,
                               float* out_rots, float* out_ops, float* out_colors, int32_t* out_count,
                               void* scratch, cudaStream_t stream);
// The same without compaction: every input slot written, the dropped ones
// parked outside the frame with zero opacity and colours (no survivor count).
cudaError_t launch_warp_canvas_parked(int n, int f, int hl, int wl, int h, int w, const float* motion, float alpha,
                                      const float* recon4, const float* pos, const float* scales, const float* rots,
                                      const float* ops, const float* colors, float* out_pos, float* out_scales,
                                      float* out_rots, float* out_ops, float* out_colors, void* scratch,
                                      cudaStream_t stream);
// Backward of launch_warp_canvas (fwd_scratch: the forward's scratch, which
// holds the survivor offsets); d_motion (LR, may be null) is written, d_hr
// planes live in `scratch` (warp_backward_scratch_bytes).
int64_t warp_backward_scratch_bytes(int64_t h, int64_t w);
cudaError_t launch_warp_canvas_backward(int n, int f, int hl, int wl, int h, int w, const float* motion, float alpha,
                                        const float* recon4, const float* pos, const float* scales, const float* rots,
                                        const void* fwd_scratch, const float* g_pos, const float* g_scales,
                                        const float* g_rots, const float* g_ops, const float* g_colors, float* d_pos,
                                        float* d_scales, float* d_rots, float* d_ops, float* d_colors,
                                        float* d_motion, void* scratch, cudaStream_t stream);
cudaError_t launch_warp_positions(int n, int h, int w, const float* motion, float alpha, const float* xy,
                                  float* out_xy, uint8_t* in_frame, cudaStream_t stream);

// ---- feather.cu --------------------------------------------------------------
// One-pass feathered overlapping-tile render.  Gaussian g becomes up to
// kFeatherVariants virtual Gaussians 4 g + k; each carries its packed forward
// record (centre of its phases), its tile hull in vaabb / vcount, and its window
// in vwin: four packed [lo, hi) tile ranges (phase 0 and phase 1 along x, then
// along y; phase-1 ranges in phase-0 tile units).  Ranges are int16.
constexpr int kFeatherVariants = 4;
constexpr int kFeatherMaxTiles = 32767;
// log2 of the normalised feather weight of an entry at tile column (or row) c
// for the phase-bit pattern p = [phase 0 covers the tile] | [phase 1 covers the
// column's phase-1 tile, left part] << 1 | [... right part] << 2; -inf where 0.
struct FeatherTable {
    float lw[8][16];
};
// Fills the table; returns 0 when the reference's clamp of the weight sum at
// 1e-6 could be active (very wide overlaps), where the separable form fails.
int feather_table(int overlap, FeatherTable* tab);
__host__ __device__ inline int pack_range(int lo, int hi) {
    return static_cast<int>((static_cast<uint32_t>(lo) & 0xffffu) | (static_cast<uint32_t>(hi) << 16));
}
__host__ __device__ inline int range_lo(int v) { return static_cast<int16_t>(v & 0xffff); }
__host__ __device__ inline int range_hi(int v) { return v >> 16; }
// Phase-bit pattern of tile index t for the packed phase-0 range r0 and
// phase-1 range r1 (see FeatherTable).
__host__ __device__ inline int feather_pattern(int r0, int r1, int t) {
    const int lo0 = range_lo(r0), hi0 = range_hi(r0), lo1 = range_lo(r1), hi1 = range_hi(r1);
    return (lo0 <= t && t < hi0 ? 1 : 0) | (lo1 <= t && t < hi1 ? 2 : 0) | (lo1 <= t + 1 && t + 1 < hi1 ? 4 : 0);
}
cudaError_t launch_prepare_feathered(int n, int h, int w, int mode, int overlap, const float* xy, const float* scale,
                                     const float* rot, int f, const float* feat, const float* opacity, float* conic,
                                     float* geo, int32_t* vaabb, int32_t* vcount, float* vprec, int32_t* vwin,
                                     long long* block_sums, int32_t* tile_count, cudaStream_t stream);

// ---- v6_front.cu -------------------------------------------------------------
// V6 front-end sanitisation in place (kept Gaussians sanitised, dropped ones
// parked outside the frame with zero features) and its backward through the
// per-Gaussian derivative flags.
cudaError_t launch_v6_sanitize(int n, int h, int w, int f_in, int f_out, int ones, const uint8_t* mask,
                               const float* pos, const float* scl, const float* rot, const float* colors,
                               float* out_xy, float* out_scale, float* out_rot, float* out_feat, uint16_t* flags,
                               cudaStream_t stream);
cudaError_t launch_v6_sanitize_backward(int n, int f_in, int f_out, int ones, const uint16_t* flags,
                                        const float* d_xy, const float* d_scale, const float* d_rot,
                                        const float* d_feat, float* d_pos, float* d_scl, float* d_rot_in,
                                        float* d_colors, cudaStream_t stream);

// ---- raster_fwd.cu / raster_bwd.cu ----------------------------------------
// Entry records (forward -> backward): floats per record for f channels.
int entry_record_floats(int f);
// prec (optional): the packed records of launch_preprocess, read instead of
// geo / feat / opacity.  slots (optional with records) needs aabb and pair_offset.
cudaError_t launch_render_forward(int f, int h, int w, const float* geo, const float* feat,
                                  const float* opacity, const int32_t* gid_sorted,
                                  const int32_t* tile_offsets, float* image, const int32_t* aabb,
                                  const int32_t* pair_offset, float* records, int32_t* slots,
                                  const float* prec, cudaStream_t stream, int frames = 1);

// The windowed forward of the one-pass feathered render over virtual Gaussians
// (launch_prepare_feathered): f <= 16.  With records, entry_pat receives each
// list entry's phase-bit patterns (x | y << 8) for the backward.
cudaError_t launch_render_forward_feathered(int f, int h, int w, const FeatherTable& tab, const float* vprec,
                                           const int32_t* vwin, const int32_t* gid_sorted, const int32_t* tile_offsets,
                                           float* image, float* records, uint16_t* entry_pat, cudaStream_t stream);

// Per-pair partial gradients.  Deterministic mode (pairgrad != null): rows
// (Sx, Sy, d_conic, dF) of pair_stride floats at pair_offset[g] + local tile
// index, entries read from the forward's records/slots when records != null.
// Atomic mode: adds into d_xy / d_conic / d_feat.  items_scratch holds the
// work-item table (backward_items_scratch_bytes): launch_render_backward_tiles
// builds it and runs the backward; the two halves are also exposed so that the
// table (which needs only tile_offsets) can be built beside the forward.
// frames > 1: `frames` stacked h x w frames (tile rows [b nty, (b+1) nty) are
// frame b's; images and dL/dimage are [frames][f][h][w]).
cudaError_t launch_backward_items(int h, int w, int64_t total_pairs, const int32_t* tile_offsets, void* items_scratch,
                                  cudaStream_t stream, int frames = 1);
cudaError_t launch_render_backward_items(int f, int h, int w, int64_t total_pairs, const float* geo,
                                         const float* feat, const float* opacity, const int32_t* gid_sorted,
                                         const int32_t* tile_offsets, const float* grad_image, const int32_t* aabb,
                                         const int32_t* pair_offset, const float* records, const int32_t* slots,
                                         float* pairgrad, int pair_stride, float* d_xy, float* d_conic, float* d_feat,
                                         void* items_scratch, cudaStream_t stream, int frames = 1);
cudaError_t launch_render_backward_tiles(int f, int h, int w, int64_t total_pairs, const float* geo,
                                         const float* feat, const float* opacity, const int32_t* gid_sorted,
                                         const int32_t* tile_offsets, const float* grad_image,
                                         const int32_t* aabb, const int32_t* pair_offset,
                                         const float* records, const int32_t* slots,
                                         float* pairgrad, int pair_stride,
                                         float* d_xy, float* d_conic, float* d_feat, void* items_scratch,
                                         cudaStream_t stream);
// The backward of the windowed feathered forward (records and entry_pat of
// launch_render_forward_feathered, items of launch_backward_items), per-pair
// rows at the virtual Gaussians' gid-major slots; f <= 16.
cudaError_t launch_render_backward_feathered(int f, int h, int w, int64_t total_pairs, const FeatherTable& tab,
                                            const int32_t* gid_sorted, const int32_t* tile_offsets,
                                            const float* grad_image, const int32_t* vaabb, const int32_t* vpair_offset,
                                            const float* records, const uint16_t* entry_pat, float* pairgrad,
                                            int pair_stride, void* items_scratch, cudaStream_t stream);
int backward_pair_stride(int f);
int64_t backward_items_scratch_bytes(int64_t total_pairs, int64_t num_tiles);
cudaError_t launch_reduce_gaussian_grads(int n, int f, const float* pairgrad, int pair_stride,
                                         const int32_t* pair_offset, const float* geo, const float* feat,
                                         const float* opacity, const float* scale, const float* rot,
                                         float* d_xy, float* d_conic, float* d_feat,
                                         float* d_opacity, float* d_scale, float* d_rot,
                                         cudaStream_t stream, bool rows_dxy = false, int vstride = 1);

// ---- raster_alpha.cu -------------------------------------------------------
// Front-to-back alpha compositing over (depth, gid)-ordered lists, its
// back-to-front backward into per-pair rows (Sx, Sy, d_conic(3), dF(F),
// d_opacity) of alpha_pair_stride(f) floats, and the per-Gaussian reduce.
int alpha_pair_stride(int f);
cudaError_t launch_render_alpha_forward(int f, int h, int w, const float* geo, const float* feat,
                                        const float* opacity, const float* background, const int32_t* gid_sorted,
                                        const int32_t* tile_offsets, float* image, float* t_final,
                                        int32_t* n_contrib, cudaStream_t stream);
cudaError_t launch_render_alpha_backward(int f, int h, int w, const float* geo, const float* feat,
                                         const float* opacity, const float* background,
                                         const int32_t* gid_sorted, const int32_t* tile_offsets,
                                         const float* t_final, const int32_t* n_contrib, const float* grad_image,
                                         const int32_t* aabb, const int32_t* pair_offset, float* pairgrad,
                                         cudaStream_t stream);
cudaError_t launch_reduce_alpha_grads(int n, int f, const float* pairgrad, const int32_t* pair_offset,
                                      const float* geo, const float* scale, const float* rot, float* d_xy,
                                      float* d_conic, float* d_feat, float* d_opacity, float* d_scale,
                                      float* d_rot, cudaStream_t stream);

}  // namespace oss
