/*
 * oss_raster.h -- C ABI of the B200 (sm_100a) 2D Gaussian-canvas tile rasterizer
 * and canvas warp.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream handle
 * (cudaStream_t passed as void*; NULL means the legacy default stream).  Nothing
 * here allocates device memory: buffers that are outputs or scratch are passed
 * in by the caller, and the *_scratch_bytes() functions say how large scratch
 * must be.  All work is enqueued on `stream`; no entry point synchronises the
 * host except where its comment says so.
 *
 * Every function returns OSS_OK (0) or an OSS_ERR_* code; oss_last_error()
 * returns a message for the last failure on the calling host thread.
 *
 * Array layouts (row-major, fp32 unless stated):
 *   xy[n][2], scale[n][2], rot[n], feat[n][f], opacity[n]
 *   conic[n][3]      = (a, b, d) of the inverse covariance
 *   aabb[n][4]       = (tx0, ty0, tx1, ty1) int32 tile rectangle, half-open
 *   image[f][h][w]   planar, pixel (px, py) evaluated at integer coordinates
 *   geo[n][8]        = (x, y, A, B, D, a, b, d) with (A, B, D) = (a, 2b, d) * (-0.5*log2 e)
 *   prec[n][r]       = (x, y, A, B, D, feat'[0..f), zeros), r = oss_entry_record_floats(f),
 *                      feat' = feat * opacity: the packed forward record of a Gaussian
 *   tile id          = ty * ceil(w/16) + tx, tiles are 16x16 pixels
 *
 * Binning modes (oss_bin_mode):
 *   OSS_BIN_TIGHT3SIGMA  tile AABB of the q = 9 ellipse (the reference's
 *                        pair_construction_only lists, rasterizer_fwd.cu:74-108)
 *   OSS_BIN_EXACT        tile AABB of the q = 176 ellipse: every pixel outside
 *                        the lists has exp(-q/2) below the smallest normal fp32 (0
 *                        under flush-to-zero), so images equal the reference's
 *                        full-tail sum (rasterizer.py:294-300) to within 1.2e-38
 *                        per Gaussian
 *   OSS_BIN_FULL         every Gaussian in every tile (the reference forward's
 *                        build_full_tile_pairs, rasterizer_fwd.cu:135-149)
 *   OSS_BIN_EXACT56      tile AABB of the q = 56 ellipse: a contribution left
 *                        out has weight exp(-q/2) < e^-28 = 6.9e-13, so the image
 *                        is the full-tail sum to within 6.9e-13 * sum |feat| of
 *                        the Gaussians left out at a pixel (2.2x the 3-sigma
 *                        lists at the BASELINE shapes, against 6.3x for q = 176)
 */
#ifndef OSS_RASTER_H
#define OSS_RASTER_H

#include <stdint.h>

#if defined(__GNUC__)
#define OSS_API __attribute__((visibility("default")))
#else
#define OSS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum oss_status {
    OSS_OK = 0,
    OSS_ERR_INVALID = 1,   /* bad argument: shape, null pointer, tile size */
    OSS_ERR_CUDA = 2,      /* a CUDA runtime call or kernel launch failed */
    OSS_ERR_RANGE = 3,     /* a size exceeds the int32 range the kernels index with */
    OSS_ERR_SCRATCH = 4    /* scratch buffer smaller than *_scratch_bytes() */
};

enum oss_bin_mode {
    OSS_BIN_TIGHT3SIGMA = 0,
    OSS_BIN_EXACT = 1,
    OSS_BIN_FULL = 2,
    OSS_BIN_EXACT56 = 3
};

#define OSS_TILE 16
#define OSS_MAX_CHANNELS 64

/* Message for the last error on this host thread ("" if none). */
OSS_API const char* oss_last_error(void);
/* ABI version of this library (bumped on any signature change). */
OSS_API int oss_abi_version(void);

/* ---------------------------------------------------------------------------
 * Per-Gaussian preprocess: conic, tile AABB, pair count.
 * Replaces _C.preprocess_only (reference oss/cuda/src/bindings.cpp:73 ->
 * rasterizer_fwd.cu:325-379, kernel preprocess_gaussians rasterizer_fwd.cu:38-109).
 * tile_size must be 16.  mode selects the AABB radius (see oss_bin_mode).
 * ------------------------------------------------------------------------- */
OSS_API int oss_preprocess(int64_t n, int64_t h, int64_t w, int64_t tile_size, int32_t mode,
                   const float* xy, const float* scale, const float* rot,
                   float* conic, int32_t* aabb, int32_t* pair_count, void* stream);

/* ---------------------------------------------------------------------------
 * Render prepare: preprocess + gid-major pair-offset scan + geo records +
 * per-tile pair counts and list offsets.
 * First half of _C.rasterize_forward (rasterizer_fwd.cu:478-545) and of
 * _C.pair_construction_only (rasterizer_fwd.cu:381-444).
 * Outputs: conic[n*3], aabb[n*4], pair_offset[n+1] (exclusive scan of the pair
 * counts; pair_offset[n] = total, valid only if total <= INT32_MAX),
 * geo[n*8], total_pairs[1] (int64, on the device), tile_offsets[T+1] (int32:
 * where each tile's list will start; tile_offsets[T] = total) and
 * tile_count[oss_tile_count_elems(T)] (the per-tile list lengths in the
 * layout oss_bin_pairs reads; it consumes them).  In OSS_BIN_FULL mode
 * tile_count and tile_offsets are not written and may be NULL.
 * prec (optional, 16-byte aligned; NULL skips it, and then f, feat and opacity
 * are ignored): the packed forward records of the additive render, so that
 * oss_render_forward gathers one record per list entry instead of geo, feat
 * and opacity separately.  opacity may be NULL (1).
 * ------------------------------------------------------------------------- */
OSS_API int64_t oss_render_prepare_scratch_bytes(int64_t n);
OSS_API int64_t oss_tile_count_elems(int64_t num_tiles);
OSS_API int oss_render_prepare(int64_t n, int64_t h, int64_t w, int32_t mode,
                       const float* xy, const float* scale, const float* rot,
                       int64_t f, const float* feat, const float* opacity,
                       float* conic, int32_t* aabb, int32_t* pair_offset, float* geo, float* prec,
                       int64_t* total_pairs, int32_t* tile_count, int32_t* tile_offsets,
                       void* scratch, int64_t scratch_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Deterministic tile binning of the pairs described by (aabb, pair_offset,
 * tile_count, tile_offsets) from oss_render_prepare: gid_sorted lists, per
 * tile in ascending tile id, the Gaussians overlapping that tile in ascending
 * gid order; tile_offsets[T+1] brackets them.  Bit-exact with the reference's
 * sort of (tile << 32 | gid) keys plus searchsorted (rasterizer_fwd.cu:446-475)
 * for the same AABBs.
 *
 * No host synchronisation: the pair total is read on the device from
 * total_pairs (oss_render_prepare's int64 output) and compared with capacity,
 * the length of gid_sorted.  If it fits, *overflow = 0.  If it does not,
 * *overflow = 1 and every tile list and every Gaussian's pair range
 * (tile_offsets, pair_offset) is emptied, so the forward and backward that
 * follow stay in bounds and produce a zero image and zero gradients; the
 * caller re-runs with capacity >= the total once it reads the flag.  In
 * OSS_BIN_FULL mode tile_offsets is written here and the total n * num_tiles
 * is checked on the host (a capacity below it is an error).  tile_count is
 * consumed (its contents are unspecified afterwards).
 * ------------------------------------------------------------------------- */
OSS_API int64_t oss_bin_pairs_scratch_bytes(int64_t n, int64_t capacity, int64_t num_tiles);
OSS_API int oss_bin_pairs(int64_t n, int64_t h, int64_t w, int32_t mode,
                  const int32_t* aabb, int32_t* pair_offset, int32_t* tile_count,
                  const int64_t* total_pairs, int64_t capacity,
                  const int32_t* sort_key, const int32_t* key_order,
                  int32_t* gid_sorted, int32_t* tile_offsets, int32_t* overflow,
                  void* scratch, int64_t scratch_bytes, void* stream);
/* sort_key / key_order (both NULL, or both set; not in OSS_BIN_FULL mode):
 * order every tile list by sort_key[g] (a permutation of [0, n)) instead of
 * gid; key_order[k] = the gid with key k.  oss_depth_order makes them for the
 * alpha-blend mode (rank and order of the Gaussians by depth). */

/* ---------------------------------------------------------------------------
 * oss_render_prepare + oss_bin_pairs in one call for a caller that already
 * knows a capacity (no host synchronisation): the same outputs (conic, aabb,
 * pair_offset[n+1], geo, prec, total_pairs, tile_offsets, gid_sorted,
 * overflow, with the same overflow rule) from the same launches.  Replaces the
 * reference's preprocess + pair construction + sort + searchsorted
 * (rasterizer_fwd.cu:381-476).  mode
 * OSS_BIN_TIGHT3SIGMA, OSS_BIN_EXACT or OSS_BIN_EXACT56; full-frame lists go through
 * oss_render_prepare + oss_bin_pairs.  tile_count[oss_tile_count_elems(T)] is
 * working memory (zeroed by the call).
 *
 * frames > 1 bins a batch: Gaussians [frame_offsets[b], frame_offsets[b+1]) of
 * the concatenated inputs (frame_offsets: frames + 1 non-decreasing int32 on
 * the device, 0 to n) are drawn into frame b, every frame h x w.  The tile
 * grid is the frames stacked: T = frames * ceil(h/16) * ceil(w/16) tiles, tile
 * rows [b ceil(h/16), (b+1) ceil(h/16)) are frame b's, and aabb rows are in
 * that stacked grid.  Each frame's lists are those a call on its Gaussians
 * alone would build, with gids offset by frame_offsets[b].  The *_frames
 * forward and backward entries render such lists into [frames][f][h][w]
 * images.  frames == 1 takes frame_offsets NULL.
 * ------------------------------------------------------------------------- */
OSS_API int64_t oss_render_bin_scratch_bytes(int64_t n, int64_t capacity, int64_t num_tiles);
OSS_API int oss_render_bin(int64_t n, int64_t h, int64_t w, int64_t frames, const int32_t* frame_offsets,
                   int32_t mode, const float* xy, const float* scale, const float* rot,
                   int64_t f, const float* feat, const float* opacity,
                   float* conic, int32_t* aabb, int32_t* pair_offset, float* geo, float* prec,
                   int64_t* total_pairs, int32_t* tile_count, int32_t* tile_offsets,
                   int64_t capacity, int32_t* gid_sorted, int32_t* overflow,
                   void* scratch, int64_t scratch_bytes, void* stream);

/* Host-side read of the pair total without a copy engine: a one-thread kernel
 * on `stream` stores *total_pairs (device) into host_total, which must be
 * pinned host memory (written through its device mapping).  Record an event
 * after it and synchronise on the event to read host_total -- unlike a
 * device-to-host copy, this does not queue behind large transfers other
 * streams have in flight. */
OSS_API int oss_publish_total(const int64_t* total_pairs, int64_t* host_total, void* stream);

/* ---------------------------------------------------------------------------
 * Stable depth order for the alpha-blend lists: order[i] = the gid at position
 * i of the Gaussians sorted by (depth, gid) ascending, rank[g] = its position
 * (-0.0 counts as +0.0; -inf first, +inf last).
 * ------------------------------------------------------------------------- */
OSS_API int64_t oss_depth_order_scratch_bytes(int64_t n);
OSS_API int oss_depth_order(int64_t n, const float* depth, int32_t* order, int32_t* rank,
                    void* scratch, int64_t scratch_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Forward additive render: image[c][p] = sum over the tile list of p of
 *   feat'[g][c] * exp(-q_g(p)/2),  feat' = feat * opacity (opacity may be NULL).
 * Replaces the rasterize_sum loop of _C.rasterize_forward
 * (rasterizer_fwd.cu:151-322, host loop :570-587).  Writes every pixel.
 *
 * Per-Gaussian inputs: prec (oss_render_prepare's packed records for this f;
 * geo, feat and opacity are then not read and may be NULL), or geo, feat and
 * opacity.
 *
 * Entry records (optional): for every list entry e in list order,
 * records[e][oss_entry_record_floats(f)] = (x, y, A, B, D, feat'(f), zero
 * padding) of its Gaussian, and, if slots is non-NULL, slots[e] = its gid-major
 * pair slot pair_offset[g] + local tile index (needs aabb and pair_offset).
 * The backward reads them instead of gathering per-Gaussian data a second time
 * (and derives the slots itself when it gets none).  records and slots hold
 * capacity entries (any upper bound of the pair total).
 * ------------------------------------------------------------------------- */
OSS_API int oss_entry_record_floats(int64_t f);
OSS_API int oss_render_forward(int64_t n, int64_t f, int64_t h, int64_t w,
                       const float* geo, const float* feat, const float* opacity, const float* prec,
                       const int32_t* gid_sorted, const int32_t* tile_offsets,
                       float* image, const int32_t* aabb, const int32_t* pair_offset,
                       float* records, int32_t* slots, void* stream);
/* The same over the lists of oss_render_bin with frames > 1: image is
 * [frames][f][h][w]. */
OSS_API int oss_render_forward_frames(int64_t n, int64_t f, int64_t h, int64_t w, int64_t frames,
                       const float* geo, const float* feat, const float* opacity, const float* prec,
                       const int32_t* gid_sorted, const int32_t* tile_offsets,
                       float* image, const int32_t* aabb, const int32_t* pair_offset,
                       float* records, int32_t* slots, void* stream);

/* ---------------------------------------------------------------------------
 * Deterministic backward for lists made by oss_bin_pairs: per-pair partial
 * gradients in a fixed order, then a per-Gaussian reduction in gid-major order,
 * fused with the d_conic -> (d_scale, d_rot) chain rule and the opacity unfold.
 * Same gradients as _C.rasterize_backward + _C.conic_to_scale_rot_grad
 * (rasterizer_bwd.cu:32-154) without atomics.
 * d_feat is the gradient w.r.t. feat (not feat'); d_opacity, d_scale, d_rot
 * may be NULL.  total_pairs may be the exact pair count or any upper bound of
 * it, such as the capacity given to oss_bin_pairs: the kernels take the list
 * lengths from tile_offsets and pair_offset on the device.  records/slots are
 * the forward's entry records and slots (records NULL: gathered through
 * gid_sorted instead; slots NULL: derived from gid_sorted, aabb, pair_offset).
 * ------------------------------------------------------------------------- */
OSS_API int64_t oss_render_backward_scratch_bytes(int64_t total_pairs, int64_t f, int64_t num_tiles);
OSS_API int oss_render_backward(int64_t n, int64_t f, int64_t h, int64_t w,
                        const float* geo, const float* feat, const float* opacity,
                        const float* scale, const float* rot,
                        const int32_t* aabb, const int32_t* pair_offset, int64_t total_pairs,
                        const int32_t* gid_sorted, const int32_t* tile_offsets,
                        const float* records, const int32_t* slots,
                        const float* grad_image,
                        float* d_xy, float* d_conic, float* d_feat, float* d_opacity,
                        float* d_scale, float* d_rot,
                        void* scratch, int64_t scratch_bytes, void* stream);

/* The two halves of oss_render_backward, for callers that keep the per-pair
 * partials: oss_render_backward_pairs writes pairgrad[total_pairs][stride]
 * (stride = oss_pair_grad_stride(f) floats: Sx, Sy (the dq-weighted offset
 * sums), d_conic(3), d_feat'(f), zero padding) in gid-major pair order;
 * oss_reduce_pair_grads sums them per Gaussian and applies the conic from geo
 * (d_xy = (a Sx + b Sy, b Sx + d Sy)).  The scratch of oss_render_backward is
 * pairgrad followed by the work-item table oss_render_backward_pairs needs. */
OSS_API int oss_pair_grad_stride(int64_t f);
OSS_API int64_t oss_render_backward_pairs_scratch_bytes(int64_t total_pairs, int64_t num_tiles);
OSS_API int oss_render_backward_pairs(int64_t n, int64_t f, int64_t h, int64_t w,
                              const float* geo, const float* feat, const float* opacity,
                              const int32_t* aabb, const int32_t* pair_offset, int64_t total_pairs,
                              const int32_t* gid_sorted, const int32_t* tile_offsets,
                              const float* records, const int32_t* slots,
                              const float* grad_image, float* pairgrad,
                              void* scratch, int64_t scratch_bytes, void* stream);
/* The backward's work-item table alone (scratch of oss_render_backward_pairs,
 * oss_render_backward_pairs_scratch_bytes(total_pairs, num_tiles) bytes).  It
 * reads only tile_offsets, so it can be built on another stream while the
 * forward runs; oss_render_backward_items then runs the per-pair backward over
 * that table (oss_render_backward_pairs = both, in order).  The table holds the
 * backward's work counter: the backward takes items through it and leaves it
 * cleared, so a table serves any number of backward launches, one at a time. */
OSS_API int oss_backward_items(int64_t h, int64_t w, int64_t total_pairs, const int32_t* tile_offsets,
                       void* items, int64_t items_bytes, void* stream);
/* Stacked frames (oss_render_bin with frames > 1): the item table over all
 * frames' tiles (items_bytes >= oss_render_backward_pairs_scratch_bytes(
 * total_pairs, frames * tiles of one frame)), and the backward reading
 * grad_image as [frames][f][h][w]. */
OSS_API int oss_backward_items_frames(int64_t h, int64_t w, int64_t frames, int64_t total_pairs,
                       const int32_t* tile_offsets, void* items, int64_t items_bytes, void* stream);
OSS_API int oss_render_backward_items_frames(int64_t n, int64_t f, int64_t h, int64_t w, int64_t frames,
                              const float* geo, const float* feat, const float* opacity,
                              const int32_t* aabb, const int32_t* pair_offset, int64_t total_pairs,
                              const int32_t* gid_sorted, const int32_t* tile_offsets,
                              const float* records, const int32_t* slots,
                              const float* grad_image, float* pairgrad,
                              void* items, int64_t items_bytes, void* stream);
OSS_API int oss_render_backward_items(int64_t n, int64_t f, int64_t h, int64_t w,
                              const float* geo, const float* feat, const float* opacity,
                              const int32_t* aabb, const int32_t* pair_offset, int64_t total_pairs,
                              const int32_t* gid_sorted, const int32_t* tile_offsets,
                              const float* records, const int32_t* slots,
                              const float* grad_image, float* pairgrad,
                              void* items, int64_t items_bytes, void* stream);
OSS_API int oss_reduce_pair_grads(int64_t n, int64_t f, const float* pairgrad,
                          const int32_t* pair_offset, const float* geo,
                          const float* feat, const float* opacity,
                          const float* scale, const float* rot,
                          float* d_xy, float* d_conic, float* d_feat, float* d_opacity,
                          float* d_scale, float* d_rot, void* stream);

/* ---------------------------------------------------------------------------
 * One-pass feathered overlapping-tile render: replaces the four phase-shifted
 * renders and the blend of oss/sr/v6/rasterizer.py:159-242
 * (V6Rasterizer._render_overlapped, _phase_feather_mask, _cosine_ramp), reached
 * through rasterize_gaussians(..., overlap=o).  Each Gaussian becomes up to four
 * virtual Gaussians 4 g + k (a second centre per axis only where the reference's
 * shifted mean x + o rounds in fp32); each carries its tile hull (vaabb, 4 ints),
 * its packed forward record (vprec, oss_entry_record_floats(f) floats, centre of
 * its phases) and its window (vwin, 4 ints: packed int16 [lo, hi) phase tile
 * ranges).  The image is the reference's sum over phases of mask * render /
 * sum of masks, evaluated once per pixel and list entry with the separable
 * feather window in the exponent.  Pipeline: prepare_feathered -> oss_bin_pairs
 * over the 4N virtual Gaussians (mode tight3sigma: the lists follow vaabb) ->
 * forward_feathered (records + entry_pat when a backward follows) ->
 * oss_backward_items + backward_feathered -> reduce_pair_grads_feathered (sums
 * the four variants' rows of each Gaussian).  F <= 16, overlap > 0, at most
 * 32767 tiles per axis; oss_feather_supported says whether a call qualifies. */
OSS_API int oss_feather_supported(int32_t overlap, int64_t f, int64_t h, int64_t w);
OSS_API int64_t oss_feather_virtual_count(int64_t n);
OSS_API int64_t oss_render_prepare_feathered_scratch_bytes(int64_t n);
OSS_API int oss_render_prepare_feathered(int64_t n, int64_t h, int64_t w, int32_t mode, int32_t overlap,
                                         const float* xy, const float* scale, const float* rot, int64_t f,
                                         const float* feat, const float* opacity, float* conic, float* geo,
                                         int32_t* vaabb, int32_t* vpair_offset, float* vprec, int32_t* vwin,
                                         int64_t* total_pairs, int32_t* tile_count, int32_t* tile_offsets,
                                         void* scratch, int64_t scratch_bytes, void* stream);
OSS_API int oss_render_forward_feathered(int64_t n, int64_t f, int64_t h, int64_t w, int32_t overlap,
                                         const float* vprec, const int32_t* vwin, const int32_t* gid_sorted,
                                         const int32_t* tile_offsets, float* image, float* records,
                                         uint16_t* entry_pat, void* stream);
OSS_API int oss_render_backward_feathered(int64_t n, int64_t f, int64_t h, int64_t w, int32_t overlap,
                                          const int32_t* vaabb, const int32_t* vpair_offset, int64_t total_pairs,
                                          const int32_t* gid_sorted, const int32_t* tile_offsets,
                                          const float* records, const uint16_t* entry_pat, const float* grad_image,
                                          float* pairgrad, void* items, int64_t items_bytes, void* stream);
OSS_API int oss_reduce_pair_grads_feathered(int64_t n, int64_t f, const float* pairgrad, const int32_t* vpair_offset,
                                            const float* geo, const float* feat, const float* opacity,
                                            const float* scale, const float* rot, float* d_xy, float* d_conic,
                                            float* d_feat, float* d_opacity, float* d_scale, float* d_rot,
                                            void* stream);

/* ---------------------------------------------------------------------------
 * Alpha-blend mode (blend="alpha"; no reference counterpart -- the reference
 * rasterizer is additive only).  Over lists ordered by (depth, gid) (sort_key
 * = rank from oss_depth_order), per pixel front to back:
 *   a = min(0.99, opacity * exp(-q/2)) (0 for q < 0 or non-finite); entries
 *   with a < 1/255 are skipped; compositing stops before the first entry whose
 *   T (1 - a) would fall below 1e-4; C += feat a T; T *= 1 - a;
 *   image = C + T * background (background: device f floats, NULL = 0;
 *   opacity NULL = 1).
 * The forward also writes t_final[h][w] (final T) and n_contrib[h][w] (1 +
 * the tile-list position of the last composited entry), which the backward
 * needs.  The backward writes deterministic per-pair rows into scratch
 * (oss_render_alpha_backward_scratch_bytes) and reduces them per Gaussian:
 * d_xy, d_conic, d_feat (w.r.t. feat), d_opacity, and d_scale / d_rot when
 * d_scale is non-null.  total_pairs may be any upper bound of the pair count.
 * ------------------------------------------------------------------------- */
OSS_API int oss_render_alpha_forward(int64_t n, int64_t f, int64_t h, int64_t w,
                             const float* geo, const float* feat, const float* opacity,
                             const float* background, const int32_t* gid_sorted,
                             const int32_t* tile_offsets, float* image, float* t_final,
                             int32_t* n_contrib, void* stream);
OSS_API int oss_alpha_pair_grad_stride(int64_t f);
OSS_API int64_t oss_render_alpha_backward_scratch_bytes(int64_t total_pairs, int64_t f);
OSS_API int oss_render_alpha_backward(int64_t n, int64_t f, int64_t h, int64_t w,
                              const float* geo, const float* feat, const float* opacity,
                              const float* background, const float* scale, const float* rot,
                              const int32_t* aabb, const int32_t* pair_offset, int64_t total_pairs,
                              const int32_t* gid_sorted, const int32_t* tile_offsets,
                              const float* t_final, const int32_t* n_contrib,
                              const float* grad_image, float* d_xy, float* d_conic, float* d_feat,
                              float* d_opacity, float* d_scale, float* d_rot,
                              void* scratch, int64_t scratch_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Backward for arbitrary caller lists (per-pair partial sums, then fp32 atomics):
 * replaces _C.rasterize_backward (bindings.cpp:66 -> rasterizer_bwd.cu:157-247).
 * d_xy, d_conic, d_feat are zeroed here.  total_pairs = tile_offsets[T], the
 * length of gid_sorted.
 * ------------------------------------------------------------------------- */
OSS_API int64_t oss_rasterize_backward_lists_scratch_bytes(int64_t n, int64_t total_pairs, int64_t num_tiles);
OSS_API int oss_rasterize_backward_lists(int64_t n, int64_t f, int64_t h, int64_t w,
                                 const float* xy, const float* conic, const float* feat,
                                 const int32_t* gid_sorted, int64_t total_pairs,
                                 const int32_t* tile_offsets, const float* grad_image,
                                 float* d_xy, float* d_conic, float* d_feat,
                                 void* scratch, int64_t scratch_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Geo records from caller conics (for oss_render_forward with an explicit conic).
 * ------------------------------------------------------------------------- */
OSS_API int oss_make_geo(int64_t n, const float* xy, const float* conic, float* geo, void* stream);

/* ---------------------------------------------------------------------------
 * d_conic -> (d_scale, d_rot): replaces _C.conic_to_scale_rot_grad
 * (bindings.cpp:67 -> rasterizer_bwd.cu:115-154, 249-289).
 * ------------------------------------------------------------------------- */
OSS_API int oss_conic_to_scale_rot_grad(int64_t n, const float* scale, const float* rot,
                                const float* d_conic, float* d_scale, float* d_rot,
                                void* stream);

/* ---------------------------------------------------------------------------
 * Full-frame lists: gid_sorted[t*n + i] = i, tile_offsets[t] = t*n
 * (build_full_tile_pairs, rasterizer_fwd.cu:135-149).  n*T must fit int32.
 * ------------------------------------------------------------------------- */
OSS_API int oss_full_tile_pairs(int64_t n, int64_t num_tiles, int32_t* gid_sorted,
                        int32_t* tile_offsets, void* stream);

/* ---------------------------------------------------------------------------
 * Stable counting sort of gid by tile_id: replaces _C.tile_bin_counting_sort
 * (bindings.cpp:75 -> tile_bin_counting_sort.cu:71-128).  Entries with a tile
 * id outside [0, num_tiles) go after all valid ones, in input order;
 * tile_offsets[num_tiles] = n as in the reference (:40-48).  Within a tile the
 * input order is kept (the reference's atomic cursor leaves it unspecified).
 * ------------------------------------------------------------------------- */
OSS_API int64_t oss_tile_bin_counting_sort_scratch_bytes(int64_t n, int64_t num_tiles);
OSS_API int oss_tile_bin_counting_sort(int64_t n, int64_t num_tiles,
                               const int32_t* tile_id, const int32_t* gid,
                               int32_t* sorted_gid, int32_t* tile_offsets,
                               void* scratch, int64_t scratch_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * oss_tile_bin_counting_sort without any allocation -- no counterpart in the
 * reference; it exists for callers that cannot allocate device memory (a
 * per-frame hook inside a host application with a fixed device memory budget,
 * or an embedding host that owns all device allocations), since the counting
 * sort needs scratch.  Same inputs, outputs and results as
 * oss_tile_bin_counting_sort, but the scratch is a fixed 5 MiB array in the
 * library's device image (held by every GPU that loads the library until
 * process exit).  Limits: n <= 262144 entries and num_tiles <= 65536; larger
 * calls fail with OSS_ERR_RANGE.  Calls no cudaMalloc/cudaFree.
 * Every call looks up the array's address in the calling thread's current
 * context (cudaGetSymbolAddress), so a device reset or a context the caller made
 * current itself is picked up; the first call in a context also loads the
 * library's device code there, so make that first call before any stream
 * capture.  All calls share the one array: calls whose GPU work
 * overlaps (e.g. on two streams at once) race and must be serialised by the
 * caller.  Each call clears what must start at zero.
 * ------------------------------------------------------------------------- */
OSS_API int oss_tile_bin_counting_sort_noalloc(int64_t n, int64_t num_tiles,
                                               const int32_t* tile_id, const int32_t* gid,
                                               int32_t* sorted_gid, int32_t* tile_offsets,
                                               void* stream);

/* ---------------------------------------------------------------------------
 * GS-STVSR canvas warp: replaces oss/sr/v6/canvas_warp.py:177-254 (warp_canvas)
 * with covariance_resampling.py:76-116.  motion_lr[2][h_lr][w_lr] is the LR
 * motion of the canvas (the reference uses the first batch item, :66-77) and
 * is multiplied by alpha before use (extrapolation at t + alpha).  The HR
 * motion is F.interpolate(bilinear, align_corners=False) of it when
 * (h_lr, w_lr) != (h, w), evaluated per Gaussian without an HR buffer.
 * recon is the 2x2 row-major Sigma_recon (HOST pointer, 4 floats).
 * Gaussians whose warped centre leaves [0,w)x[0,h) are dropped; the others are
 * written in input order to out_*; out_count (device int32) receives their
 * number.  colors is [n][f].
 * ------------------------------------------------------------------------- */
OSS_API int64_t oss_warp_canvas_scratch_bytes(int64_t n);
OSS_API int oss_warp_canvas(int64_t n, int64_t f, int64_t h_lr, int64_t w_lr, int64_t h, int64_t w,
                            const float* motion_lr, float alpha, const float* recon,
                            const float* positions, const float* scales, const float* rotations,
                            const float* opacities, const float* colors,
                            float* out_positions, float* out_scales, float* out_rotations,
                            float* out_opacities, float* out_colors, int32_t* out_count,
                            void* scratch, int64_t scratch_bytes, void* stream);
/* The same warp without compaction, for a render that follows on the device:
 * every input slot g is written at out_*[g]; a Gaussian whose warped centre
 * leaves the frame is parked at (-1e7, -1e7) with opacity and colours 0, so it
 * bins into no tile and adds nothing to an image.  No count is produced, so
 * nothing needs to be read on the host before the render.  Forward only. */
OSS_API int oss_warp_canvas_parked(int64_t n, int64_t f, int64_t h_lr, int64_t w_lr, int64_t h, int64_t w,
                            const float* motion_lr, float alpha, const float* recon,
                            const float* positions, const float* scales, const float* rotations,
                            const float* opacities, const float* colors,
                            float* out_positions, float* out_scales, float* out_rotations,
                            float* out_opacities, float* out_colors,
                            void* scratch, int64_t scratch_bytes, void* stream);

/* Backward of oss_warp_canvas: the gradients autograd takes through
 * canvas_warp.py:177-254 and covariance_resampling.py:76-116.  g_* are the
 * gradients of the compacted outputs (out_count rows; any may be null for zero);
 * d_* receive the gradients of the n inputs (dropped Gaussians get zero) and
 * d_motion_lr[2][h_lr][w_lr] that of the motion (null: not wanted; sums of
 * fp64 atomics, so its last bits may vary from run to run).  forward_scratch is the scratch
 * of the forward call, unchanged since.  The reconstruction covariance is a
 * constant here.  Where the resampled covariance is exactly isotropic the
 * rotation's gradient is 0 (atan2 has none there). */
OSS_API int64_t oss_warp_canvas_backward_scratch_bytes(int64_t h, int64_t w);
OSS_API int oss_warp_canvas_backward(int64_t n, int64_t f, int64_t h_lr, int64_t w_lr, int64_t h, int64_t w,
                                     const float* motion_lr, float alpha, const float* recon,
                                     const float* positions, const float* scales, const float* rotations,
                                     const void* forward_scratch, const float* g_positions, const float* g_scales,
                                     const float* g_rotations, const float* g_opacities, const float* g_colors,
                                     float* d_positions, float* d_scales, float* d_rotations, float* d_opacities,
                                     float* d_colors, float* d_motion_lr, void* scratch, int64_t scratch_bytes,
                                     void* stream);

/* ---------------------------------------------------------------------------
 * V6 front end: replaces the gathers and sanitisation of V6Rasterizer.forward
 * (oss/sr/v6/rasterizer.py:56-157, _sanitize_active_gaussians :244-291,
 * _token_features :319-327) without host reads.  For the n live Gaussians:
 * kept = active_mask (uint8, null: all) and finite position / scale / rotation
 * / used features and the 3 max|scale| disc overlapping the frame.  A kept
 * Gaussian is written sanitised (|scale| clamped to [1e-3, max(h, w)], position
 * clamped to [0, w - 1e-4] x [0, h - 1e-4], rotation wrapped by atan2(sin, cos),
 * features padded or truncated to f_out, then a ones channel when
 * ones_channel); a dropped one is parked outside the frame with zero features,
 * so it bins into no tile.  flags (uint16 [n]) keep what the backward needs:
 * oss_v6_sanitize_backward maps the render's input gradients (d_feat has
 * f_out + ones columns; any input may be null for zero) to the canvas tensors
 * with PyTorch's derivative conventions at clamp bounds and ties. */
OSS_API int oss_v6_sanitize(int64_t n, int64_t h, int64_t w, int64_t f_in, int64_t f_out, int32_t ones_channel,
                            const uint8_t* active_mask, const float* positions, const float* scales,
                            const float* rotations, const float* colors, float* out_xy, float* out_scale,
                            float* out_rot, float* out_feat, uint16_t* flags, void* stream);
OSS_API int oss_v6_sanitize_backward(int64_t n, int64_t f_in, int64_t f_out, int32_t ones_channel,
                                     const uint16_t* flags, const float* d_xy, const float* d_scale,
                                     const float* d_rot, const float* d_feat, float* d_positions, float* d_scales,
                                     float* d_rotations, float* d_colors, void* stream);

/* ---------------------------------------------------------------------------
 * Position-only warp: replaces oss/gaussian/canvas/warp.py:28-91
 * (warp_positions); motion[2][h][w] at the output resolution, times alpha
 * (warp_canvas(canvas, motion, alpha), :94-137).  in_frame is uint8 [n].
 * ------------------------------------------------------------------------- */
OSS_API int oss_warp_positions(int64_t n, int64_t h, int64_t w, const float* motion, float alpha,
                               const float* xy, float* out_xy, uint8_t* in_frame, void* stream);

/* ---- Analytic-Splatting pixel integral (oss/sr/v6/aa_analytic_splat.py:46-202) ----
 * Elementwise over n elements: the integral of an un-normalised 2D Gaussian with inverse covariance
 * [[s00, s01], [s10, s11]] over the unit pixel square at offset (dx, dy), with the conditioned logistic
 * CDF S(x) = 1 / (1 + exp(-1.6 x - 0.07 x^3)); the backward maps the gradient of the values onto the
 * six inputs.  oss_logistic_cdf writes S(x) (g NULL) or g * S'(x). */
OSS_API int oss_analytic_pixel_integral(int64_t n, const float* dx, const float* dy, const float* s00,
                                        const float* s01, const float* s10, const float* s11, float* out,
                                        void* stream);
OSS_API int oss_analytic_pixel_integral_backward(int64_t n, const float* dx, const float* dy, const float* s00,
                                                 const float* s01, const float* s10, const float* s11,
                                                 const float* g, float* g_dx, float* g_dy, float* g_s00,
                                                 float* g_s01, float* g_s10, float* g_s11, void* stream);
OSS_API int oss_logistic_cdf(int64_t n, const float* x, const float* g, float* out, void* stream);

/* The additive render with this integral as the weight of every list entry (instead of exp(-q/2)),
 * at integer pixel centres, over the lists and geo of oss_render_prepare / oss_bin_pairs (use exact
 * lists: the logistic tails are zero in fp32 beyond them); f <= 32.  The backward writes d_xy, d_conic
 * (of the conic entries a, b, d), d_feat, d_opacity (opacity may be NULL) and, with scale / rot given,
 * d_scale / d_rot; scratch holds the per-pair rows. */
OSS_API int oss_render_analytic_forward(int64_t n, int64_t f, int64_t h, int64_t w, const float* geo,
                                        const float* feat, const float* opacity, const int32_t* gid_sorted,
                                        const int32_t* tile_offsets, float* image, void* stream);
OSS_API int64_t oss_render_analytic_backward_scratch_bytes(int64_t total_pairs, int64_t f);
OSS_API int oss_render_analytic_backward(int64_t n, int64_t f, int64_t h, int64_t w, const float* geo,
                                         const float* feat, const float* opacity, const float* scale,
                                         const float* rot, const int32_t* aabb, const int32_t* pair_offset,
                                         int64_t total_pairs, const int32_t* gid_sorted, const int32_t* tile_offsets,
                                         const float* grad_image, float* d_xy, float* d_conic, float* d_feat,
                                         float* d_opacity, float* d_scale, float* d_rot, void* scratch,
                                         int64_t scratch_bytes, void* stream);

/* ---- v7 N-D time-slice splat (oss/sr/v7/nd_rasterizer.py:107-165) ----
 * After the time conditioning every Gaussian is a 2D Gaussian: mean xy (n x 2), inverse covariance
 * conic (n x 3: a, b, d with q = a dx^2 + 2 b dx dy + d dy^2), amplitude amp (n), features feat
 * (n x f, f <= 32) and a cull box (n x 4 int32: x0, y0, x1, y1 in pixels).  out[c](i, j) = sum over
 * Gaussians whose box holds (j, i) of feat[c] * amp * exp(-q / 2) at dx = j + 0.5 - x, dy = i + 0.5 - y.
 *
 * oss_nd_prepare is oss_render_prepare for these inputs (tiles = those the box overlaps; prec holds
 * oss_nd_record_floats(f) floats per Gaussian); bin with oss_bin_pairs(mode OSS_BIN_TIGHT3SIGMA), then
 * oss_nd_forward.  oss_nd_backward_pairs writes the per-pair rows of oss_render_backward_pairs
 * (pair_stride = oss_pair_grad_stride(f)); oss_reduce_pair_grads with opacity = amp and no scale / rot
 * turns them into d_xy, d_conic, d_feat and d_amp (its d_opacity). */
OSS_API int64_t oss_nd_record_floats(int64_t f);
/* The time conditioning that feeds the splat (nd_rasterizer.py:53-104, 168-239, 242-281): per
 * Gaussian, means (n x 3: x, y, t), covariances (n x 9, row-major 3x3) and opacities (n) ->
 * xy (n x 2), conic (n x 3), amp (n) and box (n x 4 int32), for t_query, the time falloff flag and
 * the Mip 3D / 2D variances (<= 0 turns a filter off).  The backward takes the gradients of xy,
 * conic and amp and writes those of the means, covariances and opacities. */
OSS_API int oss_nd_condition(int64_t n, int64_t h, int64_t w, const float* means, const float* covs,
                             const float* opac, float t_query, int32_t time_falloff, float mip3, float mip2,
                             float* xy, float* conic, float* amp, int32_t* box, void* stream);
OSS_API int oss_nd_condition_backward(int64_t n, const float* means, const float* covs, const float* opac,
                                      float t_query, int32_t time_falloff, float mip3, float mip2,
                                      const float* d_xy, const float* d_conic, const float* d_amp,
                                      float* d_means, float* d_covs, float* d_opac, void* stream);
OSS_API int oss_nd_prepare(int64_t n, int64_t h, int64_t w, const float* xy, const float* conic, const int32_t* box,
                           int64_t f, const float* feat, const float* amp, int32_t* aabb, int32_t* pair_offset,
                           float* geo, float* prec, int64_t* total_pairs, int32_t* tile_count,
                           int32_t* tile_offsets, void* scratch, int64_t scratch_bytes, void* stream);
OSS_API int oss_nd_forward(int64_t f, int64_t h, int64_t w, const float* prec, const int32_t* box,
                           const int32_t* gid_sorted, const int32_t* tile_offsets, float* image, void* stream);
OSS_API int oss_nd_backward_pairs(int64_t f, int64_t h, int64_t w, const float* prec, const int32_t* box,
                                  const int32_t* gid_sorted, const int32_t* tile_offsets, const int32_t* aabb,
                                  const int32_t* pair_offset, const float* grad_image, float* pairgrad,
                                  void* stream);

/* ---- Persistent-canvas lifecycle (oss/gaussian/canvas/canvas.py:191-295) ----
 * The steps around the render in PersistentCanvas.update, all on the device.
 * Masks are uint8 (0 / 1), ages int64, everything else fp32. */

/* Per-tile mean squared error (error_detection.py:26-63, per_tile_mse): tile_err[ty * (w / ts) + tx]
 * = mean over the tile's ts x ts pixels of the channel mean of (rendered - target)^2.  rendered is
 * (f, h, w); h and w must be multiples of ts.  target is (f, target_h, target_w): at (h, w) it is used
 * as is, otherwise it is the LR frame and is upsampled on the fly as F.interpolate(bilinear,
 * align_corners=False) would (canvas.py:256-263). */
OSS_API int oss_tile_mse(int64_t f, int64_t h, int64_t w, int64_t ts, const float* rendered, int64_t target_h,
                         int64_t target_w, const float* target, float* tile_err, void* stream);
/* Per-slot error (error_detection.py:66-113, gaussians_error_from_tiles): g_error[i] = the error of the
 * tile holding xy[i], +inf outside [0, w) x [0, h) or, when in_frame is given, where in_frame[i] == 0
 * (canvas.py:266-269).  With alive given: error[i] = alive[i] ? g_error[i] : 0 and
 * age[i] = alive[i] ? age[i] + 1 : 0 (canvas.py:246-249, 270).  Any output may be NULL. */
OSS_API int oss_canvas_error(int64_t n, int64_t h, int64_t w, int64_t ts, const float* xy, const uint8_t* in_frame,
                             const float* tile_err, const uint8_t* alive, int64_t* age, float* g_error,
                             float* error, void* stream);
/* Prune decision tree (prune_spawn.py:72-157, select_for_pruning) with its policy fields
 * (prune_spawn.py:36-62).  prune_idx (n int64) receives *prune_count slot indices: in slot order when
 * the selection fits max(1, floor(max_prune_frac * capacity)), else that many in descending order of
 * priority * 1e6 + error (ties in slot order).  quantiles (2 floats) receive the R2 and R3 thresholds. */
OSS_API int64_t oss_prune_scratch_bytes(int64_t n);
OSS_API int oss_select_for_pruning(int64_t n, const uint8_t* alive, const uint8_t* in_frame, const int64_t* age,
                                   const float* g_error, int64_t capacity, int64_t age_max, double age_low_error_pct,
                                   double tile_error_pct, int64_t min_age_before_prune, double max_prune_frac,
                                   int64_t* prune_idx, int64_t* prune_count, float* quantiles, void* scratch,
                                   int64_t scratch_bytes, void* stream);
/* Spawn tiles (prune_spawn.py:165-208, select_spawn_tiles): the (ty, tx) of the largest tile errors
 * (classifier_mask, nullable, sends masked tiles to -inf; ties in tile order), *take = min(n_tiles,
 * finite eligible tiles) rows of tiles_yx (th * tw x 2 int64). */
OSS_API int64_t oss_spawn_tiles_scratch_bytes(int64_t num_tiles);
OSS_API int oss_select_spawn_tiles(int64_t th, int64_t tw, const float* tile_err, const uint8_t* classifier_mask,
                                   int64_t n_tiles, int64_t* tiles_yx, int64_t* take, void* scratch,
                                   int64_t scratch_bytes, void* stream);
/* Prune/spawn slot update (prune_spawn.py:216-255, apply_prune_spawn): the first *prune_count entries
 * of prune_idx (at most max_prune) die with age and error reset, then the r-th dead slot in slot order
 * takes new Gaussian r for r < num_new (positions, scales, rotation, the first min(f, f_new) colour
 * channels; alive, age 0, error 0).  *n_spawned receives the number written.  num_new may be 0. */
OSS_API int64_t oss_prune_spawn_scratch_bytes(int64_t n);
OSS_API int oss_apply_prune_spawn(int64_t n, int64_t f, const int64_t* prune_idx, const int64_t* prune_count,
                                  int64_t max_prune, int64_t num_new, int64_t f_new, const float* new_xy,
                                  const float* new_scale, const float* new_rot, const float* new_feat,
                                  float* positions, float* scales, float* rotations, float* colors, uint8_t* alive,
                                  int64_t* age, float* error, int64_t* n_spawned, void* scratch,
                                  int64_t scratch_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* OSS_RASTER_H */
