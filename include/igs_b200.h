/*
 * igs_b200 — B200-native (sm_100a) CUDA kernels of Image-GS's per-step 2D Gaussian rasterization, behind a plain C ABI.
 *
 * Conventions shared by every entry point:
 *   - Pointers are CUDA device pointers to contiguous row-major arrays (float32 / int32 unless stated), sizes are element counts.
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream); work is enqueued asynchronously on it and nothing synchronizes.
 *   - The library never allocates device memory: outputs and workspaces are the caller's (query sizes with the *_workspace functions),
 *     so every call can be captured in a CUDA graph.
 *   - Return IGS_OK (0) or an error code; igs_last_error() gives this thread's message. No entry point exits the process.
 * Reference citations are paths inside BaylorMultimediaLab/image-gs (the gsplat fork under gsplat/gsplat/, the rate/quantization code
 * under compress/, the training step in model.py).
 */
#ifndef IGS_B200_H
#define IGS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IGS_VERSION 1

#define IGS_OK 0
#define IGS_ERR_INVALID 1     /* bad argument: caught on the host before any launch */
#define IGS_ERR_CUDA 2        /* a CUDA launch or runtime call failed */
#define IGS_ERR_UNSUPPORTED 3 /* a valid request this build does not handle */

/* Compile-time constants (gsplat/gsplat/cuda/csrc/config.h:1-10; mirrored in model.py:447-448) */
#define IGS_TILE 16
#define IGS_TOP_K 10
#define IGS_MAX_CHANNELS 12

const char *igs_last_error(void);
int igs_version(void);
/* tile side, K of the top-K lists, maximum channels, normalization epsilon */
int igs_constants(int *tile, int *top_k, int *max_channels, double *eps);

/* ---- projection ---------------------------------------------------------------------------------------------------------------- */

/* project_gaussians_2d_scale_rot_forward (gsplat/gsplat/cuda/csrc/bindings.cu:791-837, kernel foward2d.cu:9-59).
 * means2d [N,2] in [0,1) image coordinates, scales2d [N,2] in pixels, rotation [N] radians. Outputs: xys [N,2] pixel centers,
 * radii [N], conics [N,3] (upper triangle of the inverse covariance), num_tiles_hit [N]. Every output element is written. */
int igs_project_fwd(int num_points, const float *means2d, const float *scales2d, const float *rotation, int img_height, int img_width,
                    int tiles_x, int tiles_y, float *xys, int32_t *radii, float *conics, int32_t *num_tiles_hit, void *stream);

/* project_gaussians_2d_scale_rot_backward (bindings.cu:845-891, kernel backward2d.cu:53-100); the reference's means2d argument is
 * unused there and omitted. Outputs v_cov2d [N,3], v_mean2d [N,2], v_scale [N,2], v_rot [N] are fully written. */
int igs_project_bwd(int num_points, const float *scales2d, const float *rotation, int img_height, int img_width, const int32_t *radii,
                    const float *conics, const float *v_xy, const float *v_conic, float *v_cov2d, float *v_mean2d, float *v_scale,
                    float *v_rot, void *stream);

/* ---- tile binning --------------------------------------------------------------------------------------------------------------- */

/* compute_cumulative_intersects (gsplat/gsplat/utils.py:96-115): inclusive int32 prefix sum; `total` (device int32, may be NULL) gets
 * the last element without a host read-back. Workspace: igs_cumsum_workspace(n) bytes (per-block partial sums). */
size_t igs_cumsum_workspace(int n);
int igs_cumsum(int n, const int32_t *num_tiles_hit, int32_t *cum_tiles_hit, int32_t *total, void *workspace, size_t workspace_bytes,
               void *stream);

/* sort_intersects_by_tile (gsplat/gsplat/utils.py:165-186 -> bindings.cu:106-167): Gaussian IDs of the tile intersections sorted by tile,
 * increasing Gaussian ID within a tile, in `capacity` slots (intersections beyond the capacity dropped, unused slots 0), and
 * tile_bins [T,2] = [start, end) per tile ((0,0) when empty). */
size_t igs_sort_workspace(int capacity, int tiles_x, int tiles_y);
int igs_sort_intersects(int num_points, int capacity, const float *xys, const int32_t *radii, const int32_t *cum_tiles_hit, int tiles_x,
                        int tiles_y, int32_t *gaussian_ids_sorted, int32_t *tile_bins, void *workspace, size_t workspace_bytes,
                        void *stream);

/* The binning of igs_sort_intersects for callers that cannot allocate device memory and have no workspace to lend (a plugin in a host
 * application that owns all device memory, or code where an allocation would synchronize the device). No counterpart in the
 * reference. Its scratch is a fixed array inside the library, about 16 MiB in every CUDA context that runs it (the device's primary
 * context or one the host application created), held until that context or the process ends; capacity above IGS_NOALLOC_MAX_CAPACITY
 * or more than IGS_NOALLOC_MAX_TILES tiles is rejected with IGS_ERR_INVALID. The array's address belongs to one context: the first call
 * in each context looks it up (with that context current) and caches it under the context's unique ID; make that first call before any
 * stream capture. All calls in a context share the array, so calls that overlap on the GPU race; each call clears what must start at
 * zero. */
#define IGS_NOALLOC_MAX_CAPACITY 1048576
#define IGS_NOALLOC_MAX_TILES 65536
int igs_sort_intersects_noalloc(int num_points, int capacity, const float *xys, const int32_t *radii, const int32_t *cum_tiles_hit,
                                int tiles_x, int tiles_y, int32_t *gaussian_ids_sorted, int32_t *tile_bins, void *stream);

/* ---- top-K normalized rasterization ---------------------------------------------------------------------------------------------- */

/* nd_rasterize_forward_topk_norm (bindings.cu:380-437, kernel forward.cu:223-375): out_img [C,H,W] (channel-planar) and
 * pixel_topk [H,W,10] Gaussian IDs (-1 empty). colors [N,C], C <= IGS_MAX_CHANNELS. */
int igs_raster_fwd_topk(int tiles_x, int tiles_y, int img_height, int img_width, int channels, const int32_t *gaussian_ids_sorted,
                        const int32_t *tile_bins, const float *xys, const float *conics, const float *colors, float *out_img,
                        int32_t *pixel_topk, void *stream);

/* The same forward pass for the training step (rasterize_sum.py:169-267's autograd path): instead of pixel_topk, tile_topk
 * [T,10,256] uint16 holds each pixel's slots as positions in its tile's Gaussian list (0xFFFF empty), indexed by the pixel's lane in
 * the tile (warp w covers the 8x4 patch (w%2, w/2), lane l its pixel (l%8, l/8)). Tiles whose list holds 65535 entries or more are left
 * empty there; igs_raster_bwd_topk_tiles selects their lists again. max_list_len: an upper bound of the list lengths (informational). */
int igs_raster_fwd_topk_tiles(int tiles_x, int tiles_y, int img_height, int img_width, int channels, int max_list_len,
                              const int32_t *gaussian_ids_sorted, const int32_t *tile_bins, const float *xys, const float *conics,
                              const float *colors, float *out_img, uint16_t *tile_topk, void *stream);

/* igs_raster_fwd_topk_tiles with the training loss fused into its epilogue (model.py:1224-1227: loss = ratio * F.l1_loss(image,
 * target), whose gradient is sign(image - target) * ratio / numel): also reads target [C,H,W] and writes *loss and v_output [C,H,W], the
 * gradient the backward pass takes, so the image is not read again by a separate loss pass. The loss is summed per tile, then in tile
 * order by a second one-CTA kernel (deterministic). workspace: igs_raster_l1_workspace(tiles_x * tiles_y) bytes (per-tile partial sums),
 * 16-byte aligned, no initialization needed. No counterpart in the reference, which calls F.l1_loss on the returned image. */
size_t igs_raster_l1_workspace(int num_tiles);
int igs_raster_fwd_topk_tiles_l1(int tiles_x, int tiles_y, int img_height, int img_width, int channels, int max_list_len,
                                 const int32_t *gaussian_ids_sorted, const int32_t *tile_bins, const float *xys, const float *conics,
                                 const float *colors, const float *target, float ratio, float *out_img, uint16_t *tile_topk, float *loss,
                                 float *v_output, void *workspace, size_t workspace_bytes, void *stream);

/* The training step's rasterization with the L1 loss in one kernel: the top-K forward pass, loss = ratio * mean|out_img - target| (as
 * igs_raster_fwd_topk_tiles_l1) and the backward pass of that loss (as igs_raster_bwd_topk_tiles with v_output = the loss's gradient),
 * per tile back to back, so neither the top-K lists nor the image gradient are written. v_xy [N,2], v_conic [N,3], v_colors [N,C] are
 * zeroed and accumulated (float atomics); v_output [C,H,W] receives the image gradient when not null. workspace:
 * igs_raster_l1_workspace(tiles_x * tiles_y) bytes, 16-byte aligned. It replaces, for the L1 training step, the reference's
 * nd_rasterize_forward_topk_norm + F.l1_loss + nd_rasterize_backward_topk_norm (rasterize_sum.py:14-212 with model.py:1224-1227). */
int igs_raster_step_l1(int tiles_x, int tiles_y, int img_height, int img_width, int channels, int num_points,
                       const int32_t *gaussian_ids_sorted, const int32_t *tile_bins, const float *xys, const float *conics,
                       const float *colors, const float *target, float ratio, float *out_img, float *loss, float *v_output, float *v_xy,
                       float *v_conic, float *v_colors, void *workspace, size_t workspace_bytes, void *stream);

/* nd_rasterize_backward_topk_norm (bindings.cu:444-502, kernel backward.cu:187-335): v_output [C,H,W]; outputs v_xy [N,2],
 * v_conic [N,3], v_colors [N,C] are zeroed and accumulated (float atomics: the last bits vary run to run). IDs of pixel_topk outside
 * [0, N) count as empty slots (the reference reads out of bounds for IDs of N or more). */
int igs_raster_bwd_topk(int img_height, int img_width, int channels, int num_points, const float *xys, const float *conics,
                        const float *colors, const float *v_output, const int32_t *pixel_topk, float *v_xy, float *v_conic,
                        float *v_colors, void *stream);

/* The backward pass from igs_raster_fwd_topk_tiles' lists, with the same gaussian_ids_sorted / tile_bins. A list position at or past
 * the end of its tile's list counts as an empty slot. */
int igs_raster_bwd_topk_tiles(int img_height, int img_width, int channels, int num_points, const int32_t *gaussian_ids_sorted,
                              const int32_t *tile_bins, const float *xys, const float *conics, const float *colors, const float *v_output,
                              const uint16_t *tile_topk, float *v_xy, float *v_conic, float *v_colors, void *stream);

/* ---- the training step in one call (no counterpart in the reference, whose step is the sequence of the calls above: model.py:956-976,
 * 1224-1227 with gsplat's operators) --------------------------------------------------------------------------------------------- */

/* Workspace bytes of igs_train_step_l1 for `tile_rows` tile rows (the image's tiles_y, or a band's row_end - row_begin). */
size_t igs_train_step_workspace(int num_points, int capacity, int tiles_x, int tile_rows);
/* igs_project_fwd -> igs_cumsum -> igs_sort_intersects -> igs_raster_step_l1 -> igs_project_bwd for the tile rows [row_begin, row_end)
 * (the whole image: 0, tiles_y), with the stages' memsets and small passes folded into neighbouring kernels (eight kernels, no memset).
 * target and out_img hold those rows ([C, band rows, W]); tiles_hit counts the tiles of those rows (num_tiles_hit for the whole image);
 * tile_bins covers the band's tiles. v_xy, v_conic, v_colors are zeroed by the call and receive the band's gradients. With v_cov2d, v_mean2d,
 * v_scale, v_rot non-NULL the projection backward runs too and *loss is the loss; with them NULL (a band whose partials are then
 * combined across GPUs, e.g. by igs_band_reduce) *loss is the band's share. Workspace: igs_train_step_workspace, 256-byte aligned.
 * Outputs equal the per-stage calls' (the loss up to the order of its float sum). */
int igs_train_step_l1(int num_points, int channels, const float *means2d, const float *scales2d, const float *rotation, const float *colors,
                      const float *target, float ratio, int img_height, int img_width, int row_begin, int row_end, int capacity,
                      float *xys, int32_t *radii, float *conics, int32_t *tiles_hit, int32_t *cum_tiles_hit, int32_t *num_intersects,
                      int32_t *gaussian_ids_sorted, int32_t *tile_bins, float *out_img, float *loss, float *v_xy, float *v_conic,
                      float *v_colors, float *v_cov2d, float *v_mean2d, float *v_scale, float *v_rot, void *workspace,
                      size_t workspace_bytes, void *stream);

/* ---- tile-row bands (one image split over several GPUs; no counterpart in the reference, which renders on one GPU) ------------------ */

/* The tiles of rows [row_begin, row_end) that each Gaussian's rectangle covers: the band's num_tiles_hit, to prefix-sum for its binning */
int igs_band_tiles_hit(int num_points, const float *xys, const int32_t *radii, int tiles_x, int tiles_y, int row_begin, int row_end,
                       int32_t *num_tiles_hit, void *stream);

/* igs_raster_step_l1 over tile rows [row_begin, row_end): target, out_img and v_output hold the band's rows ([C, band rows, W]), tile_bins
 * and gaussian_ids_sorted come from igs_sort_intersects_band, and the loss is normalized by the whole image's C * H * W, so the bands'
 * losses and gradients add up to the whole image's. */
int igs_raster_step_l1_band(int tiles_x, int tiles_y, int img_height, int img_width, int row_begin, int row_end, int channels,
                            int num_points, const int32_t *gaussian_ids_sorted, const int32_t *tile_bins, const float *xys,
                            const float *conics, const float *colors, const float *target, float ratio, float *out_img, float *loss,
                            float *v_output, float *v_xy, float *v_conic, float *v_colors, void *workspace, size_t workspace_bytes,
                            void *stream);

/* igs_sort_intersects restricted to tile rows [row_begin, row_end): cum_tiles_hit is the prefix sum of igs_band_tiles_hit; tile_bins
 * [tiles_x * (row_end - row_begin), 2] numbers the band's tiles from its first row; workspace igs_sort_workspace(capacity, tiles_x,
 * row_end - row_begin). The lists equal the matching slice of the whole image's. */
int igs_sort_intersects_band(int num_points, int capacity, const float *xys, const int32_t *radii, const int32_t *cum_tiles_hit, int tiles_x,
                             int tiles_y, int row_begin, int row_end, int32_t *gaussian_ids_sorted, int32_t *tile_bins, void *workspace,
                             size_t workspace_bytes, void *stream);

/* igs_raster_fwd_topk_tiles for a band: out_band [C, band_h, W] with band_h = min(H, 16 row_end) - 16 row_begin, the band's tile lists;
 * pixel coordinates are the image's, so every value equals the whole image's. */
int igs_raster_fwd_topk_tiles_band(int tiles_x, int tiles_y, int img_height, int img_width, int row_begin, int row_end, int channels,
                                   int max_list_len, const int32_t *gaussian_ids_sorted, const int32_t *tile_bins, const float *xys,
                                   const float *conics, const float *colors, float *out_band, uint16_t *tile_topk, void *stream);

/* igs_raster_fwd_topk_tiles_l1 for a band: target and v_output hold the band's rows [C, band_h, W]; *loss is the band's share of the
 * whole image's loss (ratio * sum over the band of |image - target| / (C H W)), so the bands' losses sum to the image's; workspace
 * igs_raster_l1_workspace(tiles_x * (row_end - row_begin)). */
int igs_raster_fwd_topk_tiles_l1_band(int tiles_x, int tiles_y, int img_height, int img_width, int row_begin, int row_end, int channels,
                                      int max_list_len, const int32_t *gaussian_ids_sorted, const int32_t *tile_bins, const float *xys,
                                      const float *conics, const float *colors, const float *target, float ratio, float *out_img,
                                      uint16_t *tile_topk, float *loss, float *v_output, void *workspace, size_t workspace_bytes,
                                      void *stream);

/* igs_raster_bwd_topk_tiles for a band: v_output_band [C, band_h, W]; the gradients are this band's share (sum them over the bands) */
int igs_raster_bwd_topk_tiles_band(int img_height, int img_width, int row_begin, int row_end, int channels, int num_points,
                                   const int32_t *gaussian_ids_sorted, const int32_t *tile_bins, const float *xys, const float *conics,
                                   const float *colors, const float *v_output_band, const uint16_t *tile_topk, float *v_xy, float *v_conic,
                                   float *v_colors, void *stream);

/* ---- entropy coding of the bitstream (compress/rans_codec.py:93-124 over compress/csrc/rans.cpp:330-554; the container of
 * compress/__init__.py:104-156 is igs_b200/bitstream.py) ------------------------------------------------------------------------- */

#define IGS_RANS_MAX_TOKENS 4608   /* count codes per stream, at most */
#define IGS_RANS_MODEL_FIELDS 8    /* per stream: delta, zigzag_mapped, param, split_exp, msb_bits, mantissa_bits, number of codes, 0 */

/* Bytes that the payload of num_streams streams of `count` values cannot exceed. */
size_t igs_rans_payload_bound(int num_streams, int64_t count);
/* encode_streams: host arrays. streams [num_streams, count] int64; each stream is coded as its values or their differences, shifted to
 * its minimum or zigzagged around its rounded median, with the token model of the smallest estimated size, all with one rANS state;
 * the candidates are fitted on num_threads host threads (0: all). Outputs: the payload (little-endian 32-bit words), models
 * [num_streams, IGS_RANS_MODEL_FIELDS], codes [num_streams, IGS_RANS_MAX_TOKENS] (the first `number of codes` used) and each stream's
 * estimated payload bits; the bytes equal the reference's. */
int igs_rans_encode(int num_streams, int64_t count, const int64_t *streams, int num_threads, uint8_t *payload, size_t payload_capacity,
                    size_t *payload_bytes, int64_t *models, int64_t *codes, double *payload_bits);
/* decode_streams: host arrays. models and codes as igs_rans_encode writes them (only split_exp, msb_bits, mantissa_bits and the codes
 * are read: the mapping and differences are undone by the caller); values [num_streams, count] the mapped values. */
int igs_rans_decode(int num_streams, int64_t count, const int64_t *models, const int64_t *codes, const uint8_t *payload,
                    size_t payload_size, int64_t *values);
/* estimate_stream_bits (compress/rans_codec.py:83-90) of num_streams device streams [num_streams, count] int64 into bits [num_streams]
 * (host): the histograms of their tokens on the GPU, the reference's formula on the host (synchronizes the stream). Workspace:
 * igs_estimate_bits_workspace bytes, 16-byte aligned. */
size_t igs_estimate_bits_workspace(int num_streams);
int igs_estimate_stream_bits(int num_streams, int64_t count, const int64_t *streams, double *bits, void *workspace, size_t workspace_bytes,
                             void *stream);

/* ---- the bands' gradient exchange over peer memory (NVLink / NVSwitch; one process per GPU of one machine; no counterpart in the
 * reference) ------------------------------------------------------------------------------------------------------------------------ */

#define IGS_MAX_BAND_RANKS 8
#define IGS_IPC_HANDLE_BYTES 64
#define IGS_BAND_SYNC_WORDS 32     /* uint32 words of a rank's synchronisation block (igs_band_sync_bytes) */
#define IGS_BAND_SYNC_STEP 16      /* word index: exchanges this rank has completed */
#define IGS_BAND_SYNC_ERROR 17     /* word index: nonzero once a wait gave up (IGS_BAND_TIMEOUT_* bits); later exchanges do nothing */
#define IGS_BAND_TIMEOUT_READY 1u  /* a rank's partials did not arrive in time */
#define IGS_BAND_TIMEOUT_DONE 2u   /* a rank's share of the results did not arrive in time */

/* A CUDA IPC handle (IGS_IPC_HANDLE_BYTES bytes) for the device allocation that holds dev_ptr, and dev_ptr's offset in it: an allocation
 * is exported whole, so any buffer inside one (a tensor of a caching allocator) can be shared. */
int igs_ipc_export(const void *dev_ptr, void *handle, uint64_t *offset);
/* Map another process's buffer (igs_ipc_export's handle and offset) on the current device, with peer access; *dev_ptr is the buffer's
 * address here. Opening an allocation again returns the same mapping (reference-counted by CUDA); igs_ipc_close undoes one open. */
int igs_ipc_open(const void *handle, uint64_t offset, void **dev_ptr);
int igs_ipc_close(void *dev_ptr, uint64_t offset);

/* Bytes of a rank's synchronisation block (zero it once before the first exchange; 16-byte aligned) and floats of its results buffer:
 * v_cov2d [N,3], v_mean2d [N,2], v_scale [N,2], v_rot [N], v_colors [N,C] (summed over the bands), loss [1]. */
size_t igs_band_sync_bytes(void);
size_t igs_band_results_floats(int num_points, int channels);

/* The exchange that ends a band step, after igs_raster_step_l1_band (or the band's forward and backward) on every rank, in place of an
 * all-reduce of the partials followed by igs_project_bwd on every rank. partials[q] is rank q's [N (5 + C) + 1] buffer (v_xy, v_conic,
 * v_colors, loss: what the band kernels wrote), results[q] its results buffer, sync[q] its synchronisation block; entry `rank` is this
 * rank's own memory, the others are peers' buffers mapped with igs_ipc_open (world <= IGS_MAX_BAND_RANKS). This rank announces that its
 * partials are complete, waits for every rank's, sums the partials of its share of the Gaussians [N rank / world, N (rank + 1) / world)
 * in rank order, runs the projection backward on them (igs_project_bwd's arithmetic) and stores the results into every rank's results
 * buffer, adds the partial losses into its own, then announces and waits until every rank has stored its share. Every rank then holds
 * the same complete results. A wait longer than timeout_ms sets bits in the rank's error word (IGS_BAND_SYNC_ERROR) instead of hanging
 * the GPU; that step's results are invalid and later exchanges do nothing. Each rank's call must be on its own GPU. */
int igs_band_reduce(int world, int rank, int num_points, int channels, const float *const *partials, float *const *results,
                    void *const *sync, const float *scales2d, const float *rotation, int img_height, int img_width, const int32_t *radii,
                    const float *conics, int timeout_ms, void *stream);

/* topk_norm_loo_loss_increase (bindings.cu:895-936, kernel forward.cu:667-738): per Gaussian, the increase of the absolute (squared
 * when `squared`) error summed over pixels and channels when it alone leaves the top-K lists; targets [C,H,W]. IDs of N or more count
 * as empty slots. */
int igs_loo_loss_increase(int img_height, int img_width, int channels, int num_points, const float *xys, const float *conics,
                          const float *colors, const int32_t *pixel_topk, const float *targets, int squared, float eps,
                          float *loss_increase, void *stream);

/* feature_weights over _iter_topk_weights (compress/quantization.py:218-230, model.py:1404-1421): per Gaussian, the sum over pixels of
 * its squared normalized top-K weight as 64-bit fixed point with 40 fractional bits (fixed_point [N] int64, zeroed here; the weights are
 * fixed_point / 2^40). The slot weights exp(-sigma) are recomputed with the reference's IEEE float32 arithmetic from pixel_topk [H,W,10]
 * (of igs_raster_fwd_topk), normalized in double with eps (1e-4 in the reference) and rounded half to even; integer atomics make the sums
 * independent of the order of the additions. IDs outside [0, N) count as empty slots. */
int igs_feature_weights(int img_height, int img_width, int num_points, const float *xys, const float *conics, const int32_t *pixel_topk,
                        double eps, int64_t *fixed_point, void *stream);

/* nearest_neighbors / causal_neighbors of the rate model's preparation (compress/csrc/prediction.cpp:69-166, called by
 * compress/rate.py:56-66 bitstream_neighbors): for integer positions [P, 2] (int64, 16-byte aligned), the 8 nearest earlier Gaussians
 * (causal != 0: indices below the Gaussian's own, i.e. earlier in bitstream order) or the 8 nearest other Gaussians, ordered by squared
 * distance and then by index; neighbors [P, 8] int64 and, unless null, dist2 [P, 8] int64, -1 where there are fewer. workspace:
 * igs_neighbors_workspace(P) bytes, 16-byte aligned. Nothing is read back to the host. */
size_t igs_neighbors_workspace(int num_points);
int igs_nearest_neighbors(int num_points, const int64_t *positions, int causal, int64_t *neighbors, int64_t *dist2, void *workspace,
                          size_t workspace_bytes, void *stream);

/* ---- training-step losses and quantization -------------------------------------------------------------------------------------- */

/* L1 loss and its gradient in one pass (model.py:1224-1227, F.l1_loss): loss = ratio * mean|image - target| (device scalar) and
 * grad = ratio * sign(image - target) / numel. Deterministic (fixed-order block sums). partials: igs_l1_workspace bytes. */
size_t igs_l1_workspace(int64_t numel);
int igs_l1_loss(int64_t numel, const float *image, const float *target, float ratio, float *loss, float *grad, void *workspace,
                size_t workspace_bytes, void *stream);

/* The same loss keeping sign(image - target) (int8: -1, 0, 1) instead of the gradient, for autograd (F.l1_loss, model.py:1226): the
 * backward pass then forms grad = sign * (g / numel) with igs_l1_grad_from_signs from the loss's incoming gradient g (a device scalar;
 * null for 1), which is ATen's l1_loss backward product bit for bit. workspace as igs_l1_loss. */
int igs_l1_loss_signs(int64_t numel, const float *image, const float *target, float ratio, float *loss, int8_t *signs, void *workspace,
                      size_t workspace_bytes, void *stream);
int igs_l1_grad_from_signs(int64_t numel, const int8_t *signs, const float *grad_scale, float *grad, void *stream);

/* Straight-through "step" quantization of the Gaussian parameters during optimization (model.py:993-1006 with
 * compress/quantization.py:36-46,61-74,151-172,188-199; quarter turns off, log-domain scales): symbols
 * q_xy = round(xy / pos_steps), q_scale = round(log2|scale| / scale_step), q_rot = round(rot / rot_step), q_feat = round(feat / feat_steps)
 * (round half to even, IEEE division), and forward values x + (dequantize(q) - x) with dequantize(q_scale) = exp2(q_scale * scale_step).
 * xy [N,2], scale [N,2] (pixels), rot [N], feat [N,C]; pos_steps [2], feat_steps [C] device arrays. Symbol outputs may be NULL.
 * feat_transform (may be NULL): a [C,C] matrix T; then out_feat_t [N,C] = out_feat T^T as well (model.py:963-964, YUV loss space). */
int igs_quantize_ste(int num_points, int channels, const float *xy, const float *scale, const float *rot, const float *feat,
                     const float *pos_steps, float scale_step, float rot_step, const float *feat_steps, const float *feat_transform,
                     float *out_xy, float *out_scale, float *out_rot, float *out_feat, float *out_feat_t, float *q_xy, float *q_scale,
                     float *q_rot, float *q_feat, void *stream);

/* Backward of the loss-space feature transform (autograd of `feat @ loss_transform.T`, model.py:963-964) through the straight-through
 * quantizer: v_feat [N,C] = v_feat_t [N,C] T [C,C] + v_extra (may be NULL; e.g. the rate term's feature gradient). */
int igs_feat_transform_bwd(int num_points, int channels, const float *v_feat_t, const float *feat_transform, const float *v_extra,
                           float *v_feat, void *stream);

/* bitstream_order (compress/__init__.py:43-58): the order of the Gaussians along the Morton curve of their integer positions [P, 2] (int64,
 * 16-byte aligned) coarsened by refine_bits, ties by the Morton code of the full positions, then by index; order [P] int64. Reads the
 * positions' range back once (the call synchronizes the stream: not for CUDA-graph capture). Positions spanning 2^32 coarse levels or more
 * are rejected (IGS_ERR_INVALID, as the reference rejects them); a key wider than 64 bits (coordinates spanning more than about 2^16 coarse
 * and fine levels together) returns IGS_ERR_UNSUPPORTED for a host sort. Workspace: igs_bitstream_order_workspace bytes, 256-byte
 * aligned. */
size_t igs_bitstream_order_workspace(int num_points);
int igs_bitstream_order(int num_points, const int64_t *positions, int refine_bits, int64_t *order, void *workspace, size_t workspace_bytes,
                        void *stream);

/* rate_model (compress/rate.py:131-164, with predicting_sources 116-128): the fixed inputs of the rate term from the quantized Gaussians,
 * on the GPU. Inputs (device): neighbors [P,8] int64 (the bitstream-order neighbours of igs_nearest_neighbors mapped back to the
 * Gaussians' order, -1 for none), feat [P,C] the dequantized features, log2_scale [P,2] the dequantized log2 scales, q_rot [P] the rotation
 * indices (integer values), steps [C] the feature steps (> 0), channel_weights [C]; color_refs and pred_refs [C] (host) as
 * compress.quantization.get_channel_refs and compress.prediction.get_prediction_refs give them (-1 for none). Outputs (device):
 * neighbors_out [P,8] int32 (clamped to 0), weights [P,8], slope [P,C], inv_steps [C], inv_feat [C], feat_coeffs [C], inv_rot [P],
 * offsets [P+1] int32, sources [<= 8P] int32 and source_weights [<= 8P] (offsets[P] of them). Workspace: igs_rate_model_workspace bytes,
 * 16-byte aligned. Float operations follow the reference's float32 order; the means of the rounded residuals and rotation indices are
 * exact integer sums. */
size_t igs_rate_model_workspace(int num_points);
int igs_rate_model(int num_points, int channels, const int64_t *neighbors, const float *feat, const float *log2_scale, const float *q_rot,
                   const int32_t *color_refs, const int32_t *pred_refs, const float *steps, const float *channel_weights,
                   int32_t *neighbors_out, float *weights, float *slope, float *inv_steps, float *inv_feat, float *feat_coeffs,
                   float *inv_rot, int32_t *offsets, int32_t *sources, float *source_weights, void *workspace, size_t workspace_bytes,
                   void *stream);

/* rate_loss_forward (gsplat/gsplat/cuda/csrc/rate.cu:201-279; definition compress/rate.py:167-175 rate_bits): loss (device scalar)
 * = factor / max(l1_loss / l1_ratio, 1e-4) * (sum_{g,c} feat_coeffs[c] (sqrt(r^2 + 1/4) - 1/2) + sum_g rot_coeffs[g] (sqrt(t^2 + 1/4) - 1/2)),
 * own_grad [N,C] and rot_grad [N] for the backward pass. color_refs / pred_refs: C host integers each. neighbors [N,K] int32.
 * Workspace: igs_rate_workspace bytes (per-block bit sums). */
size_t igs_rate_workspace(int num_gaussians);
int igs_rate_fwd(int num_gaussians, int channels, int num_neighbors, const float *feat, const float *rot, const float *l1_loss,
                 const int32_t *neighbors, const float *weights, const float *slope, const int32_t *color_refs, const int32_t *pred_refs,
                 const float *inv_steps, const float *feat_coeffs, const float *rot_coeffs, float inv_rot_step, float l1_ratio,
                 float factor, float *loss, float *loss_weight, float *own_grad, float *rot_grad, void *workspace, size_t workspace_bytes,
                 void *stream);

/* rate_loss_backward (rate.cu:281-321): grad_feat [N,C], grad_rot [N] from the forward's own gradients and the CSR list of the
 * Gaussians that predict from each one (offsets [N+1], sources [E], source_weights [E]). Deterministic, no atomics. */
int igs_rate_bwd(int num_gaussians, int channels, const float *grad_loss, const float *loss_weight, const float *own_grad,
                 const float *rot_grad, const int32_t *offsets, const int32_t *sources, const float *source_weights, float *grad_feat,
                 float *grad_rot, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* IGS_B200_H */
