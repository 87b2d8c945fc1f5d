// Internal launchers shared between the library's files for the fused training step (step.cu, igs_train_step_l1): variants of the
// per-stage kernels that absorb the step's memsets and small passes into their neighbours, so that the step is a chain of kernels
// linked by programmatic dependent launch with no memset node between them. Not part of the C ABI.
#pragma once

#include "igs_common.cuh"

namespace igs {

// What the step's projection kernel zeroes besides projecting: the Gaussians' gradient accumulators (v_xy [N,2], v_conic [N,3],
// v_colors [N,C]) and the binning's per-tile counters
struct StepZeroing {
    float2 *v_xy;
    float *v_conic;
    float *v_colors;
    int channels;
    int *counters;
    int num_counters;
};

// The loss from the raster kernel's per-tile partial sums, formed by the last block of the projection backward: ratio * sum / numel
struct LossFinish {
    const float *partials;
    int count;
    float ratio;
    float numel;
    float *loss;
};

// project.cu: the projection with the tiles hit counted over tile rows [row_begin, row_end), one sum of them per block of 256 Gaussians
// (block_sums [ceil(n / 256)]), and the zeroing above
int project_step(int n, const float *means2d, const float *scales2d, const float *rotation, int img_height, int img_width, int tiles_x,
                 int tiles_y, int row_begin, int row_end, float *xys, int32_t *radii, float *conics, int32_t *tiles_hit,
                 unsigned *block_sums, const StepZeroing &zero, cudaStream_t s);

// project.cu: igs_project_bwd with the loss finished by its last block
int project_bwd_finish(int n, const float *scales2d, const float *rotation, int img_height, int img_width, const int32_t *radii,
                       const float *conics, const float *v_xy, const float *v_conic, float *v_cov2d, float *v_mean2d, float *v_scale,
                       float *v_rot, const LossFinish &finish, cudaStream_t s);

// binning.cu: the inclusive prefix sum of tiles_hit from project_step's block sums (one pass)
int cumsum_from_block_sums(int n, const int32_t *tiles_hit, const unsigned *block_sums, int32_t *cum, int32_t *total, cudaStream_t s);

// binning.cu: igs_sort_intersects_band with the per-tile counters (the first igs_sort_workspace region, tile_counters()) already zero
int sort_band_counters_zeroed(int num_points, int capacity, const float *xys, const int32_t *radii, const int32_t *cum_tiles_hit,
                              int tiles_x, int tiles_y, int row_begin, int row_end, int32_t *gaussian_ids_sorted, int32_t *tile_bins,
                              void *workspace, size_t workspace_bytes, cudaStream_t s);
int *tile_counters(void *sort_workspace);

// raster.cu: igs_raster_step_l1_band with the gradient accumulators already zero; finish_loss false leaves the loss to the caller (the
// per-tile partials in the workspace, LossFinish)
int raster_step_fused(int tiles_x, int tiles_y, int img_h, int img_w, int row_begin, int row_end, int channels, int num_points,
                      const int32_t *ids_sorted, const int32_t *tile_bins, const float *xys, const float *conics, const float *colors,
                      const float *target, float ratio, float *out_img, float *loss, float *v_xy, float *v_conic, float *v_colors,
                      void *workspace, size_t workspace_bytes, bool finish_loss, cudaStream_t s);

}  // namespace igs
