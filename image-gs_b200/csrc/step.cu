// The rasterization training step of one image, or of one band of tile rows, as one C-ABI call (igs_train_step_l1): the chain of
// igs_project_fwd -> igs_cumsum -> igs_sort_intersects -> igs_raster_step_l1 -> igs_project_bwd with the per-stage calls' memsets and
// small passes folded into the neighbouring kernels:
//   project_step_kernel:  projection, tiles hit (of the band's rows), one partial sum per 256 Gaussians, the gradient accumulators and
//                         the per-tile counters zeroed                                      (replaces igs_project_fwd, the first pass
//                                                                                            of igs_cumsum and two memsets)
//   cumsum_scan_kernel:   the prefix sum from those partial sums
//   count, tile scan, place, order: the binning (igs_sort_intersects without its memset)
//   raster_step_kernel:   top-K forward, L1 loss, top-K backward per tile
//   project_bwd_kernel:   the projection backward, its last block adding up the loss          (replaces l1_finish_kernel)
// Eight kernels instead of ten kernels and two memsets, all launched with programmatic dependent launch. Outputs equal the per-stage
// calls' (the loss up to the order of its float sum).
#include <algorithm>

#include "igs_common.cuh"
#include "igs_internal.cuh"

namespace {

size_t round256(size_t b) { return (b + 255) & ~(size_t)255; }

// workspace layout: per-256-Gaussian partial sums of the tiles hit, the raster kernel's per-tile loss partials, the binning's workspace
struct StepWorkspace {
    size_t l1_offset, sort_offset, l1_bytes, sort_bytes;
    StepWorkspace(int num_points, int capacity, int tiles_x, int tile_rows) {
        l1_offset = round256(sizeof(unsigned) * (size_t)std::max(1, igs::ceil_div(std::max(num_points, 0), 256)));
        l1_bytes = igs_raster_l1_workspace(tiles_x * tile_rows);
        sort_offset = l1_offset + round256(l1_bytes);
        sort_bytes = igs_sort_workspace(capacity, tiles_x, tile_rows);
    }
    size_t total() const { return sort_offset + sort_bytes; }
};

}  // namespace

extern "C" {

size_t igs_train_step_workspace(int num_points, int capacity, int tiles_x, int tile_rows) {
    return StepWorkspace(num_points, capacity, tiles_x, tile_rows).total();
}

int igs_train_step_l1(int num_points, int channels, const float *means2d, const float *scales2d, const float *rotation, const float *colors,
                      const float *target, float ratio, int img_height, int img_width, int row_begin, int row_end, int capacity,
                      float *xys, int32_t *radii, float *conics, int32_t *tiles_hit, int32_t *cum_tiles_hit, int32_t *num_intersects,
                      int32_t *gaussian_ids_sorted, int32_t *tile_bins, float *out_img, float *loss, float *v_xy, float *v_conic,
                      float *v_colors, float *v_cov2d, float *v_mean2d, float *v_scale, float *v_rot, void *workspace,
                      size_t workspace_bytes, void *stream) {
    const char *who = "igs_train_step_l1";
    IGS_REQUIRE(num_points >= 0 && img_height >= 0 && img_width >= 0, "%s: negative size", who);
    IGS_REQUIRE(channels >= 1 && channels <= igs::kMaxChannels, "%s: 1 to %d channels (got %d)", who, igs::kMaxChannels, channels);
    const int tiles_x = igs::ceil_div(img_width, igs::kTile), tiles_y = igs::ceil_div(img_height, igs::kTile);
    IGS_REQUIRE(row_begin >= 0 && row_begin <= row_end && row_end <= tiles_y, "%s: tile rows [%d, %d) outside [0, %d)", who, row_begin,
                row_end, tiles_y);
    IGS_REQUIRE(capacity >= 1, "%s: the intersection capacity must be positive", who);
    IGS_REQUIRE(num_intersects && gaussian_ids_sorted && tile_bins && loss && workspace, "%s: null pointer", who);
    IGS_REQUIRE(num_points == 0 || (means2d && scales2d && rotation && colors && xys && radii && conics && tiles_hit && cum_tiles_hit &&
                                    v_xy && v_conic && v_colors),
                "%s: null pointer", who);
    IGS_REQUIRE(num_points == 0 || (igs::aligned(means2d, 8) && igs::aligned(scales2d, 8) && igs::aligned(xys, 8) && igs::aligned(v_xy, 8)),
                "%s: [N, 2] arrays must be 8-byte aligned", who);
    const bool backward = v_cov2d != nullptr;
    IGS_REQUIRE(!backward || (v_mean2d && v_scale && v_rot), "%s: null projection gradient pointer", who);
    IGS_REQUIRE(igs::aligned(workspace, 256), "%s: workspace must be 256-byte aligned", who);
    const int rows = row_end - row_begin;
    IGS_REQUIRE(workspace_bytes >= igs_train_step_workspace(num_points, capacity, tiles_x, rows), "%s: workspace too small (%zu < %zu)",
                who, workspace_bytes, igs_train_step_workspace(num_points, capacity, tiles_x, rows));
    cudaStream_t s = igs::as_stream(stream);
    const StepWorkspace layout(num_points, capacity, tiles_x, rows);
    char *base = static_cast<char *>(workspace);
    struct {
        unsigned *block_sums;
        float *l1_partials;
        void *sort;
        size_t l1_bytes, sort_bytes;
    } w{reinterpret_cast<unsigned *>(base), reinterpret_cast<float *>(base + layout.l1_offset), base + layout.sort_offset, layout.l1_bytes,
        layout.sort_bytes};

    igs::StepZeroing zero{reinterpret_cast<float2 *>(v_xy), v_conic, v_colors, channels, igs::tile_counters(w.sort), tiles_x * rows};
    int status = igs::project_step(num_points, means2d, scales2d, rotation, img_height, img_width, tiles_x, tiles_y, row_begin, row_end, xys,
                                   radii, conics, tiles_hit, w.block_sums, zero, s);
    if (status != IGS_OK) return status;
    status = igs::cumsum_from_block_sums(num_points, tiles_hit, w.block_sums, cum_tiles_hit, num_intersects, s);
    if (status != IGS_OK) return status;
    status = igs::sort_band_counters_zeroed(num_points, capacity, xys, radii, cum_tiles_hit, tiles_x, tiles_y, row_begin, row_end,
                                            gaussian_ids_sorted, tile_bins, w.sort, w.sort_bytes, s);
    if (status != IGS_OK) return status;
    status = igs::raster_step_fused(tiles_x, tiles_y, img_height, img_width, row_begin, row_end, channels, num_points, gaussian_ids_sorted,
                                    tile_bins, xys, conics, colors, target, ratio, out_img, loss, v_xy, v_conic, v_colors, w.l1_partials,
                                    w.l1_bytes, !backward, s);
    if (status != IGS_OK || !backward) return status;
    const float numel = (float)((int64_t)channels * img_height * img_width);
    return igs::project_bwd_finish(num_points, scales2d, rotation, img_height, img_width, radii, conics, v_xy, v_conic, v_cov2d, v_mean2d,
                                   v_scale, v_rot, igs::LossFinish{w.l1_partials, tiles_x * rows, ratio, numel, loss}, s);
}

}  // extern "C"
