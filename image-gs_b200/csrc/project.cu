// 2D projection of the Gaussians: pixel centers, conics (inverse covariances), 3-sigma radii and tile footprints, and the backward pass to
// means, scales and rotations. Compiled with --use_fast_math like the reference extension (gsplat/setup.py:70), because the radius
// ceil(3 sqrt(lambda_max)) and the tile bounding box decide the tile binning, which must agree with the reference bit for bit: the same
// approximate sqrt / reciprocal / sin / cos and the same product order (glm's mat2 product, which the M2 helper of project_math.cuh reproduces so
// that the compiler contracts the same multiply-adds).
//
// One thread per Gaussian, parameters read as float2 vectors; every output element is written (the reference relies on zero-initialized
// outputs instead), so callers need no memset.
#include <algorithm>

#include "igs_common.cuh"
#include "igs_internal.cuh"
#include "project_math.cuh"

namespace {

using igs::diag;
using igs::kTile;
using igs::M2;
using igs::mul;
using igs::projection_grad;
using igs::ProjectionGrad;
using igs::rotation;
using igs::transpose;

// Tile rectangle [x0, x1) x [y0, y1) covered by a pixel center and radius, clamped to the grid (helpers.cuh:11-43)
__device__ __forceinline__ void tile_rect(float cx, float cy, float radius, unsigned tiles_x, unsigned tiles_y, unsigned &x0, unsigned &y0,
                                          unsigned &x1, unsigned &y1) {
    const float tcx = cx / (float)kTile, tcy = cy / (float)kTile;
    const float trx = radius / (float)kTile, try_ = radius / (float)kTile;
    x0 = min((unsigned)max(0, (int)(tcx - trx)), tiles_x);
    x1 = min((unsigned)max(0, (int)(tcx + trx + 1)), tiles_x);
    y0 = min((unsigned)max(0, (int)(tcy - try_)), tiles_y);
    y1 = min((unsigned)max(0, (int)(tcy + try_ + 1)), tiles_y);
}

// One Gaussian's projection: pixel center, conic, radius and tile rectangle (valid false where the covariance is singular)
struct Projected {
    float2 xy;
    float conic[3];
    int radius;
    unsigned x0, y0, x1, y1;
    bool valid;
};

__device__ __forceinline__ Projected project_one(const float2 mean, const float2 scale, const float theta, const float img_w,
                                                 const float img_h, const unsigned tiles_x, const unsigned tiles_y) {
    Projected p;
    const float cx = mean.x * img_w, cy = mean.y * img_h;
    const M2 R = rotation(cosf(theta), sinf(theta));
    const M2 M = mul(R, diag(scale.x, scale.y));
    const M2 cov = mul(M, transpose(M));
    const float a = cov.m[0][0], b = cov.m[0][1], c = cov.m[1][1];
    const float det = a * c - b * b;
    p.xy = make_float2(0.f, 0.f);
    p.conic[0] = p.conic[1] = p.conic[2] = 0.f;
    p.radius = 0;
    p.x0 = p.y0 = p.x1 = p.y1 = 0u;
    p.valid = det != 0.f;
    if (p.valid) {
        const float inv_det = 1.f / det;
        p.conic[0] = c * inv_det;
        p.conic[1] = -b * inv_det;
        p.conic[2] = a * inv_det;
        const float mid = 0.5f * (a + c);
        const float spread = sqrtf(fmaxf(0.1f, mid * mid - det));
        const float radius = ceilf(3.f * sqrtf(fmaxf(mid + spread, mid - spread)));
        p.xy = make_float2(cx, cy);
        p.radius = (int)radius;
        tile_rect(cx, cy, radius, tiles_x, tiles_y, p.x0, p.y0, p.x1, p.y1);
    }
    return p;
}

__global__ void __launch_bounds__(256) project_fwd_kernel(const int n, const float2 *__restrict__ means, const float2 *__restrict__ scales,
                                                          const float *__restrict__ rotations, const float img_w, const float img_h,
                                                          const unsigned tiles_x, const unsigned tiles_y, float2 *__restrict__ xys,
                                                          int *__restrict__ radii, float *__restrict__ conics, int *__restrict__ hits) {
    igs::wait_for_predecessor();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const Projected p = project_one(__ldg(&means[i]), __ldg(&scales[i]), __ldg(&rotations[i]), img_w, img_h, tiles_x, tiles_y);
    int tiles_hit = 0;
    if (p.valid) {
        const int area = (int)((p.x1 - p.x0) * (p.y1 - p.y0));
        tiles_hit = area > 0 ? area : 0;
    }
    xys[i] = p.xy;
    radii[i] = p.radius;
    conics[3 * i + 0] = p.conic[0];
    conics[3 * i + 1] = p.conic[1];
    conics[3 * i + 2] = p.conic[2];
    hits[i] = tiles_hit;
}

constexpr int kStepThreads = 256;

// The training step's projection (igs_train_step_l1): project_fwd_kernel's outputs with the tiles hit counted in tile rows
// [row_begin, row_end) only, plus the work of the step's first memsets and first prefix-sum pass: each block's sum of the tiles hit
// (block_sums, for cumsum_from_block_sums), the Gaussian's gradient accumulators zeroed (the raster kernel adds into them) and the
// per-tile counters of the binning zeroed
__global__ void __launch_bounds__(kStepThreads) project_step_kernel(const int n, const float2 *__restrict__ means,
                                                                    const float2 *__restrict__ scales, const float *__restrict__ rotations,
                                                                    const float img_w, const float img_h, const unsigned tiles_x,
                                                                    const unsigned tiles_y, const unsigned row_begin, const unsigned row_end,
                                                                    float2 *__restrict__ xys, int *__restrict__ radii,
                                                                    float *__restrict__ conics, int *__restrict__ hits,
                                                                    unsigned *__restrict__ block_sums, const igs::StepZeroing zero) {
    igs::wait_for_predecessor();
    __shared__ unsigned warp_sums[kStepThreads / 32];
    const int i = blockIdx.x * kStepThreads + threadIdx.x;
    unsigned tiles_hit = 0u;
    if (i < n) {
        const Projected p = project_one(__ldg(&means[i]), __ldg(&scales[i]), __ldg(&rotations[i]), img_w, img_h, tiles_x, tiles_y);
        if (p.valid) {
            const unsigned y0 = max(p.y0, row_begin), y1 = min(p.y1, row_end);
            if (y1 > y0 && p.x1 > p.x0) tiles_hit = (p.x1 - p.x0) * (y1 - y0);
        }
        xys[i] = p.xy;
        radii[i] = p.radius;
        conics[3 * i + 0] = p.conic[0];
        conics[3 * i + 1] = p.conic[1];
        conics[3 * i + 2] = p.conic[2];
        hits[i] = (int)tiles_hit;
        zero.v_xy[i] = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 3; ++k) zero.v_conic[3 * (size_t)i + k] = 0.f;
        for (int c = 0; c < zero.channels; ++c) zero.v_colors[(size_t)i * zero.channels + c] = 0.f;
    }
    for (int t = i; t < zero.num_counters; t += gridDim.x * kStepThreads) zero.counters[t] = 0;
    unsigned v = tiles_hit;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned total = 0u;
#pragma unroll
        for (int w = 0; w < kStepThreads / 32; ++w) total += warp_sums[w];
        block_sums[blockIdx.x] = total;
    }
}

// Backward of the projection, the reference's formula (backward2d.cu:53-100, helpers.cuh:71-82) term by term: v_cov2d = -X G X with the
// conic X and G built from v_conic (its off-diagonal used as is), v_scale and v_rot contract v_cov2d with dSigma/ds and dSigma/dtheta
// weighting the off-diagonal by 2, v_mean2d = v_xy (W, H). Gaussians with radius <= 0 get zeros.
template <bool kFinish>
__global__ void __launch_bounds__(256) project_bwd_kernel(const int n, const float2 *__restrict__ scales, const float *__restrict__ rotations,
                                                          const float img_w, const float img_h, const int *__restrict__ radii,
                                                          const float *__restrict__ conics, const float2 *__restrict__ v_xy,
                                                          const float *__restrict__ v_conic, float *__restrict__ v_cov2d,
                                                          float2 *__restrict__ v_mean2d, float2 *__restrict__ v_scale,
                                                          float *__restrict__ v_rot, const igs::LossFinish finish) {
    igs::wait_for_predecessor();
    if (kFinish && blockIdx.x == gridDim.x - 1) {
        // the training step's loss from the raster kernel's per-tile partial sums, in a fixed order: ratio * (sum) / numel
        __shared__ float warp_sums[8];
        float sum = 0.f;
        int t0 = 0;
        if ((reinterpret_cast<uintptr_t>(finish.partials) & 15) == 0) {
            // four partials per load, several loads in flight per thread (the sum's order stays fixed)
            const float4 *p4 = reinterpret_cast<const float4 *>(finish.partials);
            const int n4 = finish.count / 4;
#pragma unroll 4
            for (int t = threadIdx.x; t < n4; t += 256) {
                const float4 v = __ldg(&p4[t]);
                sum += (v.x + v.y) + (v.z + v.w);
            }
            t0 = 4 * n4;
        }
        for (int t = t0 + threadIdx.x; t < finish.count; t += 256) sum += __ldg(&finish.partials[t]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = sum;
        __syncthreads();
        if (threadIdx.x == 0) {
            float all = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) all += warp_sums[w];
            *finish.loss = finish.ratio * (all / finish.numel);
        }
    }
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (__ldg(&radii[i]) <= 0) {
        v_cov2d[3 * i + 0] = 0.f;
        v_cov2d[3 * i + 1] = 0.f;
        v_cov2d[3 * i + 2] = 0.f;
        v_mean2d[i] = make_float2(0.f, 0.f);
        v_scale[i] = make_float2(0.f, 0.f);
        v_rot[i] = 0.f;
        return;
    }
    const ProjectionGrad pg = projection_grad(__ldg(&scales[i]), __ldg(&rotations[i]), img_w, img_h, conics + 3 * i, v_conic + 3 * i,
                                              v_xy[i]);
    v_cov2d[3 * i + 0] = pg.cov2d[0];
    v_cov2d[3 * i + 1] = pg.cov2d[1];
    v_cov2d[3 * i + 2] = pg.cov2d[2];
    v_scale[i] = pg.scale;
    v_rot[i] = pg.rot;
    v_mean2d[i] = pg.mean2d;
}

}  // namespace

extern "C" {

int igs_project_fwd(int num_points, const float *means2d, const float *scales2d, const float *rotation, int img_height, int img_width,
                    int tiles_x, int tiles_y, float *xys, int32_t *radii, float *conics, int32_t *num_tiles_hit, void *stream) {
    IGS_REQUIRE(num_points >= 0 && img_height >= 0 && img_width >= 0 && tiles_x >= 0 && tiles_y >= 0, "igs_project_fwd: negative size");
    if (num_points == 0) return IGS_OK;
    IGS_REQUIRE(means2d && scales2d && rotation && xys && radii && conics && num_tiles_hit, "igs_project_fwd: null pointer");
    IGS_REQUIRE(igs::aligned(means2d, 8) && igs::aligned(scales2d, 8) && igs::aligned(xys, 8),
                "igs_project_fwd: means2d, scales2d and xys must be 8-byte aligned [N, 2] float32");
    igs::launch(project_fwd_kernel, igs::ceil_div(num_points, 256), 256, 0, igs::as_stream(stream), num_points,
                reinterpret_cast<const float2 *>(means2d), reinterpret_cast<const float2 *>(scales2d), rotation, (float)img_width,
                (float)img_height, (unsigned)tiles_x, (unsigned)tiles_y, reinterpret_cast<float2 *>(xys), radii, conics, num_tiles_hit);
    return igs::check_launch("igs_project_fwd");
}

int igs_project_bwd(int num_points, const float *scales2d, const float *rotation, int img_height, int img_width, const int32_t *radii,
                    const float *conics, const float *v_xy, const float *v_conic, float *v_cov2d, float *v_mean2d, float *v_scale,
                    float *v_rot, void *stream) {
    IGS_REQUIRE(num_points >= 0, "igs_project_bwd: negative size");
    if (num_points == 0) return IGS_OK;
    IGS_REQUIRE(scales2d && rotation && radii && conics && v_xy && v_conic && v_cov2d && v_mean2d && v_scale && v_rot,
                "igs_project_bwd: null pointer");
    IGS_REQUIRE(igs::aligned(scales2d, 8) && igs::aligned(v_xy, 8) && igs::aligned(v_mean2d, 8) && igs::aligned(v_scale, 8),
                "igs_project_bwd: [N, 2] tensors must be 8-byte aligned");
    igs::launch(project_bwd_kernel<false>, igs::ceil_div(num_points, 256), 256, 0, igs::as_stream(stream), num_points,
                reinterpret_cast<const float2 *>(scales2d), rotation, (float)img_width, (float)img_height, radii, conics,
                reinterpret_cast<const float2 *>(v_xy), v_conic, v_cov2d, reinterpret_cast<float2 *>(v_mean2d),
                reinterpret_cast<float2 *>(v_scale), v_rot, igs::LossFinish{});
    return igs::check_launch("igs_project_bwd");
}

}  // extern "C"

namespace igs {

int project_step(int n, const float *means2d, const float *scales2d, const float *rotation, int img_height, int img_width, int tiles_x,
                 int tiles_y, int row_begin, int row_end, float *xys, int32_t *radii, float *conics, int32_t *tiles_hit,
                 unsigned *block_sums, const StepZeroing &zero, cudaStream_t s) {
    const int blocks = std::max(1, ceil_div(n, kStepThreads));
    launch(project_step_kernel, blocks, kStepThreads, 0, s, n, reinterpret_cast<const float2 *>(means2d),
           reinterpret_cast<const float2 *>(scales2d), rotation, (float)img_width, (float)img_height, (unsigned)tiles_x, (unsigned)tiles_y,
           (unsigned)row_begin, (unsigned)row_end, reinterpret_cast<float2 *>(xys), radii, conics, tiles_hit, block_sums, zero);
    return check_launch("project (training step)");
}

int project_bwd_finish(int n, const float *scales2d, const float *rotation, int img_height, int img_width, const int32_t *radii,
                       const float *conics, const float *v_xy, const float *v_conic, float *v_cov2d, float *v_mean2d, float *v_scale,
                       float *v_rot, const LossFinish &finish, cudaStream_t s) {
    launch(project_bwd_kernel<true>, std::max(1, ceil_div(n, 256)), 256, 0, s, n, reinterpret_cast<const float2 *>(scales2d), rotation,
           (float)img_width, (float)img_height, radii, conics, reinterpret_cast<const float2 *>(v_xy), v_conic, v_cov2d,
           reinterpret_cast<float2 *>(v_mean2d), reinterpret_cast<float2 *>(v_scale), v_rot, finish);
    return check_launch("projection backward (training step)");
}

}  // namespace igs

