// Per-Gaussian feature weights from the top-K lists: the sum over pixels of each Gaussian's squared normalized top-K weight, the
// sensitivity proxy of the adaptive feature steps (compress/quantization.py:218-230 feature_weights over model.py:1404-1421
// _iter_topk_weights). One thread per pixel recomputes its slots' weights exp(-sigma) with the reference's arithmetic, normalizes them
// in double, and adds round(w^2 2^40) to the Gaussian's 64-bit fixed-point sum: integer additions, so the result does not depend on the
// order of the atomics.
//
// The reference evaluates sigma with separate ATen float32 operations (no contraction) and ATen's expf, so this file is compiled without
// fast-math and spells every operation with an explicit round-to-nearest intrinsic:
//   delta = xy[id] - pixel; sigma = 0.5 * (c0 * d0^2 + c2 * d1^2) + c1 * d0 * d1; w = exp(-sigma) * valid
//   normalized = w / (sum_k w_k + eps) in double; fixed[id] += round(normalized^2 * 2^40) for valid slots.
#include "igs_common.cuh"

namespace {

constexpr int kTopK = 10;
constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) feature_weights_kernel(const int img_h, const int img_w, const int num_points,
                                                                   const float2 *__restrict__ xys,
                                                                   const float *__restrict__ conics, const int *__restrict__ pixel_topk,
                                                                   const double eps, unsigned long long *__restrict__ fixed) {
    const int64_t p = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (p >= (int64_t)img_h * img_w) return;
    const float px = (float)(p % img_w), py = (float)(p / img_w);
    int ids[kTopK];
    const int2 *row = reinterpret_cast<const int2 *>(pixel_topk + p * kTopK);
#pragma unroll
    for (int k = 0; k < kTopK / 2; ++k) {
        // an ID outside [0, N) counts as an empty slot (the reference's indexing would fault on one of N or more)
        const int2 v = __ldg(&row[k]);
        ids[2 * k] = (unsigned)v.x < (unsigned)num_points ? v.x : -1;
        ids[2 * k + 1] = (unsigned)v.y < (unsigned)num_points ? v.y : -1;
    }
    float w[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        const int g = ids[k] >= 0 ? ids[k] : 0;  // empty slots read Gaussian 0 and are multiplied by 0, as the reference does
        const float2 xy = __ldg(&xys[g]);
        const float c0 = __ldg(&conics[3 * g]), c1 = __ldg(&conics[3 * g + 1]), c2 = __ldg(&conics[3 * g + 2]);
        const float d0 = __fsub_rn(xy.x, px), d1 = __fsub_rn(xy.y, py);
        const float quad = __fmul_rn(0.5f, __fadd_rn(__fmul_rn(c0, __fmul_rn(d0, d0)), __fmul_rn(c2, __fmul_rn(d1, d1))));
        const float sigma = __fadd_rn(quad, __fmul_rn(__fmul_rn(c1, d0), d1));
        w[k] = __fmul_rn(expf(-sigma), ids[k] >= 0 ? 1.f : 0.f);
    }
    // the row sum in the order of ATen's CUDA sum over a [P, 10] float64 row: element k into accumulator k % 8, then the accumulators
    // combined as a tree (i with i + 4, then i + 2, then i + 1); the normalized weights and their rounding follow it bit for bit
    double acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = (double)w[j];
    acc[0] = __dadd_rn(acc[0], (double)w[8]);
    acc[1] = __dadd_rn(acc[1], (double)w[9]);
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j] = __dadd_rn(acc[j], acc[j + 4]);
    acc[0] = __dadd_rn(acc[0], acc[2]);
    acc[1] = __dadd_rn(acc[1], acc[3]);
    const double denom = __dadd_rn(__dadd_rn(acc[0], acc[1]), eps);
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        if (ids[k] < 0) continue;
        const double n = __ddiv_rn((double)w[k], denom);
        const double q = rint(__dmul_rn(__dmul_rn(n, n), 1099511627776.0));  // 2^40, round half to even as torch.round
        atomicAdd(&fixed[ids[k]], (unsigned long long)(long long)q);
    }
}

}  // namespace

extern "C" int igs_feature_weights(int img_height, int img_width, int num_points, const float *xys, const float *conics,
                                   const int32_t *pixel_topk, double eps, int64_t *fixed_point, void *stream) {
    IGS_REQUIRE(img_height >= 0 && img_width >= 0 && num_points >= 0, "igs_feature_weights: negative size");
    if (num_points == 0) return IGS_OK;
    IGS_REQUIRE(fixed_point != nullptr, "igs_feature_weights: null pointer");
    cudaStream_t s = igs::as_stream(stream);
    if (cudaMemsetAsync(fixed_point, 0, sizeof(int64_t) * (size_t)num_points, s) != cudaSuccess)
        return igs::check_launch("igs_feature_weights");
    const int64_t pixels = (int64_t)img_height * img_width;
    if (pixels == 0) return IGS_OK;
    IGS_REQUIRE(xys && conics && pixel_topk, "igs_feature_weights: null pointer");
    IGS_REQUIRE(igs::aligned(xys, 8) && igs::aligned(pixel_topk, 8), "igs_feature_weights: xys and pixel_topk must be 8-byte aligned");
    const int64_t blocks = (pixels + kThreads - 1) / kThreads;
    feature_weights_kernel<<<(unsigned)blocks, kThreads, 0, s>>>(img_height, img_width, num_points, reinterpret_cast<const float2 *>(xys),
                                                               conics,
                                                               pixel_topk, eps, reinterpret_cast<unsigned long long *>(fixed_point));
    return igs::check_launch("igs_feature_weights");
}
