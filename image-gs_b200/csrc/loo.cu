// Leave-one-out loss increase per Gaussian (topk_norm_loo_loss_increase, gsplat/gsplat/cuda/csrc/forward.cu:667-738; called once per
// pruning round by compress/pruning.py:13-27): with the top-K weights w = exp(-sigma) of a pixel, S_w = sum_k w_k and S_f = sum_k w_k f_k,
// removing slot k changes the pixel from S_f / (S_w + eps) to (S_f - w_k f_k) / (S_w - w_k + eps); the change of the pixel's absolute
// (or squared) error summed over channels is added to that Gaussian.
//
// One CTA of 256 threads per 16x16 tile, one pixel per thread, each warp an 8x4 patch of the tile (neighbouring pixels share most of
// their lists). After each pixel's per-slot increases are known, the warp walks the union of its pixels' Gaussian IDs in increasing
// order (a warp-wide minimum per step: about 15 steps for a patch), adds the increases of the lanes holding the current Gaussian with
// one five-step shuffle sum, and makes one global atomic per (warp, Gaussian). Compiled with --use_fast_math like the reference.
#include "igs_common.cuh"

namespace {

using igs::kMaxChannels;
using igs::kTile;
using igs::kTopK;

constexpr int kNoId = 0x7fffffff;

template <int C>
__global__ void __launch_bounds__(256) loo_kernel(const int tiles_x, const int img_h, const int img_w, const int channels_rt,
                                                  const int num_points, const float2 *__restrict__ xys, const float *__restrict__ conics,
                                                  const float *__restrict__ colors, const int *__restrict__ pixel_topk,
                                                  const float *__restrict__ targets, const bool squared, const float eps,
                                                  float *__restrict__ loss_increase) {
    constexpr int kMaxC = C > 0 ? C : kMaxChannels;
    const int channels = C > 0 ? C : channels_rt;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // warp w covers the 8x4 patch (w % 2, w / 2) of the tile, lane l its pixel (l % 8, l / 8)
    const int i = (blockIdx.x / tiles_x) * kTile + (warp >> 1) * 4 + (lane >> 3);
    const int j = (blockIdx.x % tiles_x) * kTile + (warp & 1) * 8 + (lane & 7);
    const bool valid = i < img_h && j < img_w;
    const int num_pixels = img_h * img_w;
    const int p = valid ? i * img_w + j : 0;
    const float px = (float)j, py = (float)i;
    int ids[kTopK];
    float w[kTopK];
    float sum_w = 0.f, sum_f[kMaxC], target[kMaxC];
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) {
        sum_f[c] = 0.f;
        target[c] = (valid && c < channels) ? targets[(size_t)c * num_pixels + p] : 0.f;
    }
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        const int id = valid ? __ldg(&pixel_topk[(size_t)p * kTopK + k]) : -1;
        const int g = id < num_points ? id : -1;  // an ID of N or more counts as an empty slot instead of reading out of bounds
        ids[k] = g;
        w[k] = 0.f;
        if (g < 0) continue;
        const float2 xy = __ldg(&xys[g]);
        const float a = __ldg(&conics[3 * g]), b = __ldg(&conics[3 * g + 1]), cc = __ldg(&conics[3 * g + 2]);
        w[k] = __expf(-igs::gaussian_sigma(xy.x, xy.y, a, b, cc, px, py));
        sum_w += w[k];
#pragma unroll
        for (int c = 0; c < kMaxC; ++c)
            if (c < channels) sum_f[c] += w[k] * __ldg(&colors[(size_t)g * channels + c]);
    }
    float error = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) {
        if (c >= channels) continue;
        const float diff = sum_f[c] / (sum_w + eps) - target[c];
        error += squared ? diff * diff : fabsf(diff);
    }
    float delta[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        const int g = ids[k];
        delta[k] = 0.f;
        if (g >= 0) {
            const float inv = 1.f / (sum_w - w[k] + eps);
            float loo = 0.f;
#pragma unroll
            for (int c = 0; c < kMaxC; ++c) {
                if (c >= channels) continue;
                const float diff = (sum_f[c] - w[k] * __ldg(&colors[(size_t)g * channels + c])) * inv - target[c];
                loo += squared ? diff * diff : fabsf(diff);
            }
            delta[k] = loo - error;
        }
        ids[k] = g < 0 ? kNoId : g;
    }
    // the union of the warp's IDs in increasing order: one warp sum and one atomic per Gaussian
    while (true) {
        int head = ids[0];
#pragma unroll
        for (int k = 1; k < kTopK; ++k) head = min(head, ids[k]);
        const int cur = __reduce_min_sync(0xffffffffu, head);
        if (cur == kNoId) break;
        float v = 0.f;
#pragma unroll
        for (int k = 0; k < kTopK; ++k) {
            if (ids[k] == cur) {
                v += delta[k];  // a list holds a Gaussian once; a malformed one with repeats still adds every slot
                ids[k] = kNoId;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) atomicAdd(&loss_increase[cur], v);
    }
}

}  // namespace

extern "C" {

int igs_loo_loss_increase(int img_height, int img_width, int channels, int num_points, const float *xys, const float *conics,
                          const float *colors, const int32_t *pixel_topk, const float *targets, int squared, float eps,
                          float *loss_increase, void *stream) {
    IGS_REQUIRE(img_height >= 0 && img_width >= 0 && num_points >= 0, "igs_loo_loss_increase: negative size");
    IGS_REQUIRE(channels >= 0 && channels <= kMaxChannels, "igs_loo_loss_increase: at most %d channels", kMaxChannels);
    cudaStream_t s = igs::as_stream(stream);
    if (num_points == 0) return IGS_OK;
    IGS_REQUIRE(loss_increase, "igs_loo_loss_increase: null output");
    if (cudaMemsetAsync(loss_increase, 0, sizeof(float) * (size_t)num_points, s) != cudaSuccess) return igs::check_launch("igs_loo_loss_increase");
    const int num_pixels = img_height * img_width;
    if (num_pixels == 0) return IGS_OK;
    IGS_REQUIRE(xys && conics && (colors || channels == 0) && pixel_topk && (targets || channels == 0), "igs_loo_loss_increase: null pointer");
    IGS_REQUIRE(igs::aligned(xys, 8), "igs_loo_loss_increase: xys must be 8-byte aligned");
    const int tiles_x = igs::ceil_div(img_width, kTile), tiles_y = igs::ceil_div(img_height, kTile);
    const int blocks = tiles_x * tiles_y;
    if (channels == 3)
        loo_kernel<3><<<blocks, 256, 0, s>>>(tiles_x, img_height, img_width, channels, num_points, reinterpret_cast<const float2 *>(xys),
                                             conics, colors, pixel_topk, targets, squared != 0, eps, loss_increase);
    else
        loo_kernel<0><<<blocks, 256, 0, s>>>(tiles_x, img_height, img_width, channels, num_points, reinterpret_cast<const float2 *>(xys),
                                             conics, colors, pixel_topk, targets, squared != 0, eps, loss_increase);
    return igs::check_launch("igs_loo_loss_increase");
}

}  // extern "C"
