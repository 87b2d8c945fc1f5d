// L1 loss of the rendered image and its gradient in one pass over both images (the training loss of model.py:1224-1227,
// l1_loss_ratio * F.l1_loss(images, targets), whose autograd backward is sign(image - target) * ratio / numel).
//
// For autograd (F.l1_loss routed here) the forward pass can keep the signs instead (one byte per value) and the backward pass form
// sign * (g / numel) from the incoming gradient g, a device scalar: the product ATen's l1_loss backward forms (mean: g / numel, abs:
// times sgn), so the gradient is bit for bit ATen's, with a quarter of the bytes written and read between the two passes.
//
// Grid-stride loop with 16-byte vector loads and stores; every block writes its partial sum, and the last block to finish (an atomic
// ticket, no waiting) adds the partials in block order, so the loss is deterministic. The ticket counter is reset by that block, so
// repeated calls and CUDA-graph replays need no re-initialization beyond the first zeroing of the workspace.
#include "igs_common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kMaxBlocks = 148 * 8;

struct L1Workspace {
    unsigned int ticket;
    unsigned int pad[63];
    float partials[kMaxBlocks];
};

__device__ __forceinline__ float sgn(float d) { return d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f); }

__device__ __forceinline__ float block_sum(float v, float *scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float total = 0.f;
    if (threadIdx.x == 0)
        for (int w = 0; w < kThreads / 32; ++w) total += scratch[w];
    return total;  // valid in thread 0
}

__device__ __forceinline__ signed char sgn8(float d) { return d > 0.f ? 1 : (d < 0.f ? -1 : 0); }

// kSigns false: grad[i] = sign(d_i) * grad_value; true: signs[i] = sign(d_i) (one byte)
template <bool kSigns>
__global__ void __launch_bounds__(kThreads) l1_kernel(const int64_t numel, const float *__restrict__ image, const float *__restrict__ target,
                                                      const float ratio, const float grad_value, float *__restrict__ loss,
                                                      float *__restrict__ grad, signed char *__restrict__ signs, L1Workspace *__restrict__ ws) {
    __shared__ float scratch[kThreads / 32];
    __shared__ bool last;
    float acc = 0.f;
    const int64_t stride = (int64_t)gridDim.x * kThreads;
    const uintptr_t out_bits = kSigns ? (reinterpret_cast<uintptr_t>(signs) & 3) : (reinterpret_cast<uintptr_t>(grad) & 15);
    const bool vec = ((reinterpret_cast<uintptr_t>(image) | reinterpret_cast<uintptr_t>(target)) & 15) == 0 && out_bits == 0;
    auto put = [&](const int64_t i, const float d) {
        if constexpr (kSigns) signs[i] = sgn8(d);
        else grad[i] = sgn(d) * grad_value;
    };
    if (vec) {
        const int64_t n4 = numel / 4;
        const float4 *im4 = reinterpret_cast<const float4 *>(image), *tg4 = reinterpret_cast<const float4 *>(target);
        for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n4; i += stride) {
            const float4 a = __ldcs(&im4[i]), b = __ldcs(&tg4[i]);
            const float d0 = a.x - b.x, d1 = a.y - b.y, d2 = a.z - b.z, d3 = a.w - b.w;
            acc += fabsf(d0) + fabsf(d1) + fabsf(d2) + fabsf(d3);
            if constexpr (kSigns)
                reinterpret_cast<char4 *>(signs)[i] = make_char4(sgn8(d0), sgn8(d1), sgn8(d2), sgn8(d3));
            else
                __stcs(&reinterpret_cast<float4 *>(grad)[i],
                       make_float4(sgn(d0) * grad_value, sgn(d1) * grad_value, sgn(d2) * grad_value, sgn(d3) * grad_value));
        }
        for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * kThreads + threadIdx.x; i < numel; i += stride) {
            const float d = image[i] - target[i];
            acc += fabsf(d);
            put(i, d);
        }
    } else {
        for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < numel; i += stride) {
            const float d = image[i] - target[i];
            acc += fabsf(d);
            put(i, d);
        }
    }
    const float total = block_sum(acc, scratch);
    if (threadIdx.x == 0) {
        ws->partials[blockIdx.x] = total;
        __threadfence();
        last = atomicAdd(&ws->ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    float sum = 0.f;
    for (int b = threadIdx.x; b < (int)gridDim.x; b += kThreads) sum += *((volatile float *)&ws->partials[b]);
    __syncthreads();
    const float all = block_sum(sum, scratch);
    if (threadIdx.x == 0) {
        *loss = ratio * (all / (float)numel);
        ws->ticket = 0u;
    }
}

// grad[i] = signs[i] * (g / numel), g = *grad_scale (or 1): 4 values per thread and step from one 32-bit load
__global__ void __launch_bounds__(kThreads) l1_grad_kernel(const int64_t numel, const signed char *__restrict__ signs,
                                                           const float *__restrict__ grad_scale, float *__restrict__ grad) {
    const float v = (grad_scale ? *grad_scale : 1.f) / (float)numel;
    const int64_t stride = (int64_t)gridDim.x * kThreads;
    const bool vec = ((reinterpret_cast<uintptr_t>(signs) & 3) | (reinterpret_cast<uintptr_t>(grad) & 15)) == 0;
    const int64_t n4 = vec ? numel / 4 : 0;
    for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n4; i += stride) {
        const char4 s4 = __ldcs(&reinterpret_cast<const char4 *>(signs)[i]);
        __stcs(&reinterpret_cast<float4 *>(grad)[i], make_float4((float)s4.x * v, (float)s4.y * v, (float)s4.z * v, (float)s4.w * v));
    }
    for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * kThreads + threadIdx.x; i < numel; i += stride) grad[i] = (float)signs[i] * v;
}

int l1_blocks(int64_t numel) {
    const int64_t want = (numel / 4 + kThreads - 1) / kThreads;
    return (int)(want < 1 ? 1 : (want > kMaxBlocks ? kMaxBlocks : want));
}

}  // namespace

extern "C" {

size_t igs_l1_workspace(int64_t numel) { return sizeof(L1Workspace); }

int igs_l1_loss(int64_t numel, const float *image, const float *target, float ratio, float *loss, float *grad, void *workspace,
                size_t workspace_bytes, void *stream) {
    IGS_REQUIRE(numel > 0, "igs_l1_loss: empty images");
    IGS_REQUIRE(image && target && loss && grad && workspace, "igs_l1_loss: null pointer");
    IGS_REQUIRE(workspace_bytes >= sizeof(L1Workspace), "igs_l1_loss: workspace too small");
    IGS_REQUIRE(igs::aligned(workspace, 16), "igs_l1_loss: workspace must be 16-byte aligned");
    const float grad_value = ratio / (float)numel;
    l1_kernel<false><<<l1_blocks(numel), kThreads, 0, igs::as_stream(stream)>>>(numel, image, target, ratio, grad_value, loss, grad, nullptr,
                                                                               static_cast<L1Workspace *>(workspace));
    return igs::check_launch("igs_l1_loss");
}

int igs_l1_loss_signs(int64_t numel, const float *image, const float *target, float ratio, float *loss, int8_t *signs, void *workspace,
                      size_t workspace_bytes, void *stream) {
    IGS_REQUIRE(numel > 0, "igs_l1_loss_signs: empty images");
    IGS_REQUIRE(image && target && loss && signs && workspace, "igs_l1_loss_signs: null pointer");
    IGS_REQUIRE(workspace_bytes >= sizeof(L1Workspace), "igs_l1_loss_signs: workspace too small");
    IGS_REQUIRE(igs::aligned(workspace, 16), "igs_l1_loss_signs: workspace must be 16-byte aligned");
    l1_kernel<true><<<l1_blocks(numel), kThreads, 0, igs::as_stream(stream)>>>(numel, image, target, ratio, 0.f, loss, nullptr,
                                                                              reinterpret_cast<signed char *>(signs),
                                                                              static_cast<L1Workspace *>(workspace));
    return igs::check_launch("igs_l1_loss_signs");
}

int igs_l1_grad_from_signs(int64_t numel, const int8_t *signs, const float *grad_scale, float *grad, void *stream) {
    IGS_REQUIRE(numel > 0, "igs_l1_grad_from_signs: empty images");
    IGS_REQUIRE(signs && grad, "igs_l1_grad_from_signs: null pointer");
    l1_grad_kernel<<<l1_blocks(numel), kThreads, 0, igs::as_stream(stream)>>>(numel, reinterpret_cast<const signed char *>(signs), grad_scale,
                                                                            grad);
    return igs::check_launch("igs_l1_grad_from_signs");
}

}  // extern "C"
