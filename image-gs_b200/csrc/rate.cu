// Rate term of the training loss (compress/rate.py: rate_bits 167-175 defines it; the reference computes it in gsplat/gsplat/cuda/csrc/
// rate.cu:35-199): smooth Laplace code lengths (sqrt(r^2 + 1/4) - 1/2) / (scale ln 2) of the feature residuals r of a prediction from
// causal neighbors (weighted neighbor mean plus a CCLM slope times the Gaussian's reference-channel deviation, after subtracting colour
// reference channels) and of the canonical rotations, times factor / max(l1 / l1_ratio, 1e-4).
//
// Forward: one thread per Gaussian computes its bits and the gradient of its bits with respect to its own features (own_grad) and rotation;
// blocks write partial sums and the last block (atomic ticket, no waiting) adds them in block order and forms the loss, so the loss is
// deterministic and needs one launch. Backward: one thread per Gaussian gathers, over the Gaussians that predict from it (CSR lists), their
// own gradients times their neighbor weights; no atomics. Compiled with --use_fast_math like the reference kernels.
#include "igs_common.cuh"

namespace {

using igs::kMaxChannels;
constexpr int kThreads = 256;

struct ChannelRefs {
    int color[kMaxChannels];  // channel subtracted before the prediction, -1 for none
    int pred[kMaxChannels];   // reference channel of the CCLM term (the channel itself when it has none)
};

struct RateWorkspace {
    unsigned int ticket;
    unsigned int pad[63];
    float partials[1];  // one per block
};

template <int kMaxC>
__device__ __forceinline__ void coded(const float *__restrict__ f, const ChannelRefs &refs, int channels, float (&out)[kMaxC]) {
#pragma unroll
    for (int c = 0; c < kMaxC; ++c)
        if (c < channels) out[c] = f[c] - (refs.color[c] >= 0 ? f[refs.color[c]] : 0.f);
}

template <int C>
__global__ void __launch_bounds__(kThreads) rate_fwd_kernel(const int n, const int channels_rt, const int num_neighbors,
                                                            const ChannelRefs refs, const float *__restrict__ feat,
                                                            const float *__restrict__ rot, const float *__restrict__ l1_loss,
                                                            const int *__restrict__ neighbors, const float *__restrict__ weights,
                                                            const float *__restrict__ slope, const float *__restrict__ inv_steps,
                                                            const float *__restrict__ feat_coeffs, const float *__restrict__ rot_coeffs,
                                                            const float inv_rot_step, const float l1_ratio, const float factor,
                                                            float *__restrict__ loss, float *__restrict__ loss_weight,
                                                            float *__restrict__ own_grad, float *__restrict__ rot_grad,
                                                            RateWorkspace *__restrict__ ws) {
    constexpr int kMaxC = C > 0 ? C : kMaxChannels;
    const int channels = C > 0 ? C : channels_rt;
    __shared__ float scratch[kThreads / 32];
    __shared__ bool last;
    const int i = blockIdx.x * kThreads + threadIdx.x;
    float bits = 0.f;
    if (i < n) {
        float v[kMaxC], mean[kMaxC], nb[kMaxC], cg[kMaxC];
        coded<kMaxC>(feat + (size_t)i * channels, refs, channels, v);
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) mean[c] = 0.f, cg[c] = 0.f;
        for (int k = 0; k < num_neighbors; ++k) {
            const float w = __ldg(&weights[(size_t)i * num_neighbors + k]);
            if (w == 0.f) continue;
            coded<kMaxC>(feat + (size_t)__ldg(&neighbors[(size_t)i * num_neighbors + k]) * channels, refs, channels, nb);
#pragma unroll
            for (int c = 0; c < kMaxC; ++c)
                if (c < channels) mean[c] += w * nb[c];
        }
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) {
            if (c >= channels) continue;
            // the reference channel's deviation, selected without dynamic register indexing
            float dev = 0.f;
#pragma unroll
            for (int q = 0; q < kMaxC; ++q)
                if (q == refs.pred[c]) dev = v[q] - mean[q];
            const float sl = __ldg(&slope[(size_t)i * channels + c]);
            const float r = (v[c] - mean[c] - sl * dev) * __ldg(&inv_steps[c]);
            const float root = sqrtf(r * r + 0.25f);
            const float coeff = __ldg(&feat_coeffs[c]);
            bits += (root - 0.5f) * coeff;
            const float g = coeff * r / root * __ldg(&inv_steps[c]);
            cg[c] += g;
#pragma unroll
            for (int q = 0; q < kMaxC; ++q)
                if (q == refs.pred[c]) cg[q] -= sl * g;
        }
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) {
            if (c >= channels) continue;
            float g = cg[c];
#pragma unroll
            for (int q = 0; q < kMaxC; ++q)
                if (q < channels && refs.color[q] == c) g -= cg[q];
            own_grad[(size_t)i * channels + c] = g;
        }
        // canonical rotation in steps: quarter turns (no gradient) removed, within [-pi/4, pi/4]
        const float angle = rot[i];
        const float t = (angle - rintf(angle * (float)M_2_PI) * (float)M_PI_2) * inv_rot_step;
        const float root = sqrtf(t * t + 0.25f);
        const float rc = __ldg(&rot_coeffs[i]);
        bits += (root - 0.5f) * rc;
        rot_grad[i] = rc * t / root * inv_rot_step;
    }

    // block sum, then the last block adds the partials in block order
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) bits += __shfl_xor_sync(0xffffffffu, bits, o);
    if (lane == 0) scratch[warp] = bits;
    __syncthreads();
    if (threadIdx.x == 0) {
        float total = 0.f;
        for (int w = 0; w < kThreads / 32; ++w) total += scratch[w];
        ws->partials[blockIdx.x] = total;
        __threadfence();
        last = atomicAdd(&ws->ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    float sum = 0.f;
    for (int b = threadIdx.x; b < (int)gridDim.x; b += kThreads) sum += *((volatile float *)&ws->partials[b]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    __syncthreads();
    if (lane == 0) scratch[warp] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        float total = 0.f;
        for (int w = 0; w < kThreads / 32; ++w) total += scratch[w];
        const float weight = factor / fmaxf(l1_loss[0] / l1_ratio, 1e-4f);
        *loss = weight * total;
        *loss_weight = weight;
        ws->ticket = 0u;
    }
}

template <int C>
__global__ void __launch_bounds__(kThreads) rate_bwd_kernel(const int n, const int channels_rt, const float *__restrict__ grad_loss,
                                                            const float *__restrict__ loss_weight, const float *__restrict__ own_grad,
                                                            const float *__restrict__ rot_grad, const int *__restrict__ offsets,
                                                            const int *__restrict__ sources, const float *__restrict__ source_weights,
                                                            float *__restrict__ grad_feat, float *__restrict__ grad_rot) {
    constexpr int kMaxC = C > 0 ? C : kMaxChannels;
    const int channels = C > 0 ? C : channels_rt;
    const int j = blockIdx.x * kThreads + threadIdx.x;
    if (j >= n) return;
    const float scale = grad_loss[0] * loss_weight[0];
    float g[kMaxC];
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) g[c] = c < channels ? own_grad[(size_t)j * channels + c] : 0.f;
    const int e1 = offsets[j + 1];
    for (int e = offsets[j]; e < e1; ++e) {
        const int src = __ldg(&sources[e]);
        const float w = __ldg(&source_weights[e]);
#pragma unroll
        for (int c = 0; c < kMaxC; ++c)
            if (c < channels) g[c] -= w * __ldg(&own_grad[(size_t)src * channels + c]);
    }
#pragma unroll
    for (int c = 0; c < kMaxC; ++c)
        if (c < channels) grad_feat[(size_t)j * channels + c] = scale * g[c];
    grad_rot[j] = scale * rot_grad[j];
}

}  // namespace

extern "C" {

size_t igs_rate_workspace(int num_gaussians) {
    const int blocks = igs::ceil_div(num_gaussians > 0 ? num_gaussians : 1, kThreads);
    return sizeof(RateWorkspace) + sizeof(float) * (size_t)blocks;
}

int igs_rate_fwd(int num_gaussians, int channels, int num_neighbors, const float *feat, const float *rot, const float *l1_loss,
                 const int32_t *neighbors, const float *weights, const float *slope, const int32_t *color_refs, const int32_t *pred_refs,
                 const float *inv_steps, const float *feat_coeffs, const float *rot_coeffs, float inv_rot_step, float l1_ratio,
                 float factor, float *loss, float *loss_weight, float *own_grad, float *rot_grad, void *workspace, size_t workspace_bytes,
                 void *stream) {
    IGS_REQUIRE(num_gaussians >= 0 && num_neighbors >= 0, "igs_rate_fwd: negative size");
    IGS_REQUIRE(channels >= 1 && channels <= kMaxChannels, "igs_rate_fwd: 1 to %d feature channels", kMaxChannels);
    IGS_REQUIRE(color_refs && pred_refs, "igs_rate_fwd: null channel references");
    IGS_REQUIRE(l1_loss && loss && loss_weight && workspace, "igs_rate_fwd: null pointer");
    IGS_REQUIRE(workspace_bytes >= igs_rate_workspace(num_gaussians), "igs_rate_fwd: workspace too small");
    IGS_REQUIRE(num_gaussians == 0 || (feat && rot && (neighbors || num_neighbors == 0) && (weights || num_neighbors == 0) && slope &&
                                       inv_steps && feat_coeffs && rot_coeffs && own_grad && rot_grad),
                "igs_rate_fwd: null pointer");
    ChannelRefs refs;
    for (int c = 0; c < kMaxChannels; ++c) {
        refs.color[c] = -1;
        refs.pred[c] = c;
    }
    for (int c = 0; c < channels; ++c) {
        IGS_REQUIRE(color_refs[c] < channels && pred_refs[c] >= 0 && pred_refs[c] < channels,
                    "igs_rate_fwd: invalid reference channel for channel %d", c);
        refs.color[c] = color_refs[c];
        refs.pred[c] = pred_refs[c];
    }
    const int blocks = igs::ceil_div(num_gaussians > 0 ? num_gaussians : 1, kThreads);
    cudaStream_t s = igs::as_stream(stream);
    auto ws = static_cast<RateWorkspace *>(workspace);
    if (channels == 3)
        rate_fwd_kernel<3><<<blocks, kThreads, 0, s>>>(num_gaussians, channels, num_neighbors, refs, feat, rot, l1_loss, neighbors, weights,
                                                       slope, inv_steps, feat_coeffs, rot_coeffs, inv_rot_step, l1_ratio, factor, loss,
                                                       loss_weight, own_grad, rot_grad, ws);
    else
        rate_fwd_kernel<0><<<blocks, kThreads, 0, s>>>(num_gaussians, channels, num_neighbors, refs, feat, rot, l1_loss, neighbors, weights,
                                                       slope, inv_steps, feat_coeffs, rot_coeffs, inv_rot_step, l1_ratio, factor, loss,
                                                       loss_weight, own_grad, rot_grad, ws);
    return igs::check_launch("igs_rate_fwd");
}

int igs_rate_bwd(int num_gaussians, int channels, const float *grad_loss, const float *loss_weight, const float *own_grad,
                 const float *rot_grad, const int32_t *offsets, const int32_t *sources, const float *source_weights, float *grad_feat,
                 float *grad_rot, void *stream) {
    IGS_REQUIRE(num_gaussians >= 0, "igs_rate_bwd: negative size");
    IGS_REQUIRE(channels >= 1 && channels <= kMaxChannels, "igs_rate_bwd: 1 to %d feature channels", kMaxChannels);
    if (num_gaussians == 0) return IGS_OK;
    IGS_REQUIRE(grad_loss && loss_weight && own_grad && rot_grad && offsets && grad_feat && grad_rot, "igs_rate_bwd: null pointer");
    const int blocks = igs::ceil_div(num_gaussians, kThreads);
    cudaStream_t s = igs::as_stream(stream);
    if (channels == 3)
        rate_bwd_kernel<3><<<blocks, kThreads, 0, s>>>(num_gaussians, channels, grad_loss, loss_weight, own_grad, rot_grad, offsets, sources,
                                                       source_weights, grad_feat, grad_rot);
    else
        rate_bwd_kernel<0><<<blocks, kThreads, 0, s>>>(num_gaussians, channels, grad_loss, loss_weight, own_grad, rot_grad, offsets, sources,
                                                       source_weights, grad_feat, grad_rot);
    return igs::check_launch("igs_rate_bwd");
}

}  // extern "C"
