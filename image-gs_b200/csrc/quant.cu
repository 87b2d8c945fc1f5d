// Straight-through "step" quantization of the Gaussian parameters in the training step, one thread per Gaussian, replacing the ~20 ATen
// kernels of model.py:993-1006 (compress/quantization.py: quantize_step 36-42, dequantize 45-46, canonicalize 61-74 with quarter turns off,
// get_step_symbols 151-172, dequantize_symbols 188-199):
//   symbols   q_xy = round(xy / pos_step), q_s = round(log2|s| / scale_step), q_rot = round(rot / rot_step), q_f = round(f / feat_step)
//   values    x + (dequantize(q) - x), dequantize(q) = q * step (scale: exp2(q * scale_step))
// The symbols must equal ATen's bit for bit, so this file is compiled WITHOUT fast-math and every operation is the IEEE one ATen performs:
// correctly rounded division, log2f/exp2f from the CUDA math library (ATen's log2/exp2 on float), rintf (round half to even, as
// torch.round), and separate multiply / add / subtract with explicit round-to-nearest intrinsics so that nothing is contracted.
// Optionally also the features mapped to the loss space, out_feat T^T (model.py:963-964).
#include "igs_common.cuh"

namespace {

using igs::kMaxChannels;

__device__ __forceinline__ float ste(float x, float q) { return __fadd_rn(x, __fsub_rn(q, x)); }

template <int C>
__global__ void __launch_bounds__(256) quantize_ste_kernel(const int n, const int channels_rt, const float2 *__restrict__ xy,
                                                           const float2 *__restrict__ scale, const float *__restrict__ rot,
                                                           const float *__restrict__ feat, const float *__restrict__ pos_steps,
                                                           const float scale_step, const float rot_step, const float *__restrict__ feat_steps,
                                                           const float *__restrict__ transform, float2 *__restrict__ out_xy,
                                                           float2 *__restrict__ out_scale, float *__restrict__ out_rot,
                                                           float *__restrict__ out_feat, float *__restrict__ out_feat_t,
                                                           float2 *__restrict__ q_xy, float2 *__restrict__ q_scale, float *__restrict__ q_rot,
                                                           float *__restrict__ q_feat) {
    constexpr int kMaxC = C > 0 ? C : kMaxChannels;
    const int channels = C > 0 ? C : channels_rt;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;

    const float2 p = xy[i];
    const float sx = __ldg(&pos_steps[0]), sy = __ldg(&pos_steps[1]);
    const float qx = rintf(__fdiv_rn(p.x, sx)), qy = rintf(__fdiv_rn(p.y, sy));
    out_xy[i] = make_float2(ste(p.x, __fadd_rn(__fmul_rn(qx, sx), 0.f)), ste(p.y, __fadd_rn(__fmul_rn(qy, sy), 0.f)));

    const float2 s = scale[i];
    const float qs0 = rintf(__fdiv_rn(log2f(fabsf(s.x)), scale_step)), qs1 = rintf(__fdiv_rn(log2f(fabsf(s.y)), scale_step));
    out_scale[i] = make_float2(ste(s.x, exp2f(__fadd_rn(__fmul_rn(qs0, scale_step), 0.f))),
                               ste(s.y, exp2f(__fadd_rn(__fmul_rn(qs1, scale_step), 0.f))));

    const float r = rot[i];
    const float qr = rintf(__fdiv_rn(r, rot_step));
    out_rot[i] = ste(r, __fadd_rn(__fmul_rn(qr, rot_step), 0.f));

    float f_out[kMaxC];
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) {
        if (c >= channels) continue;
        const float f = feat[(size_t)i * channels + c];
        const float step = __ldg(&feat_steps[c]);
        const float qf = rintf(__fdiv_rn(f, step));
        f_out[c] = ste(f, __fadd_rn(__fmul_rn(qf, step), 0.f));
        out_feat[(size_t)i * channels + c] = f_out[c];
        if (q_feat) q_feat[(size_t)i * channels + c] = qf;
    }
    if (q_xy) q_xy[i] = make_float2(qx, qy);
    if (q_scale) q_scale[i] = make_float2(qs0, qs1);
    if (q_rot) q_rot[i] = qr;
    if (out_feat_t) {
#pragma unroll
        for (int d = 0; d < kMaxC; ++d) {
            if (d >= channels) continue;
            float acc = 0.f;
#pragma unroll
            for (int c = 0; c < kMaxC; ++c)
                if (c < channels) acc = __fmaf_rn(f_out[c], __ldg(&transform[d * channels + c]), acc);
            out_feat_t[(size_t)i * channels + d] = acc;
        }
    }
}

}  // namespace

extern "C" {

int igs_quantize_ste(int num_points, int channels, const float *xy, const float *scale, const float *rot, const float *feat,
                     const float *pos_steps, float scale_step, float rot_step, const float *feat_steps, const float *feat_transform,
                     float *out_xy, float *out_scale, float *out_rot, float *out_feat, float *out_feat_t, float *q_xy, float *q_scale,
                     float *q_rot, float *q_feat, void *stream) {
    IGS_REQUIRE(num_points >= 0, "igs_quantize_ste: negative size");
    IGS_REQUIRE(channels >= 0 && channels <= kMaxChannels, "igs_quantize_ste: at most %d channels", kMaxChannels);
    IGS_REQUIRE(scale_step > 0.f && rot_step > 0.f, "igs_quantize_ste: steps must be positive");
    if (num_points == 0) return IGS_OK;
    IGS_REQUIRE(xy && scale && rot && (feat || channels == 0) && pos_steps && (feat_steps || channels == 0) && out_xy && out_scale &&
                    out_rot && (out_feat || channels == 0),
                "igs_quantize_ste: null pointer");
    IGS_REQUIRE(feat_transform == nullptr || out_feat_t != nullptr, "igs_quantize_ste: feat_transform needs out_feat_t");
    IGS_REQUIRE(igs::aligned(xy, 8) && igs::aligned(scale, 8) && igs::aligned(out_xy, 8) && igs::aligned(out_scale, 8) &&
                    (q_xy == nullptr || igs::aligned(q_xy, 8)) && (q_scale == nullptr || igs::aligned(q_scale, 8)),
                "igs_quantize_ste: [N, 2] tensors must be 8-byte aligned");
    cudaStream_t s = igs::as_stream(stream);
    const int blocks = igs::ceil_div(num_points, 256);
    auto go = [&](auto kernel) {
        kernel<<<blocks, 256, 0, s>>>(num_points, channels, reinterpret_cast<const float2 *>(xy), reinterpret_cast<const float2 *>(scale),
                                      rot, feat, pos_steps, scale_step, rot_step, feat_steps, feat_transform,
                                      reinterpret_cast<float2 *>(out_xy), reinterpret_cast<float2 *>(out_scale), out_rot, out_feat,
                                      feat_transform ? out_feat_t : nullptr, reinterpret_cast<float2 *>(q_xy),
                                      reinterpret_cast<float2 *>(q_scale), q_rot, q_feat);
    };
    if (channels == 3)
        go(quantize_ste_kernel<3>);
    else
        go(quantize_ste_kernel<0>);
    return igs::check_launch("igs_quantize_ste");
}

}  // extern "C"

// Backward of the loss-space feature transform of the forward above (feat_t = feat T^T, model.py:963-964) with the straight-through
// identity: v_feat = v_feat_t T (+ v_extra, e.g. the rate term's gradient with respect to the same features), one thread per Gaussian.
namespace {

template <int C>
__global__ void __launch_bounds__(256) feat_transform_bwd_kernel(const int n, const int channels_rt, const float *__restrict__ v_feat_t,
                                                                 const float *__restrict__ transform, const float *__restrict__ v_extra,
                                                                 float *__restrict__ v_feat) {
    constexpr int kMaxC = C > 0 ? C : kMaxChannels;
    const int channels = C > 0 ? C : channels_rt;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float g[kMaxC];
#pragma unroll
    for (int d = 0; d < kMaxC; ++d) g[d] = d < channels ? v_feat_t[(size_t)i * channels + d] : 0.f;
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) {
        if (c >= channels) continue;
        float acc = v_extra ? v_extra[(size_t)i * channels + c] : 0.f;
#pragma unroll
        for (int d = 0; d < kMaxC; ++d)
            if (d < channels) acc = __fmaf_rn(g[d], __ldg(&transform[d * channels + c]), acc);
        v_feat[(size_t)i * channels + c] = acc;
    }
}

}  // namespace

extern "C" int igs_feat_transform_bwd(int num_points, int channels, const float *v_feat_t, const float *feat_transform, const float *v_extra,
                                      float *v_feat, void *stream) {
    IGS_REQUIRE(num_points >= 0, "igs_feat_transform_bwd: negative size");
    IGS_REQUIRE(channels >= 1 && channels <= kMaxChannels, "igs_feat_transform_bwd: 1 to %d channels", kMaxChannels);
    if (num_points == 0) return IGS_OK;
    IGS_REQUIRE(v_feat_t && feat_transform && v_feat, "igs_feat_transform_bwd: null pointer");
    const int blocks = igs::ceil_div(num_points, 256);
    if (channels == 3)
        feat_transform_bwd_kernel<3><<<blocks, 256, 0, igs::as_stream(stream)>>>(num_points, channels, v_feat_t, feat_transform, v_extra, v_feat);
    else
        feat_transform_bwd_kernel<0><<<blocks, 256, 0, igs::as_stream(stream)>>>(num_points, channels, v_feat_t, feat_transform, v_extra, v_feat);
    return igs::check_launch("igs_feat_transform_bwd");
}
