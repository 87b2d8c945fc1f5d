// Per-Gaussian arithmetic of the 2D projection shared by the kernels that need it (project.cu, and the bands' exchange in exchange.cu,
// which runs the projection backward on the summed gradients). Every file that includes it is compiled with --use_fast_math, like the
// reference extension (gsplat/setup.py:70), so that the same approximate sqrt / reciprocal / sin / cos and the same contracted products
// give the same bits in every kernel.
#pragma once

#include "igs_common.cuh"

namespace igs {

// 2x2 matrix stored [column][row]; product terms in glm's order: (a*b)[c][r] = a[0][r]*b[c][0] + a[1][r]*b[c][1]
struct M2 {
    float m[2][2];
};

__device__ __forceinline__ M2 mul(const M2 &a, const M2 &b) {
    M2 o;
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int r = 0; r < 2; ++r) o.m[c][r] = a.m[0][r] * b.m[c][0] + a.m[1][r] * b.m[c][1];
    return o;
}

__device__ __forceinline__ M2 transpose(const M2 &a) {
    M2 o;
    o.m[0][0] = a.m[0][0];
    o.m[0][1] = a.m[1][0];
    o.m[1][0] = a.m[0][1];
    o.m[1][1] = a.m[1][1];
    return o;
}

// Rotation by theta as in helpers.cuh:265-276 (cos on the diagonal, [0][1] = -sin), and its derivative (helpers.cuh:278-289)
__device__ __forceinline__ M2 rotation(float cs, float sn) { return M2{{{cs, -sn}, {sn, cs}}}; }
__device__ __forceinline__ M2 rotation_grad(float cs, float sn) { return M2{{{-sn, -cs}, {cs, -sn}}}; }
__device__ __forceinline__ M2 diag(float a, float b) { return M2{{{a, 0.f}, {0.f, b}}}; }

// Gradients of one Gaussian's projection (the reference's backward2d.cu:53-100 with helpers.cuh:71-82, term by term)
struct ProjectionGrad {
    float cov2d[3];  // v_cov2d = -X G X (X the conic, G from v_conic with its off-diagonal used as is): G11, G12 + G21, G22
    float2 mean2d;   // v_xy scaled by the image size (W, H)
    float2 scale;    // v_cov2d contracted with dSigma / ds, the off-diagonal weighted by 2
    float rot;       // v_cov2d contracted with dSigma / dtheta, the off-diagonal weighted by 2
};

// conic and v_conic: three floats each (upper triangle)
__device__ __forceinline__ ProjectionGrad projection_grad(const float2 s, const float theta, const float img_w, const float img_h,
                                                          const float *conic, const float *v_conic, const float2 vxy) {
    const float x = conic[0], y = conic[1], z = conic[2];
    const float gx = v_conic[0], gy = v_conic[1], gz = v_conic[2];
    const M2 X{{{x, y}, {y, z}}};
    const M2 G{{{gx, gy}, {gy, gz}}};
    const M2 negX{{{-x, -y}, {-y, -z}}};
    const M2 V = mul(mul(negX, G), X);
    const float G11 = V.m[0][0], G12 = V.m[1][0] + V.m[0][1], G22 = V.m[1][1];

    const float cs = cosf(theta), sn = sinf(theta);
    const M2 R = rotation(cs, sn);
    const M2 Rg = rotation_grad(cs, sn);
    const M2 S = diag(s.x, s.y);
    const M2 M = mul(R, S);
    const M2 t1 = mul(mul(Rg, S), transpose(M));
    const M2 t2 = mul(mul(M, transpose(S)), transpose(Rg));
    M2 th;
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int r = 0; r < 2; ++r) th.m[c][r] = t1.m[c][r] + t2.m[c][r];
    const M2 sxg = mul(mul(R, diag(2.f * s.x, 0.f)), transpose(R));
    const M2 syg = mul(mul(R, diag(0.f, 2.f * s.y)), transpose(R));

    ProjectionGrad out;
    out.cov2d[0] = G11;
    out.cov2d[1] = G12;
    out.cov2d[2] = G22;
    out.scale = make_float2(G11 * sxg.m[0][0] + 2 * G12 * sxg.m[0][1] + G22 * sxg.m[1][1],
                            G11 * syg.m[0][0] + 2 * G12 * syg.m[0][1] + G22 * syg.m[1][1]);
    out.rot = G11 * th.m[0][0] + 2 * G12 * th.m[0][1] + G22 * th.m[1][1];
    out.mean2d = make_float2(vxy.x * img_w, vxy.y * img_h);
    return out;
}

}  // namespace igs
