// g2v_cov.cuh -- covariance from per-Gaussian scale and rotation quaternion, and its gradient.
//
// The front end of GaussTR-style pipelines (reference test/gaussian_voxelizer.py:14-37, quat_to_rotmat and
// get_covariance, as called by GaussianVoxelizer.forward :176-177):
//     q = (r, x, y, z) / |q|,   R = the rotation matrix of q,   M = R diag(s),   Sigma = M M^T.
// Every operation is an explicit round-to-nearest intrinsic, so the result does not depend on the
// translation unit's flags (the preparation kernel's unit is built with --use_fast_math for the box rule,
// the standalone kernels' unit without): the fused and the standalone paths give the same bits.
//
// Gradient: with G = dL/dSigma over the nine entries taken as independent (the voxelizer's grad_cov),
// dL/dM = (G + G^T) M, dL/ds_j = sum_i dL/dM_ij R_ij, dL/dR_ij = dL/dM_ij s_j, dL/dq_hat from the
// polynomial entries of R, and dL/dq = (dL/dq_hat - q_hat (q_hat . dL/dq_hat)) / |q|.
#pragma once

namespace g2v {

struct QuatRot {
    float r, x, y, z;  // normalised quaternion
    float norm;        // |q|
    float R[9];        // row-major rotation
};

__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }

__device__ __forceinline__ QuatRot quat_rot(const float q[4]) {
    QuatRot o;
    const float n2 = add_rn(add_rn(add_rn(mul_rn(q[0], q[0]), mul_rn(q[1], q[1])), mul_rn(q[2], q[2])),
                            mul_rn(q[3], q[3]));
    o.norm = __fsqrt_rn(n2);
    o.r = __fdiv_rn(q[0], o.norm);
    o.x = __fdiv_rn(q[1], o.norm);
    o.y = __fdiv_rn(q[2], o.norm);
    o.z = __fdiv_rn(q[3], o.norm);
    const float r = o.r, x = o.x, y = o.y, z = o.z;
    const float xx = mul_rn(x, x), yy = mul_rn(y, y), zz = mul_rn(z, z);
    const float xy = mul_rn(x, y), xz = mul_rn(x, z), yz = mul_rn(y, z);
    const float rx = mul_rn(r, x), ry = mul_rn(r, y), rz = mul_rn(r, z);
    o.R[0] = sub_rn(1.f, mul_rn(2.f, add_rn(yy, zz)));
    o.R[1] = mul_rn(2.f, sub_rn(xy, rz));
    o.R[2] = mul_rn(2.f, add_rn(xz, ry));
    o.R[3] = mul_rn(2.f, add_rn(xy, rz));
    o.R[4] = sub_rn(1.f, mul_rn(2.f, add_rn(xx, zz)));
    o.R[5] = mul_rn(2.f, sub_rn(yz, rx));
    o.R[6] = mul_rn(2.f, sub_rn(xz, ry));
    o.R[7] = mul_rn(2.f, add_rn(yz, rx));
    o.R[8] = sub_rn(1.f, mul_rn(2.f, add_rn(xx, yy)));
    return o;
}

// Sigma (row-major 3x3) from scales s[3] and quaternion q[4] = (r, x, y, z).
__device__ __forceinline__ void scale_rot_to_cov(const float s[3], const float q[4], float S[9]) {
    const QuatRot Q = quat_rot(q);
    float M[9];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) M[i * 3 + j] = mul_rn(Q.R[i * 3 + j], s[j]);
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            S[i * 3 + j] = __fmaf_rn(M[i * 3 + 2], M[j * 3 + 2],
                                     __fmaf_rn(M[i * 3 + 1], M[j * 3 + 1], mul_rn(M[i * 3 + 0], M[j * 3 + 0])));
}

// dL/ds (3) and dL/dq (4) from G = dL/dSigma (row-major 3x3, entries independent).
__device__ __forceinline__ void scale_rot_grad(const float s[3], const float q[4], const float G[9], float gs[3],
                                               float gq[4]) {
    const QuatRot Q = quat_rot(q);
    float M[9], H[9];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            M[i * 3 + j] = mul_rn(Q.R[i * 3 + j], s[j]);
            H[i * 3 + j] = add_rn(G[i * 3 + j], G[j * 3 + i]);  // G + G^T
        }
    float gR[9];
#pragma unroll
    for (int j = 0; j < 3; ++j) gs[j] = 0.f;
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            // dL/dM_ij = sum_k H_ik M_kj
            const float gm = __fmaf_rn(H[i * 3 + 2], M[2 * 3 + j],
                                       __fmaf_rn(H[i * 3 + 1], M[1 * 3 + j], mul_rn(H[i * 3 + 0], M[0 * 3 + j])));
            gs[j] = __fmaf_rn(gm, Q.R[i * 3 + j], gs[j]);
            gR[i * 3 + j] = mul_rn(gm, s[j]);
        }
    const float r = Q.r, x = Q.x, y = Q.y, z = Q.z;
    // dR/d(r, x, y, z) of the entries of quat_rot, contracted with gR
    const float a13 = sub_rn(gR[3], gR[1]), p13 = add_rn(gR[1], gR[3]);
    const float a26 = sub_rn(gR[2], gR[6]), p26 = add_rn(gR[2], gR[6]);
    const float a75 = sub_rn(gR[7], gR[5]), p57 = add_rn(gR[5], gR[7]);
    const float p48 = add_rn(gR[4], gR[8]), p08 = add_rn(gR[0], gR[8]), p04 = add_rn(gR[0], gR[4]);
    const float gr = mul_rn(2.f, __fmaf_rn(z, a13, __fmaf_rn(y, a26, mul_rn(x, a75))));
    const float gx = mul_rn(2.f, __fmaf_rn(y, p13, __fmaf_rn(z, p26, __fmaf_rn(r, a75, mul_rn(-2.f * x, p48)))));
    const float gy = mul_rn(2.f, __fmaf_rn(x, p13, __fmaf_rn(r, a26, __fmaf_rn(z, p57, mul_rn(-2.f * y, p08)))));
    const float gz = mul_rn(2.f, __fmaf_rn(r, a13, __fmaf_rn(x, p26, __fmaf_rn(y, p57, mul_rn(-2.f * z, p04)))));
    // through the normalisation q_hat = q / |q|
    const float dot = __fmaf_rn(z, gz, __fmaf_rn(y, gy, __fmaf_rn(x, gx, mul_rn(r, gr))));
    const float inv = __fdiv_rn(1.f, Q.norm);
    gq[0] = mul_rn(__fmaf_rn(-r, dot, gr), inv);
    gq[1] = mul_rn(__fmaf_rn(-x, dot, gx), inv);
    gq[2] = mul_rn(__fmaf_rn(-y, dot, gy), inv);
    gq[3] = mul_rn(__fmaf_rn(-z, dot, gz), inv);
}

}  // namespace g2v
