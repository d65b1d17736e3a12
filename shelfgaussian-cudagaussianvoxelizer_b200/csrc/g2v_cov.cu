// g2v_cov.cu -- standalone covariance-from-(scale, rotation) kernels, forward and backward.
//
// Sigma = R(q) diag(s)^2 R(q)^T per Gaussian (reference test/gaussian_voxelizer.py:14-37), and the
// chain rule from dL/dSigma to dL/ds, dL/dq (g2v_cov.cuh).  One thread per Gaussian; HBM-bound
// (forward 28 B in, 36 B out; backward 64 B in, 28 B out per Gaussian).  The voxelizer's fused paths
// (g2v_forward_prepare_plan_sr / g2v_backward_sr) evaluate the same device functions inside the box
// preparation and the gradient reduction, so they never materialise Sigma or dL/dSigma.
#include "g2v_cov.cuh"
#include "g2v_internal.cuh"

namespace g2v {

namespace {
__global__ void __launch_bounds__(256) cov_from_scale_rot_kernel(const float* __restrict__ scales,
                                                                 const float* __restrict__ quats, int64_t n,
                                                                 float* __restrict__ cov) {
    const int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (g >= n) return;
    const float s[3] = {scales[g * 3 + 0], scales[g * 3 + 1], scales[g * 3 + 2]};
    const float q[4] = {quats[g * 4 + 0], quats[g * 4 + 1], quats[g * 4 + 2], quats[g * 4 + 3]};
    float S[9];
    scale_rot_to_cov(s, q, S);
#pragma unroll
    for (int k = 0; k < 9; ++k) cov[g * 9 + k] = S[k];
}

__global__ void __launch_bounds__(256) cov_from_scale_rot_backward_kernel(const float* __restrict__ scales,
                                                                          const float* __restrict__ quats,
                                                                          const float* __restrict__ grad_cov,
                                                                          int64_t n, float* __restrict__ grad_scales,
                                                                          float* __restrict__ grad_quats) {
    const int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (g >= n) return;
    const float s[3] = {scales[g * 3 + 0], scales[g * 3 + 1], scales[g * 3 + 2]};
    const float q[4] = {quats[g * 4 + 0], quats[g * 4 + 1], quats[g * 4 + 2], quats[g * 4 + 3]};
    float G[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) G[k] = grad_cov[g * 9 + k];
    float gs[3], gq[4];
    scale_rot_grad(s, q, G, gs, gq);
#pragma unroll
    for (int k = 0; k < 3; ++k) grad_scales[g * 3 + k] = gs[k];
#pragma unroll
    for (int k = 0; k < 4; ++k) grad_quats[g * 4 + k] = gq[k];
}
}  // namespace

int launch_cov_from_scale_rot(const float* scales, const float* quats, int64_t n, float* cov, cudaStream_t s) {
    if (n == 0) return 0;
    const int64_t blocks = (n + 255) / 256;
    G2V_TIMED("cov_from_scale_rot_kernel", s,
              (cov_from_scale_rot_kernel<<<(unsigned)blocks, 256, 0, s>>>(scales, quats, n, cov)));
    G2V_LAUNCH_CHECK("cov_from_scale_rot_kernel");
    return 0;
}

int launch_cov_from_scale_rot_backward(const float* scales, const float* quats, const float* grad_cov, int64_t n,
                                       float* grad_scales, float* grad_quats, cudaStream_t s) {
    if (n == 0) return 0;
    const int64_t blocks = (n + 255) / 256;
    G2V_TIMED("cov_from_scale_rot_backward_kernel", s,
              (cov_from_scale_rot_backward_kernel<<<(unsigned)blocks, 256, 0, s>>>(scales, quats, grad_cov, n,
                                                                                  grad_scales, grad_quats)));
    G2V_LAUNCH_CHECK("cov_from_scale_rot_backward_kernel");
    return 0;
}

}  // namespace g2v
