// g2v_prep.cu -- per-Gaussian voxel box, tile count and inverse covariance.
//
// This translation unit is compiled with --use_fast_math, the flag the reference builds with
// (setup.py:19-20).  The box rule below must reproduce the reference's integer boxes bit for bit, and
// those depend on the rounding of sqrtf and '/' under that flag; using the same source-level
// operations under the same flags yields the same instructions.  The inverse uses the IEEE reciprocal
// intrinsic, so it is not affected by the flag.
#include "g2v_cov.cuh"
#include "g2v_internal.cuh"

namespace g2v {

// One thread per Gaussian.  Box rule of src/cuda_gaussian_voxelizer.cu:367-532: sigma = sqrt of the
// covariance diagonal, [mu - 3 sigma, mu + 3 sigma] clamped to the range, floor((v - v0) / h), clamped
// to the grid; an empty box gives lb = 0, ub = -1, zero counts and a zero inverse.  The tile count is
// the size of the tile box (voxel box / 4).  The inverse is the adjugate over the determinant, with
// |det| < 1e-6 replaced by +1e-6 (the reference's clamp, cu:201-220).
// kScaleRot: the covariance is formed in registers from scales (n,3) and rotation quaternions (n,4)
// (g2v_cov.cuh, the same bits as cov_from_scale_rot_kernel), `cov` is unused and `scales` / `quats` are
// read instead.
template <bool kScaleRot>
__global__ void __launch_bounds__(256) prepare_boxes_kernel(const float* __restrict__ means,
                                                            const float* __restrict__ cov,
                                                            const float* __restrict__ scales,
                                                            const float* __restrict__ quats, int64_t n, Grid G,
                                                            float* __restrict__ cov_inv, int32_t* __restrict__ lb,
                                                            int32_t* __restrict__ ub, int32_t* __restrict__ nvox,
                                                            int32_t* __restrict__ ntiles,
                                                            const int32_t* __restrict__ scene_offsets,
                                                            int num_scenes) {
    const int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (g >= n) return;
    // scene of this Gaussian (last b with scene_offsets[b] <= g) and the scene's x extent
    int scene = 0;
    if (scene_offsets) {
        int lo_b = 0, hi_b = num_scenes - 1;
        while (lo_b < hi_b) {
            const int mid = (lo_b + hi_b + 1) >> 1;
            if (scene_offsets[mid] <= g) lo_b = mid;
            else hi_b = mid - 1;
        }
        scene = lo_b;
    }
    const int dims_s[3] = {G.scene_x > 0 ? G.scene_x : G.dims[0], G.dims[1], G.dims[2]};
    const int tiles_s[3] = {G.scene_x > 0 ? G.scene_x / kTile : G.tiles[0], G.tiles[1], G.tiles[2]};
    float A[9];
    if (kScaleRot) {
        const float sc[3] = {scales[g * 3 + 0], scales[g * 3 + 1], scales[g * 3 + 2]};
        const float q[4] = {quats[g * 4 + 0], quats[g * 4 + 1], quats[g * 4 + 2], quats[g * 4 + 3]};
        scale_rot_to_cov(sc, q, A);
    } else {
#pragma unroll
        for (int k = 0; k < 9; ++k) A[k] = cov[g * 9 + k];
    }

    int lo[3], hi[3];
#pragma unroll
    for (int a = 0; a < 3; ++a) {
        const float mu = means[g * 3 + a];
        const float s = sqrtf(A[4 * a]);
        float lower = mu - 3.0f * s;
        float upper = mu + 3.0f * s;
        lower = fmaxf(lower, G.r0[a]);
        upper = fminf(upper, G.r1[a]);
        // float -> int conversion saturates and maps NaN to 0 on the GPU
        const int l = (int)floorf((lower - G.r0[a]) / G.h[a]);
        const int u = (int)floorf((upper - G.r0[a]) / G.h[a]);
        lo[a] = max(l, 0);
        hi[a] = min(u, dims_s[a] - 1);
    }
    const bool empty = lo[0] > hi[0] || lo[1] > hi[1] || lo[2] > hi[2];
    if (empty) {
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            lb[g * 3 + a] = 0;
            ub[g * 3 + a] = -1;
        }
        nvox[g] = 0;
        ntiles[g] = 0;
#pragma unroll
        for (int k = 0; k < 9; ++k) cov_inv[g * 9 + k] = 0.0f;
        return;
    }
    int tcount = 1, vcount = 1;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
        const int shift = a == 0 ? scene * dims_s[0] : 0;  // stacked-batch coordinates
        lb[g * 3 + a] = lo[a] + shift;
        ub[g * 3 + a] = hi[a] + shift;
        vcount *= hi[a] - lo[a] + 1;
        const int tl = max(lo[a] / kTile, 0);
        const int th = min(hi[a] / kTile, tiles_s[a] - 1);
        tcount *= th - tl + 1;
    }
    nvox[g] = vcount;
    ntiles[g] = tcount;

    // adjugate / determinant
    const float c00 = A[4] * A[8] - A[5] * A[7];
    const float c01 = A[3] * A[8] - A[5] * A[6];
    const float c02 = A[3] * A[7] - A[4] * A[6];
    float det = A[0] * c00 - A[1] * c01 + A[2] * c02;
    if (fabsf(det) < kEps) det = kEps;
    const float r = __frcp_rn(det);
    float* o = cov_inv + g * 9;
    o[0] = c00 * r;
    o[1] = (A[2] * A[7] - A[1] * A[8]) * r;
    o[2] = (A[1] * A[5] - A[2] * A[4]) * r;
    o[3] = -c01 * r;
    o[4] = (A[0] * A[8] - A[2] * A[6]) * r;
    o[5] = (A[2] * A[3] - A[0] * A[5]) * r;
    o[6] = c02 * r;
    o[7] = (A[1] * A[6] - A[0] * A[7]) * r;
    o[8] = (A[0] * A[4] - A[1] * A[3]) * r;
}

int launch_prepare_boxes(const float* means, const float* cov, int64_t n, const Grid& G, float* cov_inv,
                         int32_t* lb, int32_t* ub, int32_t* num_voxels, int32_t* num_tiles, cudaStream_t s,
                         const float* scales, const float* quats, const int32_t* scene_offsets, int num_scenes) {
    if (n == 0) return 0;
    const int threads = 256;
    const int64_t blocks = (n + threads - 1) / threads;
    if (scales)
        G2V_TIMED("prepare_boxes_kernel", s,
                  (prepare_boxes_kernel<true><<<(unsigned)blocks, threads, 0, s>>>(
                      means, nullptr, scales, quats, n, G, cov_inv, lb, ub, num_voxels, num_tiles, scene_offsets,
                      num_scenes)));
    else
        G2V_TIMED("prepare_boxes_kernel", s,
                  (prepare_boxes_kernel<false><<<(unsigned)blocks, threads, 0, s>>>(
                      means, cov, nullptr, nullptr, n, G, cov_inv, lb, ub, num_voxels, num_tiles, scene_offsets,
                      num_scenes)));
    G2V_LAUNCH_CHECK("prepare_boxes_kernel");
    return 0;
}

}  // namespace g2v
