// g2v_splat.cu -- forward splat, one CTA per tile (FP32-FMA variant).
//
// For the 64 voxels of a tile and the K Gaussians of its Tile->Gaussian list (ascending ids):
//   w_gv = opacity_g * exp(-1/2 d^T P_g d), d = voxel centre - mean, for v inside g's voxel box
//   D_v  = sum_g w_gv                                  (density, summed in list order)
//   F_vc = (sum_g w_gv f_gc) / max(D_v, 1e-6)          (normalised grid features)
// Every voxel of the tile is written exactly once (zeros where K = 0), so the grid needs no zero fill
// and no separate normalisation pass (the reference's zero_ and clamp_min/div_, cu:1793, 1848-1849).
// Reference kernels: ComputeGaussian2VoxelTileWithFeats cu:767-966, ComputeGaussian2VoxelTile cu:7-136.
//
// Work split: the list is walked in chunks of 64 Gaussians; per chunk the CTA evaluates the 64x64
// weight block into shared memory, then every thread owns one channel and accumulates its 64 voxels
// (64 FMAs per feature load, weights read as shared-memory broadcasts).  Channels are processed 256
// at a time; the weights are re-evaluated for each group of 256 channels.
#include "g2v_internal.cuh"

namespace g2v {

namespace {
constexpr int kThreads = 256;
constexpr int kChunk = 64;

struct __align__(16) SplatSmem {
    alignas(16) float W[kChunk][kVoxPerTile];  // weights of the chunk, [gaussian][voxel]; read as float4
    float D[kVoxPerTile];          // running density
    float mx[kChunk], my[kChunk], mz[kChunk], op[kChunk];
    float ci[9][kChunk];
    int lbx[kChunk], lby[kChunk], lbz[kChunk], ubx[kChunk], uby[kChunk], ubz[kChunk];
    int gid[kChunk];
};

__device__ __forceinline__ void load_chunk(SplatSmem& sm, const int32_t* __restrict__ list, int k0, int kc,
                                           const float* __restrict__ means, const float* __restrict__ opacity,
                                           const float* __restrict__ cov_inv, const int32_t* __restrict__ lb,
                                           const int32_t* __restrict__ ub) {
    for (int k = threadIdx.x; k < kc; k += kThreads) {
        const int g = list[k0 + k];
        sm.gid[k] = g;
        sm.mx[k] = means[(int64_t)g * 3 + 0];
        sm.my[k] = means[(int64_t)g * 3 + 1];
        sm.mz[k] = means[(int64_t)g * 3 + 2];
        sm.op[k] = opacity[g];
        sm.lbx[k] = lb[(int64_t)g * 3 + 0];
        sm.lby[k] = lb[(int64_t)g * 3 + 1];
        sm.lbz[k] = lb[(int64_t)g * 3 + 2];
        sm.ubx[k] = ub[(int64_t)g * 3 + 0];
        sm.uby[k] = ub[(int64_t)g * 3 + 1];
        sm.ubz[k] = ub[(int64_t)g * 3 + 2];
    }
    for (int i = threadIdx.x; i < kc * 9; i += kThreads) {
        const int k = i / 9, j = i - k * 9;
        sm.ci[j][k] = cov_inv[(int64_t)list[k0 + k] * 9 + j];
    }
}

// W[k][v] for the chunk; zero outside the Gaussian's box (which also excludes voxels beyond the grid).
__device__ __forceinline__ void eval_chunk(SplatSmem& sm, int kc, const Grid& G, int x0, int y0, int z0) {
    const int v = threadIdx.x & 63;
    int lx, ly, lz;
    local_voxel(v, lx, ly, lz);
    const int x = x0 + lx, y = y0 + ly, z = z0 + lz;
    const float cx = voxel_centre(G, 0, x), cy = voxel_centre(G, 1, y), cz = voxel_centre(G, 2, z);
    for (int k = threadIdx.x >> 6; k < kChunk; k += kThreads / 64) {
        float w = 0.0f;
        if (k < kc && x >= sm.lbx[k] && x <= sm.ubx[k] && y >= sm.lby[k] && y <= sm.uby[k] && z >= sm.lbz[k] &&
            z <= sm.ubz[k]) {
            const float c[9] = {sm.ci[0][k], sm.ci[1][k], sm.ci[2][k], sm.ci[3][k], sm.ci[4][k],
                                sm.ci[5][k], sm.ci[6][k], sm.ci[7][k], sm.ci[8][k]};
            float qx, qy, qz;
            const float e = eval_gaussian(c, cx - sm.mx[k], cy - sm.my[k], cz - sm.mz[k], qx, qy, qz);
            w = sm.op[k] * e;
        }
        sm.W[k][v] = w;
    }
}

template <bool kFeatures>
__global__ void __launch_bounds__(kThreads) splat_tile_kernel(
    const float* __restrict__ means, const float* __restrict__ opacity, const float* __restrict__ cov_inv,
    const int32_t* __restrict__ lb, const int32_t* __restrict__ ub, const float* __restrict__ features, int C,
    const int32_t* __restrict__ tile_offsets, const int32_t* __restrict__ tile_lists, int first_tile, Grid G,
    float* __restrict__ density, float* __restrict__ grid_feats, bool zero_density) {
    __shared__ SplatSmem sm;
    const int tile = first_tile + blockIdx.x;
    int tx, ty, tz;
    decode_tile(tile, G, tx, ty, tz);
    const int x0 = tx * kTile, y0 = ty * kTile, z0 = tz * kTile;
    const int s = tile_offsets[blockIdx.x], e = tile_offsets[blockIdx.x + 1];
    const int K = e - s;
    const int tid = threadIdx.x;
    if (tid < kVoxPerTile) sm.D[tid] = 0.0f;
    __syncthreads();

    if (!kFeatures) {
        for (int k0 = 0; k0 < K; k0 += kChunk) {
            const int kc = min(kChunk, K - k0);
            load_chunk(sm, tile_lists + s, k0, kc, means, opacity, cov_inv, lb, ub);
            __syncthreads();
            eval_chunk(sm, kc, G, x0, y0, z0);
            __syncthreads();
            if (tid < kVoxPerTile) {
                float d = sm.D[tid];
                for (int k = 0; k < kc; ++k) d += sm.W[k][tid];
                sm.D[tid] = d;
            }
            __syncthreads();
        }
    } else {
        for (int c0 = 0; c0 < C; c0 += kThreads) {
            const int c = c0 + tid;
            float acc[kVoxPerTile];
#pragma unroll
            for (int v = 0; v < kVoxPerTile; ++v) acc[v] = 0.0f;
            for (int k0 = 0; k0 < K; k0 += kChunk) {
                const int kc = min(kChunk, K - k0);
                load_chunk(sm, tile_lists + s, k0, kc, means, opacity, cov_inv, lb, ub);
                __syncthreads();
                eval_chunk(sm, kc, G, x0, y0, z0);
                __syncthreads();
                if (c0 == 0 && tid < kVoxPerTile) {
                    float d = sm.D[tid];
                    for (int k = 0; k < kc; ++k) d += sm.W[k][tid];
                    sm.D[tid] = d;
                }
                if (c < C) {
                    for (int k = 0; k < kc; ++k) {
                        const float f = features[(int64_t)sm.gid[k] * C + c];
                        const float4* wr = reinterpret_cast<const float4*>(&sm.W[k][0]);
#pragma unroll
                        for (int q = 0; q < kVoxPerTile / 4; ++q) {
                            const float4 w4 = wr[q];
                            acc[4 * q + 0] = fmaf(w4.x, f, acc[4 * q + 0]);
                            acc[4 * q + 1] = fmaf(w4.y, f, acc[4 * q + 1]);
                            acc[4 * q + 2] = fmaf(w4.z, f, acc[4 * q + 2]);
                            acc[4 * q + 3] = fmaf(w4.w, f, acc[4 * q + 3]);
                        }
                    }
                }
                __syncthreads();
            }
            if (c < C) {
                const int64_t sz = C, sy = (int64_t)G.dims[2] * C, sx = (int64_t)G.dims[1] * sy;
                float* base = grid_feats + grid_row(G, x0, y0, z0) * C + c;
                const int nx = min(kTile, G.dims[0] - x0), ny = min(kTile, G.dims[1] - y0),
                          nz = min(kTile, G.dims[2] - z0);
#pragma unroll
                for (int lx = 0; lx < kTile; ++lx) {
#pragma unroll
                    for (int ly = 0; ly < kTile; ++ly) {
                        float* row = base + lx * sx + ly * sy;
#pragma unroll
                        for (int lz = 0; lz < kTile; ++lz) {
                            const int v = (lx * kTile + ly) * kTile + lz;
                            if (lx < nx && ly < ny && lz < nz) row[lz * sz] = acc[v] / fmaxf(sm.D[v], kEps);
                        }
                    }
                }
            }
            __syncthreads();
        }
    }
    if (tid < kVoxPerTile) {
        int lx, ly, lz;
        local_voxel(tid, lx, ly, lz);
        const int x = x0 + lx, y = y0 + ly, z = z0 + lz;
        if (x < G.dims[0] && y < G.dims[1] && z < G.dims[2])
            density[grid_row(G, x, y, z)] = zero_density ? 0.0f : sm.D[tid];
    }
}
}  // namespace

// features == nullptr: density only.  features != nullptr with C == 0: density left at zero (the
// reference's density sum sits inside its channel loop).
int launch_splat_simt(const float* means, const float* opacity, const float* cov_inv, const int32_t* lb,
                      const int32_t* ub, const float* features, int C, const int32_t* tile_offsets,
                      const int32_t* tile_lists, int first_tile, int num_tiles, const Grid& G, float* density,
                      float* grid_feats, cudaStream_t s) {
    if (num_tiles <= 0) return 0;
    if (features == nullptr || C == 0) {
        G2V_TIMED("splat_tile_kernel", s, splat_tile_kernel<false><<<num_tiles, kThreads, 0, s>>>(means, opacity, cov_inv, lb, ub, nullptr, 0,
                                                                tile_offsets, tile_lists, first_tile, G, density,
                                                                nullptr, features != nullptr));
    } else {
        G2V_TIMED("splat_tile_kernel", s, splat_tile_kernel<true><<<num_tiles, kThreads, 0, s>>>(means, opacity, cov_inv, lb, ub, features, C,
                                                               tile_offsets, tile_lists, first_tile, G, density,
                                                               grid_feats, false));
    }
    G2V_LAUNCH_CHECK("splat_tile_kernel");
    return 0;
}

}  // namespace g2v
