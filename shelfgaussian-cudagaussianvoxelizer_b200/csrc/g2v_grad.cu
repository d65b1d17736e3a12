// g2v_grad.cu -- backward of the splat (FP32-FMA variant), atomic-free and deterministic.
//
// With w_gv = o_g exp(-1/2 d^T P_g d), D_v = sum_g w_gv, den_v = max(D_v, 1e-6) and
// F_vc = sum_g w_gv f_gc / den_v, the upstream gradients gD_v, gF_vc give (reference
// ComputeGaussian2VoxelGradientTileWithFeats, src/cuda_gaussian_voxelizer.cu:1376-1482):
//   S_gv   = sum_c gF_vc f_gc
//   e_v    = sum_c gF_vc F_vc = sum_g (w_gv / den_v) S_gv
//   a_gv   = gD_v + (S_gv - [D_v >= eps] e_v) / den_v              (dL/dw_gv)
//   dmu_g  = sum_v a_gv w_gv P d          dSigma_g = 1/2 sum_v a_gv w_gv (P d)(P d)^T
//   do_g   = sum_v a_gv exp(...)          df_g     = sum_v gF_v w_gv / den_v
// The reference reads F back and forms e_v with a batched GEMM (cu:1996); here e_v comes from the
// S_gv that the tile pass computes anyway, so grid_feats is never read.
//
// Passes:
//   S-pass  one CTA per tile: S (64 voxels x K Gaussians, contraction over C), e_v, a_gv and the ten
//           scalar gradient partials of every (Gaussian, tile) pair, written at the pair's position
//           in the Gaussian->Tile CSR.
//   F-pass  one CTA per (block of tiles, 64 channels): df partial rows of every (Gaussian, block) pair.
//   reduce  per Gaussian, in CSR order: sums of the pair partials -> the output gradients.
#include <algorithm>

#include "g2v_cov.cuh"
#include "g2v_internal.cuh"

namespace g2v {

namespace {
constexpr int kThreads = 256;
constexpr int kChunk = 64;       // Gaussians per chunk of the S-pass
constexpr int kCh = 32;          // channels per GEMM step
constexpr int kSKeep = 256;      // lists up to this length keep S in shared memory between the phases
constexpr int kFChunk = 256;     // Gaussians per accumulation round of the F-pass
constexpr int kFCh = 64;         // channels per F-pass CTA

struct Params {
    float mx, my, mz, op;
    float c[9];
    int lb[3], ub[3];
};

__device__ __forceinline__ void load_params(Params* P, const int32_t* __restrict__ list, int k0, int kc,
                                            const float* __restrict__ means, const float* __restrict__ opacity,
                                            const float* __restrict__ cov_inv, const int32_t* __restrict__ lb,
                                            const int32_t* __restrict__ ub, int* gid) {
    for (int k = threadIdx.x; k < kc; k += blockDim.x) {
        const int64_t g = list[k0 + k];
        gid[k] = (int)g;
        Params p;
        p.mx = means[g * 3 + 0];
        p.my = means[g * 3 + 1];
        p.mz = means[g * 3 + 2];
        p.op = opacity[g];
#pragma unroll
        for (int j = 0; j < 9; ++j) p.c[j] = cov_inv[g * 9 + j];
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            p.lb[a] = lb[g * 3 + a];
            p.ub[a] = ub[g * 3 + a];
        }
        P[k] = p;
    }
}

__device__ __forceinline__ bool in_box(const Params& p, int x, int y, int z) {
    return x >= p.lb[0] && x <= p.ub[0] && y >= p.lb[1] && y <= p.ub[1] && z >= p.lb[2] && z <= p.ub[2];
}

struct SPassSmem {
    Params P[kChunk];
    int gid[kChunk];
    alignas(16) float Fs[kCh][kChunk];       // features slice [channel][gaussian]; read as float4
    alignas(16) float Gs[kCh][kVoxPerTile];  // upstream grid-feature gradient slice [channel][voxel]
    float S[kChunk][kVoxPerTile];   // S of the chunk [gaussian][voxel]
    float gD[kVoxPerTile], den[kVoxPerTile], e[kVoxPerTile], act[kVoxPerTile];
    int vox_ok[kVoxPerTile];
    int64_t vrow[kVoxPerTile];      // linear voxel index
    float red[4][kChunk][10];
};

// S[k][v] = sum_c f[gid_k][c] * gF[v][c] for the chunk (SIMT 4x4 register blocking).
__device__ void s_gemm(SPassSmem& sm, int kc, const float* __restrict__ features,
                       const float* __restrict__ grad_feats, int C) {
    const int tid = threadIdx.x;
    const int tk = tid >> 4, tv = tid & 15;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    const int r = tid >> 2, cb = (tid & 3) * 8;
    for (int c0 = 0; c0 < C; c0 += kCh) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int c = c0 + cb + q;
            sm.Fs[cb + q][r] = (r < kc && c < C) ? features[(int64_t)sm.gid[r] * C + c] : 0.0f;
            sm.Gs[cb + q][r] = (sm.vox_ok[r] && c < C) ? grad_feats[sm.vrow[r] * C + c] : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int cc = 0; cc < kCh; ++cc) {
            const float4 a = *reinterpret_cast<const float4*>(&sm.Fs[cc][tk * 4]);
            const float4 b = *reinterpret_cast<const float4*>(&sm.Gs[cc][tv * 4]);
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) sm.S[tk * 4 + i][tv * 4 + j] = acc[i][j];
    __syncthreads();
}

__global__ void __launch_bounds__(kThreads) spass_kernel(
    const float* __restrict__ grad_density, const float* __restrict__ grad_feats,
    const float* __restrict__ means, const float* __restrict__ opacity, const float* __restrict__ cov_inv,
    const int32_t* __restrict__ lb, const int32_t* __restrict__ ub, const float* __restrict__ features, int C,
    const float* __restrict__ density, const int32_t* __restrict__ g2t_offsets,
    const int32_t* __restrict__ tile_offsets, const int32_t* __restrict__ tile_lists, int first_tile, Grid G,
    float* __restrict__ partial10, int64_t pair_cap) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SPassSmem& sm = *reinterpret_cast<SPassSmem*>(smem_raw);
    float* Skeep = reinterpret_cast<float*>(smem_raw + ((sizeof(SPassSmem) + 15) & ~size_t(15)));  // [K][64]

    const int tile = first_tile + blockIdx.x;
    int tx, ty, tz;
    decode_tile(tile, G, tx, ty, tz);
    const int x0 = tx * kTile, y0 = ty * kTile, z0 = tz * kTile;
    const int s = tile_offsets[blockIdx.x], K = tile_offsets[blockIdx.x + 1] - s;
    if (K == 0) return;
    const int tid = threadIdx.x;
    const bool keep = K <= kSKeep;
    const bool feats = C > 0;
    if (tid < kVoxPerTile) {
        int lx, ly, lz;
        local_voxel(tid, lx, ly, lz);
        const int x = x0 + lx, y = y0 + ly, z = z0 + lz;
        const bool ok = x < G.dims[0] && y < G.dims[1] && z < G.dims[2];
        const int64_t row = ok ? grid_row(G, x, y, z) : 0;
        sm.vox_ok[tid] = ok;
        sm.vrow[tid] = row;
        const float D = ok ? density[row] : 0.0f;
        sm.gD[tid] = ok ? grad_density[row] : 0.0f;
        sm.den[tid] = fmaxf(D, kEps);
        sm.act[tid] = D >= kEps ? 1.0f : 0.0f;
        sm.e[tid] = 0.0f;
    }
    __syncthreads();

    // phase 1: e_v = sum_g (w_gv / den_v) S_gv
    if (feats) {
        for (int k0 = 0; k0 < K; k0 += kChunk) {
            const int kc = min(kChunk, K - k0);
            load_params(sm.P, tile_lists + s, k0, kc, means, opacity, cov_inv, lb, ub, sm.gid);
            __syncthreads();
            s_gemm(sm, kc, features, grad_feats, C);
            if (keep)
                for (int i = tid; i < kc * kVoxPerTile; i += kThreads)
                    Skeep[(k0 + i / kVoxPerTile) * kVoxPerTile + (i % kVoxPerTile)] =
                        sm.S[i / kVoxPerTile][i % kVoxPerTile];
            if (tid < kVoxPerTile) {
                int lx, ly, lz;
                local_voxel(tid, lx, ly, lz);
                const int x = x0 + lx, y = y0 + ly, z = z0 + lz;
                const float cx = voxel_centre(G, 0, x), cy = voxel_centre(G, 1, y), cz = voxel_centre(G, 2, z);
                const float rden = 1.0f / sm.den[tid];
                float ev = sm.e[tid];
                for (int k = 0; k < kc; ++k) {
                    const Params& p = sm.P[k];
                    if (!in_box(p, x, y, z)) continue;
                    float qx, qy, qz;
                    const float ex = eval_gaussian(p.c, cx - p.mx, cy - p.my, cz - p.mz, qx, qy, qz);
                    ev = fmaf(p.op * ex * rden, sm.S[k][tid], ev);
                }
                sm.e[tid] = ev;
            }
            __syncthreads();
        }
    }

    // phase 2: a_gv and the ten gradient partials of each (Gaussian, tile) pair
    for (int k0 = 0; k0 < K; k0 += kChunk) {
        const int kc = min(kChunk, K - k0);
        load_params(sm.P, tile_lists + s, k0, kc, means, opacity, cov_inv, lb, ub, sm.gid);
        __syncthreads();
        if (feats) {
            if (keep) {
                for (int i = tid; i < kc * kVoxPerTile; i += kThreads)
                    sm.S[i / kVoxPerTile][i % kVoxPerTile] =
                        Skeep[(k0 + i / kVoxPerTile) * kVoxPerTile + (i % kVoxPerTile)];
                __syncthreads();
            } else {
                s_gemm(sm, kc, features, grad_feats, C);
            }
        }
        const int k = tid & 63, quarter = tid >> 6;
        float gr[10];
#pragma unroll
        for (int j = 0; j < 10; ++j) gr[j] = 0.0f;
        if (k < kc) {
            const Params& p = sm.P[k];
            for (int v = quarter * 16; v < quarter * 16 + 16; ++v) {
                int lx, ly, lz;
                local_voxel(v, lx, ly, lz);
                const int x = x0 + lx, y = y0 + ly, z = z0 + lz;
                if (!in_box(p, x, y, z)) continue;
                float qx, qy, qz;
                const float ex = eval_gaussian(p.c, voxel_centre(G, 0, x) - p.mx, voxel_centre(G, 1, y) - p.my,
                                               voxel_centre(G, 2, z) - p.mz, qx, qy, qz);
                float a = sm.gD[v];
                if (feats) a += (sm.S[k][v] - sm.act[v] * sm.e[v]) / sm.den[v];
                const float aw = a * p.op * ex;
                gr[0] = fmaf(aw, qx, gr[0]);
                gr[1] = fmaf(aw, qy, gr[1]);
                gr[2] = fmaf(aw, qz, gr[2]);
                const float h = 0.5f * aw;
                gr[3] = fmaf(h * qx, qx, gr[3]);
                gr[4] = fmaf(h * qy, qy, gr[4]);
                gr[5] = fmaf(h * qz, qz, gr[5]);
                gr[6] = fmaf(h * qx, qy, gr[6]);
                gr[7] = fmaf(h * qx, qz, gr[7]);
                gr[8] = fmaf(h * qy, qz, gr[8]);
                gr[9] = fmaf(a, ex, gr[9]);
            }
        }
#pragma unroll
        for (int j = 0; j < 10; ++j) sm.red[quarter][k][j] = gr[j];
        __syncthreads();
        if (tid < kc) {
            const int g = sm.gid[tid];
            const Params& p = sm.P[tid];
            // position of this tile inside the Gaussian's x-major tile box
            const int tlx = p.lb[0] / kTile, tly = p.lb[1] / kTile, tlz = p.lb[2] / kTile;
            const int ey = p.ub[1] / kTile - tly + 1, ez = p.ub[2] / kTile - tlz + 1;
            const int64_t idx = (int64_t)g2t_offsets[g] + ((tx - tlx) * ey + (ty - tly)) * ez + (tz - tlz);
            if (idx < pair_cap) {  // offsets come from the caller
                float* out = partial10 + idx * 10;
#pragma unroll
                for (int j = 0; j < 10; ++j)
                    out[j] = ((sm.red[0][tid][j] + sm.red[1][tid][j]) + sm.red[2][tid][j]) + sm.red[3][tid][j];
            }
        }
        __syncthreads();
    }
}

// F-pass: df partial row of every (Gaussian, block) pair for 64 channels.
struct FParams {
    float mx, my, mz, op;
    float c[9];
    int lb[3], ub[3];
};

__global__ void __launch_bounds__(kThreads) fpass_kernel(
    const float* __restrict__ grad_feats, const float* __restrict__ means, const float* __restrict__ opacity,
    const float* __restrict__ cov_inv, const int32_t* __restrict__ lb, const int32_t* __restrict__ ub, int C,
    const float* __restrict__ density, const int32_t* __restrict__ block_offsets,
    const int32_t* __restrict__ block_lists, const int32_t* __restrict__ g2b_offsets, int bx_begin, int nby,
    int nbz, int BX, int BY, int BZ, int tx_begin, int tx_end, Grid G, float* __restrict__ partialF,
    int64_t block_pair_cap) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float* Wn = reinterpret_cast<float*>(smem_raw);                                  // [64 voxels][256]
    Params* P = reinterpret_cast<Params*>(smem_raw + sizeof(float) * kVoxPerTile * kFChunk);
    int* gid = reinterpret_cast<int*>(P + kFChunk);
    float* rden = reinterpret_cast<float*>(gid + kFChunk);                           // [64]
    int64_t* vrow = reinterpret_cast<int64_t*>(rden + kVoxPerTile);                  // [64]

    const int bl = blockIdx.x;
    const int bxr = bl / (nby * nbz), rem = bl - bxr * nby * nbz;
    const int by = rem / nbz, bz = rem - (rem / nbz) * nbz;
    const int bx = bx_begin + bxr;
    const int s = block_offsets[bl], Kb = block_offsets[bl + 1] - s;
    if (Kb == 0) return;
    const int tid = threadIdx.x;
    const int c = blockIdx.y * kFCh + (tid & 63);
    const int gg = tid >> 6;
    const int txa = max(bx * BX, tx_begin), txb = min(bx * BX + BX, min(tx_end, G.tiles[0]));
    const int tya = by * BY, tyb = min(tya + BY, G.tiles[1]);
    const int tza = bz * BZ, tzb = min(tza + BZ, G.tiles[2]);

    for (int k0 = 0; k0 < Kb; k0 += kFChunk) {
        const int kc = min(kFChunk, Kb - k0);
        load_params(P, block_lists + s, k0, kc, means, opacity, cov_inv, lb, ub, gid);
        float acc[64];
#pragma unroll
        for (int j = 0; j < 64; ++j) acc[j] = 0.0f;
        __syncthreads();
        for (int tx = txa; tx < txb; ++tx)
            for (int ty = tya; ty < tyb; ++ty)
                for (int tz = tza; tz < tzb; ++tz) {
                    const int x0 = tx * kTile, y0 = ty * kTile, z0 = tz * kTile;
                    if (tid < kVoxPerTile) {
                        int lx, ly, lz;
                        local_voxel(tid, lx, ly, lz);
                        const int x = x0 + lx, y = y0 + ly, z = z0 + lz;
                        const bool ok = x < G.dims[0] && y < G.dims[1] && z < G.dims[2];
                        const int64_t row = ok ? grid_row(G, x, y, z) : -1;
                        vrow[tid] = row;
                        rden[tid] = ok ? 1.0f / fmaxf(density[row], kEps) : 0.0f;
                    }
                    __syncthreads();
                    {
                        const int v = tid & 63;
                        int lx, ly, lz;
                        local_voxel(v, lx, ly, lz);
                        const int x = x0 + lx, y = y0 + ly, z = z0 + lz;
                        const float cx = voxel_centre(G, 0, x), cy = voxel_centre(G, 1, y), cz = voxel_centre(G, 2, z);
                        const float rd = rden[v];
                        for (int k = tid >> 6; k < kFChunk; k += 4) {
                            float w = 0.0f;
                            if (k < kc) {
                                const Params& p = P[k];
                                if (in_box(p, x, y, z)) {
                                    float qx, qy, qz;
                                    const float ex = eval_gaussian(p.c, cx - p.mx, cy - p.my, cz - p.mz, qx, qy, qz);
                                    w = p.op * ex * rd;
                                }
                            }
                            Wn[v * kFChunk + k] = w;
                        }
                    }
                    __syncthreads();
                    if (c < C) {
                        for (int v = 0; v < kVoxPerTile; ++v) {
                            const int64_t row = vrow[v];
                            if (row < 0) continue;
                            const float gv = grad_feats[row * C + c];
                            const float4* wr = reinterpret_cast<const float4*>(&Wn[v * kFChunk + gg * 64]);
#pragma unroll
                            for (int q = 0; q < 16; ++q) {
                                const float4 w4 = wr[q];
                                acc[4 * q + 0] = fmaf(w4.x, gv, acc[4 * q + 0]);
                                acc[4 * q + 1] = fmaf(w4.y, gv, acc[4 * q + 1]);
                                acc[4 * q + 2] = fmaf(w4.z, gv, acc[4 * q + 2]);
                                acc[4 * q + 3] = fmaf(w4.w, gv, acc[4 * q + 3]);
                            }
                        }
                    }
                    __syncthreads();
                }
        if (c < C) {
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                const int k = gg * 64 + j;
                if (k < kc) {
                    const Params& p = P[k];
                    const int blx = (p.lb[0] / kTile) / BX, bly = (p.lb[1] / kTile) / BY, blz = (p.lb[2] / kTile) / BZ;
                    const int ey = (p.ub[1] / kTile) / BY - bly + 1, ez = (p.ub[2] / kTile) / BZ - blz + 1;
                    const int64_t idx = (int64_t)g2b_offsets[gid[k]] + ((bx - blx) * ey + (by - bly)) * ez + (bz - blz);
                    if (idx < block_pair_cap) partialF[idx * C + c] = acc[j];
                }
            }
        }
        __syncthreads();
    }
}

// Warp per Gaussian: sums the ten partials of its (Gaussian, tile) pairs whose tile lies in the slab.
// kScaleRot: instead of dL/dSigma, write dL/dscales (n,3) into grad_cov and dL/dquats (n,4) into
// grad_quats, by the chain rule through Sigma = R(q) diag(s)^2 R(q)^T (g2v_cov.cuh).
template <bool kScaleRot>
__global__ void __launch_bounds__(256) reduce10_kernel(const float* __restrict__ partial10,
                                                       const int32_t* __restrict__ g2t_offsets,
                                                       const int32_t* __restrict__ g2t_tile_ids, int64_t n,
                                                       int tyz, int tx_begin, int tx_end,
                                                       float* __restrict__ grad_means, float* __restrict__ grad_cov,
                                                       float* __restrict__ grad_opacity,
                                                       const float* __restrict__ scales,
                                                       const float* __restrict__ quats,
                                                       float* __restrict__ grad_quats) {
    const int64_t g = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (g >= n) return;
    float s[10];
#pragma unroll
    for (int j = 0; j < 10; ++j) s[j] = 0.0f;
    const int b = g2t_offsets[g], e = g2t_offsets[g + 1];
    for (int i = b + lane; i < e; i += 32) {
        const int tx = g2t_tile_ids[i] / tyz;
        if (tx < tx_begin || tx >= tx_end) continue;
#pragma unroll
        for (int j = 0; j < 10; ++j) s[j] += partial10[(int64_t)i * 10 + j];
    }
#pragma unroll
    for (int j = 0; j < 10; ++j)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s[j] += __shfl_xor_sync(0xffffffffu, s[j], o);
    if (lane == 0) {
        grad_means[g * 3 + 0] = s[0];
        grad_means[g * 3 + 1] = s[1];
        grad_means[g * 3 + 2] = s[2];
        const float Gc[9] = {s[3], s[6], s[7], s[6], s[4], s[8], s[7], s[8], s[5]};
        if (kScaleRot) {
            const float sc[3] = {scales[g * 3 + 0], scales[g * 3 + 1], scales[g * 3 + 2]};
            const float q[4] = {quats[g * 4 + 0], quats[g * 4 + 1], quats[g * 4 + 2], quats[g * 4 + 3]};
            float gs[3], gq[4];
            scale_rot_grad(sc, q, Gc, gs, gq);
#pragma unroll
            for (int k = 0; k < 3; ++k) grad_cov[g * 3 + k] = gs[k];
#pragma unroll
            for (int k = 0; k < 4; ++k) grad_quats[g * 4 + k] = gq[k];
        } else {
#pragma unroll
            for (int k = 0; k < 9; ++k) grad_cov[g * 9 + k] = Gc[k];
        }
        grad_opacity[g] = s[9];
    }
}

// CTA per Gaussian: sums its block partial rows (blocks with x in the slab's block range).  The rows of
// one block-x column are contiguous, so each thread streams a run of rows for its 4 channels with
// 16-byte loads and four independent accumulators (several loads in flight per thread); the sum is taken
// in row order, so results do not depend on the launch shape.
template <bool kVec>
__global__ void __launch_bounds__(256) reduce_feats_kernel(const float* __restrict__ partialF,
                                                           const int32_t* __restrict__ g2b_offsets,
                                                           const int32_t* __restrict__ lb,
                                                           const int32_t* __restrict__ ub, int C, int BX, int BY,
                                                           int BZ, int bx_begin, int bx_end,
                                                           float* __restrict__ grad_features, int64_t row_cap) {
    const int64_t g = blockIdx.x;
    int tlo[3], thi[3];
    bool ok = tile_box(lb, ub, g, tlo, thi);
    int blo[3] = {0, 0, 0}, ext[3] = {0, 0, 0};
    if (ok) {
        const int B[3] = {BX, BY, BZ};
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            blo[a] = tlo[a] / B[a];
            ext[a] = thi[a] / B[a] - blo[a] + 1;
        }
    }
    const int64_t base = g2b_offsets[g];
    const int run = ext[1] * ext[2];  // rows of one block-x column
    ok = ok && base + (int64_t)ext[0] * run <= row_cap;  // rows beyond a capped call's capacity: flagged, skipped
    if (kVec) {
        const int C4 = C >> 2;
        for (int c4 = threadIdx.x; c4 < C4; c4 += blockDim.x) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            if (ok) {
                for (int lx = 0; lx < ext[0]; ++lx) {
                    const int bx = blo[0] + lx;
                    if (bx < bx_begin || bx >= bx_end) continue;
                    const float4* p = reinterpret_cast<const float4*>(partialF + (base + (int64_t)lx * run) * C) + c4;
                    int j = 0;
                    for (; j + 4 <= run; j += 4) {
                        const float4 a0 = __ldg(p + (int64_t)(j + 0) * C4), a1 = __ldg(p + (int64_t)(j + 1) * C4);
                        const float4 a2 = __ldg(p + (int64_t)(j + 2) * C4), a3 = __ldg(p + (int64_t)(j + 3) * C4);
                        acc.x += a0.x; acc.y += a0.y; acc.z += a0.z; acc.w += a0.w;
                        acc.x += a1.x; acc.y += a1.y; acc.z += a1.z; acc.w += a1.w;
                        acc.x += a2.x; acc.y += a2.y; acc.z += a2.z; acc.w += a2.w;
                        acc.x += a3.x; acc.y += a3.y; acc.z += a3.z; acc.w += a3.w;
                    }
                    for (; j < run; ++j) {
                        const float4 a0 = __ldg(p + (int64_t)j * C4);
                        acc.x += a0.x; acc.y += a0.y; acc.z += a0.z; acc.w += a0.w;
                    }
                }
            }
            reinterpret_cast<float4*>(grad_features + g * C)[c4] = acc;
        }
    } else {
        for (int c = threadIdx.x; c < C; c += blockDim.x) {
            float acc = 0.0f;
            if (ok) {
                for (int lx = 0; lx < ext[0]; ++lx) {
                    const int bx = blo[0] + lx;
                    if (bx < bx_begin || bx >= bx_end) continue;
                    const int64_t r0 = base + (int64_t)lx * run;
                    for (int j = 0; j < run; ++j) acc += partialF[(r0 + j) * C + c];
                }
            }
            grad_features[g * C + c] = acc;
        }
    }
}
}  // namespace

size_t spass_smem_bytes(bool keep) {
    size_t b = (sizeof(SPassSmem) + 15) & ~size_t(15);
    if (keep) b += sizeof(float) * kSKeep * kVoxPerTile;
    return b;
}

size_t fpass_smem_bytes() {
    return sizeof(float) * kVoxPerTile * kFChunk + sizeof(Params) * kFChunk + sizeof(int) * kFChunk +
           sizeof(float) * kVoxPerTile + sizeof(int64_t) * kVoxPerTile;
}

int launch_spass(const float* grad_density, const float* grad_feats, const float* means, const float* opacity,
                 const float* cov_inv, const int32_t* lb, const int32_t* ub, const float* features, int C,
                 const float* density, const int32_t* g2t_offsets, const int32_t* tile_offsets,
                 const int32_t* tile_lists, int first_tile, int num_tiles, const Grid& G, float* partial10,
                 int64_t pair_cap, cudaStream_t s) {
    if (num_tiles <= 0) return 0;
    const size_t smem = spass_smem_bytes(C > 0);
    // per device; cheap enough to set on every call
    G2V_CUDA(cudaFuncSetAttribute(spass_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)spass_smem_bytes(true)));
    G2V_TIMED("spass_kernel", s, spass_kernel<<<num_tiles, kThreads, smem, s>>>(grad_density, grad_feats, means, opacity, cov_inv, lb, ub,
                                                   features, C, density, g2t_offsets, tile_offsets, tile_lists,
                                                   first_tile, G, partial10, pair_cap));
    G2V_LAUNCH_CHECK("spass_kernel");
    return 0;
}

int launch_fpass(const float* grad_feats, const float* means, const float* opacity, const float* cov_inv,
                 const int32_t* lb, const int32_t* ub, int C, const float* density, const int32_t* block_offsets,
                 const int32_t* block_lists, const int32_t* g2b_offsets, int bx_begin, int nbx, int nby, int nbz,
                 const int B[3], int tx_begin, int tx_end, const Grid& G, float* partialF, int64_t block_pair_cap,
                 cudaStream_t s) {
    const int64_t nblocks = (int64_t)nbx * nby * nbz;
    if (nblocks <= 0 || C <= 0) return 0;
    const size_t smem = fpass_smem_bytes();
    G2V_CUDA(cudaFuncSetAttribute(fpass_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((unsigned)nblocks, (unsigned)((C + kFCh - 1) / kFCh));
    G2V_TIMED("fpass_kernel", s, fpass_kernel<<<grid, kThreads, smem, s>>>(grad_feats, means, opacity, cov_inv, lb, ub, C, density, block_offsets,
                                              block_lists, g2b_offsets, bx_begin, nby, nbz, B[0], B[1], B[2],
                                              tx_begin, tx_end, G, partialF, block_pair_cap));
    G2V_LAUNCH_CHECK("fpass_kernel");
    return 0;
}

int launch_reduce10(const float* partial10, const int32_t* g2t_offsets, const int32_t* g2t_tile_ids, int64_t n,
                    const Grid& G, int tx_begin, int tx_end, float* grad_means, float* grad_cov,
                    float* grad_opacity, cudaStream_t s, const float* scales, const float* quats,
                    float* grad_quats) {
    if (n == 0) return 0;
    const unsigned blocks = (unsigned)((n * 32 + 255) / 256);
    if (scales)
        G2V_TIMED("reduce10_kernel", s,
                  (reduce10_kernel<true><<<blocks, 256, 0, s>>>(partial10, g2t_offsets, g2t_tile_ids, n,
                                                                G.tiles[1] * G.tiles[2], tx_begin, tx_end,
                                                                grad_means, grad_cov, grad_opacity, scales, quats,
                                                                grad_quats)));
    else
        G2V_TIMED("reduce10_kernel", s,
                  (reduce10_kernel<false><<<blocks, 256, 0, s>>>(partial10, g2t_offsets, g2t_tile_ids, n,
                                                                 G.tiles[1] * G.tiles[2], tx_begin, tx_end,
                                                                 grad_means, grad_cov, grad_opacity, nullptr,
                                                                 nullptr, nullptr)));
    G2V_LAUNCH_CHECK("reduce10_kernel");
    return 0;
}

int launch_reduce_feats(const float* partialF, const int32_t* g2b_offsets, const int32_t* lb, const int32_t* ub,
                        int64_t n, int C, const int B[3], int bx_begin, int bx_end, float* grad_features,
                        cudaStream_t s, int64_t row_cap) {
    if (n == 0 || C == 0) return 0;
    // 16-byte rows: C % 4 == 0 and 16-byte aligned bases (the partial rows live in the library's workspace)
    const bool vec = C % 4 == 0 && (reinterpret_cast<uintptr_t>(partialF) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(grad_features) & 15) == 0;
    const int threads = vec ? std::min(256, std::max(32, ((C / 4 + 31) / 32) * 32)) : 256;
    if (vec)
        G2V_TIMED("reduce_feats_kernel", s,
                  reduce_feats_kernel<true><<<(unsigned)n, threads, 0, s>>>(partialF, g2b_offsets, lb, ub, C, B[0],
                                                                            B[1], B[2], bx_begin, bx_end,
                                                                            grad_features, row_cap));
    else
        G2V_TIMED("reduce_feats_kernel", s,
                  reduce_feats_kernel<false><<<(unsigned)n, threads, 0, s>>>(partialF, g2b_offsets, lb, ub, C, B[0],
                                                                             B[1], B[2], bx_begin, bx_end,
                                                                             grad_features, row_cap));
    G2V_LAUNCH_CHECK("reduce_feats_kernel");
    return 0;
}

}  // namespace g2v
