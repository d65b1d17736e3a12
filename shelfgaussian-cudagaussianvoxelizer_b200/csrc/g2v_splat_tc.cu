// g2v_splat_tc.cu -- forward splat on the 5th-generation tensor cores (tcgen05, kind::f16).
//
// Per tile (64 voxels) and group of 512 channels, the feature sum is the contraction
//     S[c][v] = sum_k F[g_k][c] * w[v][k]       (C x K) . (K x 64)
// computed as D^T in TMEM: M = 128 channels per MMA (4 M-blocks, 256 TMEM columns), N = 64 voxels,
// K = 16 Gaussians per step.  fp32-level accuracy comes from splitting both operands into a half
// pair, x = hi + lo (~22 bits), and accumulating hi*hi + hi*lo + lo*hi in fp32 (the dropped lo*lo
// term is ~2^-22 relative).  Range: features are scaled per channel by a power of two so that a
// channel's max |f| lies in [2^14, 2^15); weights by a per-tile power of two from the tile's max
// |opacity| (w <= |opacity|).  The epilogue undoes both exactly and divides by max(D_v, 1e-6).
//
// Operands in shared memory:
//   A = F^T slice (128 channels x 16 Gaussians) MN-major, 128-byte swizzle: 64-channel x 8-Gaussian
//       atoms of 1 KB (LBO = 1 KB between the two channel halves, SBO = 2 KB between Gaussian octets),
//       gathered row by row from the split features with cp.async (16 B = 8 channels).
//   B = w slice (64 voxels x 16 Gaussians) K-major, no swizzle: 8x8 core matrices of 128 B
//       (LBO = 128 B between Gaussian octets, SBO = 256 B between voxel octets), written by the
//       threads that evaluate the weights.
// Roles (256 threads): threads 0-127 evaluate weights (voxel = t % 64, Gaussian octet = t / 64) and
// accumulate the density; threads 128-255 issue the feature gathers one step ahead; thread 0 issues
// the 12 MMAs of a step and commits them to the stage's mbarrier.  Three stages; every wait is bounded.
#include <cstddef>

#include "g2v_internal.cuh"
#include "g2v_tc.cuh"

namespace g2v {

namespace {
constexpr int kThreads = 288;          // 4 producer warps, 4 weight warps, 1 MMA warp
constexpr int kKStep = 16;
constexpr int kMB = 4;                   // M-blocks of 128 channels per CTA
constexpr int kChGroup = kMB * 128;      // channels per CTA
constexpr int kStages = 3;
constexpr int kABytes = kMB * 4096;      // one operand half (hi or lo), one stage
constexpr int kWBytes = 2048;
constexpr int kStageBytes = 2 * kABytes + 2 * kWBytes;
constexpr uint32_t kTmemCols = kMB * 64;
constexpr uint32_t kIdesc = tc::idesc_f16_f32(128, 64, /*a MN-major*/ 1, /*b K-major*/ 0);

// The producer threads stage the GParams records of the 16 Gaussians of a step one step ahead.
struct StepParams {
    GParams g[kKStep];
};

struct TcMisc {
    uint64_t full_a[kStages];   // the stage's A operand and Gaussian parameters landed (128 producer threads)
    uint64_t full_w[kStages];   // the stage's weights written (4 weight warps)
    uint64_t empty[kStages];    // the MMAs reading the stage completed
    uint64_t mma_done;
    uint32_t tmem_base;
    int fail;
    alignas(16) float vscale[kVoxPerTile];  // 1 / (max(D_v, eps) * weight scale); read as float4
    float red[(kThreads + 31) / 32];
    StepParams prm[kStages];
};
// Two CTAs per SM: 3 stages (108 KB) + TcMisc (4.3 KB) per CTA.  The 128-byte swizzle atoms need the
// dynamic shared memory to start on a 1024-byte boundary; the kernel checks that at run time.
constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + sizeof(TcMisc);
static_assert(offsetof(TcMisc, vscale) % 16 == 0 && offsetof(TcMisc, prm) % 16 == 0,
              "vector-accessed shared fields must be 16-byte aligned");
static_assert((kStages * kStageBytes) % 1024 == 0, "TcMisc must start 1024-byte aligned");
// 228 KB per SM, 1 KB of it reserved per resident CTA: two CTAs need <= 113 KB of dynamic smem each
static_assert(kSmemBytes <= (228 * 1024) / 2 - 1024, "splat_tc_kernel no longer fits two CTAs per SM");

__device__ __forceinline__ int pow2_exponent(float m) {
    // floor(log2(m)) for a finite m > 0
    int e;
    frexpf(m, &e);
    return e - 1;
}

// Per-channel max |f| (as float bits; non-negative floats order like integers).
__global__ void __launch_bounds__(256) feature_colmax_kernel(const float* __restrict__ f, int64_t n, int C,
                                                             int rows_per_block, unsigned* __restrict__ colmax) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    const int64_t r0 = (int64_t)blockIdx.y * rows_per_block;
    const int64_t r1 = min(n, r0 + rows_per_block);
    float m = 0.0f;
    for (int64_t r = r0; r < r1; ++r) m = fmaxf(m, fabsf(f[r * C + c]));
    atomicMax(&colmax[c], __float_as_uint(m));
}

// features (N, C) fp32 -> hi / lo halves (N, Cp) scaled by 2^k_c, and unscale[c] = 2^-k_c.
__global__ void __launch_bounds__(256) feature_split_kernel(const float* __restrict__ f, int64_t n, int C, int Cp,
                                                            const unsigned* __restrict__ colmax,
                                                            __half* __restrict__ hi, __half* __restrict__ lo,
                                                            float* __restrict__ unscale) {
    const int64_t chunks = (int64_t)Cp / 8;
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n * chunks) return;
    const int64_t r = i / chunks;
    const int c8 = (int)(i - r * chunks) * 8;
    __align__(16) __half h[8], l[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int c = c8 + j;
        float x = 0.0f;
        int k = 0;
        if (c < C) {
            x = f[r * C + c];
            const float m = __uint_as_float(colmax[c]);
            k = (m > 0.0f) ? max(-100, min(100, 14 - pow2_exponent(m))) : 0;
        }
        tc::split_half(ldexpf(x, k), h[j], l[j]);
        if (r == 0) unscale[c] = ldexpf(1.0f, -k);
    }
    *reinterpret_cast<uint4*>(hi + r * Cp + c8) = *reinterpret_cast<const uint4*>(h);
    *reinterpret_cast<uint4*>(lo + r * Cp + c8) = *reinterpret_cast<const uint4*>(l);
}

// Gaussian parameters packed as GParams records (the layout the weight threads read).
__global__ void __launch_bounds__(256) pack_params_kernel(const float* __restrict__ means,
                                                          const float* __restrict__ opacity,
                                                          const float* __restrict__ cov_inv,
                                                          const int32_t* __restrict__ lb, const int32_t* __restrict__ ub,
                                                          int64_t n, GParams* __restrict__ out) {
    const int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (g >= n) return;
    const float* P = cov_inv + g * 9;
    GParams r;
    r.w[0] = make_float4(means[g * 3], means[g * 3 + 1], means[g * 3 + 2], opacity[g]);
    r.w[1] = make_float4(P[0], P[1], P[2], P[3]);
    r.w[2] = make_float4(P[4], P[5], P[6], P[7]);
    r.w[3] = make_float4(P[8], __int_as_float(lb[g * 3]), __int_as_float(lb[g * 3 + 1]), __int_as_float(lb[g * 3 + 2]));
    r.w[4] = make_float4(__int_as_float(ub[g * 3]), __int_as_float(ub[g * 3 + 1]), __int_as_float(ub[g * 3 + 2]), 0.0f);
    out[g] = r;
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = 0.0f;
#pragma unroll
    for (int w = 0; w < (kThreads + 31) / 32; ++w) m = fmaxf(m, red[w]);
    __syncthreads();
    return m;
}

// Roles: warp 0 stages step i+1 (TMA gathers of the split features into the swizzled A layout, 4-byte
// cp.async of the Gaussian parameters); warp 1 (one thread) issues the 12 MMAs of a step once its A and
// w are ready and commits them to the stage's "empty" barrier; warps 2-5 evaluate the weights of a
// step.  No CTA-wide barrier in the main loop: stages hand over through mbarriers.
__global__ void __launch_bounds__(kThreads, 1) splat_tc_kernel(
    const __half* __restrict__ Fhi, const __half* __restrict__ Flo, const float* __restrict__ unscale, int C, int Cp,
    const GParams* __restrict__ gparams,
    const float* __restrict__ opacity, const int32_t* __restrict__ tile_offsets, const int32_t* __restrict__ tile_lists,
    int first_tile, int ngroups, Grid G, float* __restrict__ density, float* __restrict__ grid_feats,
    int* __restrict__ err) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* base = smem_raw;
    TcMisc& ms = *reinterpret_cast<TcMisc*>(base + kStages * kStageBytes);
    if ((tc::smem_u32(smem_raw) & 1023u) != 0) {  // never expected; fail loudly instead of mis-swizzling
        if (threadIdx.x == 0) atomicOr(err, 2);
        return;
    }

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tl = blockIdx.x / ngroups, grp = blockIdx.x - tl * ngroups;
    int tx, ty, tz;
    decode_tile(first_tile + tl, G, tx, ty, tz);
    const int x0 = tx * kTile, y0 = ty * kTile, z0 = tz * kTile;
    const int s = tile_offsets[tl], K = tile_offsets[tl + 1] - s;
    const int32_t* list = tile_lists + s;
    const int c0 = grp * kChGroup;
    const int nx = min(kTile, G.dims[0] - x0), ny = min(kTile, G.dims[1] - y0), nz = min(kTile, G.dims[2] - z0);
    const int64_t row0 = ((int64_t)x0 * G.dims[1] + y0) * G.dims[2] + z0;
    const int64_t sx = (int64_t)G.dims[1] * G.dims[2], sy = G.dims[2];

    if (K == 0) {  // no Gaussian reaches the tile: zeros
        for (int i = tid; i < kVoxPerTile * kChGroup; i += kThreads) {
            const int v = i / kChGroup, c = c0 + (i - v * kChGroup);
            int lx, ly, lz;
            local_voxel(v, lx, ly, lz);
            if (c < C && lx < nx && ly < ny && lz < nz) grid_feats[(row0 + lx * sx + ly * sy + lz) * C + c] = 0.0f;
        }
        if (grp == 0 && tid < kVoxPerTile) {
            int lx, ly, lz;
            local_voxel(tid, lx, ly, lz);
            if (lx < nx && ly < ny && lz < nz) density[row0 + lx * sx + ly * sy + lz] = 0.0f;
        }
        return;
    }

    // per-tile weight scale: |w| <= |opacity|
    float om = 0.0f;
    for (int k = tid; k < K; k += kThreads) om = fmaxf(om, fabsf(opacity[list[k]]));
    om = block_max(om, ms.red);
    const int kt = (om > 0.0f) ? max(-100, min(100, 14 - pow2_exponent(om))) : 0;
    const float wscale = ldexpf(1.0f, kt);

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            tc::mbar_init(&ms.full_a[i], 128);
            tc::mbar_init(&ms.full_w[i], 4);
            tc::mbar_init(&ms.empty[i], 1);
        }
        tc::mbar_init(&ms.mma_done, 1);
        tc::mbar_fence_init();
        ms.fail = 0;
    }
    if (warp == 0) tc::tmem_alloc(&ms.tmem_base, kTmemCols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = ms.tmem_base;
    const int nsteps = (K + kKStep - 1) / kKStep;
    bool ok = true;
    float dsum[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // weight threads: density partials of their z-line
    int dline = 0, dkp = 0;

    auto a_stage = [&](int st, int hl) -> uint32_t {
        return tc::smem_u32(base + st * kStageBytes + hl * kABytes);
    };
    auto w_stage = [&](int st, int hl) -> unsigned char* {
        return base + st * kStageBytes + 2 * kABytes + hl * kWBytes;
    };

    if (warp < 4) {
        // ---------------- producer warps: thread = (operand half, 8-channel chunk) ----------------
        const int hl = tid >> 6, ch16 = tid & 63;
        const int mb = ch16 >> 4, a = (ch16 >> 3) & 1, j = ch16 & 7;
        const int c = c0 + ch16 * 8;
        const bool cin = c < Cp;
        const char* fbase = reinterpret_cast<const char*>(hl ? Flo : Fhi) + (int64_t)(cin ? c : 0) * 2;
        const int64_t pitch = (int64_t)Cp * 2;
        // lanes 0..15 of each producer warp hold the Gaussian ids of a step; step i+1's ids load early
        int next_row = (lane < kKStep && lane < K) ? list[lane] : 0;
        for (int i = 0; i < nsteps && ok; ++i) {
            const int st = i % kStages;
            const int k0 = i * kKStep;
            const int my_row = next_row;
            next_row = (lane < kKStep && k0 + kKStep + lane < K) ? list[k0 + kKStep + lane] : 0;
            if (i >= kStages) ok = tc::mbar_wait(&ms.empty[st], ((i / kStages) + 1) & 1, err);
            if (!ok) break;
            const uint32_t dbase = a_stage(st, hl) + mb * 4096 + a * 1024;
#pragma unroll
            for (int k = 0; k < kKStep; ++k) {
                const int row = __shfl_sync(0xffffffffu, my_row, k);
                const bool valid = cin && (k0 + k < K);
                const uint32_t dst = dbase + (k >> 3) * 2048 + (k & 7) * 128 + ((j ^ (k & 7)) << 4);
                tc::cp_async16(dst, fbase + (valid ? (int64_t)row * pitch : 0), valid ? 16u : 0u);
            }
            // Gaussian parameters: 16 records of 5 x 16 bytes (zero fill for padding)
            {
                const int k = min(tid / 5, kKStep - 1), wq = tid - (tid / 5) * 5;
                const int row = __shfl_sync(0xffffffffu, my_row, k);  // whole warp takes part
                if (tid < kKStep * 5) {
                    const bool valid = k0 + k < K;
                    tc::cp_async16(tc::smem_u32(ms.prm[st].g) + tid * 16, &gparams[valid ? row : 0].w[wq],
                                   valid ? 16u : 0u);
                }
            }
            tc::cp_async_mbar_arrive_noinc(&ms.full_a[st]);
        }
    } else if (warp == 8) {
        // ---------------- MMA warp (one thread) ----------------
        if (lane == 0) {
            for (int i = 0; i < nsteps && ok; ++i) {
                const int st = i % kStages;
                const uint32_t par = (i / kStages) & 1;
                ok = tc::mbar_wait(&ms.full_a[st], par, err) && tc::mbar_wait(&ms.full_w[st], par, err);
                if (!ok) break;
                // the A operand was written by cp.async (generic proxy); the MMA reads it through the async proxy
                tc::fence_async_smem();
                tc::tc_fence_after();
                const uint64_t bh = tc::smem_desc(tc::smem_u32(w_stage(st, 0)), 128, 256, tc::kLayoutNone);
                const uint64_t bl = tc::smem_desc(tc::smem_u32(w_stage(st, 1)), 128, 256, tc::kLayoutNone);
#pragma unroll
                for (int mb = 0; mb < kMB; ++mb) {
                    const uint64_t ah = tc::smem_desc(a_stage(st, 0) + mb * 4096, 1024, 2048, tc::kLayoutSw128);
                    const uint64_t al = tc::smem_desc(a_stage(st, 1) + mb * 4096, 1024, 2048, tc::kLayoutSw128);
                    const uint32_t d = tmem + mb * 64;
                    tc::mma_f16_ss(d, ah, bh, kIdesc, i > 0);
                    tc::mma_f16_ss(d, ah, bl, kIdesc, true);
                    tc::mma_f16_ss(d, al, bh, kIdesc, true);
                }
                tc::mma_commit(tc::smem_u32(&ms.empty[st]));
            }
            tc::mma_commit(tc::smem_u32(&ms.mma_done));
        }
        __syncwarp();
    } else {
        // ---------------- weight warps (4..7): thread = (z-line (lx, ly), Gaussian pair) ----------------
        const int t = tid - 128;
        const int line = t >> 3, kp = t & 7;  // 16 lines x 8 pairs
        const int lx = line >> 2, ly = line & 3;
        const int vx = x0 + lx, vy = y0 + ly;
        const float cx = voxel_centre(G, 0, vx), cy = voxel_centre(G, 1, vy), cz0 = voxel_centre(G, 2, z0);
        const float hz = G.h[2];
        dline = line;
        dkp = kp;
        for (int i = 0; i < nsteps && ok; ++i) {
            const int st = i % kStages;
            if (i >= kStages) ok = tc::mbar_wait(&ms.empty[st], ((i / kStages) + 1) & 1, err);
            ok = ok && tc::mbar_wait(&ms.full_a[st], (i / kStages) & 1, err);
            if (!ok) break;
            float w[2][4];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int k = 2 * kp + u;
                const GParams& gp = ms.prm[st].g[k];
                const float4 a = gp.w[0], b = gp.w[1], c = gp.w[2], d = gp.w[3], e4 = gp.w[4];
#pragma unroll
                for (int zz = 0; zz < 4; ++zz) w[u][zz] = 0.0f;
                const int zlo = max(__float_as_int(d.w) - z0, 0), zhi = min(__float_as_int(e4.z) - z0, 3);
                if (i * kKStep + k < K && vx >= __float_as_int(d.y) && vx <= __float_as_int(e4.x) &&
                    vy >= __float_as_int(d.z) && vy <= __float_as_int(e4.y) && zlo <= zhi) {
                    // maha(z0 + t) = A + t B + t^2 Q for the voxel centres of this z-line
                    const float dx = cx - a.x, dy = cy - a.y, dz = cz0 - a.z;
                    const float qx = b.x * dx + b.y * dy + b.z * dz;   // (P d)
                    const float qy = b.w * dx + c.x * dy + c.y * dz;
                    const float qz = c.z * dx + c.w * dy + d.x * dz;
                    const float A = dx * qx + dy * qy + dz * qz;
                    const float ptz = b.z * dx + c.y * dy + d.x * dz;  // (P^T d)_z
                    const float B = hz * (qz + ptz), Q = hz * hz * d.x;
#pragma unroll
                    for (int zz = 0; zz < 4; ++zz) {
                        const float m = fmaf(fmaf(Q, (float)zz, B), (float)zz, A);
                        const float ex = __expf(-0.5f * m);
                        w[u][zz] = (zz >= zlo && zz <= zhi) ? a.w * ex : 0.0f;
                    }
                }
            }
            // store the 8 weights (4 voxels x 2 Gaussians) as half2 pairs, hi and lo, in the K-major core matrices
#pragma unroll
            for (int zz = 0; zz < 4; ++zz) {
                dsum[zz] += w[0][zz] + w[1][zz];
                __half h0, l0, h1, l1;
                tc::split_half(w[0][zz] * wscale, h0, l0);
                tc::split_half(w[1][zz] * wscale, h1, l1);
                const int v = (lx * 4 + ly) * 4 + zz, k = 2 * kp;
                const int off = (v >> 3) * 256 + (k >> 3) * 128 + (v & 7) * 16 + (k & 7) * 2;
                *reinterpret_cast<__half2*>(w_stage(st, 0) + off) = __halves2half2(h0, h1);
                *reinterpret_cast<__half2*>(w_stage(st, 1) + off) = __halves2half2(l0, l1);
            }
            tc::fence_async_smem();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&ms.full_w[st]);
        }
    }
    // all MMAs are complete once mma_done has arrived
    ok = tc::mbar_wait_drain(&ms.mma_done, 0, err) && ok;
    if (!ok) ms.fail = 1;  // benign race: every writer stores 1
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    // the stage buffers are free now: density partials [pair slot][voxel] go there
    float* dpartk = reinterpret_cast<float*>(base);
    if (warp >= 4 && warp < 8) {
#pragma unroll
        for (int zz = 0; zz < 4; ++zz) dpartk[dkp * kVoxPerTile + dline * 4 + zz] = dsum[zz];
    }
    __syncthreads();
    if (tid < kVoxPerTile) {
        float D = 0.0f;
#pragma unroll
        for (int q = 0; q < 8; ++q) D += dpartk[q * kVoxPerTile + tid];
        ms.vscale[tid] = 1.0f / (fmaxf(D, kEps) * wscale);
        int lx, ly, lz;
        local_voxel(tid, lx, ly, lz);
        if (grp == 0 && lx < nx && ly < ny && lz < nz) density[row0 + lx * sx + ly * sy + lz] = D;
    }
    __syncthreads();

    // epilogue: warp w reads TMEM lanes 32*(w%4).. (channels) of M-blocks (w/4) and (w/4)+2; lane = channel,
    // the 16 columns of one load are the voxels (lx, 0..3, 0..3) of x-slice lx = j
    const bool good = !ms.fail;
    const bool full = nx == kTile && ny == kTile && nz == kTile;
    const int q = warp & 3, hh = (warp >> 2) & 1;
    int64_t off[16];  // element offsets of the 16 voxels (ly, lz) of an x-slice, relative to the slice
#pragma unroll
    for (int e = 0; e < 16; ++e) off[e] = ((int64_t)(e >> 2) * sy + (e & 3)) * C;
#pragma unroll
    for (int t = 0; t < 2 && warp < 8; ++t) {
        const int mb = hh + 2 * t;
        const int c = c0 + mb * 128 + q * 32 + lane;
        const bool cok = c < C;
        const float us = cok ? unscale[c] : 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float vals[16];
            if (good) {
                tc::tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + mb * 64 + j * 16, vals);
            } else {
#pragma unroll
                for (int e = 0; e < 16; ++e) vals[e] = 0.0f;
            }
            float* slice = grid_feats + (row0 + j * sx) * C + c;
            const float4* vs4 = reinterpret_cast<const float4*>(&ms.vscale[j * 16]);
            if (full) {
                if (cok) {
#pragma unroll
                    for (int e4 = 0; e4 < 4; ++e4) {
                        const float4 r = vs4[e4];
                        slice[off[4 * e4 + 0]] = vals[4 * e4 + 0] * (us * r.x);
                        slice[off[4 * e4 + 1]] = vals[4 * e4 + 1] * (us * r.y);
                        slice[off[4 * e4 + 2]] = vals[4 * e4 + 2] * (us * r.z);
                        slice[off[4 * e4 + 3]] = vals[4 * e4 + 3] * (us * r.w);
                    }
                }
            } else if (cok && j < nx) {
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    if ((e >> 2) < ny && (e & 3) < nz) slice[off[e]] = vals[e] * (us * ms.vscale[j * 16 + e]);
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}
}  // namespace

int launch_pack_params(const float* means, const float* opacity, const float* cov_inv, const int32_t* lb,
                       const int32_t* ub, int64_t n, GParams* out, cudaStream_t s) {
    if (n <= 0) return 0;
    G2V_TIMED("pack_params_kernel", s,
              pack_params_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(means, opacity, cov_inv, lb, ub, n, out));
    G2V_LAUNCH_CHECK("pack_params_kernel");
    return 0;
}

size_t splat_tc_split_bytes(int64_t n, int64_t C) {
    const int64_t Cp = (C + 7) / 8 * 8;
    return 2 * ((size_t)n * Cp * sizeof(__half) + 256) + 2 * ((size_t)Cp * 4 + 256) +
           ((size_t)(n > 0 ? n : 1) * sizeof(GParams) + 256);
}

// Splits the features (per-channel power-of-two scale) into `split` (splat_tc_split_bytes) and runs the
// tensor-core splat over the tiles [first_tile, first_tile + num_tiles).
int launch_splat_tc(const float* means, const float* opacity, const float* cov_inv, const int32_t* lb,
                    const int32_t* ub, const float* features, int64_t n, int C, const int32_t* tile_offsets,
                    const int32_t* tile_lists, int first_tile, int num_tiles, const Grid& G, float* density,
                    float* grid_feats, void* split, int* err, cudaStream_t s) {
    if (num_tiles <= 0) return 0;
    const int Cp = (C + 7) / 8 * 8;
    Carver cv(split);
    __half* hi = cv.take<__half>((size_t)n * Cp);
    __half* lo = cv.take<__half>((size_t)n * Cp);
    unsigned* colmax = cv.take<unsigned>((size_t)Cp);
    float* unscale = cv.take<float>((size_t)Cp);
    if (n > 0) {
        G2V_CUDA(cudaMemsetAsync(colmax, 0, sizeof(unsigned) * Cp, s));
        const int rows = 256;
        dim3 g1((C + 255) / 256, (unsigned)((n + rows - 1) / rows));
        G2V_TIMED("feature_colmax_kernel", s, feature_colmax_kernel<<<g1, 256, 0, s>>>(features, n, C, rows, colmax));
        G2V_LAUNCH_CHECK("feature_colmax_kernel");
        const int64_t total = n * (Cp / 8);
        G2V_TIMED("feature_split_kernel", s,
                  feature_split_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(features, n, C, Cp, colmax, hi,
                                                                                    lo, unscale));
        G2V_LAUNCH_CHECK("feature_split_kernel");
    }
    const int ngroups = (C + kChGroup - 1) / kChGroup;
    GParams* gp = cv.take<GParams>((size_t)(n > 0 ? n : 1));
    int rc = launch_pack_params(means, opacity, cov_inv, lb, ub, n, gp, s);
    if (rc) return rc;
    G2V_CUDA(cudaFuncSetAttribute(splat_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    const int64_t grid = (int64_t)num_tiles * ngroups;
    G2V_TIMED("splat_tc_kernel", s,
              splat_tc_kernel<<<(unsigned)grid, kThreads, kSmemBytes, s>>>(hi, lo, unscale, C, Cp, gp, opacity,
                                                                            tile_offsets, tile_lists,
                                                                            first_tile, ngroups, G, density,
                                                                            grid_feats, err));
    G2V_LAUNCH_CHECK("splat_tc_kernel");
    return 0;
}

}  // namespace g2v
