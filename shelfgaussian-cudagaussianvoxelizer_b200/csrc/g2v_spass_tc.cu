// g2v_spass_tc.cu -- tile pass of the backward on the tensor cores (tcgen05, kind::f16, bf16).
//
// For one tile and the Gaussians of its list (reference ComputeGaussian2VoxelGradientTileWithFeats,
// src/cuda_gaussian_voxelizer.cu:1376-1482, with e_v formed from S instead of reading grid_feats):
//   S_gv  = sum_c f_gc gF_vc                        (tensor cores, D = S in TMEM)
//   e_v   = sum_g (w_gv / den_v) S_gv               (epilogue, phase 1)
//   a_gv  = gD_v + (S_gv - [D_v >= eps] e_v) / den_v
//   the ten gradient partials of every (Gaussian, tile) pair = sums over the tile's voxels (phase 2),
// written at the pair's position in the Gaussian->Tile CSR like the FP32-FMA variant (g2v_grad.cu).
//
// MMA shape: M = 128 Gaussians (two M-blocks = 256 "slots" per pass), N = the tile's 64 voxels,
// K = 32 channels per pipeline step.  Both operands are K-major without swizzle (8-row x 16-byte core
// matrices): A rows are the features, pre-split once into bf16 hi/lo rows padded to Cp channels and
// copied with 16-byte cp.async; B rows are the upstream gradient of the voxels, converted fp32 -> bf16
// hi/lo by the producer threads.  hi*hi + hi*lo + lo*hi is accumulated in fp32 (~2^-16 relative per
// product; bf16 keeps the fp32 exponent range, so no scaling is needed).
//
// The upstream gradient of a step (the tile's 4x4x4 voxels x 32 channels, 8 KB) arrives in a staging
// ring through one tiled TMA load of the 4-D tensor map {C, Z, Y, X} (zero fill beyond the grid), so the
// HBM latency is hidden by the ring instead of stalling the converting threads; when the tensor map
// cannot be built (C % 4 != 0, unaligned base) the converting threads load the rows themselves.
//
// Roles (320 threads): warps 0-7 copy the feature rows and convert the staged gradient rows, warp 8
// (one thread) issues the MMAs, warp 9 (one thread) issues the TMA loads; after a pass's MMAs have
// drained, warps 0-7 run the epilogue with one thread per Gaussian slot (TMEM lane).
// Tiles with at most 512 Gaussians keep all of S in TMEM (two passes x 128 columns); longer lists run
// two sweeps (phase 1 over all passes, then the MMAs again for phase 2).  Two CTAs share an SM so that
// one's epilogue overlaps the other's main loop.  Every mbarrier wait is bounded.
#include <algorithm>
#include <cstddef>
#include <cstring>

#include "g2v_internal.cuh"
#include "g2v_tc.cuh"
#include "g2v_tmap.cuh"

namespace g2v {

namespace {
constexpr int kThreads = 320;
constexpr int kSlots = 256;                       // Gaussians per pass
constexpr int kKC = 32;                           // channels per pipeline step
constexpr int kStages = 2;
constexpr int kAHalf = kSlots * kKC * 2;          // 16 KB: 256 rows x 64 bytes
constexpr int kBHalf = kVoxPerTile * kKC * 2;     // 4 KB: 64 rows x 64 bytes
constexpr int kStageBytes = 2 * kAHalf + 2 * kBHalf;
constexpr int kRowGroupBytes = (kKC / 8) * 128;   // 8 rows x kKC channels: 4 core matrices along K
constexpr int kMBlockBytes = 16 * kRowGroupBytes; // 128 rows
constexpr int kGS = 3;                            // staging stages of the fp32 gradient
constexpr int kGBytes = kVoxPerTile * kKC * 4;    // 8 KB: [x][y][z][32 channels]
constexpr uint32_t kTmemCols = 256;
constexpr int kKeepPasses = 2;                    // passes whose S stays in TMEM (128 columns each)
constexpr uint32_t kIdesc = tc::idesc_bf16_f32(128, kVoxPerTile, /*A K-major*/ 0, /*B K-major*/ 0);

struct SMisc {
    uint64_t full_a[kStages];  // 256 cp.async arrivals (feature rows)
    uint64_t full_b[kStages];  // 8 warp arrivals (gradient rows)
    uint64_t empty[kStages];   // MMA commit
    uint64_t mma_done;
    uint64_t gfull[kGS];       // TMA bytes of a staged gradient step
    uint64_t gempty[kGS];      // 8 converter-warp arrivals
    uint32_t tmem_base;
    int fail;
    float gD[kVoxPerTile], rden[kVoxPerTile], act[kVoxPerTile], e[kVoxPerTile];
    float epart[8][kVoxPerTile];
    int64_t vrow[kVoxPerTile];  // linear voxel index, -1 outside the grid
};
constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + (size_t)kGS * kGBytes + sizeof(SMisc);
static_assert(kSmemBytes * 2 + 2048 <= 228 * 1024, "spass_tc_kernel: two CTAs per SM");

// 16 per-lane values -> each lane pair (2i, 2i+1) holds the warp sum of value i (fixed order).
__device__ __forceinline__ float warp_reduce_scatter16(float (&p)[16], int lane) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const bool up = lane & 16;
        const float send = up ? p[i] : p[i + 8];
        const float keep = up ? p[i + 8] : p[i];
        p[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const bool up = lane & 8;
        const float send = up ? p[i] : p[i + 4];
        const float keep = up ? p[i + 4] : p[i];
        p[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const bool up = lane & 4;
        const float send = up ? p[i] : p[i + 2];
        const float keep = up ? p[i + 2] : p[i];
        p[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    {
        const bool up = lane & 2;
        const float send = up ? p[0] : p[1];
        const float keep = up ? p[1] : p[0];
        p[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    }
    return p[0] + __shfl_xor_sync(0xffffffffu, p[0], 1);  // value index (lane >> 1)
}

template <bool kTma>
__global__ void __launch_bounds__(kThreads, 2) spass_tc_kernel(
    const __grid_constant__ CUtensorMap gmap, const float* __restrict__ grad_density,
    const float* __restrict__ grad_feats,
    const __nv_bfloat16* __restrict__ Fh, const __nv_bfloat16* __restrict__ Fl, int C, int Cp, int vec,
    const float* __restrict__ density, const GParams* __restrict__ gparams, const int32_t* __restrict__ g2t_offsets,
    const int32_t* __restrict__ tile_offsets, const int32_t* __restrict__ tile_lists, int first_tile, Grid G,
    float* __restrict__ partial10, int64_t pair_cap, int* __restrict__ err) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* base = smem_raw;
    unsigned char* gstage = base + kStages * kStageBytes;
    SMisc& ms = *reinterpret_cast<SMisc*>(gstage + kGS * kGBytes);
    if ((tc::smem_u32(smem_raw) & 127u) != 0) {  // never expected; fail loudly
        if (threadIdx.x == 0) atomicOr(err, 2);
        return;
    }
    const int tl = blockIdx.x;
    const int s0 = tile_offsets[tl], K = tile_offsets[tl + 1] - s0;
    if (K == 0) return;
    const int32_t* list = tile_lists + s0;
    int tx, ty, tz;
    decode_tile(first_tile + tl, G, tx, ty, tz);
    const int x0 = tx * kTile, y0 = ty * kTile, z0 = tz * kTile;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid < kVoxPerTile) {
        int lx, ly, lz;
        local_voxel(tid, lx, ly, lz);
        const int x = x0 + lx, y = y0 + ly, z = z0 + lz;
        const bool in = x < G.dims[0] && y < G.dims[1] && z < G.dims[2];
        const int64_t row = in ? ((int64_t)x * G.dims[1] + y) * G.dims[2] + z : 0;
        const float D = in ? density[row] : 0.0f;
        ms.vrow[tid] = in ? row : -1;
        ms.gD[tid] = in ? grad_density[row] : 0.0f;
        ms.rden[tid] = 1.0f / fmaxf(D, kEps);
        ms.act[tid] = D >= kEps ? 1.0f : 0.0f;
        ms.e[tid] = 0.0f;
    }
    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            tc::mbar_init(&ms.full_a[i], 256);
            tc::mbar_init(&ms.full_b[i], 8);
            tc::mbar_init(&ms.empty[i], 1);
        }
        tc::mbar_init(&ms.mma_done, 1);
        for (int i = 0; i < kGS; ++i) {
            tc::mbar_init(&ms.gfull[i], 1);
            tc::mbar_init(&ms.gempty[i], 8);
        }
        tc::mbar_fence_init();
        ms.fail = 0;
    }
    if (warp == 0) tc::tmem_alloc(&ms.tmem_base, kTmemCols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = ms.tmem_base;

    const int npass = (K + kSlots - 1) / kSlots;
    const bool keep = npass <= kKeepPasses;
    const int nsteps = Cp / kKC;
    const int64_t pitch = (int64_t)Cp * 2;  // bytes per split feature row
    bool ok = true;
    int it = 0;   // pipeline step counter (stage / parity bookkeeping), the same in every role
    int issued = 0;  // TMA thread: staged steps issued
    int ndone = 0;  // completed mma_done phases

    auto a_half = [&](int st, int hl) -> uint32_t { return tc::smem_u32(base + st * kStageBytes + hl * kAHalf); };
    auto b_half = [&](int st, int hl) -> uint32_t {
        return tc::smem_u32(base + st * kStageBytes + 2 * kAHalf + hl * kBHalf);
    };

    // ---- main loop of one pass: S of slots [p*256, p*256+256) into TMEM columns cg*128 .. +127 ----
    auto mainloop = [&](int p, int cg, bool commit_done) {
        const int ns = min(kSlots, K - p * kSlots);
        const int nmb = ns > 128 ? 2 : 1;
        if (warp < 8) {
            // feature rows: thread = (row r of each 64-row quarter, 16-byte chunk kc)
            const int kc = lane & 3;
            int64_t goff[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int slot = u * 64 + warp * 8 + (lane >> 2);
                goff[u] = slot < ns ? (int64_t)list[p * kSlots + slot] * pitch : -1;
            }
            // gradient rows: thread = (voxel v, 16-byte chunk kcb)
            const int v = tid >> 2, kcb = tid & 3;
            const int64_t vrow = ms.vrow[v];
            const uint32_t boff = (v >> 3) * kRowGroupBytes + kcb * 128 + (v & 7) * 16;
            for (int j = 0; j < nsteps && ok; ++j, ++it) {
                const int st = it % kStages;
                if (it >= kStages) ok = tc::mbar_wait(&ms.empty[st], ((it / kStages) + 1) & 1, err);
                if (!ok) break;
                const int c0 = j * kKC;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int slot = u * 64 + warp * 8 + (lane >> 2);
                    if (slot < nmb * 128) {
                        const uint32_t aoff = (slot >> 3) * kRowGroupBytes + kc * 128 + (slot & 7) * 16;
                        const int64_t src = goff[u] >= 0 ? goff[u] + (int64_t)(c0 + kc * 8) * 2 : 0;
                        const uint32_t nb = goff[u] >= 0 ? 16u : 0u;
                        tc::cp_async16(a_half(st, 0) + aoff, reinterpret_cast<const char*>(Fh) + src, nb);
                        tc::cp_async16(a_half(st, 1) + aoff, reinterpret_cast<const char*>(Fl) + src, nb);
                    }
                }
                tc::cp_async_mbar_arrive_noinc(&ms.full_a[st]);
                // B: 8 channels of the voxel's gradient row -> bf16 hi / lo
                const int c = c0 + kcb * 8;
                const int gs = it % kGS;
                float f[8];
                if (kTma) {
                    ok = tc::mbar_wait(&ms.gfull[gs], (it / kGS) & 1, err);
                    if (!ok) break;
                    const float4* src = reinterpret_cast<const float4*>(gstage + gs * kGBytes + v * (kKC * 4) + kcb * 32);
                    const float4 u0 = src[0], u1 = src[1];
                    f[0] = u0.x; f[1] = u0.y; f[2] = u0.z; f[3] = u0.w;
                    f[4] = u1.x; f[5] = u1.y; f[6] = u1.z; f[7] = u1.w;
                } else if (vrow >= 0 && vec && c + 7 < C) {
                    const float4 u0 = *reinterpret_cast<const float4*>(grad_feats + vrow * C + c);
                    const float4 u1 = *reinterpret_cast<const float4*>(grad_feats + vrow * C + c + 4);
                    f[0] = u0.x; f[1] = u0.y; f[2] = u0.z; f[3] = u0.w;
                    f[4] = u1.x; f[5] = u1.y; f[6] = u1.z; f[7] = u1.w;
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] = (vrow >= 0 && c + e < C) ? grad_feats[vrow * C + c + e] : 0.0f;
                }
                uint32_t h[4], l[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) tc::split_bf16x2(f[2 * e], f[2 * e + 1], h[e], l[e]);
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(b_half(st, 0) + boff), "r"(h[0]),
                             "r"(h[1]), "r"(h[2]), "r"(h[3])
                             : "memory");
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(b_half(st, 1) + boff), "r"(l[0]),
                             "r"(l[1]), "r"(l[2]), "r"(l[3])
                             : "memory");
                tc::fence_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tc::mbar_arrive(&ms.full_b[st]);
                    if (kTma) tc::mbar_arrive(&ms.gempty[gs]);
                }
            }
        } else if (kTma && warp == 9 && lane == 0) {
            // ---- TMA thread: the gradient box of each step into the staging ring ----
            for (int j = 0; j < nsteps && ok; ++j, ++it) {
                const int gs = it % kGS;
                if (it >= kGS) ok = tc::mbar_wait(&ms.gempty[gs], ((it / kGS) + 1) & 1, err);
                if (!ok) break;
                tc::mbar_arrive_expect_tx(&ms.gfull[gs], kGBytes);
                tc::tma_load_4d(tc::smem_u32(gstage + gs * kGBytes), &gmap, j * kKC, z0, y0, x0, &ms.gfull[gs]);
                issued = it + 1;
            }
        } else if (warp == 8 && lane == 0) {
            for (int j = 0; j < nsteps && ok; ++j, ++it) {
                const int st = it % kStages;
                const uint32_t par = (it / kStages) & 1;
                ok = tc::mbar_wait(&ms.full_a[st], par, err) && tc::mbar_wait(&ms.full_b[st], par, err);
                if (!ok) break;
                tc::tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < kKC / 16; ++ks) {
                    const uint64_t bh = tc::smem_desc(b_half(st, 0) + ks * 256, 128, kRowGroupBytes, tc::kLayoutNone);
                    const uint64_t bl = tc::smem_desc(b_half(st, 1) + ks * 256, 128, kRowGroupBytes, tc::kLayoutNone);
                    for (int mb = 0; mb < nmb; ++mb) {
                        const uint32_t ao = mb * kMBlockBytes + ks * 256;
                        const uint64_t ah = tc::smem_desc(a_half(st, 0) + ao, 128, kRowGroupBytes, tc::kLayoutNone);
                        const uint64_t al = tc::smem_desc(a_half(st, 1) + ao, 128, kRowGroupBytes, tc::kLayoutNone);
                        const uint32_t d = tmem + (uint32_t)((cg * 2 + mb) * kVoxPerTile);
                        tc::mma_f16_ss(d, ah, bh, kIdesc, j > 0 || ks > 0);
                        tc::mma_f16_ss(d, ah, bl, kIdesc, true);
                        tc::mma_f16_ss(d, al, bh, kIdesc, true);
                    }
                }
                tc::mma_commit(tc::smem_u32(&ms.empty[st]));
            }
            if (commit_done) tc::mma_commit(tc::smem_u32(&ms.mma_done));
        } else {
            it += nsteps;
        }
    };

    auto drain = [&]() {
        ok = tc::mbar_wait_drain(&ms.mma_done, ndone & 1, err) && ok;
        ++ndone;
        if (!ok) ms.fail = 1;
        tc::tc_fence_before();
        __syncthreads();
        tc::tc_fence_after();
    };

    // voxel centres of the tile along each axis
    float cxs[kTile], cys[kTile], czs[kTile];
#pragma unroll
    for (int i = 0; i < kTile; ++i) {
        cxs[i] = voxel_centre(G, 0, x0 + i);
        cys[i] = voxel_centre(G, 1, y0 + i);
        czs[i] = voxel_centre(G, 2, z0 + i);
    }

    // ---- phase 1: e_v += sum over the pass's slots of (w_gv / den_v) S_gv ----
    auto phase1 = [&](int p, int cg) {
        if (warp < 8 && !ms.fail) {
            const int mb = warp >> 2, q = warp & 3;
            const int slot0 = p * kSlots + mb * 128 + q * 32;
            if (slot0 < K) {  // warp-uniform
                const int slot = slot0 + lane;
                const bool live = slot < K;
                const GParams& gp = gparams[live ? list[slot] : list[0]];
                const float4 A = gp.w[0], P0 = gp.w[1], P1 = gp.w[2], P2 = gp.w[3], U = gp.w[4];
                const int lbx = __float_as_int(P2.y), lby = __float_as_int(P2.z), lbz = __float_as_int(P2.w);
                const int ubx = __float_as_int(U.x), uby = __float_as_int(U.y), ubz = __float_as_int(U.z);
                const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((cg * 2 + mb) * kVoxPerTile);
#pragma unroll 1
                for (int lx = 0; lx < kTile; ++lx) {
                    float Sv[16];
                    tc::tmem_ld16(taddr + lx * 16, Sv);
                    const float dx = cxs[lx] - A.x;
                    const bool inx = live && x0 + lx >= lbx && x0 + lx <= ubx;
#pragma unroll
                    for (int ly = 0; ly < kTile; ++ly) {
                        const float dy = cys[ly] - A.y;
                        const bool iny = inx && y0 + ly >= lby && y0 + ly <= uby;
                        const float tx_ = fmaf(P0.y, dy, P0.x * dx);
                        const float ty_ = fmaf(P1.x, dy, P0.w * dx);
                        const float tz_ = fmaf(P1.w, dy, P1.z * dx);
#pragma unroll
                        for (int lz = 0; lz < kTile; ++lz) {
                            const float dz = czs[lz] - A.z;
                            const float qx = fmaf(P0.z, dz, tx_), qy = fmaf(P1.y, dz, ty_), qz = fmaf(P2.x, dz, tz_);
                            const float m = dx * qx + dy * qy + dz * qz;
                            const bool in = iny && z0 + lz >= lbz && z0 + lz <= ubz;
                            const int v = ly * 4 + lz;
                            Sv[v] = in ? A.w * __expf(-0.5f * m) * ms.rden[lx * 16 + v] * Sv[v] : 0.0f;
                        }
                    }
                    const float r = warp_reduce_scatter16(Sv, lane);
                    if ((lane & 1) == 0) ms.epart[warp][lx * 16 + (lane >> 1)] = r;
                }
            } else {
                for (int v = lane; v < kVoxPerTile; v += 32) ms.epart[warp][v] = 0.0f;
            }
        }
        __syncthreads();
        if (tid < kVoxPerTile && !ms.fail) {
            float acc = ms.epart[0][tid];
#pragma unroll
            for (int w = 1; w < 8; ++w) acc += ms.epart[w][tid];
            ms.e[tid] += acc;
        }
        __syncthreads();
    };

    // ---- phase 2: the ten gradient partials of each slot's (Gaussian, tile) pair ----
    auto phase2 = [&](int p, int cg) {
        if (warp < 8 && !ms.fail) {
            const int mb = warp >> 2, q = warp & 3;
            const int slot0 = p * kSlots + mb * 128 + q * 32;
            if (slot0 < K) {  // warp-uniform
                const int slot = slot0 + lane;
                const bool live = slot < K;
                const int g = live ? list[slot] : list[0];
                const GParams& gp = gparams[g];
                const float4 A = gp.w[0], P0 = gp.w[1], P1 = gp.w[2], P2 = gp.w[3], U = gp.w[4];
                const int lbx = __float_as_int(P2.y), lby = __float_as_int(P2.z), lbz = __float_as_int(P2.w);
                const int ubx = __float_as_int(U.x), uby = __float_as_int(U.y), ubz = __float_as_int(U.z);
                const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((cg * 2 + mb) * kVoxPerTile);
                float gr[10];
#pragma unroll
                for (int i = 0; i < 10; ++i) gr[i] = 0.0f;
#pragma unroll 1
                for (int lx = 0; lx < kTile; ++lx) {
                    float Sv[16];
                    tc::tmem_ld16(taddr + lx * 16, Sv);
                    const float dx = cxs[lx] - A.x;
                    const bool inx = live && x0 + lx >= lbx && x0 + lx <= ubx;
#pragma unroll
                    for (int ly = 0; ly < kTile; ++ly) {
                        const float dy = cys[ly] - A.y;
                        const bool iny = inx && y0 + ly >= lby && y0 + ly <= uby;
                        const float tx_ = fmaf(P0.y, dy, P0.x * dx);
                        const float ty_ = fmaf(P1.x, dy, P0.w * dx);
                        const float tz_ = fmaf(P1.w, dy, P1.z * dx);
#pragma unroll
                        for (int lz = 0; lz < kTile; ++lz) {
                            const int v = ly * 4 + lz, vt = lx * 16 + v;
                            const bool in = iny && z0 + lz >= lbz && z0 + lz <= ubz;
                            if (in) {
                                const float dz = czs[lz] - A.z;
                                const float qx = fmaf(P0.z, dz, tx_), qy = fmaf(P1.y, dz, ty_),
                                            qz = fmaf(P2.x, dz, tz_);
                                const float m = dx * qx + dy * qy + dz * qz;
                                const float ex = __expf(-0.5f * m);
                                const float a = fmaf(fmaf(-ms.act[vt], ms.e[vt], Sv[v]), ms.rden[vt], ms.gD[vt]);
                                const float aw = a * A.w * ex;
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
                    }
                }
                if (live) {
                    const int tlx = lbx / kTile, tly = lby / kTile, tlz = lbz / kTile;
                    const int ey = uby / kTile - tly + 1, ez = ubz / kTile - tlz + 1;
                    const int64_t idx = (int64_t)g2t_offsets[g] + ((tx - tlx) * ey + (ty - tly)) * ez + (tz - tlz);
                    if (idx >= 0 && idx < pair_cap) {  // offsets come from the caller
                        float* out = partial10 + idx * 10;
#pragma unroll
                        for (int i = 0; i < 10; ++i) out[i] = gr[i];
                    }
                }
            }
        }
    };

    auto sync_tc = [&]() {
        tc::tc_fence_before();
        __syncthreads();
        tc::tc_fence_after();
    };

    if (keep) {
        for (int p = 0; p < npass; ++p) mainloop(p, p, p == npass - 1);
        drain();
        for (int p = 0; p < npass; ++p) phase1(p, p);
        for (int p = 0; p < npass; ++p) phase2(p, p);
    } else {
        for (int p = 0; p < npass; ++p) {
            mainloop(p, 0, true);
            drain();
            phase1(p, 0);
            sync_tc();
        }
        for (int p = 0; p < npass; ++p) {
            mainloop(p, 0, true);
            drain();
            phase2(p, 0);
            sync_tc();
        }
    }
    // no copy may still be in flight when the CTA's shared memory is released (matters after a wait gave up)
    if (kTma && warp == 9 && lane == 0)
        for (int k = max(0, issued - kGS); k < issued; ++k) tc::mbar_wait_drain(&ms.gfull[k % kGS], (k / kGS) & 1, err);
    tc::cp_async_wait<0>();
    sync_tc();
    if (warp == 0) tc::tmem_dealloc(tmem, kTmemCols);
}

// features [n][C] fp32 -> bf16 hi / lo rows of Cp channels (zero padded), 8 channels per thread
__global__ void feature_split_bf16_kernel(const float* __restrict__ f, int64_t n, int C, int Cp,
                                          __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
    const int cpr = Cp / 8;
    const int64_t total = n * cpr;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t g = i / cpr;
        const int c = (int)(i - g * cpr) * 8;
        __align__(16) __nv_bfloat16 h[8], l[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float x = c + e < C ? f[g * C + c + e] : 0.0f;
            tc::split_bf16(x, h[e], l[e]);
        }
        *reinterpret_cast<uint4*>(hi + g * Cp + c) = *reinterpret_cast<const uint4*>(h);
        *reinterpret_cast<uint4*>(lo + g * Cp + c) = *reinterpret_cast<const uint4*>(l);
    }
}
}  // namespace

int64_t spass_tc_padded_channels(int64_t C) { return (C + kKC - 1) / kKC * kKC; }

size_t spass_tc_split_bytes(int64_t n, int64_t C) {
    return (size_t)2 * (size_t)(n > 0 ? n : 1) * (size_t)spass_tc_padded_channels(C) * sizeof(__nv_bfloat16) + 256;
}

int launch_spass_tc(const float* grad_density, const float* grad_feats, const float* features, int64_t n, int C,
                    const float* density, const GParams* gparams, const int32_t* g2t_offsets,
                    const int32_t* tile_offsets, const int32_t* tile_lists, int first_tile, int num_tiles,
                    const Grid& G, float* partial10, int64_t pair_cap, void* split, int* err, cudaStream_t s) {
    if (num_tiles <= 0 || C <= 0 || n <= 0) return 0;
    const int Cp = (int)spass_tc_padded_channels(C);
    uintptr_t p = (reinterpret_cast<uintptr_t>(split) + 255) & ~uintptr_t(255);
    __nv_bfloat16* Fh = reinterpret_cast<__nv_bfloat16*>(p);
    __nv_bfloat16* Fl = Fh + n * Cp;
    {
        const int64_t total = n * (Cp / 8);
        const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
        G2V_TIMED("feature_split_bf16_kernel", s,
                  feature_split_bf16_kernel<<<blocks, 256, 0, s>>>(features, n, C, Cp, Fh, Fl));
        G2V_LAUNCH_CHECK("feature_split_bf16_kernel");
    }
    const int vec = (C % 4 == 0) && (reinterpret_cast<uintptr_t>(grad_feats) % 16 == 0);
    CUtensorMap gmap;
    memset(&gmap, 0, sizeof(gmap));
    const bool tma = encode_grid_rows_f32(&gmap, grad_feats, G.dims, C, kKC, kTile, kTile, kTile);
    auto kern = tma ? spass_tc_kernel<true> : spass_tc_kernel<false>;
    G2V_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    G2V_TIMED("spass_tc_kernel", s,
              kern<<<(unsigned)num_tiles, kThreads, kSmemBytes, s>>>(
                  gmap, grad_density, grad_feats, Fh, Fl, C, Cp, vec, density, gparams, g2t_offsets, tile_offsets,
                  tile_lists, first_tile, G, partial10, pair_cap, err));
    G2V_LAUNCH_CHECK("spass_tc_kernel");
    return 0;
}

}  // namespace g2v
