// g2v_spass_tc.cu -- tile pass of the backward on the tensor cores (tcgen05, kind::f16, bf16).
//
// For the Gaussians of a tile (reference ComputeGaussian2VoxelGradientTileWithFeats,
// src/cuda_gaussian_voxelizer.cu:1376-1482, with e_v formed from S instead of reading grid_feats):
//   S_gv  = sum_c f_gc gF_vc                        (tensor cores, S in TMEM)
//   e_v   = sum_g (w_gv / den_v) S_gv               (epilogue, phase 1)
//   a_gv  = gD_v + (S_gv - [D_v >= eps] e_v) / den_v
//   the ten gradient partials of every (Gaussian, tile) pair = sums over the tile's voxels (phase 2),
// written at the pair's position in the Gaussian->Tile CSR like the FP32-FMA variant (g2v_grad.cu).
//
// Unit of work: a pair of z-adjacent tiles (4 x 4 x 8 = 128 voxels) with the union of their Gaussian
// lists (ascending ids).  Pairing halves the feature-row gathers and doubles the MMA's N against the
// per-tile shape, at the price of the Gaussians that reach only one of the two tiles.
// MMA: M = 128 Gaussians (two M-blocks = 256 slots per pass), N = the unit's 128 voxels, K = 32
// channels per pipeline step; both operands K-major with 64-byte swizzle (a row = the step's 32
// channels; atoms of 8 rows x 64 bytes, 16-byte chunk c of row r stored at chunk c ^ ((r / 2) % 4)).
// A rows are the features, pre-split once into bf16 hi/lo rows padded to Cp channels and gathered with
// 16-byte cp.async; B rows are the upstream gradient of the unit's voxels, brought in by one tiled TMA
// load of the 4-D tensor map {C, Z, Y, X} per step and converted fp32 -> bf16 hi/lo in shared memory
// (zero fill beyond the grid).  hi*hi + hi*lo + lo*hi is accumulated in fp32 (~2^-16 relative per
// product).  When the tensor map cannot be built (C % 4 != 0, unaligned base) the converting threads
// load the gradient rows themselves.
//
// Persistent CTAs (one per SM) walk the units with a fixed stride; the S of one job (a pass of a unit)
// fills half of TMEM (256 columns), so the epilogue of one job overlaps the main loop of the next.
// Roles (576 threads): warps 0-3 gather feature rows (4-stage ring, L2 evict_last), warps 4-7 convert
// gradient rows (2-stage ring; the fp32 rows stream through L2 with evict_first), warp 8 (one thread)
// issues the MMAs, warp 9 (one thread) issues the TMA loads, warps 10-17 run the epilogue with one
// thread per Gaussian slot (TMEM lane).  A unit of one pass is one job (phase 1 then phase 2 on the same
// S); a longer list runs every pass twice, phase 1 over all passes first, then the MMAs again for
// phase 2.  Every mbarrier wait is bounded.
#include <algorithm>
#include <cstddef>
#include <cstring>

#include "g2v_internal.cuh"
#include "g2v_tc.cuh"
#include "g2v_tmap.cuh"

namespace g2v {

namespace {
constexpr int kThreads = 576;
constexpr int kSlots = 256;                       // Gaussians per pass
constexpr int kKC = 32;                           // channels per pipeline step
constexpr int kSA = 4;                            // feature-row (A) stages
constexpr int kSB = 2;                            // converted gradient-row (B) stages
constexpr int kGS = 3;                            // staging stages of the fp32 gradient
constexpr int kUV = 128;                          // voxels of a unit: x 4, y 4, z 8 (two tiles)
constexpr int kAHalf = kSlots * kKC * 2;          // 16 KB
constexpr int kBHalf = kUV * kKC * 2;             // 8 KB
constexpr int kAStage = 2 * kAHalf;               // hi + lo
constexpr int kBStage = 2 * kBHalf;
constexpr int kGBytes = kUV * kKC * 4;            // 16 KB: [x][y][z8][32 channels], 128-byte swizzle
static_assert(kKC * 4 == 128, "the staging rows are one 128-byte swizzle span");
constexpr int kRowGroupBytes = 8 * kKC * 2;       // 8 rows x kKC bf16: one 64-byte-swizzle atom
static_assert(kKC * 2 == 64, "a K-major row of the step is one 64-byte swizzle span");

// Byte offset of 16-byte chunk c of row r in a K-major 64-byte-swizzled operand.
__device__ __forceinline__ uint32_t sw64_off(int r, int c) {
    return (uint32_t)((r >> 3) * kRowGroupBytes + (r & 7) * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}
constexpr int kMBlockBytes = 16 * kRowGroupBytes; // 128 rows
constexpr uint32_t kTmemCols = 512;
constexpr int kBufCols = 256;                     // one job: 2 M-blocks x 128 voxel columns
constexpr int kEpiWarp0 = 10;                     // first epilogue warp
constexpr uint32_t kIdesc = tc::idesc_bf16_f32(128, kUV, /*A K-major*/ 0, /*B K-major*/ 0);

struct SMisc {
    uint64_t full_a[kSA];      // 128 cp.async arrivals (feature rows)
    uint64_t empty_a[kSA];     // MMA commit
    uint64_t full_b[kSB];      // 4 warp arrivals (gradient rows)
    uint64_t empty_b[kSB];     // MMA commit
    uint64_t gfull[kGS];       // TMA bytes of a staged step
    uint64_t gempty[kGS];      // 4 converter-warp arrivals
    uint64_t tfull[2];         // MMA commit: a job's S is complete in TMEM buffer b
    uint64_t tempty[2];        // 8 epilogue-warp arrivals: buffer b has been read
    uint32_t tmem_base;
    alignas(16) float lrd[kUV];   // log2(1 / max(D, eps)), -inf outside the grid
    alignas(16) float2 va[kUV];   // phase 2: a_gv = S_gv * va.x + va.y  (va.x = 1/den, va.y = gD - act e / den)
    float gD[kUV], act[kUV], rden[kUV], e[kUV];
    float epart[8][kUV];
};
constexpr size_t kSmemBytes =
    (size_t)kSA * kAStage + (size_t)kSB * kBStage + (size_t)kGS * kGBytes + sizeof(SMisc);
static_assert(kSmemBytes <= 227 * 1024, "spass_tc_kernel shared memory");

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

// Named barrier of the 8 epilogue warps (barrier 0 is __syncthreads).
__device__ __forceinline__ void epi_barrier() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Unit u of the slab -> tile coordinates (tx, ty) and z-pair index of its first tile.
struct UnitGeom {
    int tx, ty, tzp;
};
__device__ __forceinline__ UnitGeom unit_geom(int u, int ty_n, int tzp_n, int tx_begin) {
    UnitGeom g;
    const int yz = ty_n * tzp_n;
    g.tx = tx_begin + u / yz;
    const int r = u - (u / yz) * yz;
    g.ty = r / tzp_n;
    g.tzp = r - g.ty * tzp_n;
    return g;
}

template <bool kTma>
__global__ void __launch_bounds__(kThreads, 1) spass_tc_kernel(
    const __grid_constant__ CUtensorMap gmap, const float* __restrict__ grad_density,
    const float* __restrict__ grad_feats, const __nv_bfloat16* __restrict__ Fh, const __nv_bfloat16* __restrict__ Fl,
    int C, int Cp, const float* __restrict__ density, const GParams* __restrict__ gparams,
    const int32_t* __restrict__ g2t_offsets, const int32_t* __restrict__ unit_offsets,
    const int32_t* __restrict__ unit_lists, int num_units, int tx_begin, Grid G, float* __restrict__ partial10,
    int64_t pair_cap, const float* __restrict__ ev, int* __restrict__ err) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* base = smem_raw;
    unsigned char* bring = base + kSA * kAStage;
    unsigned char* gstage = bring + kSB * kBStage;
    SMisc& ms = *reinterpret_cast<SMisc*>(gstage + kGS * kGBytes);
    if ((tc::smem_u32(smem_raw) & 127u) != 0) {  // never expected; fail loudly
        if (threadIdx.x == 0) atomicOr(err, 2);
        return;
    }
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tzp_n = (G.tiles[2] + 1) / 2;
    const int nsteps = Cp / kKC;
    const int64_t pitch = (int64_t)Cp * 2;  // bytes per split feature row

    if (tid == 0) {
        for (int i = 0; i < kSA; ++i) {
            tc::mbar_init(&ms.full_a[i], 128);
            tc::mbar_init(&ms.empty_a[i], 1);
        }
        for (int i = 0; i < kSB; ++i) {
            tc::mbar_init(&ms.full_b[i], 4);
            tc::mbar_init(&ms.empty_b[i], 1);
        }
        for (int i = 0; i < kGS; ++i) {
            tc::mbar_init(&ms.gfull[i], 1);
            tc::mbar_init(&ms.gempty[i], 4);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&ms.tfull[i], 1);
            tc::mbar_init(&ms.tempty[i], 8);
        }
        tc::mbar_fence_init();
    }
    if (warp == 0) tc::tmem_alloc(&ms.tmem_base, kTmemCols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = ms.tmem_base;
    bool ok = true;

    auto a_half = [&](int st, int hl) -> uint32_t { return tc::smem_u32(base + st * kAStage + hl * kAHalf); };
    auto b_half = [&](int st, int hl) -> uint32_t { return tc::smem_u32(bring + st * kBStage + hl * kBHalf); };

    if (warp < 4) {
        // ============ feature-row producers (cp.async, kept in L2: evict_last) ============
        // lane = (row rs of an 8-row group, 16-byte chunk kc): 8 lanes fill one 128-byte core-matrix column
        const int kc = lane >> 3, rs = lane & 7;
        const uint64_t pol = tc::l2_policy_evict_last();
        int it = 0;
        for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
            const int s0 = unit_offsets[u], K = unit_offsets[u + 1] - s0;
            if (K == 0) continue;
            const int npass = (K + kSlots - 1) / kSlots;
            const int njobs = npass == 1 ? 1 : (ev ? npass : 2 * npass);
            for (int jb = 0; jb < njobs && ok; ++jb) {
                const int p = npass == 1 ? 0 : jb % npass;
                const int ns = min(kSlots, K - p * kSlots);
                const int nrows = ns > 128 ? 256 : 128;  // rows of the M-blocks in use
                int64_t goff[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const int slot = q * 32 + warp * 8 + rs;
                    goff[q] = slot < ns ? (int64_t)unit_lists[s0 + p * kSlots + slot] * pitch : -1;
                }
                for (int j = 0; j < nsteps && ok; ++j, ++it) {
                    const int sa = it % kSA;
                    if (it >= kSA) ok = tc::mbar_wait(&ms.empty_a[sa], ((it / kSA) + 1) & 1, err);
                    if (!ok) break;
                    const int c0 = j * kKC;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int slot = q * 32 + warp * 8 + rs;
                        if (slot < nrows) {
                            const uint32_t aoff = sw64_off(slot, kc);
                            const int64_t src = goff[q] >= 0 ? goff[q] + (int64_t)(c0 + kc * 8) * 2 : 0;
                            const uint32_t nb = goff[q] >= 0 ? 16u : 0u;
                            tc::cp_async16_hint(a_half(sa, 0) + aoff, reinterpret_cast<const char*>(Fh) + src, nb, pol);
                            tc::cp_async16_hint(a_half(sa, 1) + aoff, reinterpret_cast<const char*>(Fl) + src, nb, pol);
                        }
                    }
                    tc::cp_async_mbar_arrive_noinc(&ms.full_a[sa]);
                }
            }
        }
        tc::cp_async_wait<0>();  // no copy in flight when the shared memory is released
    } else if (warp < 8) {
        // ============ gradient-row converters: staged fp32 -> bf16 hi / lo; thread = voxel row v ============
        const int v = tid - 128;
        unsigned char* const bbase = bring;
        int it = 0;
        for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
            const int K = unit_offsets[u + 1] - unit_offsets[u];
            if (K == 0) continue;
            const UnitGeom ug = unit_geom(u, G.tiles[1], tzp_n, tx_begin);
            const int x = ug.tx * kTile + (v >> 5), y = ug.ty * kTile + ((v >> 3) & 3), z = ug.tzp * 8 + (v & 7);
            const bool vin = x < G.dims[0] && y < G.dims[1] && z < G.dims[2];
            const int64_t vrow = vin ? grid_row(G, x, y, z) : -1;
            const int npass = (K + kSlots - 1) / kSlots;
            const int njobs = npass == 1 ? 1 : (ev ? npass : 2 * npass);
            for (int jb = 0; jb < njobs && ok; ++jb) {
                for (int j = 0; j < nsteps && ok; ++j, ++it) {
                    const int sb = it % kSB, gs = it % kGS;
                    if (it >= kSB) ok = tc::mbar_wait(&ms.empty_b[sb], ((it / kSB) + 1) & 1, err);
                    if (kTma && ok) ok = tc::mbar_wait(&ms.gfull[gs], (it / kGS) & 1, err);
                    if (!ok) break;
                    unsigned char* bst = bbase + sb * kBStage;
                    // 128-byte swizzled staging row: logical chunk c sits at chunk c ^ (v % 8)
                    const unsigned char* row = gstage + gs * kGBytes + v * (kKC * 4);
#pragma unroll
                    for (int hv = 0; hv < 2; ++hv) {  // 16 channels at a time
                        float f[16];
                        if (kTma) {
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const float4 t =
                                    *reinterpret_cast<const float4*>(row + (((hv * 4 + q) ^ (v & 7)) << 4));
                                f[4 * q] = t.x;
                                f[4 * q + 1] = t.y;
                                f[4 * q + 2] = t.z;
                                f[4 * q + 3] = t.w;
                            }
                        } else {
                            const int c = j * kKC + hv * 16;
#pragma unroll
                            for (int e = 0; e < 16; ++e)
                                f[e] = (vrow >= 0 && c + e < C) ? grad_feats[vrow * C + c + e] : 0.0f;
                        }
                        uint4 h0, h1, l0, l1;
                        tc::split_bf16x2(f[0], f[1], h0.x, l0.x);
                        tc::split_bf16x2(f[2], f[3], h0.y, l0.y);
                        tc::split_bf16x2(f[4], f[5], h0.z, l0.z);
                        tc::split_bf16x2(f[6], f[7], h0.w, l0.w);
                        tc::split_bf16x2(f[8], f[9], h1.x, l1.x);
                        tc::split_bf16x2(f[10], f[11], h1.y, l1.y);
                        tc::split_bf16x2(f[12], f[13], h1.z, l1.z);
                        tc::split_bf16x2(f[14], f[15], h1.w, l1.w);
                        const uint32_t o0 = sw64_off(v, 2 * hv), o1 = sw64_off(v, 2 * hv + 1);
                        *reinterpret_cast<uint4*>(bst + o0) = h0;
                        *reinterpret_cast<uint4*>(bst + o1) = h1;
                        *reinterpret_cast<uint4*>(bst + kBHalf + o0) = l0;
                        *reinterpret_cast<uint4*>(bst + kBHalf + o1) = l1;
                    }
                    tc::fence_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tc::mbar_arrive(&ms.full_b[sb]);
                        if (kTma) tc::mbar_arrive(&ms.gempty[gs]);
                    }
                }
            }
        }
    } else if (warp == 8) {
        // ============ MMA thread ============
        if (lane == 0) {
            int it = 0, job = 0;
            const uint64_t adesc0 = tc::smem_desc(a_half(0, 0), 16, kRowGroupBytes, tc::kLayoutSw64);
            const uint64_t bdesc0 = tc::smem_desc(b_half(0, 0), 16, kRowGroupBytes, tc::kLayoutSw64);
            for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
                const int K = unit_offsets[u + 1] - unit_offsets[u];
                if (K == 0) continue;
                const int npass = (K + kSlots - 1) / kSlots;
                const int njobs = npass == 1 ? 1 : (ev ? npass : 2 * npass);
                for (int jb = 0; jb < njobs && ok; ++jb, ++job) {
                    const int p = npass == 1 ? 0 : jb % npass;
                    const int ns = min(kSlots, K - p * kSlots);
                    const int nmb = ns > 128 ? 2 : 1;
                    const int buf = job & 1;
                    if (job >= 2) ok = tc::mbar_wait(&ms.tempty[buf], ((job / 2) + 1) & 1, err);
                    if (!ok) break;
                    tc::tc_fence_after();
                    for (int j = 0; j < nsteps && ok; ++j, ++it) {
                        const int sa = it % kSA, sb = it % kSB;
                        ok = tc::mbar_wait(&ms.full_a[sa], (it / kSA) & 1, err) &&
                             tc::mbar_wait(&ms.full_b[sb], (it / kSB) & 1, err);
                        if (!ok) break;
                        tc::tc_fence_after();
                        // descriptors of the stage: the start-address field counts 16-byte units, so an
                        // offset within the stage is added to the stage's base descriptors
                        const uint64_t bh0 = bdesc0 + (uint64_t)((sb * kBStage) >> 4);
                        const uint64_t bl0 = bh0 + (uint64_t)(kBHalf >> 4);
                        const uint64_t ah0 = adesc0 + (uint64_t)((sa * kAStage) >> 4);
                        const uint64_t al0 = ah0 + (uint64_t)(kAHalf >> 4);
#pragma unroll
                        for (int ks = 0; ks < kKC / 16; ++ks) {
                            // K step ks = channels 16 ks .. 16 ks + 15: 32 bytes into each swizzled row
                            const uint64_t bh = bh0 + (uint64_t)(ks * 2);
                            const uint64_t bl = bl0 + (uint64_t)(ks * 2);
                            for (int mb = 0; mb < nmb; ++mb) {
                                const uint64_t ao = (uint64_t)((mb * kMBlockBytes + ks * 32) >> 4);
                                const uint64_t ah = ah0 + ao;
                                const uint64_t al = al0 + ao;
                                const uint32_t d = tmem + (uint32_t)(buf * kBufCols + mb * kUV);
                                tc::mma_f16_ss(d, ah, bh, kIdesc, j > 0 || ks > 0);
                                tc::mma_f16_ss(d, ah, bl, kIdesc, true);
                                tc::mma_f16_ss(d, al, bh, kIdesc, true);
                            }
                        }
                        tc::mma_commit(tc::smem_u32(&ms.empty_a[sa]));
                        tc::mma_commit(tc::smem_u32(&ms.empty_b[sb]));
                    }
                    tc::mma_commit(tc::smem_u32(&ms.tfull[buf]));
                }
            }
        }
    } else if (warp == 9) {
        // ============ TMA thread: the unit's gradient box of each step into the staging ring ============
        if (kTma && lane == 0) {
            int it = 0, issued = 0;
            const uint64_t pol = tc::l2_policy_evict_first();  // the gradient is streamed once per pass
            for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
                const int K = unit_offsets[u + 1] - unit_offsets[u];
                if (K == 0) continue;
                const UnitGeom ug = unit_geom(u, G.tiles[1], tzp_n, tx_begin);
                const int npass = (K + kSlots - 1) / kSlots;
                const int njobs = npass == 1 ? 1 : (ev ? npass : 2 * npass);
                for (int jb = 0; jb < njobs && ok; ++jb) {
                    for (int j = 0; j < nsteps && ok; ++j, ++it) {
                        const int gs = it % kGS;
                        if (it >= kGS) ok = tc::mbar_wait(&ms.gempty[gs], ((it / kGS) + 1) & 1, err);
                        if (!ok) break;
                        tc::mbar_arrive_expect_tx(&ms.gfull[gs], kGBytes);
                        tc::tma_load_4d_hint(tc::smem_u32(gstage + gs * kGBytes), &gmap, j * kKC, ug.tzp * 8,
                                             ug.ty * kTile, ug.tx * kTile - G.xoff, &ms.gfull[gs], pol);
                        issued = it + 1;
                    }
                }
            }
            // no copy may still be in flight when the shared memory is released
            for (int k = max(0, issued - kGS); k < issued; ++k)
                tc::mbar_wait_drain(&ms.gfull[k % kGS], (k / kGS) & 1, err);
        }
    } else {
        // ============ epilogue warps: thread = Gaussian slot (TMEM lane) ============
        const int et = tid - kEpiWarp0 * 32;     // 0..255
        const int q = warp & 3;                  // TMEM lane quarter of this warp
        const int ew = warp - kEpiWarp0;         // 0..7
        const int mb = ew >> 2;                  // M-block
        const int sl = mb * 128 + q * 32 + lane; // slot within a pass
        const float k2 = tc::kNegHalfLog2e;
        const float hz = G.h[2];
        int job = 0;
        for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
            const int s0 = unit_offsets[u], K = unit_offsets[u + 1] - s0;
            if (K == 0) continue;
            const UnitGeom ug = unit_geom(u, G.tiles[1], tzp_n, tx_begin);
            const int x0 = ug.tx * kTile, y0 = ug.ty * kTile, z0 = ug.tzp * 8;
            // voxel data of the unit (the previous unit's epilogue is complete: barrier at its end)
            if (et < kUV) {
                const int x = x0 + (et >> 5), y = y0 + ((et >> 3) & 3), z = z0 + (et & 7);
                const bool in = x < G.dims[0] && y < G.dims[1] && z < G.dims[2];
                const int64_t row = in ? grid_row(G, x, y, z) : 0;
                const float D = in ? density[row] : 0.0f;
                const float den = fmaxf(D, kEps);
                ms.lrd[et] = in ? -log2f(den) : -INFINITY;
                ms.gD[et] = in ? grad_density[row] : 0.0f;
                ms.rden[et] = in ? 1.0f / den : 0.0f;
                ms.act[et] = D >= kEps ? 1.0f : 0.0f;
                ms.e[et] = 0.0f;
                if (ev && K > kSlots) {  // e_v of a multi-pass unit, formed from grid_feats beforehand
                    const float e = in ? ev[row] : 0.0f;
                    ms.e[et] = e;
                    ms.va[et] = make_float2(ms.rden[et], fmaf(-ms.act[et] * e, ms.rden[et], ms.gD[et]));
                }
            }
            epi_barrier();
            const float cz0 = voxel_centre(G, 2, z0);
            const int npass = (K + kSlots - 1) / kSlots;
            const int njobs = npass == 1 ? 1 : (ev ? npass : 2 * npass);
            for (int jb = 0; jb < njobs; ++jb, ++job) {
                const int p = npass == 1 ? 0 : jb % npass;
                // with e_v given (multi-pass units), every job is phase 2
                const bool do1 = npass == 1 || (!ev && jb < npass);  // phase 1 of this job
                const bool do2 = npass == 1 || ev || jb >= npass;    // phase 2 of this job
                const int buf = job & 1;
                const bool good = ok && tc::mbar_wait(&ms.tfull[buf], (job / 2) & 1, err);
                if (!good) ok = false;
                tc::tc_fence_after();
                const int slot0 = p * kSlots + mb * 128 + q * 32;  // first list index of this warp
                const bool wact = good && slot0 < K;                 // warp-uniform
                const int slot = p * kSlots + sl;
                const bool live = slot < K;
                const int g = unit_lists[s0 + (live ? slot : 0)];
                const GParams& gp = gparams[g];
                const float4 A = gp.w[0], P0 = gp.w[1], P1 = gp.w[2], P2 = gp.w[3], U = gp.w[4];
                const int lbx = __float_as_int(P2.y), lby = __float_as_int(P2.z), lbz = __float_as_int(P2.w);
                const int ubx = __float_as_int(U.x), uby = __float_as_int(U.y), ubz = __float_as_int(U.z);
                const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kBufCols + mb * kUV);
                // z mask of the 8 z voxels of the unit for this Gaussian (-inf outside its box)
                float mz[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) mz[i] = (live && z0 + i >= lbz && z0 + i <= ubz) ? 0.0f : -INFINITY;
                const float dz0 = cz0 - A.z;
                // along z the exponent is a quadratic in lz: k2 (a + b lz + P8 hz^2 lz^2)
                const float Qz = k2 * hz * hz * P2.x;
                if (do1) {
                    if (wact) {
#pragma unroll 1
                        for (int lx = 0; lx < kTile; ++lx) {
                            const float dx = voxel_centre(G, 0, x0 + lx) - A.x;
                            const bool inx = live && x0 + lx >= lbx && x0 + lx <= ubx;
#pragma unroll 1
                            for (int ly2 = 0; ly2 < 2; ++ly2) {
                                float Sv[16];
                                tc::tmem_ld16(taddr + lx * 32 + ly2 * 16, Sv);
#pragma unroll
                                for (int h = 0; h < 2; ++h) {
                                    const int ly = ly2 * 2 + h;
                                    const float dy = voxel_centre(G, 1, y0 + ly) - A.y;
                                    const bool iny = inx && y0 + ly >= lby && y0 + ly <= uby;
                                    const float qx = fmaf(P0.z, dz0, fmaf(P0.y, dy, P0.x * dx));
                                    const float qy = fmaf(P1.y, dz0, fmaf(P1.x, dy, P0.w * dx));
                                    const float qz = fmaf(P2.x, dz0, fmaf(P1.w, dy, P1.z * dx));
                                    const float ptz = fmaf(P2.x, dz0, fmaf(P1.y, dy, P0.z * dx));  // (P^T d)_z
                                    const float a0 = iny ? k2 * (dx * qx + dy * qy + dz0 * qz) : -INFINITY;
                                    const float b0 = k2 * hz * (qz + ptz);
                                    const float4* L4 = reinterpret_cast<const float4*>(&ms.lrd[lx * 32 + ly * 8]);
                                    const float4 La = L4[0], Lb = L4[1];
                                    const float L[8] = {La.x, La.y, La.z, La.w, Lb.x, Lb.y, Lb.z, Lb.w};
#pragma unroll
                                    for (int lz = 0; lz < 8; ++lz) {
                                        const float m =
                                            fmaf(fmaf(Qz, (float)lz, b0), (float)lz, a0) + (L[lz] + mz[lz]);
                                        Sv[h * 8 + lz] *= A.w * tc::exp2_approx(m);
                                    }
                                }
                                const float r = warp_reduce_scatter16(Sv, lane);
                                if ((lane & 1) == 0) ms.epart[ew][lx * 32 + ly2 * 16 + (lane >> 1)] = r;
                            }
                        }
                    } else {
                        for (int i = lane; i < kUV; i += 32) ms.epart[ew][i] = 0.0f;
                    }
                    epi_barrier();
                    if (et < kUV) {
                        float acc = ms.epart[0][et];
#pragma unroll
                        for (int w = 1; w < 8; ++w) acc += ms.epart[w][et];
                        const float ev = ms.e[et] + acc;
                        ms.e[et] = ev;
                        // a = gD + (S - act e) / den = S * rden + (gD - act e rden)
                        ms.va[et] = make_float2(ms.rden[et], fmaf(-ms.act[et] * ev, ms.rden[et], ms.gD[et]));
                    }
                    epi_barrier();
                }
                if (do2 && wact) {
                    // Per x-slice of a tile, with q = P d = q0 + ly u + lz w (u = hy P e_y, w = hz P e_z):
                    //   sum aw q    = q0 M00 + u M10 + w M01
                    //   sum aw q q' = q0 q0' M00 + (q0 u' + u q0') M10 + (q0 w' + w q0') M01
                    //                 + u u' M20 + (u w' + w u') M11 + w w' M02
                    // with the moments M_ab = sum over the slice of a ex ly^a lz^b (aw = o a ex; o applied at the end)
                    const float hy = G.h[1];
                    const float ux = hy * P0.y, uy = hy * P1.x, uz = hy * P1.w;  // hy P[:, 1]
                    const float wx = hz * P0.z, wy = hz * P1.y, wz = hz * P2.x;  // hz P[:, 2]
                    const float Qyy = k2 * hy * hy * P1.x, Qyz = k2 * hy * hz * (P1.y + P1.w);
#pragma unroll
                    for (int t = 0; t < 2; ++t) {
                        const int tz = ug.tzp * 2 + t;
                        if (tz >= G.tiles[2]) break;
                        const bool tin = live && tz * kTile + 3 >= lbz && tz * kTile <= ubz;
                        if (!__any_sync(0xffffffffu, tin)) continue;
                        float gr[10];
#pragma unroll
                        for (int i = 0; i < 10; ++i) gr[i] = 0.0f;
                        const float dzt = fmaf((float)(4 * t), hz, dz0);  // slice origin z offset
                        const float dy0 = voxel_centre(G, 1, y0) - A.y;
#pragma unroll 1
                        for (int lx = 0; lx < kTile; ++lx) {
                            const float dx = voxel_centre(G, 0, x0 + lx) - A.x;
                            const bool inx = tin && x0 + lx >= lbx && x0 + lx <= ubx;
                            // slice origin: q0 = P d0, the exponent k2 (d' P d) as a quadratic in (ly, lz)
                            const float q0x = fmaf(P0.z, dzt, fmaf(P0.y, dy0, P0.x * dx));
                            const float q0y = fmaf(P1.y, dzt, fmaf(P1.x, dy0, P0.w * dx));
                            const float q0z = fmaf(P2.x, dzt, fmaf(P1.w, dy0, P1.z * dx));
                            const float pty = fmaf(P1.w, dzt, fmaf(P1.x, dy0, P0.y * dx));  // (P' d0)_y
                            const float ptz = fmaf(P2.x, dzt, fmaf(P1.y, dy0, P0.z * dx));  // (P' d0)_z
                            const float a0 = inx ? k2 * (dx * q0x + dy0 * q0y + dzt * q0z) : -INFINITY;
                            const float by = k2 * hy * (q0y + pty), bz = k2 * hz * (q0z + ptz);
                            float M00 = 0.f, M10 = 0.f, M01 = 0.f, M20 = 0.f, M11 = 0.f, M02 = 0.f;
#pragma unroll
                            for (int ly2 = 0; ly2 < 2; ++ly2) {
                                float Sv[16];
                                tc::tmem_ld16(taddr + lx * 32 + ly2 * 16, Sv);
#pragma unroll
                                for (int h = 0; h < 2; ++h) {
                                    const int ly = ly2 * 2 + h;
                                    const bool iny = y0 + ly >= lby && y0 + ly <= uby;
                                    const float ay = iny ? fmaf(fmaf(Qyy, (float)ly, by), (float)ly, a0) : -INFINITY;
                                    const float bzy = fmaf(Qyz, (float)ly, bz);
                                    const float4* V4 =
                                        reinterpret_cast<const float4*>(&ms.va[lx * 32 + ly * 8 + t * 4]);
                                    const float4 va01 = V4[0], va23 = V4[1];
                                    const float vax[4] = {va01.x, va01.z, va23.x, va23.z};
                                    const float vay[4] = {va01.y, va01.w, va23.y, va23.w};
#pragma unroll
                                    for (int lz = 0; lz < 4; ++lz) {
                                        const float m = fmaf(fmaf(Qz, (float)lz, bzy), (float)lz, ay) + mz[t * 4 + lz];
                                        const float ex = tc::exp2_approx(m);
                                        const float ae = fmaf(Sv[h * 8 + t * 4 + lz], vax[lz], vay[lz]) * ex;
                                        M00 += ae;
                                        M10 = fmaf(ae, (float)ly, M10);
                                        M01 = fmaf(ae, (float)lz, M01);
                                        M20 = fmaf(ae, (float)(ly * ly), M20);
                                        M11 = fmaf(ae, (float)(ly * lz), M11);
                                        M02 = fmaf(ae, (float)(lz * lz), M02);
                                    }
                                }
                            }
                            gr[9] += M00;
                            gr[0] = fmaf(q0x, M00, fmaf(ux, M10, fmaf(wx, M01, gr[0])));
                            gr[1] = fmaf(q0y, M00, fmaf(uy, M10, fmaf(wy, M01, gr[1])));
                            gr[2] = fmaf(q0z, M00, fmaf(uz, M10, fmaf(wz, M01, gr[2])));
                            // (i, j) component of sum aw q q'
                            auto qq = [&](float q0i, float ui, float wi, float q0j, float uj, float wj) {
                                return q0i * q0j * M00 + (q0i * uj + ui * q0j) * M10 + (q0i * wj + wi * q0j) * M01 +
                                       ui * uj * M20 + (ui * wj + wi * uj) * M11 + wi * wj * M02;
                            };
                            gr[3] += qq(q0x, ux, wx, q0x, ux, wx);
                            gr[4] += qq(q0y, uy, wy, q0y, uy, wy);
                            gr[5] += qq(q0z, uz, wz, q0z, uz, wz);
                            gr[6] += qq(q0x, ux, wx, q0y, uy, wy);
                            gr[7] += qq(q0x, ux, wx, q0z, uz, wz);
                            gr[8] += qq(q0y, uy, wy, q0z, uz, wz);
                        }
                        if (tin) {
                            const float o = A.w, oh = 0.5f * A.w;
#pragma unroll
                            for (int i = 0; i < 3; ++i) gr[i] *= o;
#pragma unroll
                            for (int i = 3; i < 9; ++i) gr[i] *= oh;
                            const int tlx = lbx / kTile, tly = lby / kTile, tlz = lbz / kTile;
                            const int ey = uby / kTile - tly + 1, ez = ubz / kTile - tlz + 1;
                            const int64_t idx =
                                (int64_t)g2t_offsets[g] + ((ug.tx - tlx) * ey + (ug.ty - tly)) * ez + (tz - tlz);
                            if (idx >= 0 && idx < pair_cap) {  // offsets come from the caller
                                float* out = partial10 + idx * 10;
#pragma unroll
                                for (int i = 0; i < 10; ++i) out[i] = gr[i];
                            }
                        }
                    }
                }
                // this job's S has been read: hand the buffer back to the MMA thread
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&ms.tempty[buf]);
            }
            epi_barrier();  // the unit's voxel data may be overwritten now
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
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
        float x[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = c + e < C ? f[g * C + c + e] : 0.0f;
        uint4 h, l;
        tc::split_bf16x2(x[0], x[1], h.x, l.x);
        tc::split_bf16x2(x[2], x[3], h.y, l.y);
        tc::split_bf16x2(x[4], x[5], h.z, l.z);
        tc::split_bf16x2(x[6], x[7], h.w, l.w);
        *reinterpret_cast<uint4*>(hi + g * Cp + c) = h;
        *reinterpret_cast<uint4*>(lo + g * Cp + c) = l;
    }
}
}  // namespace

int64_t spass_tc_padded_channels(int64_t C) { return (C + kKC - 1) / kKC * kKC; }

size_t spass_tc_split_bytes(int64_t n, int64_t C) {
    return (size_t)2 * (size_t)(n > 0 ? n : 1) * (size_t)spass_tc_padded_channels(C) * sizeof(__nv_bfloat16) + 256;
}

// The pass works on cells of 1 x 1 x 2 tiles (z pairs).
void spass_tc_unit_shape(const Grid& G, int cell[3], int ncells[3]) {
    cell[0] = 1;
    cell[1] = 1;
    cell[2] = 2;
    ncells[0] = G.tiles[0];
    ncells[1] = G.tiles[1];
    ncells[2] = (G.tiles[2] + 1) / 2;
}

namespace {
// e_v = sum_c gF_vc F_vc (F = grid_feats, the forward's output: the reference's at::bmm, cu:1996) for the
// voxels of the units with more than kSlots Gaussians, where forming e_v from S would need every slot
// pass twice.  Warp = one (unit, quad of 4 z-consecutive voxel rows) item of a grid-stride walk over all
// units: the unit check and the geometry are paid once per quad, the loads of the 4 rows are in flight
// together, and each row keeps the fixed per-lane channel order and warp reduction (deterministic).
__global__ void __launch_bounds__(256, 4) unit_ev_kernel(const int32_t* __restrict__ unit_offsets, int num_units,
                                                      int tzp_n, int tx_begin, Grid G,
                                                      const float* __restrict__ gF, const float* __restrict__ F,
                                                      int C, int vec, float* __restrict__ ev) {
    constexpr int kQuads = kUV / 4;  // 32 quads of a unit: x 4, y 4, z half 2
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t items = (int64_t)num_units * kQuads;
    for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < items; w += nw) {
        const int u = (int)(w / kQuads), q = (int)(w - (int64_t)u * kQuads);
        if (unit_offsets[u + 1] - unit_offsets[u] <= kSlots) continue;  // warp-uniform
        const UnitGeom ug = unit_geom(u, G.tiles[1], tzp_n, tx_begin);
        const int x = ug.tx * kTile + (q >> 3), y = ug.ty * kTile + ((q >> 1) & 3);
        const int z0 = ug.tzp * 8 + (q & 1) * 4;
        if (x >= G.dims[0] || y >= G.dims[1] || z0 >= G.dims[2]) continue;  // warp-uniform
        const int nz = min(4, G.dims[2] - z0);                               // rows of the quad in the grid
        int64_t rows[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) rows[i] = grid_row(G, x, y, z0 + (i < nz ? i : 0));
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (vec) {
            for (int c = 4 * lane; c < C; c += 128) {
                float4 p[4], r[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    if (i < nz) {
                        p[i] = *reinterpret_cast<const float4*>(gF + rows[i] * C + c);
                        r[i] = *reinterpret_cast<const float4*>(F + rows[i] * C + c);
                    }
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    if (i < nz) {
                        acc[i] = fmaf(p[i].x, r[i].x, acc[i]);
                        acc[i] = fmaf(p[i].y, r[i].y, acc[i]);
                        acc[i] = fmaf(p[i].z, r[i].z, acc[i]);
                        acc[i] = fmaf(p[i].w, r[i].w, acc[i]);
                    }
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if (i < nz)
                    for (int c = lane; c < C; c += 32) acc[i] = fmaf(gF[rows[i] * C + c], F[rows[i] * C + c], acc[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
            if (lane == 0 && i < nz) ev[rows[i]] = acc[i];
        }
    }
}
}  // namespace

int launch_spass_tc(const float* grad_density, const float* grad_feats, const float* features, int64_t n, int C,
                    const float* density, const GParams* gparams, const int32_t* g2t_offsets,
                    const int32_t* unit_offsets, const int32_t* unit_lists, int tile_x_begin, int tile_x_end,
                    const Grid& G, float* partial10, int64_t pair_cap, void* split, int* err, cudaStream_t s,
                    const float* grid_feats, float* ev_buf) {
    const int num_units = (tile_x_end - tile_x_begin) * G.tiles[1] * ((G.tiles[2] + 1) / 2);
    if (num_units <= 0 || C <= 0 || n <= 0) return 0;
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
    CUtensorMap gmap;
    memset(&gmap, 0, sizeof(gmap));
    const int ldims[3] = {G.xlen, G.dims[1], G.dims[2]};
    const bool tma = encode_grid_rows_f32(&gmap, grad_feats, ldims, C, kKC, 8, kTile, kTile, /*swizzle128*/ true);
    auto kern = tma ? spass_tc_kernel<true> : spass_tc_kernel<false>;
    G2V_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    int dev = 0, sms = 148;
    G2V_CUDA(cudaGetDevice(&dev));
    G2V_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int grid = std::min(num_units, sms);
    // e_v of the multi-pass units from grid_feats (when the caller passed it)
    const float* ev = nullptr;
    if (grid_feats != nullptr && ev_buf != nullptr) {
        const int vec = (C % 4 == 0) && (reinterpret_cast<uintptr_t>(grad_feats) % 16 == 0) &&
                        (reinterpret_cast<uintptr_t>(grid_feats) % 16 == 0);
        // 8 warps per block, as many blocks as are resident at once (__launch_bounds__(256, 4): four per
        // SM): the grid-stride walk covers every (unit, row quad) item
        const int64_t ev_blocks = std::min<int64_t>((int64_t)sms * 4, ((int64_t)num_units * (kUV / 4) + 7) / 8);
        G2V_TIMED("unit_ev_kernel", s,
                  unit_ev_kernel<<<(unsigned)ev_blocks, 256, 0, s>>>(unit_offsets, num_units, (G.tiles[2] + 1) / 2,
                                                                     tile_x_begin, G, grad_feats, grid_feats, C, vec,
                                                                     ev_buf));
        G2V_LAUNCH_CHECK("unit_ev_kernel");
        ev = ev_buf;
    }
    G2V_TIMED("spass_tc_kernel", s,
              kern<<<(unsigned)grid, kThreads, kSmemBytes, s>>>(gmap, grad_density, grad_feats, Fh, Fl, C, Cp,
                                                                  density, gparams, g2t_offsets, unit_offsets,
                                                                  unit_lists, num_units, tile_x_begin, G, partial10,
                                                                  pair_cap, ev, err));
    G2V_LAUNCH_CHECK("spass_tc_kernel");
    return 0;
}

}  // namespace g2v
