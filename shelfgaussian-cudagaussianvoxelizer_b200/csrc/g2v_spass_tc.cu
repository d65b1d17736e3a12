// g2v_spass_tc.cu -- tile pass of the backward on the tensor cores (tcgen05 cta_group::2, kind::f16, bf16).
//
// For the Gaussians of a unit of tiles (reference ComputeGaussian2VoxelGradientTileWithFeats,
// src/cuda_gaussian_voxelizer.cu:1376-1482, with e_v formed from S instead of reading grid_feats):
//   S_gv  = sum_c f_gc gF_vc                        (tensor cores, S in TMEM)
//   e_v   = sum_g (w_gv / den_v) S_gv               (epilogue, phase 1)
//   a_gv  = gD_v + (S_gv - [D_v >= eps] e_v) / den_v
//   the ten gradient partials of every (Gaussian, tile) pair = sums over the tile's voxels (phase 2),
// written at the pair's position in the Gaussian->Tile CSR like the FP32-FMA variant (g2v_grad.cu).
//
// Unit of work: a column of four z-consecutive tiles (4 x 4 x 16 = 256 voxels, v = (lx * 4 + ly) * 16 +
// lz) with the union of their Gaussian lists (ascending ids; the lists the forward splat built).  A
// cluster of two CTAs (a pair) shares every MMA: M = 256 Gaussian slots per pass (CTA r holds slots
// 128 r .. 128 r + 127: its A rows and its TMEM lanes), N = 256 voxels (CTA r holds the B rows of voxels
// 128 r .. 128 r + 127, i.e. lx = 2r, 2r + 1), K = 32 channels per pipeline step (two MMAs of K = 16).
// Each CTA's TMEM gets its 128 slots x all 256 voxels (256 columns), so a CTA double-buffers S in its
// 512 columns and the epilogue of a job overlaps the MMAs of the next.  Both operands are K-major with
// 64-byte swizzle (a row = the step's 32 channels; atoms of 8 rows x 64 bytes, 16-byte chunk c of row r
// at chunk c ^ ((r / 2) % 4)).  A rows are the features, pre-split once into bf16 hi/lo and stored per
// step as one 128-byte line [hi 32 channels | lo 32 channels] (rows padded to Cp channels), gathered with
// 16-byte cp.async by 8 threads per row, so one warp instruction fetches 4 whole lines; B rows are the upstream gradient of the CTA's 128 voxels,
// one tiled TMA load of the 4-D tensor map {C, Z, Y, X} per step (128-byte swizzle), converted fp32 ->
// bf16 hi/lo in shared memory (zero fill beyond the grid).  hi*hi + hi*lo + lo*hi is accumulated in fp32
// (~2^-16 relative per product).  When the tensor map cannot be built (C % 4 != 0, unaligned base) the
// converting threads load the gradient rows themselves.
//
// Roles per CTA (512 threads, 16 warps: four per SM sub-partition, 128 registers each): warps 0-1 gather
// feature rows (5-stage ring shared with the converted gradient rows, L2 evict_last), warps 2-5 convert
// gradient rows (their fp32 rows stream through a 3-stage staging ring with L2 evict_first), warp 6
// issues the pair's MMAs (leader) or forwards the completion of this CTA's stages to the leader (other
// CTA), warp 7 issues the TMA loads, warps 8-15 run the epilogue: thread = (slot, z half) of this CTA.  The e_v of a job needs the slots of both CTAs:
// each CTA sums its own slots and sends the 256 sums to the other with st.async (completion counted in
// bytes on the receiver's mbarrier); both add the two halves in rank order, so e_v is bitwise the same
// in both.  A unit of one pass is one job (phase 1 then phase 2 on the same S); a longer list runs every
// pass twice, phase 1 over all passes first, then the MMAs again for phase 2 -- or, when e_v is given
// (read from grid_feats beforehand, as the reference's bmm does), every pass once.  Every mbarrier wait
// is bounded, and both CTAs of a pair walk the same units and jobs and always meet at the closing
// cluster barrier.
#include <algorithm>
#include <cstddef>
#include <cstdlib>
#include <cstring>

#include "g2v_internal.cuh"
#include "g2v_tc.cuh"
#include "g2v_tmap.cuh"

namespace g2v {

namespace {
constexpr int kThreads = 512;
constexpr int kSlots = 256;                       // Gaussians per pass (both CTAs)
constexpr int kSlotsCta = 128;                    // Gaussians per pass held by one CTA
constexpr int kKC = 32;                           // channels per pipeline step
constexpr int kS = 5;                             // operand stages (feature rows + gradient rows)
constexpr int kGS = 3;                            // staging stages of the fp32 gradient
constexpr int kUZ = 4 * kTile;                    // voxels of a unit along z (four tiles)
constexpr int kUV = kTile * kTile * kUZ;          // 256 voxels of a unit
constexpr int kHV = kUV / 2;                      // 128 voxels (B rows) held by one CTA
constexpr int kAHalf = kSlotsCta * kKC * 2;       // 8 KB: one of hi / lo
constexpr int kBHalf = kHV * kKC * 2;             // 8 KB
constexpr int kStage = 2 * kAHalf + 2 * kBHalf;   // A hi, A lo, B hi, B lo
constexpr int kGBytes = kHV * kKC * 4;            // 16 KB: [x2][y4][z16][32 channels], 128-byte swizzle
static_assert(kKC * 4 == 128, "the staging rows are one 128-byte swizzle span");
static_assert(kKC * 2 == 64, "a K-major row of the step is one 64-byte swizzle span");
constexpr int kRowGroupBytes = 8 * kKC * 2;       // 8 rows x kKC bf16: one 64-byte-swizzle atom

// Byte offset of 16-byte chunk c of row r in a K-major 64-byte-swizzled operand.
__device__ __forceinline__ uint32_t sw64_off(int r, int c) {
    return (uint32_t)((r >> 3) * kRowGroupBytes + (r & 7) * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}
constexpr uint32_t kTmemCols = 512;               // two S buffers of 256 voxel columns
constexpr int kEpiWarp0 = 8;                      // first epilogue warp
constexpr uint32_t kIdesc = tc::idesc_bf16_f32(256, kUV, /*A K-major*/ 0, /*B K-major*/ 0);

struct SMisc {
    uint64_t full[kS];         // 64 cp.async arrivals (feature rows) + 4 converter warps
    uint64_t pfull[kS];        // leader: the other CTA's stage is full (forwarded arrival)
    uint64_t empty[kS];        // the pair's MMAs reading the stage completed (leader's commit, both CTAs)
    uint64_t gfull[kGS];       // TMA bytes of a staged step
    uint64_t gempty[kGS];      // 4 converter-warp arrivals
    uint64_t tfull[2];         // a job's S is complete in TMEM (leader's commit, both CTAs)
    uint64_t tempty[2];        // leader: 16 epilogue-warp arrivals (8 per CTA) -- S buffer read
    uint64_t xfull[2];         // the other CTA's 256 e_v sums arrived (1024 bytes) + own expect_tx
    uint32_t tmem_base;
    alignas(16) float lrd[kUV];   // log2(1 / max(D, eps)), -inf outside the grid
    alignas(16) float2 va[kUV];   // phase 2: a_gv = S_gv * va.x + va.y  (va.x = 1/den, va.y = gD - act e / den)
    float gD[kUV], act[kUV], rden[kUV], e[kUV];
    float epart[4][kUV];          // per lane quarter: sums over its 32 slots
    float xbuf[2][kUV];           // written by the other CTA (st.async)
};
constexpr size_t kSmemBytes = (size_t)kS * kStage + (size_t)kGS * kGBytes + sizeof(SMisc);
static_assert(kSmemBytes <= 227 * 1024, "spass_tc_kernel shared memory");

// 8 per-lane values -> each lane quad (4i .. 4i + 3) holds the warp sum of value i (fixed order).
__device__ __forceinline__ float warp_reduce_scatter8(float (&p)[8], int lane) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const bool up = lane & 16;
        const float send = up ? p[i] : p[i + 4];
        const float keep = up ? p[i + 4] : p[i];
        p[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const bool up = lane & 8;
        const float send = up ? p[i] : p[i + 2];
        const float keep = up ? p[i + 2] : p[i];
        p[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    {
        const bool up = lane & 4;
        const float send = up ? p[0] : p[1];
        const float keep = up ? p[1] : p[0];
        p[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    p[0] += __shfl_xor_sync(0xffffffffu, p[0], 2);
    return p[0] + __shfl_xor_sync(0xffffffffu, p[0], 1);  // value index (lane >> 2)
}

// Named barrier of the 8 epilogue warps (barrier 0 is __syncthreads).
__device__ __forceinline__ void epi_barrier() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Four 32 x 4 loads at columns taddr + 16 i (i = 0..3: the y rows of an x slice of one tile), one wait.
__device__ __forceinline__ void tmem_ld4x4(uint32_t taddr, float (&v)[4][4]) {
    uint32_t r[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(r[i][0]), "=r"(r[i][1]), "=r"(r[i][2]), "=r"(r[i][3])
                     : "r"(taddr + 16u * i));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) v[i][k] = __uint_as_float(r[i][k]);
}

// Unit u of the slab -> tile coordinates (tx, ty) and the z-quad index of its first tile.
struct UnitGeom {
    int tx, ty, tzq;
};
__device__ __forceinline__ UnitGeom unit_geom(int u, int ty_n, int tzq_n, int tx_begin) {
    UnitGeom g;
    const int yz = ty_n * tzq_n;
    g.tx = tx_begin + u / yz;
    const int r = u - (u / yz) * yz;
    g.ty = r / tzq_n;
    g.tzq = r - g.ty * tzq_n;
    return g;
}

// Number of jobs of a unit of K Gaussians: one per slot pass, or two per pass (phase 1 of all passes,
// then phase 2) when e_v is not given for a multi-pass unit.
__device__ __forceinline__ int unit_jobs(int K, bool have_ev) {
    const int npass = (K + kSlots - 1) / kSlots;
    return npass == 1 ? 1 : (have_ev ? npass : 2 * npass);
}

template <bool kTma>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1) spass_tc_kernel(
    const __grid_constant__ CUtensorMap gmap, const float* __restrict__ grad_density,
    const float* __restrict__ grad_feats, const __nv_bfloat16* __restrict__ Fs, int C, int Cp, const float* __restrict__ density, const GParams* __restrict__ gparams,
    const int32_t* __restrict__ g2t_offsets, const int32_t* __restrict__ unit_offsets,
    const int32_t* __restrict__ unit_lists, int num_units, int tx_begin, Grid G, float* __restrict__ partial10,
    int64_t pair_cap, const float* __restrict__ ev, int* __restrict__ err) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* stages = smem_raw;
    unsigned char* gstage = stages + kS * kStage;
    SMisc& ms = *reinterpret_cast<SMisc*>(gstage + kGS * kGBytes);
    // the swizzle atoms need 1 KB alignment; never expected, and the same in both CTAs of the pair, so
    // both leave before any cluster operation
    if ((tc::smem_u32(smem_raw) & 1023u) != 0) {
        if (threadIdx.x == 0) atomicOr(err, 2);
        return;
    }
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = tc::cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int tzq_n = (G.tiles[2] + 3) / 4;
    const int nsteps = Cp / kKC;
    const int64_t pitch = (int64_t)Cp * 4;  // bytes per split feature row (hi + lo)
    const bool have_ev = ev != nullptr;

    if (tid == 0) {
        for (int i = 0; i < kS; ++i) {
            tc::mbar_init(&ms.full[i], 64 + 4);
            tc::mbar_init(&ms.pfull[i], 1);
            tc::mbar_init(&ms.empty[i], 1);
        }
        for (int i = 0; i < kGS; ++i) {
            tc::mbar_init(&ms.gfull[i], 1);
            tc::mbar_init(&ms.gempty[i], 4);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&ms.tfull[i], 1);
            tc::mbar_init(&ms.tempty[i], 16);
            tc::mbar_init(&ms.xfull[i], 1);
        }
        tc::mbar_fence_init();
    }
    if (warp == 0) tc::tmem_alloc_pair(&ms.tmem_base, kTmemCols);
    tc::tc_fence_before();
    tc::cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
    tc::tc_fence_after();
    const uint32_t tmem = ms.tmem_base;
    bool ok = true;

    auto a_half = [&](int st, int hl) -> uint32_t { return tc::smem_u32(stages + st * kStage + hl * kAHalf); };
    auto b_half = [&](int st, int hl) -> unsigned char* { return stages + st * kStage + 2 * kAHalf + hl * kBHalf; };

    if (warp < 2) {
        // ============ feature-row producers (cp.async, kept in L2: evict_last) ============
        // thread = 16-byte chunk kc of the rows rg + 8 i (i = 0..15) of this CTA: chunks 0-3 are hi, 4-7 lo
        const int t = tid;
        const int kc = t & 7, rg = t >> 3;
        const char* fbase = reinterpret_cast<const char*>(Fs) + kc * 16;
        const uint64_t pol = tc::l2_policy_evict_last();
        int it = 0;
        for (int u = pair; u < num_units && ok; u += npairs) {
            const int s0 = unit_offsets[u], K = unit_offsets[u + 1] - s0;
            if (K == 0) continue;
            const int npass = (K + kSlots - 1) / kSlots;
            const int njobs = unit_jobs(K, have_ev);
            for (int jb = 0; jb < njobs && ok; ++jb) {
                const int p = npass == 1 ? 0 : jb % npass;
                int32_t grow[16];  // Gaussian of each row, -1 beyond the list (zero fill)
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int slot = p * kSlots + (int)rank * kSlotsCta + rg + 8 * i;
                    grow[i] = slot < K ? unit_lists[s0 + slot] : -1;
                }
                for (int j = 0; j < nsteps && ok; ++j, ++it) {
                    const int st = it % kS;
                    if (it >= kS) ok = tc::mbar_wait_cluster(&ms.empty[st], ((it / kS) + 1) & 1, err);
                    if (!ok) break;
                    const uint32_t dst0 = a_half(st, kc >> 2);
                    const char* fstep = fbase + (int64_t)j * 128;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int r = rg + 8 * i;
                        const bool valid = grow[i] >= 0;
                        tc::cp_async16_hint(dst0 + sw64_off(r, kc & 3), valid ? fstep + (int64_t)grow[i] * pitch : fbase,
                                            valid ? 16u : 0u, pol);
                    }
                    tc::cp_async_mbar_arrive_noinc(&ms.full[st]);
                }
            }
        }
        tc::cp_async_wait<0>();  // no copy in flight when the shared memory is released
    } else if (warp < 6) {
        // ============ gradient-row converters: staged fp32 -> bf16 hi / lo; thread = this CTA's voxel row t ============
        const int t = tid - 64;
        int it = 0;
        for (int u = pair; u < num_units && ok; u += npairs) {
            const int K = unit_offsets[u + 1] - unit_offsets[u];
            if (K == 0) continue;
            const UnitGeom ug = unit_geom(u, G.tiles[1], tzq_n, tx_begin);
            const int x = ug.tx * kTile + 2 * (int)rank + (t >> 6), y = ug.ty * kTile + ((t >> 4) & 3),
                      z = ug.tzq * kUZ + (t & 15);
            const int64_t vrow = (x < G.dims[0] && y < G.dims[1] && z < G.dims[2]) ? grid_row(G, x, y, z) : -1;
            const int njobs = unit_jobs(K, have_ev);
            for (int jb = 0; jb < njobs && ok; ++jb) {
                for (int j = 0; j < nsteps && ok; ++j, ++it) {
                    const int st = it % kS, gs = it % kGS;
                    if (it >= kS) ok = tc::mbar_wait_cluster(&ms.empty[st], ((it / kS) + 1) & 1, err);
                    if (kTma && ok) ok = tc::mbar_wait(&ms.gfull[gs], (it / kGS) & 1, err);
                    if (!ok) break;
                    unsigned char* bh = b_half(st, 0);
                    unsigned char* bl = b_half(st, 1);
#pragma unroll
                    for (int c = 0; c < 4; ++c) {  // 8 channels per 16-byte chunk of the bf16 row
                        float f[8];
                        if (kTma) {
                            // 128-byte swizzled staging row: logical chunk k sits at chunk k ^ (t % 8)
                            const unsigned char* row = gstage + gs * kGBytes + t * (kKC * 4);
                            const float4 x0 = *reinterpret_cast<const float4*>(row + (((2 * c) ^ (t & 7)) << 4));
                            const float4 x1 = *reinterpret_cast<const float4*>(row + (((2 * c + 1) ^ (t & 7)) << 4));
                            f[0] = x0.x; f[1] = x0.y; f[2] = x0.z; f[3] = x0.w;
                            f[4] = x1.x; f[5] = x1.y; f[6] = x1.z; f[7] = x1.w;
                        } else {
                            const int cc = j * kKC + c * 8;
#pragma unroll
                            for (int e = 0; e < 8; ++e)
                                f[e] = (vrow >= 0 && cc + e < C) ? grad_feats[vrow * C + cc + e] : 0.0f;
                        }
                        uint4 h4, l4;
                        tc::split_bf16x2_p(make_float2(f[0], f[1]), h4.x, l4.x);
                        tc::split_bf16x2_p(make_float2(f[2], f[3]), h4.y, l4.y);
                        tc::split_bf16x2_p(make_float2(f[4], f[5]), h4.z, l4.z);
                        tc::split_bf16x2_p(make_float2(f[6], f[7]), h4.w, l4.w);
                        const uint32_t o = sw64_off(t, c);
                        *reinterpret_cast<uint4*>(bh + o) = h4;
                        *reinterpret_cast<uint4*>(bl + o) = l4;
                    }
                    tc::fence_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tc::mbar_arrive(&ms.full[st]);
                        if (kTma) tc::mbar_arrive(&ms.gempty[gs]);
                    }
                }
            }
        }
    } else if (warp == 6) {
        if (lane == 0 && leader) {
            // ============ MMA thread of the pair ============
            int it = 0, job = 0;
            const uint64_t adesc0 = tc::smem_desc(tc::smem_u32(stages), 16, kRowGroupBytes, tc::kLayoutSw64);
            const uint64_t bdesc0 =
                tc::smem_desc(tc::smem_u32(stages + 2 * kAHalf), 16, kRowGroupBytes, tc::kLayoutSw64);
            for (int u = pair; u < num_units && ok; u += npairs) {
                const int K = unit_offsets[u + 1] - unit_offsets[u];
                if (K == 0) continue;
                const int njobs = unit_jobs(K, have_ev);
                for (int jb = 0; jb < njobs && ok; ++jb, ++job) {
                    const int buf = job & 1;
                    // the S buffer's previous job has been read by both CTAs' epilogues
                    if (job >= 2) ok = tc::mbar_wait_cluster(&ms.tempty[buf], ((job / 2) + 1) & 1, err);
                    if (!ok) break;
                    tc::tc_fence_after();
                    const uint32_t d = tmem + (uint32_t)(buf * kUV);
                    // two steps per iteration: the waits, the proxy fence and the loop are paid once per 64
                    // channels (the second step's stage is normally complete already)
                    for (int j = 0; j < nsteps && ok; j += 2) {
                        const int nj = min(2, nsteps - j);
                        const int st0 = it % kS, st1 = (it + 1) % kS;
                        ok = tc::mbar_wait(&ms.full[st0], (it / kS) & 1, err) &&
                             tc::mbar_wait_cluster(&ms.pfull[st0], (it / kS) & 1, err);
                        if (ok && nj == 2)
                            ok = tc::mbar_wait(&ms.full[st1], ((it + 1) / kS) & 1, err) &&
                                 tc::mbar_wait_cluster(&ms.pfull[st1], ((it + 1) / kS) & 1, err);
                        if (!ok) break;
                        // the A rows were written by cp.async, the B rows by ordinary stores: order them
                        // before the MMAs' async-proxy reads
                        tc::fence_async_smem();
                        tc::tc_fence_after();
                        for (int h2 = 0; h2 < nj; ++h2) {
                            const int st = h2 ? st1 : st0;
                            const uint64_t so = (uint64_t)((st * kStage) >> 4);  // start address in 16-byte units
#pragma unroll
                            for (int ks = 0; ks < kKC / 16; ++ks) {
                                // K step ks = channels 16 ks .. 16 ks + 15: 32 bytes into each swizzled row
                                const uint64_t ah = adesc0 + so + (uint64_t)(ks * 2);
                                const uint64_t al = ah + (uint64_t)(kAHalf >> 4);
                                const uint64_t bh = bdesc0 + so + (uint64_t)(ks * 2);
                                const uint64_t bl = bh + (uint64_t)(kBHalf >> 4);
                                tc::mma_f16_ss_pair<tc::kColFill>(d, ah, bh, kIdesc, j + h2 > 0 || ks > 0);
                                tc::mma_f16_ss_pair<tc::kColLastUse>(d, ah, bl, kIdesc, true);
                                tc::mma_f16_ss_pair(d, al, bh, kIdesc, true);
                            }
                            tc::mma_commit_pair(tc::smem_u32(&ms.empty[st]), (uint16_t)3);
                        }
                        it += nj;
                    }
                    tc::mma_commit_pair(tc::smem_u32(&ms.tfull[buf]), (uint16_t)3);
                }
            }
        } else if (lane == 0) {
            // ============ forwarder (second CTA): this CTA's stage is full -> the leader's pfull ============
            int it = 0;
            for (int u = pair; u < num_units && ok; u += npairs) {
                const int K = unit_offsets[u + 1] - unit_offsets[u];
                if (K == 0) continue;
                const int njobs = unit_jobs(K, have_ev);
                for (int jb = 0; jb < njobs && ok; ++jb) {
                    for (int j = 0; j < nsteps && ok; ++j, ++it) {
                        const int st = it % kS;
                        ok = tc::mbar_wait(&ms.full[st], (it / kS) & 1, err);
                        if (!ok) break;
                        // The stage's rows are complete in this CTA's shared memory (cp.async completion and
                        // the converters' stores + proxy fence, acquired through full[st]); the leader's MMAs
                        // read them after its own acquire of pfull and proxy fence.  A release arrive here
                        // adds nothing but its cost (it paced the whole pipeline).
                        tc::mbar_arrive_cluster_relaxed(tc::mapa_shared(tc::smem_u32(&ms.pfull[st]), 0));
                    }
                }
            }
        }
    } else if (warp == 7) {
        // ============ TMA thread: this CTA's half of the unit's gradient box of each step ============
        if (kTma && lane == 0) {
            int it = 0, issued = 0;
            const uint64_t pol = tc::l2_policy_evict_first();  // the gradient is streamed once per pass
            for (int u = pair; u < num_units && ok; u += npairs) {
                const int K = unit_offsets[u + 1] - unit_offsets[u];
                if (K == 0) continue;
                const UnitGeom ug = unit_geom(u, G.tiles[1], tzq_n, tx_begin);
                const int njobs = unit_jobs(K, have_ev);
                for (int jb = 0; jb < njobs && ok; ++jb) {
                    for (int j = 0; j < nsteps && ok; ++j, ++it) {
                        const int gs = it % kGS;
                        if (it >= kGS) ok = tc::mbar_wait(&ms.gempty[gs], ((it / kGS) + 1) & 1, err);
                        if (!ok) break;
                        tc::mbar_arrive_expect_tx(&ms.gfull[gs], kGBytes);
                        tc::tma_load_4d_hint(tc::smem_u32(gstage + gs * kGBytes), &gmap, j * kKC, ug.tzq * kUZ,
                                             ug.ty * kTile, ug.tx * kTile + 2 * (int)rank - G.xoff, &ms.gfull[gs],
                                             pol);
                        issued = it + 1;
                    }
                }
            }
            // no copy may still be in flight when the shared memory is released
            for (int k = max(0, issued - kGS); k < issued; ++k)
                tc::mbar_wait_drain(&ms.gfull[k % kGS], (k / kGS) & 1, err);
        }
    } else {
        // ============ epilogue warps: thread = (this CTA's slot q * 32 + lane, z half / tile pair h) ============
        const int et = tid - kEpiWarp0 * 32;     // 0..255: the voxel of the per-voxel work
        const int q = warp & 3;                  // TMEM lane quarter of this warp
        const int h = (warp - kEpiWarp0) >> 2;   // z half of phase 1, tiles 2h, 2h + 1 of phase 2
        const int sl = (int)rank * kSlotsCta + q * 32 + lane;  // slot within a pass
        const float k2 = tc::kNegHalfLog2e;
        const float hy = G.h[1], hz = G.h[2];
        const uint32_t other = rank ^ 1u;
        const uint32_t other_xbuf = tc::mapa_shared(tc::smem_u32(&ms.xbuf[0][0]), other);
        const uint32_t other_xfull = tc::mapa_shared(tc::smem_u32(&ms.xfull[0]), other);
        const uint32_t lead_tempty = tc::mapa_shared(tc::smem_u32(&ms.tempty[0]), 0);
        int job = 0, nx = 0;
        for (int u = pair; u < num_units; u += npairs) {
            const int s0 = unit_offsets[u], K = unit_offsets[u + 1] - s0;
            if (K == 0) continue;
            const UnitGeom ug = unit_geom(u, G.tiles[1], tzq_n, tx_begin);
            const int x0 = ug.tx * kTile, y0 = ug.ty * kTile, z0 = ug.tzq * kUZ;
            // voxel data of the unit (the previous unit's epilogue is complete: barrier at its end)
            {
                const int v = et;
                const int x = x0 + (v >> 6), y = y0 + ((v >> 4) & 3), z = z0 + (v & 15);
                const bool in = x < G.dims[0] && y < G.dims[1] && z < G.dims[2];
                const int64_t row = in ? grid_row(G, x, y, z) : 0;
                const float D = in ? density[row] : 0.0f;
                const float den = fmaxf(D, kEps);
                ms.lrd[v] = in ? -log2f(den) : -INFINITY;
                ms.gD[v] = in ? grad_density[row] : 0.0f;
                ms.rden[v] = in ? 1.0f / den : 0.0f;
                ms.act[v] = D >= kEps ? 1.0f : 0.0f;
                ms.e[v] = 0.0f;
                if (have_ev && K > kSlots) {  // e_v of a multi-pass unit, formed from grid_feats beforehand
                    const float e = in ? ev[row] : 0.0f;
                    ms.e[v] = e;
                    ms.va[v] = make_float2(ms.rden[v], fmaf(-ms.act[v] * e, ms.rden[v], ms.gD[v]));
                }
            }
            epi_barrier();
            const float cz0 = voxel_centre(G, 2, z0);
            const int npass = (K + kSlots - 1) / kSlots;
            const int njobs = unit_jobs(K, have_ev);
            for (int jb = 0; jb < njobs; ++jb, ++job) {
                const int p = npass == 1 ? 0 : jb % npass;
                // with e_v given (multi-pass units), every job is phase 2
                const bool do1 = npass == 1 || (!have_ev && jb < npass);  // phase 1 of this job
                const bool do2 = npass == 1 || have_ev || jb >= npass;    // phase 2 of this job
                const int buf = job & 1;
                const bool good = ok && tc::mbar_wait_cluster(&ms.tfull[buf], (job / 2) & 1, err);
                if (!good) ok = false;
                tc::tc_fence_after();
                const int slot0 = p * kSlots + (int)rank * kSlotsCta + q * 32;  // first list index of this warp
                const bool wact = good && slot0 < K;                              // warp-uniform
                const int slot = p * kSlots + sl;
                const bool live = slot < K;
                const int g = unit_lists[s0 + (live ? slot : 0)];
                const GParams& gp = gparams[g];
                const float4 A = gp.w[0], P0 = gp.w[1], P1 = gp.w[2], P2 = gp.w[3], U = gp.w[4];
                const int lbx = __float_as_int(P2.y), lby = __float_as_int(P2.z), lbz = __float_as_int(P2.w);
                const int ubx = __float_as_int(U.x), uby = __float_as_int(U.y), ubz = __float_as_int(U.z);
                const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kUV);
                // z range of this Gaussian's box within the unit (outside: weight 0 through a -inf exponent)
                const int zlo = live ? lbz - z0 : kUZ, zhi = live ? ubz - z0 : -1;
                const float dz0 = cz0 - A.z;
                // along z the exponent is a quadratic in lz: k2 (a + b lz + P8 hz^2 lz^2)
                const float Qz = k2 * hz * hz * P2.x;
                if (do1) {
                    if (wact) {
                        // Qz lz^2 plus the z box mask (0 / -inf) of this thread's z half, as z pairs
                        float2 zh[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int l0 = 8 * h + 2 * i, l1 = l0 + 1;
                            zh[i] = make_float2((l0 >= zlo && l0 <= zhi) ? Qz * (float)(l0 * l0) : -INFINITY,
                                                (l1 >= zlo && l1 <= zhi) ? Qz * (float)(l1 * l1) : -INFINITY);
                        }
#pragma unroll 1
                        for (int lx = 0; lx < kTile; ++lx) {
                            const float dx = voxel_centre(G, 0, x0 + lx) - A.x;
                            const bool inx = live && x0 + lx >= lbx && x0 + lx <= ubx;
#pragma unroll 1
                            for (int ly = 0; ly < kTile; ++ly) {
                                const int vb = lx * 64 + ly * 16 + 8 * h;  // first voxel of the row half
                                float Sv[8];
                                tc::tmem_ld8(taddr + vb, Sv);
                                const float dy = voxel_centre(G, 1, y0 + ly) - A.y;
                                const bool iny = inx && y0 + ly >= lby && y0 + ly <= uby;
                                const float qx = fmaf(P0.z, dz0, fmaf(P0.y, dy, P0.x * dx));
                                const float qy = fmaf(P1.y, dz0, fmaf(P1.x, dy, P0.w * dx));
                                const float qz = fmaf(P2.x, dz0, fmaf(P1.w, dy, P1.z * dx));
                                const float ptz = fmaf(P2.x, dz0, fmaf(P1.y, dy, P0.z * dx));  // (P^T d)_z
                                const float a0 = iny ? k2 * (dx * qx + dy * qy + dz0 * qz) : -INFINITY;
                                const float b0 = k2 * hz * (qz + ptz);
                                const float4* L4 = reinterpret_cast<const float4*>(&ms.lrd[vb]);
                                const float4 La = L4[0], Lb = L4[1];
                                const float2 L2[4] = {make_float2(La.x, La.y), make_float2(La.z, La.w),
                                                      make_float2(Lb.x, Lb.y), make_float2(Lb.z, Lb.w)};
                                const float2 A2 = make_float2(a0, a0), B2 = make_float2(b0, b0);
                                const float2 O2 = make_float2(A.w, A.w);
#pragma unroll
                                for (int i = 0; i < 4; ++i) {
                                    // m = (a0 + Qz lz^2 + z mask + log2(1/den)) + lz b0 for lz = 8 h + 2 i, + 1
                                    const float l0 = (float)(8 * h + 2 * i);
                                    const float2 m = __ffma2_rn(make_float2(l0, l0 + 1.0f), B2,
                                                                __fadd2_rn(__fadd2_rn(A2, zh[i]), L2[i]));
                                    const float2 e = make_float2(tc::exp2_approx(m.x), tc::exp2_approx(m.y));
                                    const float2 sv = __fmul2_rn(make_float2(Sv[2 * i], Sv[2 * i + 1]), __fmul2_rn(O2, e));
                                    Sv[2 * i] = sv.x;
                                    Sv[2 * i + 1] = sv.y;
                                }
                                const float r = warp_reduce_scatter8(Sv, lane);
                                if ((lane & 3) == 0) ms.epart[q][vb + (lane >> 2)] = r;
                            }
                        }
                    } else {
                        for (int i = lane; i < kUV / 2; i += 32) ms.epart[q][(i >> 3) * 16 + 8 * h + (i & 7)] = 0.0f;
                    }
                    epi_barrier();
                    {
                        // this CTA's sum over its slots, sent to the other CTA; e_v adds both in rank order
                        const int v = et;
                        const float mine = ((ms.epart[0][v] + ms.epart[1][v]) + ms.epart[2][v]) + ms.epart[3][v];
                        const int xb = nx & 1;
                        if (et == 0) tc::mbar_arrive_expect_tx(&ms.xfull[xb], kUV * 4);
                        tc::st_async_f32(other_xbuf + (uint32_t)((xb * kUV + v) * 4), mine,
                                         other_xfull + (uint32_t)(xb * 8));
                        const bool got = tc::mbar_wait_cluster(&ms.xfull[xb], (nx >> 1) & 1, err);
                        if (!got) ok = false;
                        const float theirs = got ? ms.xbuf[xb][v] : 0.0f;
                        const float both = rank == 0 ? mine + theirs : theirs + mine;
                        const float ev2 = ms.e[v] + both;
                        ms.e[v] = ev2;
                        // a = gD + (S - act e) / den = S * rden + (gD - act e rden)
                        ms.va[v] = make_float2(ms.rden[v], fmaf(-ms.act[v] * ev2, ms.rden[v], ms.gD[v]));
                    }
                    ++nx;
                    epi_barrier();
                }
                if (do2 && wact) {
                    // Per x-slice of a tile, with q = P d = q0 + ly u + lz w (u = hy P e_y, w = hz P e_z):
                    //   sum aw q    = q0 M00 + u M10 + w M01
                    //   sum aw q q' = q0 q0' M00 + (q0 u' + u q0') M10 + (q0 w' + w q0') M01
                    //                 + u u' M20 + (u w' + w u') M11 + w w' M02
                    // with the moments M_ab = sum over the slice of a ex ly^a lz^b (aw = o a ex; o applied at the end)
                    const float ux = hy * P0.y, uy = hy * P1.x, uz = hy * P1.w;  // hy P[:, 1]
                    const float wx = hz * P0.z, wy = hz * P1.y, wz = hz * P2.x;  // hz P[:, 2]
                    const float Qyy = k2 * hy * hy * P1.x, Qyz = k2 * hy * hz * (P1.y + P1.w);
#pragma unroll 1
                    for (int tt = 0; tt < 2; ++tt) {
                        const int t = 2 * h + tt;
                        const int tz = ug.tzq * (kUZ / kTile) + t;
                        if (tz >= G.tiles[2]) break;
                        const bool tin = live && tz * kTile + 3 >= lbz && tz * kTile <= ubz;
                        if (!__any_sync(0xffffffffu, tin)) continue;
                        float gr[10];
#pragma unroll
                        for (int i = 0; i < 10; ++i) gr[i] = 0.0f;
                        // Qz lz^2 plus the z box mask (0 / -inf) of the tile's four z layers
                        float zq[4];
#pragma unroll
                        for (int lz = 0; lz < kTile; ++lz) {
                            const int zz = kTile * t + lz;
                            zq[lz] = (zz >= zlo && zz <= zhi) ? Qz * (float)(lz * lz) : -INFINITY;
                        }
                        const float2 Zq01 = make_float2(zq[0], zq[1]), Zq23 = make_float2(zq[2], zq[3]);
                        const float dzt = fmaf((float)(kTile * t), hz, dz0);  // slice origin z offset
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
                            float S4[4][4];
                            tmem_ld4x4(taddr + lx * 64 + kTile * t, S4);
#pragma unroll
                            for (int ly = 0; ly < kTile; ++ly) {
                                const float* Sv = S4[ly];
                                const bool iny = y0 + ly >= lby && y0 + ly <= uby;
                                const float ay = iny ? fmaf(fmaf(Qyy, (float)ly, by), (float)ly, a0) : -INFINITY;
                                const float bzy = fmaf(Qyz, (float)ly, bz);
                                const float4* V4 = reinterpret_cast<const float4*>(&ms.va[lx * 64 + ly * 16 + kTile * t]);
                                const float4 va01 = V4[0], va23 = V4[1];
                                // z pairs (0, 1), (2, 3) in packed f32x2 arithmetic: m = (ay + Qz lz^2 + z mask) + lz bzy
                                const float2 A2 = make_float2(ay, ay), B2 = make_float2(bzy, bzy);
                                const float2 m01 = __ffma2_rn(make_float2(0.0f, 1.0f), B2, __fadd2_rn(A2, Zq01));
                                const float2 m23 = __ffma2_rn(make_float2(2.0f, 3.0f), B2, __fadd2_rn(A2, Zq23));
                                const float2 e01 = make_float2(tc::exp2_approx(m01.x), tc::exp2_approx(m01.y));
                                const float2 e23 = make_float2(tc::exp2_approx(m23.x), tc::exp2_approx(m23.y));
                                // a e = (S * va.x + va.y) e
                                const float2 a01 = __fmul2_rn(__ffma2_rn(make_float2(Sv[0], Sv[1]), make_float2(va01.x, va01.z),
                                                                         make_float2(va01.y, va01.w)), e01);
                                const float2 a23 = __fmul2_rn(__ffma2_rn(make_float2(Sv[2], Sv[3]), make_float2(va23.x, va23.z),
                                                                         make_float2(va23.y, va23.w)), e23);
                                // row sums over lz of a e, lz a e, lz^2 a e; the ly moments from them
                                const float2 s0 = __fadd2_rn(a01, a23);
                                const float2 s1 = __ffma2_rn(make_float2(2.0f, 3.0f), a23, __fmul2_rn(make_float2(0.0f, 1.0f), a01));
                                const float2 s2 = __ffma2_rn(make_float2(4.0f, 9.0f), a23, __fmul2_rn(make_float2(0.0f, 1.0f), a01));
                                const float r0 = s0.x + s0.y, r1 = s1.x + s1.y, r2 = s2.x + s2.y;
                                const float fy = (float)ly;
                                M00 += r0;
                                M10 = fmaf(fy, r0, M10);
                                M20 = fmaf(fy * fy, r0, M20);
                                M01 += r1;
                                M11 = fmaf(fy, r1, M11);
                                M02 += r2;
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
                // this job's S buffer has been read by this warp: tell the leader's MMA thread
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive_cluster(lead_tempty + (uint32_t)(buf * 8));
            }
            epi_barrier();  // the unit's voxel data may be overwritten now
        }
    }
    tc::tc_fence_before();
    tc::cluster_sync();  // neither CTA frees TMEM or leaves while the pair still works on it
    tc::tc_fence_after();
    if (warp == 0) tc::tmem_dealloc_pair(tmem, kTmemCols);
}

// features [n][C] fp32 -> split rows of Cp channels (zero padded): per 32-channel step one 128-byte line
// [hi 32 | lo 32] (bf16); 8 channels per thread
__global__ void feature_split_bf16_kernel(const float* __restrict__ f, int64_t n, int C, int Cp,
                                          __nv_bfloat16* __restrict__ out) {
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
        __nv_bfloat16* row = out + g * 2 * Cp + (c / kKC) * (2 * kKC) + (c % kKC);
        *reinterpret_cast<uint4*>(row) = h;
        *reinterpret_cast<uint4*>(row + kKC) = l;
    }
}
}  // namespace

int64_t spass_tc_padded_channels(int64_t C) { return (C + kKC - 1) / kKC * kKC; }

size_t spass_tc_split_bytes(int64_t n, int64_t C) {
    return (size_t)2 * (size_t)(n > 0 ? n : 1) * (size_t)spass_tc_padded_channels(C) * sizeof(__nv_bfloat16) + 256;
}

// The tensor-core splat and tile pass list Gaussians per cell of 1 x 1 x 4 tiles (z quads).
void tc_unit_shape(const Grid& G, int cell[3], int ncells[3]) {
    cell[0] = 1;
    cell[1] = 1;
    cell[2] = 4;
    ncells[0] = G.tiles[0];
    ncells[1] = G.tiles[1];
    ncells[2] = (G.tiles[2] + 3) / 4;
}

namespace {
// e_v = sum_c gF_vc F_vc (F = grid_feats, the forward's output: the reference's at::bmm, cu:1996) for the
// voxels of the units with more than kSlots Gaussians, where forming e_v from S would need every slot
// pass twice.  Warp = one (unit, quad of 4 z-consecutive voxel rows) item of a grid-stride walk over all
// units: the unit check and the geometry are paid once per quad, the loads of the 4 rows are in flight
// together, and each row keeps the fixed per-lane channel order and warp reduction (deterministic).
__global__ void __launch_bounds__(256, 4) unit_ev_kernel(const int32_t* __restrict__ unit_offsets, int num_units,
                                                      int tzq_n, int tx_begin, Grid G,
                                                      const float* __restrict__ gF, const float* __restrict__ F,
                                                      int C, int vec, float* __restrict__ ev) {
    constexpr int kQuads = kUV / 4;  // 64 quads of a unit: x 4, y 4, z quarter 4
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t items = (int64_t)num_units * kQuads;
    for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < items; w += nw) {
        const int u = (int)(w / kQuads), q = (int)(w - (int64_t)u * kQuads);
        if (unit_offsets[u + 1] - unit_offsets[u] <= kSlots) continue;  // warp-uniform
        const UnitGeom ug = unit_geom(u, G.tiles[1], tzq_n, tx_begin);
        const int x = ug.tx * kTile + (q >> 4), y = ug.ty * kTile + ((q >> 2) & 3);
        const int z0 = ug.tzq * kUZ + (q & 3) * 4;
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

namespace {
// Clusters of two spass_tc_kernel CTAs that fit on the device at once (the persistent grid), per device.
int spass_pair_slots(const void* kern, int dev, int sms) {
    static int cached[64] = {0};
    if (dev >= 0 && dev < 64 && cached[dev] > 0) return cached[dev];
    int n = 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(sms & ~1), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        (void)cudaGetLastError();
        n = sms / 2;
    }
    if (dev >= 0 && dev < 64) cached[dev] = n;
    return n;
}
}  // namespace

int launch_spass_tc(const float* grad_density, const float* grad_feats, const float* features, int64_t n, int C,
                    const float* density, const GParams* gparams, const int32_t* g2t_offsets,
                    const int32_t* unit_offsets, const int32_t* unit_lists, int tile_x_begin, int tile_x_end,
                    const Grid& G, float* partial10, int64_t pair_cap, void* split, int* err, cudaStream_t s,
                    const float* grid_feats, float* ev_buf) {
    const int tzq_n = (G.tiles[2] + 3) / 4;
    const int num_units = (tile_x_end - tile_x_begin) * G.tiles[1] * tzq_n;
    if (num_units <= 0 || C <= 0 || n <= 0) return 0;
    const int Cp = (int)spass_tc_padded_channels(C);
    uintptr_t p = (reinterpret_cast<uintptr_t>(split) + 255) & ~uintptr_t(255);
    __nv_bfloat16* Fs = reinterpret_cast<__nv_bfloat16*>(p);
    {
        const int64_t total = n * (Cp / 8);
        const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
        G2V_TIMED("feature_split_bf16_kernel", s,
                  feature_split_bf16_kernel<<<blocks, 256, 0, s>>>(features, n, C, Cp, Fs));
        G2V_LAUNCH_CHECK("feature_split_bf16_kernel");
    }
    CUtensorMap gmap;
    memset(&gmap, 0, sizeof(gmap));
    const int ldims[3] = {G.xlen, G.dims[1], G.dims[2]};
    // this CTA's half of a unit: 2 x 4 x 16 voxels x 32 channels
    const bool tma = encode_grid_rows_f32(&gmap, grad_feats, ldims, C, kKC, kUZ, kTile, 2, /*swizzle*/ 128);
    auto kern = tma ? spass_tc_kernel<true> : spass_tc_kernel<false>;
    G2V_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    int dev = 0, sms = 148;
    G2V_CUDA(cudaGetDevice(&dev));
    G2V_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    // one pair per unit at most; clusters of two (__cluster_dims__)
    const int grid = 2 * std::min(num_units, spass_pair_slots(reinterpret_cast<const void*>(kern), dev, sms));
    // e_v of the multi-pass units from grid_feats (when the caller passed it)
    const float* ev = nullptr;
    if (grid_feats != nullptr && ev_buf != nullptr) {
        const int vec = (C % 4 == 0) && (reinterpret_cast<uintptr_t>(grad_feats) % 16 == 0) &&
                        (reinterpret_cast<uintptr_t>(grid_feats) % 16 == 0);
        // 8 warps per block, as many blocks as are resident at once (__launch_bounds__(256, 4): four per
        // SM): the grid-stride walk covers every (unit, row quad) item
        const int64_t ev_blocks = std::min<int64_t>((int64_t)sms * 4, ((int64_t)num_units * (kUV / 4) + 7) / 8);
        G2V_TIMED("unit_ev_kernel", s,
                  unit_ev_kernel<<<(unsigned)ev_blocks, 256, 0, s>>>(unit_offsets, num_units, tzq_n, tile_x_begin, G,
                                                                     grad_feats, grid_feats, C, vec, ev_buf));
        G2V_LAUNCH_CHECK("unit_ev_kernel");
        ev = ev_buf;
    }
    G2V_TIMED("spass_tc_kernel", s,
              kern<<<(unsigned)grid, kThreads, kSmemBytes, s>>>(gmap, grad_density, grad_feats, Fs, C, Cp,
                                                                  density, gparams, g2t_offsets, unit_offsets,
                                                                  unit_lists, num_units, tile_x_begin, G, partial10,
                                                                  pair_cap, ev, err));
    G2V_LAUNCH_CHECK("spass_tc_kernel");
    return 0;
}

}  // namespace g2v
