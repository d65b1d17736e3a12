// g2v_fpass_cl.cu -- feature gradient of the backward on the tensor cores, one thread-block cluster per
// block of tiles.
//
// Same product as g2v_grad_tc.cu: for a block of tiles b and its Gaussians ("slots"),
//     dF[slot][c] = sum_{v in b} w_slot,v / max(D_v, 1e-6) * gF[v][c],
// as D^T in TMEM (M = channels, N = slots, K = 16 voxels of one x-slice per step), bf16 hi/lo split of both
// operands with hi*hi + hi*lo + lo*hi accumulated in fp32.  The difference is how the work is spread:
//   * a CTA covers 128 channels (one M-block), so its TMEM (512 columns) holds 512 slots: every block of
//     the usual workloads (up to ~360 Gaussians per 2x2x4-tile block) is done in one pass over its
//     gradient rows instead of two;
//   * the R CTAs of a cluster (R <= 8, consecutive 128-channel groups of the same block) share the
//     weights: CTA r evaluates the weights of its 1/R of the slots into its own B operand and copies them
//     into the same rows of its peers' B operands with shared::cta -> shared::cluster bulk copies
//     (completion counted on the peers' mbarriers).  A weight is therefore evaluated once per block and
//     voxel instead of once per channel group.
// Hand-offs per operand stage (all waits bounded, as everywhere in this library):
//   full_a   (local)  4 converter-warp arrivals: A (gF^T, 128 channels x 16 voxels) written;
//   full_w   (local)  8 weight-warp arrivals + one arrive.expect_tx per peer, whose bulk copies then
//                     complete the peers' weight rows;
//   empty    (local)  the MMA commit: this CTA's MMAs of the stage are done;
//   chunk    (local)  8 weight-warp arrivals: the CTA's own rows are written, the copy thread may send;
//   peer_free(local)  one arrival per cluster CTA (sent by each CTA's relay thread after its `empty`): the
//                     stage is free in every CTA, so the weight rows (local and copied) may be rewritten.
// Roles (512 threads): warps 0-3 convert A from the TMA-staged fp32 rows, warps 4-11 evaluate weights,
// warp 12 issues the MMAs, warp 13 the TMA loads, warp 14 the weight copies, warp 15 relays `empty`.
#include <cstddef>
#include <cstring>

#include "g2v.h"
#include "g2v_internal.cuh"
#include "g2v_tc.cuh"
#include "g2v_tmap.cuh"

namespace g2v {

namespace {
constexpr int kThreads = 512;
constexpr int kConvWarps = 4;
constexpr int kWWarp0 = 4, kWWarps = 8;
constexpr int kMmaWarp = 12, kTmaWarp = 13, kCopyWarp = 14, kRelayWarp = 15;
static_assert(kRelayWarp == kThreads / 32 - 1, "the relay thread is the last warp (the final role branch)");
constexpr int kSlots = 512;                     // slots per pass = TMEM columns
constexpr int kCG = 128;                        // channels per CTA
constexpr int kStages = 3;
constexpr int kAHalf = 4096;                    // 128 channels x 16 voxels x bf16
constexpr int kBHalf = kSlots * 32;             // 512 slots x 16 voxels x bf16
constexpr int kStageBytes = 2 * kAHalf + 2 * kBHalf;
constexpr uint32_t kTmemCols = 512;
constexpr int kGS = 4;                          // staging stages of the fp32 gradient
constexpr int kGBytes = 16 * kCG * 4;           // 8 KB: [ly][lz][128 channels]
constexpr int kMaxBlockTiles = 16;
constexpr int kMaxCluster = 8;

struct CMisc {
    uint64_t full_a[kStages];
    uint64_t full_w[kStages];
    uint64_t empty[kStages];
    uint64_t chunk[kStages];
    uint64_t peer_free[kStages];
    uint64_t mma_done;
    uint64_t gfull[kGS];
    uint64_t gempty[kGS];
    uint32_t tmem_base;
    int fail;
    alignas(16) GParams prm[kSlots];  // the CTA's own slots, from index 0
    int64_t rowoff[kSlots];
    alignas(16) float lrd[kMaxBlockTiles * kVoxPerTile];
    int4 org[kMaxBlockTiles];
};
constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + (size_t)kGS * kGBytes + sizeof(CMisc);
static_assert(kSmemBytes <= 227 * 1024, "fpass_cl_kernel shared memory");
static_assert(offsetof(CMisc, prm) % 16 == 0, "GParams records are read as float4");

// ---- cluster primitives ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the same shared::cta offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_peer(uint32_t saddr, uint32_t rank) {
    uint32_t d;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
    return d;
}
__device__ __forceinline__ void peer_arrive(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
__device__ __forceinline__ void peer_arrive_expect_tx(uint32_t cluster_bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(cluster_bar),
                 "r"(bytes)
                 : "memory");
}
// bulk copy of `bytes` (multiple of 16) from this CTA's shared memory to a peer's; completes on the
// peer's mbarrier (complete_tx)
__device__ __forceinline__ void copy_to_peer(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                                             uint32_t cluster_bar) {
    asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     dst_cluster),
                 "r"(src_cta), "r"(bytes), "r"(cluster_bar)
                 : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// mbar_wait with cluster-scope acquire (phases completed by arrivals of other CTAs)
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar_saddr, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(bar_saddr), "r"(parity), "r"(tc::kWaitHintNs)
        : "memory");
    return done != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err) {
    const uint32_t a = tc::smem_u32(bar);
    if (mbar_try_wait_cluster(a, parity)) return true;
    const uint64_t t0 = tc::global_ns();
    for (;;) {
        if (mbar_try_wait_cluster(a, parity)) return true;
        if (*reinterpret_cast<volatile int*>(err) != 0) return false;
        if (tc::global_ns() - t0 > tc::kWaitLimitNs) break;
    }
    atomicOr(err, tc::kErrWaitTimeout);
    return false;
}

template <bool kTma>
__global__ void __launch_bounds__(kThreads, 1) fpass_cl_kernel(
    const __grid_constant__ CUtensorMap gmap, const float* __restrict__ grad_feats, int C,
    const float* __restrict__ density, const GParams* __restrict__ gparams, const int32_t* __restrict__ block_offsets,
    const int32_t* __restrict__ block_lists, const int32_t* __restrict__ g2b_offsets, int bx_begin, int nby, int nbz,
    int BX, int BY, int BZ, int tx_begin, int tx_end, int ngroups, int R, int vec, Grid G,
    float* __restrict__ partialF, int64_t block_pair_cap, int* __restrict__ err) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* base = smem_raw;
    unsigned char* gstage = base + kStages * kStageBytes;
    CMisc& ms = *reinterpret_cast<CMisc*>(gstage + kGS * kGBytes);
    if ((tc::smem_u32(smem_raw) & 1023u) != 0) {  // the same for every CTA of the cluster
        if (threadIdx.x == 0) atomicOr(err, 2);
        return;
    }
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bl = blockIdx.x / ngroups, cg = blockIdx.x - bl * ngroups;
    const uint32_t rank = R > 1 ? cluster_rank() : 0;
    const int bxr = bl / (nby * nbz), rem = bl - bxr * nby * nbz;
    const int by = rem / nbz, bz = rem - (rem / nbz) * nbz;
    const int bx = bx_begin + bxr;
    // every CTA of a cluster belongs to the same block, so they take the same early exits
    const int s0 = block_offsets[bl], Kb = block_offsets[bl + 1] - s0;
    if (Kb == 0) return;
    const int c0 = cg * kCG;
    const int txa = max(bx * BX, tx_begin), txb = min(bx * BX + BX, min(tx_end, G.tiles[0]));
    const int tya = by * BY, tyb = min(tya + BY, G.tiles[1]);
    const int tza = bz * BZ, tzb = min(tza + BZ, G.tiles[2]);
    const int nty = tyb - tya, ntz = tzb - tza;
    const int ntiles = max(0, txb - txa) * nty * ntz;
    if (ntiles == 0) {  // no tile of this block in the slab: its partial rows are zero
        for (int sl = 0; sl < Kb; ++sl) {
            const int g = block_lists[s0 + sl];
            const GParams& gp = gparams[g];
            const int blx = (__float_as_int(gp.w[3].y) / kTile) / BX, bly = (__float_as_int(gp.w[3].z) / kTile) / BY;
            const int blz = (__float_as_int(gp.w[3].w) / kTile) / BZ;
            const int ey = (__float_as_int(gp.w[4].y) / kTile) / BY - bly + 1;
            const int ez = (__float_as_int(gp.w[4].z) / kTile) / BZ - blz + 1;
            const int64_t ro = (int64_t)g2b_offsets[g] + ((bx - blx) * ey + (by - bly)) * ez + (bz - blz);
            if (ro >= block_pair_cap) continue;
            for (int c = c0 + threadIdx.x; c < min(C, c0 + kCG); c += kThreads) partialF[ro * C + c] = 0.0f;
        }
        return;
    }
    const int nsteps = ntiles * 4;  // 4 x-slices of 16 voxels per tile
    if (ntiles > kMaxBlockTiles) {  // the host sizes blocks within the limit
        if (tid == 0) atomicOr(err, 4);
        return;
    }
    for (int i = tid; i < ntiles * kVoxPerTile; i += kThreads) {
        const int t = i >> 6;
        int lx, ly, lz;
        local_voxel(i & 63, lx, ly, lz);
        const int tzi = t % ntz, tyi = (t / ntz) % nty, txi = t / (ntz * nty);
        const int x = (txa + txi) * kTile + lx, y = (tya + tyi) * kTile + ly, z = (tza + tzi) * kTile + lz;
        float r = -INFINITY;
        if (x < G.dims[0] && y < G.dims[1] && z < G.dims[2]) r = -log2f(fmaxf(density[grid_row(G, x, y, z)], kEps));
        ms.lrd[i] = r;
    }
    for (int t = tid; t < ntiles; t += kThreads) {
        const int tzi = t % ntz, tyi = (t / ntz) % nty, txi = t / (ntz * nty);
        ms.org[t] = make_int4((txa + txi) * kTile, (tya + tyi) * kTile, (tza + tzi) * kTile, 0);
    }
    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            tc::mbar_init(&ms.full_a[i], kConvWarps);
            tc::mbar_init(&ms.full_w[i], kWWarps + (R - 1));
            tc::mbar_init(&ms.empty[i], 1);
            tc::mbar_init(&ms.chunk[i], kWWarps);
            tc::mbar_init(&ms.peer_free[i], R);
        }
        tc::mbar_init(&ms.mma_done, 1);
        for (int i = 0; i < kGS; ++i) {
            tc::mbar_init(&ms.gfull[i], 1);
            tc::mbar_init(&ms.gempty[i], kConvWarps);
        }
        tc::mbar_fence_init();
        ms.fail = 0;
    }
    if (warp == 0) tc::tmem_alloc(&ms.tmem_base, kTmemCols);
    tc::tc_fence_before();
    __syncthreads();
    if (R > 1) cluster_sync_all();  // every peer's barriers are initialised before any remote arrival
    tc::tc_fence_after();
    const uint32_t tmem = ms.tmem_base;
    bool ok = true;

    auto a_stage = [&](int st, int hl) -> unsigned char* { return base + st * kStageBytes + hl * kAHalf; };
    auto b_stage = [&](int st, int hl) -> unsigned char* {
        return base + st * kStageBytes + 2 * kAHalf + hl * kBHalf;
    };

    int it = 0;      // global step counter across passes (stage / parity bookkeeping)
    int issued = 0;  // TMA thread: staged steps issued
    const int npass = (Kb + kSlots - 1) / kSlots;
    for (int pass = 0; pass < npass; ++pass) {
        const int p0 = pass * kSlots, ns = min(kSlots, Kb - p0);
        const int nn = (ns + 15) & ~15;                     // MMA N of this pass (two MMAs above 256)
        const int cs = (((nn + R - 1) / R) + 15) & ~15;     // slots per cluster CTA
        const int t0 = min(nn, (int)rank * cs), t1 = min(nn, t0 + cs);
        for (int i = tid; i < (t1 - t0) * 5; i += kThreads) {
            const int sl = i / 5, wq = i - sl * 5;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t0 + sl < ns) v = gparams[block_lists[s0 + p0 + t0 + sl]].w[wq];
            ms.prm[sl].w[wq] = v;
        }
        for (int sl = tid; sl < kSlots; sl += kThreads) {
            int64_t ro = -1;
            if (sl < ns) {
                const int g = block_lists[s0 + p0 + sl];
                const GParams& gp = gparams[g];
                const int lbx = __float_as_int(gp.w[3].y), lby = __float_as_int(gp.w[3].z), lbz = __float_as_int(gp.w[3].w);
                const int uby = __float_as_int(gp.w[4].y), ubz = __float_as_int(gp.w[4].z);
                const int blx = (lbx / kTile) / BX, bly = (lby / kTile) / BY, blz = (lbz / kTile) / BZ;
                const int ey = (uby / kTile) / BY - bly + 1, ez = (ubz / kTile) / BZ - blz + 1;
                ro = (int64_t)g2b_offsets[g] + ((bx - blx) * ey + (by - bly)) * ez + (bz - blz);
                if (ro >= block_pair_cap) ro = -1;  // offsets come from the caller
            }
            ms.rowoff[sl] = ro;
        }
        __syncthreads();

        if (warp < kConvWarps) {
            // ---------------- converters: A = gF^T, thread = (8-channel chunk jc, voxel rows r, r + 8) ----------
            const int jc = tid & 15, rb = tid >> 4;  // rb 0..7
            const int a = jc >> 3, jj = jc & 7;
            for (int j = 0; j < nsteps && ok; ++j, ++it) {
                const int st = it % kStages, gs = it % kGS;
                const int4 o = ms.org[j >> 2];
                const int ks = j & 3;
                if (it >= kStages) ok = tc::mbar_wait(&ms.empty[st], ((it / kStages) + 1) & 1, err);
                if (kTma && ok) ok = tc::mbar_wait(&ms.gfull[gs], (it / kGS) & 1, err);
                if (!ok) break;
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const int r = rb + 8 * i;  // voxel row of the step: (ly, lz) = (r / 4, r % 4)
                    float f[8];
                    if (kTma) {
                        const float4* src = reinterpret_cast<const float4*>(gstage + gs * kGBytes + r * (kCG * 4) + jc * 32);
                        const float4 u = src[0], w4 = src[1];
                        f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w;
                        f[4] = w4.x; f[5] = w4.y; f[6] = w4.z; f[7] = w4.w;
                    } else {
                        const int x = o.x + ks, y = o.y + (r >> 2), z = o.z + (r & 3);
                        const bool vok = x < G.dims[0] && y < G.dims[1] && z < G.dims[2];
                        const int c = c0 + jc * 8;
                        const float* src = grad_feats + grid_row(G, x, y, z) * C + c;
                        if (vok && c + 7 < C && vec) {
                            const float4 u = *reinterpret_cast<const float4*>(src);
                            const float4 w4 = *reinterpret_cast<const float4*>(src + 4);
                            f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w;
                            f[4] = w4.x; f[5] = w4.y; f[6] = w4.z; f[7] = w4.w;
                        } else {
#pragma unroll
                            for (int e = 0; e < 8; ++e) f[e] = (vok && c + e < C) ? src[e] : 0.0f;
                        }
                    }
                    uint4 h, l;
                    tc::split_bf16x2(f[0], f[1], h.x, l.x);
                    tc::split_bf16x2(f[2], f[3], h.y, l.y);
                    tc::split_bf16x2(f[4], f[5], h.z, l.z);
                    tc::split_bf16x2(f[6], f[7], h.w, l.w);
                    const int g8 = r >> 3, rr = r & 7;
                    const int off = a * 1024 + g8 * 2048 + rr * 128 + ((jj ^ rr) << 4);
                    *reinterpret_cast<uint4*>(a_stage(st, 0) + off) = h;
                    *reinterpret_cast<uint4*>(a_stage(st, 1) + off) = l;
                }
                tc::fence_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tc::mbar_arrive(&ms.full_a[st]);
                    if (kTma) tc::mbar_arrive(&ms.gempty[gs]);
                }
            }
        } else if (warp < kWWarp0 + kWWarps) {
            // ---------------- weight warps: the CTA's own slots [t0, t1), 16 voxels each ----------------
            const int tw = tid - kWWarp0 * 32;
            for (int j = 0; j < nsteps && ok; ++j, ++it) {
                const int st = it % kStages;
                const int4 o = ms.org[j >> 2];
                const int ks = j & 3;
                // the stage must be free in every CTA of the cluster (its rows are copied there)
                if (it >= kStages) ok = mbar_wait_cluster(&ms.peer_free[st], ((it / kStages) + 1) & 1, err);
                if (!ok) break;
                const int x = o.x + ks;
#pragma unroll 1
                for (int t = t0 + tw; t < t1; t += kWWarps * 32) {
                    float w[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) w[e] = 0.0f;
                    const GParams& gp = ms.prm[t - t0];
                    const float4 a = gp.w[0], b = gp.w[1], c = gp.w[2], d = gp.w[3], e4 = gp.w[4];
                    const bool live = t < ns && x >= __float_as_int(d.y) && x <= __float_as_int(e4.x);
                    if (live) {
                        const float cx = voxel_centre(G, 0, x), cy0 = voxel_centre(G, 1, o.y), cz0 = voxel_centre(G, 2, o.z);
                        const float hy = G.h[1], hz = G.h[2];
                        const int ylo = __float_as_int(d.z) - o.y, yhi = __float_as_int(e4.y) - o.y;
                        const int zlo = __float_as_int(d.w) - o.z, zhi = __float_as_int(e4.z) - o.z;
                        const float dx = cx - a.x, dy = cy0 - a.y, dz = cz0 - a.z;
                        const float qx = b.x * dx + b.y * dy + b.z * dz;
                        const float qy = b.w * dx + c.x * dy + c.y * dz;
                        const float qz = c.z * dx + c.w * dy + d.x * dz;
                        const float pty = b.y * dx + c.x * dy + c.w * dz;  // (P^T d)_y
                        const float ptz = b.z * dx + c.y * dy + d.x * dz;  // (P^T d)_z
                        // base-2 exponent of voxel (ly, lz):
                        //   k (A + By ly + Qyy ly^2 + (Bz + Qyz ly) lz + Qzz lz^2) + log2(1 / den_v),  k = -log2(e) / 2
                        const float k = tc::kNegHalfLog2e;
                        const float A = k * (dx * qx + dy * qy + dz * qz);
                        const float By = k * hy * (qy + pty), Bz = k * hz * (qz + ptz);
                        const float Qyy = k * hy * hy * c.x, Qzz = k * hz * hz * d.x, Qyz = k * hy * hz * (c.y + c.w);
                        const float4* L4 = reinterpret_cast<const float4*>(&ms.lrd[(j >> 2) * kVoxPerTile + ks * 16]);
#pragma unroll
                        for (int ly = 0; ly < 4; ++ly) {
                            const float4 L = L4[ly];  // the 4 voxels (ly, 0..3); box mask: -inf outside
                            const float my = (ly >= ylo && ly <= yhi) ? 0.0f : -INFINITY;
                            const float Ay = fmaf(fmaf(Qyy, (float)ly, By), (float)ly, A) + my;
                            const float By2 = fmaf(Qyz, (float)ly, Bz);
                            const float Lz[4] = {L.x, L.y, L.z, L.w};
#pragma unroll
                            for (int lz = 0; lz < 4; ++lz) {
                                const float mz = (lz >= zlo && lz <= zhi) ? Lz[lz] : -INFINITY;
                                const float m = fmaf(fmaf(Qzz, (float)lz, By2), (float)lz, Ay) + mz;
                                w[ly * 4 + lz] = a.w * tc::exp2_approx(m);
                            }
                        }
                    }
                    uint4 h0, h1, l0, l1;
                    tc::split_bf16x2(w[0], w[1], h0.x, l0.x);
                    tc::split_bf16x2(w[2], w[3], h0.y, l0.y);
                    tc::split_bf16x2(w[4], w[5], h0.z, l0.z);
                    tc::split_bf16x2(w[6], w[7], h0.w, l0.w);
                    tc::split_bf16x2(w[8], w[9], h1.x, l1.x);
                    tc::split_bf16x2(w[10], w[11], h1.y, l1.y);
                    tc::split_bf16x2(w[12], w[13], h1.z, l1.z);
                    tc::split_bf16x2(w[14], w[15], h1.w, l1.w);
                    // K-major, 32-byte swizzle: row t = the slot's 16 voxels (32 bytes), chunk c at c ^ ((t / 4) % 2)
                    const int sw = (t >> 2) & 1;
                    const int off0 = (t >> 3) * 256 + (t & 7) * 32 + (sw << 4), off1 = off0 ^ 16;
                    *reinterpret_cast<uint4*>(b_stage(st, 0) + off0) = h0;
                    *reinterpret_cast<uint4*>(b_stage(st, 0) + off1) = h1;
                    *reinterpret_cast<uint4*>(b_stage(st, 1) + off0) = l0;
                    *reinterpret_cast<uint4*>(b_stage(st, 1) + off1) = l1;
                }
                tc::fence_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tc::mbar_arrive(&ms.full_w[st]);
                    tc::mbar_arrive(&ms.chunk[st]);
                }
            }
        } else if (warp == kMmaWarp) {
            if (lane == 0) {
                const int n0 = min(nn, 256), n1 = nn - n0;
                const uint32_t id0 = tc::idesc_bf16_f32(128, n0, /*A MN-major*/ 1, /*B K-major*/ 0);
                const uint32_t id1 = tc::idesc_bf16_f32(128, n1 > 0 ? n1 : 16, 1, 0);
                for (int j = 0; j < nsteps && ok; ++j, ++it) {
                    const int st = it % kStages;
                    const uint32_t par = (it / kStages) & 1;
                    ok = tc::mbar_wait(&ms.full_a[st], par, err) && tc::mbar_wait(&ms.full_w[st], par, err);
                    if (!ok) break;
                    tc::tc_fence_after();
                    const uint64_t ah = tc::smem_desc(tc::smem_u32(a_stage(st, 0)), 1024, 2048, tc::kLayoutSw128);
                    const uint64_t al = tc::smem_desc(tc::smem_u32(a_stage(st, 1)), 1024, 2048, tc::kLayoutSw128);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        if (h == 1 && n1 == 0) break;
                        const uint32_t boff = h * 256 * 32;  // rows 256.. of B (8 KB)
                        const uint64_t bh = tc::smem_desc(tc::smem_u32(b_stage(st, 0)) + boff, 16, 256, tc::kLayoutSw32);
                        const uint64_t blo = tc::smem_desc(tc::smem_u32(b_stage(st, 1)) + boff, 16, 256, tc::kLayoutSw32);
                        const uint32_t dcol = tmem + h * 256;
                        const uint32_t id = h == 0 ? id0 : id1;
                        tc::mma_f16_ss(dcol, ah, bh, id, j > 0);
                        tc::mma_f16_ss(dcol, ah, blo, id, true);
                        tc::mma_f16_ss(dcol, al, bh, id, true);
                    }
                    tc::mma_commit(tc::smem_u32(&ms.empty[st]));
                }
                tc::mma_commit(tc::smem_u32(&ms.mma_done));
            } else {
                it += nsteps;
            }
        } else if (warp == kTmaWarp) {
            if (kTma && lane == 0) {
                for (int j = 0; j < nsteps && ok; ++j, ++it) {
                    const int gs = it % kGS;
                    const int4 o = ms.org[j >> 2];
                    if (it >= kGS) ok = tc::mbar_wait(&ms.gempty[gs], ((it / kGS) + 1) & 1, err);
                    if (!ok) break;
                    tc::mbar_arrive_expect_tx(&ms.gfull[gs], kGBytes);
                    tc::tma_load_4d(tc::smem_u32(gstage + gs * kGBytes), &gmap, c0, o.z, o.y, o.x + (j & 3) - G.xoff,
                                    &ms.gfull[gs]);
                    issued = it + 1;
                }
            } else {
                it += nsteps;
            }
        } else if (warp == kCopyWarp) {
            // ---------------- copy thread: the CTA's weight rows into every peer's B operand ----------------
            if (R > 1 && lane == 0) {
                const uint32_t bytes = (uint32_t)(t1 - t0) * 32;  // per half (hi or lo)
                for (int j = 0; j < nsteps && ok; ++j, ++it) {
                    const int st = it % kStages;
                    ok = tc::mbar_wait(&ms.chunk[st], (it / kStages) & 1, err);
                    if (!ok) break;
                    const uint32_t src_h = tc::smem_u32(b_stage(st, 0)) + t0 * 32;
                    const uint32_t src_l = tc::smem_u32(b_stage(st, 1)) + t0 * 32;
                    const uint32_t bar = tc::smem_u32(&ms.full_w[st]);
                    for (int q = 0; q < R; ++q) {
                        if (q == (int)rank) continue;
                        const uint32_t pbar = map_peer(bar, q);
                        if (bytes == 0) {
                            peer_arrive(pbar);
                            continue;
                        }
                        peer_arrive_expect_tx(pbar, 2 * bytes);
                        copy_to_peer(map_peer(src_h, q), src_h, bytes, pbar);
                        copy_to_peer(map_peer(src_l, q), src_l, bytes, pbar);
                    }
                }
            } else {
                it += nsteps;
            }
        } else {
            // ---------------- relay thread: "stage free here" to every CTA of the cluster ----------------
            if (lane == 0) {
                const uint32_t pf = tc::smem_u32(&ms.peer_free[0]);
                for (int j = 0; j < nsteps && ok; ++j, ++it) {
                    const int st = it % kStages;
                    ok = tc::mbar_wait(&ms.empty[st], (it / kStages) & 1, err);
                    if (!ok) break;
                    const uint32_t bar = pf + st * (uint32_t)sizeof(uint64_t);
                    if (R == 1) {
                        tc::mbar_arrive(&ms.peer_free[st]);
                    } else {
                        for (int q = 0; q < R; ++q) peer_arrive(map_peer(bar, q));
                    }
                }
            } else {
                it += nsteps;
            }
        }

        ok = tc::mbar_wait_drain(&ms.mma_done, pass & 1, err) && ok;
        if (!ok) ms.fail = 1;
        tc::tc_fence_before();
        __syncthreads();
        tc::tc_fence_after();
        // epilogue: warp w < 8 reads TMEM lanes 32*(w%4).. (channels), slot columns [256 (w/4), +256)
        if (warp < 8 && !ms.fail) {
            const int q = warp & 3, h = warp >> 2;
            const int c = c0 + q * 32 + lane;
            for (int jc = h * 16; jc < h * 16 + 16; ++jc) {
                if (jc * 16 >= ns) break;  // warp-uniform
                float vals[16];
                tc::tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + jc * 16, vals);
                if (c < C) {
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const int64_t ro = ms.rowoff[jc * 16 + e];
                        if (ro >= 0) partialF[ro * C + c] = vals[e];
                    }
                }
            }
        }
        tc::tc_fence_before();
        __syncthreads();
        tc::tc_fence_after();
    }
    // no copy may still be in flight when the CTA's shared memory is released (matters after a wait gave up)
    if (kTma && warp == kTmaWarp && lane == 0)
        for (int k = max(0, issued - kGS); k < issued; ++k) tc::mbar_wait_drain(&ms.gfull[k % kGS], (k / kGS) & 1, err);
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, kTmemCols);
    // peers copy into this CTA's shared memory and arrive on its barriers: leave together
    if (R > 1) cluster_sync_all();
}

// Largest divisor of n that is at most kMaxCluster.
int cluster_size_for(int n) {
    for (int r = kMaxCluster; r > 1; --r)
        if (n % r == 0) return r;
    return 1;
}
}  // namespace

int launch_fpass_cl(const float* grad_feats, int C, const float* density, const GParams* gparams,
                    const int32_t* block_offsets, const int32_t* block_lists, const int32_t* g2b_offsets, int bx_begin,
                    int nbx, int nby, int nbz, const int B[3], int tx_begin, int tx_end, const Grid& G, float* partialF,
                    int64_t block_pair_cap, int* err, cudaStream_t s) {
    const int64_t nblocks = (int64_t)nbx * nby * nbz;
    if (nblocks <= 0 || C <= 0) return 0;
    const int ngroups = (C + kCG - 1) / kCG;
    int R = cluster_size_for(ngroups);
    const int vec = (C % 4 == 0) && (reinterpret_cast<uintptr_t>(grad_feats) % 16 == 0);
    if (B[0] * B[1] * B[2] > kMaxBlockTiles) {
        set_error("fpass_cl: block of %dx%dx%d tiles exceeds %d", B[0], B[1], B[2], kMaxBlockTiles);
        return G2V_ERROR_INVALID_VALUE;
    }
    CUtensorMap gmap;
    memset(&gmap, 0, sizeof(gmap));
    const int ldims[3] = {G.xlen, G.dims[1], G.dims[2]};
    const bool tma = encode_grid_rows_f32(&gmap, grad_feats, ldims, C, kCG, kTile, kTile, 1);
    auto kern = tma ? fpass_cl_kernel<true> : fpass_cl_kernel<false>;
    G2V_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    const int64_t grid = nblocks * ngroups;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    // the largest cluster size dividing the channel groups that the GPU can co-schedule
    for (; R > 1; --R) {
        if (ngroups % R != 0) continue;
        attr[0].val.clusterDim.x = (unsigned)R;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int nclusters = 0;
        if (cudaOccupancyMaxActiveClusters(&nclusters, kern, &cfg) == cudaSuccess && nclusters > 0) break;
        cudaGetLastError();
    }
    if (R < 1) R = 1;
    attr[0].val.clusterDim.x = (unsigned)R;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    G2V_TIMED("fpass_tc_kernel", s,
              G2V_CUDA(cudaLaunchKernelEx(&cfg, kern, gmap, grad_feats, C, density, gparams, block_offsets,
                                          block_lists, g2b_offsets, bx_begin, nby, nbz, B[0], B[1], B[2], tx_begin,
                                          tx_end, ngroups, R, vec, G, partialF, block_pair_cap, err)));
    G2V_LAUNCH_CHECK("fpass_tc_kernel");
    return 0;
}

}  // namespace g2v
