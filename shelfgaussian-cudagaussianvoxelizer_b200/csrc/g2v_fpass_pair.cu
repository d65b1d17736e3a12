// g2v_fpass_pair.cu -- feature gradient of the backward on CTA pairs (tcgen05 cta_group::2, kind::f16, bf16).
//
// Same contraction as fpass_tc_kernel (g2v_grad_tc.cu): for a block of tiles b and its Gaussians (slots),
//     dF[slot][c] = sum_{v in b} w_slot,v / max(D_v, 1e-6) * gF[v][c],
// computed as D^T in TMEM with K = 16 voxels per step, both operands split into bf16 pairs
// (hi*hi + hi*lo + lo*hi, fp32 accumulation).  A cluster of two CTAs shares each MMA (M = 256):
//   * CTA r of the pair holds 128 of the job's 256 channels: its A operand (gF^T, 128 channels x 16
//     voxels) is converted from its own 128-channel slice of the gradient rows, and the accumulator rows
//     of those channels live in its own TMEM (128 lanes x up to 512 slot columns);
//   * the slots of a pass (up to 512) form two MMA column ranges of up to 256 (N); each CTA evaluates the
//     weights of half of each range (B rows), so a pair evaluates every weight of the block once per
//     256-channel group, like one single-CTA job, but covers 512 slots in one pass: blocks of 257-512
//     Gaussians no longer stream and convert their gradient rows a second time.
// The leader (rank 0) issues the MMAs after both CTAs' producers arrived on its stage barriers (remote
// arrives through shared::cluster addresses, release/acquire at cluster scope); its commits arrive on
// the stage-free and accumulator-ready barriers of both CTAs (one tcgen05.commit for both).  The gradient
// rows are loaded by each CTA into its own staging ring (a plain per-CTA tiled load).  Every wait is bounded; the
// pair always reaches its closing cluster barrier, also after a wait gave up.
#include <cstddef>

#include <cstring>

#include "g2v.h"
#include "g2v_internal.cuh"
#include "g2v_tc.cuh"
#include "g2v_tmap.cuh"

namespace g2v {

namespace {
constexpr int kThreads = 576;
constexpr int kPassSlots = 512;                  // slots of a pass (two MMA column ranges of 256)
constexpr int kHalfRows = 128;                   // B rows of one range held by one CTA
constexpr int kCh = 128;                         // channels per CTA (A rows)
constexpr int kCG = 2 * kCh;                     // channels per pair
constexpr int kStages = 4;
constexpr int kAHalf = 4096;                     // 128 channels x 16 voxels, bf16, one half (hi or lo)
constexpr int kBRange = kHalfRows * 16 * 2;      // one range's rows of this CTA, one half
constexpr int kBHalf = 2 * kBRange;              // both ranges, one half
constexpr int kStageBytes = 2 * kAHalf + 2 * kBHalf;
constexpr uint32_t kTmemCols = 512;
// Staging stages of the fp32 gradient: a CTA streams only 8 KB per step, so the ring is deep enough to
// keep ~96 KB of loads in flight per SM (HBM latency x the per-SM share of the bandwidth).
constexpr int kGS = 12;
constexpr int kGBytes = 16 * kCh * 4;            // 8 KB: [ly][lz][128 channels]
constexpr int kMaxBlockTiles = 16;
constexpr int kWeightThreads = 256;              // 2 ranges x 128 rows

struct PMisc {
    uint64_t full_a[kStages];  // leader: converted A of both CTAs (8 + 8 warp arrivals)
    uint64_t full_w[kStages];  // leader: weights of both CTAs (8 + 8 warp arrivals)
    uint64_t empty[kStages];   // both: the pair's MMAs reading the stage completed (leader's commit)
    uint64_t mma_done;         // both: the pass's accumulators are complete
    uint32_t tmem_base;
    int fail;
    uint64_t gfull[kGS];   // TMA bytes of a staged step
    uint64_t gempty[kGS];  // 8 converter-warp arrivals
    alignas(16) GParams prm[kWeightThreads];
    int64_t rowoff[kPassSlots];
    alignas(16) float lrd[kMaxBlockTiles * kVoxPerTile];  // log2(1 / max(D, eps)), -inf outside the grid
    int4 org[kMaxBlockTiles];
};
constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + (size_t)kGS * kGBytes + sizeof(PMisc);
static_assert(kSmemBytes <= 227 * 1024, "fpass_pair_kernel shared memory");
static_assert(offsetof(PMisc, prm) % 16 == 0 && offsetof(PMisc, lrd) % 16 == 0, "vector-accessed fields");

// N of MMA column range j of a pass with ns slots: the range's slot count rounded up to 16.
__device__ __forceinline__ int range_n(int ns, int j) {
    const int k = min(256, max(0, ns - 256 * j));
    return (k + 15) & ~15;
}

template <bool kTma>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1) fpass_pair_kernel(
    const __grid_constant__ CUtensorMap gmap, const float* __restrict__ grad_feats, int C,
    const float* __restrict__ density, const GParams* __restrict__ gparams, const int32_t* __restrict__ block_offsets,
    const int32_t* __restrict__ block_lists, const int32_t* __restrict__ g2b_offsets, int bx_begin, int nby, int nbz,
    int BX, int BY, int BZ, int tx_begin, int tx_end, int ngroups, int vec, Grid G, float* __restrict__ partialF,
    int64_t block_pair_cap, int* __restrict__ err) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* base = smem_raw;
    unsigned char* gstage = base + kStages * kStageBytes;
    PMisc& ms = *reinterpret_cast<PMisc*>(gstage + kGS * kGBytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = tc::cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1;
    const int bl = pair / ngroups, cg = pair - bl * ngroups;
    const int bxr = bl / (nby * nbz), rem = bl - bxr * nby * nbz;
    const int by = rem / nbz, bz = rem - (rem / nbz) * nbz;
    const int bx = bx_begin + bxr;
    const int s0 = block_offsets[bl], Kb = block_offsets[bl + 1] - s0;
    // Both CTAs of a pair take the same early exits (they depend on the block only), before any
    // cluster-level operation.
    if (Kb == 0) return;
    const int c0 = cg * kCG + (int)rank * kCh;  // this CTA's channels
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
            for (int c = c0 + threadIdx.x; c < min(C, c0 + kCh); c += kThreads) partialF[ro * C + c] = 0.0f;
        }
        return;
    }
    if (ntiles > kMaxBlockTiles) {  // the host sizes blocks within the limit
        if (tid == 0) atomicOr(err, 4);
        return;
    }
    if ((tc::smem_u32(smem_raw) & 1023u) != 0) {  // same offset in both CTAs: both leave here
        if (tid == 0) atomicOr(err, 2);
        return;
    }
    const int nsteps = ntiles * 4;  // 4 x-slices of 16 voxels per tile
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
            tc::mbar_init(&ms.full_a[i], 16);
            tc::mbar_init(&ms.full_w[i], 16);
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
    if (warp == 0) tc::tmem_alloc_pair(&ms.tmem_base, kTmemCols);
    tc::tc_fence_before();
    tc::cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
    tc::tc_fence_after();
    const uint32_t tmem = ms.tmem_base;
    bool ok = true;

    auto a_stage = [&](int st, int hl) -> unsigned char* { return base + st * kStageBytes + hl * kAHalf; };
    auto b_stage = [&](int st, int hl) -> unsigned char* {
        return base + st * kStageBytes + 2 * kAHalf + hl * kBHalf;
    };
    // the leader's copy of a stage barrier, as a shared::cluster address
    auto leader_bar = [&](uint64_t* bar) -> uint32_t { return tc::mapa_shared(tc::smem_u32(bar), 0); };

    int it = 0;      // global step counter across passes (stage / parity bookkeeping)
    int issued = 0;  // TMA thread: staged steps issued
    const int npass = (Kb + kPassSlots - 1) / kPassSlots;
    for (int pass = 0; pass < npass; ++pass) {
        const int p0 = pass * kPassSlots, ns = min(kPassSlots, Kb - p0);
        const int n0 = range_n(ns, 0), n1 = range_n(ns, 1);
        // This CTA's B rows: h0 = n0 / 2 rows of range 0, then h1 = n1 / 2 rows of range 1.  The list is
        // dealt to the 8 weight warps in runs of rpw rows (a multiple of 8, so that a warp's 16-byte
        // stores stay conflict-free): row q = w * rpw + lane for weight warp w, so every warp has work
        // whatever the number of rows.
        const int h0 = n0 >> 1, h1 = n1 >> 1;
        const int rpw = (((h0 + h1 + 7) >> 3) + 7) & ~7;
        auto wrow = [&](int t) { return (t & 31) < rpw ? (t >> 5) * rpw + (t & 31) : 1 << 20; };
        for (int i = tid; i < kWeightThreads * 5; i += kThreads) {
            const int t = i / 5, wq = i - t * 5;
            const int q = wrow(t);
            const int j = q >= h0, lr = j ? q - h0 : q, hj = j ? h1 : h0;
            const int sl = 256 * j + (int)rank * hj + lr;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (q < h0 + h1 && sl < ns) v = gparams[block_lists[s0 + p0 + sl]].w[wq];
            ms.prm[t].w[wq] = v;
        }
        for (int sl = tid; sl < kPassSlots; sl += kThreads) {
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

        if (warp < 8) {
            // ------------- converters: A = gF^T, thread = (8-channel chunk jc, voxel row r) -------------
            const int jc = lane & 15, r = warp * 2 + (lane >> 4);  // (ly, lz) = (r / 4, r % 4)
            const int a = jc >> 3, jj = jc & 7;
            const int g8 = r >> 3, rr = r & 7;
            const int off = a * 1024 + g8 * 2048 + rr * 128 + ((jj ^ rr) << 4);
            for (int j = 0; j < nsteps && ok; ++j, ++it) {
                const int st = it % kStages, gs = it % kGS;
                if (it >= kStages) ok = tc::mbar_wait(&ms.empty[st], ((it / kStages) + 1) & 1, err);
                if (kTma && ok) ok = tc::mbar_wait(&ms.gfull[gs], (it / kGS) & 1, err);
                if (!ok) break;
                float f[8];
                if (kTma) {
                    const float4* src = reinterpret_cast<const float4*>(gstage + gs * kGBytes + r * (kCh * 4) + jc * 32);
                    const float4 u = src[0], w4 = src[1];
                    f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w;
                    f[4] = w4.x; f[5] = w4.y; f[6] = w4.z; f[7] = w4.w;
                } else {
                    const int4 o = ms.org[j >> 2];
                    const int x = o.x + (j & 3), y = o.y + (r >> 2), z = o.z + (r & 3);
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
                *reinterpret_cast<uint4*>(a_stage(st, 0) + off) = h;
                *reinterpret_cast<uint4*>(a_stage(st, 1) + off) = l;
                tc::fence_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tc::mbar_arrive_cluster(leader_bar(&ms.full_a[st]));
                    if (kTma) tc::mbar_arrive(&ms.gempty[gs]);
                }
            }
        } else if (warp < 16) {
            // ------------- weight warps: thread = one B row (slot) of a range, 16 voxels of the step -------------
            const int t = tid - 256;
            const int q = wrow(t);  // this thread's row of the CTA's list (see above)
            const int jr = q >= h0, lr = jr ? q - h0 : q, hj = jr ? h1 : h0;
            const int sl = 256 * jr + (int)rank * hj + lr;  // slot within the pass
            const bool row = q < h0 + h1;                   // rows >= N/2 of a range are not read by the MMAs
            const bool slot_live = row && sl < ns;
            const int sw = (lr >> 2) & 1;
            const int off0 = jr * kBRange + (lr >> 3) * 256 + (lr & 7) * 32 + (sw << 4), off1 = off0 ^ 16;
            for (int j = 0; j < nsteps && ok; ++j, ++it) {
                const int st = it % kStages;
                if (it >= kStages) ok = tc::mbar_wait(&ms.empty[st], ((it / kStages) + 1) & 1, err);
                if (!ok) break;
                if (row) {
                    const int4 o = ms.org[j >> 2];
                    const int ks = j & 3;
                    const int x0 = o.x, y0 = o.y, z0 = o.z;
                    float w[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) w[e] = 0.0f;
                    const GParams& gp = ms.prm[t];
                    const float4 a = gp.w[0], b = gp.w[1], c = gp.w[2], d = gp.w[3], e4 = gp.w[4];
                    const int x = x0 + ks;
                    const bool live = slot_live && x >= __float_as_int(d.y) && x <= __float_as_int(e4.x);
                    if (live) {
                        const float cx = voxel_centre(G, 0, x), cy0 = voxel_centre(G, 1, y0), cz0 = voxel_centre(G, 2, z0);
                        const float hy = G.h[1], hz = G.h[2];
                        const int ylo = __float_as_int(d.z) - y0, yhi = __float_as_int(e4.y) - y0;
                        const int zlo = __float_as_int(d.w) - z0, zhi = __float_as_int(e4.z) - z0;
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
                    // K-major, 32-byte swizzle: row lr = the slot's 16 voxels (32 bytes), chunk c at c ^ ((lr / 4) % 2)
                    *reinterpret_cast<uint4*>(b_stage(st, 0) + off0) = h0;
                    *reinterpret_cast<uint4*>(b_stage(st, 0) + off1) = h1;
                    *reinterpret_cast<uint4*>(b_stage(st, 1) + off0) = l0;
                    *reinterpret_cast<uint4*>(b_stage(st, 1) + off1) = l1;
                }
                tc::fence_async_smem();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive_cluster(leader_bar(&ms.full_w[st]));
            }
        } else if (kTma && warp == 17 && lane == 0) {
            // ------------- TMA thread: this CTA's 128-channel slice of the step's gradient rows -------------
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
        } else if (warp == 16 && lane == 0 && leader) {
            // ------------- MMA thread of the pair (leader CTA) -------------
            const uint32_t idesc0 = tc::idesc_bf16_f32(256, n0 > 0 ? n0 : 16, /*A MN-major*/ 1, /*B K-major*/ 0);
            const uint32_t idesc1 = tc::idesc_bf16_f32(256, n1 > 0 ? n1 : 16, 1, 0);
            for (int j = 0; j < nsteps && ok; ++j, ++it) {
                const int st = it % kStages;
                const uint32_t par = (it / kStages) & 1;
                ok = tc::mbar_wait(&ms.full_a[st], par, err) && tc::mbar_wait(&ms.full_w[st], par, err);
                if (!ok) break;
                tc::tc_fence_after();
                const uint64_t ah = tc::smem_desc(tc::smem_u32(a_stage(st, 0)), 1024, 2048, tc::kLayoutSw128);
                const uint64_t al = tc::smem_desc(tc::smem_u32(a_stage(st, 1)), 1024, 2048, tc::kLayoutSw128);
#pragma unroll
                for (int jr = 0; jr < 2; ++jr) {
                    if ((jr ? n1 : n0) == 0) continue;
                    const uint32_t id = jr ? idesc1 : idesc0;
                    const uint64_t bh =
                        tc::smem_desc(tc::smem_u32(b_stage(st, 0)) + jr * kBRange, 16, 256, tc::kLayoutSw32);
                    const uint64_t blo =
                        tc::smem_desc(tc::smem_u32(b_stage(st, 1)) + jr * kBRange, 16, 256, tc::kLayoutSw32);
                    const uint32_t dcol = tmem + jr * 256;
                    tc::mma_f16_ss_pair(dcol, ah, bh, id, j > 0);
                    tc::mma_f16_ss_pair(dcol, ah, blo, id, true);
                    tc::mma_f16_ss_pair(dcol, al, bh, id, true);
                }
                tc::mma_commit_pair(tc::smem_u32(&ms.empty[st]), (uint16_t)3);
            }
            tc::mma_commit_pair(tc::smem_u32(&ms.mma_done), (uint16_t)3);
        } else {
            it += nsteps;
        }

        ok = tc::mbar_wait_drain(&ms.mma_done, pass & 1, err) && ok;
        if (!ok) ms.fail = 1;
        tc::tc_fence_before();
        __syncthreads();
        tc::tc_fence_after();
        // epilogue: warp w < 8 reads lanes 32*(w%4).. (this CTA's channels) of column range w/4
        if (warp < 8 && !ms.fail) {
            const int q = warp & 3, jr = warp >> 2;
            const int c = c0 + q * 32 + lane;
            const int nsr = min(256, max(0, ns - 256 * jr));  // valid slots of the range
            for (int jc = 0; jc < 16; ++jc) {
                if (jc * 16 >= nsr) break;  // warp-uniform
                float vals[16];
                tc::tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + jr * 256 + jc * 16, vals);
                if (c < C && c < c0 + kCh) {
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const int64_t ro = ms.rowoff[256 * jr + jc * 16 + e];
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
    if (kTma && warp == 17 && lane == 0)
        for (int k = max(0, issued - kGS); k < issued; ++k) tc::mbar_wait_drain(&ms.gfull[k % kGS], (k / kGS) & 1, err);
    tc::tc_fence_before();
    tc::cluster_sync();  // neither CTA frees TMEM or leaves while the pair still works on it
    tc::tc_fence_after();
    if (warp == 0) tc::tmem_dealloc_pair(tmem, kTmemCols);
}
}  // namespace

// Feature-gradient pass on CTA pairs: grid = 2 x blocks x 256-channel groups, clusters of 2.
int launch_fpass_tc_pair(const float* grad_feats, int C, const float* density, const GParams* gparams,
                         const int32_t* block_offsets, const int32_t* block_lists, const int32_t* g2b_offsets,
                         int bx_begin, int nbx, int nby, int nbz, const int B[3], int tx_begin, int tx_end,
                         const Grid& G, float* partialF, int64_t block_pair_cap, int* err, cudaStream_t s) {
    const int64_t nblocks = (int64_t)nbx * nby * nbz;
    if (nblocks <= 0 || C <= 0) return 0;
    const int ngroups = (C + kCG - 1) / kCG;
    const int vec = (C % 4 == 0) && (reinterpret_cast<uintptr_t>(grad_feats) % 16 == 0);
    if (B[0] * B[1] * B[2] > kMaxBlockTiles) {
        set_error("fpass_pair: block of %dx%dx%d tiles exceeds %d", B[0], B[1], B[2], kMaxBlockTiles);
        return G2V_ERROR_INVALID_VALUE;
    }
    CUtensorMap gmap;
    memset(&gmap, 0, sizeof(gmap));
    const int ldims[3] = {G.xlen, G.dims[1], G.dims[2]};
    const bool tma = encode_grid_rows_f32(&gmap, grad_feats, ldims, C, kCh, kTile, kTile, 1);
    auto kern = tma ? fpass_pair_kernel<true> : fpass_pair_kernel<false>;
    G2V_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    const int64_t grid = 2 * nblocks * ngroups;
    if (grid > INT32_MAX) {
        set_error("fpass_pair: %lld CTAs", (long long)grid);
        return G2V_ERROR_INVALID_VALUE;
    }
    G2V_TIMED("fpass_tc_kernel", s,
              kern<<<(unsigned)grid, kThreads, kSmemBytes, s>>>(
                  gmap, grad_feats, C, density, gparams, block_offsets, block_lists, g2b_offsets, bx_begin, nby, nbz,
                  B[0], B[1], B[2], tx_begin, tx_end, ngroups, vec, G, partialF, block_pair_cap, err));
    G2V_LAUNCH_CHECK("fpass_pair_kernel");
    return 0;
}

}  // namespace g2v
