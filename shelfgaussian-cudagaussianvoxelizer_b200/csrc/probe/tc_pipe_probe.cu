// tc_pipe_probe.cu -- pipeline probe: the MMA thread consumes a ring of R stages (wait full -> fence -> S
// MMAs -> commit empty) while 4 producer warps refill it (wait empty -> optional shared-memory stores ->
// fence -> arrive full).  Reports cycles per step of the MMA thread.  Bounded waits throughout.
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>
#include "g2v_tc.cuh"
using namespace g2v;

constexpr int kMaxR = 8;
template <int N, int S, int R, int STORE_KB>
__global__ void __launch_bounds__(160, 1) pipe(int steps, unsigned long long* out, int* err) {
    extern __shared__ __align__(1024) unsigned char sm[];
    __shared__ uint64_t full[kMaxR], empty[kMaxR], done;
    __shared__ uint32_t tbase;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < 64 * 1024 / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(sm)[i] = 0;
    if (tid == 0) {
        for (int i = 0; i < R; ++i) { tc::mbar_init(&full[i], 4); tc::mbar_init(&empty[i], 1); }
        tc::mbar_init(&done, 1);
        tc::mbar_fence_init();
    }
    if (warp == 0) tc::tmem_alloc(&tbase, 512);
    tc::fence_async_smem();
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = tbase;
    bool ok = true;
    if (warp < 4) {
        // producers: 4 warps, each stores STORE_KB/4 KB per step into a scratch area (64 KB .. 128 KB)
        unsigned char* scratch = sm + 65536;
        for (int it = 0; it < steps && ok; ++it) {
            const int st = it % R;
            if (it >= R) ok = tc::mbar_wait(&empty[st], ((it / R) + 1) & 1, err);
            if (!ok) break;
            if (STORE_KB > 0) {
                const int per_thread = STORE_KB * 1024 / 128 / 16;  // 16-byte stores per thread
                uint4 v = make_uint4(it, tid, 0, 0);
#pragma unroll 4
                for (int q = 0; q < per_thread; ++q)
                    *reinterpret_cast<uint4*>(scratch + ((q * 128 + tid) * 16) % 65536) = v;
            }
            tc::fence_async_smem();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&full[st]);
        }
    } else if (tid == 128) {
        const uint32_t a = tc::smem_u32(sm), b = tc::smem_u32(sm + 32768);
        const uint64_t ad = tc::smem_desc(a, 1024, 2048, tc::kLayoutSw128), bd = tc::smem_desc(b, 1024, 2048, tc::kLayoutSw128);
        const uint32_t idesc = tc::idesc_bf16_f32(128, N, 1, 1);
        const long long t0 = clock64();
        for (int it = 0; it < steps && ok; ++it) {
            const int st = it % R;
            ok = tc::mbar_wait(&full[st], (it / R) & 1, err);
            if (!ok) break;
            tc::tc_fence_after();
#pragma unroll
            for (int s = 0; s < S; ++s) tc::mma_f16_ss(tmem + (uint32_t)((s & 1) * N), ad, bd, idesc, it > 0 || s > 1);
            tc::mma_commit(tc::smem_u32(&empty[st]));
        }
        tc::mma_commit(tc::smem_u32(&done));
        tc::mbar_wait_drain(&done, 0, err);
        atomicAdd(out, (unsigned long long)(clock64() - t0));
        atomicAdd(out + 1, 1ull);
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (warp == 0) tc::tmem_dealloc(tmem, 512);
}

template <int N, int S, int R, int STORE_KB>
void run(const char* name, int sms) {
    unsigned long long* out; int* err;
    cudaMalloc(&out, 16); cudaMalloc(&err, 4);
    cudaMemset(out, 0, 16); cudaMemset(err, 0, 4);
    auto k = pipe<N, S, R, STORE_KB>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 131072);
    const int steps = 4000;
    k<<<sms, 160, 131072>>>(100, out, err);
    cudaDeviceSynchronize();
    cudaMemset(out, 0, 16);
    k<<<sms, 160, 131072>>>(steps, out, err);
    cudaError_t ce = cudaDeviceSynchronize();
    unsigned long long h[2]; int herr; cudaMemcpy(h, out, 16, cudaMemcpyDeviceToHost); cudaMemcpy(&herr, err, 4, cudaMemcpyDeviceToHost);
    const double cyc = (double)h[0] / (double)(h[1] ? h[1] : 1) / steps;
    const double ideal = (double)S * 128 * N * 16 / 4096.0;
    printf("%-52s cycles/step %7.1f  (MMA ideal %5.0f, %3.0f%%)  %s err %d\n", name, cyc, ideal, 100.0 * ideal / cyc,
           cudaGetErrorString(ce), herr);
    cudaFree(out); cudaFree(err);
}

int main() {
    int sms = 0; cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    run<128, 6, 4, 0>("N128 S6 R4, no producer stores", sms);
    run<128, 6, 7, 0>("N128 S6 R7, no producer stores", sms);
    run<128, 12, 4, 0>("N128 S12 R4, no producer stores", sms);
    run<256, 6, 4, 0>("N256 S6 R4, no producer stores", sms);
    run<128, 6, 7, 16>("N128 S6 R7, producers store 16 KB/step", sms);
    run<128, 6, 7, 32>("N128 S6 R7, producers store 32 KB/step", sms);
    run<128, 12, 4, 48>("N128 S12 R4, producers store 48 KB/step", sms);
    run<128, 12, 4, 80>("N128 S12 R4, producers store 80 KB/step", sms);
    run<256, 6, 4, 32>("N256 S6 R4, producers store 32 KB/step", sms);
    run<256, 6, 4, 64>("N256 S6 R4, producers store 64 KB/step", sms);
    return 0;
}
