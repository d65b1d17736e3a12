// tc_rate_probe.cu -- tensor-pipe rate probe: one CTA per SM issues back-to-back tcgen05.mma (kind::f16,
// bf16) on zeroed shared memory for a fixed count, then one commit; reports cycles per MMA per SM.
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>
#include "g2v_tc.cuh"
using namespace g2v;

template <int M, int N, int AMN, int BMN, int LAYA, int LAYB, int PAIR, int NACC>
__global__ void __launch_bounds__(128, 1) probe(int iters, unsigned long long* out, int* err) {
    extern __shared__ __align__(1024) unsigned char sm[];
    __shared__ uint64_t bar;
    __shared__ uint32_t tbase;
    const int tid = threadIdx.x;
    for (int i = tid; i < 64 * 1024 / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(sm)[i] = 0;
    if (tid == 0) { tc::mbar_init(&bar, 1); tc::mbar_fence_init(); }
    if (tid < 32) { if (PAIR) tc::tmem_alloc_pair(&tbase, 512); else tc::tmem_alloc(&tbase, 512); }
    tc::fence_async_smem();
    tc::tc_fence_before();
    if (PAIR) tc::cluster_sync(); else __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = tbase;
    const bool leader = !PAIR || tc::cluster_ctarank() == 0;
    if (tid == 0 && leader) {
        const uint32_t a = tc::smem_u32(sm), b = tc::smem_u32(sm + 32768);
        // descriptors: SW128 MN-major (LBO 1 KB, SBO 2 KB), SW128 K-major (LBO 16, SBO 1 KB: 8 rows x 128 B),
        // SW32 K-major (LBO 16, SBO 256)
        auto desc = [&](uint32_t base, int lay) -> uint64_t {
            if (lay == 0) return tc::smem_desc(base, 1024, 2048, tc::kLayoutSw128);   // MN-major SW128
            if (lay == 1) return tc::smem_desc(base, 16, 1024, tc::kLayoutSw128);     // K-major SW128
            if (lay == 2) return tc::smem_desc(base, 16, 256, tc::kLayoutSw32);       // K-major SW32
            return tc::smem_desc(base, 16, 512, tc::kLayoutSw64);                     // K-major SW64
        };
        const uint64_t ad = desc(a, LAYA), bd = desc(b, LAYB);
        const uint32_t idesc = tc::idesc_bf16_f32(M, N, AMN, BMN);
        const long long t0 = clock64();
        for (int i = 0; i < iters; ++i) {
            const uint32_t d = tmem + (uint32_t)((i % NACC) * N);
            if (PAIR) tc::mma_f16_ss_pair(d, ad, bd, idesc, i >= NACC);
            else tc::mma_f16_ss(d, ad, bd, idesc, i >= NACC);
        }
        if (PAIR) tc::mma_commit_pair(tc::smem_u32(&bar), 3); else tc::mma_commit(tc::smem_u32(&bar));
        tc::mbar_wait_drain(&bar, 0, err);
        const long long t1 = clock64();
        atomicAdd(out, (unsigned long long)(t1 - t0));
        atomicAdd(out + 1, 1ull);
    } else if (PAIR && tid == 0) {
        tc::mbar_wait_drain(&bar, 0, err);
    }
    tc::tc_fence_before();
    if (PAIR) tc::cluster_sync(); else __syncthreads();
    tc::tc_fence_after();
    if (tid < 32) { if (PAIR) tc::tmem_dealloc_pair(tmem, 512); else tc::tmem_dealloc(tmem, 512); }
}

template <int M, int N, int AMN, int BMN, int LAYA, int LAYB, int PAIR, int NACC>
void run(const char* name, int sms) {
    unsigned long long* out; int* err;
    cudaMalloc(&out, 16); cudaMalloc(&err, 4);
    cudaMemset(out, 0, 16); cudaMemset(err, 0, 4);
    auto k = probe<M, N, AMN, BMN, LAYA, LAYB, PAIR, NACC>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 65536);
    const int iters = 20000;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(PAIR ? (sms / 2) * 2 : sms); cfg.blockDim = dim3(128); cfg.dynamicSmemBytes = 65536;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension; at[0].val.clusterDim.x = PAIR ? 2 : 1; at[0].val.clusterDim.y = 1; at[0].val.clusterDim.z = 1;
    cfg.attrs = at; cfg.numAttrs = 1;
    cudaEvent_t e0, e1; cudaEventCreate(&e0); cudaEventCreate(&e1);
    cudaLaunchKernelEx(&cfg, k, 200, out, err);  // warm-up
    cudaDeviceSynchronize();
    cudaMemset(out, 0, 16);
    cudaEventRecord(e0);
    cudaLaunchKernelEx(&cfg, k, iters, out, err);
    cudaEventRecord(e1);
    cudaError_t ce = cudaDeviceSynchronize();
    float ms; cudaEventElapsedTime(&ms, e0, e1);
    unsigned long long h[2]; int herr; cudaMemcpy(h, out, 16, cudaMemcpyDeviceToHost); cudaMemcpy(&herr, err, 4, cudaMemcpyDeviceToHost);
    const double cyc = (double)h[0] / (double)(h[1] ? h[1] : 1) / iters;
    const double macs_per_sm = (double)(PAIR ? M / 2 : M) * N * 16;
    const double ctas = PAIR ? (sms / 2) * 2 : sms;
    const double tflops = 2.0 * macs_per_sm * ctas * iters / (ms * 1e-3) / 1e12;
    printf("%-44s cycles/MMA/SM %7.1f  MAC/clk/SM %6.0f  %7.1f TFLOP/s  (%s, err %d)\n", name, cyc, macs_per_sm / cyc, tflops,
           cudaGetErrorString(ce), herr);
    cudaFree(out); cudaFree(err);
}

int main() {
    int sms = 0; cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    run<128, 128, 1, 1, 0, 0, 0, 1>("M128 N128 A,B MN SW128 (splat), 1 acc", sms);
    run<128, 128, 1, 1, 0, 0, 0, 2>("M128 N128 A,B MN SW128, 2 acc", sms);
    run<128, 128, 0, 0, 3, 3, 0, 2>("M128 N128 A,B K SW64 (spass), 2 acc", sms);
    run<128, 128, 0, 0, 1, 1, 0, 2>("M128 N128 A,B K SW128, 2 acc", sms);
    run<128, 256, 1, 0, 0, 2, 0, 1>("M128 N256 A MN SW128, B K SW32 (fpass)", sms);
    run<128, 256, 1, 0, 0, 2, 0, 2>("M128 N256 A MN SW128, B K SW32, 2 acc", sms);
    run<128, 256, 0, 0, 1, 1, 0, 2>("M128 N256 A,B K SW128, 2 acc", sms);
    run<128, 256, 1, 1, 0, 0, 0, 2>("M128 N256 A,B MN SW128, 2 acc", sms);
    run<256, 256, 0, 0, 1, 1, 1, 2>("PAIR M256 N256 A,B K SW128, 2 acc", sms);
    run<256, 256, 1, 0, 0, 2, 1, 2>("PAIR M256 N256 A MN SW128 B K SW32", sms);
    return 0;
}
