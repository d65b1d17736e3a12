// g2v_profile.cu -- per-kernel CUDA-event timing behind g2v_profile_enable / g2v_profile_read.
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "g2v.h"
#include "g2v_internal.cuh"

namespace g2v {

volatile int g_profiling = 0;

namespace {
struct Rec {
    const char* name;
    cudaEvent_t a, b;
};
std::mutex g_mu;
std::vector<Rec> g_recs;        // recorded launches since the last enable
std::vector<cudaEvent_t> g_pool;  // reusable events

cudaEvent_t get_event() {
    if (!g_pool.empty()) {
        cudaEvent_t e = g_pool.back();
        g_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

struct Agg {
    std::string name;
    double ms = 0.0;
    int64_t n = 0;
};
std::vector<Agg> g_agg;

void recycle_locked() {
    for (auto& r : g_recs) {
        g_pool.push_back(r.a);
        g_pool.push_back(r.b);
    }
    g_recs.clear();
}
}  // namespace

int prof_start(const char* name, cudaStream_t s) {
    std::lock_guard<std::mutex> lk(g_mu);
    Rec r{name, get_event(), get_event()};
    cudaEventRecord(r.a, s);
    g_recs.push_back(r);
    return (int)g_recs.size() - 1;
}

void prof_stop(int slot, cudaStream_t s) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (slot >= 0 && slot < (int)g_recs.size()) cudaEventRecord(g_recs[slot].b, s);
}

}  // namespace g2v

using namespace g2v;

extern "C" {

int g2v_profile_enable(int enabled) {
    std::lock_guard<std::mutex> lk(g_mu);
    for (auto& r : g_recs) {
        cudaEventSynchronize(r.b);
    }
    recycle_locked();
    g_agg.clear();
    g_profiling = enabled ? 1 : 0;
    return G2V_SUCCESS;
}

int g2v_profile_read(int index, char* name, size_t name_len, double* total_ms, int64_t* launches) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_recs.empty()) {
        for (auto& r : g_recs) {
            cudaError_t e = cudaEventSynchronize(r.b);
            if (e != cudaSuccess) return cuda_fail(e, "cudaEventSynchronize");
            float ms = 0.0f;
            e = cudaEventElapsedTime(&ms, r.a, r.b);
            if (e != cudaSuccess) return cuda_fail(e, "cudaEventElapsedTime");
            Agg* a = nullptr;
            for (auto& x : g_agg)
                if (x.name == r.name) a = &x;
            if (!a) {
                g_agg.push_back(Agg{r.name});
                a = &g_agg.back();
            }
            a->ms += ms;
            a->n += 1;
        }
        recycle_locked();
    }
    if (index < 0 || index >= (int)g_agg.size()) return G2V_ERROR_INVALID_VALUE;
    if (name && name_len) {
        strncpy(name, g_agg[index].name.c_str(), name_len - 1);
        name[name_len - 1] = 0;
    }
    if (total_ms) *total_ms = g_agg[index].ms;
    if (launches) *launches = g_agg[index].n;
    return G2V_SUCCESS;
}

}  // extern "C"
