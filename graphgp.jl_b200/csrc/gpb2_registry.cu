// gpb2_registry.cu -- kernel registry, launch-shape helpers and the launch profiler.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "gpb2_internal.h"
#include "gpb2_kernels.cuh"
#include "gpb2_kset.h"

namespace gpb2 {

#define GPB2_DECL(T, TN, D, K) const Ops<T>* ops_##TN##_d##D##_k##K();
GPB2_KSET(GPB2_DECL)
#undef GPB2_DECL

#define GPB2_FIND(T, TN, DD, KK) \
    if (D == DD && K == KK) return ops_##TN##_d##DD##_k##KK();
template <>
const Ops<float>* find_ops<float>(int K, int D) {
    GPB2_DK(GPB2_FIND, float, f32)
    return nullptr;
}
template <>
const Ops<double>* find_ops<double>(int K, int D) {
    GPB2_DK(GPB2_FIND, double, f64)
    return nullptr;
}
#undef GPB2_FIND

namespace {
struct KernelInfo {
    int blocks_per_sm = 0;
    size_t smem_set = 0;
};
std::mutex g_mu;
std::unordered_map<const void*, KernelInfo> g_info;  // per kernel; one device per process
int g_sms = 0;
}  // namespace

cudaError_t prepare_kernel_smem(const void* kernel, size_t smem) {
    std::lock_guard<std::mutex> lk(g_mu);
    KernelInfo& ki = g_info[kernel];
    if (smem > 48 * 1024 && smem > ki.smem_set) {
        cudaError_t e =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) {
            cudaGetLastError();  // reported here: no later call may find it pending
            return e;
        }
        ki.smem_set = smem;
        ki.blocks_per_sm = 0;
    }
    return cudaSuccess;
}

int flat_grid(const void* kernel, int threads, size_t smem, int64_t work) {
    int per_sm;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (g_sms == 0) {
            int dev = 0;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
            if (g_sms <= 0) g_sms = 1;
        }
        KernelInfo& ki = g_info[kernel];
        if (ki.blocks_per_sm == 0) {
            int b = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, threads, smem) !=
                    cudaSuccess || b <= 0)
                b = 1;
            ki.blocks_per_sm = b;
        }
        per_sm = ki.blocks_per_sm;
    }
    const int64_t need = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)per_sm * g_sms;
    return (int)(need < cap ? need : cap);
}

int coop_grid(const void* kernel, int threads, size_t smem) {
    return flat_grid(kernel, threads, smem, INT64_MAX / 2);
}

// ------------------------------------------------------------------------------------------
// Launch profiler.  Every kernel launch of the library goes through prof_begin/prof_end: the
// launch counter is always on; with profiling enabled a CUDA event pair is recorded around the
// launch on its own stream, and gpb2_profile_report sums the elapsed times per kernel kind.
// ------------------------------------------------------------------------------------------
namespace {
struct ProfRec {
    const char* name;
    cudaEvent_t a, b;
};
std::atomic<int> g_prof_on{0};
std::atomic<unsigned long long> g_launches{0};
std::mutex g_prof_mu;
std::vector<ProfRec> g_recs;
std::vector<cudaEvent_t> g_pool;

cudaEvent_t take_event() {
    if (!g_pool.empty()) {
        cudaEvent_t e = g_pool.back();
        g_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    return e;
}
}  // namespace

ProfToken prof_begin(const char* name, cudaStream_t s) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    ProfToken t{name, nullptr, nullptr};
    if (!g_prof_on.load(std::memory_order_relaxed)) return t;
    std::lock_guard<std::mutex> lk(g_prof_mu);
    t.a = take_event();
    t.b = take_event();
    if (t.a) cudaEventRecord(t.a, s);
    return t;
}

void prof_end(const ProfToken& t, cudaStream_t s) {
    if (!t.a || !t.b) return;
    cudaEventRecord(t.b, s);
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_recs.push_back({t.name, t.a, t.b});
}

}  // namespace gpb2

using namespace gpb2;

extern "C" {

int gpb2_profile_enable(int on) {
    g_prof_on.store(on ? 1 : 0);
    return GPB2_OK;
}

int gpb2_profile_reset(void) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    for (auto& r : g_recs) {
        cudaEventSynchronize(r.b);
        g_pool.push_back(r.a);
        g_pool.push_back(r.b);
    }
    g_recs.clear();
    g_launches.store(0);
    return GPB2_OK;
}

int64_t gpb2_launch_count(void) { return (int64_t)g_launches.load(); }

int gpb2_profile_report(char* buf, int64_t cap) {
    if (!buf || cap <= 0) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_profile_report: no buffer");
    std::map<std::string, std::pair<long long, double>> agg;
    {
        std::lock_guard<std::mutex> lk(g_prof_mu);
        for (auto& r : g_recs) {
            float ms = 0.f;
            if (cudaEventSynchronize(r.b) == cudaSuccess &&
                cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
                auto& e = agg[r.name];
                e.first += 1;
                e.second += ms;
            }
        }
    }
    std::string out;
    char line[256];
    for (auto& kv : agg) {
        snprintf(line, sizeof(line), "%s %lld %.6f\n", kv.first.c_str(), kv.second.first,
                 kv.second.second);
        out += line;
    }
    if ((int64_t)out.size() + 1 > cap)
        return set_error(GPB2_ERR_INVALID_ARG, "gpb2_profile_report: buffer too small (%zu)",
                         out.size() + 1);
    memcpy(buf, out.c_str(), out.size() + 1);
    return GPB2_OK;
}

}  // extern "C"
