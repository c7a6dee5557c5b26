// gpb2_sync.cuh -- grid-wide barrier for the library's cooperative (persistent) kernels.
//
// The kernels that use it are launched with cudaLaunchCooperativeKernel, so every CTA of the
// grid is resident and a barrier cannot deadlock by construction.  The wait is still bounded:
// after kSpinLimit polls a CTA records GPB2_SYNC_TIMEOUT in the shared error word and every CTA
// leaves at its next barrier, so a fault elsewhere can never turn into a hung GPU.  The host
// reads the error word after the launch and reports GPB2_ERR_TIMEOUT.
//
// Arrival is one atomic per CTA on a single word: CTA 0 adds 2^31 - (nblocks - 1), every other
// CTA adds 1, so the word's top bit flips exactly when the last CTA arrives and the low bits are
// back where they started; a CTA waits for the top bit to differ from the value it saw on
// arrival.  The word must be zero before the launch.
#pragma once
#include <cuda_runtime.h>

namespace gpb2 {

constexpr int GPB2_SYNC_TIMEOUT = 1;

struct GridSync {
    unsigned int* bar;  // arrival word (zeroed before the launch)
    int* err;           // error word (zeroed before the launch)
};

// ~2^24 polls of an L2-resident word: well over a second, far above any legitimate wait.
constexpr unsigned int kSpinLimit = 1u << 24;

__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_relaxed_gpu(const int* p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Dataflow sweeps: a field value not yet produced holds kPending (all bits set, a NaN that no
// arithmetic produces: the device's NaN results are the canonical 0x7fffffff / 0x7ff8...).
template <typename T>
struct Pending;
template <>
struct Pending<float> {
    using U = unsigned int;
    static constexpr U kBits = 0xffffffffu;
};
template <>
struct Pending<double> {
    using U = unsigned long long;
    static constexpr U kBits = 0xffffffffffffffffull;
};

__device__ __forceinline__ unsigned int ld_relaxed_bits(const float* p) {
    unsigned int v;
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed_bits(const double* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed(float* p, float v) {
    asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(__float_as_uint(v)) : "memory");
}
__device__ __forceinline__ void st_relaxed(double* p, double v) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p),
                 "l"((unsigned long long)__double_as_longlong(v))
                 : "memory");
}
__device__ __forceinline__ float bits_to(unsigned int u, float) { return __uint_as_float(u); }
__device__ __forceinline__ double bits_to(unsigned long long u, double) {
    return __longlong_as_double((long long)u);
}

// Wait (bounded) until *p has been produced.  On timeout the error word is set and NaN returned,
// so the sweep still ends and the host reports GPB2_ERR_TIMEOUT.
template <typename T>
__device__ __forceinline__ T wait_value(const T* p, int* err) {
    using U = typename Pending<T>::U;
    U u = ld_relaxed_bits(p);
    unsigned int it = 0;
    while (u == Pending<T>::kBits) {
        if ((++it & 1023u) == 0u && (it > kSpinLimit || ld_relaxed_gpu(err))) {
            atomicCAS(err, 0, GPB2_SYNC_TIMEOUT);
            return bits_to(Pending<T>::kBits >> 1, T());  // a NaN that is not kPending
        }
        u = ld_relaxed_bits(p);
    }
    return bits_to(u, T());
}

// Publish a produced value (never the pending pattern itself).
template <typename T>
__device__ __forceinline__ void publish_value(T* p, T v) {
    using U = typename Pending<T>::U;
    U u;
    memcpy(&u, &v, sizeof(U));
    if (u == Pending<T>::kBits) v = bits_to(Pending<T>::kBits >> 1, T());
    st_relaxed(p, v);
}

// All threads of all CTAs call this; returns false if the grid must stop (timeout anywhere).
__device__ __forceinline__ bool grid_sync(const GridSync& gs) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int nb = gridDim.x * gridDim.y * gridDim.z;
        const bool lead = (blockIdx.x | blockIdx.y | blockIdx.z) == 0;
        const unsigned int add = lead ? (0x80000000u - (nb - 1u)) : 1u;
        __threadfence();
        const unsigned int old = atomicAdd(gs.bar, add);
        int ok = 1;
        unsigned int it = 0;
        while (((old ^ ld_acquire_gpu(gs.bar)) & 0x80000000u) == 0u) {
            if ((++it & 1023u) == 0u && (it > kSpinLimit || ld_relaxed_gpu(gs.err))) {
                atomicCAS(gs.err, 0, GPB2_SYNC_TIMEOUT);
                ok = 0;
                break;
            }
        }
        if (ok && ld_relaxed_gpu(gs.err)) ok = 0;
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

}  // namespace gpb2
