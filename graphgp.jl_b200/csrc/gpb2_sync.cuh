// gpb2_sync.cuh -- grid-wide barrier for the library's cooperative (persistent) kernels.
//
// The kernels that use it are launched with cudaLaunchCooperativeKernel, so every CTA of the
// grid is resident and a barrier cannot deadlock by construction.  The wait is still bounded:
// after kSpinLimit polls a CTA records GPB2_SYNC_TIMEOUT in the shared error word and every CTA
// leaves at its next barrier, so a fault elsewhere can never turn into a hung GPU.  The host reads
// the error word after the launch and reports GPB2_ERR_TIMEOUT.
#pragma once
#include <cuda_runtime.h>

namespace gpb2 {

constexpr int GPB2_SYNC_TIMEOUT = 1;

struct GridSync {
    unsigned int* bar;  // [0] arrivals, [1] generation (zeroed before the launch)
    int* err;           // error word (zeroed before the launch)
};

// ~2^22 polls x ~256 ns: a few seconds at most, far above any legitimate wait.
constexpr unsigned int kSpinLimit = 1u << 22;

// All threads of all CTAs call this; returns false if the grid must stop (timeout anywhere).
__device__ __forceinline__ bool grid_sync(const GridSync& gs) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        volatile unsigned int* gen = gs.bar + 1;
        const unsigned int g = *gen;
        __threadfence();
        const unsigned int nb = gridDim.x * gridDim.y * gridDim.z;
        if (atomicAdd(gs.bar, 1u) == nb - 1) {
            atomicExch(gs.bar, 0u);
            __threadfence();
            atomicAdd(const_cast<unsigned int*>(gen), 1u);
        } else {
            unsigned int it = 0;
            while (*gen == g) {
                if (++it > kSpinLimit || *(volatile int*)gs.err) {
                    atomicCAS(gs.err, 0, GPB2_SYNC_TIMEOUT);
                    ok = 0;
                    break;
                }
                __nanosleep(256);
            }
        }
        __threadfence();
        if (*(volatile int*)gs.err) ok = 0;
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

}  // namespace gpb2
