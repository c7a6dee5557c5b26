// gpb2_noalloc.cu -- gpb2_refine_logdet_grad_vals_noalloc: refine_logdet_grad_vals whose scratch
// is a fixed device array, so that the call itself never allocates device memory.
//
// gpb2_refine_logdet_grad_vals takes its double-precision histogram from the handle's scratch,
// which the handle allocates with cudaMalloc on first use.  Some callers cannot let a library
// allocate at that point: a framework's caching allocator (CUDA.jl's pool, PyTorch's) may hold
// the free HBM, so a cudaMalloc inside the call fails, and cudaMalloc / cudaFree can synchronise
// the device in the middle of the caller's pipeline.  This variant accumulates in a file-scope
// __device__ array instead (one per device, found with cudaGetSymbolAddress on the first call
// with that device current) and performs no allocation of its own.
//
// Limits and rules:
//   * nbins <= kNoAllocMaxBins (4096); larger tables are rejected with GPB2_ERR_INVALID_ARG.
//   * The array is shared by every caller on a device: calls that overlap in time (other host
//     threads, other streams, other problems) race on it and corrupt each other's result.
//   * The first call on each device must be made outside stream capture (it resolves the
//     array's address and the kernel attributes).
//   * Everything that must start at zero (the histogram and the log-det accumulator) is cleared
//     by the call itself with cudaMemsetAsync on the caller's stream.
#include <mutex>

#include "gpb2_problem.h"

namespace gpb2 {

namespace {

constexpr int64_t kNoAllocMaxBins = 4096;
constexpr int64_t kNoAllocScalars = 8;  // log-det accumulator (+ spare), after the histogram
constexpr int kNoAllocMaxDevices = 64;

// 4096 + 8 doubles = 32.8 KB per device.
static __device__ __align__(256) double g_noalloc_acc[kNoAllocMaxBins + kNoAllocScalars];

template <typename T>
__global__ void k_noalloc_hist_to_t(const double* __restrict__ acc, T* __restrict__ out,
                                    int64_t nb) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nb;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (T)acc[i];
}

std::mutex g_addr_mu;
double* g_addr[kNoAllocMaxDevices] = {};

// Address of this device's accumulator; `device` must be current.
int noalloc_acc(int device, double** out) {
    if (device < 0 || device >= kNoAllocMaxDevices)
        return set_error(GPB2_ERR_INVALID_ARG, "noalloc: device %d out of range", device);
    std::lock_guard<std::mutex> lk(g_addr_mu);
    if (!g_addr[device]) {
        void* ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_acc);
        if (e != cudaSuccess || !ptr)
            return set_error(GPB2_ERR_CUDA, "noalloc: cudaGetSymbolAddress failed: %s",
                             cudaGetErrorString(e));
        g_addr[device] = static_cast<double*>(ptr);
    }
    *out = g_addr[device];
    return GPB2_OK;
}

template <typename T>
int run(gpb2_problem* p, T* dvals, double* ld, cudaStream_t s) {
    double* acc = nullptr;
    GPB2_TRY(noalloc_acc(p->device, &acc));
    GPB2_CUDA_TRY(cudaMemsetAsync(acc, 0, sizeof(double) * (p->nb + kNoAllocScalars), s));
    cudaError_t e = ops_of<T>(p)->logdet_grad(point_args<T>(p), acc, acc + p->nb, nullptr,
                                              Pts::all(p->m), s);
    if (e != cudaSuccess)
        return set_error(GPB2_ERR_CUDA, "noalloc logdet grad launch failed: %s",
                         cudaGetErrorString(e));
    // The same grid as the allocating form's conversion (grid-stride loop, 256 threads).
    const int64_t g = std::min<int64_t>((p->nb + 255) / 256, 148 * 16);
    k_noalloc_hist_to_t<T><<<(unsigned)std::max<int64_t>(g, 1), 256, 0, s>>>(acc, dvals, p->nb);
    GPB2_CUDA_TRY(cudaGetLastError());
    double h = 0.0;
    if (ld)
        GPB2_CUDA_TRY(cudaMemcpyAsync(&h, acc + p->nb, sizeof(double), cudaMemcpyDeviceToHost, s));
    GPB2_CUDA_TRY(cudaStreamSynchronize(s));
    if (ld) *ld = h;
    return GPB2_OK;
}

}  // namespace

}  // namespace gpb2

using namespace gpb2;

int gpb2_refine_logdet_grad_vals_noalloc(gpb2_problem* p, void* dvals, double* ld, void* stream) {
    clear_error();
    if (!p || !dvals)
        return set_error(GPB2_ERR_INVALID_ARG, "gpb2_refine_logdet_grad_vals_noalloc: NULL");
    if (p->an_grid)
        return set_error(GPB2_ERR_INVALID_ARG,
                         "gpb2_refine_logdet_grad_vals_noalloc: the anisotropic covariance "
                         "supports the forward operations only");
    if (p->nb > kNoAllocMaxBins)
        return set_error(GPB2_ERR_INVALID_ARG,
                         "gpb2_refine_logdet_grad_vals_noalloc: %lld bins exceed the fixed "
                         "accumulator of %lld bins; use gpb2_refine_logdet_grad_vals",
                         (long long)p->nb, (long long)kNoAllocMaxBins);
    DeviceGuard dg(p->device);
    if (!dg.ok) return set_error(GPB2_ERR_NO_DEVICE, "cudaSetDevice(%d) failed", p->device);
    cudaStream_t s = (cudaStream_t)stream;
    return p->dtype == GPB2_F32 ? run<float>(p, static_cast<float*>(dvals), ld, s)
                                : run<double>(p, static_cast<double*>(dvals), ld, s);
}
