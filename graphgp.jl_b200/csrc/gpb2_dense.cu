// gpb2_dense.cu -- the dense first layer (the n0 root points) on the device.
//
// Follows src/dense.jl: the n0 x n0 covariance is assembled with the same integer-distance +
// interpolation pipeline as the refine kernels (_assemble_dense_cov, :15-40) and factorised with
// the jitter ladder of _dense_chol_L (:46-67) by the exact-order kernels of gpb2_dense_chol.cu.
// generate_dense is L*xi, generate_dense_inv is L\v, generate_dense_logdet is
// sum(log(diag(L))); the triangular products and solves use cuBLAS.
//
// Adjoints:
//  * generate_grad_vals dense block (src/grad_generate_vals.jl:252-280): L-bar = tril(vb xi^T)
//    pulled back through the Cholesky.  The scalar recurrence chol_pullback_dyn! is O(n0^3)
//    sequential; here it is the equivalent blocked form S = L^-T Phi(L^T L-bar) L^-1 (Phi =
//    lower triangle with halved diagonal), whose lower-triangle gradient is S_ij + S_ji off
//    the diagonal and S_ii on it -- the same quantity the recurrence computes.
//  * _dense_logdet_grad_vals (src/dense.jl:153-183): K^-1 = L^-T L^-1 (one SYRK of the inverse
//    kept with the factor; potri when that inverse is not kept); cotangent
//    K^-1[a,b] off-diagonal, K^-1[a,a]/2 on the diagonal.
//  * _dense_inv_loss_grad_vals (src/dense.jl:244-266): alpha = K^-1 y; cotangent -alpha_a*alpha_b,
//    -alpha_a^2/2 on the diagonal.
// Every cotangent is scattered into the vals histogram through cov_lookup_weights of its pair.
#include <cmath>
#include <vector>

#include "gpb2_problem.h"

namespace gpb2 {

namespace {

// --- cuBLAS / cuSOLVER overloads -----------------------------------------------------------
inline cublasStatus_t trmv(cublasHandle_t h, cublasOperation_t op, int n, const float* A,
                           float* x) {
    return cublasStrmv(h, CUBLAS_FILL_MODE_LOWER, op, CUBLAS_DIAG_NON_UNIT, n, A, n, x, 1);
}
inline cublasStatus_t trmv(cublasHandle_t h, cublasOperation_t op, int n, const double* A,
                           double* x) {
    return cublasDtrmv(h, CUBLAS_FILL_MODE_LOWER, op, CUBLAS_DIAG_NON_UNIT, n, A, n, x, 1);
}
inline cublasStatus_t trsv(cublasHandle_t h, cublasOperation_t op, int n, const float* A,
                           float* x) {
    return cublasStrsv(h, CUBLAS_FILL_MODE_LOWER, op, CUBLAS_DIAG_NON_UNIT, n, A, n, x, 1);
}
inline cublasStatus_t trsv(cublasHandle_t h, cublasOperation_t op, int n, const double* A,
                           double* x) {
    return cublasDtrsv(h, CUBLAS_FILL_MODE_LOWER, op, CUBLAS_DIAG_NON_UNIT, n, A, n, x, 1);
}
inline cublasStatus_t trmm(cublasHandle_t h, cublasSideMode_t side, cublasOperation_t op, int n,
                           const float* A, const float* B, float* C) {
    const float one = 1.0f;
    return cublasStrmm(h, side, CUBLAS_FILL_MODE_LOWER, op, CUBLAS_DIAG_NON_UNIT, n, n, &one, A,
                       n, B, n, C, n);
}
inline cublasStatus_t trmm(cublasHandle_t h, cublasSideMode_t side, cublasOperation_t op, int n,
                           const double* A, const double* B, double* C) {
    const double one = 1.0;
    return cublasDtrmm(h, side, CUBLAS_FILL_MODE_LOWER, op, CUBLAS_DIAG_NON_UNIT, n, n, &one, A,
                       n, B, n, C, n);
}
inline cublasStatus_t trsm(cublasHandle_t h, cublasSideMode_t side, cublasOperation_t op, int n,
                           const float* A, float* B) {
    const float one = 1.0f;
    return cublasStrsm(h, side, CUBLAS_FILL_MODE_LOWER, op, CUBLAS_DIAG_NON_UNIT, n, n, &one, A,
                       n, B, n);
}
inline cublasStatus_t trsm(cublasHandle_t h, cublasSideMode_t side, cublasOperation_t op, int n,
                           const double* A, double* B) {
    const double one = 1.0;
    return cublasDtrsm(h, side, CUBLAS_FILL_MODE_LOWER, op, CUBLAS_DIAG_NON_UNIT, n, n, &one, A,
                       n, B, n);
}
// y = op(A) x (A n x n column-major).
inline cublasStatus_t gemv(cublasHandle_t h, cublasOperation_t op, int n, const float* A,
                           const float* x, float* y) {
    const float one = 1.0f, zero = 0.0f;
    return cublasSgemv(h, op, n, n, &one, A, n, x, 1, &zero, y, 1);
}
inline cublasStatus_t gemv(cublasHandle_t h, cublasOperation_t op, int n, const double* A,
                           const double* x, double* y) {
    const double one = 1.0, zero = 0.0;
    return cublasDgemv(h, op, n, n, &one, A, n, x, 1, &zero, y, 1);
}

// Lower triangle of C = A^T A (A n x n column-major).
inline cublasStatus_t syrk_tn(cublasHandle_t h, int n, const float* A, float* C) {
    const float one = 1.0f, zero = 0.0f;
    return cublasSsyrk(h, CUBLAS_FILL_MODE_LOWER, CUBLAS_OP_T, n, n, &one, A, n, &zero, C, n);
}
inline cublasStatus_t syrk_tn(cublasHandle_t h, int n, const double* A, double* C) {
    const double one = 1.0, zero = 0.0;
    return cublasDsyrk(h, CUBLAS_FILL_MODE_LOWER, CUBLAS_OP_T, n, n, &one, A, n, &zero, C, n);
}

inline cusolverStatus_t potri_ws(cusolverDnHandle_t h, int n, float* A, int* lw) {
    return cusolverDnSpotri_bufferSize(h, CUBLAS_FILL_MODE_LOWER, n, A, n, lw);
}
inline cusolverStatus_t potri_ws(cusolverDnHandle_t h, int n, double* A, int* lw) {
    return cusolverDnDpotri_bufferSize(h, CUBLAS_FILL_MODE_LOWER, n, A, n, lw);
}
inline cusolverStatus_t potri(cusolverDnHandle_t h, int n, float* A, float* w, int lw, int* info) {
    return cusolverDnSpotri(h, CUBLAS_FILL_MODE_LOWER, n, A, n, w, lw, info);
}
inline cusolverStatus_t potri(cusolverDnHandle_t h, int n, double* A, double* w, int lw,
                              int* info) {
    return cusolverDnDpotri(h, CUBLAS_FILL_MODE_LOWER, n, A, n, w, lw, info);
}

#define GPB2_BLAS_TRY(expr)                                                                     \
    do {                                                                                        \
        cublasStatus_t _b = (expr);                                                             \
        if (_b != CUBLAS_STATUS_SUCCESS)                                                        \
            return set_error(GPB2_ERR_CUDA, "%s:%d: %s -> cuBLAS status %d", __FILE__, __LINE__, \
                             #expr, (int)_b);                                                   \
    } while (0)
#define GPB2_SOLVER_TRY(expr)                                                                    \
    do {                                                                                         \
        cusolverStatus_t _c = (expr);                                                            \
        if (_c != CUSOLVER_STATUS_SUCCESS)                                                       \
            return set_error(GPB2_ERR_CUDA, "%s:%d: %s -> cuSOLVER status %d", __FILE__,         \
                             __LINE__, #expr, (int)_c);                                          \
    } while (0)

constexpr int kDenseThreads = 256;

// Radius between root points i and j (exact Int64 squared lattice distance), runtime D.
template <typename T>
__device__ __forceinline__ T pair_radius(const uint32_t* __restrict__ coords, int DS, int D,
                                         int64_t i, int64_t j, T scale) {
    long long sq = 0;
    for (int d = 0; d < D; d++) {
        const long long di = (long long)coords[i * DS + d] - (long long)coords[j * DS + d];
        sq += di * di;
    }
    return Num<T>::mul(Num<T>::sqrt(Num<T>::from_i64(sq)), scale);
}

template <typename T>
__global__ void k_dense_logdet(const T* __restrict__ L, int64_t n, double* __restrict__ acc) {
    __shared__ double red[32];
    double s = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        s += (double)Num<T>::log(L[i * n + i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += red[w];
        atomicAdd(acc, t);
    }
}

// W = tril(vb xi^T), column-major (the L-bar seed of src/grad_generate_vals.jl:258-261).
template <typename T>
__global__ void k_outer_tril(const T* __restrict__ vb, const T* __restrict__ xi, int64_t n,
                             T* __restrict__ W) {
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n * n;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = idx / n, i = idx - j * n;
        W[idx] = i >= j ? Num<T>::mul(vb[i], xi[j]) : T(0);
    }
}

// Phi: keep the lower triangle, halve the diagonal, zero the strict upper part.
template <typename T>
__global__ void k_phi(T* __restrict__ X, int64_t n) {
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n * n;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = idx / n, i = idx - j * n;
        X[idx] = i > j ? X[idx] : (i == j ? Num<T>::mul(X[idx], T(0.5)) : T(0));
    }
}

template <typename T>
__global__ void k_sum_sq_half(const T* __restrict__ z, int64_t n, double* __restrict__ acc) {
    __shared__ double red[32];
    double s = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        s += (double)z[i] * (double)z[i] * 0.5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += red[w];
        atomicAdd(acc, t);
    }
}

// Scatter a dense cotangent into the vals histogram (modes documented at the top of the file):
//   mode 0: S (full n x n):     g_ij = S_ij + S_ji (i > j), g_ii = S_ii
//   mode 1: Kinv (lower valid): g_ij = Kinv_ij,             g_ii = Kinv_ii / 2
//   mode 2: alpha (vector):     g_ij = -alpha_i * alpha_j,   g_ii = -alpha_i^2 / 2
template <typename T, typename MT>
__global__ void k_dense_scatter(TableView<T> tv, const uint32_t* __restrict__ coords, int D,
                                int DS, T scale, int64_t n, int mode, const MT* __restrict__ A,
                                double* __restrict__ gacc) {
    using N = Num<T>;
    extern __shared__ __align__(16) unsigned char smem[];
    SmemTable<T> tab;
    tab.stage(tv, smem, threadIdx.x, blockDim.x);
    double* hist = reinterpret_cast<double*>(smem + table_smem_bytes<T>(tv.nb, tv.nkeys));
    for (int i = threadIdx.x; i < tv.nb; i += blockDim.x) hist[i] = 0.0;
    __syncthreads();
    for (int64_t j = blockIdx.x; j < n; j += gridDim.x) {
        for (int64_t i = j + threadIdx.x; i < n; i += blockDim.x) {
            if constexpr (!std::is_same<MT, T>::value) {  // double S from the triangular path
                const double g = i == j ? (double)A[j * n + j]
                                        : (double)A[j * n + i] + (double)A[i * n + j];
                if (i == j) {
                    atomicAdd(&hist[0], g);
                } else {
                    T wlo, whi;
                    const int lo =
                        tab.weights(pair_radius<T>(coords, DS, D, i, j, scale), wlo, whi);
                    atomicAdd(&hist[lo], g * (double)wlo);
                    atomicAdd(&hist[lo + 1], g * (double)whi);
                }
                continue;
            } else {
            T g;
            if (mode == 0) g = i == j ? A[j * n + j] : N::add(A[j * n + i], A[i * n + j]);
            else if (mode == 1) g = i == j ? N::mul(T(0.5), A[j * n + j]) : A[j * n + i];
            else g = i == j ? N::mul(N::mul(T(-0.5), A[i]), A[i]) : N::mul(-A[i], A[j]);
            if (i == j) {
                atomicAdd(&hist[0], (double)g);  // r = 0: bin 0 with weight 1
            } else {
                T wlo, whi;
                const int lo = tab.weights(pair_radius<T>(coords, DS, D, i, j, scale), wlo, whi);
                atomicAdd(&hist[lo], (double)N::mul(g, wlo));
                atomicAdd(&hist[lo + 1], (double)N::mul(g, whi));
            }
            }
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < tv.nb; i += blockDim.x) {
        const double h = hist[i];
        if (h != 0.0) atomicAdd(&gacc[i], h);
    }
}

// Position gradient of the dense block (_dense_logdet_grad_points / _dense_inv_loss_grad_points,
// src/dense.jl:188-225, 271-297): pair (i, j), i > j, cotangent g (mode 1: Kinv_ij from the
// lower triangle of the column-major K^-1; mode 2: -alpha_i * alpha_j) times k'(r) / r times
// scale * (x_i - x_j) added to point i and subtracted from point j (coincident points and flat
// table segments add nothing).  dp is (N, D) row-major, double atomics.
template <typename T>
__global__ void __launch_bounds__(kDenseThreads)
k_dense_points(TableView<T> tv, const uint32_t* __restrict__ coords, int D, int DS, T scale,
               int64_t n, int mode, const T* __restrict__ A, double* __restrict__ dp) {
    using N = Num<T>;
    extern __shared__ __align__(16) unsigned char smem[];
    SmemTable<T> tab;
    tab.stage(tv, smem, threadIdx.x, blockDim.x);
    __syncthreads();
    for (int64_t j = blockIdx.x; j < n; j += gridDim.x) {
        for (int64_t i = j + 1 + threadIdx.x; i < n; i += blockDim.x) {
            const uint32_t* ci = coords + i * DS;
            const uint32_t* cj = coords + j * DS;
            unsigned long long sq = 0;
            for (int d = 0; d < D; d++) {
                const uint32_t di = ci[d] > cj[d] ? ci[d] - cj[d] : cj[d] - ci[d];
                sq += (unsigned long long)di * di;
            }
            if (sq == 0) continue;
            const T r = N::mul(N::sqrt(N::from_i64((long long)sq)), scale);
            const T dcov = tab.dr(r);
            if (dcov == T(0)) continue;
            const T g = mode == 1 ? A[j * n + i] : N::mul(-A[i], A[j]);
            const T factor = N::div(N::mul(g, dcov), r);
            for (int d = 0; d < D; d++) {
                const T diff = N::mul(scale, N::sub(N::from_i64((long long)ci[d]),
                                                    N::from_i64((long long)cj[d])));
                const T c = N::mul(factor, diff);
                atomicAdd(dp + i * D + d, (double)c);
                atomicAdd(dp + j * D + d, -(double)c);
            }
        }
    }
}

template <typename T>
int scatter_points(gpb2_problem* p, int mode, const T* A, double* dp, cudaStream_t s) {
    const size_t smem = table_smem_bytes<T>((int)p->nb, p->nkeys);
    GPB2_CUDA_TRY(prepare_kernel_smem((const void*)k_dense_points<T>, smem));
    const int grid = (int)std::min<int64_t>(p->n0, 2 * 148);
    GPB2_CUDA_TRY(launch_prof("dense_points", k_dense_points<T>, dim3(grid), dim3(kDenseThreads),
                              smem, s, table_view<T>(p), (const uint32_t*)p->coords, (int)p->d,
                              coord_stride((int)p->d), (T)p->scale, p->n0, mode, A, dp));
    return GPB2_OK;
}

template <typename T>
int grid_for(int64_t n) {
    int64_t g = (n + kDenseThreads - 1) / kDenseThreads;
    return (int)(g < 1 ? 1 : (g > 4096 ? 4096 : g));
}

template <typename T, typename MT = T>
int scatter(gpb2_problem* p, int mode, const MT* A, double* hist, cudaStream_t s) {
    const size_t smem = table_smem_bytes<T>((int)p->nb, p->nkeys) + sizeof(double) * p->nb;
    GPB2_CUDA_TRY(prepare_kernel_smem((const void*)k_dense_scatter<T, MT>, smem));
    const int grid = (int)std::min<int64_t>(p->n0, 2 * 148);
    GPB2_CUDA_TRY(launch_prof("dense_scatter", k_dense_scatter<T, MT>, dim3(grid),
                              dim3(kDenseThreads), smem, s, table_view<T>(p),
                              (const uint32_t*)p->coords, (int)p->d, coord_stride((int)p->d),
                              (T)p->scale, p->n0, mode, A, hist));
    return GPB2_OK;
}

}  // namespace

int ensure_dense(gpb2_problem* p) {
    const size_t ts = p->dtype == GPB2_F32 ? 4 : 8;
    const size_t nn = (size_t)p->n0 * (size_t)p->n0;
    GPB2_TRY(ensure_alloc(&p->Wd, ts * nn));
    GPB2_TRY(ensure_alloc(&p->Wd2, ts * nn));
    GPB2_TRY(ensure_alloc(reinterpret_cast<void**>(&p->dinfo), sizeof(int) * 4));
    if (!p->solver) GPB2_SOLVER_TRY(cusolverDnCreate(&p->solver));
    if (!p->blas) GPB2_BLAS_TRY(cublasCreate(&p->blas));
    if (!p->dwork) {
        int lw = 0;
        const int n = (int)p->n0;
        if (p->dtype == GPB2_F32)
            GPB2_SOLVER_TRY(potri_ws(p->solver, n, (float*)p->Wd, &lw));
        else
            GPB2_SOLVER_TRY(potri_ws(p->solver, n, (double*)p->Wd, &lw));
        p->dwork_bytes = (int64_t)ts * std::max(lw, 1);
        GPB2_TRY(ensure_alloc(&p->dwork, (size_t)p->dwork_bytes));
    }
    return GPB2_OK;
}

template <typename T>
int Dense<T>::factor(gpb2_problem* p, cudaStream_t s, bool defer_tri) {
    // The factor depends only on the coordinates (fixed) and the covariance table: a checked
    // factor of the current table is reused (the table setter clears the flag).
    if (p->dense_valid || p->dense_launched) return GPB2_OK;  // (a prefactor launched it)
    GPB2_TRY(ensure_dense(p));
    p->tri_ready = false;
    p->tri_pending = false;
    p->tri_deferred = false;
    GPB2_TRY(dense_cholesky_ladder<T>(p, s));  // gpb2_dense_chol.cu
    if (dense_tri_supported<T>(p)) {
        p->tri_deferred = true;
        if (!defer_tri) return finish_tri(p, s);
    }
    return GPB2_OK;
}

// The row-major copy, the diagonal-block inverses and L^-1 of a factor queued on s (the
// ladder's stream).  When s is the dense stream the readers of these buffers order themselves
// after ev_tri or ev_inv (wait_tri), so the preparation runs beside the caller's next kernels.
template <typename T>
int Dense<T>::finish_tri(gpb2_problem* p, cudaStream_t s) {
    if (!p->tri_deferred) return GPB2_OK;
    p->tri_deferred = false;
    const bool queued = s == p->dstream && p->ev_tri;
    GPB2_TRY(dense_tri_prepare<T>(p, s, queued ? p->ev_tri : nullptr));  // gpb2_dense_tri.cu
    p->tri_ready = true;
    if (queued) {
        GPB2_CUDA_TRY(cudaEventRecord(p->ev_inv, s));
        p->tri_pending = true;
    }
    return GPB2_OK;
}

namespace {

// Orders s after the part of a triangular preparation still queued on the dense stream that
// it reads: the row-major copy alone (inverse = false) or L^-1 as well.
int wait_tri(gpb2_problem* p, cudaStream_t s, bool inverse) {
    if (p->tri_pending && s != p->dstream)
        GPB2_CUDA_TRY(cudaStreamWaitEvent(s, inverse ? p->ev_inv : p->ev_tri, 0));
    return GPB2_OK;
}

}  // namespace

template <typename T>
int Dense<T>::apply_L(gpb2_problem* p, const T* x, T* y, cudaStream_t s) {
    if (p->tri_ready) {
        if (x == y) {
            GPB2_CUDA_TRY(cudaMemcpyAsync(p->Wd2, x, sizeof(T) * p->n0, cudaMemcpyDeviceToDevice,
                                          s));
            x = static_cast<const T*>(p->Wd2);
        }
        return dense_trmv<T>(p, false, x, y, s);
    }
    if (x != y)
        GPB2_CUDA_TRY(cudaMemcpyAsync(y, x, sizeof(T) * p->n0, cudaMemcpyDeviceToDevice, s));
    GPB2_BLAS_TRY(cublasSetStream(p->blas, s));
    GPB2_BLAS_TRY(trmv(p->blas, CUBLAS_OP_N, (int)p->n0, static_cast<const T*>(p->Ld), y));
    return GPB2_OK;
}

template <typename T>
int Dense<T>::apply_Lt(gpb2_problem* p, const T* x, T* y, cudaStream_t s) {
    if (p->tri_ready) {
        GPB2_TRY(wait_tri(p, s, false));  // reads the row-major copy
        if (x == y) {
            GPB2_CUDA_TRY(cudaMemcpyAsync(p->Wd2, x, sizeof(T) * p->n0, cudaMemcpyDeviceToDevice,
                                          s));
            x = static_cast<const T*>(p->Wd2);
        }
        return dense_trmv<T>(p, true, x, y, s);
    }
    if (x != y)
        GPB2_CUDA_TRY(cudaMemcpyAsync(y, x, sizeof(T) * p->n0, cudaMemcpyDeviceToDevice, s));
    GPB2_BLAS_TRY(cublasSetStream(p->blas, s));
    GPB2_BLAS_TRY(trmv(p->blas, CUBLAS_OP_T, (int)p->n0, static_cast<const T*>(p->Ld), y));
    return GPB2_OK;
}

template <typename T>
int Dense<T>::solve_L(gpb2_problem* p, const T* b, T* y, cudaStream_t s) {
    if (p->tri_ready && b != y) {  // y = L^-1 b with the inverse kept with the factor
        GPB2_TRY(wait_tri(p, s, true));
        GPB2_BLAS_TRY(cublasSetStream(p->blas, s));
        GPB2_BLAS_TRY(gemv(p->blas, CUBLAS_OP_N, (int)p->n0, static_cast<const T*>(p->Ainv), b, y));
        return GPB2_OK;
    }
    if (b != y)
        GPB2_CUDA_TRY(cudaMemcpyAsync(y, b, sizeof(T) * p->n0, cudaMemcpyDeviceToDevice, s));
    GPB2_BLAS_TRY(cublasSetStream(p->blas, s));
    GPB2_BLAS_TRY(trsv(p->blas, CUBLAS_OP_N, (int)p->n0, static_cast<const T*>(p->Ld), y));
    return GPB2_OK;
}

template <typename T>
int Dense<T>::logdet(gpb2_problem* p, double* acc, cudaStream_t s) {
    GPB2_CUDA_TRY(launch_prof("dense_logdet", k_dense_logdet<T>, dim3(1), dim3(kDenseThreads), 0,
                              s, static_cast<const T*>(p->Ld), p->n0, acc));
    return GPB2_OK;
}

template <typename T>
int Dense<T>::grad_vals(gpb2_problem* p, const T* vb, const T* xi, double* hist, cudaStream_t s) {
    const int n = (int)p->n0;
    const int64_t nn = (int64_t)n * n;
    T* W = static_cast<T*>(p->Wd);
    T* X = static_cast<T*>(p->Wd2);
    const T* L = static_cast<const T*>(p->Ld);
    if (p->tri_ready) {  // S = L^-T Phi(tril((L^T vb) xi^T)) L^-1 by the triangular kernels
        GPB2_TRY(wait_tri(p, s, true));
        const T* S = nullptr;
        GPB2_TRY(dense_chol_pullback_outer<T>(p, vb, xi, &S, s));
        return scatter<T>(p, 0, S, hist, s);
    }
    GPB2_CUDA_TRY(launch_prof("dense_outer", k_outer_tril<T>, dim3(grid_for<T>(nn)),
                              dim3(kDenseThreads), 0, s, vb, xi, (int64_t)n, W));
    GPB2_BLAS_TRY(cublasSetStream(p->blas, s));
    GPB2_BLAS_TRY(trmm(p->blas, CUBLAS_SIDE_LEFT, CUBLAS_OP_T, n, L, W, X));  // X = L^T W
    GPB2_CUDA_TRY(launch_prof("dense_phi", k_phi<T>, dim3(grid_for<T>(nn)), dim3(kDenseThreads),
                              0, s, X, (int64_t)n));
    GPB2_BLAS_TRY(trsm(p->blas, CUBLAS_SIDE_LEFT, CUBLAS_OP_T, n, L, X));   // X = L^-T X
    GPB2_BLAS_TRY(trsm(p->blas, CUBLAS_SIDE_RIGHT, CUBLAS_OP_N, n, L, X));  // X = X L^-1
    return scatter<T>(p, 0, X, hist, s);
}

// K^-1 (column-major, lower triangle valid) into p->Wd.
template <typename T>
static int dense_kinv(gpb2_problem* p, cudaStream_t s) {
    const int n = (int)p->n0;
    T* W = static_cast<T*>(p->Wd);
    if (p->tri_ready) {
        // K^-1 = L^-T L^-1 from the inverse kept with the factor: one symmetric rank-n update
        // (potri recomputes L^-1 and then forms the same product).
        GPB2_TRY(wait_tri(p, s, true));
        GPB2_BLAS_TRY(cublasSetStream(p->blas, s));
        GPB2_BLAS_TRY(syrk_tn(p->blas, n, static_cast<const T*>(p->Ainv), W));
        return GPB2_OK;
    }
    GPB2_CUDA_TRY(cudaMemcpyAsync(W, p->Ld, sizeof(T) * (size_t)n * n, cudaMemcpyDeviceToDevice,
                                  s));
    GPB2_SOLVER_TRY(cusolverDnSetStream(p->solver, s));
    GPB2_SOLVER_TRY(potri(p->solver, n, W, static_cast<T*>(p->dwork),
                          (int)(p->dwork_bytes / sizeof(T)), p->dinfo));
    return GPB2_OK;
}

template <typename T>
int Dense<T>::logdet_grad(gpb2_problem* p, double* hist, cudaStream_t s) {
    GPB2_TRY(dense_kinv<T>(p, s));
    return scatter<T>(p, 1, static_cast<const T*>(p->Wd), hist, s);
}

template <typename T>
int Dense<T>::logdet_points(gpb2_problem* p, double* dp, cudaStream_t s) {
    GPB2_TRY(dense_kinv<T>(p, s));
    return scatter_points<T>(p, 1, static_cast<const T*>(p->Wd), dp, s);
}

// z = L^-1 y (its half squared norm into *loss when loss is set) and alpha = L^-T z = K^-1 y;
// returns alpha (in p->Wd).
template <typename T>
static int dense_alpha(gpb2_problem* p, const T* y, double* loss, const T** alpha_out,
                       cudaStream_t s) {
    const int n = (int)p->n0;
    T* z = static_cast<T*>(p->Wd);
    if (p->tri_ready) {
        // z = L^-1 y and alpha = L^-T z as two products with the inverse kept with the factor
        // (two matrix-vector products instead of two triangular solves, each a dependent chain).
        GPB2_TRY(wait_tri(p, s, true));
        T* alpha = z + n;
        GPB2_BLAS_TRY(cublasSetStream(p->blas, s));
        GPB2_BLAS_TRY(gemv(p->blas, CUBLAS_OP_N, n, static_cast<const T*>(p->Ainv), y, z));
        if (loss)
            GPB2_CUDA_TRY(launch_prof("dense_sumsq", k_sum_sq_half<T>, dim3(1),
                                      dim3(kDenseThreads), 0, s, (const T*)z, (int64_t)n, loss));
        GPB2_BLAS_TRY(gemv(p->blas, CUBLAS_OP_T, n, static_cast<const T*>(p->Ainv), z, alpha));
        *alpha_out = alpha;
        return GPB2_OK;
    }
    GPB2_TRY(Dense<T>::solve_L(p, y, z, s));  // z = L \ y  (generate_dense_inv)
    if (loss)
        GPB2_CUDA_TRY(launch_prof("dense_sumsq", k_sum_sq_half<T>, dim3(1), dim3(kDenseThreads),
                                  0, s, (const T*)z, (int64_t)n, loss));
    GPB2_BLAS_TRY(trsv(p->blas, CUBLAS_OP_T, n, static_cast<const T*>(p->Ld), z));  // alpha
    *alpha_out = z;
    return GPB2_OK;
}

template <typename T>
int Dense<T>::inv_loss_grad(gpb2_problem* p, const T* y, double* hist, double* loss,
                            cudaStream_t s) {
    const T* alpha = nullptr;
    GPB2_TRY(dense_alpha<T>(p, y, loss, &alpha, s));
    return scatter<T>(p, 2, alpha, hist, s);
}

template <typename T>
int Dense<T>::inv_loss_points(gpb2_problem* p, const T* y, double* dp, cudaStream_t s) {
    const T* alpha = nullptr;
    GPB2_TRY(dense_alpha<T>(p, y, nullptr, &alpha, s));
    return scatter_points<T>(p, 2, alpha, dp, s);
}

template struct Dense<float>;
template struct Dense<double>;

}  // namespace gpb2
