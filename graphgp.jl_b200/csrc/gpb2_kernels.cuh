// gpb2_kernels.cuh -- the kernels of the refine path and their launchers.
//
// Two shapes:
//  * flat kernels over all M refined points (factor, inverse, logdet, the vals-gradient
//    pullbacks): persistent grid (a multiple of the SM count, sized by occupancy), grid-stride
//    over points, the interpolation table staged in shared memory once per CTA;
//  * per-depth-batch kernels (the forward and reverse sweeps and the fused forward level
//    kernel): one launch per batch, a thread per point.  Batch-mates never neighbour each
//    other (check_graph invariant 4), so a batch reads only values finished by earlier
//    launches on the same stream and the reverse sweep's atomics never touch the batch's own
//    entries.
//
// The vals-gradients accumulate a per-CTA double histogram in shared memory and flush it into a
// global double accumulator (one atomic per non-zero bin per CTA).
#pragma once
#include <cuda_runtime.h>

#include "gpb2_device.cuh"
#include "gpb2_sync.cuh"

namespace gpb2 {

// Per-point factor cache of a problem (slab layout: entry e of point m at [e * stride + m], so a
// warp's 32 consecutive points touch one contiguous run per entry): the packed Cholesky factor
// of every refined point (NT slabs) and the interpolation segment and fraction of each of its
// pair radii (NR slabs each).  The factor pass writes it; the vals-gradient kernels read it
// instead of gathering coordinates, interpolating the covariance and factorising again.  The
// entries are the bits the recomputation would produce (the same code writes them).  Null
// pointers: no cache.
template <typename T>
struct FactorCache {
    T* L = nullptr;
    T* t = nullptr;
    uint16_t* lo = nullptr;
    int64_t stride = 0;
};

template <typename T>
struct PointArgs {
    TableView<T> tab;
    const uint32_t* coords;  // (N, coord_stride(D)) uint32
    const int* nbrs;         // (M, K) int32, 0-based
    int64_t n0;
    T scale;
    FactorCache<T> fc;  // write target of k_factor / source of the gradient kernels, or none
    AnisoView<T> an;    // an anisotropic covariance (forward kernels), or none: the table
};

constexpr int kFlatThreads = 128;
constexpr int kSweepThreads = 256;

// Grid for a persistent flat kernel: resident CTAs per SM x SM count, capped by the work.
int flat_grid(const void* kernel, int threads, size_t smem, int64_t work);
cudaError_t prepare_kernel_smem(const void* kernel, size_t smem);

// Launch profiler (gpb2_registry.cu): every launch is counted; with profiling enabled a CUDA
// event pair brackets it on its stream.
struct ProfToken {
    const char* name;
    cudaEvent_t a, b;
};
ProfToken prof_begin(const char* name, cudaStream_t s);
void prof_end(const ProfToken& t, cudaStream_t s);

// Launch `kern` bracketed by the profiler; returns the launch status.
template <class Kern, class... Args>
inline cudaError_t launch_prof(const char* name, Kern kern, dim3 grid, dim3 block, size_t smem,
                               cudaStream_t s, Args... args) {
    const ProfToken t = prof_begin(name, s);
    kern<<<grid, block, smem, s>>>(args...);
    const cudaError_t e = cudaGetLastError();
    prof_end(t, s);
    return e;
}

__device__ __forceinline__ double block_sum_double(double v, double* red /*>= 32 doubles*/) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double s = 0.0;
    if (threadIdx.x == 0)
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) s += red[w];
    return s;  // valid on thread 0
}

// Where the adjoint kernels keep a point's pair radii between the assembly and the histogram
// scatter: the thread's column of a shared-memory block after the histogram when it fits (the
// radii would otherwise occupy NR registers through the whole pullback), else registers.
template <typename T, int K, int D, int NTH = kFlatThreads, size_t CAP = 36 * 1024>
struct RadiusStore {
    static constexpr int NR = PointMath<T, K, D>::NR;
    // Interpolation weights (segment + fraction) when they fit, else radii, in shared memory;
    // else radii in registers.
    static constexpr bool kWeights =
        (size_t)NR * NTH * (sizeof(T) + sizeof(uint16_t)) <= CAP;
    static constexpr bool kSmem = (size_t)NR * NTH * sizeof(T) <= CAP;
    using type = typename std::conditional<
        kWeights, SmemWeights<T>,
        typename std::conditional<kSmem, SmemCol<T>, RegArr<T, NR>>::type>::type;
    static constexpr size_t bytes =
        kWeights ? (size_t)NR * NTH * (sizeof(T) + sizeof(uint16_t))
                 : (kSmem ? (size_t)NR * NTH * sizeof(T) : 0);
    static __device__ __forceinline__ type make(unsigned char* base) {
        if constexpr (kWeights) {
            SmemWeights<T> w;
            w.t = reinterpret_cast<T*>(base) + threadIdx.x;
            w.lo = reinterpret_cast<uint16_t*>(base + (size_t)NR * NTH * sizeof(T)) +
                   threadIdx.x;
            w.stride = NTH;
            return w;
        } else if constexpr (kSmem) {
            SmemCol<T> c;
            c.p = reinterpret_cast<T*>(base) + threadIdx.x;
            c.stride = NTH;
            return c;
        } else {
            return type{};
        }
    }
};

// ---------------------------------------------------------------------------------------------
// Shared per-point preamble: neighbour list, joint coords, covariance, factor.
// ---------------------------------------------------------------------------------------------
template <typename T, int K, int D, bool KEEP_R,
          typename RT = RegArr<T, PointMath<T, K, D>::NR>>
struct PointFactor {
    using PM = PointMath<T, K, D>;
    int nb[K];
    T L[PM::NT];
    RT R;

    __device__ __forceinline__ void compute(const PointArgs<T>& a, const SmemTable<T>& tab,
                                            int64_t m) {
        load_row_i32<K>(nb, a.nbrs + m * K);
        uint32_t jc[PM::KP1][D];
        PM::gather(jc, a.coords, nb, a.n0 + m);
        PM::template assemble<KEEP_R>(L, R, jc, a.scale, tab);
        PM::chol(L);
    }
    // The same with the anisotropic covariance of a.an (src/aniso.jl: forward only).
    __device__ __forceinline__ void compute_aniso(const PointArgs<T>& a, int64_t m) {
        load_row_i32<K>(nb, a.nbrs + m * K);
        uint32_t jc[PM::KP1][D];
        PM::gather(jc, a.coords, nb, a.n0 + m);
        PM::assemble_aniso(L, jc, a.scale, a.an);
        PM::chol(L);
    }
    // Either covariance, for the forward kernels.
    __device__ __forceinline__ void compute_any(const PointArgs<T>& a, const SmemTable<T>& tab,
                                                int64_t m) {
        if (a.an.grid)
            compute_aniso(a, m);
        else
            compute(a, tab, m);
    }
    // The factor cache's slab columns of point m (R must be a SlabWeights).
    __device__ __forceinline__ void bind_cache(const PointArgs<T>& a, int64_t m) {
        R.t = a.fc.t + m;
        R.lo = a.fc.lo + m;
        R.stride = a.fc.stride;
    }
    __device__ __forceinline__ void load_cached(const PointArgs<T>& a, int64_t m) {
        load_row_i32<K>(nb, a.nbrs + m * K);
        sfor<0, PM::NT>([&](auto e_) {
            GPB2_CI(e);
            L[e] = __ldcs(a.fc.L + e * a.fc.stride + m);
        });
        bind_cache(a, m);
    }
    __device__ __forceinline__ void store_cached(const PointArgs<T>& a, int64_t m) const {
        sfor<0, PM::NT>([&](auto e_) {
            GPB2_CI(e);
            a.fc.L[e * a.fc.stride + m] = L[e];
        });
    }
};

// ---------------------------------------------------------------------------------------------
// Flat kernels.
// ---------------------------------------------------------------------------------------------

// The flat kernels visit `cnt` refined points: m = m0 + t, or m = mlist[t] when a list is given
// (the points a rank owns in a level-sharded operation: one chunk of every depth batch).
__device__ __forceinline__ int64_t point_of(int64_t t, int64_t m0, const int* __restrict__ mlist) {
    return mlist ? (int64_t)mlist[t] : m0 + t;
}

// Conditional-mean weights and std of points [m_begin, m_end) (refine_meanvec_std_kernel!,
// src/kernels.jl:61-78): mv is (M, K) point-major, sd is (M).
// With FILL the point's factor and pair weights also go to the factor cache (a.fc).
template <typename T, int K, int D, bool FILL>
__global__ void __launch_bounds__(kFlatThreads)
k_factor(PointArgs<T> a, int64_t m_begin, int64_t m_end, T* __restrict__ mv, T* __restrict__ sd) {
    extern __shared__ __align__(16) unsigned char smem[];
    SmemTable<T> tab;
    tab.stage(a.tab, smem, threadIdx.x, blockDim.x);
    __syncthreads();
    for (int64_t m = m_begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; m < m_end;
         m += (int64_t)gridDim.x * blockDim.x) {
        using RT = typename std::conditional<FILL, SlabWeights<T>,
                                             RegArr<T, PointMath<T, K, D>::NR>>::type;
        PointFactor<T, K, D, FILL, RT> f;
        if constexpr (FILL) {  // the cache is never allocated for an anisotropic problem
            f.bind_cache(a, m);
            f.compute(a, tab, m);
            f.store_cached(a, m);
        } else {
            f.compute_any(a, tab, m);
        }
        T x[K];
        PointMath<T, K, D>::solve(x, f.L, a.tab.pivc);
        store_row_t<T, K>(mv + m * K, x);
        sd[m] = f.L[tri(K, K)];
    }
}

// refine_inv_kernel! (src/kernels.jl:37-56).
template <typename T, int K, int D>
__global__ void __launch_bounds__(kFlatThreads)
k_inv(PointArgs<T> a, const T* __restrict__ values, T* __restrict__ xi_out, int64_t m0,
      int64_t cnt, const int* __restrict__ mlist) {
    using N = Num<T>;
    extern __shared__ __align__(16) unsigned char smem[];
    SmemTable<T> tab;
    tab.stage(a.tab, smem, threadIdx.x, blockDim.x);
    __syncthreads();
    for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < cnt;
         it += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = point_of(it, m0, mlist);
        PointFactor<T, K, D, false> f;
        f.compute_any(a, tab, m);
        T x[K];
        PointMath<T, K, D>::solve(x, f.L, a.tab.pivc);
        T mean = T(0);
        sfor<0, K>([&](auto j_) {
            GPB2_CI(j);
            mean = N::add(mean, N::mul(x[j], values[f.nb[j]]));
        });
        xi_out[m] = N::div(N::sub(values[a.n0 + m], mean), f.L[tri(K, K)]);
    }
}

// refine_logdet_kernel! (src/kernels.jl:25-35) + the sum, accumulated in double.
template <typename T, int K, int D>
__global__ void __launch_bounds__(kFlatThreads)
k_logdet(PointArgs<T> a, T* __restrict__ terms, double* __restrict__ acc, int64_t m0,
         int64_t cnt, const int* __restrict__ mlist) {
    using N = Num<T>;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ double red[32];
    SmemTable<T> tab;
    tab.stage(a.tab, smem, threadIdx.x, blockDim.x);
    __syncthreads();
    double s = 0.0;
    for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < cnt;
         it += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = point_of(it, m0, mlist);
        PointFactor<T, K, D, false> f;
        f.compute_any(a, tab, m);
        const T t = N::log(f.L[tri(K, K)]);
        if (terms) terms[m] = t;
        s += (double)t;
    }
    s = block_sum_double(s, red);
    if (threadIdx.x == 0) atomicAdd(acc, s);
}

// Scatter a point's A-bar (lower triangle, in B) into the CTA histogram: the diagonal sum into
// bin 0, each off-diagonal through the interpolation weights of its radius
// (_scatter_Abar_hist!, src/kernels_adjoint.jl:50-74).  The diagonal sum goes to the thread's
// own accumulator `bin0` (added to bin 0 once per thread: every point hits that bin).
template <typename T, int K, int D, typename RT>
__device__ __forceinline__ void scatter_hist(double* hist, double& bin0,
                                             const T (&B)[PointMath<T, K, D>::NT], const RT& R,
                                             const SmemTable<T>& tab) {
    using N = Num<T>;
    constexpr int KP1 = K + 1;
    sfor<0, KP1>([&](auto a_) {
        GPB2_CI(a);
        bin0 += (double)B[tri(a, a)];
    });
    sfor<1, KP1>([&](auto a_) {
        GPB2_CI(a);
        sfor<0, a>([&](auto b_) {
            GPB2_CI(b);
            T wlo, whi;
            int lo;
            if constexpr (is_weight_store<RT>::value) {
                const auto i = tri(a - 1, b) * R.stride;
                const T t = R.t[i];
                lo = R.lo[i];
                wlo = N::sub(T(1), t);
                whi = t;
            } else {
                lo = tab.weights(R[tri(a - 1, b)], wlo, whi);
            }
            const T g = B[tri(a, b)];
            atomicAdd(&hist[lo], (double)N::mul(g, wlo));
            atomicAdd(&hist[lo + 1], (double)N::mul(g, whi));
        });
    });
}

__device__ __forceinline__ void flush_hist(double* __restrict__ gacc, const double* hist, int nb) {
    for (int i = threadIdx.x; i < nb; i += blockDim.x) {
        const double h = hist[i];
        if (h != 0.0) atomicAdd(&gacc[i], h);
    }
}

// Block shape of the histogram kernels (k_logdet_grad, k_grad_vals, k_inv_loss_grad): 320
// threads, two blocks per SM (20 warps, within both the register file at <= 102 registers and
// shared memory), when the interpolation weights of 320 threads fit in 72 KB; else the flat
// kernels' 128 threads.
template <typename T, int K, int D>
struct GradShape {
    static constexpr int kWide = 320;
    static constexpr bool kUse =
        (size_t)PointMath<T, K, D>::NR * kWide * (sizeof(T) + sizeof(uint16_t)) <= 72 * 1024;
    static constexpr int kThreads = kUse ? kWide : kFlatThreads;
    static constexpr int kMinBlocks = kUse ? 2 : 1;
    // The factor-cache form keeps no pair weights in shared memory and its loop is latency-bound:
    // more resident warps pay more than the registers they cost.  Measured at C4 (f32, K = 8,
    // 2e7 points): k_grad_vals 7.1 ms at 256 threads x 3 blocks per SM against 7.9 ms at the
    // 320 x 2 shape; k_logdet_grad 5.6 ms at 256 x 4 against 7.5 ms.  Other shapes keep the
    // recompute form's block.
    static constexpr bool kCachedWide = kUse && std::is_same<T, float>::value;
    static constexpr int kCachedThreads = kCachedWide ? 256 : kThreads;
    static constexpr int kCachedBlocks = kCachedWide ? 3 : kMinBlocks;        // grad_vals, inv_loss
    static constexpr int kCachedBlocksLogdet = kCachedWide ? 4 : kMinBlocks;  // logdet_grad
    static constexpr int threads(bool cached) { return cached ? kCachedThreads : kThreads; }
    using Store = RadiusStore<T, K, D, kThreads, kUse ? 72 * 1024 : 36 * 1024>;
    // The point factor of a histogram kernel: recomputed (pair weights in Store), or read from
    // the factor cache (pair weights in its slabs).
    template <bool CACHED>
    using Factor = PointFactor<T, K, D, true,
                               typename std::conditional<CACHED, SlabWeights<T>,
                                                         typename Store::type>::type>;
};

// Shared-memory layout of the histogram kernels: [table][histogram][pair-weight store] when the
// factor is recomputed, the histogram alone when it comes from the factor cache (the cached
// weights replace every table search).
template <typename T, bool CACHED>
__device__ __forceinline__ void grad_smem(const PointArgs<T>& a, SmemTable<T>& tab,
                                          unsigned char* smem, double*& hist,
                                          unsigned char*& rbase) {
    if constexpr (CACHED) {
        hist = reinterpret_cast<double*>(smem);
        rbase = nullptr;
    } else {
        tab.stage(a.tab, smem, threadIdx.x, blockDim.x);
        hist = reinterpret_cast<double*>(smem + table_smem_bytes<T>(a.tab.nb, a.tab.nkeys));
        rbase = smem + table_smem_bytes<T>(a.tab.nb, a.tab.nkeys) + sizeof(double) * a.tab.nb;
    }
}

template <typename T, int K, int D, bool CACHED, typename F>
__device__ __forceinline__ void grad_factor(F& f, const PointArgs<T>& a, const SmemTable<T>& tab,
                                            unsigned char* rbase, int64_t m) {
    if constexpr (CACHED) {
        f.load_cached(a, m);
    } else {
        f.R = GradShape<T, K, D>::Store::make(rbase);
        f.compute(a, tab, m);
    }
}

// Each histogram kernel handles a point in two forms: FAST (DivChecked: the adjoint's divisions
// without per-operation range checks, then one check of the point's operands) and exact
// (DivExact, the same arithmetic with div_r's check and IEEE fallback in every division).  The
// FAST form does the whole point and returns true, or, when an operand lay outside the window,
// returns false having written nothing; the kernel then calls the exact form, kept out of line
// (point_exact) so that the rare path does not enlarge the hot loop.  Both give the same bits
// wherever the FAST form accepts a point.

// One point of k_logdet_grad: the log-pivot (its term, into *s) and the Abar scatter.
template <typename T, int K, int D, bool CACHED, bool FAST>
__device__ __forceinline__ bool logdet_grad_point(const PointArgs<T>& a, const SmemTable<T>& tab,
                                                  unsigned char* rbase, int64_t m, double* hist,
                                                  double& bin0, T* terms, double& s) {
    using N = Num<T>;
    using PM = PointMath<T, K, D>;
    typename GradShape<T, K, D>::template Factor<CACHED> f;
    grad_factor<T, K, D, CACHED>(f, a, tab, rbase, m);
    T B[PM::NT];
    sfor<0, PM::NT>([&](auto i_) {
        GPB2_CI(i);
        B[i] = T(0);
    });
    T rp[PM::KP1];
    PM::pivot_recips(rp, f.L);
    B[tri(K, K)] = rp[K];  // chol_logdet_pullback! seed 1/L[K][K] (src/linalg.jl:137-146)
    if constexpr (FAST) {
        DivChecked<T> dv;
        PM::pullback(B, f.L, rp, dv);
        if (!dv.template ok<PM::KP1>(f.L)) return false;
    } else {
        PM::pullback(B, f.L, rp);
    }
    const T t = N::log(f.L[tri(K, K)]);
    if (terms) terms[m] = t;
    s += (double)t;
    scatter_hist<T, K, D>(hist, bin0, B, f.R, tab);
    return true;
}

// One point of k_grad_vals.
template <typename T, int K, int D, bool CACHED, bool FAST>
__device__ __forceinline__ bool grad_vals_point(const PointArgs<T>& a, const SmemTable<T>& tab,
                                                unsigned char* rbase, int64_t m,
                                                const T* __restrict__ v, const T* __restrict__ xih,
                                                const T* __restrict__ vb,
                                                const T* __restrict__ mv, double* hist,
                                                double& bin0) {
    using N = Num<T>;
    using PM = PointMath<T, K, D>;
    const int64_t p = a.n0 + m;
    const T vbp = vb[p];
    typename GradShape<T, K, D>::template Factor<CACHED> f;
    grad_factor<T, K, D, CACHED>(f, a, tab, rbase, m);
    const T pivfloor = N::mul(a.tab.pivc, f.L[0]);
    T B[PM::NT];
    sfor<0, PM::NT>([&](auto i_) {
        GPB2_CI(i);
        B[i] = T(0);
    });
    B[tri(K, K)] = N::mul(vbp, xih[p]);
    T z[K];
    sfor<0, K>([&](auto j_) {
        GPB2_CI(j);
        z[j] = N::mul(vbp, v[f.nb[j]]);
    });
    T rp[PM::KP1];
    PM::pivot_recips(rp, f.L);
    T x[K];  // mean_vec of the point: k_factor's output, the same solve bit for bit
    sfor<0, K>([&](auto j_) {
        GPB2_CI(j);
        x[j] = mv[m * K + j];
    });
    if constexpr (FAST) {
        DivChecked<T> dv;
        PM::template forward_subst<true>(z, f.L, rp, pivfloor, dv);
        PM::seed_from_solve(B, z, x);
        PM::pullback(B, f.L, rp, dv);
        if (!dv.template ok<PM::KP1>(f.L)) return false;
    } else {
        PM::template forward_subst<true>(z, f.L, rp, pivfloor);
        PM::seed_from_solve(B, z, x);
        PM::pullback(B, f.L, rp);
    }
    scatter_hist<T, K, D>(hist, bin0, B, f.R, tab);
    return true;
}

// One point of k_inv_loss_grad: its xi (into xi_out), its loss term (into *ls), the scatter.
template <typename T, int K, int D, bool CACHED, bool FAST>
__device__ __forceinline__ bool inv_loss_grad_point(const PointArgs<T>& a,
                                                    const SmemTable<T>& tab, unsigned char* rbase,
                                                    int64_t m, const T* __restrict__ values,
                                                    double* hist, double& bin0, T* xi_out,
                                                    double& ls) {
    using N = Num<T>;
    using PM = PointMath<T, K, D>;
    typename GradShape<T, K, D>::template Factor<CACHED> f;
    grad_factor<T, K, D, CACHED>(f, a, tab, rbase, m);
    T x[K];
    PM::solve(x, f.L, a.tab.pivc);
    const T sd = f.L[tri(K, K)];
    T vn[K];
    T mean = T(0);
    sfor<0, K>([&](auto j_) {
        GPB2_CI(j);
        vn[j] = values[f.nb[j]];
        mean = N::add(mean, N::mul(x[j], vn[j]));
    });
    const T xim = N::div(N::sub(values[a.n0 + m], mean), sd);
    T B[PM::NT];
    sfor<0, PM::NT>([&](auto i_) {
        GPB2_CI(i);
        B[i] = T(0);
    });
    B[tri(K, K)] = N::div(N::mul(-xim, xim), sd);
    T z[K];
    sfor<0, K>([&](auto j_) {
        GPB2_CI(j);
        z[j] = N::div(N::mul(-xim, vn[j]), sd);
    });
    T rp[PM::KP1];
    PM::pivot_recips(rp, f.L);
    if constexpr (FAST) {
        DivChecked<T> dv;
        PM::template forward_subst<false>(z, f.L, rp, T(0), dv);
        PM::seed_from_solve(B, z, x);
        PM::pullback(B, f.L, rp, dv);
        if (!dv.template ok<PM::KP1>(f.L)) return false;
    } else {
        PM::template forward_subst<false>(z, f.L, rp, T(0));
        PM::seed_from_solve(B, z, x);
        PM::pullback(B, f.L, rp);
    }
    if (xi_out) xi_out[m] = xim;
    ls += (double)N::div(N::mul(xim, xim), T(2));
    scatter_hist<T, K, D>(hist, bin0, B, f.R, tab);
    return true;
}

// The exact forms, out of line: each returns its point's contributions to the thread's
// bin-0 share and scalar accumulator through the two-element array acc.
template <typename T, int K, int D, bool CACHED>
__device__ __noinline__ void logdet_grad_exact(PointArgs<T> a, SmemTable<T> tab,
                                               unsigned char* rbase, int64_t m, double* hist,
                                               T* terms, double* acc) {
    double b0 = 0.0, s = 0.0;
    logdet_grad_point<T, K, D, CACHED, false>(a, tab, rbase, m, hist, b0, terms, s);
    acc[0] = b0;
    acc[1] = s;
}
template <typename T, int K, int D, bool CACHED>
__device__ __noinline__ double grad_vals_exact(PointArgs<T> a, SmemTable<T> tab,
                                               unsigned char* rbase, int64_t m, const T* v,
                                               const T* xih, const T* vb, const T* mv,
                                               double* hist) {
    double b0 = 0.0;
    grad_vals_point<T, K, D, CACHED, false>(a, tab, rbase, m, v, xih, vb, mv, hist, b0);
    return b0;
}
template <typename T, int K, int D, bool CACHED>
__device__ __noinline__ void inv_loss_grad_exact(PointArgs<T> a, SmemTable<T> tab,
                                                 unsigned char* rbase, int64_t m, const T* values,
                                                 double* hist, T* xi_out, double* acc) {
    double b0 = 0.0, ls = 0.0;
    inv_loss_grad_point<T, K, D, CACHED, false>(a, tab, rbase, m, values, hist, b0, xi_out, ls);
    acc[0] = b0;
    acc[1] = ls;
}

// refine_logdet_and_grad_hist_kernel! (src/kernels_adjoint.jl:117-152), seed 1.
template <typename T, int K, int D, bool CACHED>
__global__ void __launch_bounds__(GradShape<T, K, D>::threads(CACHED),
                                  CACHED ? GradShape<T, K, D>::kCachedBlocksLogdet
                                         : GradShape<T, K, D>::kMinBlocks)
k_logdet_grad(PointArgs<T> a, double* __restrict__ gacc, double* __restrict__ ld_acc,
              T* __restrict__ terms, int64_t m0, int64_t cnt, const int* __restrict__ mlist) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ double red[32];
    SmemTable<T> tab;
    double* hist;
    unsigned char* rbase;
    grad_smem<T, CACHED>(a, tab, smem, hist, rbase);
    for (int i = threadIdx.x; i < a.tab.nb; i += blockDim.x) hist[i] = 0.0;
    __syncthreads();
    double bin0 = 0.0;  // this thread's share of histogram bin 0
    double s = 0.0;
    for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < cnt;
         it += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = point_of(it, m0, mlist);
        if (!logdet_grad_point<T, K, D, CACHED, true>(a, tab, rbase, m, hist, bin0, terms, s)) {
            double acc[2];
            logdet_grad_exact<T, K, D, CACHED>(a, tab, rbase, m, hist, terms, acc);
            bin0 += acc[0];
            s += acc[1];
        }
    }
    s = block_sum_double(s, red);
    if (threadIdx.x == 0 && ld_acc) atomicAdd(ld_acc, s);
    atomicAdd(&hist[0], bin0);
    __syncthreads();
    flush_hist(gacc, hist, a.tab.nb);
}

// Per-point vals-gradient of generate (generate_grad_vals_rev_kernel!,
// src/kernels_adjoint.jl:484-553), run over ALL points after the reverse sweep has finalised
// vb: every point's cotangent seed (vb[p]*xi[p], vb[p]*v[nbr]) is then known, and the point's
// pullback needs nothing else, so the batches need not be visited in order.

template <typename T, int K, int D, bool CACHED>
__global__ void __launch_bounds__(GradShape<T, K, D>::threads(CACHED),
                                  CACHED ? GradShape<T, K, D>::kCachedBlocks
                                         : GradShape<T, K, D>::kMinBlocks)
k_grad_vals(PointArgs<T> a, const T* __restrict__ v, const T* __restrict__ xih,
            const T* __restrict__ vb, const T* __restrict__ mv, double* __restrict__ gacc,
            int64_t m0, int64_t cnt, const int* __restrict__ mlist) {
    extern __shared__ __align__(16) unsigned char smem[];
    SmemTable<T> tab;
    double* hist;
    unsigned char* rbase;
    grad_smem<T, CACHED>(a, tab, smem, hist, rbase);
    for (int i = threadIdx.x; i < a.tab.nb; i += blockDim.x) hist[i] = 0.0;
    __syncthreads();
    double bin0 = 0.0;  // this thread's share of histogram bin 0
    for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < cnt;
         it += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = point_of(it, m0, mlist);
        if (!grad_vals_point<T, K, D, CACHED, true>(a, tab, rbase, m, v, xih, vb, mv, hist, bin0))
            bin0 += grad_vals_exact<T, K, D, CACHED>(a, tab, rbase, m, v, xih, vb, mv, hist);
    }
    atomicAdd(&hist[0], bin0);
    __syncthreads();
    flush_hist(gacc, hist, a.tab.nb);
}

// refine_inv_loss_grad_hist_kernel! (src/kernels_adjoint.jl:155-221): loss 0.5*sum(xi^2) and its
// vals-gradient; the z-bar solve has no pivot guard, as in the reference.
template <typename T, int K, int D, bool CACHED>
__global__ void __launch_bounds__(GradShape<T, K, D>::threads(CACHED),
                                  CACHED ? GradShape<T, K, D>::kCachedBlocks
                                         : GradShape<T, K, D>::kMinBlocks)
k_inv_loss_grad(PointArgs<T> a, const T* __restrict__ values, double* __restrict__ gacc,
                double* __restrict__ loss_acc, T* __restrict__ xi_out, int64_t m0, int64_t cnt,
                const int* __restrict__ mlist) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ double red[32];
    SmemTable<T> tab;
    double* hist;
    unsigned char* rbase;
    grad_smem<T, CACHED>(a, tab, smem, hist, rbase);
    for (int i = threadIdx.x; i < a.tab.nb; i += blockDim.x) hist[i] = 0.0;
    __syncthreads();
    double bin0 = 0.0;  // this thread's share of histogram bin 0
    double ls = 0.0;
    for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < cnt;
         it += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = point_of(it, m0, mlist);
        if (!inv_loss_grad_point<T, K, D, CACHED, true>(a, tab, rbase, m, values, hist, bin0,
                                                        xi_out, ls)) {
            double acc[2];
            inv_loss_grad_exact<T, K, D, CACHED>(a, tab, rbase, m, values, hist, xi_out, acc);
            bin0 += acc[0];
            ls += acc[1];
        }
    }
    ls = block_sum_double(ls, red);
    if (threadIdx.x == 0 && loss_acc) atomicAdd(loss_acc, ls);
    atomicAdd(&hist[0], bin0);
    __syncthreads();
    flush_hist(gacc, hist, a.tab.nb);
}

// Point-position gradients of the refined points (refine_logdet_grad_points_kernel! and
// refine_inv_loss_grad_points_kernel!, src/kernels_adjoint.jl:254-324; INV: the inverse loss
// with `values`, else the log-determinant): the point's Abar, then every off-diagonal pair's
// Abar * k'(r) / r * scale * (x_a - x_b) added to point a and subtracted from point b
// (_scatter_Abar_points_atomic!, src/kernels_adjoint.jl:226-251; coincident points and flat
// table segments add nothing).  dp is (N, D) row-major in library positions, double atomics
// (the terms are T products, summed in double as the d(vals) histogram is).
template <typename T, int K, int D, bool INV>
__global__ void __launch_bounds__(kFlatThreads)
k_points_grad(PointArgs<T> pa, const T* __restrict__ values, double* __restrict__ dp, int64_t m0,
              int64_t cnt, const int* __restrict__ mlist) {
    using N = Num<T>;
    using PM = PointMath<T, K, D>;
    extern __shared__ __align__(16) unsigned char smem[];
    SmemTable<T> tab;
    tab.stage(pa.tab, smem, threadIdx.x, blockDim.x);
    __syncthreads();
    for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < cnt;
         it += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = point_of(it, m0, mlist);
        int nb[K];
        load_row_i32<K>(nb, pa.nbrs + m * K);
        uint32_t jc[PM::KP1][D];
        PM::gather(jc, pa.coords, nb, pa.n0 + m);
        T L[PM::NT];
        RegArr<T, PM::NR> R;
        PM::template assemble<false>(L, R, jc, pa.scale, tab);
        PM::chol(L);
        T B[PM::NT];
        sfor<0, PM::NT>([&](auto i_) {
            GPB2_CI(i);
            B[i] = T(0);
        });
        T rp[PM::KP1];
        PM::pivot_recips(rp, L);
        if constexpr (INV) {
            T x[K];
            PM::solve(x, L, pa.tab.pivc);
            const T sd = L[tri(K, K)];
            T vn[K];
            T mean = T(0);
            sfor<0, K>([&](auto j_) {
                GPB2_CI(j);
                vn[j] = values[nb[j]];
                mean = N::add(mean, N::mul(x[j], vn[j]));
            });
            const T xim = N::div(N::sub(values[pa.n0 + m], mean), sd);
            B[tri(K, K)] = N::div(N::mul(-xim, xim), sd);
            T z[K];
            sfor<0, K>([&](auto j_) {
                GPB2_CI(j);
                z[j] = N::div(N::mul(-xim, vn[j]), sd);
            });
            PM::template forward_subst<false>(z, L, rp, T(0));
            PM::seed_from_solve(B, z, x);
        } else {
            B[tri(K, K)] = rp[K];  // chol_logdet_pullback! seed 1/L[K][K]
        }
        PM::pullback(B, L, rp);
        sfor<1, PM::KP1>([&](auto a_) {
            GPB2_CI(a);
            const int64_t ga = a < K ? (int64_t)nb[a] : pa.n0 + m;
            sfor<0, a>([&](auto b_) {
                GPB2_CI(b);
                const T r = PM::radius(jc[a], jc[b], pa.scale);
                if (r == T(0)) return;
                const T dcov = tab.dr(r);
                if (dcov == T(0)) return;
                const int64_t gb = (int64_t)nb[b];  // b < a <= K: always a neighbour
                const T factor = N::div(N::mul(B[tri(a, b)], dcov), r);
                sfor<0, D>([&](auto d_) {
                    GPB2_CI(d);
                    const T diff = N::mul(pa.scale, N::sub(N::from_i64((long long)jc[a][d]),
                                                           N::from_i64((long long)jc[b][d])));
                    const T c = N::mul(factor, diff);
                    atomicAdd(dp + ga * D + d, (double)c);
                    atomicAdd(dp + gb * D + d, -(double)c);
                });
            });
        });
    }
}

// Grid-wide lane index of the persistent sweeps: a warp takes 32 consecutive points (its loads
// are contiguous and, in library order, its points' neighbours are close together), and
// consecutive warps sit on consecutive CTAs (one per SM), so a small batch still spreads over
// every SM's load units instead of queueing on the first few.
__device__ __forceinline__ int64_t sweep_gtid() {
    return ((int64_t)(threadIdx.x >> 5) * gridDim.x + blockIdx.x) * 32 + (threadIdx.x & 31);
}

// ---------------------------------------------------------------------------------------------
// Per-batch kernels.
// ---------------------------------------------------------------------------------------------

// Fused forward for tree positions [p_lo, p_hi) (refine_apply_fused_kernel!,
// src/kernels.jl:101-119): values[p] = std*xi + sum_j mv[j]*values[nbr_j], in that order.
template <typename T, int K, int D>
__global__ void __launch_bounds__(kFlatThreads)
k_fused_fwd(PointArgs<T> a, T* __restrict__ values, const T* __restrict__ xi_ref, int64_t p_lo,
            int64_t p_hi) {
    using N = Num<T>;
    extern __shared__ __align__(16) unsigned char smem[];
    SmemTable<T> tab;
    tab.stage(a.tab, smem, threadIdx.x, blockDim.x);
    __syncthreads();
    for (int64_t p = p_lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < p_hi;
         p += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = p - a.n0;
        PointFactor<T, K, D, false> f;
        f.compute_any(a, tab, m);
        T x[K];
        PointMath<T, K, D>::solve(x, f.L, a.tab.pivc);
        T acc = N::mul(f.L[tri(K, K)], xi_ref[m]);
        sfor<0, K>([&](auto j_) {
            GPB2_CI(j);
            acc = N::add(acc, N::mul(x[j], values[f.nb[j]]));
        });
        values[p] = acc;
    }
}

// Forward sweep step from materialised weights (refine_apply_kernel!, src/kernels.jl:83-94,
// with the fused kernel's accumulation order: std*xi first).
template <typename T, int K>
__global__ void __launch_bounds__(kSweepThreads)
k_sweep_fwd(T* __restrict__ values, const T* __restrict__ xi_ref, const T* __restrict__ mv,
            const T* __restrict__ sd, const int* __restrict__ nbrs, int64_t n0, int64_t p_lo,
            int64_t p_hi) {
    using N = Num<T>;
    const int64_t p = p_lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= p_hi) return;
    const int64_t m = p - n0;
    int nb[K];
    T w[K];
    load_row_i32<K>(nb, nbrs + m * K);
    load_row_t<T, K>(w, mv + m * K);
    T acc = N::mul(__ldg(sd + m), __ldg(xi_ref + m));
#pragma unroll
    for (int j = 0; j < K; j++) acc = N::add(acc, N::mul(w[j], values[nb[j]]));
    values[p] = acc;
}

// Reverse sweep step (refine_reverse_apply_kernel!, src/kernels_adjoint.jl:433-447):
// xg[p] = std*vb[p]; vb[nbr_j] += mv[j]*vb[p] (atomic: batch-mates can share a neighbour).
template <typename T, int K>
__global__ void __launch_bounds__(kSweepThreads)
k_sweep_rev(T* __restrict__ xg, T* __restrict__ vb, const T* __restrict__ mv,
            const T* __restrict__ sd, const int* __restrict__ nbrs, int64_t n0, int64_t p_lo,
            int64_t p_hi) {
    using N = Num<T>;
    const int64_t p = p_lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= p_hi) return;
    const int64_t m = p - n0;
    int nb[K];
    T w[K];
    load_row_i32<K>(nb, nbrs + m * K);
    load_row_t<T, K>(w, mv + m * K);
    const T vbp = vb[p];
    if (xg) xg[p] = N::mul(__ldg(sd + m), vbp);
#pragma unroll
    for (int j = 0; j < K; j++) atomicAdd(vb + nb[j], N::mul(w[j], vbp));
}

// ---------------------------------------------------------------------------------------------
// Persistent sweeps: one cooperative launch per full sweep.  The grid walks the depth batches in
// order with a grid barrier between consecutive batches.  Each thread holds the read-only inputs
// (weights, neighbour list, std, xi) of two points in registers: while the current point's
// neighbour gathers are in flight, the next point's inputs are already being loaded, so a point
// costs one round of memory latency instead of two chained ones.  The first point of the next
// batch is loaded before the barrier.  Field values and cotangents cross the barrier through L2
// (ld/st .cg), never through an SM's L1.
// ---------------------------------------------------------------------------------------------
constexpr int kPersistThreads = 1024;  // k_sweep_fwd_flow

// The transposed graph of the pull-form reverse sweep (built by gpb2_rev.cu): the edges of
// point q are off[q] .. off[q + 1]; edge e comes from refined point mj[e] / K (slot
// mj[e] % K) with weight w[e] = mean_vec of that slot.  off == nullptr: the atomic push.
template <typename T>
struct RevGraph {
    const uint32_t* off = nullptr;
    const int* mj = nullptr;
    const T* w = nullptr;
};

// One point's read-only sweep inputs (a pulled reverse point keeps its edge range in nb[0..1]).
template <typename T, int K>
struct SweepIn {
    int nb[K];
    T w[K];
    T sd;
    T xi;  // forward only
    __device__ __forceinline__ void load(const T* __restrict__ mv, const T* __restrict__ sdv,
                                         const T* __restrict__ xiv, const int* __restrict__ nbrs,
                                         int64_t m) {
        load_row_i32<K>(nb, nbrs + m * K);
        load_row_t<T, K>(w, mv + m * K);
        sd = __ldg(sdv + m);
        if (xiv) xi = __ldg(xiv + m);
    }
    __device__ __forceinline__ void load_pull(const RevGraph<T>& rg, const T* __restrict__ sdv,
                                              int64_t p, int64_t n0) {
        nb[0] = (int)__ldg(rg.off + p);
        nb[1] = (int)__ldg(rg.off + p + 1);
        sd = p >= n0 ? __ldg(sdv + (p - n0)) : T(0);
    }
};

// Block shape of the persistent sweeps: as many threads as the register file holds with two
// points' inputs, K gathered values and ~16 registers of bookkeeping per thread.
template <typename T, int K>
struct SweepShape {
    static constexpr int kWords = (int)sizeof(T) / 4;
    static constexpr int kRegs = 2 * (K + K * kWords + 2 * kWords) + K * kWords + 16;
    static constexpr int kThreads =
        kRegs <= 56 ? 1024 : (kRegs <= 85 ? 768 : (kRegs <= 128 ? 512 : 256));
};

// The incoming terms of point p in the pull-form reverse sweep, in edge order (the serial
// sweep's order): acc = vb[p] + w_0 vb[c_0] + w_1 vb[c_1] + ..., eight edges' loads in flight.
// The children's cotangents are final (written in earlier steps, or by earlier launches) and
// are read through L1 (ld.global.ca), where a child shared by several parents of the CTA hits:
// see the forward gathers in sweep_pipe for why the L1 holds no stale line.
template <typename T, int K>
__device__ __forceinline__ T pull_sum(T acc, const RevGraph<T>& rg, const T* __restrict__ vb,
                                      int64_t n0, uint32_t e, uint32_t end) {
    using N = Num<T>;
    constexpr int U = 8;
    for (; e + U <= end; e += U) {
        int mj[U];
        T w[U], v[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            mj[u] = __ldg(rg.mj + e + u);
            w[u] = __ldg(rg.w + e + u);
        }
#pragma unroll
        for (int u = 0; u < U; u++) v[u] = __ldca(vb + n0 + mj[u] / K);
#pragma unroll
        for (int u = 0; u < U; u++) acc = N::add(acc, N::mul(w[u], v[u]));
    }
    for (; e < end; e++) acc = N::add(acc, N::mul(__ldg(rg.w + e), __ldca(vb + n0 + __ldg(rg.mj + e) / K)));
    return acc;
}

// Step i of a sweep visits forward batch i (F) and reverse batch nbatch-1-i (R); one grid
// barrier per step.  A thread's tasks within a step are F_0, R_0, F_1, R_1, ... (F_k: point
// offs[i] + gtid + k*gsz when below offs[i+1]; R_k likewise in the reverse batch), the absent
// ones skipped; neither kind reads the other's output, so their interleaving is free.  Per
// point the arithmetic and its order are those of the per-batch kernels k_sweep_fwd /
// k_sweep_rev: forward values[p] = std*xi + sum_j mv[j]*values[nbr_j]; reverse
// xg[p] = std*vb[p], vb[nbr_j] += mv[j]*vb[p] -- pushed as atomic additions, or, with PULL, as
// every point's own sum of its incoming terms in the serial order (pull_sum), which needs one
// more step for the dense block [0, n0) after batch 0.
template <typename T, int K, bool F, bool R, bool PULL>
__device__ __forceinline__ void sweep_pipe(T* __restrict__ values, const T* __restrict__ xi_ref,
                                           T* __restrict__ vb, T* __restrict__ xg,
                                           const T* __restrict__ mv, const T* __restrict__ sd,
                                           const int* __restrict__ nbrs, int64_t n0,
                                           const int64_t* __restrict__ offs, int nbatch,
                                           RevGraph<T> rg, GridSync gs) {
    using N = Num<T>;
    const int64_t gtid = sweep_gtid();
    const int64_t gsz = (int64_t)gridDim.x * blockDim.x;
    const int nstep = nbatch + (R && PULL ? 1 : 0);

    int64_t f0 = 0, fhi = 0, r0 = 0, rhi = 0;  // this step's first points and batch ends
    auto set_step = [&](int i) {
        if (i < nbatch) {
            f0 = offs[i] + gtid;
            fhi = offs[i + 1];
            r0 = offs[nbatch - 1 - i] + gtid;
            rhi = offs[nbatch - i];
        } else {  // the pulled dense block
            f0 = fhi = 0;
            r0 = gtid;
            rhi = n0;
        }
    };
    auto has = [&](bool fwd, int64_t k) {
        return fwd ? (F && f0 + k * gsz < fhi) : (R && r0 + k * gsz < rhi);
    };
    auto load = [&](SweepIn<T, K>& in, bool fwd, int64_t k) {
        const int64_t p = (fwd ? f0 : r0) + k * gsz;
        if (!fwd && PULL)
            in.load_pull(rg, sd, p, n0);
        else
            in.load(mv, sd, fwd ? xi_ref : nullptr, nbrs, p - n0);
    };

    SweepIn<T, K> cur, nxt;
    bool fwd, valid;
    int64_t k = 0;
    set_step(0);
    valid = has(true, 0) || has(false, 0);
    fwd = has(true, 0);
    if (valid) load(cur, fwd, 0);
    for (int i = 0; i < nstep; i++) {
        while (valid) {
            // The task after (fwd, k): R_k after F_k, else F_{k+1}, else R_{k+1}.
            bool nfwd = false, nvalid = true;
            int64_t nk = k;
            if (fwd && has(false, k)) {
                nfwd = false;
            } else if (has(true, k + 1)) {
                nfwd = true;
                nk = k + 1;
            } else if (has(false, k + 1)) {
                nfwd = false;
                nk = k + 1;
            } else {
                nvalid = false;
            }
            if (F && fwd) {
                const int64_t p = f0 + k * gsz;
                // The neighbours' values were written in earlier steps, by other CTAs.  They are
                // read through L1 (ld.global.ca: neighbours shared by the CTA's points hit there,
                // -19 % sweep time at C4 1e8): each step begins after grid_sync, whose acquire
                // load (thread 0) and block barrier order these loads after every earlier
                // step's writes, so no stale L1 line is read; lines written during this step
                // hold only this batch's values, which no point of the step reads (batch-mates
                // never neighbour each other).
                T v[K];
                sfor<0, K>([&](auto j_) {
                    GPB2_CI(j);
                    v[j] = __ldca(values + cur.nb[j]);
                });
                if (nvalid) load(nxt, nfwd, nk);
                T acc = N::mul(cur.sd, cur.xi);
                sfor<0, K>([&](auto j_) {
                    GPB2_CI(j);
                    acc = N::add(acc, N::mul(cur.w[j], v[j]));
                });
                __stcg(values + p, acc);
            } else if (R) {
                const int64_t p = r0 + k * gsz;
                if constexpr (PULL) {
                    const T vb0 = __ldcg(vb + p);
                    if (nvalid) load(nxt, nfwd, nk);
                    const T acc = pull_sum<T, K>(vb0, rg, vb, n0, (uint32_t)cur.nb[0],
                                                 (uint32_t)cur.nb[1]);
                    __stcg(vb + p, acc);
                    if (xg && p >= n0) xg[p] = N::mul(cur.sd, acc);
                } else {
                    const T vbp = __ldcg(vb + p);
                    if (nvalid) load(nxt, nfwd, nk);
                    if (xg) xg[p] = N::mul(cur.sd, vbp);
                    sfor<0, K>([&](auto j_) {
                        GPB2_CI(j);
                        atomicAdd(vb + cur.nb[j], N::mul(cur.w[j], vbp));
                    });
                }
            }
            cur = nxt;
            fwd = nfwd;
            k = nk;
            valid = nvalid;
        }
        if (i + 1 < nstep) {
            set_step(i + 1);
            k = 0;
            valid = has(true, 0) || has(false, 0);
            fwd = has(true, 0);
            if (valid) load(cur, fwd, 0);
            if (!grid_sync(gs)) return;
        }
    }
}

template <typename T, int K>
__global__ void __launch_bounds__(SweepShape<T, K>::kThreads)
k_sweep_fwd_all(T* __restrict__ values, const T* __restrict__ xi_ref, const T* __restrict__ mv,
                const T* __restrict__ sd, const int* __restrict__ nbrs, int64_t n0,
                const int64_t* __restrict__ offs, int nbatch, GridSync gs) {
    sweep_pipe<T, K, true, false, false>(values, xi_ref, nullptr, nullptr, mv, sd, nbrs, n0, offs,
                                         nbatch, RevGraph<T>{}, gs);
}

template <typename T, int K, bool PULL>
__global__ void __launch_bounds__(SweepShape<T, K>::kThreads)
k_sweep_rev_all(T* __restrict__ xg, T* __restrict__ vb, const T* __restrict__ mv,
                const T* __restrict__ sd, const int* __restrict__ nbrs, int64_t n0,
                const int64_t* __restrict__ offs, int nbatch, RevGraph<T> rg, GridSync gs) {
    sweep_pipe<T, K, false, true, PULL>(nullptr, nullptr, vb, xg, mv, sd, nbrs, n0, offs, nbatch,
                                        rg, gs);
}

// generate_grad_vals needs both the forward field v (from xi) and the reverse cotangent vb (from
// vbar); neither sweep reads the other's output, so one persistent kernel runs them together:
// step i sweeps forward batch i and reverse batch nbatch-1-i, one grid barrier per step instead
// of one per batch of each sweep.
template <typename T, int K, bool PULL>
__global__ void __launch_bounds__(SweepShape<T, K>::kThreads)
k_sweep_fwdrev_all(T* __restrict__ values, const T* __restrict__ xi_ref, T* __restrict__ vb,
                   const T* __restrict__ mv, const T* __restrict__ sd,
                   const int* __restrict__ nbrs, int64_t n0, const int64_t* __restrict__ offs,
                   int nbatch, RevGraph<T> rg, GridSync gs) {
    sweep_pipe<T, K, true, true, PULL>(values, xi_ref, vb, nullptr, mv, sd, nbrs, n0, offs,
                                       nbatch, rg, gs);
}

template <typename T, int K>
struct SweepPoint {
    int nb[K];
    T w[K];
    T a;  // std * xi (the first product of the forward sum)
    __device__ __forceinline__ void load_fwd(const T* __restrict__ mv, const T* __restrict__ sd,
                                             const T* __restrict__ xi_ref,
                                             const int* __restrict__ nbrs, int64_t m) {
        load_row_i32<K>(nb, nbrs + m * K);
        load_row_t<T, K>(w, mv + m * K);
        a = Num<T>::mul(__ldg(sd + m), __ldg(xi_ref + m));
    }
};

// Dataflow forward sweep: one cooperative launch and no barrier.  values[n0:N] are set to the
// pending pattern before the launch; each point waits only for its own K neighbour values, so
// the sweep's critical path is the graph's dependency chain rather than one grid barrier per
// batch.  Points are dealt in rounds (round k: p = n0 + gtid + k*gsz); every point depends only
// on earlier batches, i.e. on smaller tree positions, so with the whole grid resident the
// earliest unfinished point can always proceed.  Inside a warp the lanes poll together: each
// pass, every lane whose neighbours are all published computes and publishes its point, and the
// warp moves to the next round when all lanes are done -- so a lane never blocks while another
// lane of its own warp still has to publish the value it needs.  Bit-identical to the other
// sweeps (same arithmetic, same order).
template <typename T, int K>
__global__ void __launch_bounds__(kPersistThreads)
k_sweep_fwd_flow(T* __restrict__ values, const T* __restrict__ xi_ref, const T* __restrict__ mv,
                 const T* __restrict__ sd, const int* __restrict__ nbrs, int64_t n0, int64_t n,
                 int* __restrict__ err) {
    using N = Num<T>;
    using U = typename Pending<T>::U;
    const int64_t gtid = (int64_t)threadIdx.x * gridDim.x + blockIdx.x;
    const int64_t gsz = (int64_t)gridDim.x * blockDim.x;
    const int64_t rounds = (n - n0 + gsz - 1) / gsz;
    SweepPoint<T, K> sp;
    for (int64_t k = 0; k < rounds; k++) {
        const int64_t p = n0 + gtid + k * gsz;
        bool done = p >= n;
        if (!done) sp.load_fwd(mv, sd, xi_ref, nbrs, p - n0);
        unsigned int it = 0;
        while (true) {
            if (!done) {
                T v[K];
                bool ready = true;
                sfor<0, K>([&](auto j_) {
                    GPB2_CI(j);
                    const U u = ld_relaxed_bits(values + sp.nb[j]);
                    ready = ready && u != Pending<T>::kBits;
                    v[j] = bits_to(u, T());
                });
                if (ready) {
                    T acc = sp.a;
                    sfor<0, K>([&](auto j_) {
                        GPB2_CI(j);
                        acc = N::add(acc, N::mul(sp.w[j], v[j]));
                    });
                    publish_value(values + p, acc);
                    done = true;
                }
            }
            if (__all_sync(0xffffffffu, done)) break;
            if ((++it & 255u) == 0u) {  // `it` is warp-uniform, so is this test
                const bool stop = it > kSpinLimit || ld_relaxed_gpu(err) != 0;
                if (__any_sync(0xffffffffu, stop)) {
                    if ((threadIdx.x & 31) == 0) atomicCAS(err, 0, GPB2_SYNC_TIMEOUT);
                    return;
                }
            }
        }
    }
}

// Co-resident grid of a cooperative kernel (occupancy x SM count).
int coop_grid(const void* kernel, int threads, size_t smem);

// ---------------------------------------------------------------------------------------------
// Launchers, bundled per (T, K, D) into an Ops table.
// ---------------------------------------------------------------------------------------------
// The refined points a flat kernel visits: [m0, m0 + cnt), or list[0 .. cnt) when list is set.
struct Pts {
    int64_t m0 = 0;
    int64_t cnt = 0;
    const int* list = nullptr;
    static Pts all(int64_t M) { return Pts{0, M, nullptr}; }
};

template <typename T>
struct Ops {
    cudaError_t (*factor)(const PointArgs<T>&, int64_t, int64_t, T*, T*, cudaStream_t);
    cudaError_t (*inv)(const PointArgs<T>&, const T*, T*, Pts, cudaStream_t);
    cudaError_t (*logdet)(const PointArgs<T>&, T*, double*, Pts, cudaStream_t);
    cudaError_t (*logdet_grad)(const PointArgs<T>&, double*, double*, T*, Pts, cudaStream_t);
    cudaError_t (*grad_vals)(const PointArgs<T>&, const T*, const T*, const T*, const T*, double*,
                             Pts, cudaStream_t);
    cudaError_t (*inv_loss_grad)(const PointArgs<T>&, const T*, double*, double*, T*, Pts,
                                 cudaStream_t);
    cudaError_t (*fused_fwd)(const PointArgs<T>&, T*, const T*, int64_t, int64_t, cudaStream_t);
    cudaError_t (*sweep_fwdrev_all)(T*, const T*, T*, const T*, const T*, const int*, int64_t,
                                    const int64_t*, int, RevGraph<T>, GridSync, cudaStream_t);
    cudaError_t (*sweep_fwd_flow)(T*, const T*, const T*, const T*, const int*, int64_t, int64_t,
                                  int*, cudaStream_t);
    cudaError_t (*sweep_fwd)(T*, const T*, const T*, const T*, const int*, int64_t, int64_t,
                             int64_t, cudaStream_t);
    cudaError_t (*sweep_rev)(T*, T*, const T*, const T*, const int*, int64_t, int64_t, int64_t,
                             cudaStream_t);
    cudaError_t (*sweep_fwd_all)(T*, const T*, const T*, const T*, const int*, int64_t,
                                 const int64_t*, int, GridSync, cudaStream_t);
    cudaError_t (*sweep_rev_all)(T*, T*, const T*, const T*, const int*, int64_t, const int64_t*,
                                 int, RevGraph<T>, GridSync, cudaStream_t);
    cudaError_t (*points_grad)(const PointArgs<T>&, const T*, double*, Pts, cudaStream_t);
};

template <typename T>
inline size_t flat_smem(const PointArgs<T>& a, bool hist) {
    return table_smem_bytes<T>(a.tab.nb, a.tab.nkeys) + (hist ? sizeof(double) * a.tab.nb : 0);
}

template <typename T, int K, int D>
struct Launch {
    template <class Kern, class... Args>
    static cudaError_t flat(const char* name, Kern kern, size_t smem, int64_t work,
                            cudaStream_t s, Args... args) {
        if (work <= 0) return cudaSuccess;
        cudaError_t e = prepare_kernel_smem((const void*)kern, smem);
        if (e != cudaSuccess) return e;
        const int grid = flat_grid((const void*)kern, kFlatThreads, smem, work);
        return launch_prof(name, kern, dim3(grid), dim3(kFlatThreads), smem, s, args...);
    }
    static cudaError_t factor(const PointArgs<T>& a, int64_t mb, int64_t me, T* mv, T* sd,
                              cudaStream_t s) {
        if (a.fc.L)
            return flat("factor", k_factor<T, K, D, true>, flat_smem(a, false), me - mb, s, a, mb,
                        me, mv, sd);
        return flat("factor", k_factor<T, K, D, false>, flat_smem(a, false), me - mb, s, a, mb, me,
                    mv, sd);
    }
    // A histogram kernel (k_logdet_grad, k_grad_vals, k_inv_loss_grad) over r.cnt points: the
    // instantiation that reads the factor cache when the arguments carry one.
    template <class KernC, class KernR, class... Args>
    static cudaError_t hist_kernel(const char* name, KernC kc, KernR kr, const PointArgs<T>& a,
                                   int64_t work, cudaStream_t s, Args... args) {
        if (work <= 0) return cudaSuccess;
        using G = GradShape<T, K, D>;
        const bool cached = a.fc.L != nullptr;
        const void* kern = cached ? (const void*)kc : (const void*)kr;
        const size_t smem = cached ? sizeof(double) * a.tab.nb
                                   : flat_smem(a, true) + G::Store::bytes;
        cudaError_t e = prepare_kernel_smem(kern, smem);
        if (e != cudaSuccess) return e;
        const int threads = G::threads(cached);
        const int grid = flat_grid(kern, threads, smem, work);
        if (cached)
            return launch_prof(name, kc, dim3(grid), dim3(threads), smem, s, a, args...);
        return launch_prof(name, kr, dim3(grid), dim3(threads), smem, s, a, args...);
    }
    static cudaError_t inv(const PointArgs<T>& a, const T* values, T* xi, Pts r,
                           cudaStream_t s) {
        return flat("inv", k_inv<T, K, D>, flat_smem(a, false), r.cnt, s, a, values, xi, r.m0,
                    r.cnt, r.list);
    }
    static cudaError_t logdet(const PointArgs<T>& a, T* terms, double* acc, Pts r,
                              cudaStream_t s) {
        return flat("logdet", k_logdet<T, K, D>, flat_smem(a, false), r.cnt, s, a, terms, acc,
                    r.m0, r.cnt, r.list);
    }
    static cudaError_t logdet_grad(const PointArgs<T>& a, double* gacc, double* ld, T* terms,
                                   Pts r, cudaStream_t s) {
        return hist_kernel("logdet_grad", k_logdet_grad<T, K, D, true>,
                           k_logdet_grad<T, K, D, false>, a, r.cnt, s, gacc, ld, terms, r.m0,
                           r.cnt, r.list);
    }
    static cudaError_t grad_vals(const PointArgs<T>& a, const T* v, const T* xih, const T* vb,
                                 const T* mv, double* gacc, Pts r, cudaStream_t s) {
        return hist_kernel("grad_vals", k_grad_vals<T, K, D, true>, k_grad_vals<T, K, D, false>,
                           a, r.cnt, s, v, xih, vb, mv, gacc, r.m0, r.cnt, r.list);
    }
    static cudaError_t inv_loss_grad(const PointArgs<T>& a, const T* values, double* gacc,
                                     double* loss, T* xi_out, Pts r, cudaStream_t s) {
        return hist_kernel("inv_loss_grad", k_inv_loss_grad<T, K, D, true>,
                           k_inv_loss_grad<T, K, D, false>, a, r.cnt, s, values, gacc, loss,
                           xi_out, r.m0, r.cnt, r.list);
    }
    static cudaError_t fused_fwd(const PointArgs<T>& a, T* values, const T* xi_ref, int64_t lo,
                                 int64_t hi, cudaStream_t s) {
        return flat("fused_fwd", k_fused_fwd<T, K, D>, flat_smem(a, false), hi - lo, s, a,
                    values, xi_ref, lo, hi);
    }
    static cudaError_t sweep_fwd(T* values, const T* xi_ref, const T* mv, const T* sd,
                                 const int* nbrs, int64_t n0, int64_t lo, int64_t hi,
                                 cudaStream_t s) {
        if (hi <= lo) return cudaSuccess;
        const int64_t grid = (hi - lo + kSweepThreads - 1) / kSweepThreads;
        return launch_prof("sweep_fwd", k_sweep_fwd<T, K>, dim3((unsigned)grid),
                           dim3(kSweepThreads), 0, s, values, xi_ref, mv, sd, nbrs, n0, lo, hi);
    }
    static cudaError_t sweep_rev(T* xg, T* vb, const T* mv, const T* sd, const int* nbrs,
                                 int64_t n0, int64_t lo, int64_t hi, cudaStream_t s) {
        if (hi <= lo) return cudaSuccess;
        const int64_t grid = (hi - lo + kSweepThreads - 1) / kSweepThreads;
        return launch_prof("sweep_rev", k_sweep_rev<T, K>, dim3((unsigned)grid),
                           dim3(kSweepThreads), 0, s, xg, vb, mv, sd, nbrs, n0, lo, hi);
    }
    template <class Kern, class... Args>
    static cudaError_t coop(const char* name, Kern kern, int threads, size_t smem, cudaStream_t s,
                            Args... args) {
        if (smem) {
            const cudaError_t e = prepare_kernel_smem((const void*)kern, smem);
            if (e != cudaSuccess) return e;
        }
        const int grid = coop_grid((const void*)kern, threads, smem);
        void* argv[] = {(void*)&args...};
        const ProfToken t = prof_begin(name, s);
        const cudaError_t e =
            cudaLaunchCooperativeKernel((const void*)kern, grid, threads, argv, smem, s);
        prof_end(t, s);
        return e;
    }
    using SS = SweepShape<T, K>;
    static cudaError_t sweep_fwd_all(T* values, const T* xi_ref, const T* mv, const T* sd,
                                     const int* nbrs, int64_t n0, const int64_t* offs, int nbatch,
                                     GridSync gs, cudaStream_t s) {
        if (nbatch <= 0) return cudaSuccess;
        return coop("sweep_fwd_all", k_sweep_fwd_all<T, K>, SS::kThreads, 0, s, values, xi_ref, mv, sd, nbrs, n0,
                    offs, nbatch, gs);
    }
    static cudaError_t sweep_fwd_flow(T* values, const T* xi_ref, const T* mv, const T* sd,
                                      const int* nbrs, int64_t n0, int64_t n, int* err,
                                      cudaStream_t s) {
        if (n <= n0) return cudaSuccess;
        return coop("sweep_fwd_flow", k_sweep_fwd_flow<T, K>, kPersistThreads, 0, s, values, xi_ref, mv, sd, nbrs,
                    n0, n, err);
    }
    // rg.off set: the pull-form reverse sweep (an extra step for the dense block), else push.
    static cudaError_t sweep_fwdrev_all(T* values, const T* xi_ref, T* vb, const T* mv,
                                        const T* sd, const int* nbrs, int64_t n0,
                                        const int64_t* offs, int nbatch, RevGraph<T> rg,
                                        GridSync gs, cudaStream_t s) {
        if (nbatch <= 0) return cudaSuccess;
        if (rg.off)
            return coop("sweep_fwdrev_all", k_sweep_fwdrev_all<T, K, true>, SS::kThreads, 0, s,
                        values, xi_ref, vb, mv, sd, nbrs, n0, offs, nbatch, rg, gs);
        return coop("sweep_fwdrev_all", k_sweep_fwdrev_all<T, K, false>, SS::kThreads, 0, s,
                    values, xi_ref, vb, mv, sd, nbrs, n0, offs, nbatch, rg, gs);
    }
    static cudaError_t sweep_rev_all(T* xg, T* vb, const T* mv, const T* sd, const int* nbrs,
                                     int64_t n0, const int64_t* offs, int nbatch, RevGraph<T> rg,
                                     GridSync gs, cudaStream_t s) {
        if (nbatch <= 0) return cudaSuccess;
        if (rg.off)
            return coop("sweep_rev_all", k_sweep_rev_all<T, K, true>, SS::kThreads, 0, s, xg, vb,
                        mv, sd, nbrs, n0, offs, nbatch, rg, gs);
        return coop("sweep_rev_all", k_sweep_rev_all<T, K, false>, SS::kThreads, 0, s, xg, vb, mv,
                    sd, nbrs, n0, offs, nbatch, rg, gs);
    }
    // values != nullptr: the inverse-loss position gradient, else the log-determinant's.
    static cudaError_t points_grad(const PointArgs<T>& a, const T* values, double* dp, Pts r,
                                   cudaStream_t s) {
        if (values)
            return flat("points_grad", k_points_grad<T, K, D, true>, flat_smem(a, false), r.cnt,
                        s, a, values, dp, r.m0, r.cnt, r.list);
        return flat("points_grad", k_points_grad<T, K, D, false>, flat_smem(a, false), r.cnt, s,
                    a, values, dp, r.m0, r.cnt, r.list);
    }
    static const Ops<T>* ops() {
        static const Ops<T> o = {factor,        inv,           logdet,
                                 logdet_grad,   grad_vals,     inv_loss_grad,
                                 fused_fwd,     sweep_fwdrev_all, sweep_fwd_flow,
                                 sweep_fwd,     sweep_rev,     sweep_fwd_all,
                                 sweep_rev_all, points_grad};
        return &o;
    }
};

// Registry: the (K, D) pairs with a compiled kernel set (gpb2_inst_*.cu).
template <typename T>
const Ops<T>* find_ops(int K, int D);

}  // namespace gpb2
