// gpb2_dense_chol.cu -- the dense block's Cholesky factorisation with the reference's jitter
// ladder (_dense_chol_L, src/dense.jl:46-67), as one cooperative kernel.
//
// Exact order.  The reference factorises with LAPACK; the oracle restates it as the unblocked
// left-looking recurrence  L[i][j] = (A[i][j] - sum_{p<j} L[i][p]*L[j][p]) / L[j][j],  the sum
// taken as sequential subtractions p = 0, 1, ..., j-1.  A right-looking elimination applies to
// every entry (i, j) exactly the same subtractions in exactly the same order (column p's update
// reaches (i, j) after columns 0..p-1 and before p+1..j-1), so the blocked phases below --
// diagonal block, panel rows, trailing update, each subtracting one product at a time with
// round-to-nearest and no contraction -- reproduce the oracle's factor bit for bit, including
// the column at which a non-positive pivot makes an attempt fail.
//
// Ladder.  Candidate 0 is K itself, candidates 1..8 are K + eps*mean(diag) on the diagonal for
// eps = 1e-9, 1e-8, ..., 1e-2 (the sequence evaluated in T, as the reference writes it).  For a
// block up to kSpecMax all candidates are factorised in the same launch -- one n0 x n0
// factorisation is latency-bound and leaves most of the device idle -- and the first success is
// selected on the device; a larger block tries the candidates one after another.  A candidate
// that fails stops at its failing panel.
//
// Schedule (one cooperative launch, bounded grid barriers between phases), per 32-wide panel:
//   D  one warp per live candidate factors the 32 x 32 diagonal block, a row per lane;
//   P  (candidate, 256-row chunk) tasks: each thread solves one row of the panel below the block;
//   U  (candidate, 64 x 64 lower tile) tasks: the trailing update with the panel's 32 columns.
#include <cmath>
#include <vector>

#include "gpb2_problem.h"

namespace gpb2 {

namespace {

constexpr int kB = 32;          // panel width (= warp size: one row per lane in phase D)
constexpr int kSpecMax = 4096;  // concurrent ladder up to this n0
constexpr int kCholThreads = 256;
constexpr int kRowChunk = kCholThreads;

template <typename T>
__host__ __device__ constexpr int tile_of() { return sizeof(T) == 4 ? 64 : 32; }  // smem < 48 KB

template <typename T>
struct CholArgs {
    T* base;          // nc candidates, each n x n column-major (lower triangle)
    int64_t n;
    int nc;
    int* fail;        // fail[c] = failing column + 1, 0 while alive
    int* sel;         // first live candidate, -1 if none
    GridSync gs;
};

// Phase D: candidate c's diagonal block [p0, p0+bs)^2, lane i holding row i in registers.
template <typename T>
__device__ void chol_diag_warp(const CholArgs<T>& a, int c, int p0) {
    using N = Num<T>;
    const int lane = threadIdx.x & 31;
    T* L = a.base + (int64_t)c * a.n * a.n;
    const int bs = a.n - p0 < kB ? (int)(a.n - p0) : kB;
    T r[kB];
    sfor<0, kB>([&](auto j_) {
        GPB2_CI(j);
        r[j] = (lane < bs && j <= lane) ? __ldcg(L + (p0 + lane) + (int64_t)(p0 + j) * a.n)
                                        : T(0);
    });
    int bad = 0;
    sfor<0, kB>([&](auto j_) {
        GPB2_CI(j);
        if (j < bs && !bad) {
            const T s = __shfl_sync(0xffffffffu, r[j], j);
            if (!(s > T(0))) {  // LAPACK potrf's failure test (also catches NaN)
                bad = p0 + j + 1;
            } else {
                const T d = N::sqrt(s);
                if (lane == j) r[j] = d;
                else if (lane > j) r[j] = N::div(r[j], d);
                sfor<j + 1, kB>([&](auto q_) {
                    GPB2_CI(q);
                    const T lqj = __shfl_sync(0xffffffffu, r[j], q);
                    if (lane >= q) r[q] = N::sub(r[q], N::mul(r[j], lqj));
                });
            }
        }
    });
    if (bad) {
        if (lane == 0) a.fail[c] = bad;
        return;
    }
    sfor<0, kB>([&](auto j_) {
        GPB2_CI(j);
        if (lane < bs && j <= lane) __stcg(L + (p0 + lane) + (int64_t)(p0 + j) * a.n, r[j]);
    });
}

// Phase P: rows [r0, r0 + kRowChunk) below candidate c's diagonal block.
template <typename T>
__device__ void chol_panel_rows(const CholArgs<T>& a, int c, int p0, int64_t r0, T (*Dg)[kB + 1]) {
    using N = Num<T>;
    T* L = a.base + (int64_t)c * a.n * a.n;
    for (int e = threadIdx.x; e < kB * kB; e += blockDim.x) {
        const int i = e % kB, j = e / kB;
        Dg[i][j] = (i >= j) ? __ldcg(L + (p0 + i) + (int64_t)(p0 + j) * a.n) : T(0);
    }
    __syncthreads();
    const int64_t i = r0 + threadIdx.x;
    if (i < a.n) {
        T x[kB];
        sfor<0, kB>([&](auto j_) {
            GPB2_CI(j);
            x[j] = __ldcg(L + i + (int64_t)(p0 + j) * a.n);
        });
        sfor<0, kB>([&](auto j_) {
            GPB2_CI(j);
            x[j] = N::div(x[j], Dg[j][j]);
            sfor<j + 1, kB>([&](auto q_) {
                GPB2_CI(q);
                x[q] = N::sub(x[q], N::mul(x[j], Dg[q][j]));
            });
        });
        sfor<0, kB>([&](auto j_) {
            GPB2_CI(j);
            __stcg(L + i + (int64_t)(p0 + j) * a.n, x[j]);
        });
    }
    __syncthreads();
}

// Phase U: lower tile (bi, bj) of candidate c's trailing matrix [t0, n)^2.
template <typename T>
__device__ void chol_update_tile(const CholArgs<T>& a, int c, int p0, int bi, int bj,
                                 T (*Li)[kB + 1], T (*Lj)[kB + 1]) {
    using N = Num<T>;
    constexpr int TL = tile_of<T>();
    constexpr int R = TL / 16;
    T* L = a.base + (int64_t)c * a.n * a.n;
    const int64_t t0 = p0 + kB;
    const int64_t r0 = t0 + (int64_t)bi * TL, c0 = t0 + (int64_t)bj * TL;
    for (int e = threadIdx.x; e < TL * kB; e += blockDim.x) {
        const int rr = e % TL, p = e / TL;
        const int64_t gi = r0 + rr, gj = c0 + rr;
        Li[rr][p] = gi < a.n ? __ldcg(L + gi + (int64_t)(p0 + p) * a.n) : T(0);
        Lj[rr][p] = gj < a.n ? __ldcg(L + gj + (int64_t)(p0 + p) * a.n) : T(0);
    }
    __syncthreads();
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    T acc[R][R];
    bool live[R][R];
#pragma unroll
    for (int u = 0; u < R; u++)
#pragma unroll
        for (int v = 0; v < R; v++) {
            const int64_t gi = r0 + ty + 16 * u, gj = c0 + tx + 16 * v;
            live[u][v] = gi < a.n && gj < a.n && gi >= gj;
            acc[u][v] = live[u][v] ? __ldcg(L + gi + gj * a.n) : T(0);
        }
#pragma unroll 4
    for (int p = 0; p < kB; p++) {
        T li[R], lj[R];
#pragma unroll
        for (int u = 0; u < R; u++) li[u] = Li[ty + 16 * u][p];
#pragma unroll
        for (int v = 0; v < R; v++) lj[v] = Lj[tx + 16 * v][p];
#pragma unroll
        for (int u = 0; u < R; u++)
#pragma unroll
            for (int v = 0; v < R; v++) acc[u][v] = N::sub(acc[u][v], N::mul(li[u], lj[v]));
    }
#pragma unroll
    for (int u = 0; u < R; u++)
#pragma unroll
        for (int v = 0; v < R; v++)
            if (live[u][v]) __stcg(L + (r0 + ty + 16 * u) + (c0 + tx + 16 * v) * a.n, acc[u][v]);
    __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(kCholThreads) k_chol_ladder(CholArgs<T> a) {
    constexpr int TL = tile_of<T>();
    __shared__ T S1[TL][kB + 1];
    __shared__ T S2[TL][kB + 1];
    __shared__ int s_live;
    const int npanels = (int)((a.n + kB - 1) / kB);
    for (int k = 0; k < npanels; k++) {
        const int p0 = k * kB;
        // D: warp 0 of CTA c handles candidate c.
        if (blockIdx.x < (unsigned)a.nc && threadIdx.x < 32 && !__ldcg(a.fail + blockIdx.x))
            chol_diag_warp(a, blockIdx.x, p0);
        if (!grid_sync(a.gs)) return;
        const int64_t rows = a.n - p0 - kB;
        if (rows <= 0) break;
        // P: (candidate, row chunk) tasks.
        const int64_t chunks = (rows + kRowChunk - 1) / kRowChunk;
        for (int64_t t = blockIdx.x; t < chunks * a.nc; t += gridDim.x) {
            const int c = (int)(t / chunks);
            if (threadIdx.x == 0) s_live = !__ldcg(a.fail + c);
            __syncthreads();
            if (s_live)
                chol_panel_rows(a, c, p0, p0 + kB + (t % chunks) * kRowChunk, S1);
            __syncthreads();
        }
        if (!grid_sync(a.gs)) return;
        // U: (candidate, lower tile) tasks.
        const int64_t nt = (rows + TL - 1) / TL;
        const int64_t tiles = nt * (nt + 1) / 2;
        for (int64_t t = blockIdx.x; t < tiles * a.nc; t += gridDim.x) {
            const int c = (int)(t / tiles);
            const int64_t tt = t % tiles;
            int bi = (int)((sqrt(8.0 * (double)tt + 1.0) - 1.0) * 0.5);
            while ((int64_t)(bi + 1) * (bi + 2) / 2 <= tt) bi++;
            while ((int64_t)bi * (bi + 1) / 2 > tt) bi--;
            const int bj = (int)(tt - (int64_t)bi * (bi + 1) / 2);
            if (threadIdx.x == 0) s_live = !__ldcg(a.fail + c);
            __syncthreads();
            if (s_live) chol_update_tile(a, c, p0, bi, bj, S1, S2);
            __syncthreads();
        }
        if (!grid_sync(a.gs)) return;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        int s = -1;
        for (int c = 0; c < a.nc; c++)
            if (!__ldcg(a.fail + c)) {
                s = c;
                break;
            }
        a.sel[0] = s;
    }
}

// Candidates 0..nc-1 of the ladder: K with jit[c] added to the diagonal (exact T sum).  Only the
// lower triangle is written: nothing downstream reads the upper one.
template <typename T>
__global__ void k_ladder_assemble(TableView<T> tv, const uint32_t* __restrict__ coords, int D,
                                  int DS, T scale, int64_t n, const T* __restrict__ jit, int nc,
                                  T* __restrict__ base) {
    extern __shared__ __align__(16) unsigned char smem[];
    SmemTable<T> tab;
    tab.stage(tv, smem, threadIdx.x, blockDim.x);
    __syncthreads();
    const T diag = tab.lookup(T(0));
    const int64_t nn = n * n;
    for (int64_t j = blockIdx.x; j < n; j += gridDim.x) {
        for (int64_t i = j + threadIdx.x; i < n; i += blockDim.x) {
            if (i == j) {
                for (int c = 0; c < nc; c++)
                    base[c * nn + j * n + j] = jit[c] == T(0) ? diag : Num<T>::add(diag, jit[c]);
            } else {
                long long sq = 0;
                for (int d = 0; d < D; d++) {
                    const long long di =
                        (long long)coords[i * DS + d] - (long long)coords[j * DS + d];
                    sq += di * di;
                }
                const T r = Num<T>::mul(Num<T>::sqrt(Num<T>::from_i64(sq)), scale);
                const T v = tab.lookup(r);
                for (int c = 0; c < nc; c++) base[c * nn + j * n + i] = v;
            }
        }
    }
}

}  // namespace

template <typename T>
int dense_cholesky_ladder(gpb2_problem* p, cudaStream_t s) {
    const int64_t n = p->n0;
    const int ncand = 9;
    // The ladder's jitters, evaluated in T exactly as src/dense.jl:50-64 writes them.
    std::vector<T> jit(ncand, T(0)), epsv(ncand, T(0));
    int ncand_used = 1;
    {
        T dmean = T(0);
        const T v0 = (T)p->v0;  // every diagonal entry is cov_lookup(0)
        for (int64_t i = 0; i < n; i++) dmean = dmean + v0;
        dmean = dmean / (T)(n > 1 ? n : 1);
        for (T eps = T(1e-9); eps <= T(1e-2) && ncand_used < ncand; eps *= T(10)) {
            epsv[ncand_used] = eps;
            jit[ncand_used++] = eps * dmean;
        }
    }
    const bool spec = n <= kSpecMax;
    const int batch = spec ? ncand : 1;
    const size_t nn = (size_t)n * (size_t)n;
    GPB2_TRY(ensure_alloc(&p->Lcand, sizeof(T) * nn * batch));
    // lad: fail[16] | sel[1] (+pad) | barrier words[4] | jitters (T x 16)
    GPB2_TRY(ensure_alloc(reinterpret_cast<void**>(&p->lad), sizeof(int) * 32 + sizeof(T) * 16));
    int* fail = p->lad;
    int* sel = p->lad + 16;
    unsigned int* bar = reinterpret_cast<unsigned int*>(p->lad + 20);
    T* djit = reinterpret_cast<T*>(p->lad + 32);
    T* base = static_cast<T*>(p->Lcand);
    const size_t smem = table_smem_bytes<T>((int)p->nb, p->nkeys);
    GPB2_CUDA_TRY(prepare_kernel_smem((const void*)k_ladder_assemble<T>, smem));
    const int grid = coop_grid((const void*)k_chol_ladder<T>, kCholThreads, 0);

    for (int first = 0; first < ncand_used; first += batch) {
        const int nc = std::min(batch, ncand_used - first);
        GPB2_CUDA_TRY(cudaMemcpyAsync(djit, jit.data() + first, sizeof(T) * nc,
                                      cudaMemcpyHostToDevice, s));
        GPB2_CUDA_TRY(cudaMemsetAsync(p->lad, 0, sizeof(int) * 32, s));
        GPB2_CUDA_TRY(launch_prof("dense_assemble", k_ladder_assemble<T>,
                                  dim3((unsigned)std::min<int64_t>(n, 4 * 148)), dim3(256), smem,
                                  s, table_view<T>(p), (const uint32_t*)p->coords, (int)p->d,
                                  coord_stride((int)p->d), (T)p->scale, n, (const T*)djit, nc,
                                  base));
        CholArgs<T> args{base, n, nc, fail, sel, GridSync{bar, reinterpret_cast<int*>(bar + 2)}};
        void* argv[] = {&args};
        const ProfToken t = prof_begin("dense_chol", s);
        cudaError_t e = cudaLaunchCooperativeKernel((const void*)k_chol_ladder<T>, grid,
                                                    kCholThreads, argv, 0, s);
        prof_end(t, s);
        GPB2_CUDA_TRY(e);
        int h[8] = {-1, 0, 0, 0, 0, 0, 0, 0};
        GPB2_CUDA_TRY(cudaMemcpyAsync(h, sel, sizeof(int) * 8, cudaMemcpyDeviceToHost, s));
        GPB2_CUDA_TRY(cudaStreamSynchronize(s));
        if (h[6] != 0)  // error word of the barrier (lad[22])
            return set_error(GPB2_ERR_TIMEOUT, "dense factorisation barrier timed out");
        if (h[0] >= 0) {
            p->Ld = base + (size_t)h[0] * nn;
            p->dense_jitter = (double)epsv[first + h[0]];
            p->dense_candidate = first + h[0];
            return GPB2_OK;
        }
    }
    return set_error(GPB2_ERR_NOT_PD,
                     "dense first-layer covariance is not positive definite even with 1e-2 "
                     "relative jitter; increase the kernel `jitter` or reduce n0");
}

template int dense_cholesky_ladder<float>(gpb2_problem*, cudaStream_t);
template int dense_cholesky_ladder<double>(gpb2_problem*, cudaStream_t);

}  // namespace gpb2
