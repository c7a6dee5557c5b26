// gpb2_dense_chol.cu -- the dense block's Cholesky factorisation with the reference's jitter
// ladder (_dense_chol_L, src/dense.jl:46-67), one thread-block cluster per ladder candidate.
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
// Schedule: one thread-block cluster per candidate, phases separated by the cluster barrier; per
// 32-wide panel:
//   D  one warp of the cluster factors the 32 x 32 diagonal block, a row per lane;
//   P  256-row chunks over the cluster's CTAs: each thread solves one row below the block;
//   U  64 x 64 lower tiles over the cluster's CTAs: the trailing update with the panel's columns.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include <cooperative_groups.h>

#include "gpb2_problem.h"
#include "gpb2_sync.cuh"

namespace cg = cooperative_groups;

namespace gpb2 {

namespace {

constexpr int kB = 32;          // panel width (= warp size: a lane per row or column)
constexpr int kSpecMax = 4096;  // concurrent ladder up to this n0
constexpr int kGridMin = 2048;  // one candidate at a time on the whole GPU above this n0

template <typename T>
__host__ __device__ constexpr int chol_threads() { return 512; }

// Per-slot data of one ladder launch, passed by value as kernel arguments (no host-to-device
// copy per factorisation: such small copies would queue in the copy engine behind whatever
// large transfers the caller has in flight).
struct SlotOrder {
    int v[16];  // ladder index of slot c
};
template <typename T>
struct SlotJit {
    T v[16];  // jitter added to slot c's diagonal
};

template <typename T>
struct CholArgs {
    T* base;          // nc candidates, each n x n column-major (lower triangle)
    int64_t n;
    int nc;
    int first;        // ladder index of candidate 0 of this launch
    int* fail;        // fail[c] = failing column + 1 (or stop column + 1), 0 while alive
    int* sel;         // sel[0]: ladder index of the first success (-1: none yet); sel[1]: its slot
    int* done;        // done[c] = 1 once candidate c is fully factorised
    int* dflag;       // dflag[c]: last panel whose diagonal block candidate c has published
    int* err;         // error word: a bounded wait gave up
    int order[16];    // order[c]: ladder index of candidate slot c (a kernel argument)
    unsigned long long* trace;  // diagnostics (GPB2_TRACE_DENSE): phase timestamps, or NULL
    GridSync gs;      // whole-grid form: barrier words
    unsigned int* gctr;  // whole-grid form: the trailing-tile counters (by panel parity)
};

__device__ __forceinline__ void st_release_gpu(int* p, int v) {
    asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_gpu_s32(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Bounded wait until *flag >= v (one thread); on timeout the error word is set and the wait
// ends, so a failure elsewhere never hangs the cluster.
__device__ __forceinline__ void wait_flag_gpu(const int* flag, int v, int* err) {
    for (unsigned int it = 0; ld_acquire_gpu_s32(flag) < v; it++) {
        if ((it & 1023u) == 1023u && (it > (1u << 24) || ld_acquire_gpu_s32(err) != 0)) {
            atomicCAS(err, 0, 1);
            return;
        }
    }
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// x / d for d > 0, bit for bit as Num<T>::div.  A zero dividend gives a zero of its own sign;
// the division sequence reaches that case only through its slow path (several times the
// latency), and zeros are common here (padding rows, negligible covariances).
template <typename T>
__device__ __forceinline__ T div_pos(T x, T d) {
    const T q = Num<T>::div(x == T(0) ? T(1) : x, d);
    return x == T(0) ? x : q;
}

// Phase D (whole CTA): factor candidate c's diagonal block [p0, p0+bs)^2.  The CTA stages the
// block in shared memory in one coalesced pass (unless `staged`: the caller left it in S), warp 0
// eliminates it in registers, and the CTA writes it back.  Returns false (and records the
// column) if a pivot fails.
template <typename T>
__device__ __noinline__ bool chol_diag(const CholArgs<T>& a, int c, int64_t p0, T (*S)[kB + 1],
                                       int* s_bad, unsigned long long* st = nullptr,
                                       bool staged = false) {
    using N = Num<T>;
    constexpr int NTH = chol_threads<T>();
    T* L = a.base + (int64_t)c * a.n * a.n;
    const int bs = a.n - p0 < kB ? (int)(a.n - p0) : kB;
    if (!staged) {
#pragma unroll
        for (int e0 = 0; e0 < kB * kB; e0 += NTH) {
            const int e = e0 + threadIdx.x, i = e % kB, j = e / kB;
            if (i < bs && j <= i) S[i][j] = __ldcg(L + (p0 + i) + (p0 + j) * a.n);
        }
    }
    __syncthreads();
    if (st) st[0] = global_ns();
    if (threadIdx.x < 32) {
        // Row `lane` in registers; column j's pivot and multipliers travel by shuffle; finished
        // entries go to S.  Fully unrolled: about 500 update steps that follow the triangle, so
        // the serial chain (pivot -> sqrt -> divisions -> next pivot) has the issue slots to
        // itself.  Entries above the diagonal (lane < q) take meaningless values: they are never
        // a pivot, a multiplier or stored.
        const int lane = threadIdx.x;
        int bad = 0;
        T r[kB];
        sfor<0, kB>([&](auto q_) {
            GPB2_CI(q);
            r[q] = (lane < bs && q <= lane) ? S[lane][q] : T(0);
        });
        sfor<0, kB>([&](auto j_) {
            GPB2_CI(j);
            if (j < bs && !bad) {
                const T sjj = __shfl_sync(0xffffffffu, r[j], j);
                if (!(sjj > T(0))) {  // LAPACK potrf's failure test (also catches NaN)
                    bad = (int)p0 + j + 1;
                } else {
                    const T d = N::sqrt(sjj);
                    const T qv = div_pos(lane > j ? r[j] : T(1), d);  // branch-free
                    r[j] = lane == j ? d : qv;                         // L[lane][j], lane >= j
                    if (lane >= j) S[lane][j] = r[j];
                    sfor<j + 1, kB>([&](auto q_) {
                        GPB2_CI(q);
                        const T lqj = __shfl_sync(0xffffffffu, r[j], q);
                        r[q] = N::sub(r[q], N::mul(r[j], lqj));
                    });
                }
            }
        });
        if (lane == 0) {
            *s_bad = bad;
            if (bad) a.fail[c] = bad;
        }
    }
    __syncthreads();
    if (st) st[1] = global_ns();
    const bool ok = *s_bad == 0;
    if (ok) {
#pragma unroll
        for (int e0 = 0; e0 < kB * kB; e0 += NTH) {
            const int e = e0 + threadIdx.x, i = e % kB, j = e / kB;
            if (i < bs && j <= i) __stcg(L + (p0 + i) + (p0 + j) * a.n, S[i][j]);
        }
    }
    __syncthreads();
    return ok;
}

// Phase P (whole CTA): the rows below candidate c's diagonal block, X <- X * Dg^-T.  Rows go in
// 32-row blocks, block b to cluster rank b % CL and warp (b / CL) % NW, a row per lane (loads
// and stores along the contiguous dimension); each lane runs the forward substitution over its
// row in registers, column by column -- the oracle's order for each entry.
template <typename T>
__device__ void chol_panel(const CholArgs<T>& a, int c, int64_t p0, int rank, int CL,
                           T* Dg, unsigned long long* st = nullptr) {
    using N = Num<T>;
    constexpr int NTH = chol_threads<T>(), NW = NTH / 32;
    T* L = a.base + (int64_t)c * a.n * a.n;
    const int64_t r0 = p0 + kB;
    const int64_t nrb = (a.n - r0 + kB - 1) / kB;
    if (rank >= nrb) return;  // CTA-uniform
#pragma unroll
    for (int e0 = 0; e0 < kB * kB; e0 += NTH) {
        const int e = e0 + threadIdx.x, i = e % kB, j = e / kB;
        Dg[j * kB + i] = (i >= j) ? __ldcg(L + (p0 + i) + (p0 + j) * a.n) : T(0);
    }
    if (threadIdx.x < kB) Dg[kB * kB + threadIdx.x] = T(0);
    __syncthreads();
    if (st) st[0] = global_ns();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int64_t b = rank + (int64_t)CL * warp; b < nrb; b += (int64_t)CL * NW) {
        const int64_t i = r0 + b * kB + lane;
        const bool live = i < a.n;
        T* Li = L + i + p0 * a.n;
        // Fully unrolled (unlike the diagonal block: many warps run this code, and the unrolled
        // form lets column j+1's division start while column j's updates are in flight).
        T x[kB];
        sfor<0, kB>([&](auto q_) {
            GPB2_CI(q);
            x[q] = live ? __ldcg(Li + q * a.n) : T(0);
        });
        sfor<0, kB>([&](auto j_) {
            GPB2_CI(j);
            const T* dj = Dg + j * kB;  // dj[q] = L[p0 + q][p0 + j]
            x[j] = div_pos(x[j], dj[j]);
            sfor<j + 1, kB>([&](auto q_) {
                GPB2_CI(q);
                x[q] = N::sub(x[q], N::mul(x[j], dj[q]));
            });
        });
        if (live) {
            sfor<0, kB>([&](auto q_) {
                GPB2_CI(q);
                __stcg(Li + q * a.n, x[q]);
            });
        }
    }
    __syncthreads();
    if (st) st[1] = global_ns();
}

// The panel's diagonal factor, transposed, into Dg (whole CTA; row j = column j of the factor,
// zero above the diagonal, plus a zero row).
template <typename T>
__device__ __forceinline__ void load_diag_t(const CholArgs<T>& a, int c, int64_t p0, T* Dg) {
    constexpr int NTH = chol_threads<T>();
    const T* L = a.base + (int64_t)c * a.n * a.n;
#pragma unroll
    for (int e0 = 0; e0 < kB * kB; e0 += NTH) {
        const int e = e0 + threadIdx.x, i = e % kB, j = e / kB;
        Dg[j * kB + i] = (i >= j && p0 + i < a.n) ? __ldcg(L + (p0 + i) + (p0 + j) * a.n) : T(0);
    }
    if (threadIdx.x < kB) Dg[kB * kB + threadIdx.x] = T(0);
}

// Panel rows [r_lo, r_hi) (at most one tile: warp w takes rows r_lo + 32w + lane) solved against
// the transposed diagonal factor Dg, as in chol_panel.  With Sr the rows come from shared memory
// (row i at Sr[i - p0], as the tile holding them left them) instead of global memory.
template <typename T>
__device__ void chol_rows(const CholArgs<T>& a, int c, int64_t p0, int64_t r_lo, int64_t r_hi,
                          const T* Dg, const T (*Sr)[kB + 1] = nullptr) {
    using N = Num<T>;
    T* L = a.base + (int64_t)c * a.n * a.n;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if ((int64_t)warp * 32 >= r_hi - r_lo) return;  // warp-uniform
    const int64_t i = r_lo + warp * 32 + lane;
    const bool live = i < r_hi;
    T* Li = L + i + p0 * a.n;
    T x[kB];
    if (Sr) {
        sfor<0, kB>([&](auto q_) {
            GPB2_CI(q);
            x[q] = live ? Sr[i - p0][q] : T(0);
        });
    } else {
        sfor<0, kB>([&](auto q_) {
            GPB2_CI(q);
            x[q] = live ? __ldcg(Li + q * a.n) : T(0);
        });
    }
    sfor<0, kB>([&](auto j_) {
        GPB2_CI(j);
        const T* dj = Dg + j * kB;
        x[j] = div_pos(x[j], dj[j]);
        sfor<j + 1, kB>([&](auto q_) {
            GPB2_CI(q);
            x[q] = N::sub(x[q], N::mul(x[j], dj[q]));
        });
    });
    if (live) {
        sfor<0, kB>([&](auto q_) {
            GPB2_CI(q);
            __stcg(Li + q * a.n, x[q]);
        });
    }
}

// Packed single-precision pairs: mul.rn.f32x2 rounds each lane exactly as __fmul_rn does
// (denormals included).  The subtraction stays scalar: a packed multiply whose only use is a
// packed subtraction is contracted into a fused multiply-add by the code generator, which would
// round once instead of twice.
__device__ __forceinline__ unsigned long long pk2(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void upk2(unsigned long long v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long mul2_rn(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// Phase U: lower tile (bi, bj) of candidate c's trailing matrix [p0 + kB, n)^2, one subtraction
// per panel column in order.  Thread (tx, ty) owns rows tx + 32*u (lanes along the contiguous
// dimension) and RV columns col(v): ty + TY*v, or in single precision adjacent pairs
// 2*ty + 2*TY*w + {0, 1}, updated as packed pairs.  A tile's operands are fetched into
// registers (fetch) while the previous tile computes, then staged in shared memory (stage) and
// consumed (compute).
template <typename T, int TL>
struct TileWork {
    static constexpr int NTH = chol_threads<T>();
    static constexpr int TY = NTH / 32;
    static constexpr int RU = TL / 32, RV = TL / TY;
    static constexpr int NP = TL * kB / NTH;  // panel entries per thread per side
    static constexpr bool kPair = sizeof(T) == 4;
    static_assert(RU * 32 == TL && RV * TY == TL && NP * NTH == TL * kB, "tile shape");
    static_assert(!kPair || RV % 2 == 0, "column pairs");
    T li[NP], lj[NP];
    T acc[RU][RV];
    int64_t r0, c0;

    // After compute() and a barrier: the tile's first kB columns into S[row][col] (the diagonal
    // block and the rows below it of tile (0, 0), as chol_diag and chol_rows read them).
    __device__ __forceinline__ void stash_first_cols(T (*S)[kB + 1]) const {
        const int tx = threadIdx.x % 32;
#pragma unroll
        for (int u = 0; u < RU; u++)
#pragma unroll
            for (int v = 0; v < RV; v++)
                if (col(v) < kB) S[tx + 32 * u][col(v)] = acc[u][v];
    }
    static __device__ __forceinline__ int col(int v) {
        const int ty = threadIdx.x / 32;
        return kPair ? 2 * ty + 2 * TY * (v / 2) + (v % 2) : ty + TY * v;
    }

    __device__ __forceinline__ void fetch(const CholArgs<T>& a, int c, int64_t p0, int bi,
                                          int bj) {
        const T* L = a.base + (int64_t)c * a.n * a.n;
        const int64_t t0 = p0 + kB;
        r0 = t0 + (int64_t)bi * TL;
        c0 = t0 + (int64_t)bj * TL;
#pragma unroll
        for (int q = 0; q < NP; q++) {
            const int e = q * NTH + threadIdx.x, rr = e % TL, pp = e / TL;
            const int64_t gi = r0 + rr, gj = c0 + rr;
            li[q] = gi < a.n ? __ldcg(L + gi + (p0 + pp) * a.n) : T(0);
            lj[q] = gj < a.n ? __ldcg(L + gj + (p0 + pp) * a.n) : T(0);
        }
        const int tx = threadIdx.x % 32;
#pragma unroll
        for (int u = 0; u < RU; u++)
#pragma unroll
            for (int v = 0; v < RV; v++) {
                const int64_t gi = r0 + tx + 32 * u, gj = c0 + col(v);
                acc[u][v] = (gi < a.n && gi >= gj) ? __ldcg(L + gi + gj * a.n) : T(0);
            }
    }
    // Li[rr][pp] = L[r0 + rr][p0 + pp]; the column side likewise, or in single precision
    // transposed (LjT[pp * TL + rr]) so that a column pair is one 8-byte load.
    __device__ __forceinline__ void stage(T (*Li)[kB + 1], T (*Lj)[kB + 1]) const {
        T* LjT = &Lj[0][0];
#pragma unroll
        for (int q = 0; q < NP; q++) {
            const int e = q * NTH + threadIdx.x, rr = e % TL, pp = e / TL;
            Li[rr][pp] = li[q];
            if constexpr (kPair)
                LjT[pp * TL + rr] = lj[q];
            else
                Lj[rr][pp] = lj[q];
        }
    }
    // After stage() and a barrier: subtract the panel's products and store the tile.
    __device__ __forceinline__ void compute(const CholArgs<T>& a, int c, T (*Li)[kB + 1],
                                            T (*Lj)[kB + 1]) {
        using N = Num<T>;
        T* L = a.base + (int64_t)c * a.n * a.n;
        const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;
        if constexpr (kPair) {
            const float* LjT = reinterpret_cast<const float*>(&Lj[0][0]);
#pragma unroll 4
            for (int p = 0; p < kB; p++) {
                unsigned long long xb[RU], xj[RV / 2];
#pragma unroll
                for (int u = 0; u < RU; u++) {
                    const float x = Li[tx + 32 * u][p];
                    xb[u] = pk2(x, x);
                }
#pragma unroll
                for (int w = 0; w < RV / 2; w++)
                    xj[w] = *reinterpret_cast<const unsigned long long*>(LjT + p * TL + 2 * ty +
                                                                         2 * TY * w);
#pragma unroll
                for (int u = 0; u < RU; u++)
#pragma unroll
                    for (int w = 0; w < RV / 2; w++) {
                        float plo, phi;
                        upk2(mul2_rn(xb[u], xj[w]), plo, phi);
                        acc[u][2 * w] = N::sub(acc[u][2 * w], plo);
                        acc[u][2 * w + 1] = N::sub(acc[u][2 * w + 1], phi);
                    }
            }
        } else {
#pragma unroll 4
            for (int p = 0; p < kB; p++) {
                T xi[RU], xj[RV];
#pragma unroll
                for (int u = 0; u < RU; u++) xi[u] = Li[tx + 32 * u][p];
#pragma unroll
                for (int v = 0; v < RV; v++) xj[v] = Lj[ty + TY * v][p];
#pragma unroll
                for (int u = 0; u < RU; u++)
#pragma unroll
                    for (int v = 0; v < RV; v++)
                        acc[u][v] = N::sub(acc[u][v], N::mul(xi[u], xj[v]));
            }
        }
#pragma unroll
        for (int u = 0; u < RU; u++)
#pragma unroll
            for (int v = 0; v < RV; v++) {
                const int64_t gi = r0 + tx + 32 * u, gj = c0 + col(v);
                if (gi < a.n && gi >= gj) __stcg(L + gi + gj * a.n, acc[u][v]);
            }
    }
};

// Tile index t of panel k's trailing matrix (nt x nt tiles, lower triangle) -> (bi, bj): tile
// 0 is (0, 0); then the inner triangle (bj >= 1); the first tile column last.
__device__ __forceinline__ void tile_of_index(unsigned int t, int64_t nt, int& bi, int& bj) {
    const unsigned int inner = (unsigned int)((nt - 1) * nt / 2);
    if (t == 0) {
        bi = bj = 0;
    } else if (t - 1 < inner) {
        const int64_t u = t - 1;
        int q = (int)((sqrt(8.0 * (double)u + 1.0) - 1.0) * 0.5);
        while ((int64_t)(q + 1) * (q + 2) / 2 <= u) q++;
        while ((int64_t)q * (q + 1) / 2 > u) q--;
        bi = q + 1;
        bj = (int)(u - (int64_t)q * (q + 1) / 2) + 1;
    } else {
        bi = (int)(t - inner);
        bj = 0;
    }
}

// Whether candidate c stops before the panel whose trailing block starts at column `lim`.  Rank 0
// records a stop (a failed pivot, or a supersede) as that column + 1 while other CTAs may still
// be reading the word for the previous panel; filtering by column makes every thread of the
// cluster take the same decision after the same barrier, so they all leave together.
template <class T>
__device__ __forceinline__ bool chol_stopped(const CholArgs<T>& a, int c, int64_t lim) {
    const int f = __ldcg(a.fail + c);
    return f != 0 && (int64_t)f - 1 < lim;
}

// One group of CTAs per ladder candidate.  kGrid = false: a thread-block cluster per candidate,
// its CTAs meeting at the hardware cluster barrier (release/acquire at cluster scope), so
// candidates proceed independently (the concurrent ladder of blocks up to a few thousand).
// kGrid = true: one candidate per cooperative launch on every SM, meeting at the bounded grid
// barrier (the first layers of the 1e8 / 1e9-point configurations, where one factorisation
// has enough tiles for the whole GPU).  One barrier per panel: rank 0 updates tile (0, 0) --
// which holds the next diagonal block -- factors that block, publishes it and solves the tile's
// rows below it; the other CTAs take the remaining trailing tiles from an atomic counter (in
// rank 0's shared memory, or in global memory for the grid), the tiles of the first tile column
// (which hold the next panel's rows) last, and whoever updates one of those then solves its rows
// against the published block.  At the barrier the next panel is final.
template <typename T, int TL, bool kGrid>
__global__ void __launch_bounds__(chol_threads<T>()) k_chol_cluster(CholArgs<T> a) {
    __shared__ __align__(16) T S[2 * TL][kB + 1];
    __shared__ __align__(16) T Dg[(kB + 1) * kB];
    __shared__ int s_bad;
    __shared__ unsigned int s_ctr[2];   // rank 0: next trailing tile (by panel parity)
    __shared__ unsigned int s_next[2];  // this CTA's next tile (double-buffered)
    __shared__ int s_dg;                // panel whose diagonal factor Dg holds (-1: none)
    int CL, rank, c;
    if constexpr (kGrid) {
        CL = (int)gridDim.x;
        rank = (int)blockIdx.x;
        c = 0;
    } else {
        cg::cluster_group cl = cg::this_cluster();
        CL = (int)cl.num_blocks();
        rank = (int)cl.block_rank();
        c = (int)(blockIdx.x / CL);
    }
    // The group's barrier; false when the grid form's bounded wait gave up (its error word is
    // set and every CTA leaves).
    auto group_sync = [&]() -> bool {
        if constexpr (kGrid) {
            return grid_sync(a.gs);
        } else {
            cg::this_cluster().sync();
            return true;
        }
    };
    auto tile_counter = [&](int parity) -> unsigned int* {
        if constexpr (kGrid)
            return a.gctr + parity;
        else
            return cg::this_cluster().map_shared_rank(&s_ctr[parity], 0);
    };
    // A previous launch of the ladder already succeeded (sel is only written between launches).
    if (__ldcg(a.sel) >= 0) return;
    const int npanels = (int)((a.n + kB - 1) / kB);
    int* dflag = a.dflag + c;  // last panel whose diagonal block is published
    unsigned long long* tr =
        (a.trace && c == a.nc - 1 && rank == 0 && threadIdx.x == 0) ? a.trace : nullptr;
    // Diagnostics: each candidate's start and end times and how it ended, after the panel trace.
    unsigned long long* life =
        (a.trace && rank == 0 && threadIdx.x == 0) ? a.trace + 8 * npanels + 3 * c : nullptr;
    if (life) life[0] = global_ns();
    auto leave = [&](unsigned long long how) {
        if (life) {
            life[1] = global_ns();
            life[2] = how;
        }
    };
    if (threadIdx.x == 0) {
        s_ctr[0] = 1u;  // tile 0 of every panel is rank 0's
        s_ctr[1] = 1u;
        s_dg = -1;
        if (kGrid && rank == 0) {
            a.gctr[0] = 1u;
            a.gctr[1] = 1u;
        }
    }
    // Panel 0: its diagonal block, then its rows.
    if (rank == 0) chol_diag(a, c, 0, S, &s_bad);
    if (!group_sync()) return leave(3000);
    if (chol_stopped(a, c, kB)) return leave(1);
    chol_panel<T>(a, c, 0, rank, CL, Dg, nullptr);
    if (!group_sync()) return leave(3000);
    for (int k = 0; k < npanels; k++) {
        const int64_t p0 = (int64_t)k * kB;
        unsigned long long* st = tr ? tr + 8 * k : nullptr;
        if (st) st[0] = global_ns();
        if (chol_stopped(a, c, p0 + kB)) return leave(2 + k);  // the whole cluster leaves together
        const int64_t rows = a.n - p0 - kB;
        if (rows <= 0) break;
        const int64_t t0 = p0 + kB;        // trailing matrix [t0, n)^2
        const int64_t nt = (rows + TL - 1) / TL;
        const unsigned int tiles = (unsigned int)(nt * (nt + 1) / 2);
        const unsigned int inner = (unsigned int)((nt - 1) * nt / 2);  // tiles with bj >= 1
        unsigned int* ctr = tile_counter(k & 1);
        unsigned int t = 0u;
        if (rank != 0) {
            if (threadIdx.x == 0) s_next[0] = atomicAdd(ctr, 1u);
            __syncthreads();
            t = s_next[0];
        }
        TileWork<T, TL> cur;
        int bi = 0, bj = 0;
        if (t < tiles) {
            tile_of_index(t, nt, bi, bj);
            cur.fetch(a, c, p0, bi, bj);
        }
        // Rank 0 takes only tile 0 (then the diagonal block and its rows: the critical path);
        // the other CTAs share every other tile.  Each tile's successor is fetched into
        // registers while the tile computes.
        for (int it = 1; t < tiles; it++) {
            if (threadIdx.x == 0) s_next[it & 1] = rank == 0 ? tiles : atomicAdd(ctr, 1u);
            cur.stage(S, S + TL);
            __syncthreads();
            const unsigned int tn = s_next[it & 1];
            int bin = 0, bjn = 0;
            TileWork<T, TL> nxt;
            if (tn < tiles) {
                tile_of_index(tn, nt, bin, bjn);
                nxt.fetch(a, c, p0, bin, bjn);
            }
            cur.compute(a, c, S, S + TL);
            __syncthreads();
            if (t == 0) {  // the next diagonal block is final: factorise it and publish it
                if (st) st[4] = global_ns();
                cur.stash_first_cols(S);  // block and rows straight from registers
                chol_diag(a, c, t0, S, &s_bad, st ? st + 5 : nullptr, true);  // ends with a barrier
                if (threadIdx.x == 0) {
                    __threadfence();
                    st_release_gpu(dflag, k + 1);  // published even on failure: waiters go on
                }
                // This CTA's copy of the block, transposed, straight from shared memory.
                for (int e = threadIdx.x; e < kB * kB; e += chol_threads<T>()) {
                    const int i = e % kB, j = e / kB;
                    Dg[j * kB + i] = (i >= j && t0 + i < a.n) ? S[i][j] : T(0);
                }
                if (threadIdx.x < kB) Dg[kB * kB + threadIdx.x] = T(0);
                __syncthreads();
                if (threadIdx.x == 0) s_dg = k + 1;
                __syncthreads();
            }
            if (bj == 0) {  // rows of the next panel in this tile: solve them
                const int64_t r_lo = t0 + (int64_t)bi * TL > t0 + kB ? t0 + (int64_t)bi * TL : t0 + kB;
                const int64_t r_hi = t0 + (int64_t)(bi + 1) * TL < a.n ? t0 + (int64_t)(bi + 1) * TL : a.n;
                if (r_lo < r_hi) {
                    if (s_dg != k + 1) {
                        if (threadIdx.x == 0) wait_flag_gpu(dflag, k + 1, a.err);
                        __syncthreads();
                        load_diag_t(a, c, t0, Dg);
                        __syncthreads();
                        if (threadIdx.x == 0) s_dg = k + 1;
                    }
                    chol_rows(a, c, t0, r_lo, r_hi, Dg, t == 0 ? S : nullptr);
                    __syncthreads();
                }
            }
            cur = nxt;
            t = tn;
            bi = bin;
            bj = bjn;
        }
        if (rank == 0 && threadIdx.x == 0) {
            s_ctr[(k + 1) & 1] = 1u;  // the next panel's counter
            if (kGrid) a.gctr[(k + 1) & 1] = 1u;
            // Superseded: a smaller ladder step has already factorised, so this candidate can no
            // longer be selected -- stop (after the barrier, with the whole cluster) and free its
            // SMs for candidates still waiting for a slot.
            bool sup = false;
            for (int c2 = 0; c2 < a.nc; c2++)
                sup = sup || (a.order[c2] < a.order[c] && __ldcg(a.done + c2));
            if (sup && !__ldcg(a.fail + c)) a.fail[c] = (int)(p0 + kB) + 1;
        }
        if (st) st[7] = global_ns();
        if (!group_sync()) return leave(3000);
    }
    if (rank == 0 && threadIdx.x == 0 && !__ldcg(a.fail + c)) a.done[c] = 1;
    leave(1000);
}

// After a launch: record the first candidate (in ladder order) that factorised, unless an
// earlier launch already did.
__global__ void k_ladder_mark(const int* __restrict__ done, SlotOrder order, int nc,
                              int* __restrict__ sel) {
    if (sel[0] >= 0) return;
    int best = -1;
    for (int c = 0; c < nc; c++)  // the smallest ladder index that factorised
        if (done[c] && (best < 0 || order.v[c] < order.v[best])) best = c;
    if (best >= 0) {
        sel[0] = order.v[best];
        sel[1] = best;
    }
}

// Copy the selected candidate into the fixed factor buffer (the triangular products and solves
// downstream read it there); with no success the status word records it and the call fails.
template <typename T>
__global__ void k_ladder_pick(const T* __restrict__ base, const int* __restrict__ sel,
                              int64_t nn, T* __restrict__ L, int* __restrict__ status) {
    const int s = __ldcg(sel + 1);
    if (__ldcg(sel) < 0) {
        if (blockIdx.x == 0 && threadIdx.x == 0) *status = 1;
        return;
    }
    const T* src = base + (int64_t)s * nn;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nn;
         i += (int64_t)gridDim.x * blockDim.x)
        L[i] = src[i];
}

// Candidates 0..nc-1 of the ladder: K with jit[c] added to the diagonal (exact T sum).  Only the
// lower triangle is written: nothing downstream reads the upper one.
template <typename T>
__global__ void k_ladder_assemble(TableView<T> tv, AnisoView<T> av,
                                  const uint32_t* __restrict__ coords, int D, int DS, T scale,
                                  int64_t n, SlotJit<T> jit, int nc, T* __restrict__ base,
                                  const int* __restrict__ sel) {
    // A later launch of the ladder must not overwrite the slots once a candidate is selected.
    if (__ldcg(sel) >= 0) return;
    extern __shared__ __align__(16) unsigned char smem[];
    SmemTable<T> tab;
    tab.stage(tv, smem, threadIdx.x, blockDim.x);
    __syncthreads();
    // An anisotropic covariance (av.grid set) replaces the table (_assemble_dense_cov_aniso,
    // src/aniso.jl:218-244).
    const T diag = av.grid ? av.lookup(T(0), T(0)) : tab.lookup(T(0));
    const int64_t nn = n * n;
    for (int64_t j = blockIdx.x; j < n; j += gridDim.x) {
        for (int64_t i = j + threadIdx.x; i < n; i += blockDim.x) {
            if (i == j) {
                for (int c = 0; c < nc; c++)
                    base[c * nn + j * n + j] =
                        jit.v[c] == T(0) ? diag : Num<T>::add(diag, jit.v[c]);
            } else if (av.grid) {
                const T v = av.pair_rt(coords + i * DS, coords + j * DS, D, scale);
                for (int c = 0; c < nc; c++) base[c * nn + j * n + i] = v;
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

// Largest cluster (16 with the non-portable opt-in, else 8, 4, ...) the factorisation kernel can
// be resident with; decided once per precision.
template <typename T, int TL>
int cluster_size() {
    static const int cs = [] {
        cudaFuncSetAttribute((const void*)k_chol_cluster<T, TL, false>,
                             cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        for (int c = 16; c >= 1; c /= 2) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)c);
            cfg.blockDim = dim3(chol_threads<T>());
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = (unsigned)c;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int nclusters = 0;
            if (cudaOccupancyMaxActiveClusters(&nclusters, (const void*)k_chol_cluster<T, TL, false>, &cfg) ==
                    cudaSuccess &&
                nclusters > 0)
                return c;
            cudaGetLastError();
        }
        return 0;
    }();
    return cs;
}

}  // namespace

// Large first layers: the ladder's candidates one at a time in ladder order, each factorised by
// the whole GPU (the grid form of k_chol_cluster, a cooperative launch) directly in the factor
// buffer; once one succeeds the later launches return at once (they read the selection first),
// so the usual case -- K itself factorises -- costs one factorisation and a few empty launches.
template <typename T>
int ladder_grid(gpb2_problem* p, cudaStream_t s, const std::vector<T>& jit, int ncand_used) {
    const int64_t n = p->n0;
    const size_t nn = (size_t)n * (size_t)n;
    GPB2_TRY(ensure_alloc(&p->Ld, sizeof(T) * nn));
    GPB2_TRY(ensure_alloc(reinterpret_cast<void**>(&p->lad), sizeof(int) * kLadInts + sizeof(T) * 16));
    int* sel = p->lad + kLadSel;
    T* base = static_cast<T*>(p->Ld);
    const size_t smem = table_smem_bytes<T>((int)p->nb, p->nkeys);
    GPB2_CUDA_TRY(prepare_kernel_smem((const void*)k_ladder_assemble<T>, smem));
    constexpr int kTile = sizeof(T) == 4 ? 128 : 64;
    void (*kern)(CholArgs<T>) = k_chol_cluster<T, kTile, true>;
    const int grid = coop_grid((const void*)kern, chol_threads<T>(), 0);
    if (grid <= 0) return set_error(GPB2_ERR_CUDA, "no resident grid for the dense factorisation");
    GPB2_CUDA_TRY(cudaMemsetAsync(p->lad, 0, sizeof(int) * kLadInts, s));
    GPB2_CUDA_TRY(cudaMemsetAsync(sel, 0xff, sizeof(int) * 2, s));
    for (int c = 0; c < ncand_used; c++) {
        // Per-candidate words (slot 0): failure column, completion, published panel, barrier.
        GPB2_CUDA_TRY(cudaMemsetAsync(p->lad + kLadFail, 0, sizeof(int), s));
        GPB2_CUDA_TRY(cudaMemsetAsync(p->lad + kLadDone, 0, sizeof(int), s));
        GPB2_CUDA_TRY(cudaMemsetAsync(p->lad + kLadDflag, 0, sizeof(int), s));
        GPB2_CUDA_TRY(cudaMemsetAsync(p->lad + kLadGridBar, 0, sizeof(int), s));
        SlotJit<T> sj{};
        sj.v[0] = jit[c];
        GPB2_CUDA_TRY(launch_prof("dense_assemble", k_ladder_assemble<T>,
                                  dim3((unsigned)std::min<int64_t>(n, 4 * 148)), dim3(256), smem,
                                  s, table_view<T>(p), aniso_view<T>(p),
                                  (const uint32_t*)p->coords, (int)p->d,
                                  coord_stride((int)p->d), (T)p->scale, n, sj, 1, base,
                                  (const int*)sel));
        CholArgs<T> args{base, n, 1, c, p->lad + kLadFail, sel, p->lad + kLadDone,
                         p->lad + kLadDflag, p->lad + kLadBarErr, {}, nullptr,
                         GridSync{reinterpret_cast<unsigned int*>(p->lad + kLadGridBar),
                                  p->lad + kLadBarErr},
                         reinterpret_cast<unsigned int*>(p->lad + kLadGridCtr)};
        args.order[0] = c;
        void* argv[] = {(void*)&args};
        const ProfToken t = prof_begin("dense_chol", s);
        const cudaError_t e = cudaLaunchCooperativeKernel((const void*)kern, grid,
                                                          chol_threads<T>(), argv, 0, s);
        prof_end(t, s);
        GPB2_CUDA_TRY(e);
        SlotOrder so{};
        so.v[0] = c;
        GPB2_CUDA_TRY(launch_prof("dense_mark", k_ladder_mark, dim3(1), dim3(1), 0, s,
                                  (const int*)(p->lad + kLadDone), so, 1, sel));
    }
    // No candidate factorised: the status word records it (the pick kernel copies nothing else:
    // the factor already sits in its buffer).
    GPB2_CUDA_TRY(launch_prof("dense_pick", k_ladder_pick<T>, dim3(1), dim3(32), 0, s,
                              (const T*)base, (const int*)sel, (int64_t)0,
                              static_cast<T*>(p->Ld), p->lad + kLadNotPD));
    return GPB2_OK;
}

template <typename T>
int dense_cholesky_ladder(gpb2_problem* p, cudaStream_t s) {
    const int64_t n = p->n0;
    const int ncand = 9;
    // The ladder's jitters, evaluated in T exactly as src/dense.jl:50-64 writes them.
    std::vector<T> jit(ncand, T(0)), epsv(ncand, T(0));
    int ncand_used = 1;
    {
        T dmean = T(0);
        // every diagonal entry is cov_lookup(0) (aniso_lookup(0, 0) for an anisotropic model)
        const T v0 = (T)(p->an_grid ? p->an_diag : p->v0);
        for (int64_t i = 0; i < n; i++) dmean = dmean + v0;
        dmean = dmean / (T)(n > 1 ? n : 1);
        for (T eps = T(1e-9); eps <= T(1e-2) && ncand_used < ncand; eps *= T(10)) {
            epsv[ncand_used] = eps;
            jit[ncand_used++] = eps * dmean;
        }
    }
    // Whole-GPU factorisation above this size (GPB2_DENSE_GRID_MIN overrides it).
    int64_t grid_min = kGridMin;
    if (const char* e = std::getenv("GPB2_DENSE_GRID_MIN")) grid_min = std::atoll(e);
    if (n > grid_min) {
        GPB2_TRY(ladder_grid<T>(p, s, jit, ncand_used));
        p->ladder_eps.assign(epsv.begin(), epsv.begin() + ncand_used);
        p->dense_pending = true;  // outcome checked by the call's finishing synchronisation
        p->dense_launched = true;
        return GPB2_OK;
    }
    int64_t spec_max = kSpecMax;  // GPB2_DENSE_SPEC_MAX overrides it (tests: force sequential)
    if (const char* e = std::getenv("GPB2_DENSE_SPEC_MAX")) spec_max = std::atoll(e);
    const bool spec = n <= spec_max;
    const int batch = spec ? ncand : 1;
    const size_t nn = (size_t)n * (size_t)n;
    GPB2_TRY(ensure_capacity(&p->Lcand, &p->lcand_bytes, sizeof(T) * nn * batch));
    GPB2_TRY(ensure_alloc(&p->Ld, sizeof(T) * nn));
    GPB2_TRY(ensure_alloc(reinterpret_cast<void**>(&p->lad), sizeof(int) * kLadInts + sizeof(T) * 16));
    int* fail = p->lad + kLadFail;
    int* done = p->lad + kLadDone;
    int* sel = p->lad + kLadSel;
    T* base = static_cast<T*>(p->Lcand);
    const size_t smem = table_smem_bytes<T>((int)p->nb, p->nkeys);
    GPB2_CUDA_TRY(prepare_kernel_smem((const void*)k_ladder_assemble<T>, smem));
    // Trailing-update tile: the small one balances the cluster's CTAs better on small blocks.
    constexpr int kTileS = sizeof(T) == 4 ? 64 : 32, kTileL = 2 * kTileS;
    int tile = n <= 2048 ? kTileS : kTileL;
    if (const char* e = std::getenv("GPB2_CHOL_TILE")) tile = std::atoi(e) == kTileL ? kTileL : kTileS;
    void (*kern)(CholArgs<T>) =
        tile == kTileS ? k_chol_cluster<T, kTileS, false> : k_chol_cluster<T, kTileL, false>;
    const int csize = tile == kTileS ? cluster_size<T, kTileS>() : cluster_size<T, kTileL>();
    if (csize <= 0) return set_error(GPB2_ERR_CUDA, "no thread-block cluster shape fits");

    // Fresh status: no selection (-1), no failure or completion flags, no error.
    GPB2_CUDA_TRY(cudaMemsetAsync(p->lad, 0, sizeof(int) * kLadInts, s));
    GPB2_CUDA_TRY(cudaMemsetAsync(sel, 0xff, sizeof(int) * 2, s));
    // Candidate slots in launch order.  Only some clusters are resident at once; the rest start
    // as slots free up.  A speculative launch starts with the ladder step that succeeded last
    // time (it runs to the end), then the smaller steps, which must all be seen to fail and fail
    // sooner the smaller they are, and last the larger steps, needed only if the hint fails and
    // otherwise superseded as soon as it completes.  Every slot is still examined, so the first
    // success in ladder order is selected whatever the order.  Sequential launches keep ladder
    // order.
    std::vector<int> order;
    order.reserve(ncand_used);
    const bool hinted = spec && p->ladder_hint >= 0 && p->ladder_hint < ncand_used;
    const int hint = hinted ? p->ladder_hint : 0;
    if (spec && !hinted) {
        // No hint yet: step 0 first (a well-conditioned block needs no jitter, and its success
        // supersedes every other candidate), then the largest steps down, so that whichever
        // step succeeds is among the resident clusters while the small ones, which fail early,
        // wait for a slot.
        order.push_back(0);
        for (int i = ncand_used - 1; i >= 1; i--) order.push_back(i);
    } else {
        for (int i = hint; i >= 0; i--) order.push_back(i);
        for (int i = hint + 1; i < ncand_used; i++) order.push_back(i);
    }
    std::vector<T> jit_slot(ncand_used);
    for (int i = 0; i < ncand_used; i++) jit_slot[i] = jit[order[i]];
    auto slot_jit = [&](int first, int nc) {
        SlotJit<T> j{};
        for (int c = 0; c < nc; c++) j.v[c] = jit_slot[first + c];
        return j;
    };
    auto slot_order = [&](int first, int nc) {
        SlotOrder o{};
        for (int c = 0; c < nc; c++) o.v[c] = order[first + c];
        return o;
    };
    // Launches: one candidate each (sequential), or all at once (speculative) -- except that
    // with a hint the steps above it get a second launch, which does nothing (every CTA returns
    // at once) when the hint or a step below it succeeded: they would only have competed with
    // the hinted candidate for the L2 and the cluster slots.
    std::vector<std::pair<int, int>> launches;  // (first slot, candidates)
    if (!spec) {
        for (int f = 0; f < ncand_used; f++) launches.push_back({f, 1});
    } else if (hinted && hint + 1 < ncand_used) {
        launches.push_back({0, hint + 1});
        launches.push_back({hint + 1, ncand_used - hint - 1});
    } else {
        launches.push_back({0, ncand_used});
    }
    for (const auto& ln : launches) {
        const int first = ln.first, nc = ln.second;
        if (first > 0) {
            GPB2_CUDA_TRY(cudaMemsetAsync(fail, 0, sizeof(int) * 16, s));
            GPB2_CUDA_TRY(cudaMemsetAsync(done, 0, sizeof(int) * 16, s));
            GPB2_CUDA_TRY(cudaMemsetAsync(p->lad + kLadDflag, 0, sizeof(int) * 16, s));
        }
        GPB2_CUDA_TRY(launch_prof("dense_assemble", k_ladder_assemble<T>,
                                  dim3((unsigned)std::min<int64_t>(n, 4 * 148)), dim3(256), smem,
                                  s, table_view<T>(p), aniso_view<T>(p),
                                  (const uint32_t*)p->coords, (int)p->d,
                                  coord_stride((int)p->d), (T)p->scale, n,
                                  slot_jit(first, nc), nc, base, (const int*)sel));
        unsigned long long* trace = nullptr;
        const int npan = (int)((n + kB - 1) / kB);
        if (std::getenv("GPB2_TRACE_DENSE")) {
            const size_t tn = 8 * (size_t)npan + 3 * 16;
            GPB2_TRY(ensure_alloc(&p->trace, sizeof(unsigned long long) * tn));
            GPB2_CUDA_TRY(cudaMemsetAsync(p->trace, 0, sizeof(unsigned long long) * tn, s));
            trace = static_cast<unsigned long long*>(p->trace);
        }
        CholArgs<T> args{base,  n,    nc,   first, fail, sel, done, p->lad + kLadDflag,
                         p->lad + kLadBarErr, {}, trace};
        const SlotOrder so = slot_order(first, nc);
        for (int c = 0; c < 16; c++) args.order[c] = so.v[c];
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(nc * csize));
        cfg.blockDim = dim3(chol_threads<T>());
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = (unsigned)csize;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const ProfToken t = prof_begin("dense_chol", s);
        cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args);
        prof_end(t, s);
        GPB2_CUDA_TRY(e);
        GPB2_CUDA_TRY(launch_prof("dense_mark", k_ladder_mark, dim3(1), dim3(1), 0, s,
                                  (const int*)done, so, nc,
                                  sel));
        if (trace) {  // diagnostics: per-phase totals of the last candidate of this launch
            std::vector<unsigned long long> h(8 * (size_t)npan + 3 * 16);
            GPB2_CUDA_TRY(cudaMemcpyAsync(h.data(), trace, sizeof(unsigned long long) * h.size(),
                                          cudaMemcpyDeviceToHost, s));
            GPB2_CUDA_TRY(cudaStreamSynchronize(s));
            // Per-panel intervals of rank 0: P load, P solve, P store, barrier + U tile 0, D load,
            // D factor, D store + U rest, barrier.
            double sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            int kk = 0;
            for (; kk + 1 < npan && h[8 * (kk + 1)] != 0; kk++)
                for (int q = 0; q < 8; q++) {
                    const unsigned long long t1 = q < 7 ? h[8 * kk + q + 1] : h[8 * (kk + 1)];
                    if (t1 && h[8 * kk + q]) sum[q] += (double)(t1 - h[8 * kk + q]);
                }
            std::fprintf(stderr,
                         "gpb2 dense trace: n0=%lld cluster=%d tile=%d panels=%d/%d us: Pload %.1f "
                         "Psolve %.1f Pstore %.1f bar+tile0 %.1f Dload %.1f Dfactor %.1f "
                         "Dstore+Urest %.1f bar %.1f\n",
                         (long long)n, csize, tile, kk, npan, sum[0] / 1e3, sum[1] / 1e3,
                         sum[2] / 1e3, sum[3] / 1e3, sum[4] / 1e3, sum[5] / 1e3, sum[6] / 1e3,
                         sum[7] / 1e3);
            if (std::atoi(std::getenv("GPB2_TRACE_DENSE")) >= 2) {
                // Candidate lifetimes relative to the first start (us); end code 1000 = done,
                // 1 = failed in panel 0's block, 2 + k = stopped at the top of panel k.
                unsigned long long t00 = ~0ull;
                for (int q = 0; q < nc; q++)
                    if (h[8 * npan + 3 * q]) t00 = std::min(t00, h[8 * npan + 3 * q]);
                for (int q = 0; q < nc; q++) {
                    const unsigned long long* lf = h.data() + 8 * npan + 3 * q;
                    std::fprintf(stderr, "  slot %d ladder %d: start %.1f end %.1f how %llu\n", q,
                                 order[first + q], lf[0] ? (lf[0] - t00) / 1e3 : -1.0,
                                 lf[1] ? (lf[1] - t00) / 1e3 : -1.0, lf[2]);
                }
                for (int q = 0; q < 8; q++) {
                    std::fprintf(stderr, "  interval %d:", q);
                    for (int k2 = 0; k2 < kk; k2++) {
                        const unsigned long long t1 =
                            q < 7 ? h[8 * k2 + q + 1] : h[8 * (k2 + 1)];
                        std::fprintf(stderr, " %.1f",
                                     (t1 && h[8 * k2 + q]) ? (t1 - h[8 * k2 + q]) / 1e3 : -1.0);
                    }
                    std::fprintf(stderr, "\n");
                }
            }
        }
    }
    GPB2_CUDA_TRY(launch_prof("dense_pick", k_ladder_pick<T>, dim3(4 * 148), dim3(256), 0, s,
                              (const T*)base, (const int*)sel, (int64_t)nn,
                              static_cast<T*>(p->Ld), p->lad + kLadNotPD));
    p->ladder_eps.assign(epsv.begin(), epsv.begin() + ncand_used);
    p->dense_pending = true;  // outcome checked by the call's finishing synchronisation
    p->dense_launched = true;
    return GPB2_OK;
}

template int dense_cholesky_ladder<float>(gpb2_problem*, cudaStream_t);
template int dense_cholesky_ladder<double>(gpb2_problem*, cudaStream_t);

}  // namespace gpb2
