/*
 * gp_oracle.c -- CPU restatement of GraphGP.jl's per-point Vecchia refine path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for libgraphgp_b200.so and the
 * timed CPU baseline of bench.py.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may load it.  The product (the CUDA library and the
 * Python mirror of the reference API) never calls into it.
 *
 * Compiled twice from this one source (see oracle/Makefile): -DGP_F32 gives the Float32 entry
 * points (suffix _f32), the default gives Float64 (suffix _f64).  Built with -O2
 * -ffp-contract=off so the floating-point operation order below is exactly the written order
 * (no FMA contraction), which makes the restatement deterministic for a given thread count.
 *
 * Every routine follows a named reference function (paths are inside the GraphGP.jl tree):
 *   cov_lookup            src/interp.jl:10-34
 *   cov_lookup_weights    src/interp.jl:62-83
 *   assemble_cov          src/linalg.jl:15-29   (exact Int64 squared distances)
 *   chol_lower            src/linalg.jl:38-73  (pivot floor eps(T)*A11, zeroed column)
 *   mean_vec_solve        src/linalg.jl:85-103  (weight zeroed at 1.5*sqrt(eps)*L11)
 *   chol_pullback         src/linalg.jl:112-134
 *   refine (forward)      src/kernels.jl:101-119 + src/api.jl:113-141 + src/cpu_native.jl:86-112
 *   refine_inv            src/kernels.jl:37-56, src/cpu_native.jl:46-63
 *   refine_logdet_terms   src/kernels.jl:25-35, src/cpu_native.jl:33-44
 *   generate_grad_xi core src/grad.jl:392-465 (materialised mean_vec/std + serial reverse sweep)
 *   generate_grad_vals    src/grad_generate_vals.jl:44-101,111-213 and the device per-point
 *                         body src/kernels_adjoint.jl:484-553 (pivfloor guard in the z-bar solve)
 *   refine_logdet_grad    src/grad.jl:32-87 (privatised per-chunk histograms)
 *   refine_inv_loss_grad  src/grad.jl:533-641
 *   dense layer           src/dense.jl:15-67,112-183,227-266 and chol_pullback_dyn!
 *                         src/grad_generate_vals.jl:18-39
 *
 * Layout (identical to the reference's memory layout):
 *   coords    (N, D) row-major uint32   == Julia (D, N) column-major
 *   nbrs      (M, K) row-major int64, 0-based == Julia (K, M) column-major minus one
 *   offsets   [n_off] int64, offsets[0] = n0, batch b covers positions [offsets[b-1], offsets[b])
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#ifdef GP_F32
typedef float T;
#define SFX(name) name##_f32
#define T_EPS FLT_EPSILON
#define SQRT_T sqrtf
#define LOG_T logf
#else
typedef double T;
#define SFX(name) name##_f64
#define T_EPS DBL_EPSILON
#define SQRT_T sqrt
#define LOG_T log
#endif

#define KMAX 64
#define DMAX 8

/* ---------------------------------------------------------------------------------------- */
/* L0: scalar numerics                                                                       */
/* ---------------------------------------------------------------------------------------- */

/* src/interp.jl:10-34.  Clamp at both ends; binary search for bins[lo] <= r < bins[lo+1]. */
static inline T cov_lookup(T r, const T* bins, const T* vals, int64_t n) {
    if (r <= bins[0]) return vals[0];
    if (r >= bins[n - 1]) return vals[n - 1];
    int64_t lo = 0, hi = n - 1;
    while (hi - lo > 1) {
        int64_t mid = (lo + hi) >> 1;
        if (bins[mid] <= r) lo = mid; else hi = mid;
    }
    T x0 = bins[lo], x1 = bins[lo + 1];
    T y0 = vals[lo], y1 = vals[lo + 1];
    T slope = (y1 - y0) / (x1 - x0);
    return y0 + slope * (r - x0);
}

/* src/interp.jl:62-83.  Returns lo (0-based) and the two interpolation weights. */
static inline int64_t cov_lookup_weights(T r, const T* bins, int64_t n, T* wlo, T* whi) {
    if (r <= bins[0]) { *wlo = (T)1; *whi = (T)0; return 0; }
    if (r >= bins[n - 1]) { *wlo = (T)0; *whi = (T)1; return n - 2; }
    int64_t lo = 0, hi = n - 1;
    while (hi - lo > 1) {
        int64_t mid = (lo + hi) >> 1;
        if (bins[mid] <= r) lo = mid; else hi = mid;
    }
    T x0 = bins[lo], x1 = bins[lo + 1];
    T t = (r - x0) / (x1 - x0);
    *wlo = (T)1 - t;
    *whi = t;
    return lo;
}

/* Anisotropic covariance (src/aniso.jl), consulted by assemble_cov and gpo_dense_cov while set
 * by gpo_set_aniso (this checker handles one problem at a time). */
static struct {
    const T* sb;
    int64_t ns;
    const T* zb;
    int64_t nz;
    const T* grid; /* (ns, nz) column-major */
    T alpha;
    int on;
} g_an;

int SFX(gpo_set_aniso)(const T* sb, int64_t ns, const T* zb, int64_t nz, const T* grid,
                       T alpha, int on) {
    g_an.sb = sb;
    g_an.ns = ns;
    g_an.zb = zb;
    g_an.nz = nz;
    g_an.grid = grid;
    g_an.alpha = alpha;
    g_an.on = on;
    return 0;
}

/* _frac_index (src/aniso.jl:42-57): 0-based, clamped to [0, n - 1]. */
static inline T frac_index(T d, const T* bins, int64_t n) {
    if (d <= bins[0]) return (T)0;
    if (d >= bins[n - 1]) return (T)(n - 1);
    int64_t lo = 0, hi = n - 1;
    while (hi - lo > 1) {
        int64_t mid = (lo + hi) >> 1;
        if (bins[mid] <= d) lo = mid; else hi = mid;
    }
    T x0 = bins[lo], x1 = bins[lo + 1];
    return (T)lo + (d - x0) / (x1 - x0);
}

/* aniso_lookup (src/aniso.jl:67-85). */
static inline T aniso_lookup(T ds, T dz) {
    T fx = frac_index(ds, g_an.sb, g_an.ns), fz = frac_index(dz, g_an.zb, g_an.nz);
    int64_t i0 = (int64_t)fx, j0 = (int64_t)fz;
    int64_t i1 = i0 + 1 < g_an.ns ? i0 + 1 : g_an.ns - 1;
    int64_t j1 = j0 + 1 < g_an.nz ? j0 + 1 : g_an.nz - 1;
    T tx = fx - (T)i0, tz = fz - (T)j0;
    const T* g = g_an.grid;
    int64_t ns = g_an.ns;
    T g00 = g[i0 + j0 * ns], g10 = g[i1 + j0 * ns], g01 = g[i0 + j1 * ns], g11 = g[i1 + j1 * ns];
    return (g00 * ((T)1 - tx) + g10 * tx) * ((T)1 - tz) + (g01 * ((T)1 - tx) + g11 * tx) * tz;
}

/* aniso_lookup on arrays (the model set by gpo_set_aniso). */
int SFX(gpo_aniso_lookup)(const T* ds, const T* dz, int64_t n, T* out) {
    for (int64_t i = 0; i < n; i++) out[i] = aniso_lookup(ds[i], dz[i]);
    return 0;
}

/* The pair's covariance under the anisotropic model (src/aniso.jl:88-105): spatial distance
 * over the first D - 1 coordinates, radial |dz| * scale / alpha over the last. */
static inline T aniso_pair(const uint32_t* a, const uint32_t* b, int D, T scale) {
    int64_t sqs = 0;
    for (int d = 0; d < D - 1; d++) {
        int64_t di = (int64_t)a[d] - (int64_t)b[d];
        sqs += di * di;
    }
    int64_t dzi = (int64_t)a[D - 1] - (int64_t)b[D - 1];
    T dsp = SQRT_T((T)sqs) * scale;
    T tz = (T)dzi;
    T dz = (tz < 0 ? -tz : tz) * scale / g_an.alpha;
    return aniso_lookup(dsp, dz);
}

/* Radius between two lattice points: exact Int64 squared distance, then T(sq), sqrt, * scale
 * (src/linalg.jl:19-24). */
static inline T lattice_radius(const uint32_t* a, const uint32_t* b, int D, T scale) {
    int64_t sq = 0;
    for (int d = 0; d < D; d++) {
        int64_t di = (int64_t)a[d] - (int64_t)b[d];
        sq += di * di;
    }
    return SQRT_T((T)sq) * scale;
}

/* Gather the joint coordinates: rows 0..K-1 = neighbours, row K = the refined point
 * (src/kernels.jl:9-23). */
static inline void gather_joint(uint32_t* jc, const uint32_t* coords, const int64_t* nb, int K,
                                int D, int64_t fine) {
    for (int j = 0; j < K; j++)
        for (int d = 0; d < D; d++) jc[j * D + d] = coords[nb[j] * D + d];
    for (int d = 0; d < D; d++) jc[K * D + d] = coords[fine * D + d];
}

/* src/linalg.jl:15-29.  A is KP1 x KP1 row-major; only the lower triangle is written. */
static inline void assemble_cov(T* A, const uint32_t* jc, int KP1, int D, T scale,
                                const T* bins, const T* vals, int64_t nb) {
    if (g_an.on) { /* assemble_cov! of src/aniso.jl:88-105 */
        T diag = aniso_lookup((T)0, (T)0);
        for (int a = 0; a < KP1; a++) {
            A[a * KP1 + a] = diag;
            for (int b = 0; b < a; b++) A[a * KP1 + b] = aniso_pair(jc + a * D, jc + b * D, D, scale);
        }
        return;
    }
    for (int a = 0; a < KP1; a++) {
        A[a * KP1 + a] = cov_lookup((T)0, bins, vals, nb);
        for (int b = 0; b < a; b++) {
            T r = lattice_radius(jc + a * D, jc + b * D, D, scale);
            A[a * KP1 + b] = cov_lookup(r, bins, vals, nb);
        }
    }
}

/* src/linalg.jl:38-73.  Left-looking Cholesky with the relative pivot floor.  Returns the
 * number of clamped pivots (diagnostics only). */
static inline int chol_lower(T* A, int KP1) {
    int clamped = 0;
    T pivmin = T_EPS * A[0];
    for (int j = 0; j < KP1; j++) {
        T s = A[j * KP1 + j];
        for (int p = 0; p < j; p++) s -= A[j * KP1 + p] * A[j * KP1 + p];
        if (s > pivmin) {
            T d = SQRT_T(s);
            A[j * KP1 + j] = d;
            for (int i = j + 1; i < KP1; i++) {
                T t = A[i * KP1 + j];
                for (int p = 0; p < j; p++) t -= A[i * KP1 + p] * A[j * KP1 + p];
                A[i * KP1 + j] = t / d;
            }
        } else {
            A[j * KP1 + j] = SQRT_T(pivmin);
            for (int i = j + 1; i < KP1; i++) A[i * KP1 + j] = (T)0;
            clamped++;
        }
    }
    return clamped;
}

/* The constant 1.5*sqrt(eps(T)) of src/linalg.jl:88, evaluated in T left to right. */
static inline T pivfloor_coeff(void) { return (T)1.5 * SQRT_T(T_EPS); }

/* src/linalg.jl:85-103.  Back substitution L[0:K,0:K]^T x = L[K, 0:K]. */
static inline void mean_vec_solve(T* x, const T* L, int K) {
    int KP1 = K + 1;
    T pivfloor = pivfloor_coeff() * L[0];
    for (int i = K - 1; i >= 0; i--) {
        T d = L[i * KP1 + i];
        if (d > pivfloor) {
            T s = L[K * KP1 + i];
            for (int j = i + 1; j < K; j++) s -= L[j * KP1 + i] * x[j];
            x[i] = s / d;
        } else {
            x[i] = (T)0;
        }
    }
}

/* src/linalg.jl:112-134.  Reverse of chol_lower; Lbar consumed, Abar lower triangle. */
static void chol_pullback(T* Abar, T* Lbar, const T* L, int n) {
    for (int j = n - 1; j >= 0; j--) {
        T ljj = L[j * n + j];
        for (int i = n - 1; i >= j + 1; i--) {
            T lbij = Lbar[i * n + j];
            T tbar = lbij / ljj;
            Lbar[j * n + j] -= lbij * L[i * n + j] / ljj;
            Abar[i * n + j] = tbar;
            for (int p = 0; p < j; p++) {
                Lbar[i * n + p] -= tbar * L[j * n + p];
                Lbar[j * n + p] -= tbar * L[i * n + p];
            }
        }
        T sbar = Lbar[j * n + j] / (2 * ljj);
        Abar[j * n + j] = sbar;
        for (int p = 0; p < j; p++) Lbar[j * n + p] -= 2 * sbar * L[j * n + p];
    }
}

/* One refined point's factor: gather + assemble + chol + solve.  Returns std. */
static inline T point_factor(T* A, T* mv, uint32_t* jc, const uint32_t* coords, const int64_t* nbrs,
                             int64_t m, int64_t n0, int K, int D, T scale, const T* bins,
                             const T* vals, int64_t nb) {
    int KP1 = K + 1;
    gather_joint(jc, coords, nbrs + m * K, K, D, n0 + m);
    assemble_cov(A, jc, KP1, D, scale, bins, vals, nb);
    chol_lower(A, KP1);
    if (mv) mean_vec_solve(mv, A, K);
    return A[K * KP1 + K];
}

/* Scatter the lower-triangle cotangent Abar into dv through the interpolation weights, in the
 * CPU order of src/grad.jl:39-53 (row a: diagonal into bin 0, then the row's off-diagonals).
 * acc_t == 1 accumulates in T, the reference's accumulator type: the T-rounded running value is
 * stored back into the double slot, so the arithmetic is exactly T arithmetic.  acc_t == 0
 * accumulates the same T-valued products in double. */
static inline void scatter_abar(double* dv, const T* Abar, const uint32_t* jc, int KP1, int D,
                                T scale, const T* bins, int64_t nb, int acc_t) {
    for (int a = 0; a < KP1; a++) {
        if (acc_t) dv[0] = (double)((T)dv[0] + Abar[a * KP1 + a]);
        else dv[0] += (double)Abar[a * KP1 + a];
        for (int b = 0; b < a; b++) {
            T r = lattice_radius(jc + a * D, jc + b * D, D, scale);
            T wlo, whi;
            int64_t lo = cov_lookup_weights(r, bins, nb, &wlo, &whi);
            T g = Abar[a * KP1 + b];
            if (acc_t) {
                dv[lo] = (double)((T)dv[lo] + g * wlo);
                dv[lo + 1] = (double)((T)dv[lo + 1] + g * whi);
            } else {
                dv[lo] += (double)(g * wlo);
                dv[lo + 1] += (double)(g * whi);
            }
        }
    }
}

/* ---------------------------------------------------------------------------------------- */
/* L1/L2: refine-layer operations                                                            */
/* ---------------------------------------------------------------------------------------- */

static int nthreads_of(int requested) {
#ifdef _OPENMP
    return requested > 0 ? requested : omp_get_max_threads();
#else
    (void)requested;
    return 1;
#endif
}

int SFX(gpo_cov_lookup)(const T* r, int64_t n, const T* bins, const T* vals, int64_t nb, T* out) {
    for (int64_t i = 0; i < n; i++) out[i] = cov_lookup(r[i], bins, vals, nb);
    return 0;
}

int SFX(gpo_cov_lookup_weights)(const T* r, int64_t n, const T* bins, int64_t nb, int64_t* lo,
                                 T* wlo, T* whi) {
    for (int64_t i = 0; i < n; i++) lo[i] = cov_lookup_weights(r[i], bins, nb, &wlo[i], &whi[i]);
    return 0;
}

/* chol_lower + mean_vec_solve on an explicit (K+1)x(K+1) matrix (row-major, lower used). */
int SFX(gpo_chol_solve)(T* A, int KP1, T* mv) {
    chol_lower(A, KP1);
    if (mv) mean_vec_solve(mv, A, KP1 - 1);
    return 0;
}

/* Forward refine over the depth batches (src/api.jl:113-141 with the fused CPU body of
 * src/cpu_native.jl:86-112).  values[0:n0] preset; xi_ref indexed by m. */
int SFX(gpo_refine)(T* values, const T* xi_ref, const uint32_t* coords, const int64_t* nbrs,
                    const int64_t* offsets, int64_t n_off, int64_t n0, int K, int D, T scale,
                    const T* bins, const T* vals, int64_t nb, int nthreads) {
    if (K > KMAX || D > DMAX) return 2;
    int nt = nthreads_of(nthreads);
    for (int64_t b = 1; b < n_off; b++) {
        int64_t lo = offsets[b - 1], hi = offsets[b];
        if (hi <= lo) continue;
#pragma omp parallel num_threads(nt)
        {
            T A[(KMAX + 1) * (KMAX + 1)], mv[KMAX];
            uint32_t jc[(KMAX + 1) * DMAX];
#pragma omp for schedule(static)
            for (int64_t p = lo; p < hi; p++) {
                int64_t m = p - n0;
                T sd = point_factor(A, mv, jc, coords, nbrs, m, n0, K, D, scale, bins, vals, nb);
                T acc = sd * xi_ref[m];
                for (int j = 0; j < K; j++) acc += mv[j] * values[nbrs[m * K + j]];
                values[p] = acc;
            }
        }
    }
    return 0;
}

/* Diagnostics of the near-singular regime (no reference counterpart): over the refined points,
 * out[0] = points whose chol_lower clamped at least one pivot, out[1] = clamped pivots in all,
 * out[2] = points sharing a lattice site with one of their neighbours (a collision),
 * out[3] = neighbour weights zeroed by mean_vec_solve's pivot floor. */
int SFX(gpo_clamp_stats)(int64_t* out, const uint32_t* coords, const int64_t* nbrs, int64_t M,
                         int64_t n0, int K, int D, T scale, const T* bins, const T* vals,
                         int64_t nb, int nthreads) {
    if (K > KMAX || D > DMAX) return 2;
    int nt = nthreads_of(nthreads);
    int64_t pts = 0, piv = 0, col = 0, zw = 0;
#pragma omp parallel num_threads(nt) reduction(+ : pts, piv, col, zw)
    {
        T A[(KMAX + 1) * (KMAX + 1)], mv[KMAX];
        uint32_t jc[(KMAX + 1) * DMAX];
#pragma omp for schedule(static)
        for (int64_t m = 0; m < M; m++) {
            const int KP1 = K + 1;
            gather_joint(jc, coords, nbrs + m * K, K, D, n0 + m);
            int hit = 0;
            for (int j = 0; j < K && !hit; j++) {
                int same = 1;
                for (int d = 0; d < D; d++) same &= jc[j * D + d] == jc[K * D + d];
                hit = same;
            }
            col += hit;
            assemble_cov(A, jc, KP1, D, scale, bins, vals, nb);
            const int c = chol_lower(A, KP1);
            pts += c > 0;
            piv += c;
            mean_vec_solve(mv, A, K);
            const T pivfloor = pivfloor_coeff() * A[0];
            for (int i = 0; i < K; i++) zw += !(A[i * KP1 + i] > pivfloor);
        }
    }
    out[0] = pts;
    out[1] = piv;
    out[2] = col;
    out[3] = zw;
    return 0;
}

/* Materialised mean_vec (M,K) and std (M) (src/kernels.jl:61-78, src/cpu_native.jl:65-84). */
int SFX(gpo_meanvec_std)(T* mean_vec, T* stdv, const uint32_t* coords, const int64_t* nbrs,
                         int64_t M, int64_t n0, int K, int D, T scale, const T* bins,
                         const T* vals, int64_t nb, int nthreads) {
    if (K > KMAX || D > DMAX) return 2;
    int nt = nthreads_of(nthreads);
#pragma omp parallel num_threads(nt)
    {
        T A[(KMAX + 1) * (KMAX + 1)];
        uint32_t jc[(KMAX + 1) * DMAX];
#pragma omp for schedule(static)
        for (int64_t m = 0; m < M; m++)
            stdv[m] = point_factor(A, mean_vec + m * K, jc, coords, nbrs, m, n0, K, D, scale,
                                   bins, vals, nb);
    }
    return 0;
}

/* refine_inv (src/kernels.jl:37-56): xi[m] = (values[n0+m] - mv . values[nbrs]) / std. */
int SFX(gpo_refine_inv)(T* xi_out, const T* values, const uint32_t* coords, const int64_t* nbrs,
                        int64_t M, int64_t n0, int K, int D, T scale, const T* bins,
                        const T* vals, int64_t nb, int nthreads) {
    if (K > KMAX || D > DMAX) return 2;
    int nt = nthreads_of(nthreads);
#pragma omp parallel num_threads(nt)
    {
        T A[(KMAX + 1) * (KMAX + 1)], mv[KMAX];
        uint32_t jc[(KMAX + 1) * DMAX];
#pragma omp for schedule(static)
        for (int64_t m = 0; m < M; m++) {
            T sd = point_factor(A, mv, jc, coords, nbrs, m, n0, K, D, scale, bins, vals, nb);
            T mean = (T)0;
            for (int j = 0; j < K; j++) mean += mv[j] * values[nbrs[m * K + j]];
            xi_out[m] = (values[n0 + m] - mean) / sd;
        }
    }
    return 0;
}

/* refine_logdet_terms (src/kernels.jl:25-35). */
int SFX(gpo_refine_logdet_terms)(T* terms, const uint32_t* coords, const int64_t* nbrs, int64_t M,
                                 int64_t n0, int K, int D, T scale, const T* bins, const T* vals,
                                 int64_t nb, int nthreads) {
    if (K > KMAX || D > DMAX) return 2;
    int nt = nthreads_of(nthreads);
#pragma omp parallel num_threads(nt)
    {
        T A[(KMAX + 1) * (KMAX + 1)];
        uint32_t jc[(KMAX + 1) * DMAX];
#pragma omp for schedule(static)
        for (int64_t m = 0; m < M; m++)
            terms[m] = LOG_T(point_factor(A, NULL, jc, coords, nbrs, m, n0, K, D, scale, bins,
                                          vals, nb));
    }
    return 0;
}

/* Reverse depth-batch sweep of generate_grad_xi in tree order (src/grad.jl:430-446): on entry
 * vb is the field cotangent (tree order); on exit xg[n0:N] = std*vb and vb[0:n0] holds the
 * cotangent reaching the dense block.  Serial, latest batch first, as in the reference. */
int SFX(gpo_reverse_sweep)(T* xg, T* vb, const T* mean_vec, const T* stdv, const int64_t* nbrs,
                           const int64_t* offsets, int64_t n_off, int64_t n0, int K) {
    for (int64_t b = n_off - 1; b >= 1; b--) {
        int64_t lo = offsets[b - 1], hi = offsets[b];
        for (int64_t p = hi - 1; p >= lo; p--) {
            int64_t m = p - n0;
            xg[p] = stdv[m] * vb[p];
            for (int j = 0; j < K; j++) {
                int64_t nbj = nbrs[m * K + j];
                if (nbj < 0) continue;
                vb[nbj] += mean_vec[m * K + j] * vb[p];
            }
        }
    }
    return 0;
}

/* Per-point body of the generate vals-gradient (src/grad_generate_vals.jl:44-101 with the
 * pivfloor guard of src/kernels_adjoint.jl:520-530). */
static void generate_point_vals(double* dv, T* A, T* Abar, T* Lbar, T* zbar, T* mv, uint32_t* jc,
                                const uint32_t* coords, const int64_t* nbrs, T scale,
                                const T* bins, const T* vals, int64_t nb, int64_t n0, int64_t m,
                                const T* v, T vbp, T stdbar, int K, int D, int acc_t) {
    int KP1 = K + 1;
    point_factor(A, mv, jc, coords, nbrs, m, n0, K, D, scale, bins, vals, nb);
    T pivfloor = pivfloor_coeff() * A[0];
    for (int i = 0; i < KP1 * KP1; i++) Lbar[i] = (T)0;
    Lbar[K * KP1 + K] = stdbar;
    for (int j = 0; j < K; j++) zbar[j] = vbp * v[nbrs[m * K + j]];
    for (int i = 0; i < K; i++) {
        if (A[i * KP1 + i] > pivfloor) {
            T s = zbar[i];
            for (int p = 0; p < i; p++) s -= A[i * KP1 + p] * zbar[p];
            zbar[i] = s / A[i * KP1 + i];
        } else {
            zbar[i] = (T)0;
        }
    }
    for (int j = 0; j < K; j++) {
        Lbar[K * KP1 + j] += zbar[j];
        for (int i = 0; i <= j; i++) Lbar[j * KP1 + i] -= zbar[i] * mv[j];
    }
    chol_pullback(Abar, Lbar, A, KP1);
    scatter_abar(dv, Abar, jc, KP1, D, scale, bins, nb, acc_t);
}

/* Refined part of generate_grad_vals in tree order (src/grad_generate_vals.jl:173-186):
 * v = forward field, xih = xi (tree order), vb = cotangent (tree order, updated in place so
 * that on exit vb[0:n0] is the dense block's cotangent).  dv (double) accumulates the
 * histogram; acc_t = 1 rounds every accumulation to T as the reference does. */
int SFX(gpo_generate_grad_vals_refine)(double* dv, T* vb, const T* v, const T* xih,
                                       const T* mean_vec, const uint32_t* coords,
                                       const int64_t* nbrs, const int64_t* offsets, int64_t n_off,
                                       int64_t n0, int K, int D, T scale, const T* bins,
                                       const T* vals, int64_t nb, int acc_t) {
    if (K > KMAX || D > DMAX) return 2;
    int KP1 = K + 1;
    T* A = (T*)malloc(sizeof(T) * KP1 * KP1 * 3);
    T* Abar = A + KP1 * KP1;
    T* Lbar = Abar + KP1 * KP1;
    T zbar[KMAX], mv[KMAX];
    uint32_t jc[(KMAX + 1) * DMAX];
    for (int64_t b = n_off - 1; b >= 1; b--) {
        int64_t lo = offsets[b - 1], hi = offsets[b];
        for (int64_t p = hi - 1; p >= lo; p--) {
            int64_t m = p - n0;
            T vbp = vb[p];
            generate_point_vals(dv, A, Abar, Lbar, zbar, mv, jc, coords, nbrs, scale, bins, vals,
                                nb, n0, m, v, vbp, vbp * xih[p], K, D, acc_t);
            for (int j = 0; j < K; j++) {
                int64_t nbj = nbrs[m * K + j];
                if (nbj < 0) continue;
                vb[nbj] += mean_vec[m * K + j] * vbp;
            }
        }
    }
    free(A);
    return 0;
}

/* refine_logdet_grad_vals + logdet sum (src/grad.jl:32-87): chunks of cld(M, nchunks) points,
 * one private histogram per chunk, then summed in chunk order. */
int SFX(gpo_refine_logdet_grad_vals)(double* dv_out, double* logdet_out, const uint32_t* coords,
                                     const int64_t* nbrs, int64_t M, int64_t n0, int K, int D,
                                     T scale, const T* bins, const T* vals, int64_t nb,
                                     int nthreads, int acc_t) {
    if (K > KMAX || D > DMAX) return 2;
    int nt = nthreads_of(nthreads);
    int64_t nchunks = nt < M ? nt : (M > 0 ? M : 1);
    int64_t csz = (M + nchunks - 1) / nchunks;
    double* priv = (double*)calloc((size_t)nchunks * nb, sizeof(double));
    double* ldp = (double*)calloc((size_t)nchunks, sizeof(double));
    int KP1 = K + 1;
#pragma omp parallel for schedule(static, 1) num_threads(nt)
    for (int64_t c = 0; c < nchunks; c++) {
        T* A = (T*)malloc(sizeof(T) * KP1 * KP1 * 3);
        T* Abar = A + KP1 * KP1;
        T* Lbar = Abar + KP1 * KP1;
        uint32_t jc[(KMAX + 1) * DMAX];
        double* dv = priv + c * nb;
        T ld = (T)0;
        int64_t lo = c * csz, hi = lo + csz < M ? lo + csz : M;
        for (int64_t m = lo; m < hi; m++) {
            T sd = point_factor(A, NULL, jc, coords, nbrs, m, n0, K, D, scale, bins, vals, nb);
            ld += LOG_T(sd);
            for (int i = 0; i < KP1 * KP1; i++) Lbar[i] = (T)0;
            Lbar[K * KP1 + K] = (T)1 / A[K * KP1 + K];
            chol_pullback(Abar, Lbar, A, KP1);
            scatter_abar(dv, Abar, jc, KP1, D, scale, bins, nb, acc_t);
        }
        ldp[c] = (double)ld;
        free(A);
    }
    double ldsum = 0.0;
    for (int64_t i = 0; i < nb; i++) dv_out[i] = 0.0;
    for (int64_t c = 0; c < nchunks; c++) {
        ldsum += ldp[c];
        for (int64_t i = 0; i < nb; i++) {
            if (acc_t) dv_out[i] = (double)((T)dv_out[i] + (T)priv[c * nb + i]);
            else dv_out[i] += priv[c * nb + i];
        }
    }
    if (logdet_out) *logdet_out = ldsum;
    free(priv);
    free(ldp);
    return 0;
}

/* refine_inv_loss_grad_vals (src/grad.jl:533-641): loss = 0.5*sum(xi^2) and its vals-gradient.
 * Note the reference's inverse-loss z-bar solve has NO pivfloor guard (src/grad.jl:574-580). */
int SFX(gpo_refine_inv_loss_grad_vals)(double* dv_out, double* loss_out, const T* values,
                                       const uint32_t* coords, const int64_t* nbrs, int64_t M,
                                       int64_t n0, int K, int D, T scale, const T* bins,
                                       const T* vals, int64_t nb, int nthreads, int acc_t) {
    if (K > KMAX || D > DMAX) return 2;
    int nt = nthreads_of(nthreads);
    int64_t nchunks = nt < M ? nt : (M > 0 ? M : 1);
    int64_t csz = (M + nchunks - 1) / nchunks;
    double* priv = (double*)calloc((size_t)nchunks * nb, sizeof(double));
    double* lp = (double*)calloc((size_t)nchunks, sizeof(double));
    int KP1 = K + 1;
#pragma omp parallel for schedule(static, 1) num_threads(nt)
    for (int64_t c = 0; c < nchunks; c++) {
        T* A = (T*)malloc(sizeof(T) * KP1 * KP1 * 3);
        T* Abar = A + KP1 * KP1;
        T* Lbar = Abar + KP1 * KP1;
        T mv[KMAX], zbar[KMAX];
        uint32_t jc[(KMAX + 1) * DMAX];
        double* dv = priv + c * nb;
        T loss = (T)0;
        int64_t lo = c * csz, hi = lo + csz < M ? lo + csz : M;
        for (int64_t m = lo; m < hi; m++) {
            T sd = point_factor(A, mv, jc, coords, nbrs, m, n0, K, D, scale, bins, vals, nb);
            T mean = (T)0;
            for (int j = 0; j < K; j++) mean += mv[j] * values[nbrs[m * K + j]];
            T xim = (values[n0 + m] - mean) / sd;
            for (int i = 0; i < KP1 * KP1; i++) Lbar[i] = (T)0;
            Lbar[K * KP1 + K] = -xim * xim / sd;
            for (int j = 0; j < K; j++) zbar[j] = -xim * values[nbrs[m * K + j]] / sd;
            for (int i = 0; i < K; i++) {
                T s = zbar[i];
                for (int p = 0; p < i; p++) s -= A[i * KP1 + p] * zbar[p];
                zbar[i] = s / A[i * KP1 + i];
            }
            for (int j = 0; j < K; j++) {
                Lbar[K * KP1 + j] += zbar[j];
                for (int i = 0; i <= j; i++) Lbar[j * KP1 + i] -= zbar[i] * mv[j];
            }
            chol_pullback(Abar, Lbar, A, KP1);
            scatter_abar(dv, Abar, jc, KP1, D, scale, bins, nb, acc_t);
            loss += xim * xim / 2;
        }
        lp[c] = (double)loss;
        free(A);
    }
    double lsum = 0.0;
    for (int64_t i = 0; i < nb; i++) dv_out[i] = 0.0;
    for (int64_t c = 0; c < nchunks; c++) {
        lsum += lp[c];
        for (int64_t i = 0; i < nb; i++) {
            if (acc_t) dv_out[i] = (double)((T)dv_out[i] + (T)priv[c * nb + i]);
            else dv_out[i] += priv[c * nb + i];
        }
    }
    if (loss_out) *loss_out = lsum;
    free(priv);
    free(lp);
    return 0;
}

/* ---------------------------------------------------------------------------------------- */
/* L3: dense first layer (src/dense.jl)                                                      */
/* ---------------------------------------------------------------------------------------- */

/* _assemble_dense_cov (src/dense.jl:15-40): full symmetric n x n, row-major.  Entries are
 * independent, so the columns are spread over the host threads. */
int SFX(gpo_dense_cov)(T* K, const uint32_t* coords, int64_t n, int D, T scale, const T* bins,
                       const T* vals, int64_t nb) {
    /* _assemble_dense_cov_aniso (src/aniso.jl:218-244) while the anisotropic model is set. */
#pragma omp parallel for schedule(dynamic, 16)
    for (int64_t j = 0; j < n; j++) {
        K[j * n + j] = g_an.on ? aniso_lookup((T)0, (T)0) : cov_lookup((T)0, bins, vals, nb);
        for (int64_t i = j + 1; i < n; i++) {
            T v;
            if (g_an.on) {
                v = aniso_pair(coords + i * D, coords + j * D, D, scale);
            } else {
                T r = lattice_radius(coords + i * D, coords + j * D, D, scale);
                v = cov_lookup(r, bins, vals, nb);
            }
            K[i * n + j] = v;
            K[j * n + i] = v;
        }
    }
    return 0;
}

/* Left-looking Cholesky (lower, row-major); returns 0 on success, j+1 at the first
 * non-positive (or NaN) pivot like LAPACK potrf's info.  Every entry receives exactly the
 * subtractions of the unblocked recurrence
 *     L[i][j] = (A[i][j] - L[i][0]L[j][0] - L[i][1]L[j][1] - ... - L[i][j-1]L[j][j-1]) / L[j][j]
 * in that order (p ascending, each product rounded, then the subtraction rounded), so the factor
 * does not depend on the blocking or the thread count.  Columns are taken in panels of PB: the
 * products with the finished columns p < j0 are subtracted first for the whole panel (the panel's
 * rows read once per row below it, from a transposed copy), then the panel is finished column by
 * column (p = j0 .. j-1).  Rows are independent and spread over the host threads. */
#define PB 32
static int64_t dense_potrf(T* L, int64_t n) {
    T* Wt = (T*)malloc(sizeof(T) * (size_t)PB * (size_t)(n > 0 ? n : 1));
    if (!Wt) return -1;
    for (int64_t j0 = 0; j0 < n; j0 += PB) {
        const int64_t nb = (n - j0) < PB ? (n - j0) : PB;
        /* Wt[p][jj] = L[j0+jj][p] for the finished columns p < j0. */
        for (int64_t p = 0; p < j0; p++)
            for (int64_t jj = 0; jj < nb; jj++) Wt[p * PB + jj] = L[(j0 + jj) * n + p];
        /* Phase 1: subtract the products with columns p < j0 from every entry (i, j) of the
         * panel, i >= j >= j0. */
#pragma omp parallel for schedule(static) if ((n - j0) * j0 > 65536)
        for (int64_t i = j0; i < n; i++) {
            T t[PB];
            T* Li = L + i * n;
            const int64_t w = (i - j0 + 1) < nb ? (i - j0 + 1) : nb;
            for (int64_t jj = 0; jj < w; jj++) t[jj] = Li[j0 + jj];
            for (int64_t p = 0; p < j0; p++) {
                const T lip = Li[p];
                const T* wp = Wt + p * PB;
                for (int64_t jj = 0; jj < w; jj++) t[jj] -= lip * wp[jj];
            }
            for (int64_t jj = 0; jj < w; jj++) Li[j0 + jj] = t[jj];
        }
        /* Phase 2a: the diagonal block, column by column (p = j0 .. j-1). */
        for (int64_t j = j0; j < j0 + nb; j++) {
            T* Lj = L + j * n;
            T s = Lj[j];
            for (int64_t p = j0; p < j; p++) s -= Lj[p] * Lj[p];
            if (!(s > (T)0)) {
                free(Wt);
                return j + 1;
            }
            const T d = SQRT_T(s);
            Lj[j] = d;
            for (int64_t i = j + 1; i < j0 + nb; i++) {
                T* Li = L + i * n;
                T t = Li[j];
                for (int64_t p = j0; p < j; p++) t -= Li[p] * Lj[p];
                Li[j] = t / d;
            }
        }
        /* Phase 2b: the rows below the block, each finishing the panel's columns in order. */
#pragma omp parallel for schedule(static) if ((n - j0 - nb) * nb > 4096)
        for (int64_t i = j0 + nb; i < n; i++) {
            T* Li = L + i * n;
            for (int64_t j = j0; j < j0 + nb; j++) {
                const T* Lj = L + j * n;
                T t = Li[j];
                for (int64_t p = j0; p < j; p++) t -= Li[p] * Lj[p];
                Li[j] = t / Lj[j];
            }
        }
    }
    free(Wt);
    for (int64_t i = 0; i < n; i++)
        for (int64_t j = i + 1; j < n; j++) L[i * n + j] = (T)0;
    return 0;
}
#undef PB

/* _dense_chol_L (src/dense.jl:46-67): factor, else retry with K + eps*mean(diag) for
 * eps = 1e-9, 1e-8, ..., 1e-2 (the sequence evaluated in T).  Returns 0, or 1 when even 1e-2
 * fails.  *jitter_used receives the eps that succeeded (0 for none). */
int SFX(gpo_dense_chol)(T* L, const T* Kmat, int64_t n, T* jitter_used) {
    memcpy(L, Kmat, sizeof(T) * n * n);
    if (dense_potrf(L, n) == 0) { if (jitter_used) *jitter_used = 0; return 0; }
    T dmean = (T)0;
    for (int64_t i = 0; i < n; i++) dmean += Kmat[i * n + i];
    dmean = dmean / (T)(n > 1 ? n : 1);
    T eps = (T)1e-9;
    while (eps <= (T)1e-2) {
        memcpy(L, Kmat, sizeof(T) * n * n);
        for (int64_t i = 0; i < n; i++) L[i * n + i] = Kmat[i * n + i] + eps * dmean;
        if (dense_potrf(L, n) == 0) { if (jitter_used) *jitter_used = eps; return 0; }
        eps *= (T)10;
    }
    return 1;
}

/* out = L * x (generate_dense, src/dense.jl:112-119). */
int SFX(gpo_trmv_lower)(T* out, const T* L, const T* x, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        T acc = (T)0;
        for (int64_t j = 0; j <= i; j++) acc += L[i * n + j] * x[j];
        out[i] = acc;
    }
    return 0;
}

/* out = L^T * x (dense adjoint of generate_grad_xi, src/grad.jl:448-453). */
int SFX(gpo_trmv_lower_t)(T* out, const T* L, const T* x, int64_t n) {
    for (int64_t j = 0; j < n; j++) {
        T acc = (T)0;
        for (int64_t i = j; i < n; i++) acc += L[i * n + j] * x[i];
        out[j] = acc;
    }
    return 0;
}

/* out = L \ y (generate_dense_inv, src/dense.jl:127-134). */
int SFX(gpo_trsv_lower)(T* out, const T* L, const T* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        T s = y[i];
        for (int64_t j = 0; j < i; j++) s -= L[i * n + j] * out[j];
        out[i] = s / L[i * n + i];
    }
    return 0;
}

/* chol_pullback_dyn! (src/grad_generate_vals.jl:18-39) on an n x n lower factor. */
int SFX(gpo_chol_pullback_dense)(T* Abar, T* Lbar, const T* L, int64_t n) {
    chol_pullback(Abar, Lbar, L, (int)n);
    return 0;
}

/* Dense block of generate_grad_vals (src/grad_generate_vals.jl:188-210): Lbar = tril(vb xi^T),
 * pullback, scatter into dv (accumulated into the caller's double array). */
int SFX(gpo_dense_grad_vals)(double* dv, const T* L, const T* vb, const T* xi,
                             const uint32_t* coords, int64_t n, int D, T scale, const T* bins,
                             int64_t nb, int acc_t) {
    T* Lbar = (T*)calloc((size_t)n * n, sizeof(T));
    T* Kbar = (T*)calloc((size_t)n * n, sizeof(T));
    for (int64_t j = 0; j < n; j++)
        for (int64_t i = j; i < n; i++) Lbar[i * n + j] = vb[i] * xi[j];
    chol_pullback(Kbar, Lbar, L, (int)n);
    for (int64_t j = 0; j < n; j++) {
        if (acc_t) dv[0] = (double)((T)dv[0] + Kbar[j * n + j]);
        else dv[0] += (double)Kbar[j * n + j];
        for (int64_t i = j + 1; i < n; i++) {
            T r = lattice_radius(coords + i * D, coords + j * D, D, scale);
            T wlo, whi;
            int64_t lo = cov_lookup_weights(r, bins, nb, &wlo, &whi);
            T g = Kbar[i * n + j];
            if (acc_t) {
                dv[lo] = (double)((T)dv[lo] + g * wlo);
                dv[lo + 1] = (double)((T)dv[lo + 1] + g * whi);
            } else {
                dv[lo] += (double)(g * wlo);
                dv[lo + 1] += (double)(g * whi);
            }
        }
    }
    free(Lbar);
    free(Kbar);
    return 0;
}

/* Scatter a dense cotangent given in double (G, n x n row-major: G[i][j], i > j, the pair's
 * cotangent; G[i][i] the diagonal's) into dv through cov_lookup_weights of each pair's radius
 * (the histogram step of src/grad_generate_vals.jl:252-280 and src/dense.jl:153-183).  Used by
 * the blocked dense pullback of oracle.py for large first layers; rows are spread over the host
 * threads, each with a private histogram. */
int SFX(gpo_dense_scatter)(double* dv, const double* G, const uint32_t* coords, int64_t n, int D,
                           T scale, const T* bins, int64_t nb) {
#pragma omp parallel
    {
        double* h = (double*)calloc((size_t)nb, sizeof(double));
#pragma omp for schedule(dynamic, 16)
        for (int64_t i = 0; i < n; i++) {
            h[0] += G[i * n + i];
            for (int64_t j = 0; j < i; j++) {
                T r = lattice_radius(coords + i * D, coords + j * D, D, scale);
                T wlo, whi;
                int64_t lo = cov_lookup_weights(r, bins, nb, &wlo, &whi);
                const double g = G[i * n + j];
                h[lo] += g * (double)wlo;
                h[lo + 1] += g * (double)whi;
            }
        }
#pragma omp critical
        for (int64_t b = 0; b < nb; b++) dv[b] += h[b];
        free(h);
    }
    return 0;
}

/* _dense_logdet_grad_vals (src/dense.jl:153-183): g = K^{-1}[a,b], half on the diagonal. */
int SFX(gpo_dense_logdet_grad_vals)(double* dv, const T* L, const uint32_t* coords, int64_t n,
                                    int D, T scale, const T* bins, int64_t nb, int acc_t) {
    T* Li = (T*)calloc((size_t)n * n, sizeof(T));
    /* Linv = inv(LowerTriangular(L)), column by column (forward substitution on e_j). */
    for (int64_t j = 0; j < n; j++) {
        for (int64_t i = j; i < n; i++) {
            T s = (i == j) ? (T)1 : (T)0;
            for (int64_t p = j; p < i; p++) s -= L[i * n + p] * Li[p * n + j];
            Li[i * n + j] = s / L[i * n + i];
        }
    }
    for (int64_t b = 0; b < n; b++) {
        for (int64_t a = b; a < n; a++) {
            T kinv = (T)0;
            for (int64_t kk = 0; kk < n; kk++) kinv += Li[kk * n + a] * Li[kk * n + b];
            T r = lattice_radius(coords + a * D, coords + b * D, D, scale);
            T wlo, whi;
            int64_t lo = cov_lookup_weights(r, bins, nb, &wlo, &whi);
            T g = (a == b) ? (T)0.5 * kinv : kinv;
            if (acc_t) {
                dv[lo] = (double)((T)dv[lo] + g * wlo);
                dv[lo + 1] = (double)((T)dv[lo + 1] + g * whi);
            } else {
                dv[lo] += (double)(g * wlo);
                dv[lo + 1] += (double)(g * whi);
            }
        }
    }
    free(Li);
    return 0;
}

/* sum(log, diag(L)) (src/dense.jl:142-147). */
double SFX(gpo_dense_logdet)(const T* L, int64_t n) {
    T s = (T)0;
    for (int64_t i = 0; i < n; i++) s += LOG_T(L[i * n + i]);
    return (double)s;
}

/* ---------------------------------------------------------------------------------------- */
/* Point-position gradients (src/grad.jl:168-377, src/kernels_adjoint.jl:226-324,            */
/* src/dense.jl:184-297).  d(.)/dx for the continuous positions x = scale * coords, tree      */
/* order, (N, D) row-major (Julia's (D, N) column-major), accumulated in double.               */
/* ---------------------------------------------------------------------------------------- */

/* cov_lookup_dr (src/interp.jl:43-60): the slope of the segment holding r; 0 at and beyond
 * both ends of the table. */
static inline T cov_lookup_dr(T r, const T* bins, const T* vals, int64_t n) {
    if (r <= bins[0] || r >= bins[n - 1]) return (T)0;
    int64_t lo = 0, hi = n - 1;
    while (hi - lo > 1) {
        int64_t mid = (lo + hi) >> 1;
        if (bins[mid] <= r) lo = mid; else hi = mid;
    }
    return (vals[lo + 1] - vals[lo]) / (bins[lo + 1] - bins[lo]);
}

/* One pair's term (src/kernels_adjoint.jl:226-251): c_d = (g * k'(r) / r) * scale * (x_a - x_b)
 * into point a, -c_d into point b; coincident points and flat segments contribute nothing. */
static inline void pair_points(double* dp, T g, const uint32_t* xa, const uint32_t* xb,
                               int64_t ga, int64_t gb, int D, T scale, const T* bins,
                               const T* vals, int64_t nb) {
    int64_t sq = 0;
    for (int d = 0; d < D; d++) {
        int64_t di = (int64_t)xa[d] - (int64_t)xb[d];
        sq += di * di;
    }
    if (sq == 0) return;
    T r = SQRT_T((T)sq) * scale;
    T dcov = cov_lookup_dr(r, bins, vals, nb);
    if (dcov == (T)0) return;
    T factor = g * dcov / r;
    for (int d = 0; d < D; d++) {
        T diff = scale * ((T)(int64_t)xa[d] - (T)(int64_t)xb[d]);
        T c = factor * diff;
        dp[ga * D + d] += (double)c;
        dp[gb * D + d] -= (double)c;
    }
}

/* A refined point's off-diagonal Abar through k'(r) into its K + 1 points (rows 0..K-1 the
 * neighbours, row K the point itself). */
static void scatter_abar_points(double* dp, const T* Abar, const uint32_t* jc, const int64_t* nbm,
                                int64_t fine, int KP1, int D, T scale, const T* bins,
                                const T* vals, int64_t nb) {
    int K = KP1 - 1;
    for (int a = 1; a < KP1; a++) {
        int64_t ga = a < K ? nbm[a] : fine;
        for (int b = 0; b < a; b++) {
            int64_t gb = b < K ? nbm[b] : fine;
            pair_points(dp, Abar[a * KP1 + b], jc + a * D, jc + b * D, ga, gb, D, scale, bins,
                        vals, nb);
        }
    }
}

/* refine_logdet_grad_points (src/grad.jl:186-233): seed 1 / L[K][K], chol_pullback, scatter. */
int SFX(gpo_refine_logdet_grad_points)(double* dp, const uint32_t* coords, const int64_t* nbrs,
                                       int64_t M, int64_t n0, int K, int D, T scale,
                                       const T* bins, const T* vals, int64_t nb) {
    if (K > KMAX || D > DMAX) return 2;
    int KP1 = K + 1;
    T* A = (T*)malloc(sizeof(T) * KP1 * KP1 * 3);
    T* Abar = A + KP1 * KP1;
    T* Lbar = Abar + KP1 * KP1;
    uint32_t jc[(KMAX + 1) * DMAX];
    for (int64_t m = 0; m < M; m++) {
        point_factor(A, NULL, jc, coords, nbrs, m, n0, K, D, scale, bins, vals, nb);
        for (int i = 0; i < KP1 * KP1; i++) Lbar[i] = (T)0;
        Lbar[K * KP1 + K] = (T)1 / A[K * KP1 + K];
        chol_pullback(Abar, Lbar, A, KP1);
        scatter_abar_points(dp, Abar, jc, nbrs + m * K, n0 + m, KP1, D, scale, bins, vals, nb);
    }
    free(A);
    return 0;
}

/* refine_inv_loss_grad_points (src/grad.jl:259-358): the seeds of the inverse-loss vals
 * gradient (no pivot guard in the z-bar solve), chol_pullback, scatter into the points. */
int SFX(gpo_refine_inv_loss_grad_points)(double* dp, const T* values, const uint32_t* coords,
                                         const int64_t* nbrs, int64_t M, int64_t n0, int K, int D,
                                         T scale, const T* bins, const T* vals, int64_t nb) {
    if (K > KMAX || D > DMAX) return 2;
    int KP1 = K + 1;
    T* A = (T*)malloc(sizeof(T) * KP1 * KP1 * 3);
    T* Abar = A + KP1 * KP1;
    T* Lbar = Abar + KP1 * KP1;
    T mv[KMAX], zbar[KMAX];
    uint32_t jc[(KMAX + 1) * DMAX];
    for (int64_t m = 0; m < M; m++) {
        T sd = point_factor(A, mv, jc, coords, nbrs, m, n0, K, D, scale, bins, vals, nb);
        T mean = (T)0;
        for (int j = 0; j < K; j++) mean += mv[j] * values[nbrs[m * K + j]];
        T xim = (values[n0 + m] - mean) / sd;
        for (int i = 0; i < KP1 * KP1; i++) Lbar[i] = (T)0;
        Lbar[K * KP1 + K] = -xim * xim / sd;
        for (int j = 0; j < K; j++) zbar[j] = -xim * values[nbrs[m * K + j]] / sd;
        for (int i = 0; i < K; i++) {
            T s = zbar[i];
            for (int p = 0; p < i; p++) s -= A[i * KP1 + p] * zbar[p];
            zbar[i] = s / A[i * KP1 + i];
        }
        for (int j = 0; j < K; j++) {
            Lbar[K * KP1 + j] += zbar[j];
            for (int i = 0; i <= j; i++) Lbar[j * KP1 + i] -= zbar[i] * mv[j];
        }
        chol_pullback(Abar, Lbar, A, KP1);
        scatter_abar_points(dp, Abar, jc, nbrs + m * K, n0 + m, KP1, D, scale, bins, vals, nb);
    }
    free(A);
    return 0;
}

/* The dense block's position gradients (src/dense.jl:188-225, 271-297): the off-diagonal
 * cotangent g[a][b] (a > b) through k'(r) into points a and b.  mode 0: g = K^{-1}[a][b] from
 * the block's factor L (row-major lower); mode 1: g = -alpha[a] * alpha[b] with
 * alpha = L^{-T} L^{-1} y. */
int SFX(gpo_dense_grad_points)(double* dp, const T* L, const T* y, const uint32_t* coords,
                               int64_t n, int D, T scale, const T* bins, const T* vals,
                               int64_t nb, int mode) {
    T* Li = NULL;
    T* alpha = NULL;
    if (mode == 0) {
        Li = (T*)calloc((size_t)n * n, sizeof(T));
        for (int64_t j = 0; j < n; j++)
            for (int64_t i = j; i < n; i++) {
                T s = (i == j) ? (T)1 : (T)0;
                for (int64_t p = j; p < i; p++) s -= L[i * n + p] * Li[p * n + j];
                Li[i * n + j] = s / L[i * n + i];
            }
    } else {
        T* xi = (T*)malloc(sizeof(T) * n);
        alpha = (T*)malloc(sizeof(T) * n);
        for (int64_t i = 0; i < n; i++) {
            T s = y[i];
            for (int64_t p = 0; p < i; p++) s -= L[i * n + p] * xi[p];
            xi[i] = s / L[i * n + i];
        }
        for (int64_t i = n - 1; i >= 0; i--) {
            T s = xi[i];
            for (int64_t p = i + 1; p < n; p++) s -= L[p * n + i] * alpha[p];
            alpha[i] = s / L[i * n + i];
        }
        free(xi);
    }
    for (int64_t b = 0; b < n; b++)
        for (int64_t a = b + 1; a < n; a++) {
            T g;
            if (mode == 0) {
                g = (T)0;
                for (int64_t kk = 0; kk < n; kk++) g += Li[kk * n + a] * Li[kk * n + b];
            } else {
                g = -alpha[a] * alpha[b];
            }
            pair_points(dp, g, coords + a * D, coords + b * D, a, b, D, scale, bins, vals, nb);
        }
    free(Li);
    free(alpha);
    return 0;
}
