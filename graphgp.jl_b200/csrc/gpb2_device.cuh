// gpb2_device.cuh -- per-point Vecchia numerics for sm_100a, one thread per refined point.
//
// Each refined point conditions on its K nearest preceding neighbours.  A thread gathers the
// (K+1) lattice coordinates, assembles the (K+1)x(K+1) covariance by table interpolation,
// factorises it (left-looking Cholesky with the reference's pivot floor), solves for the
// conditional-mean weights and, for the adjoints, runs the exact reverse of the factorisation.
// The packed lower triangle lives in registers (all loops are unrolled over the compile-time K).
//
// Arithmetic: every operation is an explicit round-to-nearest IEEE operation (__fmul_rn,
// __fadd_rn, __fdiv_rn, __fsqrt_rn and the double forms) in the written order, so nothing is
// contracted into an FMA and each point's result is the same bit pattern the scalar restatement
// produces.  Operation order follows:
//   cov_lookup / cov_lookup_weights     src/interp.jl:10-34, 62-83
//   assemble_cov!                       src/linalg.jl:15-29
//   chol_lower!                         src/linalg.jl:38-73
//   mean_vec_solve!                     src/linalg.jl:85-103
//   chol_pullback!                      src/linalg.jl:112-134
//
// Interpolation table.  The reference finds the bracketing bin with a binary search (about
// log2(nbins) dependent loads per covariance entry).  Here the table is staged in shared memory
// as segments {x0, x1, y0, slope} with slope = (y1 - y0) / (x1 - x0) evaluated once per segment
// in T (the same IEEE quotient the reference forms per lookup), plus a bucket index keyed on the
// high bits of r's IEEE representation (monotone in r for r > 0).  A lookup reads the bucket's
// first segment and steps forward while x1 <= r: the bracket found is the unique lo with
// bins[lo] <= r < bins[lo+1], i.e. exactly the binary search's, for any strictly increasing
// table.  The interpolated value is y0 + slope*(r - x0) in that order, as in the reference.
#pragma once
#include <cfloat>
#include <cstdint>
#include <cuda_runtime.h>
#include <type_traits>

namespace gpb2 {

// ------------------------------------------------------------------------------------------
// IEEE round-to-nearest arithmetic that the compiler may not contract.
// ------------------------------------------------------------------------------------------
template <typename T> struct Num;

template <> struct Num<float> {
    using U = uint32_t;
    static __device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
    static __device__ __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }
    static __device__ __forceinline__ float sub(float a, float b) { return __fsub_rn(a, b); }
    static __device__ __forceinline__ float div(float a, float b) { return __fdiv_rn(a, b); }
    static __device__ __forceinline__ float sqrt(float a) { return __fsqrt_rn(a); }
    // c - a*b with one rounding (adjoint arithmetic only: not part of any exact-order path)
    static __device__ __forceinline__ float fms(float a, float b, float c) { return fmaf(-a, b, c); }
    static __device__ __forceinline__ float div_fast(float a, float b) { return __fdividef(a, b); }
    // a / b rounded to nearest, given r = RN(1/b): Markstein's correction q0 = RN(a r),
    // e = a - q0 b (exact with one fused multiply-add), q = RN(q0 + e r) is the correctly rounded
    // quotient when nothing over- or underflows; operands outside a safe exponent window (and a
    // zero dividend, whose sign the sequence would lose) take the IEEE division itself.
    static __device__ __forceinline__ float div_r(float a, float b, float r) {
        const float q0 = __fmul_rn(a, r);
        const float e = __fmaf_rn(-q0, b, a);
        const float q = __fmaf_rn(e, r, q0);
        const unsigned ea = (__float_as_uint(a) >> 23) & 0xffu, eb = (__float_as_uint(b) >> 23) & 0xffu;
        const bool safe = (ea - 31u) < 130u && (eb - 97u) < 60u;  // |a| in [2^-96, 2^34), b in [2^-30, 2^30)
        return safe ? q : __fdiv_rn(a, b);
    }
    // The corrected quotient of div_r without its per-operation range check, for callers that
    // check a whole point's operands at once (DivChecked): exact when quot_a_ok(a) and b and 2b
    // pass quot_b_ok, div_r's window.
    static __device__ __forceinline__ float div_q(float a, float b, float r) {
        const float q0 = __fmul_rn(a, r);
        const float e = __fmaf_rn(-q0, b, a);
        return __fmaf_rn(e, r, q0);
    }
    static __device__ __forceinline__ bool quot_a_ok(float a) {
        return (((__float_as_uint(a) >> 23) & 0xffu) - 31u) < 130u;
    }
    static __device__ __forceinline__ bool quot_b_ok(float b) {
        return (((__float_as_uint(b) >> 23) & 0xffu) - 97u) < 60u;
    }
    // RN(1 / a): the same bits as div(1, a).
    static __device__ __forceinline__ float rcp(float a) { return __frcp_rn(a); }
    static __device__ __forceinline__ float log(float a) { return logf(a); }
    static __device__ __forceinline__ float from_i64(long long x) { return __ll2float_rn(x); }
    static __device__ __forceinline__ U bits(float x) { return __float_as_uint(x); }
    static __host__ __device__ constexpr float eps() { return FLT_EPSILON; }
};

template <> struct Num<double> {
    using U = unsigned long long;
    static __device__ __forceinline__ double mul(double a, double b) { return __dmul_rn(a, b); }
    static __device__ __forceinline__ double add(double a, double b) { return __dadd_rn(a, b); }
    static __device__ __forceinline__ double sub(double a, double b) { return __dsub_rn(a, b); }
    static __device__ __forceinline__ double div(double a, double b) { return __ddiv_rn(a, b); }
    static __device__ __forceinline__ double sqrt(double a) { return __dsqrt_rn(a); }
    static __device__ __forceinline__ double fms(double a, double b, double c) {
        return fma(-a, b, c);
    }
    static __device__ __forceinline__ double div_fast(double a, double b) { return a / b; }
    static __device__ __forceinline__ double div_r(double a, double b, double r) {
        const double q0 = __dmul_rn(a, r);
        const double e = __fma_rn(-q0, b, a);
        const double q = __fma_rn(e, r, q0);
        const unsigned long long ua = (unsigned long long)__double_as_longlong(a);
        const unsigned long long ub = (unsigned long long)__double_as_longlong(b);
        const unsigned ea = (unsigned)((ua >> 52) & 0x7ffu), eb = (unsigned)((ub >> 52) & 0x7ffu);
        const bool safe = (ea - 223u) < 1024u && (eb - 923u) < 200u;  // |a| in [2^-800, 2^224), b in [2^-100, 2^100)
        return safe ? q : __ddiv_rn(a, b);
    }
    static __device__ __forceinline__ double div_q(double a, double b, double r) {
        const double q0 = __dmul_rn(a, r);
        const double e = __fma_rn(-q0, b, a);
        return __fma_rn(e, r, q0);
    }
    static __device__ __forceinline__ bool quot_a_ok(double a) {
        const unsigned long long u = (unsigned long long)__double_as_longlong(a);
        return ((unsigned)((u >> 52) & 0x7ffu) - 223u) < 1024u;
    }
    static __device__ __forceinline__ bool quot_b_ok(double b) {
        const unsigned long long u = (unsigned long long)__double_as_longlong(b);
        return ((unsigned)((u >> 52) & 0x7ffu) - 923u) < 200u;
    }
    static __device__ __forceinline__ double rcp(double a) { return __drcp_rn(a); }
    static __device__ __forceinline__ double log(double a) { return ::log(a); }
    static __device__ __forceinline__ double from_i64(long long x) { return __ll2double_rn(x); }
    static __device__ __forceinline__ U bits(double x) {
        return (unsigned long long)__double_as_longlong(x);
    }
    static __host__ __device__ constexpr double eps() { return DBL_EPSILON; }
};

// Storage of a point's pair radii (kept by the adjoint kernels for their histogram scatter):
// registers (compile-time indices), or the thread's column of a shared-memory block, which
// frees registers for occupancy.
template <typename T, int NR>
struct RegArr {
    T v[NR];
    __device__ __forceinline__ T& operator[](int i) { return v[i]; }
    __device__ __forceinline__ const T& operator[](int i) const { return v[i]; }
};
template <typename T>
struct SmemCol {
    T* p = nullptr;
    int stride = 0;
    __device__ __forceinline__ T& operator[](int i) const { return p[i * stride]; }
};
// Per-thread columns of interpolation weights in shared memory: for entry i, the segment index
// lo[i] and the fraction t[i] of the radius across it (w_lo = 1 - t, w_hi = t).  Kept by the
// covariance assembly so the adjoint's histogram scatter needs no second table search.
template <typename T>
struct SmemWeights {
    T* t = nullptr;
    uint16_t* lo = nullptr;
    int stride = 0;
};
// The same weights in the problem's factor cache: one slab of M entries per pair (entry i of
// point m at [i * stride + m], so a warp's 32 points read one contiguous run per entry).
template <typename T>
struct SlabWeights {
    T* t = nullptr;
    uint16_t* lo = nullptr;
    int64_t stride = 0;
};
template <typename RT>
struct is_weight_store : std::false_type {};
template <typename T>
struct is_weight_store<SmemWeights<T>> : std::true_type {};
template <typename T>
struct is_weight_store<SlabWeights<T>> : std::true_type {};

// ------------------------------------------------------------------------------------------
// Interpolation table (built on the host by the problem handle, see gpb2_problem.cu).
// ------------------------------------------------------------------------------------------
template <typename T>
struct TableView {
    const T* seg;              // device, 4 * (nb - 1): {x0, x1, y0, slope} per segment
    const uint16_t* start;     // device, nkeys: first segment to probe for each bucket
    typename Num<T>::U base;   // bucket of bins[1]
    int nb, nkeys, shift;
    T b0, b1, bN, v0, vN;      // bins[0], bins[1], bins[nb-1], vals[0], vals[nb-1]
    T pivc;                    // T(1.5) * sqrt(eps(T)), evaluated in T on the host
};

// Anisotropic covariance K(d_spatial, d_z) (src/aniso.jl): grid[i + j * ns] =
// K(spatial_bins[i], z_bins[j]) (the reference's (ns, nz) column-major grid), bilinear at the
// fractional bin indices of the two separations.  grid == nullptr: the isotropic table.
template <typename T>
struct AnisoView {
    const T* sb = nullptr;
    const T* zb = nullptr;
    const T* grid = nullptr;
    int ns = 0, nz = 0;
    T alpha = T(1);

    // _frac_index (src/aniso.jl:42-57): 0-based, clamped to [0, n - 1].
    static __device__ __forceinline__ T frac_index(T d, const T* __restrict__ bins, int n) {
        using N = Num<T>;
        if (d <= __ldg(bins)) return T(0);
        if (d >= __ldg(bins + n - 1)) return T(n - 1);
        int lo = 0, hi = n - 1;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (__ldg(bins + mid) <= d) lo = mid; else hi = mid;
        }
        const T x0 = __ldg(bins + lo), x1 = __ldg(bins + lo + 1);
        return N::add(T(lo), N::div(N::sub(d, x0), N::sub(x1, x0)));
    }

    // aniso_lookup (src/aniso.jl:67-85), in its operation order.
    __device__ __forceinline__ T lookup(T ds, T dz) const {
        using N = Num<T>;
        const T fx = frac_index(ds, sb, ns), fz = frac_index(dz, zb, nz);
        const int i0 = (int)fx, j0 = (int)fz;  // truncation = floor: both are >= 0
        const int i1 = i0 + 1 < ns ? i0 + 1 : ns - 1;
        const int j1 = j0 + 1 < nz ? j0 + 1 : nz - 1;
        const T tx = N::sub(fx, T(i0)), tz = N::sub(fz, T(j0));
        const T ux = N::sub(T(1), tx), uz = N::sub(T(1), tz);
        const T g00 = __ldg(grid + i0 + j0 * ns), g10 = __ldg(grid + i1 + j0 * ns);
        const T g01 = __ldg(grid + i0 + j1 * ns), g11 = __ldg(grid + i1 + j1 * ns);
        return N::add(N::mul(N::add(N::mul(g00, ux), N::mul(g10, tx)), uz),
                      N::mul(N::add(N::mul(g01, ux), N::mul(g11, tx)), tz));
    }

    // The pair's separations (src/aniso.jl:88-105): spatial over the first D - 1 coordinates,
    // radial |dz| * scale / alpha over the last; squares summed exactly (modulo 2^64, as Int64).
    template <int D>
    __device__ __forceinline__ T pair(const uint32_t (&a)[D], const uint32_t (&b)[D],
                                      T scale) const {
        using N = Num<T>;
        unsigned long long sq = 0;
#pragma unroll
        for (int d = 0; d < D - 1; d++) {
            const uint32_t di = a[d] > b[d] ? a[d] - b[d] : b[d] - a[d];
            sq += (unsigned long long)di * di;
        }
        const long long dzi = (long long)a[D - 1] - (long long)b[D - 1];
        const T ds = N::mul(N::sqrt(N::from_i64((long long)sq)), scale);
        const T dz = N::div(N::mul(N::from_i64(dzi < 0 ? -dzi : dzi), scale), alpha);
        return lookup(ds, dz);
    }
    // The same for coordinates in memory and a run-time D (the dense block's assembly).
    __device__ __forceinline__ T pair_rt(const uint32_t* __restrict__ a,
                                         const uint32_t* __restrict__ b, int D, T scale) const {
        using N = Num<T>;
        unsigned long long sq = 0;
        for (int d = 0; d < D - 1; d++) {
            const uint32_t di = a[d] > b[d] ? a[d] - b[d] : b[d] - a[d];
            sq += (unsigned long long)di * di;
        }
        const long long dzi = (long long)a[D - 1] - (long long)b[D - 1];
        const T ds = N::mul(N::sqrt(N::from_i64((long long)sq)), scale);
        const T dz = N::div(N::mul(N::from_i64(dzi < 0 ? -dzi : dzi), scale), alpha);
        return lookup(ds, dz);
    }
};

// Bytes of dynamic shared memory a kernel needs for the staged table.
template <typename T>
__host__ __device__ inline size_t table_smem_bytes(int nb, int nkeys) {
    size_t segb = sizeof(T) * 4 * (size_t)(nb - 1);
    size_t keyb = ((sizeof(uint16_t) * (size_t)nkeys) + 15) & ~size_t(15);
    return segb + keyb;
}

template <typename T>
struct SmemTable {
    using N = Num<T>;
    using U = typename N::U;
    const T* seg;
    const uint16_t* start;
    U base;
    int nb, last_key, shift;
    T b0, b1, bN, v0, vN;

    // Cooperative copy of the table into shared memory; the caller synchronises afterwards.
    __device__ __forceinline__ void stage(const TableView<T>& tv, unsigned char* smem, int tid,
                                          int nthr) {
        const int nseg4 = 4 * (tv.nb - 1);
        T* s = reinterpret_cast<T*>(smem);
        const int nvec = (int)((sizeof(T) * nseg4) / 16);
        const int4* src = reinterpret_cast<const int4*>(tv.seg);
        int4* dst = reinterpret_cast<int4*>(s);
        for (int i = tid; i < nvec; i += nthr) dst[i] = __ldg(src + i);
        uint16_t* st = reinterpret_cast<uint16_t*>(smem + sizeof(T) * nseg4);
        for (int i = tid; i < tv.nkeys; i += nthr) st[i] = __ldg(tv.start + i);
        seg = s;
        start = st;
        base = tv.base;
        nb = tv.nb;
        last_key = tv.nkeys - 1;
        shift = tv.shift;
        b0 = tv.b0; b1 = tv.b1; bN = tv.bN; v0 = tv.v0; vN = tv.vN;
    }

    // Segment index lo with bins[lo] <= r < bins[lo+1]; requires bins[0] < r < bins[nb-1].
    __device__ __forceinline__ int locate(T r) const {
        if (r < b1) return 0;
        U key = (N::bits(r) >> shift) - base;
        int ki = key > (U)last_key ? last_key : (int)key;
        int lo = start[ki];
        while (seg[4 * lo + 1] <= r) ++lo;  // terminates: seg[nb-2].x1 == bins[nb-1] > r
        return lo;
    }

    // cov_lookup (src/interp.jl:10-34).
    __device__ __forceinline__ T lookup(T r) const {
        if (r <= b0) return v0;
        if (r >= bN) return vN;
        const int lo = locate(r);
        const T x0 = seg[4 * lo + 0];
        const T y0 = seg[4 * lo + 2];
        const T slope = seg[4 * lo + 3];
        return N::add(y0, N::mul(slope, N::sub(r, x0)));
    }

    // cov_lookup_dr (src/interp.jl:43-60): the slope of the segment holding r, 0 at and beyond
    // both ends of the table.
    __device__ __forceinline__ T dr(T r) const {
        if (r <= b0 || r >= bN) return T(0);
        return seg[4 * locate(r) + 3];
    }

    // cov_lookup_weights (src/interp.jl:62-83): returns lo, writes w_lo and w_hi.
    __device__ __forceinline__ int weights(T r, T& wlo, T& whi) const {
        if (r <= b0) { wlo = T(1); whi = T(0); return 0; }
        if (r >= bN) { wlo = T(0); whi = T(1); return nb - 2; }
        const int lo = locate(r);
        const T x0 = seg[4 * lo + 0];
        const T x1 = seg[4 * lo + 1];
        const T t = N::div(N::sub(r, x0), N::sub(x1, x0));
        wlo = N::sub(T(1), t);
        whi = t;
        return lo;
    }
    // lookup() that also returns weights()'s segment and fraction t (w_lo = 1 - t, w_hi = t),
    // from the same segment search: the value and both weights bit for bit as the two calls.
    __device__ __forceinline__ T lookup_w(T r, int& lo_out, T& t_out) const {
        if (r <= b0) { lo_out = 0; t_out = T(0); return v0; }
        if (r >= bN) { lo_out = nb - 2; t_out = T(1); return vN; }
        const int lo = locate(r);
        const T x0 = seg[4 * lo + 0];
        const T x1 = seg[4 * lo + 1];
        const T y0 = seg[4 * lo + 2];
        const T slope = seg[4 * lo + 3];
        lo_out = lo;
        t_out = N::div(N::sub(r, x0), N::sub(x1, x0));
        return N::add(y0, N::mul(slope, N::sub(r, x0)));
    }

};

// ------------------------------------------------------------------------------------------
// Device-side layout helpers.
// ------------------------------------------------------------------------------------------

// Row stride (uint32 words) of the device coordinate copy: D = 3 is padded to 16 bytes so a
// point's coordinates are one aligned vector load that never straddles a 32-byte sector.
__host__ __device__ constexpr int coord_stride(int D) { return D == 3 ? 4 : D; }

template <int D>
__device__ __forceinline__ void load_coords(uint32_t (&c)[D], const uint32_t* __restrict__ coords,
                                            int64_t p) {
    constexpr int DS = coord_stride(D);
    if constexpr (D == 2) {
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(coords) + p);
        c[0] = v.x; c[1] = v.y;
    } else if constexpr (DS == 4) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(coords) + p);
        c[0] = v.x; c[1] = v.y; c[2] = v.z;
        if constexpr (D == 4) c[3] = v.w;
    } else {
#pragma unroll
        for (int d = 0; d < D; d++) c[d] = __ldg(coords + p * DS + d);
    }
}

// K consecutive int32 (a refined point's neighbour list), vectorised when K allows.
template <int K>
__device__ __forceinline__ void load_row_i32(int (&o)[K], const int* __restrict__ base) {
    if constexpr (K % 4 == 0) {
#pragma unroll
        for (int j = 0; j < K / 4; j++) {
            const int4 v = __ldg(reinterpret_cast<const int4*>(base) + j);
            o[4 * j] = v.x; o[4 * j + 1] = v.y; o[4 * j + 2] = v.z; o[4 * j + 3] = v.w;
        }
    } else if constexpr (K % 2 == 0) {
#pragma unroll
        for (int j = 0; j < K / 2; j++) {
            const int2 v = __ldg(reinterpret_cast<const int2*>(base) + j);
            o[2 * j] = v.x; o[2 * j + 1] = v.y;
        }
    } else {
#pragma unroll
        for (int j = 0; j < K; j++) o[j] = __ldg(base + j);
    }
}

// K consecutive T (a point's conditional-mean weights).
template <typename T, int K>
__device__ __forceinline__ void load_row_t(T (&o)[K], const T* __restrict__ base) {
    constexpr int PER = 16 / sizeof(T);
    if constexpr (K % PER == 0) {
#pragma unroll
        for (int j = 0; j < K / PER; j++) {
            const int4 v = __ldg(reinterpret_cast<const int4*>(base) + j);
            const T* t = reinterpret_cast<const T*>(&v);
#pragma unroll
            for (int q = 0; q < PER; q++) o[PER * j + q] = t[q];
        }
    } else {
#pragma unroll
        for (int j = 0; j < K; j++) o[j] = __ldg(base + j);
    }
}

template <typename T, int K>
__device__ __forceinline__ void store_row_t(T* __restrict__ base, const T (&o)[K]) {
    constexpr int PER = 16 / sizeof(T);
    if constexpr (K % PER == 0) {
#pragma unroll
        for (int j = 0; j < K / PER; j++) {
            int4 v;
            T* t = reinterpret_cast<T*>(&v);
#pragma unroll
            for (int q = 0; q < PER; q++) t[q] = o[PER * j + q];
            reinterpret_cast<int4*>(base)[j] = v;
        }
    } else {
#pragma unroll
        for (int j = 0; j < K; j++) base[j] = o[j];
    }
}

// ------------------------------------------------------------------------------------------
// The per-point factorisation.  Loop nests use sfor (compile-time recursion) rather than
// `#pragma unroll`, so every index into the packed triangle is a constant and the arrays stay in
// registers whatever the unroller's size heuristics decide.
// ------------------------------------------------------------------------------------------
__host__ __device__ constexpr int tri(int i, int j) { return i * (i + 1) / 2 + j; }

template <int B, int E, class F>
__device__ __forceinline__ void sfor(F&& f) {
    if constexpr (B < E) {
        f(std::integral_constant<int, B>{});
        sfor<B + 1, E>(f);
    }
}
// Descending: E-1, E-2, ..., B.
template <int B, int E, class F>
__device__ __forceinline__ void sfor_down(F&& f) {
    if constexpr (B < E) {
        f(std::integral_constant<int, E - 1>{});
        sfor_down<B, E - 1>(f);
    }
}
#define GPB2_CI(name) constexpr int name = decltype(name##_)::value

// Division policies of the adjoint arithmetic (forward_subst, pullback), both giving the
// correctly rounded quotient a / b from r = RN(1/b).  DivExact: div_r, whose range check and IEEE
// fallback come with every division.  DivChecked: the bare corrected quotient (div_q), each
// dividend's exponent tested against div_r's window into one flag; ok() then adds the pivots
// (the divisors L[j][j] and 2 L[j][j]) and says whether every operation of the point lay in the
// window where div_q is exact.  A point that fails is redone with DivExact (rare: clamped
// pivots, zero or extreme cotangents), so the results are DivExact's bit for bit.  The window
// is tested on the exponent bits, exactly as div_r tests it.
template <typename T>
struct DivExact {
    __device__ __forceinline__ T operator()(T a, T b, T r) { return Num<T>::div_r(a, b, r); }
};
template <typename T>
struct DivChecked {
    bool bad = false;
    __device__ __forceinline__ T operator()(T a, T b, T r) {
        bad |= !Num<T>::quot_a_ok(a);
        return Num<T>::div_q(a, b, r);
    }
    template <int KP1, int NT>
    __device__ __forceinline__ bool ok(const T (&L)[NT]) const {
        bool pb = false;
        sfor<0, KP1>([&](auto j_) {
            GPB2_CI(j);
            pb |= !Num<T>::quot_b_ok(L[tri(j, j)]) || !Num<T>::quot_b_ok(Num<T>::mul(T(2), L[tri(j, j)]));
        });
        return !bad && !pb;
    }
};

template <typename T, int K, int D>
struct PointMath {
    using N = Num<T>;
    static constexpr int KP1 = K + 1;
    static constexpr int NT = KP1 * (KP1 + 1) / 2;
    static constexpr int NR = NT - KP1;  // off-diagonal pairs

    // Joint coordinates: rows 0..K-1 are the neighbours, row K the refined point
    // (_gather_joint!, src/kernels.jl:9-23).
    static __device__ __forceinline__ void gather(uint32_t (&jc)[KP1][D],
                                                  const uint32_t* __restrict__ coords,
                                                  const int (&nb)[K], int64_t self) {
        sfor<0, K>([&](auto j_) {
            GPB2_CI(j);
            load_coords<D>(jc[j], coords, nb[j]);
        });
        load_coords<D>(jc[K], coords, self);
    }

    // r = sqrt(T(sq)) * scale with sq the exact Int64 squared lattice distance.  The squares are
    // formed as |a - b|^2 from 32-bit differences by one widening multiply-add each; the sum
    // wraps modulo 2^64 exactly as the Int64 sum of (a - b)^2 does, so sq has the same bits.
    static __device__ __forceinline__ T radius(const uint32_t (&a)[D], const uint32_t (&b)[D],
                                               T scale) {
        unsigned long long sq = 0;
        sfor<0, D>([&](auto d_) {
            GPB2_CI(d);
            const uint32_t di = a[d] > b[d] ? a[d] - b[d] : b[d] - a[d];
            sq += (unsigned long long)di * di;
        });
        return N::mul(N::sqrt(N::from_i64((long long)sq)), scale);
    }

    // assemble_cov! (src/linalg.jl:15-29).  With KEEP_R the radius of pair (a, b), b < a, is
    // kept in R[tri(a-1, b)] for the adjoint's scatter -- or, with a weight store, its
    // interpolation segment and fraction.
    template <bool KEEP_R, typename RT>
    static __device__ __forceinline__ void assemble(T (&L)[NT], RT& R,
                                                    const uint32_t (&jc)[KP1][D], T scale,
                                                    const SmemTable<T>& tab) {
        const T diag = tab.lookup(T(0));
        sfor<0, KP1>([&](auto a_) {
            GPB2_CI(a);
            L[tri(a, a)] = diag;
            sfor<0, a>([&](auto b_) {
                GPB2_CI(b);
                const T r = radius(jc[a], jc[b], scale);
                if constexpr (KEEP_R && is_weight_store<RT>::value) {
                    int lo;
                    T t;
                    L[tri(a, b)] = tab.lookup_w(r, lo, t);
                    const auto i = tri(a - 1, b) * R.stride;
                    R.lo[i] = (uint16_t)lo;
                    R.t[i] = t;
                } else {
                    if constexpr (KEEP_R) R[tri(a - 1, b)] = r;
                    L[tri(a, b)] = tab.lookup(r);
                }
            });
        });
    }

    // assemble_cov! for an anisotropic covariance (src/aniso.jl:88-105).
    static __device__ __forceinline__ void assemble_aniso(T (&L)[NT], const uint32_t (&jc)[KP1][D],
                                                          T scale, const AnisoView<T>& av) {
        const T diag = av.lookup(T(0), T(0));
        sfor<0, KP1>([&](auto a_) {
            GPB2_CI(a);
            L[tri(a, a)] = diag;
            sfor<0, a>([&](auto b_) {
                GPB2_CI(b);
                L[tri(a, b)] = av.template pair<D>(jc[a], jc[b], scale);
            });
        });
    }

    // chol_lower! (src/linalg.jl:38-73).  A degenerate column (s <= eps*A11, or NaN) gets
    // the diagonal sqrt(eps*A11) and a zeroed column; selects keep the thread branch-free.
    static __device__ __forceinline__ void chol(T (&L)[NT]) {
        const T pivmin = N::mul(N::eps(), L[0]);
        sfor<0, KP1>([&](auto j_) {
            GPB2_CI(j);
            T s = L[tri(j, j)];
            sfor<0, j>([&](auto p_) {
                GPB2_CI(p);
                s = N::sub(s, N::mul(L[tri(j, p)], L[tri(j, p)]));
            });
            const bool ok = s > pivmin;
            const T d = N::sqrt(ok ? s : pivmin);
            L[tri(j, j)] = d;
            // t / d for the column's entries: the correctly rounded quotients, from one rounded
            // reciprocal of the pivot (div_r), the same bits as the IEEE divisions.
            const T rd = N::rcp(d);
            sfor<j + 1, KP1>([&](auto i_) {
                GPB2_CI(i);
                T t = L[tri(i, j)];
                sfor<0, j>([&](auto p_) {
                    GPB2_CI(p);
                    t = N::sub(t, N::mul(L[tri(i, p)], L[tri(j, p)]));
                });
                L[tri(i, j)] = ok ? N::div_r(t, d, rd) : T(0);
            });
        });
    }

    // mean_vec_solve! (src/linalg.jl:85-103): L[0:K,0:K]^T x = L[K,0:K], weight zeroed where
    // the pivot sits at the clamp floor.
    static __device__ __forceinline__ void solve(T (&x)[K], const T (&L)[NT], T pivc) {
        const T pivfloor = N::mul(pivc, L[0]);
        sfor_down<0, K>([&](auto i_) {
            GPB2_CI(i);
            const T d = L[tri(i, i)];
            T s = L[tri(K, i)];
            sfor<i + 1, K>([&](auto j_) {
                GPB2_CI(j);
                s = N::sub(s, N::mul(L[tri(j, i)], x[j]));
            });
            x[i] = d > pivfloor ? N::div(s, d) : T(0);
        });
    }

    // Reciprocals of the factor's pivots (the adjoint arithmetic below multiplies by them).
    static __device__ __forceinline__ void pivot_recips(T (&rp)[KP1], const T (&L)[NT]) {
        sfor<0, KP1>([&](auto j_) {
            GPB2_CI(j);
            rp[j] = N::rcp(L[tri(j, j)]);
        });
    }

    // Adjoint of mean_vec_solve!: forward substitution L[0:K,0:K] z = z_in, optionally with
    // the pivot guard (src/kernels_adjoint.jl:520-530) or without it (src/grad.jl:574-580).
    // The adjoint arithmetic (here and in seed_from_solve / pullback) is the reference's
    // operation order with every operation rounded to nearest, as the forward's: each division
    // by a pivot is the correctly rounded quotient (div_r, from the pivot's reciprocal), so a
    // point's cotangents equal the CPU restatement's bit for bit.
    template <bool GUARD, typename Div = DivExact<T>>
    static __device__ __forceinline__ void forward_subst(T (&z)[K], const T (&L)[NT],
                                                         const T (&rp)[KP1], T pivfloor,
                                                         Div&& div = Div()) {
        sfor<0, K>([&](auto i_) {
            GPB2_CI(i);
            T s = z[i];
            sfor<0, i>([&](auto q_) {
                GPB2_CI(q);
                s = N::sub(s, N::mul(L[tri(i, q)], z[q]));
            });
            if constexpr (GUARD)
                z[i] = L[tri(i, i)] > pivfloor ? div(s, L[tri(i, i)], rp[i]) : T(0);
            else
                z[i] = div(s, L[tri(i, i)], rp[i]);
        });
    }

    // Seed of the factor cotangent from the solve's adjoint: B[K][j] += z[j],
    // B[j][i] -= z[i]*mv[j] for i <= j (src/kernels_adjoint.jl:531-536).
    static __device__ __forceinline__ void seed_from_solve(T (&B)[NT], const T (&z)[K],
                                                           const T (&x)[K]) {
        sfor<0, K>([&](auto j_) {
            GPB2_CI(j);
            B[tri(K, j)] = N::add(B[tri(K, j)], z[j]);
            sfor<0, j + 1>([&](auto i_) {
                GPB2_CI(i);
                B[tri(j, i)] = N::sub(B[tri(j, i)], N::mul(z[i], x[j]));
            });
        });
    }

    // chol_pullback! (src/linalg.jl:112-134), in place: on entry B holds L-bar (lower), on
    // exit B holds A-bar.  Each L-bar[i][j] is last read exactly where A-bar[i][j] is written,
    // so one array serves both.
    template <typename Div = DivExact<T>>
    static __device__ __forceinline__ void pullback(T (&B)[NT], const T (&L)[NT],
                                                    const T (&rp)[KP1], Div&& div = Div()) {
        sfor_down<0, KP1>([&](auto j_) {
            GPB2_CI(j);
            const T ljj = L[tri(j, j)];
            const T rj = rp[j];
            sfor_down<j + 1, KP1>([&](auto i_) {
                GPB2_CI(i);
                const T lbij = B[tri(i, j)];
                const T tbar = div(lbij, ljj, rj);
                B[tri(j, j)] = N::sub(B[tri(j, j)], div(N::mul(lbij, L[tri(i, j)]), ljj, rj));
                B[tri(i, j)] = tbar;
                sfor<0, j>([&](auto p_) {
                    GPB2_CI(p);
                    B[tri(i, p)] = N::sub(B[tri(i, p)], N::mul(tbar, L[tri(j, p)]));
                    B[tri(j, p)] = N::sub(B[tri(j, p)], N::mul(tbar, L[tri(i, p)]));
                });
            });
            // 1 / (2 ljj) rounded is rj / 2 exactly (a power-of-two scaling).
            const T sbar = div(B[tri(j, j)], N::mul(T(2), ljj), N::mul(T(0.5), rj));
            B[tri(j, j)] = sbar;
            const T s2 = N::mul(T(2), sbar);
            sfor<0, j>([&](auto p_) {
                GPB2_CI(p);
                B[tri(j, p)] = N::sub(B[tri(j, p)], N::mul(s2, L[tri(j, p)]));
            });
        });
    }
};

}  // namespace gpb2
