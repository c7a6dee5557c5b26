// gpb2_graph_cuda.cu -- build_graph on the device (the input producer of the refine path for the
// 1e8 / 1e9-point configurations), byte-identical to the host restatement in graph_build.cpp and
// therefore to the reference's build_graph (src/graph_build.jl:256-288).
//
// Steps, each the device form of the host step it reproduces:
//   1. heap-order ("special order") k-d tree, level by level (src/tree_special.jl:165-227):
//      a. the split dimension of every node of the level: the widest extent of its points
//         (src/tree_special.jl:41-65).  A node's points are one contiguous run whose bounds follow
//         from the previous level's layout (left child [st, mid), right child (mid, st + len) of
//         the parent's run), so the extents need no node-indexed scratch: one CTA slice per node
//         on the early levels (few, long runs), one warp per node on the later ones;
//      b. the level's order (node id, coordinate along the node's split dimension, position): a
//         total order, produced as two stable radix sorts (by coordinate, then by node id);
//      c. gather of points, node ids and original indices; the even-by-id relabel
//         (src/tree_special.jl:74-99).
//   2. preceding k-NN of every refined point: one thread per query runs the same stackless
//      traversal as the host (src/tree_special.jl:231-293) in exact double arithmetic (no
//      contraction), then orders its k results by (distance, index).
//   3. longest-path depths (src/graph_build.jl:78-107): every refined point's neighbours precede
//      it, so the depth is the least fixed point of depth[p] = 1 + max depth[nbr]; it is reached
//      by repeated in-place sweeps (monotone), each a flat kernel, until a sweep changes nothing.
//   4. stable order by depth (a stable radix sort) and the neighbour remap
//      (src/graph_build.jl:160-200); batch offsets from the depth histogram (:213-222).
//   5. 21-bit lattice quantisation with round-half-even (src/graph_build.jl:231-242).
// Every comparison and every floating-point operation is the host builder's, in its order, so the
// coordinates, neighbours, permutation and offsets are the same bytes.
#include <cub/cub.cuh>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <vector>

#include "gpb2_problem.h"

struct gpb2_dgraph {
    int device = 0;
    int64_t n = 0, d = 0, n0 = 0, k = 0;
    double scale = 0.0;
    uint32_t* coords = nullptr;  // (N, D) point-major, depth order
    int* nbrs = nullptr;         // (M, K) 0-based, -1 = unset
    int* indices = nullptr;      // (N) tree position -> original index (0-based)
    std::vector<int64_t> offsets;
};

namespace gpb2 {

namespace {

constexpr int kThreads = 256;
constexpr int kDepthSmem = 8192;  // depths counted in shared memory up to this

inline unsigned grid_for(int64_t n, int per_thread = 1) {
    int64_t g = (n + (int64_t)kThreads * per_thread - 1) / ((int64_t)kThreads * per_thread);
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(g, 148 * 32));
}

// ----------------------------------------------------------------------------------- tree

__device__ __forceinline__ int flevel_d(long long x) { return 63 - __clzll(x); }
__device__ __forceinline__ long long sp_parent_d(long long c) {
    if (c == 0) return -1;
    const int level = flevel_d(c + 1);
    const long long n_above = (1ll << level) - 1, n_parent_level = 1ll << (level - 1);
    return c < n_above + n_parent_level ? c - n_parent_level : c - 2 * n_parent_level;
}
__device__ __forceinline__ long long sp_left_d(long long c) { return c + (1ll << flevel_d(c + 1)); }
__device__ __forceinline__ long long sp_right_d(long long c) {
    return c + 2 * (1ll << flevel_d(c + 1));
}

// The run [a, b) of node ii (index within level `level`) in the layout the previous level's
// sort and relabel left: the left or right part of the parent's run around its median.
struct RunGeom {
    long long N;
    int level;
    __device__ __forceinline__ void run(long long ii, long long& a, long long& b) const {
        if (level == 0) {
            a = 0;
            b = N;
            return;
        }
        const long long nlp = 1ll << (level - 1), nap = nlp - 1;
        const long long nrem = N - nap, q = nrem / nlp, r = nrem % nlp;
        const bool left = ii < nlp;
        const long long pii = left ? ii : ii - nlp;
        const long long st = nap + (pii < r ? pii * (q + 1) : r * (q + 1) + (pii - r) * q);
        const long long len = pii < r ? q + 1 : q;
        const long long mid = st + (pii < r ? (q + 1) / 2 : q / 2);
        if (left) {
            a = st;
            b = len > 0 ? mid : st;
        } else {
            a = mid + 1;
            b = st + len;
        }
        if (b < a) b = a;
    }
};

// Order-preserving integer image of a double (for atomic min / max); -0.0 is folded into +0.0
// first (the host compares with < and >, for which the two zeros are equal).
__device__ __forceinline__ unsigned long long ord_key(double v) {
    const unsigned long long b = (unsigned long long)__double_as_longlong(v + 0.0);
    return (b >> 63) ? ~b : (b | 0x8000000000000000ull);
}
__device__ __forceinline__ double ord_val(unsigned long long o) {
    const unsigned long long b = (o >> 63) ? (o & 0x7fffffffffffffffull) : ~o;
    return __longlong_as_double((long long)b);
}

// Split dimension from the per-dimension maxima and minima: the first dimension with the
// largest range (strict >, from -inf), exactly the host's loop.
__device__ __forceinline__ int best_dim(const double* mx, const double* mn, int D) {
    int bestd = 0;
    double bestr = -INFINITY;
    for (int d = 0; d < D; d++) {
        const double rr = __dsub_rn(mx[d], mn[d]);
        if (rr > bestr) {
            bestr = rr;
            bestd = d;
        }
    }
    return bestd;
}

// Early levels: node ii's run is cut into `parts` slices, one CTA each; slices fold their
// extents into per-node slots with atomics.
__global__ void k_extent_slices(const double* __restrict__ pts, RunGeom g, long long n_above,
                                long long n_nodes, int D, int parts,
                                unsigned long long* __restrict__ smx,
                                unsigned long long* __restrict__ smn) {
    const long long ii = blockIdx.x / parts;
    const int part = blockIdx.x - (int)(ii * parts);
    if (ii >= n_nodes) return;
    long long a, b;
    g.run(ii, a, b);
    const long long len = b - a, per = (len + parts - 1) / parts;
    const long long s0 = a + part * per, s1 = min(b, s0 + per);
    double mx[8], mn[8];
    for (int d = 0; d < D; d++) {
        mx[d] = -INFINITY;
        mn[d] = INFINITY;
    }
    for (long long i = s0 + threadIdx.x; i < s1; i += blockDim.x)
        for (int d = 0; d < D; d++) {
            const double v = pts[i * D + d];
            mx[d] = fmax(mx[d], v);
            mn[d] = fmin(mn[d], v);
        }
    __shared__ unsigned long long bmx[8], bmn[8];
    if (threadIdx.x < 8) {
        bmx[threadIdx.x] = 0ull;
        bmn[threadIdx.x] = ~0ull;
    }
    __syncthreads();
    for (int d = 0; d < D; d++) {
        unsigned long long kx = ord_key(mx[d]), kn = ord_key(mn[d]);
        for (int o = 16; o > 0; o >>= 1) {
            kx = max(kx, __shfl_xor_sync(0xffffffffu, kx, o));
            kn = min(kn, __shfl_xor_sync(0xffffffffu, kn, o));
        }
        if ((threadIdx.x & 31) == 0 && s0 < s1) {
            atomicMax(&bmx[d], kx);
            atomicMin(&bmn[d], kn);
        }
    }
    __syncthreads();
    if (threadIdx.x < D && s0 < s1) {
        atomicMax(&smx[ii * D + threadIdx.x], bmx[threadIdx.x]);
        atomicMin(&smn[ii * D + threadIdx.x], bmn[threadIdx.x]);
    }
}

__global__ void k_split_from_slots(const unsigned long long* __restrict__ smx,
                                   const unsigned long long* __restrict__ smn, RunGeom g,
                                   long long n_above, long long n_nodes, int D,
                                   unsigned char* __restrict__ split) {
    for (long long ii = (long long)blockIdx.x * blockDim.x + threadIdx.x; ii < n_nodes;
         ii += (long long)gridDim.x * blockDim.x) {
        long long a, b;
        g.run(ii, a, b);
        int bd = 0;
        if (b > a) {
            double mx[8], mn[8];
            for (int d = 0; d < D; d++) {
                mx[d] = ord_val(smx[ii * D + d]);
                mn[d] = ord_val(smn[ii * D + d]);
            }
            bd = best_dim(mx, mn, D);
        }
        split[n_above + ii] = (unsigned char)bd;
    }
}

// Later levels: one warp per node (runs are short).
__global__ void k_extent_warps(const double* __restrict__ pts, RunGeom g, long long n_above,
                               long long n_nodes, long long N, int D,
                               unsigned char* __restrict__ split) {
    const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long ii = warp; ii < n_nodes; ii += nwarps) {
        if (n_above + ii >= N) continue;
        long long a, b;
        g.run(ii, a, b);
        double mx[8], mn[8];
        for (int d = 0; d < D; d++) {
            mx[d] = -INFINITY;
            mn[d] = INFINITY;
        }
        for (long long i = a + lane; i < b; i += 32)
            for (int d = 0; d < D; d++) {
                const double v = pts[i * D + d];
                mx[d] = fmax(mx[d], v);
                mn[d] = fmin(mn[d], v);
            }
        for (int d = 0; d < D; d++)
            for (int o = 16; o > 0; o >>= 1) {
                mx[d] = fmax(mx[d], __shfl_xor_sync(0xffffffffu, mx[d], o));
                mn[d] = fmin(mn[d], __shfl_xor_sync(0xffffffffu, mn[d], o));
            }
        if (lane == 0) split[n_above + ii] = (unsigned char)(b > a ? best_dim(mx, mn, D) : 0);
    }
}

// Sort keys of the level: the point's coordinate along its node's split dimension (zeros folded
// to +0.0, which the host's < treats alike), with the current positions as values.
__global__ void k_level_keys(const double* __restrict__ pts, const unsigned* __restrict__ nodes,
                             const unsigned char* __restrict__ split, long long N, int D,
                             double* __restrict__ key, unsigned* __restrict__ pos) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < N;
         i += (long long)gridDim.x * blockDim.x) {
        const unsigned s = nodes[i];
        key[i] = pts[i * D + split[s < N ? s : 0]] + 0.0;
        pos[i] = (unsigned)i;
    }
}

__global__ void k_iota(unsigned* __restrict__ x, long long N) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < N;
         i += (long long)gridDim.x * blockDim.x)
        x[i] = (unsigned)i;
}

__global__ void k_gather_u32(const unsigned* __restrict__ src, const unsigned* __restrict__ perm,
                             unsigned* __restrict__ dst, long long N) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < N;
         i += (long long)gridDim.x * blockDim.x)
        dst[i] = src[perm[i]];
}

// Gather of the level's order plus the even-by-id relabel (src/tree_special.jl:74-99).
__global__ void k_level_gather(const double* __restrict__ pts, const unsigned* __restrict__ nodes,
                               const unsigned* __restrict__ idx, const unsigned* __restrict__ perm,
                               long long N, int D, long long n_above, long long n_level,
                               double* __restrict__ pts_s, unsigned* __restrict__ nodes_s,
                               unsigned* __restrict__ idx_s) {
    const long long n_rem = N - n_above, q = n_rem / n_level, rr = n_rem % n_level;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < N;
         i += (long long)gridDim.x * blockDim.x) {
        const long long p = perm[i];
        for (int d = 0; d < D; d++) pts_s[i * D + d] = pts[p * D + d];
        idx_s[i] = idx[p];
        const long long s = nodes[p];
        const long long ii = s - n_above;
        const long long mid =
            (ii < rr ? ii * (q + 1) + (q + 1) / 2 : rr * (q + 1) + (ii - rr) * q + q / 2) + n_above;
        nodes_s[i] = (unsigned)((i < n_above || i == mid) ? s : (i < mid ? s + n_level : s + 2 * n_level));
    }
}

// ------------------------------------------------------------------------------------ k-NN

// Preceding k nearest neighbours of every refined point (tree positions [n0, N)), the host's
// stackless traversal (query_one) with max_index = the query itself, then the k results in
// (distance, index) order.  KM is the compiled capacity; slots k..KM-1 hold -inf and never win.
template <int KM>
__global__ void __launch_bounds__(128) k_knn(const double* __restrict__ sp,
                                             const unsigned char* __restrict__ split, long long N,
                                             long long n0, int D, int k, int* __restrict__ out) {
    for (long long query = n0 + (long long)blockIdx.x * blockDim.x + threadIdx.x; query < N;
         query += (long long)gridDim.x * blockDim.x) {
        double cd[KM];
        int ci[KM];
#pragma unroll
        for (int j = 0; j < KM; j++) {
            cd[j] = j < k ? INFINITY : -INFINITY;
            ci[j] = -1;
        }
        double q[8];
        for (int d = 0; d < D; d++) q[d] = sp[query * D + d];
        double square_radius = INFINITY;
        const long long max_index = query;
        long long current = 0, previous = -1;
        while (current != -1) {
            const long long parent = sp_parent_d(current);
            if (previous == parent) {
                double sq = 0.0;
                for (int d = 0; d < D; d++) {
                    const double dv = __dsub_rn(q[d], sp[current * D + d]);
                    sq = __dadd_rn(sq, __dmul_rn(dv, dv));
                }
                int wpos = 0;
                double wval = cd[0];
#pragma unroll
                for (int j = 1; j < KM; j++)
                    if (cd[j] > wval) {
                        wval = cd[j];
                        wpos = j;
                    }
                if (sq < wval) {
#pragma unroll
                    for (int j = 0; j < KM; j++)
                        if (j == wpos) {
                            cd[j] = sq;
                            ci[j] = (int)current;
                        }
                    double m = cd[0];
#pragma unroll
                    for (int j = 1; j < KM; j++) m = cd[j] > m ? cd[j] : m;
                    square_radius = m;
                } else {
                    square_radius = wval;
                }
            }
            const int sd = split[current];
            const double split_distance = __dsub_rn(q[sd], sp[current * D + sd]);
            const long long nearc = split_distance < 0 ? sp_left_d(current) : sp_right_d(current);
            const long long farc = split_distance < 0 ? sp_right_d(current) : sp_left_d(current);
            const bool far_in_range = __dmul_rn(split_distance, split_distance) <= square_radius;
            long long nxt;
            if (previous == nearc || (previous == parent && nearc >= max_index))
                nxt = (farc < max_index && far_in_range) ? farc : parent;
            else
                nxt = previous == parent ? nearc : parent;
            previous = current;
            current = nxt;
        }
        // (distance, index) order; equal pairs (only unset slots) keep slot order.
        int* o = out + (query - n0) * k;
#pragma unroll
        for (int j = 0; j < KM; j++) {
            if (j >= k) break;
            int rank = 0;
#pragma unroll
            for (int i = 0; i < KM; i++) {
                if (i >= k) break;
                const bool less = cd[i] < cd[j] || (cd[i] == cd[j] && ci[i] < ci[j]);
                const bool tie = cd[i] == cd[j] && ci[i] == ci[j] && i < j;
                rank += (less || tie) ? 1 : 0;
            }
            o[rank] = ci[j];
        }
    }
}

// ---------------------------------------------------------------------------------- depths

__global__ void k_depth_sweep(const int* __restrict__ nb, long long M, int K, long long n0,
                              int* depth, int* __restrict__ changed) {
    int ch = 0;
    for (long long m = (long long)blockIdx.x * blockDim.x + threadIdx.x; m < M;
         m += (long long)gridDim.x * blockDim.x) {
        int mx = 0;
        for (int j = 0; j < K; j++) {
            const int v = nb[m * K + j];
            if (v < 0) continue;
            const int dv = ((volatile int*)depth)[v];
            mx = dv > mx ? dv : mx;
        }
        const int nd = mx + 1;
        if (depth[n0 + m] != nd) {
            depth[n0 + m] = nd;
            ch = 1;
        }
    }
    if (__syncthreads_or(ch) && threadIdx.x == 0) atomicExch(changed, 1);
}

// Sort keys (depths) with positions, and the histogram of depths (a shared-memory histogram
// per block when the depths fit, else global atomics).
__global__ void k_depth_keys(const int* __restrict__ depth, long long N, unsigned* __restrict__ key,
                             unsigned* __restrict__ pos, unsigned long long* __restrict__ hist,
                             int maxd) {
    extern __shared__ unsigned sh[];
    const bool local = maxd < kDepthSmem;
    if (local)
        for (int i = threadIdx.x; i <= maxd; i += blockDim.x) sh[i] = 0u;
    __syncthreads();
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < N;
         i += (long long)gridDim.x * blockDim.x) {
        const int d = depth[i];
        key[i] = (unsigned)d;
        pos[i] = (unsigned)i;
        if (local)
            atomicAdd(&sh[d], 1u);
        else
            atomicAdd(&hist[d], 1ull);
    }
    __syncthreads();
    if (local)
        for (int i = threadIdx.x; i <= maxd; i += blockDim.x)
            if (sh[i]) atomicAdd(&hist[i], (unsigned long long)sh[i]);
}

__global__ void k_max_int(const int* __restrict__ x, long long n, int* __restrict__ out) {
    int m = 0;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        m = max(m, x[i]);
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(out, m);
}

__global__ void k_inverse(const unsigned* __restrict__ perm, long long N, unsigned* __restrict__ inv) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < N;
         i += (long long)gridDim.x * blockDim.x)
        inv[perm[i]] = (unsigned)i;
}

__global__ void k_final_indices(const unsigned* __restrict__ sort_perm,
                                const unsigned* __restrict__ idx_tree, long long N,
                                int* __restrict__ out) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < N;
         i += (long long)gridDim.x * blockDim.x)
        out[i] = (int)idx_tree[sort_perm[i]];
}

__global__ void k_remap_nbrs(const int* __restrict__ nb_old, const unsigned* __restrict__ inv,
                             long long M, int K, long long n0, long long n0_new,
                             int* __restrict__ nb_new) {
    for (long long m = (long long)blockIdx.x * blockDim.x + threadIdx.x; m < M;
         m += (long long)gridDim.x * blockDim.x) {
        const long long m_new = (long long)inv[n0 + m] - n0_new;
        if (m_new < 0) continue;
        for (int j = 0; j < K; j++) {
            const int o = nb_old[m * K + j];
            nb_new[m_new * K + j] = o < 0 ? -1 : (int)inv[o];
        }
    }
}

// ------------------------------------------------------------------------------ quantisation

__global__ void k_minmax(const double* __restrict__ pts, long long N, int D,
                         unsigned long long* __restrict__ gmx, unsigned long long* __restrict__ gmn) {
    double mx[8], mn[8];
    for (int d = 0; d < D; d++) {
        mx[d] = -INFINITY;
        mn[d] = INFINITY;
    }
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < N;
         i += (long long)gridDim.x * blockDim.x)
        for (int d = 0; d < D; d++) {
            const double v = pts[i * D + d];
            mx[d] = fmax(mx[d], v);
            mn[d] = fmin(mn[d], v);
        }
    for (int d = 0; d < D; d++) {
        unsigned long long kx = ord_key(mx[d]), kn = ord_key(mn[d]);
        for (int o = 16; o > 0; o >>= 1) {
            kx = max(kx, __shfl_xor_sync(0xffffffffu, kx, o));
            kn = min(kn, __shfl_xor_sync(0xffffffffu, kn, o));
        }
        if ((threadIdx.x & 31) == 0) {
            atomicMax(&gmx[d], kx);
            atomicMin(&gmn[d], kn);
        }
    }
}

struct Origin {
    double v[8];
};

__global__ void k_quantise(const double* __restrict__ pts, const unsigned* __restrict__ sort_perm,
                           long long N, int D, Origin origin, double scale, double lmax,
                           uint32_t* __restrict__ coords) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < N;
         i += (long long)gridDim.x * blockDim.x) {
        const long long src = sort_perm[i];
        for (int d = 0; d < D; d++) {
            const double cf = __ddiv_rn(__dsub_rn(pts[src * D + d], origin.v[d]), scale);
            const double rnd = rint(cf);  // round half to even
            long long c = (long long)rnd;
            if (c < 0) c = 0;
            if (c > (long long)lmax) c = (long long)lmax;
            coords[i * D + d] = (uint32_t)c;
        }
    }
}

__global__ void k_to_point_major(const double* __restrict__ src, long long N, int D,
                                 double* __restrict__ dst) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < N * D;
         i += (long long)gridDim.x * blockDim.x) {
        const long long p = i / D;
        const int d = (int)(i - p * D);
        dst[i] = src[(long long)d * N + p];
    }
}

// ------------------------------------------------------------------------------- plumbing

// Device buffers of the build, freed on every exit path.
struct Bufs {
    std::vector<void*> v;
    ~Bufs() {
        for (void* p : v)
            if (p) cudaFree(p);
    }
    template <typename X>
    int get(X** p, size_t count) {
        void* q = nullptr;
        const cudaError_t e = cudaMalloc(&q, std::max<size_t>(count * sizeof(X), 16));
        if (e != cudaSuccess) {
            cudaGetLastError();
            *p = nullptr;
            return set_error(e == cudaErrorMemoryAllocation ? GPB2_ERR_OOM : GPB2_ERR_CUDA,
                             "graph build: cudaMalloc(%zu bytes) failed: %s", count * sizeof(X),
                             cudaGetErrorString(e));
        }
        v.push_back(q);
        *p = static_cast<X*>(q);
        return GPB2_OK;
    }
    void release(void* p) {
        for (auto& q : v)
            if (q == p) {
                cudaFree(q);
                q = nullptr;
            }
    }
    void* take(void* p) {
        for (auto& q : v)
            if (q == p) q = nullptr;
        return p;
    }
};

int bits_for(unsigned long long x) {
    int b = 1;
    while (b < 64 && (x >> b) != 0) b++;
    return b;
}

// Stable radix sort of (keys, values) with CUB; the sorted arrays end in *keys / *vals (the
// double buffers are swapped as needed).
template <typename KT>
int sort_pairs(Bufs& B, KT** keys, KT** keys_alt, unsigned** vals, unsigned** vals_alt,
               long long n, int end_bit, void** temp, size_t* temp_bytes, cudaStream_t s) {
    cub::DoubleBuffer<KT> dk(*keys, *keys_alt);
    cub::DoubleBuffer<unsigned> dv(*vals, *vals_alt);
    size_t need = 0;
    GPB2_CUDA_TRY(cub::DeviceRadixSort::SortPairs(nullptr, need, dk, dv, (int64_t)n, 0, end_bit, s));
    if (need > *temp_bytes) {
        if (*temp) B.release(*temp);
        unsigned char* t = nullptr;
        GPB2_TRY(B.get(&t, need));
        *temp = t;
        *temp_bytes = need;
    }
    GPB2_CUDA_TRY(
        cub::DeviceRadixSort::SortPairs(*temp, *temp_bytes, dk, dv, (int64_t)n, 0, end_bit, s));
    if (dk.Current() != *keys) std::swap(*keys, *keys_alt);
    if (dv.Current() != *vals) std::swap(*vals, *vals_alt);
    return GPB2_OK;
}

template <int KM>
int launch_knn(const double* sp, const unsigned char* split, long long N, long long n0, int D,
               int k, int* out, cudaStream_t s) {
    const long long nq = N - n0;
    const unsigned g = (unsigned)std::max<long long>(1, std::min<long long>((nq + 127) / 128, 1ll << 30));
    k_knn<KM><<<g, 128, 0, s>>>(sp, split, N, n0, D, k, out);
    GPB2_CUDA_TRY(cudaGetLastError());
    return GPB2_OK;
}

int build(const double* points, int64_t N, int D, bool dim_major, int64_t n0, int K,
          int lattice_bits, cudaStream_t s, gpb2_dgraph* g) {
    Bufs B;
    // Points in tree order (double buffered), node ids, original indices.
    double *pts = nullptr, *pts_s = nullptr;
    unsigned *nodes = nullptr, *nodes_s = nullptr, *idx = nullptr, *idx_s = nullptr;
    unsigned char* split = nullptr;
    GPB2_TRY(B.get(&pts, (size_t)N * D));
    GPB2_TRY(B.get(&pts_s, (size_t)N * D));
    GPB2_TRY(B.get(&nodes, (size_t)N));
    GPB2_TRY(B.get(&nodes_s, (size_t)N));
    GPB2_TRY(B.get(&idx, (size_t)N));
    GPB2_TRY(B.get(&idx_s, (size_t)N));
    GPB2_TRY(B.get(&split, (size_t)N));
    if (dim_major)
        k_to_point_major<<<grid_for(N * D), kThreads, 0, s>>>(points, N, D, pts);
    else
        GPB2_CUDA_TRY(cudaMemcpyAsync(pts, points, sizeof(double) * N * D,
                                      cudaMemcpyDeviceToDevice, s));
    GPB2_CUDA_TRY(cudaMemsetAsync(nodes, 0, sizeof(unsigned) * N, s));
    GPB2_CUDA_TRY(cudaMemsetAsync(split, 0, (size_t)N, s));
    k_iota<<<grid_for(N), kThreads, 0, s>>>(idx, N);  // original indices
    double *key = nullptr, *key_alt = nullptr;
    unsigned *pos = nullptr, *pos_alt = nullptr, *nkey = nullptr, *nkey_alt = nullptr;
    GPB2_TRY(B.get(&key, (size_t)N));
    GPB2_TRY(B.get(&key_alt, (size_t)N));
    GPB2_TRY(B.get(&pos, (size_t)N));
    GPB2_TRY(B.get(&pos_alt, (size_t)N));
    GPB2_TRY(B.get(&nkey, (size_t)N));
    GPB2_TRY(B.get(&nkey_alt, (size_t)N));
    void* temp = nullptr;
    size_t temp_bytes = 0;
    constexpr long long kSlotNodes = 2048;  // early levels: per-node slots
    unsigned long long *smx = nullptr, *smn = nullptr;
    GPB2_TRY(B.get(&smx, (size_t)kSlotNodes * D));
    GPB2_TRY(B.get(&smn, (size_t)kSlotNodes * D));
    const int node_bits = bits_for((unsigned long long)N);

    const int n_levels = N > 0 ? (63 - __builtin_clzll((unsigned long long)N)) + 1 : 0;
    for (int level = 0; level < n_levels; level++) {
        const long long n_above = (1ll << level) - 1, n_level = 1ll << level;
        const long long n_nodes = std::min<long long>(n_level, N - n_above);
        const RunGeom geom{N, level};
        if (n_level <= kSlotNodes) {
            GPB2_CUDA_TRY(cudaMemsetAsync(smx, 0, sizeof(unsigned long long) * n_nodes * D, s));
            GPB2_CUDA_TRY(cudaMemsetAsync(smn, 0xff, sizeof(unsigned long long) * n_nodes * D, s));
            const long long avg = (N - n_above) / n_level + 1;
            const int parts = (int)std::max<long long>(
                1, std::min<long long>((avg + 8191) / 8192, (148 * 8 + n_nodes - 1) / n_nodes));
            k_extent_slices<<<(unsigned)(n_nodes * parts), kThreads, 0, s>>>(
                pts, geom, n_above, n_nodes, D, parts, smx, smn);
            k_split_from_slots<<<grid_for(n_nodes), kThreads, 0, s>>>(smx, smn, geom, n_above,
                                                                      n_nodes, D, split);
        } else {
            const long long warps = n_nodes;
            const unsigned gw = (unsigned)std::max<long long>(
                1, std::min<long long>((warps * 32 + kThreads - 1) / kThreads, 148 * 64));
            k_extent_warps<<<gw, kThreads, 0, s>>>(pts, geom, n_above, n_nodes, N, D, split);
        }
        GPB2_CUDA_TRY(cudaGetLastError());
        // (node, key, position) order: stable by key, then stable by node id.
        k_level_keys<<<grid_for(N), kThreads, 0, s>>>(pts, nodes, split, N, D, key, pos);
        GPB2_TRY(sort_pairs<double>(B, &key, &key_alt, &pos, &pos_alt, N, 64, &temp, &temp_bytes,
                                    s));
        k_gather_u32<<<grid_for(N), kThreads, 0, s>>>(nodes, pos, nkey, N);
        GPB2_TRY(sort_pairs<unsigned>(B, &nkey, &nkey_alt, &pos, &pos_alt, N, node_bits, &temp,
                                      &temp_bytes, s));
        k_level_gather<<<grid_for(N), kThreads, 0, s>>>(pts, nodes, idx, pos, N, D, n_above,
                                                        n_level, pts_s, nodes_s, idx_s);
        GPB2_CUDA_TRY(cudaGetLastError());
        std::swap(pts, pts_s);
        std::swap(nodes, nodes_s);
        std::swap(idx, idx_s);
    }
    B.release(key);
    B.release(key_alt);
    B.release(nkey);
    B.release(nkey_alt);
    B.release(pts_s);
    B.release(nodes);
    B.release(nodes_s);
    B.release(idx_s);
    B.release(smx);
    B.release(smn);

    // k-NN (tree positions).
    const long long M = N - n0;
    int* nb_old = nullptr;
    GPB2_TRY(B.get(&nb_old, (size_t)M * K));
    if (M > 0) {
        if (K <= 8)
            GPB2_TRY(launch_knn<8>(pts, split, N, n0, D, K, nb_old, s));
        else if (K <= 16)
            GPB2_TRY(launch_knn<16>(pts, split, N, n0, D, K, nb_old, s));
        else
            GPB2_TRY(launch_knn<32>(pts, split, N, n0, D, K, nb_old, s));
    }
    B.release(split);

    // Depths: in-place monotone sweeps until one changes nothing.
    int* depth = nullptr;
    int* flag = nullptr;
    GPB2_TRY(B.get(&depth, (size_t)N));
    GPB2_TRY(B.get(&flag, 2));
    GPB2_CUDA_TRY(cudaMemsetAsync(depth, 0, sizeof(int) * N, s));
    int* hflag = nullptr;
    GPB2_CUDA_TRY(cudaMallocHost(reinterpret_cast<void**>(&hflag), 2 * sizeof(int)));
    struct HostFree {
        int* p;
        ~HostFree() { cudaFreeHost(p); }
    } hf{hflag};
    const long long sweep_limit = N + 2;  // the longest path has at most N - n0 + 1 points
    for (long long it = 0;; it++) {
        if (it > sweep_limit)
            return set_error(GPB2_ERR_GRAPH, "graph build: depth sweeps did not converge");
        GPB2_CUDA_TRY(cudaMemsetAsync(flag, 0, sizeof(int), s));
        if (M > 0)
            k_depth_sweep<<<grid_for(M, 4), kThreads, 0, s>>>(nb_old, M, K, n0, depth, flag);
        GPB2_CUDA_TRY(cudaMemcpyAsync(hflag, flag, sizeof(int), cudaMemcpyDeviceToHost, s));
        GPB2_CUDA_TRY(cudaStreamSynchronize(s));
        if (hflag[0] == 0) break;
    }
    GPB2_CUDA_TRY(cudaMemsetAsync(flag, 0, sizeof(int), s));
    k_max_int<<<grid_for(N, 4), kThreads, 0, s>>>(depth, N, flag);
    GPB2_CUDA_TRY(cudaMemcpyAsync(hflag, flag, sizeof(int), cudaMemcpyDeviceToHost, s));
    GPB2_CUDA_TRY(cudaStreamSynchronize(s));
    const int maxd = hflag[0];

    // Stable order by depth, histogram of depths.
    unsigned *dkey = nullptr, *dkey_alt = nullptr, *sp = nullptr, *sp_alt = nullptr;
    unsigned long long* hist = nullptr;
    GPB2_TRY(B.get(&dkey, (size_t)N));
    GPB2_TRY(B.get(&dkey_alt, (size_t)N));
    GPB2_TRY(B.get(&sp, (size_t)N));
    GPB2_TRY(B.get(&sp_alt, (size_t)N));
    GPB2_TRY(B.get(&hist, (size_t)maxd + 1));
    GPB2_CUDA_TRY(cudaMemsetAsync(hist, 0, sizeof(unsigned long long) * (maxd + 1), s));
    k_depth_keys<<<grid_for(N, 8), kThreads,
                   maxd < kDepthSmem ? sizeof(unsigned) * (maxd + 1) : 0, s>>>(depth, N, dkey, sp,
                                                                              hist, maxd);
    GPB2_TRY(sort_pairs<unsigned>(B, &dkey, &dkey_alt, &sp, &sp_alt, N, bits_for((unsigned)maxd),
                                  &temp, &temp_bytes, s));
    std::vector<unsigned long long> hh((size_t)maxd + 1);
    GPB2_CUDA_TRY(cudaMemcpyAsync(hh.data(), hist, sizeof(unsigned long long) * (maxd + 1),
                                  cudaMemcpyDeviceToHost, s));
    B.release(depth);
    B.release(dkey);
    B.release(dkey_alt);
    B.release(sp_alt);
    unsigned* inv = nullptr;
    GPB2_TRY(B.get(&inv, (size_t)N));
    k_inverse<<<grid_for(N), kThreads, 0, s>>>(sp, N, inv);
    GPB2_CUDA_TRY(cudaStreamSynchronize(s));  // hh is read below
    const long long n0_new = (long long)hh[0];

    // Outputs: original indices in depth order, remapped neighbours, lattice coordinates.
    int* out_idx = nullptr;
    int* out_nb = nullptr;
    uint32_t* out_coords = nullptr;
    GPB2_TRY(B.get(&out_idx, (size_t)N));
    k_final_indices<<<grid_for(N), kThreads, 0, s>>>(sp, idx, N, out_idx);
    B.release(idx);
    const long long M_new = N - n0_new;
    GPB2_TRY(B.get(&out_nb, (size_t)M_new * K));
    GPB2_CUDA_TRY(cudaMemsetAsync(out_nb, 0xff, sizeof(int) * (size_t)M_new * K, s));
    if (M > 0)
        k_remap_nbrs<<<grid_for(M), kThreads, 0, s>>>(nb_old, inv, M, K, n0, n0_new, out_nb);
    B.release(nb_old);
    B.release(inv);

    unsigned long long* mm = nullptr;
    GPB2_TRY(B.get(&mm, 16));
    GPB2_CUDA_TRY(cudaMemsetAsync(mm, 0, sizeof(unsigned long long) * 8, s));
    GPB2_CUDA_TRY(cudaMemsetAsync(mm + 8, 0xff, sizeof(unsigned long long) * 8, s));
    k_minmax<<<grid_for(N, 8), kThreads, 0, s>>>(pts, N, D, mm, mm + 8);
    unsigned long long hm[16];
    GPB2_CUDA_TRY(cudaMemcpyAsync(hm, mm, sizeof(hm), cudaMemcpyDeviceToHost, s));
    GPB2_CUDA_TRY(cudaStreamSynchronize(s));
    auto unord = [](unsigned long long o) {
        const unsigned long long b = (o >> 63) ? (o & 0x7fffffffffffffffull) : ~o;
        double v;
        std::memcpy(&v, &b, 8);
        return v;
    };
    Origin origin{};
    double extent = -std::numeric_limits<double>::infinity();
    for (int d = 0; d < D; d++) {
        origin.v[d] = unord(hm[8 + d]);
        extent = std::max(extent, unord(hm[d]) - origin.v[d]);
    }
    const double lmax = double((int64_t(1) << lattice_bits) - 1);
    const double scale = extent > 0 ? extent / lmax : 1.0 / lmax;
    GPB2_TRY(B.get(&out_coords, (size_t)N * D));
    k_quantise<<<grid_for(N), kThreads, 0, s>>>(pts, sp, N, D, origin, scale, lmax, out_coords);
    GPB2_CUDA_TRY(cudaGetLastError());
    GPB2_CUDA_TRY(cudaStreamSynchronize(s));

    g->n = N;
    g->d = D;
    g->k = K;
    g->n0 = n0_new;
    g->scale = scale;
    g->offsets.resize((size_t)maxd + 1);
    unsigned long long acc = 0;
    for (int dd = 0; dd <= maxd; dd++) {
        acc += hh[dd];
        g->offsets[dd] = (int64_t)acc;
    }
    g->coords = static_cast<uint32_t*>(B.take(out_coords));
    g->nbrs = static_cast<int*>(B.take(out_nb));
    g->indices = static_cast<int*>(B.take(out_idx));
    return GPB2_OK;
}

}  // namespace

}  // namespace gpb2

using namespace gpb2;

extern "C" {

int gpb2_build_graph_device(const double* points_dev, int64_t n, int64_t d,
                            int64_t points_dim_major, int64_t n0, int64_t k, int64_t lattice_bits,
                            int device, void* stream, gpb2_dgraph** out) {
    clear_error();
    if (!out) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_build_graph_device: out is NULL");
    *out = nullptr;
    if (!points_dev || n <= 0 || d < 1 || d > 8 || k < 1 || k > 32 || n0 < 1 || n0 >= n ||
        lattice_bits < 1 || lattice_bits > 31 || n > (int64_t)INT32_MAX)
        return set_error(GPB2_ERR_INVALID_ARG,
                         "gpb2_build_graph_device: need points, 1<=d<=8, 1<=k<=32, 1<=n0<n<2^31, "
                         "1<=lattice_bits<=31 (got n=%lld d=%lld n0=%lld k=%lld bits=%lld)",
                         (long long)n, (long long)d, (long long)n0, (long long)k,
                         (long long)lattice_bits);
    DeviceGuard dg(device);
    if (!dg.ok) return set_error(GPB2_ERR_NO_DEVICE, "cudaSetDevice(%d) failed", device);
    auto* g = new gpb2_dgraph();
    g->device = device;
    const int st = build(points_dev, n, (int)d, points_dim_major != 0, n0, (int)k,
                         (int)lattice_bits, (cudaStream_t)stream, g);
    if (st != GPB2_OK) {
        cudaGetLastError();
        delete g;
        return st;
    }
    *out = g;
    return GPB2_OK;
}

int64_t gpb2_dgraph_n_offsets(const gpb2_dgraph* g) { return g ? (int64_t)g->offsets.size() : -1; }
int64_t gpb2_dgraph_n0(const gpb2_dgraph* g) { return g ? g->n0 : -1; }

int gpb2_dgraph_export(const gpb2_dgraph* g, uint32_t* coords_dev, int32_t* nbrs_dev,
                       int32_t* indices_dev, int64_t* offsets_host, double* scale,
                       void* stream) {
    clear_error();
    if (!g) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_dgraph_export: graph is NULL");
    DeviceGuard dg(g->device);
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t M = g->n - g->n0;
    if (coords_dev)
        GPB2_CUDA_TRY(cudaMemcpyAsync(coords_dev, g->coords, sizeof(uint32_t) * g->n * g->d,
                                      cudaMemcpyDeviceToDevice, s));
    if (nbrs_dev)
        GPB2_CUDA_TRY(cudaMemcpyAsync(nbrs_dev, g->nbrs, sizeof(int) * M * g->k,
                                      cudaMemcpyDeviceToDevice, s));
    if (indices_dev)
        GPB2_CUDA_TRY(cudaMemcpyAsync(indices_dev, g->indices, sizeof(int) * g->n,
                                      cudaMemcpyDeviceToDevice, s));
    if (offsets_host) std::copy(g->offsets.begin(), g->offsets.end(), offsets_host);
    if (scale) *scale = g->scale;
    return GPB2_OK;
}

void gpb2_dgraph_free(gpb2_dgraph* g) {
    if (!g) return;
    DeviceGuard dg(g->device);
    cudaDeviceSynchronize();
    if (g->coords) cudaFree(g->coords);
    if (g->nbrs) cudaFree(g->nbrs);
    if (g->indices) cudaFree(g->indices);
    delete g;
}

}  // extern "C"
