// gpb2_order.cu -- the library's internal point order.
//
// The reference's tree order puts a depth batch's points in heap order, which scatters them in
// space: consecutive positions are far apart, so a warp's 32 points have 256 unrelated
// neighbours and every gather lands on its own sector.  Inside the library each depth batch is
// therefore re-sorted by the Morton code of its points' lattice coordinates ("library order"):
// a warp then handles 32 neighbouring points, which share most of their neighbours, and those
// neighbours sit close together in the earlier batches -- the gathers of coordinates and values
// and the reverse sweep's atomics become largely coalesced.  Nothing else changes: the batches
// keep their bounds, the dense first layer (positions [0, n0)) keeps the tree order its factor
// depends on, each point keeps its neighbour list in the reference's order (only renumbered),
// and the per-point arithmetic is the same, so every result is the same bit for bit.
//
// The problem's device arrays (coords, nbrs, indices) are held in library order; p->lib_tree maps
// a library position to its tree position.  The operations in original order compose the
// original <-> tree permutation with this one (p->indices becomes library -> original); the
// tree-order entry points (refine!, refine_inv!, ...) gather and scatter through lib_tree.
#include <cub/cub.cuh>

#include <algorithm>
#include <cstdlib>

#include "gpb2_problem.h"

namespace gpb2 {

namespace {

constexpr int kThreads = 256;

inline unsigned grid_of(int64_t n) {
    const int64_t g = (n + kThreads - 1) / kThreads;
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(g, 148 * 16));
}

__global__ void k_max_coord(const uint32_t* __restrict__ coords, int64_t n0, int64_t n, int D,
                            int DS, unsigned* __restrict__ out) {
    unsigned m = 0;
    for (int64_t i = n0 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        for (int d = 0; d < D; d++) m = max(m, coords[i * DS + d]);
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(out, m);
}

// Sort key of refined point m: its batch in the top bits, then the Morton code of its
// coordinates (their `bits` highest significant bits, interleaved dimension by dimension).
__global__ void k_order_keys(const uint32_t* __restrict__ coords, const int64_t* __restrict__ offs,
                             int64_t n_off, int64_t n0, int64_t M, int D, int DS, int cshift,
                             int bits, int bshift, unsigned long long* __restrict__ key,
                             int* __restrict__ val) {
    for (int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; m < M;
         m += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = n0 + m;
        int64_t lo = 0, hi = n_off - 1;  // the batch: the last offs[b] <= p
        while (lo < hi) {
            const int64_t mid = (lo + hi + 1) >> 1;
            if (offs[mid] <= p) lo = mid; else hi = mid - 1;
        }
        unsigned long long code = 0;
        for (int b = bits - 1; b >= 0; b--)
            for (int d = 0; d < D; d++)
                code = (code << 1) | ((coords[p * DS + d] >> (cshift + b)) & 1u);
        key[m] = ((unsigned long long)lo << bshift) | code;
        val[m] = (int)m;
    }
}

__global__ void k_order_inverse(const int* __restrict__ perm, int64_t M, int* __restrict__ inv) {
    for (int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; m < M;
         m += (int64_t)gridDim.x * blockDim.x)
        inv[perm[m]] = (int)m;
}

// Library arrays from the tree-order ones: lib_tree (library -> tree position), coords, the
// neighbour rows (renumbered into library positions) and library -> original indices.
__global__ void k_order_apply(const int* __restrict__ perm, const int* __restrict__ inv,
                              int64_t n0, int64_t N, int K, int DS,
                              const uint32_t* __restrict__ coords_t, const int* __restrict__ nbrs_t,
                              const int* __restrict__ idx_t, int* __restrict__ lib_tree,
                              uint32_t* __restrict__ coords_l, int* __restrict__ nbrs_l,
                              int* __restrict__ idx_l) {
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < N;
         q += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = q < n0 ? q : n0 + perm[q - n0];
        lib_tree[q] = (int)t;
        for (int d = 0; d < DS; d++) coords_l[q * DS + d] = coords_t[t * DS + d];
        idx_l[q] = idx_t ? idx_t[t] : (int)t;
        if (q >= n0) {
            const int* src = nbrs_t + (t - n0) * K;
            int* dst = nbrs_l + (q - n0) * K;
            for (int j = 0; j < K; j++) {
                const int v = src[j];
                dst[j] = v < n0 ? v : (int)(n0 + inv[v - n0]);
            }
        }
    }
}

}  // namespace

int library_order(gpb2_problem* p, cudaStream_t s) {
    const int64_t N = p->n, n0 = p->n0, M = p->m, K = p->k;
    const int D = (int)p->d, DS = coord_stride(D);
    if (const char* e = std::getenv("GPB2_TREE_ORDER"))
        if (std::atoi(e) != 0) return GPB2_OK;  // keep the reference's tree order
    if (M < 2) return GPB2_OK;
    unsigned long long *k0 = nullptr, *k1 = nullptr;
    int *v0 = nullptr, *v1 = nullptr, *inv = nullptr, *lib_tree = nullptr, *nbrs_l = nullptr,
        *idx_l = nullptr;
    uint32_t* coords_l = nullptr;
    unsigned* dmax = nullptr;
    void* tmp = nullptr;
    int st = GPB2_OK;
    do {
        if ((st = ensure_alloc(reinterpret_cast<void**>(&dmax), sizeof(unsigned)))) break;
        cudaMemsetAsync(dmax, 0, sizeof(unsigned), s);
        k_max_coord<<<grid_of(M), kThreads, 0, s>>>(p->coords, n0, N, D, DS, dmax);
        unsigned hmax = 0;
        cudaMemcpyAsync(&hmax, dmax, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
        if (cudaStreamSynchronize(s) != cudaSuccess) {
            st = set_error(GPB2_ERR_CUDA, "library order: %s", cudaGetErrorString(cudaGetLastError()));
            break;
        }
        int cbits = 1;
        while (cbits < 32 && (hmax >> cbits) != 0) cbits++;
        const int nbatch = (int)p->offsets.size() - 1;
        int bbits = 1;
        while ((1ll << bbits) < nbatch) bbits++;
        const int bits = std::min(cbits, (64 - bbits) / D);  // per dimension
        const int cshift = cbits - bits;
        const int bshift = 64 - bbits;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&k0), sizeof(unsigned long long) * M))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&k1), sizeof(unsigned long long) * M))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&v0), sizeof(int) * M))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&v1), sizeof(int) * M))) break;
        k_order_keys<<<grid_of(M), kThreads, 0, s>>>(p->coords, p->d_offsets,
                                                     (int64_t)p->offsets.size(), n0, M, D, DS,
                                                     cshift, bits, bshift, k0, v0);
        cub::DoubleBuffer<unsigned long long> dk(k0, k1);
        cub::DoubleBuffer<int> dv(v0, v1);
        size_t tb = 0;
        if (cub::DeviceRadixSort::SortPairs(nullptr, tb, dk, dv, M, 0, 64, s) != cudaSuccess) {
            st = set_error(GPB2_ERR_CUDA, "library order: sort sizing failed");
            break;
        }
        if ((st = ensure_alloc(&tmp, tb))) break;
        if (cub::DeviceRadixSort::SortPairs(tmp, tb, dk, dv, M, 0, 64, s) != cudaSuccess) {
            st = set_error(GPB2_ERR_CUDA, "library order: sort failed");
            break;
        }
        const int* perm = dv.Current();  // library m -> tree m
        if ((st = ensure_alloc(reinterpret_cast<void**>(&inv), sizeof(int) * M))) break;
        k_order_inverse<<<grid_of(M), kThreads, 0, s>>>(perm, M, inv);
        if ((st = ensure_alloc(reinterpret_cast<void**>(&lib_tree), sizeof(int) * N))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&coords_l), sizeof(uint32_t) * N * DS))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&nbrs_l), sizeof(int) * M * K))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&idx_l), sizeof(int) * N))) break;
        k_order_apply<<<grid_of(N), kThreads, 0, s>>>(perm, inv, n0, N, (int)K, DS, p->coords,
                                                      p->nbrs, p->indices, lib_tree, coords_l,
                                                      nbrs_l, idx_l);
        const cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) {
            st = set_error(GPB2_ERR_CUDA, "library order: %s", cudaGetErrorString(e));
            break;
        }
        std::swap(p->coords, coords_l);
        std::swap(p->nbrs, nbrs_l);
        std::swap(p->indices, idx_l);  // now library -> original
        p->lib_tree = lib_tree;
        lib_tree = nullptr;
    } while (0);
    for (void* b : {(void*)k0, (void*)k1, (void*)v0, (void*)v1, (void*)inv, (void*)lib_tree,
                    (void*)nbrs_l, (void*)idx_l, (void*)coords_l, (void*)dmax, tmp})
        if (b) cudaFree(b);
    return st;
}

}  // namespace gpb2
