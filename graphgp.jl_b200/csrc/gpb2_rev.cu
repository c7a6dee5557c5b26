// gpb2_rev.cu -- the transposed graph of the pull-form reverse sweep.
//
// The reverse sweep of generate_grad_xi / generate_grad_vals (src/grad.jl:430-446,
// src/grad_generate_vals.jl:173-186) adds mean_vec[m][j] * vb[n0 + m] into vb[nbrs[m][j]] for
// every refined point m, latest batch first.  Pushed, that is K scattered atomic additions per
// point, in no fixed order.  Pulled, every point q adds up its own incoming terms when its turn
// comes (all of them come from later batches, so they are final by then):
//     vb[q] += w_e * vb[child_e]  for the edges e of q in descending tree order of the child
// (and, for one child listing q twice, in slot order) -- the order of the serial reverse sweep,
// so the sums are the host checker's bit for bit, and reproducible from run to run.
//
// Per problem (once): the edges of all refined points, generated in descending tree order of the
// child and slot order, stably sorted by target q: rev_mj[e] = m * K + j (the child and its
// slot), rev_off[q] .. rev_off[q + 1] the edges of q (N + 1 offsets; dense points included).
// Per table: rev_w[e] = mean_vec[m][j], gathered once after the table's factor pass.
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

// Edge (m, j) goes to position e = (M - 1 - t) * K + j, t = the tree index of refined point m:
// descending tree order of the child, slot order within it.
__global__ void k_rev_edges(const int* __restrict__ nbrs, const int* __restrict__ lib_tree,
                            int64_t n0, int64_t M, int K, unsigned* __restrict__ key,
                            int* __restrict__ val) {
    for (int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; m < M;
         m += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = lib_tree ? (int64_t)lib_tree[n0 + m] - n0 : m;
        const int64_t e0 = (M - 1 - t) * K;
        for (int j = 0; j < K; j++) {
            key[e0 + j] = (unsigned)nbrs[m * K + j];
            val[e0 + j] = (int)(m * K + j);
        }
    }
}

// CSR offsets from the sorted targets: off[q] = the first edge whose target is >= q.
__global__ void k_rev_offsets(const unsigned* __restrict__ key, int64_t E, int64_t N,
                              uint32_t* __restrict__ off) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e <= E;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t lo = e == 0 ? 0 : (int64_t)key[e - 1] + 1;  // targets with no edge below e
        const int64_t hi = e == E ? N : (int64_t)key[e];          // ... up to this edge's target
        for (int64_t q = lo; q <= hi; q++) off[q] = (uint32_t)e;
    }
}

template <typename T>
__global__ void k_rev_weights(const int* __restrict__ mj, const T* __restrict__ mv, int64_t E,
                              T* __restrict__ w) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < E;
         e += (int64_t)gridDim.x * blockDim.x)
        w[e] = __ldg(mv + __ldcs(mj + e));
}

}  // namespace

size_t rev_graph_bytes(const gpb2_problem* p) {
    const size_t ts = p->dtype == GPB2_F32 ? 4 : 8;
    const size_t E = (size_t)p->m * p->k;
    return E * (4 + ts) + 4 * ((size_t)p->n + 1);
}

// Mode 2 pulls from this many refined points up (GPB2_PULL_MIN overrides): below it the pushed
// sweep is faster (small batches leave the pull's two dependent loads per point exposed; the
// measured crossover on B200 is at about 2e7 points).
static int64_t pull_min() {
    static const int64_t v = [] {
        const char* e = std::getenv("GPB2_PULL_MIN");
        return e ? (int64_t)std::atoll(e) : (int64_t)20000000;
    }();
    return v;
}

int ensure_rev_graph(gpb2_problem* p, cudaStream_t s) {
    if (p->rev_off || p->rev_mode == 0 || p->m <= 0) return GPB2_OK;
    if (p->rev_mode == 2 && p->m < pull_min()) return GPB2_OK;
    const int64_t N = p->n, M = p->m, K = p->k, E = M * K;
    if (E >= ((int64_t)1 << 31) || N >= ((int64_t)1 << 32) - 1) return GPB2_OK;  // 32-bit CSR
    const size_t ts = p->dtype == GPB2_F32 ? 4 : 8;
    // The build holds two key and two value buffers and the sort's temporary storage.
    const size_t build = (size_t)E * 16 + (size_t)E * 8;
    if (p->rev_mode == 2) {
        size_t fr = 0, tot = 0;
        if (cudaMemGetInfo(&fr, &tot) != cudaSuccess) {
            cudaGetLastError();
            return GPB2_OK;
        }
        const size_t margin = std::max(tot / 10, (size_t)8 << 30);
        if (fr < rev_graph_bytes(p) + build + margin) return GPB2_OK;  // atomic push instead
    }
    unsigned *k0 = nullptr, *k1 = nullptr;
    int *v0 = nullptr, *v1 = nullptr;
    void* tmp = nullptr;
    uint32_t* off = nullptr;
    int* mj = nullptr;
    void* w = nullptr;
    int st = GPB2_OK;
    do {
        if ((st = ensure_alloc(reinterpret_cast<void**>(&k0), sizeof(unsigned) * E))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&k1), sizeof(unsigned) * E))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&v0), sizeof(int) * E))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&v1), sizeof(int) * E))) break;
        k_rev_edges<<<grid_of(M), kThreads, 0, s>>>(p->nbrs, p->lib_tree, p->n0, M, (int)K, k0,
                                                    v0);
        cub::DoubleBuffer<unsigned> dk(k0, k1);
        cub::DoubleBuffer<int> dv(v0, v1);
        int bits = 1;
        while (bits < 32 && ((N - 1) >> bits) != 0) bits++;
        size_t tb = 0;
        if (cub::DeviceRadixSort::SortPairs(nullptr, tb, dk, dv, E, 0, bits, s) != cudaSuccess) {
            st = set_error(GPB2_ERR_CUDA, "transposed graph: sort sizing failed");
            break;
        }
        if ((st = ensure_alloc(&tmp, tb))) break;
        if (cub::DeviceRadixSort::SortPairs(tmp, tb, dk, dv, E, 0, bits, s) != cudaSuccess) {
            st = set_error(GPB2_ERR_CUDA, "transposed graph: sort failed");
            break;
        }
        if ((st = ensure_alloc(reinterpret_cast<void**>(&off), sizeof(uint32_t) * (N + 1)))) break;
        k_rev_offsets<<<grid_of(E + 1), kThreads, 0, s>>>(dk.Current(), E, N, off);
        if ((st = ensure_alloc(reinterpret_cast<void**>(&mj), sizeof(int) * E))) break;
        GPB2_CUDA_TRY(cudaMemcpyAsync(mj, dv.Current(), sizeof(int) * E,
                                      cudaMemcpyDeviceToDevice, s));
        if ((st = ensure_alloc(&w, ts * E))) break;
        const cudaError_t e = cudaStreamSynchronize(s);  // the temporaries are freed below
        if (e != cudaSuccess) {
            st = set_error(GPB2_ERR_CUDA, "transposed graph: %s", cudaGetErrorString(e));
            break;
        }
        p->rev_off = off;
        p->rev_mj = mj;
        p->rev_w = w;
        off = nullptr;
        mj = nullptr;
        w = nullptr;
        p->rev_w_valid = false;
    } while (0);
    for (void* b : {(void*)k0, (void*)k1, (void*)v0, (void*)v1, tmp, (void*)off, (void*)mj, w})
        if (b) cudaFree(b);
    if (st && p->rev_mode == 2) {  // no room after all: stay with the atomic push
        clear_error();
        return GPB2_OK;
    }
    return st;
}

template <typename T>
int ensure_rev_weights(gpb2_problem* p, cudaStream_t s) {
    if (!p->rev_off || p->rev_w_valid) return GPB2_OK;
    const int64_t E = p->m * p->k;
    k_rev_weights<T><<<grid_of(E), kThreads, 0, s>>>(p->rev_mj, static_cast<const T*>(p->mv), E,
                                                     static_cast<T*>(p->rev_w));
    GPB2_CUDA_TRY(cudaGetLastError());
    p->rev_w_valid = true;
    return GPB2_OK;
}

template int ensure_rev_weights<float>(gpb2_problem*, cudaStream_t);
template int ensure_rev_weights<double>(gpb2_problem*, cudaStream_t);

}  // namespace gpb2
