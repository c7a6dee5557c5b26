// gpb2_perm.cu -- the original <-> tree permutation of generate & co. (src/orchestrate.jl:19-97:
// xi[indices] on the way in, out[indices] = values on the way out) for large problems.
//
// Applied directly, a random permutation of N values costs a 32-byte sector per 4-byte value
// (gathers) or a read-modify-write of one (scatters) once the field outgrows the L2.  Here each
// direction is applied in two passes through a staging buffer split into destination blocks of
// kBlock values (16 MB in single precision, L2-resident):
//   pass 1 reads the input in order and writes value i to stage[pos[i]] -- the block of its
//          destination, at the next free slot of that block, in input order, so every block is
//          filled front to back (a few dozen write streams, combined in the L2);
//   pass 2 writes the output in order, out[d] = stage[block(d) + q[d]], gathering within one
//          block at a time (the grid walks the output front to back, so the block it reads is in
//          the L2).
// pos and q come from one stable sort of the inputs by destination block, once per problem and
// direction: the sources of block b are exactly the kBlock destinations of that block, so block
// b of the staging buffer is [b * kBlock, (b + 1) * kBlock) and q[d] is the source's rank there.
#include <cub/cub.cuh>

#include <cstdlib>

#include "gpb2_problem.h"

namespace gpb2 {

namespace {

constexpr int kShift = 22;  // 2^22 values per destination block (GPB2_PERM_BLOCK_SHIFT overrides)
constexpr int kThreads = 256;

inline unsigned grid_of(int64_t n) {
    const int64_t g = (n + kThreads - 1) / kThreads;
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(g, 148 * 16));
}

// dst(i) of the two directions: tree -> original, dst(i) = idx[i]; original -> tree, the
// inverse permutation, dst(j) = inv[j] with inv[idx[i]] = i.
__global__ void k_perm_inverse(const int* __restrict__ idx, int64_t n, int* __restrict__ inv) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        inv[idx[i]] = (int)i;
}

__global__ void k_perm_keys(const int* __restrict__ dst, int64_t n, int shift,
                            unsigned short* __restrict__ key, int* __restrict__ val) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        key[i] = (unsigned short)(dst[i] >> shift);
        val[i] = (int)i;
    }
}

// From the inputs sorted by destination block (src_sorted[j], j in block order): pos[src] = j and
// q[dst(src)] = j mod kBlock.
__global__ void k_perm_plan(const int* __restrict__ src_sorted, const int* __restrict__ dst,
                            int64_t n, int shift, int* __restrict__ pos, int* __restrict__ q) {
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n;
         j += (int64_t)gridDim.x * blockDim.x) {
        const int src = src_sorted[j];
        pos[src] = (int)j;
        q[dst[src]] = (int)(j & ((1ll << shift) - 1));
    }
}

template <typename T>
__global__ void k_perm_pass1(const T* __restrict__ in, const int* __restrict__ pos, int64_t n,
                             T* __restrict__ stage) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        stage[pos[i]] = in[i];
}

template <typename T>
__global__ void k_perm_pass2(const T* __restrict__ stage, const int* __restrict__ q, int64_t n,
                             int shift, T* __restrict__ out) {
    for (int64_t d = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; d < n;
         d += (int64_t)gridDim.x * blockDim.x)
        out[d] = stage[((d >> shift) << shift) + q[d]];
}

// One direction's plan from its destination map.
int make_plan(const int* dst, int64_t n, int shift, int* pos, int* q, cudaStream_t s) {
    unsigned short *k0 = nullptr, *k1 = nullptr;
    int *v0 = nullptr, *v1 = nullptr;
    void* tmp = nullptr;
    int st = GPB2_OK;
    do {
        if ((st = ensure_alloc(reinterpret_cast<void**>(&k0), sizeof(unsigned short) * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&k1), sizeof(unsigned short) * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&v0), sizeof(int) * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&v1), sizeof(int) * n))) break;
        k_perm_keys<<<grid_of(n), kThreads, 0, s>>>(dst, n, shift, k0, v0);
        cub::DoubleBuffer<unsigned short> dk(k0, k1);
        cub::DoubleBuffer<int> dv(v0, v1);
        int bits = 1;
        while (bits < 16 && ((n - 1) >> shift) >> bits) bits++;
        size_t tb = 0;
        if (cub::DeviceRadixSort::SortPairs(nullptr, tb, dk, dv, n, 0, bits, s) != cudaSuccess) {
            st = set_error(GPB2_ERR_CUDA, "permutation plan: sort sizing failed");
            break;
        }
        if ((st = ensure_alloc(&tmp, tb))) break;
        if (cub::DeviceRadixSort::SortPairs(tmp, tb, dk, dv, n, 0, bits, s) != cudaSuccess) {
            st = set_error(GPB2_ERR_CUDA, "permutation plan: sort failed");
            break;
        }
        k_perm_plan<<<grid_of(n), kThreads, 0, s>>>(dv.Current(), dst, n, shift, pos, q);
        const cudaError_t e = cudaStreamSynchronize(s);  // the temporaries are freed below
        if (e != cudaSuccess) st = set_error(GPB2_ERR_CUDA, "permutation plan: %s", cudaGetErrorString(e));
    } while (0);
    for (void* b : {(void*)k0, (void*)k1, (void*)v0, (void*)v1, tmp})
        if (b) cudaFree(b);
    return st;
}

}  // namespace

// Fields above 48 MB (GPB2_PERM_TWO_PASS_MIN, in bytes, overrides the threshold).
bool perm_two_pass(const gpb2_problem* p) {
    const size_t ts = p->dtype == GPB2_F32 ? 4 : 8;
    size_t lim = (size_t)48 << 20;
    if (const char* e = std::getenv("GPB2_PERM_TWO_PASS_MIN")) lim = (size_t)std::atoll(e);
    return p->indices && (size_t)p->n * ts > lim;
}

int ensure_perm_plan(gpb2_problem* p, cudaStream_t s) {
    if (p->perm_pos_g) return GPB2_OK;
    const size_t ts = p->dtype == GPB2_F32 ? 4 : 8;
    const int64_t n = p->n;
    int* inv = nullptr;
    int st = GPB2_OK;
    int shift = kShift;
    if (const char* e = std::getenv("GPB2_PERM_BLOCK_SHIFT")) shift = std::atoi(e);
    // At most 2^16 blocks (16-bit sort keys), at least 16 values per block.
    while (shift < 30 && (((n - 1) >> shift) >> 16) != 0) shift++;
    shift = std::max(shift, 4);
    p->perm_shift = shift;
    do {
        if ((st = ensure_alloc(&p->perm_stage, ts * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&p->perm_pos_s), sizeof(int) * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&p->perm_q_s), sizeof(int) * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&p->perm_q_g), sizeof(int) * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&inv), sizeof(int) * n))) break;
        // tree -> original: input i (tree), destination idx[i].
        if ((st = make_plan(p->indices, n, shift, p->perm_pos_s, p->perm_q_s, s))) break;
        // original -> tree: input j (original), destination inv[j].
        k_perm_inverse<<<grid_of(n), kThreads, 0, s>>>(p->indices, n, inv);
        int* pos_g = nullptr;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&pos_g), sizeof(int) * n))) break;
        if ((st = make_plan(inv, n, shift, pos_g, p->perm_q_g, s))) {
            cudaFree(pos_g);
            break;
        }
        p->perm_pos_g = pos_g;  // set last: its presence marks a complete plan
    } while (0);
    if (inv) cudaFree(inv);
    return st;
}

template <typename T>
int perm_apply(gpb2_problem* p, bool to_tree, const T* in, T* out, cudaStream_t s) {
    GPB2_TRY(ensure_perm_plan(p, s));
    const int* pos = to_tree ? p->perm_pos_g : p->perm_pos_s;
    const int* q = to_tree ? p->perm_q_g : p->perm_q_s;
    T* stage = static_cast<T*>(p->perm_stage);
    GPB2_CUDA_TRY(launch_prof(to_tree ? "gather" : "scatter", k_perm_pass1<T>, dim3(grid_of(p->n)),
                              dim3(kThreads), 0, s, in, pos, p->n, stage));
    GPB2_CUDA_TRY(launch_prof(to_tree ? "gather" : "scatter", k_perm_pass2<T>, dim3(grid_of(p->n)),
                              dim3(kThreads), 0, s, (const T*)stage, q, p->n, p->perm_shift,
                              out));
    return GPB2_OK;
}

template int perm_apply<float>(gpb2_problem*, bool, const float*, float*, cudaStream_t);
template int perm_apply<double>(gpb2_problem*, bool, const double*, double*, cudaStream_t);

}  // namespace gpb2
