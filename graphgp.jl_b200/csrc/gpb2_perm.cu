// gpb2_perm.cu -- the original <-> library-order permutation of generate & co.
// (src/orchestrate.jl:19-97: xi[indices] on the way in, out[indices] = values on the way out) for
// large problems.
//
// Applied directly, a random permutation of N values costs a 32-byte sector per 4-byte value
// (gathers) or a read-modify-write of one (scatters) once the field outgrows the L2.  Here each
// direction is applied in two passes through a staging buffer split into destination blocks of
// 2^shift values (64 KB: 2^14 floats or 2^13 doubles), so that a block fits in one CTA's shared
// memory:
//   pass 1 reads the input in order and writes value i to stage[pos[i]] -- the block of its
//          destination, at the next free slot of that block, in input order, so every block is
//          filled front to back (each block's write front advances by a few hundred contiguous
//          values per grid sweep, combined into whole sectors in the L2);
//   pass 2 gives each CTA whole blocks: it reads block b of the staging buffer into shared
//          memory (contiguous, vectorised) and writes the output in order,
//          out[b * 2^shift + t] = block[q[b * 2^shift + t]] (q a 16-bit index into the block).
// Both passes stream their inputs and output once; only pass 1's scattered stores touch the L2
// one sector per value.  pos and q come from one stable sort of the inputs by destination block,
// once per problem and direction: the sources of block b are exactly the destinations of block b,
// so block b of the staging buffer is [b * 2^shift, (b + 1) * 2^shift) and q[d] is the rank of
// d's source there.
#include <cub/cub.cuh>

#include <cstdlib>

#include "gpb2_problem.h"

namespace gpb2 {

int coop_grid(const void* kernel, int threads, size_t smem);  // co-resident CTAs of a kernel
cudaError_t prepare_kernel_smem(const void* kernel, size_t smem);

namespace {

constexpr int kThreads = 256;    // plan kernels and pass 1
constexpr int kP2Threads = 512;  // pass 2
constexpr int kBlockBytes = 64 * 1024;

inline unsigned grid_of(int64_t n) {
    const int64_t g = (n + kThreads - 1) / kThreads;
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(g, 148 * 16));
}

// dst(i) of the two directions: library -> original, dst(i) = idx[i]; original -> library, the
// inverse permutation, dst(j) = inv[j] with inv[idx[i]] = i.
__global__ void k_perm_inverse(const int* __restrict__ idx, int64_t n, int* __restrict__ inv) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        inv[idx[i]] = (int)i;
}

__global__ void k_perm_keys(const int* __restrict__ dst, int64_t n, int shift,
                            unsigned* __restrict__ key, int* __restrict__ val) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        key[i] = (unsigned)(dst[i] >> shift);
        val[i] = (int)i;
    }
}

// From the inputs sorted by destination block (src_sorted[j], j in block order): pos[src] = j and
// q[dst(src)] = j mod 2^shift.
__global__ void k_perm_plan(const int* __restrict__ src_sorted, const int* __restrict__ dst,
                            int64_t n, int shift, int* __restrict__ pos,
                            uint16_t* __restrict__ q) {
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n;
         j += (int64_t)gridDim.x * blockDim.x) {
        const int src = src_sorted[j];
        pos[src] = (int)j;
        q[dst[src]] = (uint16_t)(j & ((1ll << shift) - 1));
    }
}

// Four consecutive values as one 16- (float) or two 16-byte (double) accesses, read or written
// once (evict-first loads, streaming stores).
template <typename T>
struct Quad {
    T v[4];
    __device__ __forceinline__ void load_stream(const T* p);
    __device__ __forceinline__ void store_stream(T* p) const;
};
template <>
__device__ __forceinline__ void Quad<float>::load_stream(const float* p) {
    const float4 a = __ldcs(reinterpret_cast<const float4*>(p));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}
template <>
__device__ __forceinline__ void Quad<float>::store_stream(float* p) const {
    __stcs(reinterpret_cast<float4*>(p), make_float4(v[0], v[1], v[2], v[3]));
}
template <>
__device__ __forceinline__ void Quad<double>::load_stream(const double* p) {
    const double2 a = __ldcs(reinterpret_cast<const double2*>(p));
    const double2 b = __ldcs(reinterpret_cast<const double2*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
template <>
__device__ __forceinline__ void Quad<double>::store_stream(double* p) const {
    __stcs(reinterpret_cast<double2*>(p), make_double2(v[0], v[1]));
    __stcs(reinterpret_cast<double2*>(p) + 1, make_double2(v[2], v[3]));
}

// Pass 1: groups of four consecutive inputs per thread, kUnroll groups in flight (their loads
// all issued before the first store), a grid-stride walk over the groups; the last n % 4 inputs
// go to the first threads of the grid.  The vector form needs a 16-byte aligned input, which the
// launcher checks (else kVec = false: one input per step).
constexpr int kUnroll = 2;

template <typename T, bool kVec>
__global__ void __launch_bounds__(kThreads)
k_perm_pass1(const T* __restrict__ in, const int* __restrict__ pos, int64_t n,
             T* __restrict__ stage) {
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nth = (int64_t)gridDim.x * blockDim.x;
    if constexpr (kVec) {
        const int64_t ng = n >> 2;
        for (int64_t g0 = tid; g0 < ng; g0 += kUnroll * nth) {
            Quad<T> v[kUnroll];
            int4 ps[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; u++) {
                const int64_t g = g0 + u * nth;
                if (g < ng) {
                    v[u].load_stream(in + 4 * g);
                    ps[u] = __ldcs(reinterpret_cast<const int4*>(pos) + g);
                }
            }
#pragma unroll
            for (int u = 0; u < kUnroll; u++) {
                if (g0 + u * nth < ng) {
                    stage[ps[u].x] = v[u].v[0];
                    stage[ps[u].y] = v[u].v[1];
                    stage[ps[u].z] = v[u].v[2];
                    stage[ps[u].w] = v[u].v[3];
                }
            }
        }
        const int64_t i = 4 * ng + tid;
        if (i < n) stage[__ldcs(pos + i)] = __ldcs(in + i);
    } else {
        for (int64_t i = tid; i < n; i += nth) stage[__ldcs(pos + i)] = __ldcs(in + i);
    }
}

// Pass 2: CTA-wide, one destination block at a time (grid-stride over the blocks).  The block's
// staging values are read into shared memory with 16-byte loads; then each thread writes four
// consecutive outputs per step from a 4 x 16-bit index load.  kVec = false (a caller's output
// not 16-byte aligned) writes one output per step.
template <typename T, bool kVec>
__global__ void __launch_bounds__(kP2Threads)
k_perm_pass2(const T* __restrict__ stage, const uint16_t* __restrict__ q, int64_t n, int shift,
             T* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char smem[];
    T* blk = reinterpret_cast<T*>(smem);
    const int64_t bsz = 1ll << shift;
    const int64_t nblk = (n + bsz - 1) >> shift;
    for (int64_t b = blockIdx.x; b < nblk; b += gridDim.x) {
        const int64_t base = b << shift;
        const int len = (int)(n - base < bsz ? n - base : bsz);
        const int nq = len >> 2;  // whole quads; base is a multiple of 2^shift >= 16 values
        for (int i = threadIdx.x; i < nq; i += blockDim.x) {
            Quad<T> v;
            v.load_stream(stage + base + 4 * i);
#pragma unroll
            for (int u = 0; u < 4; u++) blk[4 * i + u] = v.v[u];
        }
        for (int i = 4 * nq + threadIdx.x; i < len; i += blockDim.x)
            blk[i] = __ldcs(stage + base + i);
        __syncthreads();
        if constexpr (kVec) {
            for (int i = threadIdx.x; i < nq; i += blockDim.x) {
                const ushort4 qq = __ldcs(reinterpret_cast<const ushort4*>(q + base) + i);
                Quad<T> v;
                v.v[0] = blk[qq.x];
                v.v[1] = blk[qq.y];
                v.v[2] = blk[qq.z];
                v.v[3] = blk[qq.w];
                v.store_stream(out + base + 4 * i);
            }
            for (int i = 4 * nq + threadIdx.x; i < len; i += blockDim.x)
                __stcs(out + base + i, blk[__ldcs(q + base + i)]);
        } else {
            for (int i = threadIdx.x; i < len; i += blockDim.x)
                __stcs(out + base + i, blk[__ldcs(q + base + i)]);
        }
        __syncthreads();  // the block buffer is reused for the next block
    }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Pass 1 runs on a grid of exactly the co-resident CTAs, so the whole grid walks the input front
// to back together and every block's write front stays compact (its sectors are completed in the
// L2 before they are written back).
template <class Kern>
unsigned resident_grid(Kern kern, int threads, size_t smem, int64_t work) {
    const int64_t g = std::max<int64_t>(1, (work + threads - 1) / threads);
    return (unsigned)std::min<int64_t>(g, coop_grid((const void*)kern, threads, smem));
}

// One direction's plan from its destination map.
int make_plan(const int* dst, int64_t n, int shift, int* pos, uint16_t* q, cudaStream_t s) {
    unsigned *k0 = nullptr, *k1 = nullptr;
    int *v0 = nullptr, *v1 = nullptr;
    void* tmp = nullptr;
    int st = GPB2_OK;
    do {
        if ((st = ensure_alloc(reinterpret_cast<void**>(&k0), sizeof(unsigned) * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&k1), sizeof(unsigned) * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&v0), sizeof(int) * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&v1), sizeof(int) * n))) break;
        k_perm_keys<<<grid_of(n), kThreads, 0, s>>>(dst, n, shift, k0, v0);
        cub::DoubleBuffer<unsigned> dk(k0, k1);
        cub::DoubleBuffer<int> dv(v0, v1);
        int bits = 1;
        while (bits < 32 && ((n - 1) >> shift) >> bits) bits++;
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
    // 64 KB blocks; GPB2_PERM_BLOCK_SHIFT may only make them smaller (>= 16 values).
    const int full = ts == 4 ? 14 : 13;
    int shift = full;
    if (const char* e = std::getenv("GPB2_PERM_BLOCK_SHIFT")) shift = std::atoi(e);
    shift = std::min(std::max(shift, 4), full);
    p->perm_shift = shift;
    do {
        if ((st = ensure_alloc(&p->perm_stage, ts * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&p->perm_pos_s), sizeof(int) * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&p->perm_q_s), sizeof(uint16_t) * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&p->perm_q_g), sizeof(uint16_t) * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&inv), sizeof(int) * n))) break;
        // library -> original: input i (library), destination idx[i].
        if ((st = make_plan(p->indices, n, shift, p->perm_pos_s, p->perm_q_s, s))) break;
        // original -> library: input j (original), destination inv[j].
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
    const uint16_t* q = to_tree ? p->perm_q_g : p->perm_q_s;
    T* stage = static_cast<T*>(p->perm_stage);
    const char* name = to_tree ? "gather" : "scatter";
    const int64_t n = p->n;
    // pos, q and the staging buffer come from cudaMalloc; the caller's arrays may not be aligned.
    const int64_t nv = (n + 4 * kUnroll - 1) / (4 * kUnroll);
    if (aligned16(in)) {
        auto k = k_perm_pass1<T, true>;
        GPB2_CUDA_TRY(launch_prof(name, k, dim3(resident_grid(k, kThreads, 0, nv)),
                                  dim3(kThreads), 0, s, in, pos, n, stage));
    } else {
        auto k = k_perm_pass1<T, false>;
        GPB2_CUDA_TRY(launch_prof(name, k, dim3(resident_grid(k, kThreads, 0, n)),
                                  dim3(kThreads), 0, s, in, pos, n, stage));
    }
    const size_t smem = sizeof(T) << p->perm_shift;  // <= kBlockBytes
    const int64_t nblk = (n + (1ll << p->perm_shift) - 1) >> p->perm_shift;
    auto k2 = aligned16(out) ? k_perm_pass2<T, true> : k_perm_pass2<T, false>;
    GPB2_CUDA_TRY(prepare_kernel_smem((const void*)k2, kBlockBytes));
    const unsigned g2 = (unsigned)std::min<int64_t>(
        nblk, coop_grid((const void*)k2, kP2Threads, kBlockBytes));
    GPB2_CUDA_TRY(launch_prof(name, k2, dim3(g2), dim3(kP2Threads), smem, s, (const T*)stage, q,
                              n, p->perm_shift, out));
    return GPB2_OK;
}

template int perm_apply<float>(gpb2_problem*, bool, const float*, float*, cudaStream_t);
template int perm_apply<double>(gpb2_problem*, bool, const double*, double*, cudaStream_t);

}  // namespace gpb2
