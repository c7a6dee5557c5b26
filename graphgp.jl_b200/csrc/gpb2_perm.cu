// gpb2_perm.cu -- the original <-> library-order permutation of generate & co.
// (src/orchestrate.jl:19-97: xi[indices] on the way in, out[indices] = values on the way out) for
// large problems.
//
// Applied directly, a random permutation of N values costs a 32-byte sector per 4-byte value
// (gathers) or a read-modify-write of one (scatters) once the field outgrows the L2.  Here each
// direction is applied in two passes through a staging buffer split into destination blocks of
// 2^shift values (128 KB: 2^15 floats or 2^14 doubles), each of which fits in one CTA's shared
// memory.  Staging slot of input i: in the block of its destination, at the next free slot of
// that block in input order.
//   pass 1 gives each CTA whole source tiles of 2^shift inputs: it reads a tile into shared
//          memory (contiguous, vectorised) and writes it out in slot order,
//          stage[pos[k]] = tile[from[k]] for k = 0, 1, ... -- the tile's inputs that go to one
//          block occupy consecutive slots, so consecutive threads store runs of consecutive
//          slots (about N / 2^(2 shift) values per run: ~10 at 1e8 floats) rather than one
//          scattered sector each;
//   pass 2 gives each CTA whole destination blocks: it reads block b of the staging buffer into
//          shared memory and writes the output in order,
//          out[b * 2^shift + t] = block[q[b * 2^shift + t]] (q a 16-bit index into the block).
// Every array is streamed once.  The plan comes from two stable sorts per problem and
// direction: the inputs by destination block (slots; q) and each tile's inputs by destination
// block (the slot order of the tile: from, pos).  The sources of block b are exactly the
// destinations of block b, so block b of the staging buffer is [b * 2^shift, (b + 1) * 2^shift).
#include <cub/cub.cuh>

#include <cstdlib>

#include "gpb2_problem.h"

namespace gpb2 {

int coop_grid(const void* kernel, int threads, size_t smem);  // co-resident CTAs of a kernel
cudaError_t prepare_kernel_smem(const void* kernel, size_t smem);

namespace {

constexpr int kThreads = 256;     // plan kernels
constexpr int kP1Threads = 1024;  // pass 1
constexpr int kP2Threads = 1024;  // pass 2
constexpr int kBlockBytes = 128 * 1024;  // a source tile (pass 1) or destination block (pass 2)

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

// Load values [base, base + len) of src into shared memory (16-byte loads when aligned).
template <typename T, bool kVec>
__device__ __forceinline__ void load_tile(T* __restrict__ tile, const T* __restrict__ src,
                                          int64_t base, int len) {
    int done = 0;
    if constexpr (kVec) {
        const int nq = len >> 2;
        for (int i = threadIdx.x; i < nq; i += blockDim.x) {
            Quad<T> v;
            v.load_stream(src + base + 4 * i);
#pragma unroll
            for (int u = 0; u < 4; u++) tile[4 * i + u] = v.v[u];
        }
        done = 4 * nq;
    }
    for (int i = done + threadIdx.x; i < len; i += blockDim.x) tile[i] = __ldcs(src + base + i);
}

// Pass 1: CTA-wide, one source tile of 2^tshift values at a time (grid-stride over the tiles).
// The tile is read into shared memory; then slot k of the tile's destination order (the
// tile's values sorted by their staging position) is written: stage[dst[k]] = tile[from[k]].
// Consecutive threads take consecutive k, so their stores fall in runs of consecutive staging
// slots (one run per destination block the tile feeds) instead of one sector each.
template <typename T, bool kVec>
__global__ void __launch_bounds__(kP1Threads)
k_perm_pass1(const T* __restrict__ in, const uint16_t* __restrict__ from,
             const int* __restrict__ dst, int64_t n, int tshift, T* __restrict__ stage) {
    extern __shared__ __align__(16) unsigned char smem[];
    T* tile = reinterpret_cast<T*>(smem);
    const int64_t tsz = 1ll << tshift;
    const int64_t ntile = (n + tsz - 1) >> tshift;
    for (int64_t t = blockIdx.x; t < ntile; t += gridDim.x) {
        const int64_t base = t << tshift;
        const int len = (int)(n - base < tsz ? n - base : tsz);
        load_tile<T, kVec>(tile, in, base, len);
        __syncthreads();
        for (int k = threadIdx.x; k < len; k += blockDim.x)
            stage[__ldcs(dst + base + k)] = tile[__ldcs(from + base + k)];
        __syncthreads();  // the tile buffer is reused for the next tile
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
        load_tile<T, true>(blk, stage, base, len);
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

__global__ void k_tile_keys(const int* __restrict__ dmap, int64_t n, int shift, int bbits,
                            unsigned long long* __restrict__ key, int* __restrict__ val) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        key[i] = ((unsigned long long)(i >> shift) << bbits) | (unsigned)(dmap[i] >> shift);
        val[i] = (int)i;
    }
}

// From each tile's sources sorted by destination block (sorted[k], k in tile order): the
// in-tile offset of the k-th source and its staging slot.
__global__ void k_tile_plan(const int* __restrict__ sorted, const int* __restrict__ pos,
                            int64_t n, int shift, uint16_t* __restrict__ from,
                            int* __restrict__ dst) {
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n;
         k += (int64_t)gridDim.x * blockDim.x) {
        const int src = sorted[k];
        from[k] = (uint16_t)(src & ((1 << shift) - 1));
        dst[k] = pos[src];
    }
}

template <typename K>
int sort_pairs(cub::DoubleBuffer<K>& dk, cub::DoubleBuffer<int>& dv, int64_t n, int bits,
               void*& tmp, size_t& tmp_bytes, cudaStream_t s) {
    size_t tb = 0;
    if (cub::DeviceRadixSort::SortPairs(nullptr, tb, dk, dv, n, 0, bits, s) != cudaSuccess)
        return set_error(GPB2_ERR_CUDA, "permutation plan: sort sizing failed");
    if (tb > tmp_bytes) {
        if (tmp) cudaFree(tmp);
        tmp = nullptr;
        tmp_bytes = 0;
        GPB2_TRY(ensure_alloc(&tmp, tb));
        tmp_bytes = tb;
    }
    if (cub::DeviceRadixSort::SortPairs(tmp, tb, dk, dv, n, 0, bits, s) != cudaSuccess)
        return set_error(GPB2_ERR_CUDA, "permutation plan: sort failed");
    return GPB2_OK;
}

inline int bits_for(int64_t count) {  // bits of the largest index below count
    int b = 1;
    while (b < 62 && ((count - 1) >> b) != 0) b++;
    return b;
}

// One direction's plan from its destination map (dmap[i]: where input i goes): pass 1's
// (from, dst) in tile order and pass 2's q.
int make_plan(const int* dmap, int64_t n, int shift, uint16_t* from, int* dst, uint16_t* q,
              cudaStream_t s) {
    unsigned long long *k0 = nullptr, *k1 = nullptr;
    int *v0 = nullptr, *v1 = nullptr, *pos = nullptr;
    void* tmp = nullptr;
    size_t tmp_bytes = 0;
    int st = GPB2_OK;
    const int nb_bits = bits_for((n + (1ll << shift) - 1) >> shift);  // block (= tile) index
    do {
        if ((st = ensure_alloc(reinterpret_cast<void**>(&k0), sizeof(unsigned long long) * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&k1), sizeof(unsigned long long) * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&v0), sizeof(int) * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&v1), sizeof(int) * n))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&pos), sizeof(int) * n))) break;
        // Staging slots: the inputs stably sorted by destination block.
        {
            unsigned* kk0 = reinterpret_cast<unsigned*>(k0);
            unsigned* kk1 = reinterpret_cast<unsigned*>(k1);
            k_perm_keys<<<grid_of(n), kThreads, 0, s>>>(dmap, n, shift, kk0, v0);
            cub::DoubleBuffer<unsigned> dk(kk0, kk1);
            cub::DoubleBuffer<int> dv(v0, v1);
            if ((st = sort_pairs(dk, dv, n, nb_bits, tmp, tmp_bytes, s))) break;
            k_perm_plan<<<grid_of(n), kThreads, 0, s>>>(dv.Current(), dmap, n, shift, pos, q);
        }
        // Pass 1's order: every tile's inputs stably sorted by destination block, i.e. by slot.
        {
            k_tile_keys<<<grid_of(n), kThreads, 0, s>>>(dmap, n, shift, nb_bits, k0, v0);
            cub::DoubleBuffer<unsigned long long> dk(k0, k1);
            cub::DoubleBuffer<int> dv(v0, v1);
            if ((st = sort_pairs(dk, dv, n, 2 * nb_bits, tmp, tmp_bytes, s))) break;
            k_tile_plan<<<grid_of(n), kThreads, 0, s>>>(dv.Current(), pos, n, shift, from, dst);
        }
        const cudaError_t e = cudaStreamSynchronize(s);  // the temporaries are freed below
        if (e != cudaSuccess) st = set_error(GPB2_ERR_CUDA, "permutation plan: %s", cudaGetErrorString(e));
    } while (0);
    for (void* b : {(void*)k0, (void*)k1, (void*)v0, (void*)v1, (void*)pos, tmp})
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
    // 128 KB tiles and blocks; GPB2_PERM_BLOCK_SHIFT may only make them smaller (>= 16 values).
    const int full = ts == 4 ? 15 : 14;
    int shift = full;
    if (const char* e = std::getenv("GPB2_PERM_BLOCK_SHIFT")) shift = std::atoi(e);
    shift = std::min(std::max(shift, 4), full);
    p->perm_shift = shift;
    int* dst_g = nullptr;
    do {
        if ((st = ensure_alloc(&p->perm_stage, ts * n))) break;
        for (void** b : {(void**)&p->perm_pos_s, (void**)&dst_g})
            if ((st = ensure_alloc(b, sizeof(int) * n))) break;
        if (st) break;
        for (void** b : {(void**)&p->perm_from_s, (void**)&p->perm_from_g, (void**)&p->perm_q_s,
                         (void**)&p->perm_q_g})
            if ((st = ensure_alloc(b, sizeof(uint16_t) * n))) break;
        if (st) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&inv), sizeof(int) * n))) break;
        // library -> original: input i (library), destination idx[i].
        if ((st = make_plan(p->indices, n, shift, p->perm_from_s, p->perm_pos_s, p->perm_q_s, s)))
            break;
        // original -> library: input j (original), destination inv[j].
        k_perm_inverse<<<grid_of(n), kThreads, 0, s>>>(p->indices, n, inv);
        if ((st = make_plan(inv, n, shift, p->perm_from_g, dst_g, p->perm_q_g, s))) break;
        p->perm_pos_g = dst_g;  // set last: its presence marks a complete plan
        dst_g = nullptr;
    } while (0);
    if (dst_g) cudaFree(dst_g);
    if (inv) cudaFree(inv);
    return st;
}

template <typename T>
int perm_apply(gpb2_problem* p, bool to_tree, const T* in, T* out, cudaStream_t s) {
    GPB2_TRY(ensure_perm_plan(p, s));
    const int* dst = to_tree ? p->perm_pos_g : p->perm_pos_s;
    const uint16_t* from = to_tree ? p->perm_from_g : p->perm_from_s;
    const uint16_t* q = to_tree ? p->perm_q_g : p->perm_q_s;
    T* stage = static_cast<T*>(p->perm_stage);
    const char* name = to_tree ? "gather" : "scatter";
    const int64_t n = p->n;
    const int shift = p->perm_shift;
    const size_t smem = sizeof(T) << shift;  // <= kBlockBytes
    const int64_t nblk = (n + (1ll << shift) - 1) >> shift;  // tiles = blocks
    // The staging buffer and the plan come from cudaMalloc; the caller's arrays may not be
    // aligned (then the element-wise forms).
    auto k1 = aligned16(in) ? k_perm_pass1<T, true> : k_perm_pass1<T, false>;
    GPB2_CUDA_TRY(prepare_kernel_smem((const void*)k1, kBlockBytes));
    const unsigned g1 = (unsigned)std::min<int64_t>(
        nblk, coop_grid((const void*)k1, kP1Threads, kBlockBytes));
    GPB2_CUDA_TRY(launch_prof(name, k1, dim3(g1), dim3(kP1Threads), smem, s, in, from, dst, n,
                              shift, stage));
    auto k2 = aligned16(out) ? k_perm_pass2<T, true> : k_perm_pass2<T, false>;
    GPB2_CUDA_TRY(prepare_kernel_smem((const void*)k2, kBlockBytes));
    const unsigned g2 = (unsigned)std::min<int64_t>(
        nblk, coop_grid((const void*)k2, kP2Threads, kBlockBytes));
    GPB2_CUDA_TRY(launch_prof(name, k2, dim3(g2), dim3(kP2Threads), smem, s, (const T*)stage, q,
                              n, shift, out));
    return GPB2_OK;
}

template int perm_apply<float>(gpb2_problem*, bool, const float*, float*, cudaStream_t);
template int perm_apply<double>(gpb2_problem*, bool, const double*, double*, cudaStream_t);

}  // namespace gpb2
