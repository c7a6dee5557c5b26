// gpb2_problem.cu -- problem handle: upload, layout conversion, graph validation, interpolation
// table, scratch management, error plumbing.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <string>
#include <vector>

#include "gpb2_problem.h"

namespace gpb2 {

static thread_local std::string g_last_error;

int set_error(int status, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

void clear_error() { g_last_error.clear(); }

int ensure_alloc(void** ptr, size_t bytes) {
    if (*ptr) return GPB2_OK;
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e != cudaSuccess) {
        *ptr = nullptr;
        cudaGetLastError();
        return set_error(e == cudaErrorMemoryAllocation ? GPB2_ERR_OOM : GPB2_ERR_CUDA,
                         "cudaMalloc(%zu bytes) failed: %s", bytes, cudaGetErrorString(e));
    }
    return GPB2_OK;
}

int ensure_capacity(void** ptr, size_t* cap, size_t bytes) {
    if (*ptr && *cap >= bytes) return GPB2_OK;
    if (*ptr) {
        cudaFree(*ptr);  // waits for the device: work already queued on the old buffer finishes
        *ptr = nullptr;
    }
    *cap = 0;
    GPB2_TRY(ensure_alloc(ptr, bytes));
    *cap = bytes;
    return GPB2_OK;
}

static size_t tsize(const gpb2_problem* p) { return p->dtype == GPB2_F32 ? 4 : 8; }

size_t factor_cache_bytes(const gpb2_problem* p) {
    const size_t ts = tsize(p);
    const size_t nt = (size_t)(p->k + 1) * (p->k + 2) / 2, nr = nt - (size_t)(p->k + 1);
    return (size_t)p->m * (nt * ts + nr * (ts + 2));
}

int ensure_scratch(gpb2_problem* p, bool need_mv) {
    const size_t ts = tsize(p);
    GPB2_TRY(ensure_alloc(&p->buf_a, ts * p->n));
    GPB2_TRY(ensure_alloc(&p->buf_b, ts * p->n));
    GPB2_TRY(ensure_alloc(&p->buf_c, ts * p->n));
    GPB2_TRY(ensure_alloc(&p->buf_d, ts * p->n));
    GPB2_TRY(ensure_alloc(reinterpret_cast<void**>(&p->dacc), sizeof(double) * (p->nb + 8)));
    if (need_mv) {
        GPB2_TRY(ensure_alloc(&p->mv, ts * p->m * p->k));
        GPB2_TRY(ensure_alloc(&p->sd, ts * p->m));
    }
    return GPB2_OK;
}

// ------------------------------------------------------------------------------------------
// Conversion / validation kernels.
// ------------------------------------------------------------------------------------------
__global__ void k_convert_coords(const uint32_t* __restrict__ src, uint32_t* __restrict__ dst,
                                 int64_t n, int D, int DS) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n * DS;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t pnt = i / DS;
        const int d = (int)(i - pnt * DS);
        dst[i] = d < D ? src[pnt * D + d] : 0u;
    }
}

// Neighbour conversion to int32 0-based, checking the invariants the batch kernels rely on
// (check_graph, src/graph_build.jl:20-57): every neighbour of a point at tree position p lies
// strictly before the start of p's depth batch (hence before p).  Unset entries (index < 0
// after rebasing) are rejected too: the forward path reads every neighbour.
template <typename IT>
__global__ void k_convert_nbrs(const IT* __restrict__ src, int base, int64_t M, int K,
                               int64_t n0, const int64_t* __restrict__ offs, int64_t n_off,
                               int* __restrict__ dst, unsigned long long* __restrict__ bad,
                               unsigned long long* __restrict__ first_bad) {
    for (int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; m < M;
         m += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = n0 + m;
        // Batch b with offs[b-1] <= p < offs[b]: the last index with offs[idx] <= p.
        int64_t lo = 0, hi = n_off - 1;
        while (lo < hi) {
            const int64_t mid = (lo + hi + 1) >> 1;
            if (offs[mid] <= p) lo = mid; else hi = mid - 1;
        }
        const int64_t lstart = offs[lo];
        for (int j = 0; j < K; j++) {
            const long long v = (long long)src[m * K + j] - base;
            const bool ok = v >= 0 && v < lstart;
            dst[m * K + j] = ok ? (int)v : 0;
            if (!ok) {
                atomicAdd(bad, 1ull);
                atomicMin(first_bad, (unsigned long long)(m * K + j));
            }
        }
    }
}

// Device-side permutation check and conversion to int32 0-based: every value in [0, N) exactly
// once (a bitmap of seen values).
template <typename IT>
__global__ void k_convert_perm(const IT* __restrict__ src, int base, int64_t n,
                               unsigned* __restrict__ seen, int* __restrict__ dst,
                               unsigned long long* __restrict__ bad) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const long long v = (long long)src[i] - base;
        bool ok = v >= 0 && v < n;
        if (ok) {
            const unsigned bit = 1u << (v & 31);
            ok = (atomicOr(&seen[v >> 5], bit) & bit) == 0;
        }
        dst[i] = ok ? (int)v : 0;
        if (!ok) atomicAdd(bad, 1ull);
    }
}

// ------------------------------------------------------------------------------------------
// Interpolation table (see gpb2_device.cuh).
// ------------------------------------------------------------------------------------------
template <typename T> struct HostBits;
template <> struct HostBits<float> {
    using U = uint32_t;
    static U bits(float x) { U u; std::memcpy(&u, &x, 4); return u; }
    static float from(U u) { float x; std::memcpy(&x, &u, 4); return x; }
};
template <> struct HostBits<double> {
    using U = uint64_t;
    static U bits(double x) { U u; std::memcpy(&u, &x, 8); return u; }
    static double from(U u) { double x; std::memcpy(&x, &u, 8); return x; }
};

constexpr int kMaxKeys = 4096;
constexpr size_t kMaxSmem = 220 * 1024;

template <typename T>
static int build_table(gpb2_problem* p, const T* hb, const T* hv, cudaStream_t s) {
    using HB = HostBits<T>;
    using U = typename HB::U;
    const int64_t nb = p->nb;
    if (nb < 2)
        return set_error(GPB2_ERR_UNSUPPORTED_TABLE, "covariance table needs >= 2 bins (got %lld)",
                         (long long)nb);
    if (nb - 2 > 65535)
        return set_error(GPB2_ERR_UNSUPPORTED_TABLE, "at most 65537 bins are supported");
    for (int64_t i = 0; i < nb; i++)
        if (!std::isfinite((double)hb[i]) || !std::isfinite((double)hv[i]))
            return set_error(GPB2_ERR_UNSUPPORTED_TABLE, "bins/vals[%lld] is not finite",
                             (long long)i);
    for (int64_t i = 1; i < nb; i++)
        if (!(hb[i] > hb[i - 1]))
            return set_error(GPB2_ERR_UNSUPPORTED_TABLE,
                             "bins must be strictly increasing (bins[%lld] <= bins[%lld])",
                             (long long)i, (long long)(i - 1));
    if (!(hb[1] > T(0)))
        return set_error(GPB2_ERR_UNSUPPORTED_TABLE, "bins[1] must be > 0");

    // Segments {x0, x1, y0, slope}; slope is the quotient cov_lookup forms, in T.
    std::vector<T> seg(4 * (nb - 1));
    for (int64_t lo = 0; lo < nb - 1; lo++) {
        const T x0 = hb[lo], x1 = hb[lo + 1], y0 = hv[lo], y1 = hv[lo + 1];
        const T dy = y1 - y0;
        const T dx = x1 - x0;
        seg[4 * lo + 0] = x0;
        seg[4 * lo + 1] = x1;
        seg[4 * lo + 2] = y0;
        seg[4 * lo + 3] = dy / dx;
    }
    // Bucket index on the IEEE bits of r (monotone for r > 0).
    const U k1 = HB::bits(hb[1]), kN = HB::bits(hb[nb - 1]);
    int shift = 0;
    while (shift < (int)(8 * sizeof(U)) - 1 && (uint64_t)((kN >> shift) - (k1 >> shift)) + 1 >
                                                   (uint64_t)kMaxKeys)
        shift++;
    const U base = k1 >> shift;
    const int nkeys = (int)((kN >> shift) - base + 1);
    std::vector<uint16_t> start(nkeys);
    int64_t l = 0;
    for (int i = 0; i < nkeys; i++) {
        const T vmin = HB::from((U)(base + (U)i) << shift);
        while (l + 1 <= nb - 2 && hb[l + 1] <= vmin) l++;
        start[i] = (uint16_t)l;
    }
    const size_t smem = table_smem_bytes<T>((int)nb, nkeys) + sizeof(double) * nb;
    if (smem > kMaxSmem)
        return set_error(GPB2_ERR_UNSUPPORTED_TABLE,
                         "covariance table of %lld bins needs %zu bytes of shared memory "
                         "(limit %zu)", (long long)nb, smem, kMaxSmem);

    GPB2_TRY(ensure_alloc(&p->seg, sizeof(T) * seg.size()));
    GPB2_TRY(ensure_alloc(reinterpret_cast<void**>(&p->start), sizeof(uint16_t) * kMaxKeys));
    GPB2_CUDA_TRY(cudaMemcpyAsync(p->seg, seg.data(), sizeof(T) * seg.size(),
                                  cudaMemcpyHostToDevice, s));
    GPB2_CUDA_TRY(cudaMemcpyAsync(p->start, start.data(), sizeof(uint16_t) * nkeys,
                                  cudaMemcpyHostToDevice, s));
    // The host vectors die at return: finish the copies first.
    GPB2_CUDA_TRY(cudaStreamSynchronize(s));
    p->nkeys = nkeys;
    p->shift = shift;
    p->key_base = (uint64_t)base;
    p->b0 = (double)hb[0];
    p->b1 = (double)hb[1];
    p->bN = (double)hb[nb - 1];
    p->v0 = (double)hv[0];
    p->vN = (double)hv[nb - 1];
    const T pivc = T(1.5) * std::sqrt(std::numeric_limits<T>::epsilon());
    p->pivc = (double)pivc;
    return GPB2_OK;
}

static int load_table(gpb2_problem* p, const void* vals_dev, cudaStream_t s) {
    const size_t ts = tsize(p);
    p->dense_valid = false;   // the dense factor belongs to the previous table
    p->dense_launched = false;
    p->factor_valid = false;  // and so do the per-point mean_vec / std
    p->sh_factor_valid = false;
    p->fc_valid = false;      // and the factor cache
    p->fc_sh_valid = false;
    p->rev_w_valid = false;   // and the transposed graph's weights
    GPB2_CUDA_TRY(cudaMemcpyAsync(p->vals, vals_dev, ts * p->nb, cudaMemcpyDeviceToDevice, s));
    // The bins do not change after creation: they are read back once, the values every time.
    const bool first = p->hbins.size() != ts * p->nb;
    if (first) p->hbins.assign(ts * p->nb, 0);
    std::vector<unsigned char> hv(ts * p->nb);
    const std::vector<unsigned char>& hb = p->hbins;
    if (first && cudaMemcpyAsync(p->hbins.data(), p->bins, ts * p->nb, cudaMemcpyDeviceToHost,
                                 s) != cudaSuccess) {
        p->hbins.clear();
        GPB2_CUDA_TRY(cudaGetLastError());
        return set_error(GPB2_ERR_CUDA, "reading the bins back failed");
    }
    const cudaError_t e1 = cudaMemcpyAsync(hv.data(), p->vals, ts * p->nb, cudaMemcpyDeviceToHost, s);
    const cudaError_t e2 = cudaStreamSynchronize(s);
    if (first && (e1 != cudaSuccess || e2 != cudaSuccess)) p->hbins.clear();  // read again next time
    GPB2_CUDA_TRY(e1);
    GPB2_CUDA_TRY(e2);
    if (p->dtype == GPB2_F32)
        return build_table<float>(p, reinterpret_cast<const float*>(hb.data()),
                                  reinterpret_cast<const float*>(hv.data()), s);
    return build_table<double>(p, reinterpret_cast<const double*>(hb.data()),
                               reinterpret_cast<const double*>(hv.data()), s);
}

static void free_problem(gpb2_problem* p) {
    void* bufs[] = {p->coords, p->nbrs, p->indices, p->bins, p->vals,  p->seg,
                    p->start,  p->mv,   p->sd,      p->buf_a, p->buf_b, p->buf_c,
                    p->buf_d,  p->dacc, p->Lcand,   p->lad,  p->Wd,    p->Wd2,
                    p->dwork,  p->dinfo, p->d_offsets, p->dsync, p->Ld,    p->trace,
                    p->Ldr,    p->Dinv,  p->Wtri, p->Ainv,  p->sh_v, p->sh_vb,
                    p->sh_xg,  p->sh_own, p->perm_stage, p->perm_pos_g, p->perm_q_g,
                    p->perm_pos_s, p->perm_q_s, p->perm_from_g, p->perm_from_s, p->lib_tree, p->fc_L, p->fc_t, p->fc_lo,
                    p->rev_off, p->rev_mj, p->rev_w, p->dpts, p->an_sb, p->an_zb, p->an_grid};
    for (void* b : bufs)
        if (b) cudaFree(b);
    if (p->solver) cusolverDnDestroy(p->solver);
    if (p->blas) cublasDestroy(p->blas);
    if (p->hstat) cudaFreeHost(p->hstat);
    if (p->hscal) cudaFreeHost(p->hscal);
    if (p->ev_fork) cudaEventDestroy(p->ev_fork);
    if (p->ev_join) cudaEventDestroy(p->ev_join);
    if (p->ev_tri) cudaEventDestroy(p->ev_tri);
    if (p->ev_inv) cudaEventDestroy(p->ev_inv);
    if (p->dstream) cudaStreamDestroy(p->dstream);
    delete p;
}

}  // namespace gpb2

using namespace gpb2;

namespace gpb2 {
// aniso_lookup(0, 0): the diagonal of an anisotropic covariance, for the dense jitter ladder.
template <typename T>
__global__ void k_aniso_diag(AnisoView<T> av, double* out) {
    *out = (double)av.lookup(T(0), T(0));
}
}  // namespace gpb2

extern "C" {

int gpb2_version(void) { return GPB2_VERSION; }

const char* gpb2_last_error(void) { return g_last_error.c_str(); }

static int create_impl(gpb2_problem** out, int dtype, int device, const uint32_t* coords_dev,
                       int64_t d, int64_t n, const void* neighbors_dev, int neighbor_bytes,
                       int neighbor_base, int64_t k, const int64_t* offsets_host,
                       int64_t n_offsets, int64_t n0, double scale, const void* bins_dev,
                       const void* vals_dev, int64_t nbins, const int64_t* indices_host,
                       const void* indices_dev, int indices_bytes, int indices_base,
                       void* stream) {
    clear_error();
    if (!out) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_problem_create: out is NULL");
    *out = nullptr;
    if (dtype != GPB2_F32 && dtype != GPB2_F64)
        return set_error(GPB2_ERR_INVALID_ARG, "dtype must be GPB2_F32 or GPB2_F64");
    if (!coords_dev || !neighbors_dev || !offsets_host || !bins_dev || !vals_dev)
        return set_error(GPB2_ERR_INVALID_ARG, "gpb2_problem_create: NULL array argument");
    if (n <= 0 || n0 <= 0 || n0 > n || k <= 0 || nbins <= 0 || n > (int64_t)INT32_MAX)
        return set_error(GPB2_ERR_INVALID_ARG,
                         "invalid sizes n=%lld n0=%lld k=%lld nbins=%lld (need 0<n0<=n<2^31)",
                         (long long)n, (long long)n0, (long long)k, (long long)nbins);
    if (neighbor_bytes != 4 && neighbor_bytes != 8)
        return set_error(GPB2_ERR_INVALID_ARG, "neighbor_bytes must be 4 or 8");
    if (neighbor_base != 0 && neighbor_base != 1)
        return set_error(GPB2_ERR_INVALID_ARG, "neighbor_base must be 0 or 1");
    if (!(scale > 0.0) || !std::isfinite(scale))
        return set_error(GPB2_ERR_INVALID_ARG, "scale must be finite and > 0");
    if (n_offsets < 1 || offsets_host[0] != n0 || offsets_host[n_offsets - 1] != n)
        return set_error(GPB2_ERR_GRAPH, "offsets must start at n0 (%lld) and end at N (%lld)",
                         (long long)n0, (long long)n);
    for (int64_t b = 1; b < n_offsets; b++)
        if (offsets_host[b] < offsets_host[b - 1])
            return set_error(GPB2_ERR_GRAPH, "offsets must be non-decreasing (offsets[%lld])",
                             (long long)b);
    if (d < 1 || d > 8) return set_error(GPB2_ERR_UNSUPPORTED_D, "unsupported D=%lld", (long long)d);

    auto* p = new gpb2_problem();
    if (const char* e = std::getenv("GPB2_FACTOR_CACHE"))  // default mode of new handles
        p->fc_mode = std::min(std::max(std::atoi(e), 0), 2);
    if (const char* e = std::getenv("GPB2_REVERSE_MODE"))  // likewise
        p->rev_mode = std::min(std::max(std::atoi(e), 0), 2);
    p->dtype = dtype;
    p->device = device;
    p->n = n;
    p->n0 = n0;
    p->m = n - n0;
    p->k = k;
    p->d = d;
    p->nb = nbins;
    p->scale = scale;
    p->offsets.assign(offsets_host, offsets_host + n_offsets);
    if (dtype == GPB2_F32) {
        p->ops32 = find_ops<float>((int)k, (int)d);
        if (!p->ops32) {
            delete p;
            return set_error(GPB2_ERR_UNSUPPORTED_K, "no f32 kernels compiled for K=%lld, D=%lld",
                             (long long)k, (long long)d);
        }
    } else {
        p->ops64 = find_ops<double>((int)k, (int)d);
        if (!p->ops64) {
            delete p;
            return set_error(GPB2_ERR_UNSUPPORTED_K, "no f64 kernels compiled for K=%lld, D=%lld",
                             (long long)k, (long long)d);
        }
    }

    DeviceGuard dg(device);
    if (!dg.ok) {
        delete p;
        return set_error(GPB2_ERR_NO_DEVICE, "cudaSetDevice(%d) failed", device);
    }
    cudaStream_t s = (cudaStream_t)stream;
    int st = GPB2_OK;
    do {
        const int DS = coord_stride((int)d);
        if ((st = ensure_alloc(reinterpret_cast<void**>(&p->coords), sizeof(uint32_t) * n * DS)))
            break;
        k_convert_coords<<<(unsigned)std::min<int64_t>((n * DS + 255) / 256, 65535), 256, 0, s>>>(
            coords_dev, p->coords, n, (int)d, DS);
        // Neighbours.
        const int64_t M = p->m;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&p->nbrs), sizeof(int) * M * k))) break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&p->d_offsets),
                               sizeof(int64_t) * n_offsets)))
            break;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&p->dsync), 4 * sizeof(unsigned int))))
            break;
        cudaMemsetAsync(p->dsync, 0, 4 * sizeof(unsigned int), s);
        int64_t* doffs = p->d_offsets;
        unsigned long long* dbad = nullptr;
        if ((st = ensure_alloc(reinterpret_cast<void**>(&dbad), 2 * sizeof(unsigned long long))))
            break;
        unsigned long long hbad[2] = {0ull, ~0ull};
        cudaMemcpyAsync(doffs, offsets_host, sizeof(int64_t) * n_offsets, cudaMemcpyHostToDevice,
                        s);
        cudaMemcpyAsync(dbad, hbad, sizeof(hbad), cudaMemcpyHostToDevice, s);
        const unsigned g = (unsigned)std::min<int64_t>((M + 255) / 256, 65535);
        if (M > 0) {
            if (neighbor_bytes == 8)
                k_convert_nbrs<long long><<<g, 256, 0, s>>>(
                    (const long long*)neighbors_dev, neighbor_base, M, (int)k, n0, doffs,
                    n_offsets, p->nbrs, dbad, dbad + 1);
            else
                k_convert_nbrs<int><<<g, 256, 0, s>>>((const int*)neighbors_dev, neighbor_base, M,
                                                      (int)k, n0, doffs, n_offsets, p->nbrs, dbad,
                                                      dbad + 1);
        }
        cudaMemcpyAsync(hbad, dbad, sizeof(hbad), cudaMemcpyDeviceToHost, s);
        cudaError_t e = cudaStreamSynchronize(s);
        cudaFree(dbad);
        if (e != cudaSuccess) {
            st = set_error(GPB2_ERR_CUDA, "neighbour upload failed: %s", cudaGetErrorString(e));
            break;
        }
        if (hbad[0] != 0) {
            const long long fb = (long long)hbad[1];
            st = set_error(GPB2_ERR_GRAPH,
                           "%llu neighbour entries are unset or not in an earlier depth batch "
                           "(first: refined point %lld, slot %lld)",
                           hbad[0], fb / k, fb % k);
            break;
        }
        // Permutation.
        if (indices_dev) {
            if (indices_bytes != 4 && indices_bytes != 8) {
                st = set_error(GPB2_ERR_INVALID_ARG, "indices_bytes must be 4 or 8");
                break;
            }
            unsigned* seen = nullptr;
            unsigned long long* pbad = nullptr;
            if ((st = ensure_alloc(reinterpret_cast<void**>(&p->indices), sizeof(int) * n))) break;
            if ((st = ensure_alloc(reinterpret_cast<void**>(&seen), sizeof(unsigned) * ((n + 31) / 32))))
                break;
            if ((st = ensure_alloc(reinterpret_cast<void**>(&pbad), sizeof(unsigned long long)))) {
                cudaFree(seen);
                break;
            }
            cudaMemsetAsync(seen, 0, sizeof(unsigned) * ((n + 31) / 32), s);
            cudaMemsetAsync(pbad, 0, sizeof(unsigned long long), s);
            const unsigned gp = (unsigned)std::min<int64_t>((n + 255) / 256, 65535);
            if (indices_bytes == 8)
                k_convert_perm<long long><<<gp, 256, 0, s>>>((const long long*)indices_dev,
                                                             indices_base, n, seen, p->indices, pbad);
            else
                k_convert_perm<int><<<gp, 256, 0, s>>>((const int*)indices_dev, indices_base, n,
                                                       seen, p->indices, pbad);
            unsigned long long hb = 0;
            cudaMemcpyAsync(&hb, pbad, sizeof(hb), cudaMemcpyDeviceToHost, s);
            const cudaError_t e = cudaStreamSynchronize(s);
            cudaFree(seen);
            cudaFree(pbad);
            if (e != cudaSuccess) {
                st = set_error(GPB2_ERR_CUDA, "indices upload failed: %s", cudaGetErrorString(e));
                break;
            }
            if (hb != 0) {
                st = set_error(GPB2_ERR_INVALID_ARG,
                               "indices is not a permutation of 0..N-1 (%llu bad entries)", hb);
                break;
            }
        } else if (indices_host) {
            std::vector<int> idx(n);
            std::vector<unsigned char> seen(n, 0);
            for (int64_t i = 0; i < n; i++) {
                const int64_t v = indices_host[i] - indices_base;
                if (v < 0 || v >= n || seen[v]) {
                    st = set_error(GPB2_ERR_INVALID_ARG,
                                   "indices is not a permutation of 0..N-1 (entry %lld)",
                                   (long long)i);
                    break;
                }
                seen[v] = 1;
                idx[i] = (int)v;
            }
            if (st) break;
            if ((st = ensure_alloc(reinterpret_cast<void**>(&p->indices), sizeof(int) * n))) break;
            if (cudaMemcpyAsync(p->indices, idx.data(), sizeof(int) * n, cudaMemcpyHostToDevice,
                                s) != cudaSuccess ||
                cudaStreamSynchronize(s) != cudaSuccess) {
                st = set_error(GPB2_ERR_CUDA, "indices upload failed");
                break;
            }
        }
        // Library order: every depth batch sorted by Morton code (all arrays above).
        if ((st = library_order(p, s))) break;
        // Table.
        const size_t ts = tsize(p);
        if ((st = ensure_alloc(&p->bins, ts * nbins))) break;
        if ((st = ensure_alloc(&p->vals, ts * nbins))) break;
        if (cudaMemcpyAsync(p->bins, bins_dev, ts * nbins, cudaMemcpyDeviceToDevice, s) !=
            cudaSuccess) {
            st = set_error(GPB2_ERR_CUDA, "bins copy failed");
            break;
        }
        if ((st = load_table(p, vals_dev, s))) break;
    } while (0);
    if (st != GPB2_OK) {
        cudaGetLastError();
        free_problem(p);
        return st;
    }
    *out = p;
    return GPB2_OK;
}

int gpb2_problem_create(gpb2_problem** out, int dtype, int device, const uint32_t* coords_dev,
                        int64_t d, int64_t n, const void* neighbors_dev, int neighbor_bytes,
                        int neighbor_base, int64_t k, const int64_t* offsets_host,
                        int64_t n_offsets, int64_t n0, double scale, const void* bins_dev,
                        const void* vals_dev, int64_t nbins, const int64_t* indices_host,
                        int indices_base, void* stream) {
    return create_impl(out, dtype, device, coords_dev, d, n, neighbors_dev, neighbor_bytes,
                       neighbor_base, k, offsets_host, n_offsets, n0, scale, bins_dev, vals_dev,
                       nbins, indices_host, nullptr, 0, indices_base, stream);
}

int gpb2_problem_create_dev(gpb2_problem** out, int dtype, int device, const uint32_t* coords_dev,
                            int64_t d, int64_t n, const void* neighbors_dev, int neighbor_bytes,
                            int neighbor_base, int64_t k, const int64_t* offsets_host,
                            int64_t n_offsets, int64_t n0, double scale, const void* bins_dev,
                            const void* vals_dev, int64_t nbins, const void* indices_dev,
                            int indices_bytes, int indices_base, void* stream) {
    return create_impl(out, dtype, device, coords_dev, d, n, neighbors_dev, neighbor_bytes,
                       neighbor_base, k, offsets_host, n_offsets, n0, scale, bins_dev, vals_dev,
                       nbins, nullptr, indices_dev, indices_bytes, indices_base, stream);
}

int gpb2_problem_set_vals(gpb2_problem* p, const void* vals_dev, void* stream) {
    clear_error();
    if (!p || !vals_dev) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_problem_set_vals: NULL");
    DeviceGuard dg(p->device);
    return load_table(p, vals_dev, (cudaStream_t)stream);
}

int gpb2_problem_set_factor_cache(gpb2_problem* p, int mode) {
    clear_error();
    if (!p) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_problem_set_factor_cache: NULL problem");
    if (mode < 0 || mode > 2)
        return set_error(GPB2_ERR_INVALID_ARG, "gpb2_problem_set_factor_cache: mode %d", mode);
    p->fc_mode = mode;
    if (mode == 0 && p->fc_L) {  // give the memory back (cudaFree waits for the device)
        DeviceGuard dg(p->device);
        for (void* b : {p->fc_L, p->fc_t, (void*)p->fc_lo})
            if (b) cudaFree(b);
        p->fc_L = p->fc_t = nullptr;
        p->fc_lo = nullptr;
        p->fc_valid = false;
        p->fc_sh_valid = false;
    }
    return GPB2_OK;
}

int gpb2_problem_set_aniso(gpb2_problem* p, const void* spatial_bins_dev, int64_t ns,
                           const void* z_bins_dev, int64_t nz, const void* grid_dev,
                           double alpha, void* stream) {
    clear_error();
    if (!p || !spatial_bins_dev || !z_bins_dev || !grid_dev)
        return set_error(GPB2_ERR_INVALID_ARG, "gpb2_problem_set_aniso: NULL");
    if (ns < 1 || nz < 1 || ns > (1 << 20) || nz > (1 << 20) || !(alpha > 0.0))
        return set_error(GPB2_ERR_INVALID_ARG,
                         "gpb2_problem_set_aniso: ns %lld, nz %lld, alpha %g", (long long)ns,
                         (long long)nz, alpha);
    DeviceGuard dg(p->device);
    if (!dg.ok) return set_error(GPB2_ERR_NO_DEVICE, "cudaSetDevice(%d) failed", p->device);
    cudaStream_t s = (cudaStream_t)stream;
    const size_t ts = tsize(p);
    GPB2_CUDA_TRY(cudaStreamSynchronize(s));  // earlier work may still read the old arrays
    for (void** b : {&p->an_sb, &p->an_zb, &p->an_grid})
        if (*b) {
            cudaFree(*b);
            *b = nullptr;
        }
    GPB2_TRY(ensure_alloc(&p->an_sb, ts * ns));
    GPB2_TRY(ensure_alloc(&p->an_zb, ts * nz));
    GPB2_TRY(ensure_alloc(&p->an_grid, ts * ns * nz));
    GPB2_CUDA_TRY(cudaMemcpyAsync(p->an_sb, spatial_bins_dev, ts * ns, cudaMemcpyDeviceToDevice, s));
    GPB2_CUDA_TRY(cudaMemcpyAsync(p->an_zb, z_bins_dev, ts * nz, cudaMemcpyDeviceToDevice, s));
    GPB2_CUDA_TRY(
        cudaMemcpyAsync(p->an_grid, grid_dev, ts * ns * nz, cudaMemcpyDeviceToDevice, s));
    p->an_ns = (int)ns;
    p->an_nz = (int)nz;
    p->an_alpha = alpha;
    // The ladder's diagonal value, aniso_lookup(0, 0), evaluated on the device.
    double* d0 = nullptr;
    GPB2_TRY(ensure_alloc(reinterpret_cast<void**>(&d0), sizeof(double)));
    if (p->dtype == GPB2_F32)
        k_aniso_diag<float><<<1, 1, 0, s>>>(aniso_view<float>(p), d0);
    else
        k_aniso_diag<double><<<1, 1, 0, s>>>(aniso_view<double>(p), d0);
    double h0 = 0;
    cudaMemcpyAsync(&h0, d0, sizeof(double), cudaMemcpyDeviceToHost, s);
    const cudaError_t e = cudaStreamSynchronize(s);
    cudaFree(d0);
    GPB2_CUDA_TRY(e);
    p->an_diag = h0;
    // Every factor belongs to the previous covariance.
    p->dense_valid = false;
    p->dense_launched = false;
    p->ladder_hint = -1;
    p->factor_valid = false;
    p->sh_factor_valid = false;
    p->fc_valid = false;
    p->fc_sh_valid = false;
    p->rev_w_valid = false;
    return GPB2_OK;
}

int gpb2_problem_set_reverse_mode(gpb2_problem* p, int mode) {
    clear_error();
    if (!p) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_problem_set_reverse_mode: NULL problem");
    if (mode < 0 || mode > 2)
        return set_error(GPB2_ERR_INVALID_ARG, "gpb2_problem_set_reverse_mode: mode %d", mode);
    p->rev_mode = mode;
    if (mode == 0 && p->rev_off) {  // give the memory back (cudaFree waits for the device)
        DeviceGuard dg(p->device);
        for (void* b : {(void*)p->rev_off, (void*)p->rev_mj, p->rev_w})
            if (b) cudaFree(b);
        p->rev_off = nullptr;
        p->rev_mj = nullptr;
        p->rev_w = nullptr;
        p->rev_w_valid = false;
    }
    return GPB2_OK;
}

int gpb2_problem_reverse_mode(const gpb2_problem* p, int* mode, int* built, int64_t* bytes) {
    if (!p) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_problem_reverse_mode: NULL problem");
    if (mode) *mode = p->rev_mode;
    if (built) *built = p->rev_off ? 1 : 0;
    if (bytes) *bytes = (int64_t)rev_graph_bytes(p);
    return GPB2_OK;
}

int gpb2_problem_factor_cache(const gpb2_problem* p, int* mode, int* valid, int64_t* bytes) {
    if (!p) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_problem_factor_cache: NULL problem");
    if (mode) *mode = p->fc_mode;
    if (valid) *valid = !p->fc_L ? 0 : (p->fc_valid ? 1 : (p->fc_sh_valid ? 2 : 0));
    if (bytes) *bytes = (int64_t)factor_cache_bytes(p);
    return GPB2_OK;
}

int gpb2_problem_info(const gpb2_problem* p, int64_t* n, int64_t* m, int64_t* k, int64_t* d,
                      int64_t* n_batches) {
    if (!p) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_problem_info: NULL problem");
    if (n) *n = p->n;
    if (m) *m = p->m;
    if (k) *k = p->k;
    if (d) *d = p->d;
    if (n_batches) *n_batches = (int64_t)p->offsets.size() - 1;
    return GPB2_OK;
}

int gpb2_problem_order(const gpb2_problem* p, int32_t* lib_tree_dev, int32_t* lib_orig_dev,
                       void* stream) {
    clear_error();
    if (!p) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_problem_order: NULL problem");
    DeviceGuard dg(p->device);
    cudaStream_t s = (cudaStream_t)stream;
    std::vector<int> iota;
    auto fill = [&](int32_t* dst, const int* src) -> int {
        if (!dst) return GPB2_OK;
        if (src) {
            GPB2_CUDA_TRY(cudaMemcpyAsync(dst, src, sizeof(int) * p->n, cudaMemcpyDeviceToDevice, s));
            return GPB2_OK;
        }
        if (iota.empty()) {
            iota.resize((size_t)p->n);
            for (int64_t i = 0; i < p->n; i++) iota[(size_t)i] = (int)i;
        }
        GPB2_CUDA_TRY(cudaMemcpyAsync(dst, iota.data(), sizeof(int) * p->n, cudaMemcpyHostToDevice, s));
        GPB2_CUDA_TRY(cudaStreamSynchronize(s));  // iota is a host temporary
        return GPB2_OK;
    };
    GPB2_TRY(fill(lib_tree_dev, p->lib_tree));
    GPB2_TRY(fill(lib_orig_dev, p->indices));
    return GPB2_OK;
}

int gpb2_problem_dense_jitter(const gpb2_problem* p, double* eps) {
    if (!p || !eps) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_problem_dense_jitter: NULL");
    *eps = -1.0;
    if (!p->lad || p->ladder_eps.empty()) return GPB2_OK;
    DeviceGuard dg(p->device);
    int sel = -1;
    GPB2_CUDA_TRY(cudaMemcpy(&sel, p->lad + kLadSel, sizeof(int), cudaMemcpyDeviceToHost));
    if (sel >= 0 && sel < (int)p->ladder_eps.size()) *eps = p->ladder_eps[sel];
    return GPB2_OK;
}

int gpb2_problem_dense_factor(const gpb2_problem* p, void* out, void* stream) {
    if (!p || !out) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_problem_dense_factor: NULL");
    if (!p->Ld) return set_error(GPB2_ERR_INVALID_ARG, "no dense factorisation yet");
    DeviceGuard dg(p->device);
    GPB2_CUDA_TRY(cudaMemcpyAsync(out, p->Ld, tsize(p) * p->n0 * p->n0, cudaMemcpyDeviceToDevice,
                                  (cudaStream_t)stream));
    return GPB2_OK;
}

int gpb2_problem_destroy(gpb2_problem* p) {
    if (!p) return GPB2_OK;
    DeviceGuard dg(p->device);
    cudaDeviceSynchronize();
    free_problem(p);
    return GPB2_OK;
}

}  // extern "C"
