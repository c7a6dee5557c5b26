// gpb2_ops.cu -- the C-ABI operations: orchestration of the refine kernels, the dense layer and
// the tree<->original permutation (src/orchestrate.jl, src/api.jl, src/grad.jl,
// src/grad_generate_vals.jl).
//
// Forward and reverse depth sweeps.  The conditional-mean weights and std of every refined point
// depend only on the graph and the table, not on the field, so they are produced by one flat
// kernel over all M points (full-GPU occupancy regardless of batch sizes) and the depth batches
// are then swept by a light kernel per batch (K gathers and K multiply-adds per point).  The
// reference's fused per-batch kernel (refine_apply_fused_kernel!) recomputes the factor inside
// the sweep; it is kept as the "fused" forward mode (GPB2_FWD=fused) and gives the identical
// result bit for bit: both evaluate the same per-point arithmetic in the same order.
//
// generate_grad_vals.  Every point's contribution to d(vals) is linear in its final cotangent
// vb[p]; once the reverse sweep has finalised vb for all points, the per-point pullbacks are
// independent and run as one flat kernel instead of one launch per batch.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <string>

#include "gpb2_comm.h"
#include "gpb2_nvtx.h"
#include "gpb2_problem.h"

namespace gpb2 {

namespace {

template <typename T>
__global__ void k_gather(const T* __restrict__ src, const int* __restrict__ idx,
                         T* __restrict__ dst, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = src[idx[i]];
}

template <typename T>
__global__ void k_scatter(const T* __restrict__ src, const int* __restrict__ idx,
                          T* __restrict__ dst, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[idx[i]] = src[i];
}

// Between the reference's tree order and the library's (gpb2_order.cu), over positions
// [base, base + n): to_lib: dst[q] = src[map[base + q] - base]; else dst[map[base + q] - base] =
// src[q].
// (N, D) rows from library positions to tree positions, rounded to T:
// dst[lib_tree[q]] = src[q] (the identity without a library order).
template <typename T>
__global__ void k_rows_to_tree(const double* __restrict__ src, T* __restrict__ dst,
                               const int* __restrict__ lib_tree, int64_t n, int D) {
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n;
         q += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = lib_tree ? (int64_t)lib_tree[q] : q;
        for (int d = 0; d < D; d++) dst[t * D + d] = (T)src[q * D + d];
    }
}

template <typename T>
__global__ void k_lib_move(const T* __restrict__ src, T* __restrict__ dst,
                           const int* __restrict__ map, int64_t base, int64_t n, int to_lib) {
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n;
         q += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = (int64_t)map[base + q] - base;
        if (to_lib)
            dst[q] = src[t];
        else
            dst[t] = src[q];
    }
}

template <typename T>
__global__ void k_hist_to_t(const double* __restrict__ acc, T* __restrict__ out, int64_t nb) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nb;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (T)acc[i];
}

inline unsigned grid1d(int64_t n) {
    int64_t g = (n + 255) / 256;
    return (unsigned)(g < 1 ? 1 : (g > 148 * 16 ? 148 * 16 : g));
}

// Process-wide sweep strategy (GPB2_FWD=persistent|fused|batched at load time, or
// gpb2_set_forward_mode()): 0 = one cooperative kernel per sweep, 1 = the reference's fused
// per-batch forward kernel, 2 = one light kernel launch per batch.
enum class FwdMode { Persistent = 0, Fused = 1, Batched = 2, Flow = 3 };

std::atomic<int> g_fwd_mode{[] {
    const char* e = std::getenv("GPB2_FWD");
    if (e && std::strcmp(e, "fused") == 0) return 1;
    if (e && std::strcmp(e, "batched") == 0) return 2;
    if (e && std::strcmp(e, "flow") == 0) return 3;
    return 0;
}()};

FwdMode fwd_mode() { return static_cast<FwdMode>(g_fwd_mode.load()); }

// Process-wide call mode (GPB2_SYNC=0 at load time, or gpb2_set_synchronous()): 1 = every call
// waits for its work and reports its status; 0 = calls return once their work is queued and
// gpb2_problem_check() waits and reports (calls that return host values still wait for them).
std::atomic<int> g_sync{[] {
    const char* e = std::getenv("GPB2_SYNC");
    return (e && std::strcmp(e, "0") == 0) ? 0 : 1;
}()};

// Whether the dense first-layer work runs beside the per-point kernels on the problem's second
// stream (GPB2_OVERLAP=0 at load time, or gpb2_set_overlap(0), runs it on the call's stream).
std::atomic<bool> g_overlap_flag{[] {
    const char* e = std::getenv("GPB2_OVERLAP");
    return !(e && std::strcmp(e, "0") == 0);
}()};

// The problem's high-priority stream and its two events, created on first use.
static int ensure_dense_stream(gpb2_problem* p) {
    if (p->dstream) return GPB2_OK;
    int least = 0, greatest = 0;
    GPB2_CUDA_TRY(cudaDeviceGetStreamPriorityRange(&least, &greatest));
    GPB2_CUDA_TRY(cudaEventCreateWithFlags(&p->ev_fork, cudaEventDisableTiming));
    GPB2_CUDA_TRY(cudaEventCreateWithFlags(&p->ev_join, cudaEventDisableTiming));
    GPB2_CUDA_TRY(cudaEventCreateWithFlags(&p->ev_tri, cudaEventDisableTiming));
    GPB2_CUDA_TRY(cudaEventCreateWithFlags(&p->ev_inv, cudaEventDisableTiming));
    GPB2_CUDA_TRY(cudaStreamCreateWithPriority(&p->dstream, cudaStreamNonBlocking, greatest));
    return GPB2_OK;
}

}  // namespace

template <typename T>
struct Impl {
    using P = gpb2_problem;

    static int check_launch(cudaError_t e, const char* what) {
        if (e != cudaSuccess)
            return set_error(GPB2_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
        return GPB2_OK;
    }

    // original -> tree: dst[i] = src[indices[i]]
    static int gather(P* p, const T* src, T* dst, cudaStream_t s) {
        if (perm_two_pass(p)) return perm_apply<T>(p, true, src, dst, s);
        return check_launch(launch_prof("gather", k_gather<T>, dim3(grid1d(p->n)), dim3(256), 0,
                                        s, src, (const int*)p->indices, dst, p->n),
                            "gather");
    }
    // tree -> original: dst[indices[i]] = src[i]
    static int scatter(P* p, const T* src, T* dst, cudaStream_t s) {
        if (perm_two_pass(p)) return perm_apply<T>(p, false, src, dst, s);
        return check_launch(launch_prof("scatter", k_scatter<T>, dim3(grid1d(p->n)), dim3(256), 0,
                                        s, src, (const int*)p->indices, dst, p->n),
                            "scatter");
    }

    // mean_vec / std of every refined point.  They depend only on the graph and the table, so
    // they are computed once per table and reused by every call until the table changes.
    // With the factor cache allocated (mode 1 allocates it here), the same pass fills it.
    static int factor_all(P* p, cudaStream_t s) {
        if (p->factor_valid) return GPB2_OK;
        if (p->fc_mode == 1) GPB2_TRY(alloc_factor_cache(p));
        GPB2_TRY(check_launch(ops_of<T>(p)->factor(point_args<T>(p, FcUse::Fill), 0, p->m,
                                                   (T*)p->mv, (T*)p->sd, s),
                              "factor"));
        p->factor_valid = true;
        p->fc_valid = p->fc_L != nullptr;
        return GPB2_OK;
    }

    // The factor cache's buffers, as the mode allows: mode 1 always (an allocation failure is
    // the caller's error), mode 2 only when the device keeps a margin of free memory beyond it
    // (else, or on a failed allocation, nothing: the kernels recompute).
    static int alloc_factor_cache(P* p) {
        if (p->fc_L || p->fc_mode == 0 || p->m <= 0 || p->an_grid) return GPB2_OK;
        const size_t ts = sizeof(T);
        const size_t nt = (size_t)(p->k + 1) * (p->k + 2) / 2, nr = nt - (size_t)(p->k + 1);
        if (p->fc_mode == 2) {
            size_t fr = 0, tot = 0;
            if (cudaMemGetInfo(&fr, &tot) != cudaSuccess) {
                cudaGetLastError();
                return GPB2_OK;
            }
            const size_t margin = std::max(tot / 10, (size_t)8 << 30);
            if (fr < factor_cache_bytes(p) + margin) return GPB2_OK;
        }
        int st = ensure_alloc(&p->fc_L, ts * nt * p->m);
        if (!st) st = ensure_alloc(&p->fc_t, ts * nr * p->m);
        if (!st) st = ensure_alloc(reinterpret_cast<void**>(&p->fc_lo), 2 * nr * p->m);
        if (st) {
            for (void* b : {p->fc_L, p->fc_t, (void*)p->fc_lo})
                if (b) cudaFree(b);
            p->fc_L = p->fc_t = nullptr;
            p->fc_lo = nullptr;
            if (p->fc_mode == 1) return st;
            clear_error();
        }
        return GPB2_OK;
    }

    // Before generate_grad_vals' per-point kernel: the factor cache of the current table,
    // allocated as the mode allows and, when the factor pass of this table ran without it, filled
    // by a second factor pass (mean_vec / std are written again with the same bits).  The later
    // calls on the same table, and the factor passes of later tables, then read and fill it.
    static int ensure_factor_cache(P* p, cudaStream_t s) {
        if (p->fc_valid || p->fc_mode == 0 || p->m <= 0) return GPB2_OK;
        GPB2_TRY(alloc_factor_cache(p));
        if (!p->fc_L) return GPB2_OK;
        GPB2_TRY(ensure_scratch(p, true));
        GPB2_TRY(check_launch(ops_of<T>(p)->factor(point_args<T>(p, FcUse::Fill), 0, p->m,
                                                   (T*)p->mv, (T*)p->sd, s),
                              "factor cache"));
        p->factor_valid = true;
        p->fc_valid = true;
        return GPB2_OK;
    }

    // Both factors of the current table: the dense first-layer Cholesky and the per-point
    // mean_vec / std.  They are independent, and the dense ladder is a few thread-block clusters
    // whose candidates mostly stop early, leaving most SMs idle for most of its run.  When both
    // are stale the ladder runs on the problem's high-priority stream (its waiting clusters take
    // SMs as they free up, ahead of the other kernel's blocks) while the per-point factor fills
    // the remaining SMs on the call's stream; the call's stream then waits for the ladder.
    // Neither kernel waits on the other, so any co-scheduling is correct.
    static int factor_both(P* p, cudaStream_t s) {
        if (!g_overlap_flag.load() || p->dense_valid || p->factor_valid) {
            GPB2_TRY(Dense<T>::factor(p, s));
            return factor_all(p, s);
        }
        GPB2_TRY(ensure_dense_stream(p));
        GPB2_CUDA_TRY(cudaEventRecord(p->ev_fork, s));
        GPB2_CUDA_TRY(cudaStreamWaitEvent(p->dstream, p->ev_fork, 0));
        const int sd = Dense<T>::factor(p, p->dstream, true);
        const int sf = sd == GPB2_OK ? factor_all(p, s) : GPB2_OK;
        // The join is recorded whatever happened, so no kernel of the ladder outlives the stream.
        const cudaError_t e1 = cudaEventRecord(p->ev_join, p->dstream);
        const cudaError_t e2 = cudaStreamWaitEvent(s, p->ev_join, 0);
        GPB2_TRY(sd);
        GPB2_TRY(sf);
        GPB2_CUDA_TRY(e1);
        GPB2_CUDA_TRY(e2);
        // The triangular preparation needs only the factor and is queued after the join: it
        // runs beside the caller's next kernels (a forward sweep needs only the factor), and its
        // readers, and the call's final status read, wait for it.
        return Dense<T>::finish_tri(p, p->dstream);
    }

    // values[0:n0] preset; fills values[n0:N] batch by batch.
    static int refine_sweep(P* p, T* values, const T* xi_ref, bool have_factor, cudaStream_t s) {
        const Ops<T>* o = ops_of<T>(p);
        if (fwd_mode() == FwdMode::Fused && !have_factor) {
            const PointArgs<T> a = point_args<T>(p);
            for (size_t b = 1; b < p->offsets.size(); b++) {
                NvtxRange r("forward", (long long)b - 1);
                GPB2_TRY(check_launch(
                    o->fused_fwd(a, values, xi_ref, p->offsets[b - 1], p->offsets[b], s),
                    "fused forward"));
            }
            return GPB2_OK;
        }
        if (!have_factor) GPB2_TRY(factor_all(p, s));
        if (fwd_mode() == FwdMode::Flow) {
            GPB2_CUDA_TRY(cudaMemsetAsync(values + p->n0, 0xff, sizeof(T) * (p->n - p->n0), s));
            GPB2_TRY(check_launch(o->sweep_fwd_flow(values, xi_ref, (const T*)p->mv,
                                                    (const T*)p->sd, p->nbrs, p->n0, p->n,
                                                    reinterpret_cast<int*>(p->dsync + 2), s),
                                  "forward sweep"));
            return GPB2_OK;  // the wait error word is read when the call finishes
        }
        if (fwd_mode() == FwdMode::Persistent) {
            GPB2_TRY(arm_sync(p, s));
            GPB2_TRY(check_launch(o->sweep_fwd_all(values, xi_ref, (const T*)p->mv,
                                                   (const T*)p->sd, p->nbrs, p->n0, p->d_offsets,
                                                   nbatch(p), grid_sync_of(p), s),
                                  "forward sweep"));
            return GPB2_OK;  // the barrier's error word is read when the call finishes
        }
        for (size_t b = 1; b < p->offsets.size(); b++) {
            NvtxRange r("forward", (long long)b - 1);
            GPB2_TRY(check_launch(o->sweep_fwd(values, xi_ref, (const T*)p->mv,
                                               (const T*)p->sd, p->nbrs, p->n0,
                                               p->offsets[b - 1], p->offsets[b], s),
                                  "forward sweep"));
        }
        return GPB2_OK;
    }

    // The transposed graph of the pull-form reverse sweep (built on first use, its weights once
    // per table -- after the table's factor pass), or none: the atomic push.
    static int rev_graph(P* p, RevGraph<T>& rg, cudaStream_t s) {
        rg = RevGraph<T>{};
        if (p->rev_mode == 0) return GPB2_OK;
        GPB2_TRY(ensure_rev_graph(p, s));
        if (!p->rev_off) return GPB2_OK;
        GPB2_TRY(ensure_rev_weights<T>(p, s));
        rg.off = p->rev_off;
        rg.mj = p->rev_mj;
        rg.w = static_cast<const T*>(p->rev_w);
        return GPB2_OK;
    }

    // Reverse sweep over the batches, latest first; xg may be NULL.
    static int reverse_sweep(P* p, T* xg, T* vb, cudaStream_t s) {
        const Ops<T>* o = ops_of<T>(p);
        if (fwd_mode() == FwdMode::Persistent || fwd_mode() == FwdMode::Flow) {
            RevGraph<T> rg;
            GPB2_TRY(rev_graph(p, rg, s));
            GPB2_TRY(arm_sync(p, s));
            GPB2_TRY(check_launch(o->sweep_rev_all(xg, vb, (const T*)p->mv, (const T*)p->sd,
                                                   p->nbrs, p->n0, p->d_offsets, nbatch(p), rg,
                                                   grid_sync_of(p), s),
                                  "reverse sweep"));
            return GPB2_OK;
        }
        for (size_t b = p->offsets.size() - 1; b >= 1; b--) {
            NvtxRange r("reverse", (long long)b - 1);
            GPB2_TRY(check_launch(o->sweep_rev(xg, vb, (const T*)p->mv, (const T*)p->sd, p->nbrs,
                                               p->n0, p->offsets[b - 1], p->offsets[b], s),
                                  "reverse sweep"));
        }
        return GPB2_OK;
    }

    static int nbatch(P* p) { return (int)p->offsets.size() - 1; }
    static GridSync grid_sync_of(P* p) {
        return GridSync{p->dsync, reinterpret_cast<int*>(p->dsync + 2)};
    }
    // Zero the barrier words before a cooperative launch (the error word accumulates over the
    // call and is cleared by finish_call).
    static int arm_sync(P* p, cudaStream_t s) {
        GPB2_CUDA_TRY(cudaMemsetAsync(p->dsync, 0, 2 * sizeof(unsigned int), s));
        return GPB2_OK;
    }

    static int finish_hist(P* p, T* dvals, cudaStream_t s) {
        return check_launch(launch_prof("hist_to_t", k_hist_to_t<T>, dim3(grid1d(p->nb)),
                                        dim3(256), 0, s, (const double*)p->dacc, dvals, p->nb),
                            "histogram convert");
    }

    static int zero_acc(P* p, cudaStream_t s) {
        GPB2_CUDA_TRY(cudaMemsetAsync(p->dacc, 0, sizeof(double) * (p->nb + 8), s));
        return GPB2_OK;
    }

    // The four scalar accumulators after the histogram, through pinned host memory.
    static int read_scalars(P* p, double* h, cudaStream_t s) {
        if (!p->hscal)
            GPB2_CUDA_TRY(cudaMallocHost(reinterpret_cast<void**>(&p->hscal), 4 * sizeof(double)));
        GPB2_CUDA_TRY(cudaMemcpyAsync(p->hscal, p->dacc + p->nb, sizeof(double) * 4,
                                      cudaMemcpyDeviceToHost, s));
        GPB2_CUDA_TRY(cudaStreamSynchronize(s));
        for (int i = 0; i < 4; i++) h[i] = p->hscal[i];
        return GPB2_OK;
    }

    // ---------------------------------------------------------------- tree order <-> library order
    static int lib_move(P* p, const T* src, T* dst, int64_t base, int64_t n, bool to_lib,
                        cudaStream_t s) {
        return check_launch(launch_prof("order", k_lib_move<T>, dim3(grid1d(n)), dim3(256), 0, s,
                                        src, dst, (const int*)p->lib_tree, base, n,
                                        to_lib ? 1 : 0),
                            "order");
    }
    // The reference's tree-order entry points: inputs into library order, the operation, outputs
    // back (positions [0, n0) are the same in both orders).
    static int refine_tree(P* p, T* values, const T* xi_ref, cudaStream_t s) {
        if (!p->lib_tree) return refine(p, values, xi_ref, s);
        GPB2_TRY(ensure_scratch(p, true));
        T* vl = (T*)p->buf_a;
        T* xl = (T*)p->buf_b;
        GPB2_TRY(lib_move(p, xi_ref, xl, p->n0, p->m, true, s));
        GPB2_CUDA_TRY(cudaMemcpyAsync(vl, values, sizeof(T) * p->n0, cudaMemcpyDeviceToDevice, s));
        GPB2_TRY(refine(p, vl, xl, s));
        return lib_move(p, vl + p->n0, values + p->n0, p->n0, p->m, false, s);
    }
    static int refine_inv_tree(P* p, const T* values, T* xi_ref, cudaStream_t s) {
        if (!p->lib_tree) return refine_inv(p, values, xi_ref, s);
        GPB2_TRY(ensure_scratch(p, false));
        T* vl = (T*)p->buf_a;
        T* xl = (T*)p->buf_b;
        GPB2_TRY(lib_move(p, values, vl, 0, p->n, true, s));
        GPB2_TRY(refine_inv(p, vl, xl, s));
        return lib_move(p, xl, xi_ref, p->n0, p->m, false, s);
    }
    static int refine_logdet_tree(P* p, T* terms, double* out, cudaStream_t s) {
        if (!p->lib_tree || !terms) return refine_logdet(p, terms, out, s);
        GPB2_TRY(ensure_scratch(p, false));
        T* tl = (T*)p->buf_b;
        GPB2_TRY(refine_logdet(p, tl, out, s));
        return lib_move(p, tl, terms, p->n0, p->m, false, s);
    }
    // ------------------------------------------------- point-position gradients, tree order
    // (src/grad.jl:168-377).  Accumulated in library positions (N, D), the refined points'
    // part (values_lib: the inverse loss, else the log-determinant) and, with `dense`, the dense
    // block's (y_dense: its first n0 values); then the rows go to tree order.
    static int points_grad(P* p, const T* values_lib, bool dense, const T* y_dense, T* dp_tree,
                           cudaStream_t s) {
        const int D = (int)p->d;
        const size_t bytes = sizeof(double) * (size_t)p->n * D;
        GPB2_TRY(ensure_alloc(reinterpret_cast<void**>(&p->dpts), bytes));
        double* dl = p->dpts;
        GPB2_CUDA_TRY(cudaMemsetAsync(dl, 0, bytes, s));
        GPB2_TRY(check_launch(ops_of<T>(p)->points_grad(point_args<T>(p), values_lib, dl,
                                                        Pts::all(p->m), s),
                              "points grad"));
        if (dense) {
            GPB2_TRY(Dense<T>::factor(p, s));
            if (values_lib)
                GPB2_TRY(Dense<T>::inv_loss_points(p, y_dense, dl, s));
            else
                GPB2_TRY(Dense<T>::logdet_points(p, dl, s));
        }
        return check_launch(launch_prof("order", k_rows_to_tree<T>, dim3(grid1d(p->n)), dim3(256),
                                        0, s, (const double*)dl, dp_tree, (const int*)p->lib_tree,
                                        p->n, D),
                            "order");
    }
    static int refine_logdet_grad_points(P* p, T* dp, cudaStream_t s) {
        return points_grad(p, nullptr, false, nullptr, dp, s);
    }
    static int generate_logdet_grad_points(P* p, T* dp, cudaStream_t s) {
        return points_grad(p, nullptr, true, nullptr, dp, s);
    }
    static int refine_inv_loss_grad_points(P* p, const T* values, T* dp, cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, false));
        const T* vl = values;
        if (p->lib_tree) {
            GPB2_TRY(lib_move(p, values, (T*)p->buf_b, 0, p->n, true, s));
            vl = (const T*)p->buf_b;
        }
        return points_grad(p, vl, false, nullptr, dp, s);
    }
    static int generate_inv_loss_grad_points(P* p, const T* data, T* dp, cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, false));
        const T* yl = data;
        if (p->indices) {
            GPB2_TRY(gather(p, data, (T*)p->buf_a, s));
            yl = (const T*)p->buf_a;
        }
        return points_grad(p, yl, true, yl, dp, s);
    }

    static int refine_inv_loss_tree(P* p, const T* values, T* dvals, double* loss,
                                    cudaStream_t s) {
        if (!p->lib_tree) return refine_inv_loss_grad_vals(p, values, dvals, loss, s);
        GPB2_TRY(ensure_scratch(p, false));
        T* vl = (T*)p->buf_b;
        GPB2_TRY(lib_move(p, values, vl, 0, p->n, true, s));
        return refine_inv_loss_grad_vals(p, vl, dvals, loss, s);
    }

    // ---------------------------------------------------------------- refine layer (library order)
    static int refine(P* p, T* values, const T* xi_ref, cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, true));
        return refine_sweep(p, values, xi_ref, false, s);
    }

    static int refine_inv(P* p, const T* values, T* xi_ref, cudaStream_t s) {
        return check_launch(ops_of<T>(p)->inv(point_args<T>(p), values, xi_ref, Pts::all(p->m), s),
                            "refine_inv");
    }

    static int refine_logdet(P* p, T* terms, double* out, cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, false));
        GPB2_TRY(zero_acc(p, s));
        GPB2_TRY(check_launch(
            ops_of<T>(p)->logdet(point_args<T>(p), terms, p->dacc + p->nb, Pts::all(p->m), s), "logdet"));
        if (out) {
            double h[4];
            GPB2_TRY(read_scalars(p, h, s));
            *out = h[0];
        }
        return GPB2_OK;
    }

    static int refine_logdet_grad_vals(P* p, T* dvals, double* ld, cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, false));
        GPB2_TRY(zero_acc(p, s));
        GPB2_TRY(check_launch(ops_of<T>(p)->logdet_grad(point_args<T>(p, FcUse::Read), p->dacc,
                                                        p->dacc + p->nb, nullptr, Pts::all(p->m), s),
                              "logdet grad"));
        GPB2_TRY(finish_hist(p, dvals, s));
        if (ld) {
            double h[4];
            GPB2_TRY(read_scalars(p, h, s));
            *ld = h[0];
        }
        return GPB2_OK;
    }

    static int refine_inv_loss_grad_vals(P* p, const T* values, T* dvals, double* loss,
                                         cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, false));
        GPB2_TRY(zero_acc(p, s));
        GPB2_TRY(check_launch(ops_of<T>(p)->inv_loss_grad(point_args<T>(p, FcUse::Read), values, p->dacc,
                                                          p->dacc + p->nb + 1, nullptr, Pts::all(p->m), s),
                              "inverse-loss grad"));
        GPB2_TRY(finish_hist(p, dvals, s));
        if (loss) {
            double h[4];
            GPB2_TRY(read_scalars(p, h, s));
            *loss = h[1];
        }
        return GPB2_OK;
    }

    // ---------------------------------------------------------------- ranges of one depth batch
    // (the building blocks of a level-sharded sweep: each rank runs its slice of a batch, the
    // caller exchanges the batch's values between ranks; asynchronous on `s`)
    static int refine_range(P* p, T* values, const T* xi_ref, int64_t lo, int64_t hi,
                            cudaStream_t s) {
        return check_launch(
            ops_of<T>(p)->fused_fwd(point_args<T>(p), values, xi_ref, lo, hi, s), "refine range");
    }

    static int reverse_range(P* p, T* xg, T* vb, int64_t lo, int64_t hi, cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, true));
        if (!p->factor_valid)
            GPB2_TRY(check_launch(ops_of<T>(p)->factor(point_args<T>(p), lo - p->n0, hi - p->n0,
                                                       (T*)p->mv, (T*)p->sd, s),
                                  "factor range"));
        return check_launch(ops_of<T>(p)->sweep_rev(xg, vb, (const T*)p->mv, (const T*)p->sd,
                                                    p->nbrs, p->n0, lo, hi, s),
                            "reverse range");
    }

    // Both factorisations of the current table, queued on s without waiting for them.
    static int prefactor(P* p, cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, true));
        return factor_both(p, s);
    }

    static int dense_apply(P* p, int trans, const T* x, T* y, cudaStream_t s) {
        GPB2_TRY(Dense<T>::factor(p, s));
        return trans ? Dense<T>::apply_Lt(p, x, y, s) : Dense<T>::apply_L(p, x, y, s);
    }

    // ---------------------------------------------------------------- orchestrated (original order)
    static int generate(P* p, const T* xi, T* out, cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, true));
        const T* xt = xi;
        if (p->indices) {
            GPB2_TRY(gather(p, xi, (T*)p->buf_b, s));
            xt = (const T*)p->buf_b;
        }
        T* values = p->indices ? (T*)p->buf_a : out;
        GPB2_TRY(fwd_mode() == FwdMode::Fused ? Dense<T>::factor(p, s) : factor_both(p, s));
        GPB2_TRY(Dense<T>::apply_L(p, xt, values, s));
        GPB2_TRY(refine_sweep(p, values, xt + p->n0, false, s));
        if (p->indices) GPB2_TRY(scatter(p, values, out, s));
        return GPB2_OK;
    }

    static int generate_inv(P* p, const T* values, T* xi, cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, false));
        const T* vt = values;
        if (p->indices) {
            GPB2_TRY(gather(p, values, (T*)p->buf_a, s));
            vt = (const T*)p->buf_a;
        }
        T* xt = p->indices ? (T*)p->buf_b : xi;
        GPB2_TRY(refine_inv(p, vt, xt + p->n0, s));
        GPB2_TRY(Dense<T>::factor(p, s));
        GPB2_TRY(Dense<T>::solve_L(p, vt, xt, s));
        if (p->indices) GPB2_TRY(scatter(p, xt, xi, s));
        return GPB2_OK;
    }

    static int generate_logdet(P* p, double* out, cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, false));
        GPB2_TRY(zero_acc(p, s));
        GPB2_TRY(Dense<T>::factor(p, s));
        GPB2_TRY(Dense<T>::logdet(p, p->dacc + p->nb + 2, s));
        GPB2_TRY(check_launch(
            ops_of<T>(p)->logdet(point_args<T>(p), nullptr, p->dacc + p->nb, Pts::all(p->m), s), "logdet"));
        double h[4];
        GPB2_TRY(read_scalars(p, h, s));
        *out = h[2] + h[0];
        return GPB2_OK;
    }

    static int generate_grad_xi(P* p, const T* vbar, T* xbar, cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, true));
        T* vb = (T*)p->buf_c;
        if (p->indices)
            GPB2_TRY(gather(p, vbar, vb, s));
        else
            GPB2_CUDA_TRY(
                cudaMemcpyAsync(vb, vbar, sizeof(T) * p->n, cudaMemcpyDeviceToDevice, s));
        T* xg = p->indices ? (T*)p->buf_d : xbar;
        GPB2_TRY(factor_both(p, s));
        GPB2_TRY(reverse_sweep(p, xg, vb, s));
        GPB2_TRY(Dense<T>::apply_Lt(p, vb, xg, s));
        if (p->indices) GPB2_TRY(scatter(p, xg, xbar, s));
        return GPB2_OK;
    }

    static int generate_grad_vals(P* p, const T* xi, const T* vbar, T* dvals, cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, true));
        const T* xt = xi;
        if (p->indices) {
            GPB2_TRY(gather(p, xi, (T*)p->buf_b, s));
            xt = (const T*)p->buf_b;
        }
        T* v = (T*)p->buf_a;
        T* vb = (T*)p->buf_c;
        GPB2_TRY(factor_both(p, s));
        GPB2_TRY(Dense<T>::apply_L(p, xt, v, s));
        if (p->indices)
            GPB2_TRY(gather(p, vbar, vb, s));
        else
            GPB2_CUDA_TRY(
                cudaMemcpyAsync(vb, vbar, sizeof(T) * p->n, cudaMemcpyDeviceToDevice, s));
        if (fwd_mode() == FwdMode::Persistent) {  // both sweeps in one persistent kernel
            RevGraph<T> rg;
            GPB2_TRY(rev_graph(p, rg, s));
            GPB2_TRY(arm_sync(p, s));
            GPB2_TRY(check_launch(ops_of<T>(p)->sweep_fwdrev_all(
                                      v, xt + p->n0, vb, (const T*)p->mv, (const T*)p->sd,
                                      p->nbrs, p->n0, p->d_offsets, nbatch(p), rg,
                                      grid_sync_of(p), s),
                                  "forward+reverse sweep"));
        } else {
            GPB2_TRY(refine_sweep(p, v, xt + p->n0, true, s));
            GPB2_TRY(reverse_sweep(p, nullptr, vb, s));
        }
        GPB2_TRY(ensure_factor_cache(p, s));
        GPB2_TRY(zero_acc(p, s));
        auto per_point = [&](cudaStream_t st) {
            return check_launch(ops_of<T>(p)->grad_vals(point_args<T>(p, FcUse::Read), v, xt, vb,
                                                        (const T*)p->mv, p->dacc, Pts::all(p->m), st),
                                "grad_vals");
        };
        GPB2_TRY(hist_and_dense(p, per_point, true, vb, xt, s));
        return finish_hist(p, dvals, s);
    }

    // The per-point histogram kernel and (when `dense`) the dense block's pullback: independent,
    // both adding into p->dacc.  The dense chain (a short run of small kernels) goes first, on
    // the high-priority stream, and runs beside the per-point kernel (one after the other with
    // the overlap off: GPB2_OVERLAP=0, gpb2_set_overlap(0)).
    template <class PerPoint>
    static int hist_and_dense(P* p, PerPoint per_point, bool dense, const T* vb, const T* xt,
                              cudaStream_t s) {
        if (!dense) return per_point(s);
        if (!g_overlap_flag.load()) {
            GPB2_TRY(per_point(s));
            return Dense<T>::grad_vals(p, vb, xt, p->dacc, s);
        }
        GPB2_TRY(ensure_dense_stream(p));
        GPB2_CUDA_TRY(cudaEventRecord(p->ev_fork, s));
        GPB2_CUDA_TRY(cudaStreamWaitEvent(p->dstream, p->ev_fork, 0));
        const int sd = Dense<T>::grad_vals(p, vb, xt, p->dacc, p->dstream);
        const int sp = sd == GPB2_OK ? per_point(s) : GPB2_OK;
        const cudaError_t e1 = cudaEventRecord(p->ev_join, p->dstream);
        const cudaError_t e2 = cudaStreamWaitEvent(s, p->ev_join, 0);
        GPB2_TRY(sd);
        GPB2_TRY(sp);
        GPB2_CUDA_TRY(e1);
        GPB2_CUDA_TRY(e2);
        return GPB2_OK;
    }

    static int generate_logdet_grad_vals(P* p, T* dvals, double* ld, cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, false));
        GPB2_TRY(zero_acc(p, s));
        GPB2_TRY(check_launch(ops_of<T>(p)->logdet_grad(point_args<T>(p, FcUse::Read), p->dacc,
                                                        p->dacc + p->nb, nullptr, Pts::all(p->m), s),
                              "logdet grad"));
        GPB2_TRY(Dense<T>::factor(p, s));
        GPB2_TRY(Dense<T>::logdet(p, p->dacc + p->nb + 2, s));
        GPB2_TRY(Dense<T>::logdet_grad(p, p->dacc, s));
        GPB2_TRY(finish_hist(p, dvals, s));
        if (ld) {
            double h[4];
            GPB2_TRY(read_scalars(p, h, s));
            *ld = h[2] + h[0];
        }
        return GPB2_OK;
    }

    static int generate_inv_loss_grad_vals(P* p, const T* data, T* dvals, double* loss,
                                           cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, false));
        const T* yt = data;
        if (p->indices) {
            GPB2_TRY(gather(p, data, (T*)p->buf_a, s));
            yt = (const T*)p->buf_a;
        }
        GPB2_TRY(zero_acc(p, s));
        GPB2_TRY(check_launch(ops_of<T>(p)->inv_loss_grad(point_args<T>(p, FcUse::Read), yt, p->dacc,
                                                          p->dacc + p->nb + 1, nullptr, Pts::all(p->m), s),
                              "inverse-loss grad"));
        GPB2_TRY(Dense<T>::factor(p, s));
        GPB2_TRY(Dense<T>::inv_loss_grad(p, yt, p->dacc, p->dacc + p->nb + 1, s));
        GPB2_TRY(finish_hist(p, dvals, s));
        if (loss) {
            double h[4];
            GPB2_TRY(read_scalars(p, h, s));
            *loss = h[1];
        }
        return GPB2_OK;
    }
};

// Every call ends here: one synchronisation of the stream, after which the status words the
// device left behind are read -- a grid barrier that timed out (persistent sweeps, dense
// factorisation) or a dense block that no ladder step could factorise (src/dense.jl:65-66).
// The reference's drivers also synchronise before returning (e.g. src/api.jl:139).
static int finish_call(gpb2_problem* p, cudaStream_t s) {
    // Status words land in pinned host memory: the copies queue behind the call's kernels and
    // one synchronisation waits for all of them (copies to pageable memory would each wait).
    if (!p->hstat) GPB2_CUDA_TRY(cudaMallocHost(reinterpret_cast<void**>(&p->hstat), 4 * sizeof(int)));
    // Nothing the call queued on the dense stream outlives it: the status reads below (and the
    // synchronisation) come after the triangular preparation.
    const bool tri = p->tri_pending;
    if (tri) GPB2_CUDA_TRY(cudaStreamWaitEvent(s, p->ev_inv, 0));
    int* h = p->hstat;
    h[0] = 0;
    h[1] = 0;
    h[2] = 0;
    h[3] = -1;
    GPB2_CUDA_TRY(cudaMemcpyAsync(&h[0], p->dsync + 2, sizeof(int), cudaMemcpyDeviceToHost, s));
    const bool dense = p->dense_pending && p->lad;
    if (dense) {
        GPB2_CUDA_TRY(
            cudaMemcpyAsync(&h[1], p->lad + kLadNotPD, sizeof(int), cudaMemcpyDeviceToHost, s));
        GPB2_CUDA_TRY(
            cudaMemcpyAsync(&h[2], p->lad + kLadBarErr, sizeof(int), cudaMemcpyDeviceToHost, s));
        GPB2_CUDA_TRY(
            cudaMemcpyAsync(&h[3], p->lad + kLadSel, sizeof(int), cudaMemcpyDeviceToHost, s));
    }
    GPB2_CUDA_TRY(cudaStreamSynchronize(s));
    if (tri) p->tri_pending = false;
    p->dense_pending = false;
    if (dense) {
        p->dense_valid = h[0] == 0 && h[1] == 0 && h[2] == 0;
        if (!p->dense_valid) p->dense_launched = false;  // the next call factorises again
    }
    // The selected ladder step orders the next factorisation's speculative candidates.
    if (dense && h[3] >= 0) p->ladder_hint = h[3];
    if (h[0] != 0) {
        cudaMemsetAsync(p->dsync + 2, 0, sizeof(int), s);
        return set_error(GPB2_ERR_TIMEOUT, "a grid barrier of a persistent sweep timed out");
    }
    if (dense && h[2] != 0)
        return set_error(GPB2_ERR_TIMEOUT, "a grid barrier of the dense factorisation timed out");
    if (dense && h[1] != 0)
        return set_error(GPB2_ERR_NOT_PD,
                         "dense first-layer covariance is not positive definite even with 1e-2 "
                         "relative jitter; increase the kernel `jitter` or reduce n0");
    return GPB2_OK;
}

// ---------------------------------------------------------------------------------------------
// Level-sharded operations over the ranks of a gpb2_comm (one process or thread per GPU).
//
// Every rank holds the same problem (graph, table, dense factor) and the whole field; inputs and
// outputs are full length, in original order, on every rank.  Depth batch b = [lo, hi) of at
// least min_shard points is cut into `ranks` chunks of c = ceil((hi - lo) / ranks) points;
// rank r owns [lo + r c, lo + (r+1) c) (clipped to hi).  Smaller batches are not split for the
// forward sweep (every rank computes them, no exchange).  This is the reference's distributed
// per-level loop (src/distributed.jl:281-331), whose sum-Allreduce per level becomes an
// in-place all-gather of the owners' chunks.
//
// Forward: per batch, the owners' chunks, then an in-place NCCL all-gather completes the batch
// everywhere (the gather may spill past hi into later batches' slots, rewritten when they are
// computed, and past N into slack).
// Reverse (generate_grad_xi, and generate_grad_vals' cotangent sweep): each rank keeps a partial
// cotangent vb; rank 0 starts with vbar, the others with 0.  Latest batch first: its segment is
// summed over the ranks (in-place reduce-scatter for a sharded batch, all-reduce for a small
// one), then every rank scatters the contributions of the points it owns (a small batch's points
// are split for this step only, so that each is scattered once).  The dense block's cotangents
// and the xi-cotangents are summed over the ranks at the end.
// generate_grad_vals: every rank then runs the per-point vals-gradient on the points it owns
// (their cotangents are complete there); the dense block's pullback runs on rank 0; one
// all-reduce of the nbins double histogram.
// Fitting reductions (scheme A of src/distributed.jl:129-247): the refined points are split into
// contiguous per-rank ranges; one all-reduce of the nbins + 4 double accumulators.
struct ShardBatch {
    int64_t lo, hi, chunk;
    bool sharded;
};

struct ShardPlan {
    std::vector<ShardBatch> b;
    int64_t slack = 0;
    int ranks = 1, rank = 0;

    static ShardPlan make(const std::vector<int64_t>& offs, int ranks, int rank, int64_t min_shard) {
        ShardPlan pl;
        pl.ranks = ranks;
        pl.rank = rank;
        const int64_t n = offs.back();
        for (size_t i = 1; i < offs.size(); i++) {
            const int64_t lo = offs[i - 1], hi = offs[i], size = hi - lo;
            const bool sh = ranks > 1 && size >= std::max<int64_t>(min_shard, ranks);
            const int64_t c = sh ? (size + ranks - 1) / ranks : size;
            pl.b.push_back(ShardBatch{lo, hi, c, sh});
            if (sh) pl.slack = std::max(pl.slack, lo + ranks * c - n);
        }
        return pl;
    }
    // The points of batch b this rank computes in the forward sweep.
    void fwd_range(const ShardBatch& x, int64_t& a, int64_t& e) const {
        if (!x.sharded) {
            a = x.lo;
            e = x.hi;
            return;
        }
        a = std::min(x.hi, x.lo + rank * x.chunk);
        e = std::min(x.hi, a + x.chunk);
    }
    // The points of batch b whose cotangents this rank scatters (each point on one rank).
    void own_range(const ShardBatch& x, int64_t& a, int64_t& e) const {
        const int64_t c = x.sharded ? x.chunk : (x.hi - x.lo + ranks - 1) / ranks;
        a = std::min(x.hi, x.lo + rank * c);
        e = std::min(x.hi, a + c);
    }
};

template <typename T>
struct Shard {
    using P = gpb2_problem;
    static constexpr bool kF64 = sizeof(T) == 8;

    // Buffers with slack and the rank's own point list (built once per sharding).
    static int prepare(P* p, gpb2_comm* c, const ShardPlan& pl) {
        GPB2_TRY(ensure_scratch(p, true));
        const int64_t len = p->n + pl.slack + 1;
        if (p->sh_len < len) {
            void* bufs[3] = {p->sh_v, p->sh_vb, p->sh_xg};
            for (void* b : bufs)
                if (b) cudaFree(b);
            p->sh_v = p->sh_vb = p->sh_xg = nullptr;
            p->sh_len = 0;
            GPB2_TRY(ensure_alloc(&p->sh_v, sizeof(T) * len));
            GPB2_TRY(ensure_alloc(&p->sh_vb, sizeof(T) * len));
            GPB2_TRY(ensure_alloc(&p->sh_xg, sizeof(T) * len));
            p->sh_len = len;
        }
        const int64_t key[3] = {pl.ranks, pl.rank, comm_min_shard(c)};
        if (p->sh_own && std::equal(key, key + 3, p->sh_key)) return GPB2_OK;
        std::vector<int> own;
        own.reserve((size_t)(p->m / pl.ranks + p->offsets.size() + 16));
        for (const ShardBatch& x : pl.b) {
            int64_t a, e;
            pl.own_range(x, a, e);
            for (int64_t q = a; q < e; q++) own.push_back((int)(q - p->n0));
        }
        if (p->sh_own) cudaFree(p->sh_own);
        p->sh_own = nullptr;
        p->sh_own_cnt = 0;
        GPB2_TRY(ensure_alloc(reinterpret_cast<void**>(&p->sh_own), sizeof(int) * std::max<size_t>(own.size(), 1)));
        GPB2_CUDA_TRY(cudaMemcpy(p->sh_own, own.data(), sizeof(int) * own.size(),
                                 cudaMemcpyHostToDevice));
        p->sh_own_cnt = (int64_t)own.size();
        std::copy(key, key + 3, p->sh_key);
        p->sh_factor_valid = false;
        p->fc_sh_valid = false;
        return GPB2_OK;
    }

    // mean_vec / std of the points this rank's sweeps read: its forward ranges (which contain
    // its reverse ranges and the points it owns).  Nothing when every point's factor is current
    // -- unless the vals-gradient wants the factor cache (allocated as its mode allows), which
    // the same pass then fills for those ranges.
    static int factor(P* p, const ShardPlan& pl, cudaStream_t s, bool want_cache = false) {
        if (want_cache) GPB2_TRY(Impl<T>::alloc_factor_cache(p));
        const bool fill = want_cache && p->fc_L && !p->fc_valid && !p->fc_sh_valid;
        if ((p->factor_valid || p->sh_factor_valid) && !fill) return GPB2_OK;
        const Ops<T>* o = ops_of<T>(p);
        const PointArgs<T> a = point_args<T>(p, fill ? FcUse::Fill : FcUse::None);
        for (const ShardBatch& x : pl.b) {
            int64_t lo, hi;
            pl.fwd_range(x, lo, hi);
            if (hi > lo)
                GPB2_TRY(Impl<T>::check_launch(
                    o->factor(a, lo - p->n0, hi - p->n0, (T*)p->mv, (T*)p->sd, s), "factor"));
        }
        if (!p->factor_valid) p->sh_factor_valid = true;
        if (fill) p->fc_sh_valid = true;
        return GPB2_OK;
    }

    static int forward(P* p, gpb2_comm* c, const ShardPlan& pl, const T* xt, T* v,
                       cudaStream_t s) {
        const Ops<T>* o = ops_of<T>(p);
        GPB2_TRY(Dense<T>::apply_L(p, xt, v, s));
        for (const ShardBatch& x : pl.b) {
            NvtxRange r("forward", (long long)(&x - pl.b.data()));
            int64_t a, e;
            pl.fwd_range(x, a, e);
            GPB2_TRY(Impl<T>::check_launch(o->sweep_fwd(v, xt + p->n0, (const T*)p->mv,
                                                        (const T*)p->sd, p->nbrs, p->n0, a, e, s),
                                           "forward sweep"));
            if (x.sharded) GPB2_TRY(comm_all_gather(c, v, x.lo, x.chunk, kF64, s));
        }
        return GPB2_OK;
    }

    // On entry vb holds this rank's share of the cotangent (full length); on exit the points this
    // rank owns hold their complete cotangents, vb[0:n0] the dense block's (summed), and xg (if
    // given) the xi-cotangents of the refined points, summed over the ranks.
    static int reverse(P* p, gpb2_comm* c, const ShardPlan& pl, T* vb, T* xg, cudaStream_t s) {
        const Ops<T>* o = ops_of<T>(p);
        for (size_t i = pl.b.size(); i-- > 0;) {
            const ShardBatch& x = pl.b[i];
            if (x.hi <= x.lo) continue;
            NvtxRange r("reverse", (long long)i);
            if (x.sharded)
                GPB2_TRY(comm_reduce_scatter(c, vb, x.lo, x.chunk, kF64, s));
            else
                GPB2_TRY(comm_all_reduce(c, vb + x.lo, x.hi - x.lo, kF64, s));
            int64_t a, e;
            pl.own_range(x, a, e);
            GPB2_TRY(Impl<T>::check_launch(o->sweep_rev(xg, vb, (const T*)p->mv, (const T*)p->sd,
                                                        p->nbrs, p->n0, a, e, s),
                                           "reverse sweep"));
        }
        GPB2_TRY(comm_all_reduce(c, vb, p->n0, kF64, s));
        if (xg) GPB2_TRY(comm_all_reduce(c, xg + p->n0, p->m, kF64, s));
        return GPB2_OK;
    }

    static const T* to_tree(P* p, const T* x, T* buf, cudaStream_t s, int* st) {
        if (!p->indices) return x;
        *st = Impl<T>::gather(p, x, buf, s);
        return buf;
    }

    static int generate(P* p, gpb2_comm* c, const T* xi, T* out, cudaStream_t s) {
        const ShardPlan pl = ShardPlan::make(p->offsets, comm_size(c), comm_rank(c),
                                             comm_min_shard(c));
        GPB2_TRY(prepare(p, c, pl));
        int st = GPB2_OK;
        const T* xt = to_tree(p, xi, (T*)p->buf_b, s, &st);
        GPB2_TRY(st);
        GPB2_TRY(Dense<T>::factor(p, s));
        GPB2_TRY(factor(p, pl, s));
        T* v = (T*)p->sh_v;
        GPB2_TRY(forward(p, c, pl, xt, v, s));
        if (p->indices) return Impl<T>::scatter(p, v, out, s);
        GPB2_CUDA_TRY(cudaMemcpyAsync(out, v, sizeof(T) * p->n, cudaMemcpyDeviceToDevice, s));
        return GPB2_OK;
    }

    // The rank's share of the upstream cotangent in tree order: vbar on rank 0, zero elsewhere.
    static int seed_cotangent(P* p, gpb2_comm* c, const T* vbar, T* vb, cudaStream_t s) {
        GPB2_CUDA_TRY(cudaMemsetAsync(vb, 0, sizeof(T) * p->sh_len, s));
        if (comm_rank(c) != 0) return GPB2_OK;
        if (p->indices) return Impl<T>::gather(p, vbar, vb, s);
        GPB2_CUDA_TRY(cudaMemcpyAsync(vb, vbar, sizeof(T) * p->n, cudaMemcpyDeviceToDevice, s));
        return GPB2_OK;
    }

    static int grad_xi(P* p, gpb2_comm* c, const T* vbar, T* xbar, cudaStream_t s) {
        const ShardPlan pl = ShardPlan::make(p->offsets, comm_size(c), comm_rank(c),
                                             comm_min_shard(c));
        GPB2_TRY(prepare(p, c, pl));
        T* vb = (T*)p->sh_vb;
        T* xg = (T*)p->sh_xg;
        GPB2_TRY(seed_cotangent(p, c, vbar, vb, s));
        GPB2_CUDA_TRY(cudaMemsetAsync(xg, 0, sizeof(T) * p->sh_len, s));
        GPB2_TRY(Dense<T>::factor(p, s));
        GPB2_TRY(factor(p, pl, s));
        GPB2_TRY(reverse(p, c, pl, vb, xg, s));
        GPB2_TRY(Dense<T>::apply_Lt(p, vb, xg, s));
        if (p->indices) return Impl<T>::scatter(p, xg, xbar, s);
        GPB2_CUDA_TRY(cudaMemcpyAsync(xbar, xg, sizeof(T) * p->n, cudaMemcpyDeviceToDevice, s));
        return GPB2_OK;
    }

    static int grad_vals(P* p, gpb2_comm* c, const T* xi, const T* vbar, T* dvals,
                         cudaStream_t s) {
        const ShardPlan pl = ShardPlan::make(p->offsets, comm_size(c), comm_rank(c),
                                             comm_min_shard(c));
        GPB2_TRY(prepare(p, c, pl));
        int st = GPB2_OK;
        const T* xt = to_tree(p, xi, (T*)p->buf_b, s, &st);
        GPB2_TRY(st);
        GPB2_TRY(Dense<T>::factor(p, s));
        GPB2_TRY(factor(p, pl, s, true));
        T* v = (T*)p->sh_v;
        T* vb = (T*)p->sh_vb;
        GPB2_TRY(forward(p, c, pl, xt, v, s));
        GPB2_TRY(seed_cotangent(p, c, vbar, vb, s));
        GPB2_TRY(reverse(p, c, pl, vb, nullptr, s));
        GPB2_TRY(Impl<T>::zero_acc(p, s));
        auto per_point = [&](cudaStream_t st) {
            return Impl<T>::check_launch(
                ops_of<T>(p)->grad_vals(point_args<T>(p, FcUse::ReadShard), v, xt, vb,
                                        (const T*)p->mv, p->dacc,
                                        Pts{0, p->sh_own_cnt, p->sh_own}, st),
                "grad_vals");
        };
        // The dense block's pullback on rank 0 only (the all-reduce below adds it in once).
        GPB2_TRY(Impl<T>::hist_and_dense(p, per_point, comm_rank(c) == 0, vb, xt, s));
        GPB2_TRY(comm_all_reduce(c, p->dacc, p->nb, true, s));
        return Impl<T>::finish_hist(p, dvals, s);
    }

    // Contiguous per-rank ranges of the refined points (scheme A): the first M mod ranks ranks
    // take one point more (_balanced_range, ext/GraphGPMPIExt.jl:25-36).
    static Pts flat_share(P* p, gpb2_comm* c) {
        const int64_t W = comm_size(c), r = comm_rank(c);
        const int64_t base = p->m / W, rem = p->m % W;
        const int64_t a = r < rem ? r * (base + 1) : rem * (base + 1) + (r - rem) * base;
        return Pts{a, r < rem ? base + 1 : base, nullptr};
    }

    static int logdet(P* p, gpb2_comm* c, double* out, cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, false));
        GPB2_TRY(Impl<T>::zero_acc(p, s));
        GPB2_TRY(Dense<T>::factor(p, s));
        if (comm_rank(c) == 0) GPB2_TRY(Dense<T>::logdet(p, p->dacc + p->nb + 2, s));
        GPB2_TRY(Impl<T>::check_launch(ops_of<T>(p)->logdet(point_args<T>(p), nullptr,
                                                            p->dacc + p->nb, flat_share(p, c), s),
                                       "logdet"));
        GPB2_TRY(comm_all_reduce(c, p->dacc + p->nb, 4, true, s));
        double h[4];
        GPB2_TRY(Impl<T>::read_scalars(p, h, s));
        *out = h[2] + h[0];
        return GPB2_OK;
    }

    static int logdet_grad(P* p, gpb2_comm* c, T* dvals, double* ld, cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, false));
        GPB2_TRY(Impl<T>::zero_acc(p, s));
        GPB2_TRY(Impl<T>::check_launch(ops_of<T>(p)->logdet_grad(point_args<T>(p, FcUse::Read), p->dacc,
                                                                 p->dacc + p->nb, nullptr,
                                                                 flat_share(p, c), s),
                                       "logdet grad"));
        GPB2_TRY(Dense<T>::factor(p, s));
        if (comm_rank(c) == 0) {
            GPB2_TRY(Dense<T>::logdet(p, p->dacc + p->nb + 2, s));
            GPB2_TRY(Dense<T>::logdet_grad(p, p->dacc, s));
        }
        GPB2_TRY(comm_all_reduce(c, p->dacc, p->nb + 4, true, s));
        GPB2_TRY(Impl<T>::finish_hist(p, dvals, s));
        if (ld) {
            double h[4];
            GPB2_TRY(Impl<T>::read_scalars(p, h, s));
            *ld = h[2] + h[0];
        }
        return GPB2_OK;
    }

    static int inv_loss_grad(P* p, gpb2_comm* c, const T* data, T* dvals, double* loss,
                             cudaStream_t s) {
        GPB2_TRY(ensure_scratch(p, false));
        int st = GPB2_OK;
        const T* yt = to_tree(p, data, (T*)p->buf_a, s, &st);
        GPB2_TRY(st);
        GPB2_TRY(Impl<T>::zero_acc(p, s));
        GPB2_TRY(Impl<T>::check_launch(
            ops_of<T>(p)->inv_loss_grad(point_args<T>(p, FcUse::Read), yt, p->dacc, p->dacc + p->nb + 1,
                                        nullptr, flat_share(p, c), s),
            "inverse-loss grad"));
        GPB2_TRY(Dense<T>::factor(p, s));
        if (comm_rank(c) == 0)
            GPB2_TRY(Dense<T>::inv_loss_grad(p, yt, p->dacc, p->dacc + p->nb + 1, s));
        GPB2_TRY(comm_all_reduce(c, p->dacc, p->nb + 4, true, s));
        GPB2_TRY(Impl<T>::finish_hist(p, dvals, s));
        if (loss) {
            double h[4];
            GPB2_TRY(Impl<T>::read_scalars(p, h, s));
            *loss = h[1];
        }
        return GPB2_OK;
    }
};

}  // namespace gpb2

using namespace gpb2;

#define GPB2_DISPATCH(p, CALL32, CALL64)                                                       \
    do {                                                                                       \
        clear_error();                                                                         \
        if (!(p)) return set_error(GPB2_ERR_INVALID_ARG, "%s: NULL problem", __func__);         \
        DeviceGuard _dg((p)->device);                                                          \
        if (!_dg.ok) return set_error(GPB2_ERR_NO_DEVICE, "cudaSetDevice(%d) failed", (p)->device); \
        NvtxRange _nvtx(__func__);                                                             \
        cudaStream_t s = (cudaStream_t)stream;                                                 \
        const int _st = (p)->dtype == GPB2_F32 ? (CALL32) : (CALL64);                           \
        if (_st != GPB2_OK) {                                                                  \
            p->dense_pending = false;                                                          \
            p->dense_launched = p->dense_valid;                                                \
            return _st;                                                                        \
        }                                                                                      \
        if (!g_sync.load()) return GPB2_OK;                                                    \
        return finish_call(p, s);                                                              \
    } while (0)

#define F32(x) static_cast<float*>(const_cast<void*>(x))
#define F64(x) static_cast<double*>(const_cast<void*>(x))
#define CF32(x) static_cast<const float*>(x)
#define CF64(x) static_cast<const double*>(x)

// The vals and position gradients are defined for the isotropic table only: the reference's
// anisotropic covariance is forward-only (src/aniso.jl:17).
static int iso_only(const gpb2_problem* p, const char* fn) {
    if (p && p->an_grid)
        return set_error(GPB2_ERR_INVALID_ARG,
                         "%s: the anisotropic covariance supports the forward operations only", fn);
    return GPB2_OK;
}

static int need(const void* ptr, const char* name) {
    return ptr ? GPB2_OK : set_error(GPB2_ERR_INVALID_ARG, "%s is NULL", name);
}

extern "C" {

int gpb2_set_synchronous(int on) {
    g_sync.store(on ? 1 : 0);
    return GPB2_OK;
}

int gpb2_problem_check(gpb2_problem* p, void* stream) {
    clear_error();
    if (!p) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_problem_check: NULL problem");
    DeviceGuard dg(p->device);
    if (!dg.ok) return set_error(GPB2_ERR_NO_DEVICE, "cudaSetDevice(%d) failed", p->device);
    return finish_call(p, (cudaStream_t)stream);
}

int gpb2_set_overlap(int on) {
    g_overlap_flag.store(on != 0);
    return GPB2_OK;
}

int gpb2_set_forward_mode(int mode) {
    if (mode < 0 || mode > 3)
        return set_error(GPB2_ERR_INVALID_ARG,
                         "forward mode must be 0 (persistent), 1 (fused), 2 (batched) or 3 (flow)");
    g_fwd_mode.store(mode);
    return GPB2_OK;
}

int gpb2_refine(gpb2_problem* p, void* values, const void* xi_ref, void* stream) {
    GPB2_TRY(need(values, "values") | need(xi_ref, "xi_ref"));
    GPB2_DISPATCH(p, Impl<float>::refine_tree(p, F32(values), CF32(xi_ref), s),
                  Impl<double>::refine_tree(p, F64(values), CF64(xi_ref), s));
}

// [lo, hi) must lie inside one depth batch (the ranges of a level-sharded sweep).
static int check_range(const gpb2_problem* p, int64_t lo, int64_t hi, const char* what) {
    if (!p) return set_error(GPB2_ERR_INVALID_ARG, "%s: NULL problem", what);
    if (lo < p->n0 || hi > p->n || lo > hi)
        return set_error(GPB2_ERR_INVALID_ARG, "%s: range [%lld, %lld) outside [n0, N) = [%lld, %lld)",
                         what, (long long)lo, (long long)hi, (long long)p->n0, (long long)p->n);
    if (lo == hi) return GPB2_OK;
    const auto it = std::upper_bound(p->offsets.begin(), p->offsets.end(), lo);
    if (it == p->offsets.end() || hi > *it)
        return set_error(GPB2_ERR_INVALID_ARG, "%s: range [%lld, %lld) spans depth batches", what,
                         (long long)lo, (long long)hi);
    return GPB2_OK;
}

#define GPB2_ASYNC(p, CALL32, CALL64)                                                          \
    do {                                                                                       \
        DeviceGuard _dg((p)->device);                                                          \
        if (!_dg.ok) return set_error(GPB2_ERR_NO_DEVICE, "cudaSetDevice(%d) failed", (p)->device); \
        NvtxRange _nvtx(__func__);                                                             \
        cudaStream_t s = (cudaStream_t)stream;                                                 \
        return (p)->dtype == GPB2_F32 ? (CALL32) : (CALL64);                                    \
    } while (0)

int gpb2_refine_range(gpb2_problem* p, void* values, const void* xi_ref, int64_t lo, int64_t hi,
                      void* stream) {
    clear_error();
    GPB2_TRY(check_range(p, lo, hi, "gpb2_refine_range"));
    GPB2_TRY(need(values, "values") | need(xi_ref, "xi_ref"));
    if (lo == hi) return GPB2_OK;
    GPB2_ASYNC(p, Impl<float>::refine_range(p, F32(values), CF32(xi_ref), lo, hi, s),
               Impl<double>::refine_range(p, F64(values), CF64(xi_ref), lo, hi, s));
}

int gpb2_refine_reverse_range(gpb2_problem* p, void* xg, void* vb, int64_t lo, int64_t hi,
                              void* stream) {
    clear_error();
    GPB2_TRY(check_range(p, lo, hi, "gpb2_refine_reverse_range"));
    GPB2_TRY(need(vb, "vb"));
    if (lo == hi) return GPB2_OK;
    GPB2_ASYNC(p, Impl<float>::reverse_range(p, F32(xg), F32(vb), lo, hi, s),
               Impl<double>::reverse_range(p, F64(xg), F64(vb), lo, hi, s));
}

int gpb2_problem_prefactor(gpb2_problem* p, void* stream) {
    clear_error();
    if (!p) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_problem_prefactor: NULL problem");
    GPB2_ASYNC(p, Impl<float>::prefactor(p, s), Impl<double>::prefactor(p, s));
}

int gpb2_dense_apply(gpb2_problem* p, int trans, const void* x, void* y, void* stream) {
    GPB2_TRY(need(x, "x") | need(y, "y"));
    GPB2_DISPATCH(p, Impl<float>::dense_apply(p, trans, CF32(x), F32(y), s),
                  Impl<double>::dense_apply(p, trans, CF64(x), F64(y), s));
}

int gpb2_refine_inv(gpb2_problem* p, const void* values, void* xi_ref, void* stream) {
    GPB2_TRY(need(values, "values") | need(xi_ref, "xi_ref"));
    GPB2_DISPATCH(p, Impl<float>::refine_inv_tree(p, CF32(values), F32(xi_ref), s),
                  Impl<double>::refine_inv_tree(p, CF64(values), F64(xi_ref), s));
}

int gpb2_refine_logdet_terms(gpb2_problem* p, void* terms, void* stream) {
    GPB2_TRY(need(terms, "terms"));
    GPB2_DISPATCH(p, Impl<float>::refine_logdet_tree(p, F32(terms), nullptr, s),
                  Impl<double>::refine_logdet_tree(p, F64(terms), nullptr, s));
}

int gpb2_refine_logdet(gpb2_problem* p, double* out, void* stream) {
    GPB2_TRY(need(out, "logdet_host"));
    GPB2_DISPATCH(p, Impl<float>::refine_logdet(p, nullptr, out, s),
                  Impl<double>::refine_logdet(p, nullptr, out, s));
}

int gpb2_refine_logdet_grad_vals(gpb2_problem* p, void* dvals, double* ld, void* stream) {
    GPB2_TRY(iso_only(p, __func__));
    GPB2_TRY(need(dvals, "dvals"));
    GPB2_DISPATCH(p, Impl<float>::refine_logdet_grad_vals(p, F32(dvals), ld, s),
                  Impl<double>::refine_logdet_grad_vals(p, F64(dvals), ld, s));
}

int gpb2_refine_inv_loss_grad_vals(gpb2_problem* p, const void* values, void* dvals,
                                   double* loss, void* stream) {
    GPB2_TRY(iso_only(p, __func__));
    GPB2_TRY(need(values, "values") | need(dvals, "dvals"));
    GPB2_DISPATCH(p, Impl<float>::refine_inv_loss_tree(p, CF32(values), F32(dvals), loss, s),
                  Impl<double>::refine_inv_loss_tree(p, CF64(values), F64(dvals), loss, s));
}

int gpb2_generate(gpb2_problem* p, const void* xi, void* out, void* stream) {
    GPB2_TRY(need(xi, "xi") | need(out, "out"));
    GPB2_DISPATCH(p, Impl<float>::generate(p, CF32(xi), F32(out), s),
                  Impl<double>::generate(p, CF64(xi), F64(out), s));
}

int gpb2_generate_inv(gpb2_problem* p, const void* values, void* xi, void* stream) {
    GPB2_TRY(need(values, "values") | need(xi, "xi"));
    GPB2_DISPATCH(p, Impl<float>::generate_inv(p, CF32(values), F32(xi), s),
                  Impl<double>::generate_inv(p, CF64(values), F64(xi), s));
}

int gpb2_generate_logdet(gpb2_problem* p, double* out, void* stream) {
    GPB2_TRY(need(out, "logdet_host"));
    GPB2_DISPATCH(p, Impl<float>::generate_logdet(p, out, s),
                  Impl<double>::generate_logdet(p, out, s));
}

int gpb2_generate_grad_xi(gpb2_problem* p, const void* vbar, void* xbar, void* stream) {
    GPB2_TRY(need(vbar, "vbar") | need(xbar, "xbar"));
    GPB2_DISPATCH(p, Impl<float>::generate_grad_xi(p, CF32(vbar), F32(xbar), s),
                  Impl<double>::generate_grad_xi(p, CF64(vbar), F64(xbar), s));
}

int gpb2_generate_grad_vals(gpb2_problem* p, const void* xi, const void* vbar, void* dvals,
                            void* stream) {
    GPB2_TRY(iso_only(p, __func__));
    GPB2_TRY(need(xi, "xi") | need(vbar, "vbar") | need(dvals, "dvals"));
    GPB2_DISPATCH(p, Impl<float>::generate_grad_vals(p, CF32(xi), CF32(vbar), F32(dvals), s),
                  Impl<double>::generate_grad_vals(p, CF64(xi), CF64(vbar), F64(dvals), s));
}

int gpb2_generate_logdet_grad_vals(gpb2_problem* p, void* dvals, double* ld, void* stream) {
    GPB2_TRY(iso_only(p, __func__));
    GPB2_TRY(need(dvals, "dvals"));
    GPB2_DISPATCH(p, Impl<float>::generate_logdet_grad_vals(p, F32(dvals), ld, s),
                  Impl<double>::generate_logdet_grad_vals(p, F64(dvals), ld, s));
}

int gpb2_generate_inv_loss_grad_vals(gpb2_problem* p, const void* data, void* dvals,
                                     double* loss, void* stream) {
    GPB2_TRY(iso_only(p, __func__));
    GPB2_TRY(need(data, "data") | need(dvals, "dvals"));
    GPB2_DISPATCH(p, Impl<float>::generate_inv_loss_grad_vals(p, CF32(data), F32(dvals), loss, s),
                  Impl<double>::generate_inv_loss_grad_vals(p, CF64(data), F64(dvals), loss, s));
}

int gpb2_refine_logdet_grad_points(gpb2_problem* p, void* d_points, void* stream) {
    GPB2_TRY(iso_only(p, __func__));
    GPB2_TRY(need(d_points, "d_points"));
    GPB2_DISPATCH(p, Impl<float>::refine_logdet_grad_points(p, F32(d_points), s),
                  Impl<double>::refine_logdet_grad_points(p, F64(d_points), s));
}

int gpb2_generate_logdet_grad_points(gpb2_problem* p, void* d_points, void* stream) {
    GPB2_TRY(iso_only(p, __func__));
    GPB2_TRY(need(d_points, "d_points"));
    GPB2_DISPATCH(p, Impl<float>::generate_logdet_grad_points(p, F32(d_points), s),
                  Impl<double>::generate_logdet_grad_points(p, F64(d_points), s));
}

int gpb2_refine_inv_loss_grad_points(gpb2_problem* p, const void* values, void* d_points,
                                     void* stream) {
    GPB2_TRY(iso_only(p, __func__));
    GPB2_TRY(need(values, "values") | need(d_points, "d_points"));
    GPB2_DISPATCH(p, Impl<float>::refine_inv_loss_grad_points(p, CF32(values), F32(d_points), s),
                  Impl<double>::refine_inv_loss_grad_points(p, CF64(values), F64(d_points), s));
}

int gpb2_generate_inv_loss_grad_points(gpb2_problem* p, const void* data, void* d_points,
                                       void* stream) {
    GPB2_TRY(iso_only(p, __func__));
    GPB2_TRY(need(data, "data") | need(d_points, "d_points"));
    GPB2_DISPATCH(p, Impl<float>::generate_inv_loss_grad_points(p, CF32(data), F32(d_points), s),
                  Impl<double>::generate_inv_loss_grad_points(p, CF64(data), F64(d_points), s));
}

// ------------------------------------------------------------------------------ level-sharded

#define GPB2_SHARDED(p, c, CALL32, CALL64)                                                     \
    do {                                                                                       \
        if (!(c)) return set_error(GPB2_ERR_INVALID_ARG, "%s: NULL communicator", __func__);   \
        GPB2_DISPATCH(p, CALL32, CALL64);                                                      \
    } while (0)

int gpb2_generate_sharded(gpb2_problem* p, gpb2_comm* c, const void* xi, void* out,
                          void* stream) {
    GPB2_TRY(need(xi, "xi") | need(out, "out"));
    GPB2_SHARDED(p, c, Shard<float>::generate(p, c, CF32(xi), F32(out), s),
                 Shard<double>::generate(p, c, CF64(xi), F64(out), s));
}

int gpb2_generate_grad_xi_sharded(gpb2_problem* p, gpb2_comm* c, const void* vbar, void* xbar,
                                  void* stream) {
    GPB2_TRY(need(vbar, "vbar") | need(xbar, "xbar"));
    GPB2_SHARDED(p, c, Shard<float>::grad_xi(p, c, CF32(vbar), F32(xbar), s),
                 Shard<double>::grad_xi(p, c, CF64(vbar), F64(xbar), s));
}

int gpb2_generate_grad_vals_sharded(gpb2_problem* p, gpb2_comm* c, const void* xi,
                                    const void* vbar, void* dvals, void* stream) {
    GPB2_TRY(iso_only(p, __func__));
    GPB2_TRY(need(xi, "xi") | need(vbar, "vbar") | need(dvals, "dvals"));
    GPB2_SHARDED(p, c, Shard<float>::grad_vals(p, c, CF32(xi), CF32(vbar), F32(dvals), s),
                 Shard<double>::grad_vals(p, c, CF64(xi), CF64(vbar), F64(dvals), s));
}

int gpb2_generate_logdet_sharded(gpb2_problem* p, gpb2_comm* c, double* out, void* stream) {
    GPB2_TRY(need(out, "logdet_host"));
    GPB2_SHARDED(p, c, Shard<float>::logdet(p, c, out, s), Shard<double>::logdet(p, c, out, s));
}

int gpb2_generate_logdet_grad_vals_sharded(gpb2_problem* p, gpb2_comm* c, void* dvals,
                                           double* ld, void* stream) {
    GPB2_TRY(iso_only(p, __func__));
    GPB2_TRY(need(dvals, "dvals"));
    GPB2_SHARDED(p, c, Shard<float>::logdet_grad(p, c, F32(dvals), ld, s),
                 Shard<double>::logdet_grad(p, c, F64(dvals), ld, s));
}

int gpb2_generate_inv_loss_grad_vals_sharded(gpb2_problem* p, gpb2_comm* c, const void* data,
                                             void* dvals, double* loss, void* stream) {
    GPB2_TRY(iso_only(p, __func__));
    GPB2_TRY(need(data, "data") | need(dvals, "dvals"));
    GPB2_SHARDED(p, c, Shard<float>::inv_loss_grad(p, c, CF32(data), F32(dvals), loss, s),
                 Shard<double>::inv_loss_grad(p, c, CF64(data), F64(dvals), loss, s));
}

int gpb2_shard_plan(const int64_t* offsets, int64_t n_offsets, int nranks, int rank,
                    int64_t min_shard, int64_t* fwd_lo, int64_t* fwd_hi, int64_t* own_lo,
                    int64_t* own_hi, int* sharded, int64_t* slack) {
    clear_error();
    if (!offsets || n_offsets < 1 || nranks < 1 || rank < 0 || rank >= nranks || min_shard < 1)
        return set_error(GPB2_ERR_INVALID_ARG, "gpb2_shard_plan: invalid arguments");
    const ShardPlan pl = ShardPlan::make(std::vector<int64_t>(offsets, offsets + n_offsets),
                                         nranks, rank, min_shard);
    for (size_t i = 0; i < pl.b.size(); i++) {
        int64_t a, e;
        pl.fwd_range(pl.b[i], a, e);
        if (fwd_lo) fwd_lo[i] = a;
        if (fwd_hi) fwd_hi[i] = e;
        pl.own_range(pl.b[i], a, e);
        if (own_lo) own_lo[i] = a;
        if (own_hi) own_hi[i] = e;
        if (sharded) sharded[i] = pl.b[i].sharded ? 1 : 0;
    }
    if (slack) *slack = pl.slack;
    return GPB2_OK;
}

}  // extern "C"
