/*
 * graphgp_b200.h -- C ABI of libgraphgp_b200.so, the B200 (sm_100a) implementation of
 * GraphGP.jl's per-point Vecchia refine path and its analytic adjoints.
 *
 * Drop-in boundary.  The reference reaches CUDA through KernelAbstractions launches selected by
 * `_is_cpu(backend)` (src/cpu_native.jl:13) and through the opt-in ccall bridge
 * ext/GraphGPCUDAExt.jl:39-64 over csrc/graphgp_capi.cu:70-119.  Every entry point below names
 * the reference function (path:line inside the GraphGP.jl tree) whose device work it replaces.
 *
 * Conventions
 *  - Every function returns a gpb2_status; nothing aborts or exits.  The message of the last
 *    failure on the calling thread is available from gpb2_last_error().
 *  - Arrays use the reference's memory layout: coords is Julia's (D, N) column-major uint32
 *    (a point's D coordinates contiguous); neighbors is Julia's (K, M) column-major (a refined
 *    point's K neighbour indices contiguous), int64 or int32, 1-based (Julia) or 0-based.
 *    offsets is the reference's host Vector{Int}: offsets[0] == n0, offsets[last] == N, depth
 *    batch b covers tree positions [offsets[b-1], offsets[b]).  indices (host, optional) is
 *    the tree->original permutation: indices[tree_pos] = original_pos.
 *  - Floating-point buffers are float (dtype GPB2_F32) or double (GPB2_F64), matching the
 *    problem's dtype.  Buffers named *_dev are device pointers on the problem's device; the
 *    *_host outputs are host scalars (those calls synchronise the stream).
 *  - Calls are ordered on the caller's `stream` (a cudaStream_t; NULL = legacy default
 *    stream).  One problem handle must not be used by two threads at once.
 *  - In/out device buffers are caller-owned; the library owns only the problem handle's
 *    internal copies and scratch, released by gpb2_problem_destroy.
 */
#ifndef GRAPHGP_B200_H
#define GRAPHGP_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GPB2_VERSION 1

typedef enum gpb2_status {
    GPB2_OK = 0,
    GPB2_ERR_INVALID_ARG = 1,
    GPB2_ERR_UNSUPPORTED_K = 2,     /* same code as csrc/graphgp_capi.cu:53-68 ("unsupported k") */
    GPB2_ERR_UNSUPPORTED_D = 3,     /* same code as csrc/graphgp_capi.cu:53-68 ("unsupported D") */
    GPB2_ERR_OOM = 4,
    GPB2_ERR_CUDA = 5,
    GPB2_ERR_NCCL = 6,
    GPB2_ERR_TIMEOUT = 7,
    GPB2_ERR_GRAPH = 8,             /* check_graph invariant violated (src/graph_build.jl:20-57) */
    GPB2_ERR_NOT_PD = 9,            /* dense block not PD at 1e-2 jitter (src/dense.jl:65-66) */
    GPB2_ERR_UNSUPPORTED_TABLE = 10,/* bins not strictly increasing / too many bins */
    GPB2_ERR_NO_DEVICE = 11
} gpb2_status;

typedef enum gpb2_dtype { GPB2_F32 = 0, GPB2_F64 = 1 } gpb2_dtype;

typedef struct gpb2_problem gpb2_problem;
typedef struct gpb2_graph gpb2_graph;

/* Library version (GPB2_VERSION) and the last error message on this thread ("" if none). */
int gpb2_version(void);
const char* gpb2_last_error(void);

/* ------------------------------------------------------------------------------------------
 * Problem handle.  Replaces the per-call `_prep` conversion of ext/GraphGPCUDAExt.jl:27-35
 * (float positions, 0-based Int64 neighbours) with a one-time upload: the library keeps a
 * 0-based int32 copy of the neighbours, a padded copy of the coords, the level table and the
 * interpolation table, and validates the graph invariants of check_graph
 * (src/graph_build.jl:20-57) on the device.  Mirrors the GraphGPProblem constructor
 * (src/types.jl:22-60) and `to_backend` (src/types.jl:97-106).
 * ---------------------------------------------------------------------------------------- */
int gpb2_problem_create(gpb2_problem** out, int dtype, int device,
                        const uint32_t* coords_dev, int64_t d, int64_t n,
                        const void* neighbors_dev, int neighbor_bytes, int neighbor_base,
                        int64_t k, const int64_t* offsets_host, int64_t n_offsets, int64_t n0,
                        double scale, const void* bins_dev, const void* vals_dev, int64_t nbins,
                        const int64_t* indices_host, int indices_base, void* stream);

/* gpb2_problem_create with the permutation given on the device: indices_dev holds N int32
 * (indices_bytes = 4) or int64 (8) values, base 0 or 1, checked on the device to be a
 * permutation.  For graphs built on the device (gpb2_build_graph_device), whose arrays never
 * pass through host memory; the reference's problems keep `indices` on the host
 * (src/types.jl:22-60), which gpb2_problem_create covers. */
int gpb2_problem_create_dev(gpb2_problem** out, int dtype, int device,
                            const uint32_t* coords_dev, int64_t d, int64_t n,
                            const void* neighbors_dev, int neighbor_bytes, int neighbor_base,
                            int64_t k, const int64_t* offsets_host, int64_t n_offsets, int64_t n0,
                            double scale, const void* bins_dev, const void* vals_dev,
                            int64_t nbins, const void* indices_dev, int indices_bytes,
                            int indices_base, void* stream);

/* The library's internal point order.  Inside the handle every depth batch is sorted by the
 * Morton code of its points (the batches, the dense first layer's positions [0, n0) and every
 * point's neighbour list are unchanged, so every result is the same; the gathers of a warp's
 * points become coalesced).  The operations in original order and the tree-order refine entry
 * points translate at the boundary; the range entry points (gpb2_refine_range,
 * gpb2_refine_reverse_range) work in library order.  This call copies the two maps, N int32 each,
 * into device buffers: lib_tree_dev[q] = tree position of library position q, lib_orig_dev[q] =
 * original index (either may be NULL).  No reference counterpart. */
int gpb2_problem_order(const gpb2_problem* prob, int32_t* lib_tree_dev, int32_t* lib_orig_dev,
                       void* stream);

/* Replace the covariance values (`_set_vals`, src/chainrules.jl:18-21). */
int gpb2_problem_set_vals(gpb2_problem* prob, const void* vals_dev, void* stream);

/* Queue both factorisations of the current table (the dense first-layer Cholesky with its
 * jitter ladder, and every refined point's mean_vec / std) on `stream` and return without
 * waiting.  No separate counterpart in the reference: its generate factors the dense block
 * at its start (src/api.jl:113-141); every operation here also factors a table that is not
 * factorised yet, so this call only lets a caller start that work early, e.g. while the next
 * inputs are still being copied to the device.  A numerical failure (no ladder step
 * factorises the dense block) is reported by the next operation that uses the factor. */
int gpb2_problem_prefactor(gpb2_problem* prob, void* stream);

/* Anisotropic covariance K(d_spatial, d_z) (src/aniso.jl; the problem constructor of
 * src/types.jl:62-68 with an AnisoCov): a 2-D table grid[i + j*ns] = K(spatial_bins[i],
 * z_bins[j]) ((ns, nz) column-major, as the reference's Matrix; the caller applies the
 * jitter to grid[0], as build_anisotropic_covariance does), bilinear interpolation at the
 * fractional bin indices (aniso_lookup, src/aniso.jl:67-85) of d_spatial = |x_a - x_b| over
 * the first D - 1 coordinates and d_z = |z_a - z_b| / alpha over the last (times scale).  From
 * this call on, the forward operations (generate, generate_inv, generate_logdet, refine*, and
 * generate_grad_xi, their adjoint) assemble every covariance -- the dense block's included --
 * from it; the vals and position gradients return GPB2_ERR_INVALID_ARG (the reference's
 * anisotropic path is forward-only).  All arrays are the problem's T, on the device; they are
 * copied. */
int gpb2_problem_set_aniso(gpb2_problem* prob, const void* spatial_bins_dev, int64_t ns,
                           const void* z_bins_dev, int64_t nz, const void* grid_dev, double alpha,
                           void* stream);

/* Per-point factor cache: the packed (K+1)x(K+1) Cholesky factor of every refined point and
 * the interpolation segment and fraction of each of its K(K+1)/2 pair radii, kept in device
 * memory (M * (NT*sizeof(T) + NR*(sizeof(T)+2)) bytes, NT = (K+1)(K+2)/2, NR = NT - K - 1;
 * 396 bytes per point at K = 8 in single precision) so that the vals-gradient kernels
 * (generate_grad_vals, refine_logdet_grad_vals, refine_inv_loss_grad_vals and their generate_
 * forms) read each point's factor instead of gathering its neighbours' coordinates,
 * interpolating the covariance and factorising again.  The per-point factor pass of a table
 * fills it; the cached entries are the bits the recomputation gives, so results do not depend
 * on the mode.  mode 0: off (frees it); 1: always; 2 (default; GPB2_FACTOR_CACHE in the
 * environment sets the default of new handles): allocated by the first generate_grad_vals
 * when the device keeps max(10 %, 8 GB) of its memory free beyond it, else not used.  No
 * reference counterpart (the reference recomputes every factor in every kernel). */
int gpb2_problem_set_factor_cache(gpb2_problem* prob, int mode);
/* The mode, what the cache holds (valid: 0 nothing current, 1 the current table's factors of
 * every point, 2 those of this rank's level-sharded ranges), and its size in bytes. */
int gpb2_problem_factor_cache(const gpb2_problem* prob, int* mode, int* valid, int64_t* bytes);

/* Reverse sweep of generate_grad_xi / generate_grad_vals.  mode 0: every refined point pushes
 * its K terms mean_vec[j] * vb[p] into its neighbours' cotangents with atomic additions (the
 * reference's form; sums in no fixed order).  1: every point pulls its incoming terms through
 * the transposed graph, in the serial sweep's order (descending tree order of the child, slot
 * order) -- sums bit for bit those of the serial reference sweep and reproducible -- at the
 * cost of (4 + sizeof(T)) bytes per edge plus 4 per point of device memory (the graph is built
 * once, its weights once per table).  2 (default; GPB2_REVERSE_MODE in the environment sets the
 * default of new handles): 1 from 2e7 refined points up (GPB2_PULL_MIN overrides; below it the
 * push is faster) when the graph fits with a margin of free memory, else 0.  The per-batch
 * sweep modes and the level-sharded operations always push.  No reference counterpart. */
int gpb2_problem_set_reverse_mode(gpb2_problem* prob, int mode);
/* The mode, whether the transposed graph is built, and its size in bytes. */
int gpb2_problem_reverse_mode(const gpb2_problem* prob, int* mode, int* built, int64_t* bytes);

/* Sizes: N, M = N - n0, K, D, number of depth batches (n_offsets - 1). */
int gpb2_problem_info(const gpb2_problem* prob, int64_t* n, int64_t* m, int64_t* k, int64_t* d,
                      int64_t* n_batches);

int gpb2_problem_destroy(gpb2_problem* prob);

/* The relative jitter eps of the dense block's last factorisation: 0 when K itself factorised,
 * else the first of 1e-9, 1e-8, ..., 1e-2 for which K + eps*mean(diag(K)) did
 * (_dense_chol_L, src/dense.jl:46-67); -1 before any dense operation. */
int gpb2_problem_dense_jitter(const gpb2_problem* prob, double* eps);

/* Copy the dense block's last Cholesky factor (n0 x n0, column-major; lower triangle valid,
 * upper triangle unspecified) into factor_dev.  No reference counterpart: the factor is internal
 * to src/dense.jl; exposed for inspection and parity tests. */
int gpb2_problem_dense_factor(const gpb2_problem* prob, void* factor_dev, void* stream);

/* Launch profiler, process-wide (no reference counterpart; the reference times with
 * CUDA.@elapsed around whole calls, bench/compare/run_gradmem.jl:19-36).  Every kernel the
 * library launches is counted (gpb2_launch_count); with profiling enabled each launch is also
 * bracketed by a CUDA event pair on its own stream.  gpb2_profile_report synchronises those
 * events and writes one line per kernel kind, "name launches total_ms\n", into buf. */
int gpb2_profile_enable(int on);
int gpb2_profile_reset(void);
int gpb2_profile_report(char* buf, int64_t cap);
int64_t gpb2_launch_count(void);

/* Depth-sweep strategy, process-wide.  The conditional-mean weights and std of all refined
 * points come from one flat kernel; then 0 = one cooperative (persistent) kernel per sweep with a
 * bounded grid barrier between depth batches (default); 2 = one light kernel launch per batch.
 * 1 = the reference's fused per-batch forward kernel (refine_apply_fused_kernel!,
 * src/kernels.jl:101-119), which recomputes the factor inside each batch.  3 = dataflow: one
 * cooperative kernel with no barrier, each point waiting (bounded) for its own neighbours' values
 * (the reverse sweep then runs as in mode 0).  All four give bit-identical forward values.  A
 * barrier or wait that times out makes the call return GPB2_ERR_TIMEOUT. */
int gpb2_set_forward_mode(int mode);

/* Whether the dense first layer's work (the jitter ladder, the dense pullback) runs on the
 * handle's second stream beside the per-point kernels (1, default; GPB2_OVERLAP=0 at load time
 * sets 0) or in sequence on the call's stream (0: per-launch profiles then time each kernel
 * alone).  Process-wide; results are the same either way.  No reference counterpart. */
int gpb2_set_overlap(int on);

/* Call mode, process-wide (default 1; GPB2_SYNC=0 in the environment at load time sets 0).
 * 1: every operation waits for its work and returns its status, including the numerical ones
 *    (a dense block that no jitter step factorises, a grid barrier that timed out).
 * 0: operations return once their work is queued on the stream, as CUDA launches do (the
 *    reference's CUDA.jl path is asynchronous the same way: ext/GraphGPCUDAExt.jl:39-64);
 *    launch errors are still returned, the numerical status is reported by the next
 *    gpb2_problem_check on the handle.  Operations that return host values (logdets, losses)
 *    still wait for them.  No counterpart in the reference's C API. */
int gpb2_set_synchronous(int on);

/* Wait for the handle's queued work on `stream` and return its status (see
 * gpb2_set_synchronous).  No counterpart in the reference. */
int gpb2_problem_check(gpb2_problem* prob, void* stream);

/* ------------------------------------------------------------------------------------------
 * Refine layer, tree order.
 * ---------------------------------------------------------------------------------------- */

/* refine!: values_dev[0:n0] preset, values_dev[n0:N] written; xi_ref_dev has M entries.
 * Replaces the per-batch refine_apply_fused_kernel! launches of src/api.jl:113-141. */
int gpb2_refine(gpb2_problem* prob, void* values_dev, const void* xi_ref_dev, void* stream);

/* Ranges of one depth batch, the building blocks of a level-sharded sweep over several GPUs
 * (each rank runs its slice of a batch, the caller exchanges the batch between ranks; the
 * exchange replaces the reference's MPI/serial level loop, src/distributed.jl:293-322 and
 * src/api.jl:113-141).  [lo, hi) are tree-order point indices inside one batch (n0 <= lo).
 * Positions are the library's order (gpb2_problem_order): the batches' bounds are the tree
 * order's, the points inside a batch are permuted.
 * Asynchronous on `stream` (no synchronisation; launch errors are returned).
 *   refine_range:          values[p] = std_p*xi_ref[p-n0] + sum_j mv_pj*values[nbr_pj]
 *                          (refine_apply_fused_kernel!, src/kernels.jl:101-119)
 *   refine_reverse_range:  xg[p] = std_p*vb[p] (xg may be NULL); vb[nbr_pj] += mv_pj*vb[p]
 *                          (refine_reverse_apply_fused_kernel!, src/kernels_adjoint.jl:453-474) */
int gpb2_refine_range(gpb2_problem* prob, void* values_dev, const void* xi_ref_dev, int64_t lo,
                      int64_t hi, void* stream);
int gpb2_refine_reverse_range(gpb2_problem* prob, void* xg_dev, void* vb_dev, int64_t lo,
                              int64_t hi, void* stream);

/* Dense first layer: y[0:n0] = L x[0:n0] (trans = 0, generate_dense, src/dense.jl:112-119) or
 * L^T x[0:n0] (trans = 1, the dense adjoint of generate_grad_xi, src/grad.jl:448-453); the
 * block is factorised (with the jitter ladder) if the table changed.  Synchronous. */
int gpb2_dense_apply(gpb2_problem* prob, int trans, const void* x_dev, void* y_dev, void* stream);

/* refine_inv!: xi_ref_dev[m] = (values[n0+m] - mean) / std.  Replaces src/api.jl:66-97
 * (refine_inv_kernel!, src/kernels.jl:37-56) and gpcuda_refine_inv_f32 (csrc/graphgp_capi.cu:90-99). */
int gpb2_refine_inv(gpb2_problem* prob, const void* values_dev, void* xi_ref_dev, void* stream);

/* refine_logdet_terms: terms_dev[m] = log(std_m).  Replaces src/api.jl:30-57. */
int gpb2_refine_logdet_terms(gpb2_problem* prob, void* terms_dev, void* stream);

/* refine_logdet: sum of the terms, accumulated in double.  Replaces src/api.jl:24-28 and
 * gpcuda_refine_logdet_f32 (csrc/graphgp_capi.cu:76-88).  Synchronous. */
int gpb2_refine_logdet(gpb2_problem* prob, double* logdet_host, void* stream);

/* refine_logdet_grad_vals: d(refine_logdet)/d(vals) into dvals_dev (nbins, problem dtype);
 * logdet_host (optional) receives the fused logdet sum (refine_logdet_and_grad_hist_kernel!).
 * Replaces src/grad.jl:96-119 and the fused src/grad.jl:680-715 device branch. */
int gpb2_refine_logdet_grad_vals(gpb2_problem* prob, void* dvals_dev, double* logdet_host,
                                 void* stream);

/* refine_logdet_grad_vals_noalloc: the same result as gpb2_refine_logdet_grad_vals, computed
 * without allocating any device memory during the call.  It has no counterpart in the
 * reference; it serves callers whose framework allocator (CUDA.jl's pool, PyTorch's caching
 * allocator) holds the free HBM, or who cannot afford the device synchronisation of a cudaMalloc,
 * at the point of the call.  The histogram lives in a fixed __device__ array of 4096 + 8 doubles
 * per device, cleared by the call on `stream`.  Limits: nbins <= 4096 (else
 * GPB2_ERR_INVALID_ARG); calls that overlap in time on one device (other threads, streams or
 * problems) race on the shared array.  The first call on each device resolves the array's address
 * (cudaGetSymbolAddress): make it before any stream capture.  The call always waits for its own
 * work before returning
 * (whatever gpb2_set_synchronous says), and it does not read the status words that earlier
 * asynchronous calls on the handle left behind: call gpb2_problem_check for those. */
int gpb2_refine_logdet_grad_vals_noalloc(gpb2_problem* prob, void* dvals_dev,
                                         double* logdet_host, void* stream);

/* refine_inv_loss_grad_vals: loss = 0.5*||refine_inv(values)||^2 and its vals-gradient.
 * Replaces src/grad.jl:643-678 (refine_inv_loss_grad_hist_kernel!, src/kernels_adjoint.jl:155-221). */
int gpb2_refine_inv_loss_grad_vals(gpb2_problem* prob, const void* values_dev, void* dvals_dev,
                                   double* loss_host, void* stream);

/* ------------------------------------------------------------------------------------------
 * Orchestrated operations, ORIGINAL point order in and out (src/orchestrate.jl): the
 * tree<->original permutation, the dense n0 block (on the device) and the refine layer.
 * ---------------------------------------------------------------------------------------- */

/* generate(prob, xi) -> out (src/orchestrate.jl:19-42). */
int gpb2_generate(gpb2_problem* prob, const void* xi_dev, void* out_dev, void* stream);

/* generate_inv(prob, values) -> xi (src/orchestrate.jl:53-81). */
int gpb2_generate_inv(gpb2_problem* prob, const void* values_dev, void* xi_dev, void* stream);

/* generate_logdet(prob) (src/orchestrate.jl:89-97).  Synchronous. */
int gpb2_generate_logdet(gpb2_problem* prob, double* logdet_host, void* stream);

/* generate_grad_xi(prob, vbar) -> xbar (src/grad.jl:392-506). */
int gpb2_generate_grad_xi(gpb2_problem* prob, const void* vbar_dev, void* xbar_dev, void* stream);

/* generate_grad_vals(prob, xi, vbar) -> dvals (nbins) (src/grad_generate_vals.jl:111-282). */
int gpb2_generate_grad_vals(gpb2_problem* prob, const void* xi_dev, const void* vbar_dev,
                            void* dvals_dev, void* stream);

/* generate_logdet_grad_vals (src/grad.jl:149-154) and the fused
 * generate_logdet_and_grad_vals (src/grad.jl:680-715; logdet_host may be NULL). */
int gpb2_generate_logdet_grad_vals(gpb2_problem* prob, void* dvals_dev, double* logdet_host,
                                   void* stream);

/* generate_inv_loss_grad_vals (src/grad.jl:514-526): loss and vals-gradient of
 * 0.5*||generate_inv(data)||^2; data in original order. */
int gpb2_generate_inv_loss_grad_vals(gpb2_problem* prob, const void* data_dev, void* dvals_dev,
                                     double* loss_host, void* stream);

/* Point-position gradients: d/dx of the log-determinant or of the inverse loss
 * 0.5*||xi||^2 for the continuous positions x = scale * coords (the lattice enters only
 * through the radii: the reference's straight-through convention).  d_points_dev is (D, N)
 * column-major = (N, D) row-major T in TREE order, overwritten.  Every off-diagonal pair of a
 * point's (K+1)x(K+1) block (and of the dense block, generate_ forms) adds
 * Abar * k'(r) / r * scale * (x_a - x_b) to point a and subtracts it from point b, k' the
 * table's segment slope (0 at and beyond both ends; coincident points add nothing); the
 * additions are atomic.
 * refine_logdet_grad_points (src/grad.jl:168-233, kernel src/kernels_adjoint.jl:254-270). */
int gpb2_refine_logdet_grad_points(gpb2_problem* prob, void* d_points_dev, void* stream);
/* generate_logdet_grad_points (src/grad.jl:234-247): plus the dense block's
 * (_dense_logdet_grad_points, src/dense.jl:188-225: cotangent K^-1[a][b]). */
int gpb2_generate_logdet_grad_points(gpb2_problem* prob, void* d_points_dev, void* stream);
/* refine_inv_loss_grad_points (src/grad.jl:259-358, kernel src/kernels_adjoint.jl:273-324);
 * values_dev: the field in tree order. */
int gpb2_refine_inv_loss_grad_points(gpb2_problem* prob, const void* values_dev,
                                     void* d_points_dev, void* stream);
/* generate_inv_loss_grad_points (src/grad.jl:360-377): plus the dense block's
 * (_dense_inv_loss_grad_points, src/dense.jl:271-297: cotangent -alpha_a * alpha_b,
 * alpha = K^-1 y); data_dev in the original order. */
int gpb2_generate_inv_loss_grad_points(gpb2_problem* prob, const void* data_dev,
                                       void* d_points_dev, void* stream);

/* ------------------------------------------------------------------------------------------
 * Level-sharded operations over several GPUs, one process (or thread) per GPU.  Replaces the
 * reference's distributed per-level loop (src/distributed.jl:281-331: a host loop over depth
 * levels with an MPI sum-Allreduce of each level's new values, through the shims of
 * ext/GraphGPMPIExt.jl:99-115) and its fitting reductions (scheme A, src/distributed.jl:129-247,
 * ext/GraphGPMPIExt.jl:46-115).  The communicator is NCCL over NVLink, created by the library
 * from a unique id that rank 0 makes and the caller distributes (MPI, a file, a store):
 *   gpb2_comm_unique_id(id)                 on one rank; id has GPB2_COMM_ID_BYTES bytes
 *   gpb2_comm_create(&c, nranks, rank, id, device, timeout_s)   on every rank (collective; a
 *                                           rank missing after timeout_s ends it with
 *                                           GPB2_ERR_TIMEOUT; timeout_s <= 0 waits without limit)
 * Every rank holds the same problem and calls the same operations in the same order, with
 * full-length inputs in original order; outputs are full length on every rank.  A depth batch of
 * at least min_shard points (gpb2_comm_set_min_shard, default 65536) is split into one chunk per
 * rank and completed by an in-place all-gather; smaller batches are computed by every rank.  The
 * reverse sweeps sum the batch's cotangents over the ranks (reduce-scatter) before scattering;
 * the vals-gradients end with one all-reduce of the double histogram.  The fitting reductions
 * split the refined points into contiguous per-rank ranges and end with one all-reduce of
 * nbins + 4 doubles.  Results equal the single-GPU operations' (the forward bit for bit; sums in
 * another order within tolerance).
 * ---------------------------------------------------------------------------------------- */
#define GPB2_COMM_ID_BYTES 128
typedef struct gpb2_comm gpb2_comm;
int gpb2_comm_unique_id(unsigned char* id);
int gpb2_comm_create(gpb2_comm** out, int nranks, int rank, const unsigned char* id, int device,
                     double timeout_s);
int gpb2_comm_set_min_shard(gpb2_comm* comm, int64_t min_shard);
int gpb2_comm_info(const gpb2_comm* comm, int* nranks, int* rank);
int gpb2_comm_destroy(gpb2_comm* comm);

/* generate / generate_grad_xi / generate_grad_vals with level-sharded sweeps
 * (src/distributed.jl:281-331; single-GPU forms src/orchestrate.jl:19-42, src/grad.jl:392-506,
 * src/grad_generate_vals.jl:111-282). */
int gpb2_generate_sharded(gpb2_problem* prob, gpb2_comm* comm, const void* xi_dev, void* out_dev,
                          void* stream);
int gpb2_generate_grad_xi_sharded(gpb2_problem* prob, gpb2_comm* comm, const void* vbar_dev,
                                  void* xbar_dev, void* stream);
int gpb2_generate_grad_vals_sharded(gpb2_problem* prob, gpb2_comm* comm, const void* xi_dev,
                                    const void* vbar_dev, void* dvals_dev, void* stream);
/* Fitting reductions, scheme A (src/distributed.jl:129-247): generate_logdet,
 * generate_logdet_(and_)grad_vals, generate_inv_loss_grad_vals. */
int gpb2_generate_logdet_sharded(gpb2_problem* prob, gpb2_comm* comm, double* logdet_host,
                                 void* stream);
int gpb2_generate_logdet_grad_vals_sharded(gpb2_problem* prob, gpb2_comm* comm, void* dvals_dev,
                                           double* logdet_host, void* stream);
int gpb2_generate_inv_loss_grad_vals_sharded(gpb2_problem* prob, gpb2_comm* comm,
                                             const void* data_dev, void* dvals_dev,
                                             double* loss_host, void* stream);
/* The sharding plan of a rank (host only, no GPU): per depth batch b, the forward range
 * [fwd_lo[b], fwd_hi[b]) the rank computes, the range [own_lo[b], own_hi[b]) whose cotangents it
 * scatters, whether the batch is split (sharded[b]), and the slack past N the collectives may
 * touch.  Arrays have n_offsets - 1 entries; any may be NULL. */
int gpb2_shard_plan(const int64_t* offsets, int64_t n_offsets, int nranks, int rank,
                    int64_t min_shard, int64_t* fwd_lo, int64_t* fwd_hi, int64_t* own_lo,
                    int64_t* own_hi, int* sharded, int64_t* slack);

/* ------------------------------------------------------------------------------------------
 * Graph build (host, the input producer of the path).  Restates build_graph
 * (src/graph_build.jl:256-288: special-order tree, preceding k-NN, depths, stable order by
 * depth, 21-bit quantisation, offsets); its output is byte-identical to the reference's.
 * Replaces gpcuda_build_graph_f32 (csrc/graphgp_capi.cu:100-117) as the graph source.
 * points: N x D float64, dim-major (Julia's (N, D) column-major) when points_dim_major != 0,
 * else point-major.  Export: coords (N*D uint32, point-major), nbrs (M*K int64, 0-based, -1 =
 * unset), indices (N int64, 0-based tree->original), offsets (gpb2_graph_n_offsets entries).
 * ---------------------------------------------------------------------------------------- */
int gpb2_build_graph(const double* points, int64_t n, int64_t d, int64_t points_dim_major,
                     int64_t n0, int64_t k, int64_t lattice_bits, int64_t nthreads,
                     gpb2_graph** out);
int64_t gpb2_graph_n_offsets(const gpb2_graph* g);
int64_t gpb2_graph_n0(const gpb2_graph* g);
int gpb2_graph_export(const gpb2_graph* g, uint32_t* coords, int64_t* nbrs, int64_t* indices,
                      int64_t* offsets, double* scale);
void gpb2_graph_free(gpb2_graph* g);

/* build_graph on the device: the same graph, byte for byte, as gpb2_build_graph (and so as the
 * reference's build_graph), built by sm_100a kernels from points already on `device`
 * (points_dev: N x D float64, dim-major when points_dim_major != 0, else point-major), ordered
 * on `stream`; the call waits for its work.  k <= 32, N < 2^31.  Replaces the reference's
 * device builder gpcuda_build_graph_f32 (csrc/graphgp_capi.cu:100-117), which does not
 * reproduce build_graph's output; this one does.  The arrays stay on the device:
 * gpb2_dgraph_export copies coords (N*D uint32, point-major), nbrs (M*K int32, 0-based, -1 =
 * unset), indices (N int32, 0-based tree->original) into caller buffers on the same device (any
 * pointer may be NULL) and the offsets and scale to the host. */
typedef struct gpb2_dgraph gpb2_dgraph;
int gpb2_build_graph_device(const double* points_dev, int64_t n, int64_t d,
                            int64_t points_dim_major, int64_t n0, int64_t k, int64_t lattice_bits,
                            int device, void* stream, gpb2_dgraph** out);
int64_t gpb2_dgraph_n_offsets(const gpb2_dgraph* g);
int64_t gpb2_dgraph_n0(const gpb2_dgraph* g);
int gpb2_dgraph_export(const gpb2_dgraph* g, uint32_t* coords_dev, int32_t* nbrs_dev,
                       int32_t* indices_dev, int64_t* offsets_host, double* scale, void* stream);
void gpb2_dgraph_free(gpb2_dgraph* g);

#ifdef __cplusplus
}
#endif

#endif /* GRAPHGP_B200_H */
