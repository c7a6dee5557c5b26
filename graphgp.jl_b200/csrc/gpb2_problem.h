// gpb2_problem.h -- the problem handle behind gpb2_problem* (internal).
#pragma once
#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <cusolverDn.h>

#include <cstdint>
#include <vector>

#include "gpb2_internal.h"
#include "gpb2_kernels.cuh"

struct gpb2_problem {
    int dtype = GPB2_F32;
    int device = 0;
    int64_t n = 0, m = 0, k = 0, d = 0, n0 = 0, nb = 0;
    double scale = 0.0;
    std::vector<int64_t> offsets;  // host: offsets[0] == n0, offsets.back() == n
    int64_t* d_offsets = nullptr;  // device copy of offsets
    unsigned int* dsync = nullptr; // grid barrier of the persistent kernels: [0] arrivals,
                                   // [1] generation, [2] error word

    // Device copies owned by the handle.
    uint32_t* coords = nullptr;  // (N, coord_stride(D))
    int* nbrs = nullptr;         // (M, K) int32, 0-based
    int* indices = nullptr;      // (N) library -> original, 0-based; nullptr = identity
    int* lib_tree = nullptr;     // (N) library -> tree position (gpb2_order.cu); nullptr = the
                                 // tree order itself (the arrays above are in library order)
    void* bins = nullptr;        // (nb) T
    void* vals = nullptr;        // (nb) T
    void* seg = nullptr;         // 4 * (nb - 1) T
    uint16_t* start = nullptr;   // nkeys
    int nkeys = 0, shift = 0;
    uint64_t key_base = 0;
    double b0 = 0, b1 = 0, bN = 0, v0 = 0, vN = 0, pivc = 0;  // exact T values, widened

    // Scratch, allocated on first use and kept until destroy.
    void* mv = nullptr;      // (M, K) T
    void* sd = nullptr;      // (M) T
    void* buf_a = nullptr;   // (N) T   tree-order field / values
    void* buf_b = nullptr;   // (N) T   tree-order xi
    void* buf_c = nullptr;   // (N) T   tree-order cotangent
    void* buf_d = nullptr;   // (N) T   tree-order xbar
    double* dacc = nullptr;  // nb histogram + 8 scalars (double accumulators)
    double* dpts = nullptr;  // (N, D) point-position gradient, library positions
    bool factor_valid = false;  // mv / sd hold the current table's per-point factors

    // Per-point factor cache (FactorCache): the packed Cholesky factor and the pair weights of
    // every refined point, in slabs of M entries.  Mode 0 off, 1 on, 2 (default) on from the
    // first vals-gradient call when it fits in the device's free memory with a margin.
    void* fc_L = nullptr;        // NT slabs of T
    void* fc_t = nullptr;        // NR slabs of T
    uint16_t* fc_lo = nullptr;   // NR slabs of uint16
    int fc_mode = 2;
    bool fc_valid = false;       // the cache holds the current table's factors of all points
    bool fc_sh_valid = false;    // ... of the points of this rank's level-sharded forward ranges

    // Anisotropic covariance (src/aniso.jl), when set: the forward operations assemble from it
    // instead of the table (bins/vals stay as given and unused).  (ns), (nz), (ns, nz) T.
    void* an_sb = nullptr;
    void* an_zb = nullptr;
    void* an_grid = nullptr;
    int an_ns = 0, an_nz = 0;
    double an_alpha = 1.0, an_diag = 0.0;  // alpha; aniso_lookup(0, 0) (the ladder's diagonal)

    // Transposed graph of the pull-form reverse sweep (gpb2_rev.cu): rev_off (N + 1) delimits
    // each point's incoming edges in rev_mj (child m * K + slot j, in the serial sweep's order)
    // and rev_w (that slot's mean_vec, per table).  Mode 0: atomic push; 1: pull; 2 (default):
    // pull when the graph fits in free memory with a margin.
    uint32_t* rev_off = nullptr;
    int* rev_mj = nullptr;
    void* rev_w = nullptr;
    int rev_mode = 2;
    bool rev_w_valid = false;    // rev_w holds the current table's weights

    // Dense n0 block.
    void* Ld = nullptr;       // (n0, n0) column-major lower: the selected ladder candidate
    void* Lcand = nullptr;    // ladder candidates, each (n0, n0) column-major lower
    int* lad = nullptr;       // ladder status (layout: kLad* in gpb2::) + jitters
    std::vector<unsigned char> hbins;  // host copy of the bins (fixed for the handle's life)
    std::vector<double> ladder_eps;  // eps of each ladder index of the last factorisation
    void* trace = nullptr;           // diagnostics buffer (GPB2_TRACE_DENSE)
    size_t lcand_bytes = 0;          // capacity of Lcand (its candidate count can change per call)
    bool dense_pending = false;      // a factorisation was launched and not yet checked
    int* hstat = nullptr;            // pinned host copy of the status words (4 ints)
    double* hscal = nullptr;         // pinned host copy of the scalar accumulators (4 doubles)
    bool dense_launched = false;     // the current table's factorisation is launched (checked or
                                     // not); cleared by a new table and by a failed check
    bool dense_valid = false;        // Ld holds the checked factor of the current table; reused
                                     // by every call until the table changes
    int dense_candidate = -1;
    void* Ldr = nullptr;      // row-major copy of Ld, rows padded to 32 (triangular kernels)
    void* Dinv = nullptr;     // transposed inverses of Ld's 32x32 diagonal blocks
    void* Wtri = nullptr;     // 2 n0^2 + n0 T: the triangular kernels' work
    void* Ainv = nullptr;     // (n0, n0) column-major L^-1 of the current factor
    bool tri_ready = false;   // Ldr / Dinv belong to the current Ld
    bool tri_deferred = false;  // the ladder is queued and Ldr / Dinv / Ainv are not yet
    bool tri_pending = false;   // Ldr / Dinv / Ainv are queued on dstream up to ev_tri
    void* Wd = nullptr;       // (n0, n0) work
    void* Wd2 = nullptr;      // (n0, n0) work
    void* dwork = nullptr;    // cuSOLVER workspace
    int64_t dwork_bytes = 0;
    int* dinfo = nullptr;     // cuSOLVER info
    cusolverDnHandle_t solver = nullptr;
    cublasHandle_t blas = nullptr;
    cudaStream_t dstream = nullptr;   // high-priority stream of the overlapped dense factor
    cudaEvent_t ev_fork = nullptr;    // call stream -> dstream
    cudaEvent_t ev_join = nullptr;    // dstream -> call stream
    cudaEvent_t ev_tri = nullptr;     // Ldr written (triangular preparation on dstream)
    cudaEvent_t ev_inv = nullptr;     // Dinv and Ainv written (end of the preparation)
    double dense_jitter = 0.0;  // eps of the ladder that succeeded on the last factorisation
    int ladder_hint = -1;       // ladder index that succeeded last time (-1: none yet)

    const gpb2::Ops<float>* ops32 = nullptr;
    const gpb2::Ops<double>* ops64 = nullptr;

    // Level-sharded operations (gpb2_shard.cu): full-length buffers with slack for the
    // collectives' spill, the list of refined points this rank owns, and which sharding they
    // were built for.
    void* sh_v = nullptr;        // (N + slack) T   field
    void* sh_vb = nullptr;       // (N + slack) T   cotangent (partial per rank)
    void* sh_xg = nullptr;       // (N + slack) T   xi-cotangent
    int64_t sh_len = 0;          // entries of each of the three
    int* sh_own = nullptr;       // refined points (m) this rank's kernels visit
    int64_t sh_own_cnt = 0;
    int64_t sh_key[3] = {-1, -1, -1};  // (ranks, rank, min_shard) of sh_own
    bool sh_factor_valid = false;       // mv / sd hold this rank's points for the current table

    // Two-pass permutation plan of large problems (gpb2_perm.cu): staging buffer (N T) and, per
    // direction (g: original -> tree, s: tree -> original), each input's staging slot and each
    // output's rank in its destination block.
    // Two-pass permutation plans, original -> library (_g) and library -> original (_s):
    // pass 1 writes stage[pos[k]] = tile[from[k]] for slot k of each source tile, pass 2
    // out[d] = block[q[d]] for each destination block (tiles and blocks of 2^perm_shift values).
    void* perm_stage = nullptr;
    int* perm_pos_g = nullptr;
    uint16_t* perm_from_g = nullptr;
    uint16_t* perm_q_g = nullptr;
    int* perm_pos_s = nullptr;
    uint16_t* perm_from_s = nullptr;
    uint16_t* perm_q_s = nullptr;
    int perm_shift = 15;
};

namespace gpb2 {

// Layout of gpb2_problem::lad (ints), then 16 T of ladder jitters.
constexpr int kLadFail = 0;     // [0, 16): per-candidate failing column + 1
constexpr int kLadDone = 16;    // [16, 32): per-candidate completion flags
constexpr int kLadSel = 32;     // ladder index of the first success (-1: none), then its slot
constexpr int kLadNotPD = 34;   // set when no candidate succeeded
constexpr int kLadBarErr = 36;  // error word of the factorisation (0: none)
constexpr int kLadDflag = 48;   // [48, 64): per-candidate last published diagonal panel
constexpr int kLadOrder = 64;   // [64, 80): ladder index of each candidate slot of a launch
constexpr int kLadGridBar = 80; // grid barrier word of the whole-GPU factorisation
constexpr int kLadGridCtr = 84; // [84, 86): its trailing-tile counters (by panel parity)
constexpr int kLadInts = 96;

// RAII: make the problem's device current for the duration of a call, restore afterwards.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

template <typename T>
TableView<T> table_view(const gpb2_problem* p) {
    TableView<T> tv;
    tv.seg = static_cast<const T*>(p->seg);
    tv.start = p->start;
    tv.base = (typename Num<T>::U)p->key_base;
    tv.nb = (int)p->nb;
    tv.nkeys = p->nkeys;
    tv.shift = p->shift;
    tv.b0 = (T)p->b0;
    tv.b1 = (T)p->b1;
    tv.bN = (T)p->bN;
    tv.v0 = (T)p->v0;
    tv.vN = (T)p->vN;
    tv.pivc = (T)p->pivc;
    return tv;
}

// The kernels' view of the problem.  With a cache the arguments also carry the factor cache:
// as the target of the factor pass (FcUse::Fill, when it is allocated) or as the source of the
// vals-gradient kernels (FcUse::Read, when it holds the current table).
enum class FcUse { None, Fill, Read, ReadShard };

template <typename T>
AnisoView<T> aniso_view(const gpb2_problem* p) {
    AnisoView<T> av;
    if (p->an_grid) {
        av.sb = static_cast<const T*>(p->an_sb);
        av.zb = static_cast<const T*>(p->an_zb);
        av.grid = static_cast<const T*>(p->an_grid);
        av.ns = p->an_ns;
        av.nz = p->an_nz;
        av.alpha = (T)p->an_alpha;
    }
    return av;
}

template <typename T>
PointArgs<T> point_args(const gpb2_problem* p, FcUse fc = FcUse::None) {
    PointArgs<T> a;
    a.an = aniso_view<T>(p);
    a.tab = table_view<T>(p);
    a.coords = p->coords;
    a.nbrs = p->nbrs;
    a.n0 = p->n0;
    a.scale = (T)p->scale;
    // ReadShard: a level-sharded kernel over this rank's points, which the rank's own factor
    // pass may have filled.
    if (p->fc_L && (fc == FcUse::Fill || (fc == FcUse::Read && p->fc_valid) ||
                    (fc == FcUse::ReadShard && (p->fc_valid || p->fc_sh_valid)))) {
        a.fc.L = static_cast<T*>(p->fc_L);
        a.fc.t = static_cast<T*>(p->fc_t);
        a.fc.lo = p->fc_lo;
        a.fc.stride = p->m;
    }
    return a;
}

// Allocate the factor cache as the mode allows (mode 2: if it fits in free memory with a margin)
// and fill it for the current table; a no-op when it is valid or not to be used.  Called by the
// vals-gradient operations before their per-point kernel.
int ensure_factor_cache(gpb2_problem* p, cudaStream_t s);
// Bytes of the factor cache of a problem.
size_t factor_cache_bytes(const gpb2_problem* p);

// The transposed graph of the pull-form reverse sweep: built once per problem when the mode
// allows (mode 2: if it fits in free memory with a margin); its weights once per table, after
// the table's per-point factor pass.
int ensure_rev_graph(gpb2_problem* p, cudaStream_t s);
template <typename T>
int ensure_rev_weights(gpb2_problem* p, cudaStream_t s);
size_t rev_graph_bytes(const gpb2_problem* p);

template <typename T>
const Ops<T>* ops_of(const gpb2_problem* p);
template <>
inline const Ops<float>* ops_of<float>(const gpb2_problem* p) { return p->ops32; }
template <>
inline const Ops<double>* ops_of<double>(const gpb2_problem* p) { return p->ops64; }

int ensure_alloc(void** ptr, size_t bytes);
// Like ensure_alloc, but reallocates when the buffer (of *cap bytes) is smaller than `bytes`.
int ensure_capacity(void** ptr, size_t* cap, size_t bytes);
int ensure_scratch(gpb2_problem* p, bool need_mv);
int ensure_dense(gpb2_problem* p);

// The original <-> tree permutation in two streaming passes (gpb2_perm.cu), for problems whose
// field outgrows the L2 (perm_two_pass); the plan is built on first use.
bool perm_two_pass(const gpb2_problem* p);

// Re-sorts every depth batch of a freshly uploaded problem by Morton code (gpb2_order.cu).
int library_order(gpb2_problem* p, cudaStream_t s);
template <typename T>
int perm_apply(gpb2_problem* p, bool to_tree, const T* in, T* out, cudaStream_t s);

// Dense first layer (gpb2_dense.cu).  All on `s`; factor() synchronises once to read the
// Cholesky status (the jitter ladder of src/dense.jl:46-67 branches on it).
template <typename T>
int dense_cholesky_ladder(gpb2_problem* p, cudaStream_t s);

// Triangular kernels of the dense layer (gpb2_dense_tri.cu).
template <typename T>
bool dense_tri_supported(const gpb2_problem* p);
template <typename T>
// Ldr + Dinv + Ainv from Ld; after_ldr (if any) is recorded once Ldr is written.
int dense_tri_prepare(gpb2_problem* p, cudaStream_t s, cudaEvent_t after_ldr = nullptr);
template <typename T>
int dense_trmv(gpb2_problem* p, bool trans, const T* x, T* y, cudaStream_t s);
template <typename T>
int dense_chol_pullback_outer(gpb2_problem* p, const T* vb, const T* xi, const T** S,
                              cudaStream_t s);

template <typename T>
struct Dense {
    // defer_tri: queue only the ladder; finish_tri() then queues Ldr / Dinv / Ainv.
    static int factor(gpb2_problem* p, cudaStream_t s, bool defer_tri = false);
    static int finish_tri(gpb2_problem* p, cudaStream_t s);
    static int apply_L(gpb2_problem* p, const T* x, T* y, cudaStream_t s);   // y = L x
    static int apply_Lt(gpb2_problem* p, const T* x, T* y, cudaStream_t s);  // y = L^T x
    static int solve_L(gpb2_problem* p, const T* b, T* y, cudaStream_t s);   // y = L \ b
    static int logdet(gpb2_problem* p, double* acc, cudaStream_t s);         // acc += sum log diag
    static int grad_vals(gpb2_problem* p, const T* vb, const T* xi, double* hist, cudaStream_t s);
    // Position gradients of the dense block into dp ((N, D) row-major, added).
    static int logdet_points(gpb2_problem* p, double* dp, cudaStream_t s);
    static int inv_loss_points(gpb2_problem* p, const T* y, double* dp, cudaStream_t s);
    static int logdet_grad(gpb2_problem* p, double* hist, cudaStream_t s);
    static int inv_loss_grad(gpb2_problem* p, const T* y, double* hist, double* loss,
                             cudaStream_t s);
};

}  // namespace gpb2
