// gpb2_comm.cu -- the NCCL communicator of the level-sharded operations (one process or thread
// per GPU).  The reference's distributed layer exchanges each depth level's new values with an
// MPI sum-Allreduce issued from a host loop (src/distributed.jl:281-331, ext/GraphGPMPIExt.jl
// shims :99-115); here the exchange is NCCL over NVLink, issued by the library itself on the
// caller's stream between the batch kernels, so the whole per-batch schedule is one C call.
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <thread>

#include "gpb2_comm.h"
#include "gpb2_problem.h"

struct gpb2_comm {
    ncclComm_t nccl = nullptr;
    int nranks = 1;
    int rank = 0;
    int device = 0;
    int64_t min_shard = 65536;
};

namespace gpb2 {

#define GPB2_NCCL_TRY(expr)                                                                    \
    do {                                                                                       \
        ncclResult_t _r = (expr);                                                              \
        if (_r != ncclSuccess)                                                                 \
            return set_error(GPB2_ERR_NCCL, "%s:%d: %s -> %s", __FILE__, __LINE__, #expr,      \
                             ncclGetErrorString(_r));                                          \
    } while (0)

int comm_rank(const gpb2_comm* c) { return c->rank; }
int comm_size(const gpb2_comm* c) { return c->nranks; }
int64_t comm_min_shard(const gpb2_comm* c) { return c->min_shard; }

static ncclDataType_t nccl_type(bool f64) { return f64 ? ncclFloat64 : ncclFloat32; }

// The communicator is non-blocking (so that its creation can time out): a call may return
// ncclInProgress, and the next call on the communicator may only be made once the state has
// left ncclInProgress.  Bounded at 60 s.
static int settle(gpb2_comm* c, ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return GPB2_OK;
    if (r != ncclInProgress)
        return set_error(GPB2_ERR_NCCL, "%s: %s", what, ncclGetErrorString(r));
    const auto t0 = std::chrono::steady_clock::now();
    ncclResult_t state = ncclInProgress;
    while (true) {
        const ncclResult_t q = ncclCommGetAsyncError(c->nccl, &state);
        if (q != ncclSuccess)
            return set_error(GPB2_ERR_NCCL, "%s: %s", what, ncclGetErrorString(q));
        if (state != ncclInProgress) break;
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > 60)
            return set_error(GPB2_ERR_TIMEOUT, "%s: NCCL did not settle within 60 s", what);
        std::this_thread::yield();
    }
    if (state != ncclSuccess)
        return set_error(GPB2_ERR_NCCL, "%s: %s", what, ncclGetErrorString(state));
    return GPB2_OK;
}

int comm_all_gather(gpb2_comm* c, void* buf, int64_t lo, int64_t count, bool f64,
                    cudaStream_t s) {
    const size_t es = f64 ? 8 : 4;
    char* base = static_cast<char*>(buf) + es * lo;
    return settle(c, ncclAllGather(base + es * count * c->rank, base, (size_t)count,
                                   nccl_type(f64), c->nccl, s),
                  "ncclAllGather");
}

int comm_reduce_scatter(gpb2_comm* c, void* buf, int64_t lo, int64_t count, bool f64,
                        cudaStream_t s) {
    const size_t es = f64 ? 8 : 4;
    char* base = static_cast<char*>(buf) + es * lo;
    return settle(c, ncclReduceScatter(base, base + es * count * c->rank, (size_t)count,
                                       nccl_type(f64), ncclSum, c->nccl, s),
                  "ncclReduceScatter");
}

int comm_all_reduce(gpb2_comm* c, void* buf, int64_t count, bool f64, cudaStream_t s) {
    return settle(c, ncclAllReduce(buf, buf, (size_t)count, nccl_type(f64), ncclSum, c->nccl, s),
                  "ncclAllReduce");
}

}  // namespace gpb2

using namespace gpb2;

extern "C" {

int gpb2_comm_unique_id(unsigned char* id) {
    clear_error();
    if (!id) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_comm_unique_id: NULL");
    static_assert(sizeof(ncclUniqueId) == GPB2_COMM_ID_BYTES, "NCCL unique id size");
    ncclUniqueId u;
    GPB2_NCCL_TRY(ncclGetUniqueId(&u));
    std::memcpy(id, &u, sizeof(u));
    return GPB2_OK;
}

int gpb2_comm_create(gpb2_comm** out, int nranks, int rank, const unsigned char* id, int device,
                     double timeout_s) {
    clear_error();
    if (!out || !id) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_comm_create: NULL");
    *out = nullptr;
    if (nranks < 1 || rank < 0 || rank >= nranks)
        return set_error(GPB2_ERR_INVALID_ARG, "gpb2_comm_create: rank %d of %d", rank, nranks);
    DeviceGuard dg(device);
    if (!dg.ok) return set_error(GPB2_ERR_NO_DEVICE, "cudaSetDevice(%d) failed", device);
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    // Non-blocking initialisation polled against a deadline, so that a rank that never joins
    // ends the call with an error instead of a wait without end.
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclComm_t comm = nullptr;
    ncclResult_t r = ncclCommInitRankConfig(&comm, nranks, u, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress)
        return set_error(GPB2_ERR_NCCL, "ncclCommInitRankConfig: %s", ncclGetErrorString(r));
    const auto t0 = std::chrono::steady_clock::now();
    ncclResult_t state = ncclInProgress;
    while (true) {
        r = ncclCommGetAsyncError(comm, &state);
        if (r != ncclSuccess || state != ncclInProgress) break;
        const double el =
            std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (timeout_s > 0 && el > timeout_s) {
            ncclCommAbort(comm);
            return set_error(GPB2_ERR_TIMEOUT,
                             "gpb2_comm_create: not every rank joined within %.0f s", timeout_s);
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    if (r != ncclSuccess || state != ncclSuccess) {
        ncclCommAbort(comm);
        return set_error(GPB2_ERR_NCCL, "NCCL communicator initialisation failed: %s",
                         ncclGetErrorString(r != ncclSuccess ? r : state));
    }
    auto* c = new gpb2_comm();
    c->nccl = comm;
    c->nranks = nranks;
    c->rank = rank;
    c->device = device;
    *out = c;
    return GPB2_OK;
}

int gpb2_comm_set_min_shard(gpb2_comm* c, int64_t min_shard) {
    if (!c || min_shard < 1) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_comm_set_min_shard");
    c->min_shard = min_shard;
    return GPB2_OK;
}

int gpb2_comm_info(const gpb2_comm* c, int* nranks, int* rank) {
    if (!c) return set_error(GPB2_ERR_INVALID_ARG, "gpb2_comm_info: NULL");
    if (nranks) *nranks = c->nranks;
    if (rank) *rank = c->rank;
    return GPB2_OK;
}

int gpb2_comm_destroy(gpb2_comm* c) {
    if (!c) return GPB2_OK;
    DeviceGuard dg(c->device);
    ncclResult_t r = ncclSuccess;
    if (c->nccl) {
        // The communicator is non-blocking: finalize, then wait for it before destroying.
        r = ncclCommFinalize(c->nccl);
        if (r == ncclInProgress) r = ncclSuccess;
        ncclResult_t state = ncclInProgress;
        const auto t0 = std::chrono::steady_clock::now();
        while (r == ncclSuccess) {
            if (ncclCommGetAsyncError(c->nccl, &state) != ncclSuccess || state != ncclInProgress)
                break;
            if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > 60)
                break;
            std::this_thread::sleep_for(std::chrono::milliseconds(1));
        }
        if (r == ncclSuccess && state == ncclSuccess)
            ncclCommDestroy(c->nccl);
        else
            ncclCommAbort(c->nccl);
    }
    delete c;
    return r == ncclSuccess ? GPB2_OK : set_error(GPB2_ERR_NCCL, "ncclCommFinalize failed");
}

}  // extern "C"
