// Tensor-parallel communication for the sm_100a backend: NCCL, loaded at run
// time (no link-time dependency; in a process that already holds an NCCL
// library, e.g. through PyTorch, the same copy is reused).  The model's
// communicator performs the all-reduce after the row-parallel projections
// (o_proj, down_proj) and the all-gather of the vocabulary-sharded logits.
// The reference engine has no multi-GPU path; this is new in this backend.
#include "hc_internal.h"
#include "hc_comm.h"

#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

namespace hc {

namespace {

struct NcclApi {
    void* handle = nullptr;
    decltype(&ncclGetUniqueId) getUniqueId = nullptr;
    decltype(&ncclCommInitRankConfig) commInitRankConfig = nullptr;
    decltype(&ncclCommDestroy) commDestroy = nullptr;
    decltype(&ncclCommAbort) commAbort = nullptr;
    decltype(&ncclCommGetAsyncError) commGetAsyncError = nullptr;
    decltype(&ncclAllReduce) allReduce = nullptr;
    decltype(&ncclAllGather) allGather = nullptr;
    decltype(&ncclGetErrorString) getErrorString = nullptr;
    bool ok = false;
};

NcclApi& api() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        const char* names[] = {"libnccl.so.2", "libnccl.so"};
        for (const char* n : names) {
            a.handle = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
            if (a.handle) break;
        }
        if (!a.handle) return;
#define HC_SYM(field, name) a.field = reinterpret_cast<decltype(a.field)>(dlsym(a.handle, name))
        HC_SYM(getUniqueId, "ncclGetUniqueId");
        HC_SYM(commInitRankConfig, "ncclCommInitRankConfig");
        HC_SYM(commDestroy, "ncclCommDestroy");
        HC_SYM(commAbort, "ncclCommAbort");
        HC_SYM(commGetAsyncError, "ncclCommGetAsyncError");
        HC_SYM(allReduce, "ncclAllReduce");
        HC_SYM(allGather, "ncclAllGather");
        HC_SYM(getErrorString, "ncclGetErrorString");
#undef HC_SYM
        a.ok = a.getUniqueId && a.commInitRankConfig && a.commDestroy && a.commAbort && a.commGetAsyncError &&
               a.allReduce && a.allGather && a.getErrorString;
    });
    return a;
}

int nccl_fail(ncclResult_t r, const char* what) {
    hc_set_error("NCCL %s failed: %s (%d)", what, api().getErrorString ? api().getErrorString(r) : "?", (int)r);
    return HC_ERR_CUDA;
}

}  // namespace

struct Comm {
    ncclComm_t comm = nullptr;
    int rank = 0, size = 1;
    double timeout_s = 60.0;
    bool aborted = false;
};

int comm_unique_id(uint8_t* out128) {
    NcclApi& a = api();
    HC_CHECK(a.ok, HC_ERR_UNSUPPORTED, "NCCL library (libnccl.so.2) not found");
    ncclUniqueId id;
    ncclResult_t r = a.getUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail(r, "GetUniqueId");
    std::memcpy(out128, id.internal, NCCL_UNIQUE_ID_BYTES);
    return HC_OK;
}

// Non-blocking communicator: collectives return at once and a host watchdog
// (comm_wait) can abort a communicator whose peer stopped participating.
int comm_init(Comm** out, const uint8_t* id128, int rank, int size, double timeout_s) {
    NcclApi& a = api();
    HC_CHECK(a.ok, HC_ERR_UNSUPPORTED, "NCCL library (libnccl.so.2) not found");
    ncclUniqueId id;
    std::memcpy(id.internal, id128, NCCL_UNIQUE_ID_BYTES);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    Comm* c = new Comm();
    c->rank = rank;
    c->size = size;
    c->timeout_s = timeout_s;
    ncclResult_t r = a.commInitRankConfig(&c->comm, size, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        delete c;
        return nccl_fail(r, "CommInitRankConfig");
    }
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclInProgress;
        a.commGetAsyncError(c->comm, &st);
        if (st == ncclSuccess) break;
        if (st != ncclInProgress) {
            a.commAbort(c->comm);
            delete c;
            return nccl_fail(st, "communicator initialisation");
        }
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s) {
            a.commAbort(c->comm);
            delete c;
            hc_set_error("NCCL communicator initialisation timed out after %.0f s", timeout_s);
            return HC_ERR_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    *out = c;
    return HC_OK;
}

void comm_free(Comm* c) {
    if (!c) return;
    if (c->comm) {
        if (c->aborted) api().commAbort(c->comm);
        else api().commDestroy(c->comm);
    }
    delete c;
}

// Waits for an in-progress non-blocking enqueue.  The first collective of a
// communicator also sets up its peer connections, which can take far longer
// than later enqueues, so the bound is the communicator's own timeout; on
// expiry the communicator is aborted.
static int comm_enqueue_ok(Comm* c, ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return HC_OK;
    if (r != ncclInProgress) return nccl_fail(r, what);
    auto t0 = std::chrono::steady_clock::now();
    for (int i = 0;; i++) {
        ncclResult_t st = ncclInProgress;
        api().commGetAsyncError(c->comm, &st);
        if (st == ncclSuccess) return HC_OK;
        if (st != ncclInProgress) return nccl_fail(st, what);
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > c->timeout_s) break;
        if (i < 1000) std::this_thread::yield();
        else std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    api().commAbort(c->comm);
    c->aborted = true;
    hc_set_error("NCCL %s: enqueue did not complete within %.0f s; communicator aborted", what, c->timeout_s);
    return HC_ERR_TIMEOUT;
}

int comm_allreduce_sum(Comm* c, float* buf, size_t count, cudaStream_t s) {
    HC_CHECK(c && !c->aborted, HC_ERR_STATE, "communicator unavailable");
    return comm_enqueue_ok(c, api().allReduce(buf, buf, count, ncclFloat32, ncclSum, c->comm, s), "AllReduce");
}

int comm_allgather(Comm* c, const float* send, float* recv, size_t count, cudaStream_t s) {
    HC_CHECK(c && !c->aborted, HC_ERR_STATE, "communicator unavailable");
    return comm_enqueue_ok(c, api().allGather(send, recv, count, ncclFloat32, c->comm, s), "AllGather");
}

int comm_allgather_host(Comm* c, const void* send, void* recv, size_t bytes) {
    HC_CHECK(c && !c->aborted, HC_ERR_STATE, "communicator unavailable");
    uint8_t* d = nullptr;
    HC_CUDA(cudaMalloc((void**)&d, bytes * (size_t)(c->size + 1)));
    cudaStream_t s = nullptr;
    int rc = HC_OK;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) {
        cudaFree(d);
        return hc_cuda_fail(cudaGetLastError(), "cudaStreamCreate", __FILE__, __LINE__);
    }
    uint8_t* dsend = d + bytes * (size_t)c->size;
    if (cudaMemcpyAsync(dsend, send, bytes, cudaMemcpyHostToDevice, s) != cudaSuccess)
        rc = hc_cuda_fail(cudaGetLastError(), "cudaMemcpyAsync", __FILE__, __LINE__);
    if (rc == HC_OK) rc = comm_enqueue_ok(c, api().allGather(dsend, d, bytes, ncclUint8, c->comm, s), "AllGather");
    if (rc == HC_OK) rc = comm_wait(c, s, c->timeout_s);
    if (rc == HC_OK && cudaMemcpy(recv, d, bytes * (size_t)c->size, cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = hc_cuda_fail(cudaGetLastError(), "cudaMemcpy", __FILE__, __LINE__);
    cudaStreamDestroy(s);
    cudaFree(d);
    return rc;
}

// Host watchdog: waits for the stream while polling the communicator; a peer
// that stopped participating (or an NCCL error) ends in ncclCommAbort after
// timeout_s and HC_ERR_TIMEOUT, instead of a wait without end.
int comm_wait(Comm* c, cudaStream_t s, double timeout_s) {
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return HC_OK;
        if (e != cudaErrorNotReady) return hc_cuda_fail(e, "cudaStreamQuery", __FILE__, __LINE__);
        if (c && c->comm && !c->aborted) {
            ncclResult_t st = ncclSuccess;
            api().commGetAsyncError(c->comm, &st);
            if (st != ncclSuccess && st != ncclInProgress) {
                api().commAbort(c->comm);
                c->aborted = true;
                return nccl_fail(st, "collective");
            }
        }
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s) {
            if (c && c->comm && !c->aborted) {
                api().commAbort(c->comm);
                c->aborted = true;
            }
            hc_set_error("tensor-parallel step did not finish within %.1f s; communicator aborted", timeout_s);
            return HC_ERR_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // namespace hc
