// qsamp_comm.cpp -- the candidate exchange of vocab-sharded selection over a
// non-blocking NCCL communicator whose every wait has a deadline
// (include/qsamp_comm.h). Host code: no kernels of its own; the all-gather
// runs NCCL's.
#include <cuda_runtime.h>
#include <nccl.h>

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <thread>

#include "../../include/qsamp_comm.h"

struct qsamp_comm {
    ncclComm_t comm = nullptr;
    int nranks = 0, rank = 0, device = 0;
    int64_t timeout_ms = 0;
    bool aborted = false;
    std::string err;
};

namespace {

void put(char* err, size_t n, const char* fmt, ...) {
    if (!err || !n) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, n, fmt, ap);
    va_end(ap);
}

// The calls one bounded wait makes: the communicator's asynchronous error,
// whether the awaited work is done (1), pending (0) or failed (-1), and the
// abort. The real communicator and the self-test's fake supply them.
struct WaitOps {
    ncclResult_t (*async_error)(void* h, ncclResult_t* out);
    int (*done)(void* h);
    void (*abort)(void* h);
    void* h;
};

enum WaitResult { W_DONE = 0, W_ERROR = 1, W_TIMEOUT = 2 };

// Polls until the work is done, an asynchronous error appears or timeout_ms
// pass; an error or the deadline aborts. *nerr: the NCCL error seen.
WaitResult bounded_wait(const WaitOps& o, int64_t timeout_ms, ncclResult_t* nerr) {
    const auto t0 = std::chrono::steady_clock::now();
    int spins = 0;
    *nerr = ncclSuccess;
    while (true) {
        ncclResult_t ae = ncclSuccess;
        const ncclResult_t q = o.async_error(o.h, &ae);
        if (q != ncclSuccess || (ae != ncclSuccess && ae != ncclInProgress)) {
            *nerr = q != ncclSuccess ? q : ae;
            o.abort(o.h);
            return W_ERROR;
        }
        if (ae == ncclSuccess) {
            const int d = o.done(o.h);
            if (d > 0) return W_DONE;
            if (d < 0) {
                o.abort(o.h);
                return W_ERROR;
            }
        }
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0)
                            .count();
        if (ms >= timeout_ms) {
            o.abort(o.h);
            return W_TIMEOUT;
        }
        // spin briefly (a collective usually completes in microseconds), then yield
        if (++spins > 64) std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

// ---- the real communicator
struct RealWait {
    qsamp_comm* c;
    bool use_stream;      // false: wait for the communicator alone (init, enqueue)
    cudaStream_t stream;  // (handle 0, the default stream, is a stream like any other)
};
ncclResult_t real_async_error(void* h, ncclResult_t* out) {
    return ncclCommGetAsyncError(static_cast<RealWait*>(h)->c->comm, out);
}
int real_done(void* h) {
    RealWait* w = static_cast<RealWait*>(h);
    if (!w->use_stream) return 1;
    const cudaError_t e = cudaStreamQuery(w->stream);
    if (e == cudaSuccess) return 1;
    if (e == cudaErrorNotReady) return 0;
    return -1;
}
void real_abort(void* h) {
    qsamp_comm* c = static_cast<RealWait*>(h)->c;
    if (c->comm) ncclCommAbort(c->comm);
    c->comm = nullptr;
    c->aborted = true;
}

qsamp_status wait_real(qsamp_comm* c, bool use_stream, cudaStream_t stream, const char* what) {
    RealWait rw{c, use_stream, stream};
    WaitOps ops{real_async_error, real_done, real_abort, &rw};
    ncclResult_t nerr = ncclSuccess;
    const WaitResult r = bounded_wait(ops, c->timeout_ms, &nerr);
    if (r == W_DONE) return QSAMP_OK;
    char buf[256];
    if (r == W_TIMEOUT) {
        snprintf(buf, sizeof buf, "%s: not complete after %lld ms (a rank did not join, or a peer failed); "
                 "communicator aborted", what, (long long)c->timeout_ms);
        c->err = buf;
        return QSAMP_ERR_TIMEOUT;
    }
    snprintf(buf, sizeof buf, "%s: %s; communicator aborted", what,
             nerr != ncclSuccess ? ncclGetErrorString(nerr) : "the stream reported an error");
    c->err = buf;
    return QSAMP_ERR_COMM;
}

}  // namespace

extern "C" {

qsamp_status qsamp_comm_unique_id(unsigned char id[QSAMP_COMM_ID_BYTES]) {
    if (!id) return QSAMP_ERR_INVALID_ARG;
    static_assert(sizeof(ncclUniqueId) == QSAMP_COMM_ID_BYTES, "NCCL unique id size");
    ncclUniqueId u;
    if (ncclGetUniqueId(&u) != ncclSuccess) return QSAMP_ERR_COMM;
    std::memcpy(id, &u, sizeof u);
    return QSAMP_OK;
}

qsamp_status qsamp_comm_create(int32_t nranks, int32_t rank, const unsigned char id[QSAMP_COMM_ID_BYTES],
                               int32_t device, int64_t timeout_ms, qsamp_comm** out, char* err, size_t err_len) {
    if (err && err_len) err[0] = '\0';
    if (!out) return put(err, err_len, "out: expected non-NULL"), QSAMP_ERR_INVALID_ARG;
    *out = nullptr;
    if (nranks < 1) return put(err, err_len, "nranks: expected >= 1, got %d", nranks), QSAMP_ERR_INVALID_ARG;
    if (rank < 0 || rank >= nranks)
        return put(err, err_len, "rank: expected [0,%d), got %d", nranks, rank), QSAMP_ERR_INVALID_ARG;
    if (!id) return put(err, err_len, "id: expected non-NULL"), QSAMP_ERR_INVALID_ARG;
    if (timeout_ms <= 0)
        return put(err, err_len, "timeout_ms: expected > 0, got %lld", (long long)timeout_ms), QSAMP_ERR_INVALID_ARG;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
        cudaGetLastError();
        return put(err, err_len, "device: expected [0,%d), got %d", ndev, device), QSAMP_ERR_INVALID_ARG;
    }
    qsamp_comm* c = new (std::nothrow) qsamp_comm();
    if (!c) return QSAMP_ERR_NO_MEMORY;
    c->nranks = nranks;
    c->rank = rank;
    c->device = device;
    c->timeout_ms = timeout_ms;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // every NCCL call returns at once; the waits below poll
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof u);
    const ncclResult_t r = ncclCommInitRankConfig(&c->comm, nranks, u, rank, &cfg);
    qsamp_status s = QSAMP_OK;
    if (r != ncclSuccess && r != ncclInProgress) {
        put(err, err_len, "ncclCommInitRankConfig: %s", ncclGetErrorString(r));
        if (c->comm) ncclCommAbort(c->comm);
        c->comm = nullptr;
        s = QSAMP_ERR_COMM;
    } else {
        s = wait_real(c, false, nullptr, "communicator initialisation");
        if (s != QSAMP_OK) put(err, err_len, "%s", c->err.c_str());
    }
    cudaSetDevice(prev);
    if (s != QSAMP_OK) {
        delete c;
        return s;
    }
    *out = c;
    return QSAMP_OK;
}

qsamp_status qsamp_comm_allgather_candidates(qsamp_comm* c, const float* vals, const int32_t* ids,
                                             int64_t per_rank, float* all_vals, int32_t* all_ids, void* stream) {
    if (!c) return QSAMP_ERR_INVALID_ARG;
    if (c->aborted) return c->err = "the communicator was aborted: destroy it and create a new one", QSAMP_ERR_COMM;
    if (per_rank < 0) {
        c->err = "per_rank: expected >= 0";
        return QSAMP_ERR_INVALID_ARG;
    }
    if (per_rank == 0) return QSAMP_OK;
    if (!vals || !ids || !all_vals || !all_ids) {
        c->err = "vals/ids/all_vals/all_ids: expected non-NULL";
        return QSAMP_ERR_INVALID_ARG;
    }
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != c->device) cudaSetDevice(c->device);
    cudaStream_t st = (cudaStream_t)stream;
    ncclResult_t r = ncclGroupStart();
    if (r == ncclSuccess)
        r = ncclAllGather(vals, all_vals, (size_t)per_rank, ncclFloat32, c->comm, st);
    if (r == ncclSuccess || r == ncclInProgress)
        r = ncclAllGather(ids, all_ids, (size_t)per_rank, ncclInt32, c->comm, st);
    const ncclResult_t g = ncclGroupEnd();
    qsamp_status s = QSAMP_OK;
    if ((r != ncclSuccess && r != ncclInProgress) || (g != ncclSuccess && g != ncclInProgress)) {
        c->err = std::string("ncclAllGather: ") + ncclGetErrorString(r != ncclSuccess && r != ncclInProgress ? r : g);
        if (c->comm) ncclCommAbort(c->comm);
        c->comm = nullptr;
        c->aborted = true;
        s = QSAMP_ERR_COMM;
    } else {
        s = wait_real(c, false, nullptr, "enqueueing the candidate all-gather");
    }
    if (prev != c->device) cudaSetDevice(prev);
    return s;
}

qsamp_status qsamp_comm_wait(qsamp_comm* c, void* stream) {
    if (!c) return QSAMP_ERR_INVALID_ARG;
    if (c->aborted) return c->err = "the communicator was aborted: destroy it and create a new one", QSAMP_ERR_COMM;
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != c->device) cudaSetDevice(c->device);
    const qsamp_status s = wait_real(c, true, (cudaStream_t)stream, "the stream's work");
    if (prev != c->device) cudaSetDevice(prev);
    return s;
}

qsamp_status qsamp_comm_status(const qsamp_comm* c) {
    if (!c) return QSAMP_ERR_INVALID_ARG;
    return c->aborted ? QSAMP_ERR_COMM : QSAMP_OK;
}

const char* qsamp_comm_last_error(const qsamp_comm* c) { return c ? c->err.c_str() : "no communicator"; }

void qsamp_comm_destroy(qsamp_comm* c) {
    if (!c) return;
    if (c->comm) {
        int prev = 0;
        cudaGetDevice(&prev);
        if (prev != c->device) cudaSetDevice(c->device);
        // (an orderly finalize would wait on the peers; abort does not)
        ncclCommAbort(c->comm);
        if (prev != c->device) cudaSetDevice(prev);
    }
    delete c;
}

qsamp_status qsamp_comm_selftest(int32_t scenario, int64_t timeout_ms, int32_t* aborted) {
    if (scenario < 0 || scenario > 2 || timeout_ms <= 0 || !aborted) return QSAMP_ERR_INVALID_ARG;
    struct Fake {
        int scenario, polls, aborts;
    } f{scenario, 0, 0};
    WaitOps ops{
        [](void* h, ncclResult_t* out) -> ncclResult_t {
            Fake* x = static_cast<Fake*>(h);
            ++x->polls;
            *out = (x->scenario == 1 && x->polls >= 3) ? ncclRemoteError : ncclSuccess;
            return ncclSuccess;
        },
        [](void* h) -> int {
            const Fake* x = static_cast<Fake*>(h);
            return (x->scenario == 2 && x->polls >= 3) ? 1 : 0;
        },
        [](void* h) { ++static_cast<Fake*>(h)->aborts; },
        &f};
    ncclResult_t nerr = ncclSuccess;
    const WaitResult r = bounded_wait(ops, timeout_ms, &nerr);
    *aborted = f.aborts;
    return r == W_DONE ? QSAMP_OK : (r == W_TIMEOUT ? QSAMP_ERR_TIMEOUT : QSAMP_ERR_COMM);
}

}  // extern "C"
