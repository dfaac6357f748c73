// Communicators for the tensor-parallel o_proj exchange: NCCL behind the C ABI, with failure
// detection.
//
// The reference runs every layer on one device (QwenRunner.cpp:236,328) and has no collective.
// Sharding attention by KV-head group (tensor parallel) makes o_proj (Attention.h:322-325) a sum
// of per-rank partials, and these entry points carry that sum -- and the all-gather of the
// sequence-parallel form of the same exchange -- between the ranks' processes over NVLink.
//
// Failure detection.  Every communicator is created non-blocking (ncclConfig_t.blocking = 0), so
// no NCCL call can block the host indefinitely, and gets a watchdog thread (comm_watchdog.h).
// Each collective is tracked by an event recorded behind it; the thread polls every 5 ms for an
// asynchronous NCCL error and for a collective that has run past the communicator's deadline,
// and aborts the communicator (ncclCommAbort, which ends its kernels) in either case.  From then
// on every call on it returns MLLM_ERR_COMM (an asynchronous error, or an abort on request) or
// MLLM_ERR_COMM_TIMEOUT, and the caller rebuilds its communicator.  Set-up and tear-down are
// bounded by the same deadline.  Collectives enqueued while the stream is being captured into a
// CUDA graph are not tracked (they run when the graph is launched), and the watchdog's own
// queries run in relaxed capture mode, so they never invalidate a graph being recorded.
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include "comm_watchdog.h"
#include "host_util.h"

struct mllm_comm;

namespace mllm_b200 {
namespace {

double now_s() {
    using namespace std::chrono;
    return duration<double>(steady_clock::now().time_since_epoch()).count();
}

// The watchdog's view of one communicator (see comm_watchdog.h for the contract).
struct NcclOps {
    using Event = cudaEvent_t;
    mllm_comm* c;
    int async_error();
    bool done(cudaEvent_t e) { return cudaEventQuery(e) != cudaErrorNotReady; }
    void release(cudaEvent_t e);
    void abort();
    double now() { return now_s(); }
};

}  // namespace
}  // namespace mllm_b200

using namespace mllm_b200;

struct mllm_comm {
    ncclComm_t nccl = nullptr;
    int device = 0, rank = 0, nranks = 0;
    double timeout_s = 0;
    std::atomic<bool> aborted{false};
    std::unique_ptr<CommWatchdog<NcclOps>> wd;
    std::thread thread;
    std::atomic<bool> stop{false};
    std::mutex pool_mu;
    std::vector<cudaEvent_t> pool;   // idle events
    std::vector<cudaEvent_t> all;    // every event created, destroyed at the end
};

namespace mllm_b200 {
namespace {

int NcclOps::async_error() {
    if (c->aborted.load()) return 2;
    ncclResult_t r = ncclSuccess;
    if (ncclCommGetAsyncError(c->nccl, &r) != ncclSuccess) return 2;
    return r == ncclSuccess ? 0 : (r == ncclInProgress ? 1 : 2);
}

void NcclOps::release(cudaEvent_t e) {
    std::lock_guard<std::mutex> lock(c->pool_mu);
    c->pool.push_back(e);
}

void NcclOps::abort() {
    if (!c->aborted.exchange(true)) ncclCommAbort(c->nccl);
}

// Sets the calling thread's stream-capture interaction mode to relaxed for its lifetime: the
// watchdog queries events, which a thread in the default (global) mode may not do while any
// thread records a CUDA graph in global mode -- the query would invalidate that recording.  In
// relaxed mode the query is allowed and the other thread's capture is unaffected.
struct RelaxedCapture {
    cudaStreamCaptureMode prev = cudaStreamCaptureModeRelaxed;
    RelaxedCapture() { cudaThreadExchangeStreamCaptureMode(&prev); }
    ~RelaxedCapture() { cudaThreadExchangeStreamCaptureMode(&prev); }
};

int state_status(CommState s) {
    switch (s) {
        case CommState::kHealthy: return MLLM_OK;
        case CommState::kTimedOut:
            return fail(MLLM_ERR_COMM_TIMEOUT, "communicator aborted: a collective ran past its deadline");
        case CommState::kAsyncError:
            return fail(MLLM_ERR_COMM, "communicator aborted after an asynchronous NCCL error (a peer failed or left)");
        default: return fail(MLLM_ERR_COMM, "communicator was aborted");
    }
}

// Polls a non-blocking communicator until its last call has finished on the host side.
int settle(ncclComm_t comm, double deadline, const char* what) {
    for (;;) {
        ncclResult_t r = ncclSuccess;
        if (ncclCommGetAsyncError(comm, &r) != ncclSuccess) return fail(MLLM_ERR_COMM, std::string(what) + ": NCCL query failed");
        if (r == ncclSuccess) return MLLM_OK;
        if (r != ncclInProgress)
            return fail(MLLM_ERR_COMM, std::string(what) + ": " + ncclGetErrorString(r));
        if (now_s() > deadline) return fail(MLLM_ERR_COMM_TIMEOUT, std::string(what) + ": did not finish in time");
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

int nccl_status(ncclResult_t r, const char* what) {
    if (r == ncclSuccess || r == ncclInProgress) return MLLM_OK;
    return fail(MLLM_ERR_COMM, std::string(what) + ": " + ncclGetErrorString(r));
}

int take_event(mllm_comm* c, cudaEvent_t* e) {
    {
        std::lock_guard<std::mutex> lock(c->pool_mu);
        if (!c->pool.empty()) {
            *e = c->pool.back();
            c->pool.pop_back();
            return MLLM_OK;
        }
    }
    if (int st = check_cuda(cudaEventCreateWithFlags(e, cudaEventDisableTiming), "comm: cudaEventCreate")) return st;
    std::lock_guard<std::mutex> lock(c->pool_mu);
    c->all.push_back(*e);
    return MLLM_OK;
}

// Common tail of every collective: settle the non-blocking call, then track it.
int after_collective(mllm_comm* c, ncclResult_t r, cudaStream_t s, const char* what) {
    if (int st = nccl_status(r, what)) {
        c->wd->abort();
        return st;
    }
    if (r == ncclInProgress) {
        if (int st = settle(c->nccl, now_s() + c->timeout_s, what)) {
            c->wd->abort();
            return st;
        }
    }
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (int st = check_cuda(cudaStreamIsCapturing(s, &cap), "comm: cudaStreamIsCapturing")) return st;
    if (cap != cudaStreamCaptureStatusNone) return ok();
    cudaEvent_t e;
    if (int st = take_event(c, &e)) return st;
    if (int st = check_cuda(cudaEventRecord(e, s), "comm: cudaEventRecord")) {
        NcclOps{c}.release(e);
        return st;
    }
    if (!c->wd->track(e)) return state_status(c->wd->state());
    return ok();
}

int usable(mllm_comm* c) {
    if (!c) return fail(MLLM_ERR_INVALID_ARGUMENT, "comm: null communicator");
    int dev = -1;
    if (int st = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return st;
    if (dev != c->device) return fail(MLLM_ERR_INVALID_ARGUMENT, "comm: the current device is not the communicator's");
    return state_status(c->wd->state());
}

}  // namespace
}  // namespace mllm_b200

extern "C" int mllm_comm_unique_id(void* id) {
    if (!id) return fail(MLLM_ERR_INVALID_ARGUMENT, "comm_unique_id: null pointer");
    static_assert(sizeof(ncclUniqueId) == MLLM_COMM_ID_BYTES, "ncclUniqueId size");
    ncclUniqueId u;
    if (int st = nccl_status(ncclGetUniqueId(&u), "ncclGetUniqueId")) return st;
    memcpy(id, &u, sizeof(u));
    return ok();
}

extern "C" int mllm_comm_init(const void* id, int nranks, int rank, double timeout_s, mllm_comm_t* out) {
    if (!id || !out || nranks < 1 || rank < 0 || rank >= nranks || !(timeout_s > 0))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "comm_init: bad arguments");
    *out = nullptr;
    if (int st = require_sm100()) return st;
    auto c = std::make_unique<mllm_comm>();
    if (int st = check_cuda(cudaGetDevice(&c->device), "cudaGetDevice")) return st;
    c->rank = rank;
    c->nranks = nranks;
    c->timeout_s = timeout_s;
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = ncclCommInitRankConfig(&c->nccl, nranks, u, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) return nccl_status(r, "ncclCommInitRankConfig");
    if (int st = settle(c->nccl, now_s() + timeout_s, "ncclCommInitRankConfig")) {
        ncclCommAbort(c->nccl);
        return st;
    }
    c->wd = std::make_unique<CommWatchdog<NcclOps>>(NcclOps{c.get()}, timeout_s);
    mllm_comm* raw = c.get();
    c->thread = std::thread([raw] {
        cudaSetDevice(raw->device);
        RelaxedCapture relaxed;   // never disturbs a graph recorded by another thread
        while (!raw->stop.load()) {
            raw->wd->poll();
            std::this_thread::sleep_for(std::chrono::milliseconds(5));
        }
    });
    *out = c.release();
    return ok();
}

extern "C" int mllm_comm_all_reduce_bf16(mllm_comm_t comm, const void* send, void* recv, size_t count,
                                         mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_comm_all_reduce_bf16");
    if (int st = usable(comm)) return st;
    if (count == 0) return ok();
    if (!send || !recv) return fail(MLLM_ERR_INVALID_ARGUMENT, "comm_all_reduce: null buffer");
    cudaStream_t s = (cudaStream_t)stream;
    ncclResult_t r = ncclAllReduce(send, recv, count, ncclBfloat16, ncclSum, comm->nccl, s);
    return after_collective(comm, r, s, "ncclAllReduce");
}

extern "C" int mllm_comm_all_gather_bf16(mllm_comm_t comm, const void* send, void* recv, size_t send_count,
                                         mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_comm_all_gather_bf16");
    if (int st = usable(comm)) return st;
    if (send_count == 0) return ok();
    if (!send || !recv) return fail(MLLM_ERR_INVALID_ARGUMENT, "comm_all_gather: null buffer");
    cudaStream_t s = (cudaStream_t)stream;
    ncclResult_t r = ncclAllGather(send, recv, send_count, ncclBfloat16, comm->nccl, s);
    return after_collective(comm, r, s, "ncclAllGather");
}

extern "C" int mllm_comm_status(mllm_comm_t comm) {
    if (!comm) return fail(MLLM_ERR_INVALID_ARGUMENT, "comm_status: null communicator");
    RelaxedCapture relaxed;
    if (int st = state_status(comm->wd->poll())) return st;
    return ok();
}

extern "C" int mllm_comm_in_flight(mllm_comm_t comm) {
    if (!comm) return -1;
    return (int)comm->wd->in_flight();
}

extern "C" int mllm_comm_abort(mllm_comm_t comm) {
    if (!comm) return fail(MLLM_ERR_INVALID_ARGUMENT, "comm_abort: null communicator");
    comm->wd->abort();
    return ok();
}

extern "C" int mllm_comm_destroy(mllm_comm_t comm) {
    if (!comm) return ok();
    std::unique_ptr<mllm_comm> c(comm);
    c->stop.store(true);
    if (c->thread.joinable()) c->thread.join();
    int st = MLLM_OK;
    if (c->wd->state() == CommState::kHealthy) {
        // finish the queued collectives, then free; abort if that does not end in time
        ncclResult_t r = ncclCommFinalize(c->nccl);
        st = nccl_status(r, "ncclCommFinalize");
        if (st == MLLM_OK) st = settle(c->nccl, now_s() + c->timeout_s, "ncclCommFinalize");
        if (st == MLLM_OK) {
            st = nccl_status(ncclCommDestroy(c->nccl), "ncclCommDestroy");
        } else {
            c->wd->abort();
        }
    }
    for (cudaEvent_t e : c->all) cudaEventDestroy(e);
    return st == MLLM_OK ? ok() : st;
}
