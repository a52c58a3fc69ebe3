// comm.cu -- the engine's NCCL communicator, with bounded host waits.
//
// A partitioned network exchanges spikes with one NCCL all-gather per
// window.  Left alone, any rank that dies, stops early or disagrees on the
// exchange layout would hang every other rank inside NCCL.  Here every host
// wait on the communicator polls with a time limit: its set-up (run on a
// helper thread, since the communicator is blocking so that its
// collectives can be captured in CUDA graphs), a call that returns
// ncclInProgress, and the engine stream of a partitioned run (polling
// cudaStreamQuery and ncclCommGetAsyncError).  On an NCCL error or a
// timeout the communicator is aborted on a helper thread (ncclCommAbort
// ends the NCCL kernels still waiting for a peer) and the call returns
// NRN_ERR_COMM; the engine then refuses further runs.  The reference has no
// counterpart: its runner is single-device (src/simulation/runner.cpp).
#include <cuda_runtime.h>
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <memory>
#include <string>
#include <thread>

#include "common.cuh"
#include "internal.h"

namespace nrn {
namespace {

// An error code that the next query of a communicator's asynchronous state
// reports instead of NCCL's own (nrn_comm_fake_async_error; tests only).
std::atomic<int> g_fake_async{0};

ncclResult_t async_state(ncclComm_t c) {
    const int f = g_fake_async.exchange(0);
    if (f != 0) return static_cast<ncclResult_t>(f);
    ncclResult_t st = ncclSuccess;
    const ncclResult_t r = ncclCommGetAsyncError(c, &st);
    return r != ncclSuccess ? r : st;
}

struct AsyncPoll {
    ncclComm_t comm;
    ncclResult_t last = ncclSuccess;
};

int poll_async(void* ctx) {
    auto* p = static_cast<AsyncPoll*>(ctx);
    p->last = async_state(p->comm);
    if (p->last == ncclSuccess) return 1;
    if (p->last == ncclInProgress) return 0;
    return -1;
}

struct StreamPoll {
    ncclComm_t comm;
    cudaStream_t stream;
    ncclResult_t nccl = ncclSuccess;
    cudaError_t cuda = cudaSuccess;
};

int poll_stream(void* ctx) {
    auto* p = static_cast<StreamPoll*>(ctx);
    p->cuda = cudaStreamQuery(p->stream);
    if (p->cuda == cudaSuccess) {
        // the stream is done; an error the NCCL proxy saw meanwhile still counts
        p->nccl = async_state(p->comm);
        return p->nccl == ncclSuccess || p->nccl == ncclInProgress ? 1 : -1;
    }
    if (p->cuda != cudaErrorNotReady) return -1;
    p->nccl = async_state(p->comm);
    return p->nccl == ncclSuccess || p->nccl == ncclInProgress ? 0 : -1;
}

}  // namespace

// Aborts the communicator on a helper thread, waiting for it at most
// kAbortWait seconds: an abort that does not end (it may wait on peers) is
// abandoned, the communicator being unusable either way.
constexpr double kAbortWait = 30.0;

nrn_status_t comm_abort(ncclComm_t* c) {
    if (*c == nullptr) return NRN_OK;
    struct Job {
        ncclComm_t comm;
        std::atomic<bool> done{false};
    };
    auto job = std::make_shared<Job>();
    job->comm = *c;
    *c = nullptr;
    int dev = 0;
    cudaGetDevice(&dev);
    std::thread([job, dev] {
        cudaSetDevice(dev);
        ncclCommAbort(job->comm);
        job->done.store(true);
    }).detach();
    nrn_comm_bounded_wait([](void* ctx) -> int { return static_cast<Job*>(ctx)->done.load() ? 1 : 0; }, job.get(),
                          kAbortWait);
    return NRN_OK;
}

nrn_status_t comm_init(ncclComm_t* out, int world, const uint8_t id[128], int rank, double timeout_s) {
    // The communicator is blocking (its collectives are captured in CUDA
    // graphs like any kernel launch); its set-up, which waits for every
    // rank, runs on a helper thread so that the wait is bounded.  A set-up
    // that times out is left to finish or fail on its own: its thread and
    // communicator are abandoned.
    struct Job {
        ncclComm_t comm = nullptr;
        ncclResult_t r = ncclSuccess;
        std::atomic<bool> done{false};
    };
    auto job = std::make_shared<Job>();
    ncclUniqueId u;
    static_assert(sizeof(u) == 128, "NCCL unique id size");
    std::memcpy(&u, id, sizeof(u));
    int dev = 0;
    cudaGetDevice(&dev);
    std::thread([job, u, world, rank, dev] {
        cudaSetDevice(dev);
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 1;
        ncclComm_t c = nullptr;
        job->r = ncclCommInitRankConfig(&c, world, u, rank, &cfg);
        job->comm = c;
        job->done.store(true);
    }).detach();
    const nrn_status_t st = nrn_comm_bounded_wait(
        [](void* ctx) -> int { return static_cast<Job*>(ctx)->done.load() ? 1 : 0; }, job.get(), timeout_s);
    if (st != NRN_OK)
        return fail(NRN_ERR_COMM, "NCCL communicator set-up timed out after " + std::to_string(timeout_s) +
                                      " s: every rank must call nrn_engine_set_partition with the same id");
    if (job->r != ncclSuccess) {
        ncclComm_t c = job->comm;
        comm_abort(&c);
        return fail(NRN_ERR_COMM, std::string("NCCL communicator set-up: ") + ncclGetErrorString(job->r));
    }
    *out = job->comm;
    return NRN_OK;
}

nrn_status_t comm_settle(ncclComm_t* c, ncclResult_t r, double timeout_s, const char* what) {
    if (r == ncclSuccess) return NRN_OK;
    if (r == ncclInProgress) {
        AsyncPoll p{*c};
        const nrn_status_t st = nrn_comm_bounded_wait(poll_async, &p, timeout_s);
        if (st == NRN_OK) return NRN_OK;
        r = p.last;
        comm_abort(c);
        if (st == NRN_ERR_TIMEOUT)
            return fail(NRN_ERR_COMM, std::string(what) + ": timed out; communicator aborted");
        return fail(NRN_ERR_COMM, std::string(what) + ": " + ncclGetErrorString(r) + "; communicator aborted");
    }
    comm_abort(c);
    return fail(NRN_ERR_COMM, std::string(what) + ": " + ncclGetErrorString(r) + "; communicator aborted");
}

nrn_status_t comm_wait_stream(ncclComm_t* c, cudaStream_t s, double timeout_s, bool* stuck) {
    if (stuck) *stuck = false;
    StreamPoll p{*c, s};
    const nrn_status_t st = nrn_comm_bounded_wait(poll_stream, &p, timeout_s);
    if (st == NRN_OK) return NRN_OK;
    if (p.cuda != cudaSuccess && p.cuda != cudaErrorNotReady) return cuda_fail(p.cuda, "engine stream");
    comm_abort(c);
    // The aborted NCCL kernels end and the rest of the stream's work drains;
    // that wait is bounded too (a stream still busy then is reported, and the
    // engine then skips every later wait on it).
    StreamPoll q{nullptr, s};
    const nrn_status_t drained = nrn_comm_bounded_wait(
        [](void* ctx) -> int {
            auto* p = static_cast<StreamPoll*>(ctx);
            p->cuda = cudaStreamQuery(p->stream);
            return p->cuda == cudaSuccess ? 1 : p->cuda == cudaErrorNotReady ? 0 : -1;
        },
        &q, timeout_s < 30.0 ? timeout_s : 30.0);
    cudaGetLastError();
    if (stuck) *stuck = drained != NRN_OK;
    if (st == NRN_ERR_TIMEOUT)
        return fail(NRN_ERR_COMM, "partitioned run: the spike exchange did not complete within " +
                                      std::to_string(timeout_s) +
                                      " s (a rank stopped, ran other step counts or failed); communicator aborted");
    return fail(NRN_ERR_COMM, std::string("partitioned run: NCCL reported ") + ncclGetErrorString(p.nccl) +
                                  "; communicator aborted");
}

nrn_status_t comm_destroy(ncclComm_t* c, double timeout_s) {
    // Called with nothing of this communicator in flight (the engine stream
    // was drained, within the time limit, before).  Its teardown may wait
    // for peers that already left: it runs on a helper thread, and one that
    // does not end in time is abandoned.
    if (*c == nullptr) return NRN_OK;
    struct Job {
        ncclComm_t comm;
        std::atomic<bool> done{false};
    };
    auto job = std::make_shared<Job>();
    job->comm = *c;
    *c = nullptr;
    int dev = 0;
    cudaGetDevice(&dev);
    std::thread([job, dev] {
        cudaSetDevice(dev);
        ncclCommDestroy(job->comm);
        job->done.store(true);
    }).detach();
    nrn_comm_bounded_wait([](void* ctx) -> int { return static_cast<Job*>(ctx)->done.load() ? 1 : 0; }, job.get(),
                          timeout_s);
    return NRN_OK;
}

}  // namespace nrn

extern "C" nrn_status_t nrn_comm_bounded_wait(int (*poll)(void*), void* ctx, double timeout_s) {
    using namespace nrn;
    NRN_CHECK_ARG(poll != nullptr, "nrn_comm_bounded_wait: null poll function");
    NRN_CHECK_ARG(timeout_s >= 0.0, "nrn_comm_bounded_wait: negative timeout");
    const auto t0 = std::chrono::steady_clock::now();
    // spin briefly (a window exchange completes in tens of microseconds),
    // then sleep between polls
    for (long k = 0;; ++k) {
        const int r = poll(ctx);
        if (r > 0) return NRN_OK;
        if (r < 0) return fail(NRN_ERR_COMM, "nrn_comm_bounded_wait: the polled operation failed");
        const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el >= timeout_s) return fail(NRN_ERR_TIMEOUT, "nrn_comm_bounded_wait: timed out");
        if (k > 2000) std::this_thread::sleep_for(std::chrono::microseconds(k > 20000 ? 1000 : 50));
    }
}

extern "C" nrn_status_t nrn_comm_fake_async_error(int32_t nccl_result) {
    nrn::g_fake_async.store(nccl_result);
    return NRN_OK;
}
