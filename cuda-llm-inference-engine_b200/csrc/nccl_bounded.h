// Bounded NCCL host calls for the tensor-parallel engine.
//
// A communicator made with ncclCommInitRank blocks until every rank has joined, so one rank
// that never starts hangs the others forever. Here the communicator is created in NCCL's
// non-blocking mode (ncclConfig_t.blocking = 0): ncclCommInitRankConfig returns at once,
// and the caller polls ncclCommGetAsyncError until the state leaves ncclInProgress or a
// deadline passes; on a timeout or an error the half-made communicator is aborted
// (ncclCommAbort) and the engine reports B2_ERR_TIMEOUT / B2_ERR_CUDA instead of hanging.
// In non-blocking mode any later NCCL call may also return ncclInProgress while it is
// being enqueued; nccl_call_bounded waits for those with the same bound.
//
// Header-only and templated on the function table, so a host test can drive it with fake
// NCCL functions (no GPU, no NCCL library).
#pragma once
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <thread>

#include "b2decode.h"

namespace b2 {

// Seconds a rank waits for its peers (creation, or an enqueue that stays in progress);
// B2_NCCL_TIMEOUT_S overrides the default.
inline double nccl_timeout_s() {
    const char* env = getenv("B2_NCCL_TIMEOUT_S");
    const double v = env ? atof(env) : 0.0;
    return v > 0.0 ? v : 300.0;
}

// Polls the communicator's asynchronous state until it is not ncclInProgress or
// `timeout_s` passes. Returns the state (ncclInProgress on a timeout).
template <class Api>
ncclResult_t nccl_wait_ready(const Api& api, ncclComm_t comm, double timeout_s) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t state = ncclInProgress;
        const ncclResult_t r = api.GetAsyncError(comm, &state);
        if (r != ncclSuccess) return r;
        if (state != ncclInProgress) return state;
        const std::chrono::duration<double> waited = std::chrono::steady_clock::now() - t0;
        if (waited.count() > timeout_s) return ncclInProgress;
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

// Creates rank `rank` of a `world`-rank communicator in non-blocking mode and waits for it
// with a bound. On success *comm is ready; otherwise the communicator is aborted, *comm is
// null and the result is B2_ERR_TIMEOUT (a peer did not join in time) or B2_ERR_CUDA.
template <class Api>
int comm_init_bounded(const Api& api, ncclComm_t* comm, int world, ncclUniqueId id, int rank, double timeout_s) {
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    *comm = nullptr;
    ncclResult_t r = api.CommInitRankConfig(comm, world, id, rank, &cfg);
    if (r == ncclSuccess || r == ncclInProgress) r = *comm ? nccl_wait_ready(api, *comm, timeout_s) : ncclInternalError;
    if (r == ncclSuccess) return B2_OK;
    if (*comm) api.CommAbort(*comm);
    *comm = nullptr;
    return r == ncclInProgress ? B2_ERR_TIMEOUT : B2_ERR_CUDA;
}

// Issues one NCCL call on a non-blocking communicator; an ncclInProgress answer is waited
// out with the bound. B2_OK once the operation is enqueued, B2_ERR_TIMEOUT if it stays in
// progress, B2_ERR_CUDA on an NCCL error.
template <class Api, class Call>
int nccl_call_bounded(const Api& api, ncclComm_t comm, Call&& call, double timeout_s) {
    ncclResult_t r = call();
    if (r == ncclInProgress) r = nccl_wait_ready(api, comm, timeout_s);
    if (r == ncclSuccess) return B2_OK;
    return r == ncclInProgress ? B2_ERR_TIMEOUT : B2_ERR_CUDA;
}

// Tears a non-blocking communicator down: ncclCommFinalize flushes its operations, the
// state is polled until the communicator is quiescent, then ncclCommDestroy frees it; if
// that does not happen within the bound (a peer is gone), ncclCommAbort frees it instead.
// Returns B2_OK, or B2_ERR_TIMEOUT / B2_ERR_CUDA after an abort.
template <class Api>
int comm_destroy_bounded(const Api& api, ncclComm_t comm, double timeout_s) {
    if (!comm) return B2_OK;
    ncclResult_t r = api.CommFinalize(comm);
    if (r == ncclSuccess || r == ncclInProgress) r = nccl_wait_ready(api, comm, timeout_s);
    if (r == ncclSuccess) return api.CommDestroy(comm) == ncclSuccess ? B2_OK : B2_ERR_CUDA;
    api.CommAbort(comm);
    return r == ncclInProgress ? B2_ERR_TIMEOUT : B2_ERR_CUDA;
}

}  // namespace b2
