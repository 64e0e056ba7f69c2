// Drives the bounded NCCL helpers (cuda-llm-inference-engine_b200/csrc/nccl_bounded.h) with
// fake NCCL functions on the host; built and run by tests/test_nccl_bounded_cpu.py.
// Prints one line per scenario: "<name> <b2 status> <aborted> <seconds>".
#include <chrono>
#include <cstdio>

#include "nccl_bounded.h"

namespace {
int g_polls_left = 0;      // GetAsyncError answers ncclInProgress this many times (-1: forever)
ncclResult_t g_init = ncclSuccess;
ncclResult_t g_final = ncclSuccess;
int g_aborted = 0;
int g_blocking_seen = -1;
char g_comm_storage;

int g_destroyed = 0;

struct FakeApi {
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
    ncclResult_t (*GetAsyncError)(ncclComm_t, ncclResult_t*);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*CommFinalize)(ncclComm_t);
    ncclResult_t (*CommDestroy)(ncclComm_t);
};

ncclResult_t fake_init(ncclComm_t* comm, int, ncclUniqueId, int, ncclConfig_t* cfg) {
    g_blocking_seen = cfg->blocking;
    *comm = reinterpret_cast<ncclComm_t>(&g_comm_storage);
    return g_init;
}
ncclResult_t fake_async(ncclComm_t, ncclResult_t* state) {
    if (g_polls_left != 0) {
        if (g_polls_left > 0) --g_polls_left;
        *state = ncclInProgress;
    } else {
        *state = g_final;
    }
    return ncclSuccess;
}
ncclResult_t fake_abort(ncclComm_t) {
    ++g_aborted;
    return ncclSuccess;
}
ncclResult_t fake_finalize(ncclComm_t) { return ncclInProgress; }
ncclResult_t fake_destroy(ncclComm_t) {
    ++g_destroyed;
    return ncclSuccess;
}

void run_init(const char* name, int polls, ncclResult_t init, ncclResult_t fin, double timeout_s) {
    g_polls_left = polls;
    g_init = init;
    g_final = fin;
    g_aborted = 0;
    FakeApi api{fake_init, fake_async, fake_abort, fake_finalize, fake_destroy};
    ncclComm_t comm = nullptr;
    ncclUniqueId id{};
    const auto t0 = std::chrono::steady_clock::now();
    const int st = b2::comm_init_bounded(api, &comm, 2, id, 0, timeout_s);
    const std::chrono::duration<double> dt = std::chrono::steady_clock::now() - t0;
    printf("%s %d %d %.3f %d %d\n", name, st, g_aborted, dt.count(), comm != nullptr ? 1 : 0, g_blocking_seen);
}
}  // namespace

int main() {
    run_init("joins_after_polls", 5, ncclInProgress, ncclSuccess, 2.0);
    run_init("never_joins", -1, ncclInProgress, ncclSuccess, 0.3);
    run_init("init_error", 0, ncclInvalidArgument, ncclSuccess, 2.0);
    run_init("async_error", 3, ncclInProgress, ncclRemoteError, 2.0);
    // an enqueue answered with ncclInProgress: waited out, or a timeout if it never settles
    FakeApi api{fake_init, fake_async, fake_abort, fake_finalize, fake_destroy};
    ncclComm_t comm = reinterpret_cast<ncclComm_t>(&g_comm_storage);
    g_polls_left = 4;
    g_final = ncclSuccess;
    printf("enqueue_in_progress %d\n", b2::nccl_call_bounded(api, comm, [] { return ncclInProgress; }, 2.0));
    g_polls_left = -1;
    printf("enqueue_stuck %d\n", b2::nccl_call_bounded(api, comm, [] { return ncclInProgress; }, 0.2));
    printf("enqueue_error %d\n", b2::nccl_call_bounded(api, comm, [] { return ncclSystemError; }, 0.2));
    // teardown: quiescent after a few polls -> destroyed; never quiescent -> aborted
    g_polls_left = 3;
    g_aborted = g_destroyed = 0;
    int st = b2::comm_destroy_bounded(api, comm, 2.0);
    printf("destroy_quiescent %d %d %d\n", st, g_destroyed, g_aborted);
    g_polls_left = -1;
    g_aborted = g_destroyed = 0;
    st = b2::comm_destroy_bounded(api, comm, 0.2);
    printf("destroy_peer_gone %d %d %d\n", st, g_destroyed, g_aborted);
    return 0;
}
