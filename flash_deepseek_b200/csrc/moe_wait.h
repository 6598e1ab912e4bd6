// moe_wait.h -- the host-side wait of libmoe_cuda.so for a step whose stream
// holds NCCL kernels (the expert-parallel prefill, and the decode exchange
// when the peers could not be mapped).  NCCL's kernels have no bounded wait,
// so the host polls instead of blocking: it queries the stream, checks the
// communicator's asynchronous error, and after a time limit (or on such an
// error) aborts the communicator, which ends its kernels.
//
// The policy is a template over the three calls it makes, so that it runs
// unchanged against fakes on a machine without a GPU (tests/wait_policy.cc).
#pragma once
#include <chrono>
#include <thread>

enum MoeWaitOutcome {
    MOE_WAIT_DONE = 0,     // the stream finished
    MOE_WAIT_STREAM_ERROR, // the stream query reported an error (not "not ready")
    MOE_WAIT_NCCL_ERROR,   // the communicator reported an asynchronous error: aborted
    MOE_WAIT_TIMEOUT,      // the limit passed first: aborted
};

// query():      0 = finished, 1 = not ready, any other value = error
// async_err():  true when the communicator holds an asynchronous error
// abort_comm(): aborts the communicator (called at most once)
template <typename Query, typename AsyncErr, typename Abort>
MoeWaitOutcome moe_wait_poll(Query &&query, AsyncErr &&async_err, Abort &&abort_comm, double limit_s) {
    const auto t0 = std::chrono::steady_clock::now();
    for (unsigned it = 0;; it++) {
        const int q = query();
        if (q == 0) return MOE_WAIT_DONE;
        if (q != 1) return MOE_WAIT_STREAM_ERROR;
        const bool nccl_err = async_err();
        const double waited = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (nccl_err || waited > limit_s) {
            abort_comm();
            return nccl_err ? MOE_WAIT_NCCL_ERROR : MOE_WAIT_TIMEOUT;
        }
        if (it < 1000) std::this_thread::yield();
        else std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}
