// CPU check of the host wait that libmoe_cuda.so runs for a step whose stream
// holds NCCL kernels (flash_deepseek_b200/csrc/moe_wait.h), against fakes of
// the stream query, the communicator's asynchronous error and its abort.
// Prints one line per scenario: outcome, query calls, aborts.
#include <cstdio>

#include "../flash_deepseek_b200/csrc/moe_wait.h"

struct Fake {
    int done_after;   // query reports "finished" on this call (-1: never)
    int error_at;     // query reports an error on this call (-1: never)
    int nccl_err_at;  // the communicator reports an error on this poll (-1: never)
    int queries = 0, polls = 0, aborts = 0;
};

static void run(const char *name, Fake f, double limit) {
    const MoeWaitOutcome o = moe_wait_poll(
        [&]() {
            f.queries++;
            if (f.error_at >= 0 && f.queries >= f.error_at) return 2;
            return (f.done_after >= 0 && f.queries >= f.done_after) ? 0 : 1;
        },
        [&]() { return f.nccl_err_at >= 0 && ++f.polls >= f.nccl_err_at; },
        [&]() { f.aborts++; }, limit);
    printf("%s outcome=%d queries=%d aborts=%d\n", name, (int)o, f.queries, f.aborts);
}

int main() {
    run("finishes", Fake{5, -1, -1}, 10.0);
    run("stream_error", Fake{-1, 3, -1}, 10.0);
    run("nccl_error", Fake{-1, -1, 4}, 10.0);
    run("timeout", Fake{-1, -1, -1}, 0.2);
    return 0;
}
