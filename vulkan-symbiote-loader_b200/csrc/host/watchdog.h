// Bounded host waits on work that depends on other tensor-parallel ranks.
//
// NCCL's kernels wait for their peers without a time limit, so a rank that died or never
// reaches a collective would leave the others' streams waiting for good. The engine never
// blocks on such a stream directly: it polls the stream, watches the communicator's
// asynchronous error, and aborts the communicator (ncclCommAbort makes NCCL's kernels give
// up, so the stream drains and the CUDA context stays usable) when the communicator reports
// an error or the wait passes its deadline. The reference declares an ErrorHandler /
// RecoveryAction pair for this role and never uses it
// (vk_symbiote/include/vk_symbiote/Common.h:251-282); here the recovery is fixed: the engine
// reports the failure and must be recreated.
//
// The logic is written over callables so that it is tested on the host with fakes of the
// stream and the communicator (tests/cpp/watchdog_check.cpp).
#pragma once

#include "../../../include/vsl.h"

namespace vsl {

enum class StreamPoll { Done, Pending, Error };

// query(): state of the awaited stream; comm_failed(): true once the communicator reports an
// asynchronous error; abort(): abort the communicator (called at most once); now(): seconds
// on a monotonic clock; pause(): called between polls. Returns VSL_OK when the stream
// finished, VSL_ERR_CUDA when it failed, VSL_ERR_NCCL when the communicator failed (after
// aborting it) and VSL_ERR_TIMEOUT after timeout_s seconds (after aborting it).
template <class Query, class CommFailed, class Abort, class Now, class Pause>
int watched_wait(Query query, CommFailed comm_failed, Abort abort, double timeout_s, Now now, Pause pause) {
    const double t0 = now();
    for (unsigned long long it = 0;; it++) {
        const StreamPoll p = query();
        if (p == StreamPoll::Done) return VSL_OK;
        if (p == StreamPoll::Error) return VSL_ERR_CUDA;
        // the communicator and the clock are checked every 64 polls: a poll of a finished
        // stream must stay cheap on the decode path
        if ((it & 63) == 63) {
            if (comm_failed()) {
                abort();
                return VSL_ERR_NCCL;
            }
            if (now() - t0 > timeout_s) {
                abort();
                return VSL_ERR_TIMEOUT;
            }
        }
        pause(it);
    }
}

}  // namespace vsl
