// Host logic of the bounded tensor-parallel wait (vulkan-symbiote-loader_b200/csrc/host/watchdog.h),
// driven with fakes of the stream, the communicator and the clock; built by tests/test_watchdog.py
// (no GPU). Prints one line per case: "<case> ok" or "<case> FAIL ...".
#include <cstdio>

#include "watchdog.h"

using vsl::StreamPoll;
using vsl::watched_wait;

struct Fake {
    int done_after = -1;       // the stream finishes at this poll (-1: never)
    int error_at = -1;         // the stream reports a CUDA error at this poll
    int comm_error_at = -1;    // the communicator reports an asynchronous error from this poll on
    double seconds_per_poll = 0.001;
    int polls = 0, aborts = 0, comm_checks = 0;
    double clock = 0.0;
    int run(double timeout) {
        return watched_wait(
            [&] {
                const int p = polls++;
                clock += seconds_per_poll;
                if (error_at >= 0 && p >= error_at) return StreamPoll::Error;
                if (done_after >= 0 && p >= done_after) return StreamPoll::Done;
                return StreamPoll::Pending;
            },
            [&] {
                comm_checks++;
                return comm_error_at >= 0 && polls > comm_error_at;
            },
            [&] { aborts++; }, timeout, [&] { return clock; }, [](unsigned long long) {});
    }
};

static int failures = 0;
static void expect(const char* name, bool ok, const Fake& f, int rc) {
    if (ok) {
        printf("%s ok\n", name);
    } else {
        printf("%s FAIL rc=%d polls=%d aborts=%d comm_checks=%d\n", name, rc, f.polls, f.aborts, f.comm_checks);
        failures++;
    }
}

int main() {
    {  // a finished stream returns at once, without touching the communicator
        Fake f;
        f.done_after = 0;
        int rc = f.run(1.0);
        expect("finished", rc == VSL_OK && f.polls == 1 && f.aborts == 0 && f.comm_checks == 0, f, rc);
    }
    {  // work that ends within the bound
        Fake f;
        f.done_after = 500;
        int rc = f.run(1.0);
        expect("finishes_in_time", rc == VSL_OK && f.polls == 501 && f.aborts == 0, f, rc);
    }
    {  // a peer never arrives: the deadline aborts the communicator once
        Fake f;
        int rc = f.run(0.5);
        expect("deadline_aborts", rc == VSL_ERR_TIMEOUT && f.aborts == 1 && f.polls >= 500 && f.polls <= 600, f, rc);
    }
    {  // NCCL reports an asynchronous error before the deadline
        Fake f;
        f.comm_error_at = 100;
        int rc = f.run(60.0);
        expect("comm_error_aborts", rc == VSL_ERR_NCCL && f.aborts == 1 && f.polls <= 200, f, rc);
    }
    {  // a failing stream is a CUDA error, and the communicator is left alone
        Fake f;
        f.error_at = 10;
        int rc = f.run(60.0);
        expect("stream_error", rc == VSL_ERR_CUDA && f.aborts == 0, f, rc);
    }
    {  // a stream that finishes just as the communicator fails is still a success
        Fake f;
        f.done_after = 63;
        f.comm_error_at = 0;
        int rc = f.run(60.0);
        expect("done_wins", rc == VSL_OK && f.aborts == 0, f, rc);
    }
    return failures ? 1 : 0;
}
