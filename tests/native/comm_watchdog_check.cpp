// CPU check of the communicator watchdog (mllm_b200/csrc/comm_watchdog.h) against fake NCCL and
// CUDA operations: a clock the test moves by hand, events the test completes, an asynchronous
// error the test raises, and a counter of aborts.  Prints one "name ok" line per scenario and
// exits nonzero on the first failure.  Built and run by tests/test_comm_watchdog.py.
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <set>
#include <thread>
#include <vector>

#include "comm_watchdog.h"

using mllm_b200::CommState;
using mllm_b200::CommWatchdog;

struct Fake {
    std::atomic<double> clock{0.0};
    std::atomic<int> error{0};
    std::atomic<int> aborts{0};
    std::set<int> done;       // completed events
    std::set<int> released;   // events returned to the pool
    std::mutex mu;
};

struct FakeOps {
    using Event = int;
    Fake* f;
    int async_error() { return f->error.load(); }
    bool done(int e) {
        std::lock_guard<std::mutex> l(f->mu);
        return f->done.count(e) > 0;
    }
    void release(int e) {
        std::lock_guard<std::mutex> l(f->mu);
        f->released.insert(e);
    }
    void abort() { f->aborts++; }
    double now() { return f->clock.load(); }
};

#define CHECK(c)                                                        \
    do {                                                                \
        if (!(c)) {                                                     \
            std::printf("FAIL %s:%d %s\n", __FILE__, __LINE__, #c);     \
            std::exit(1);                                               \
        }                                                               \
    } while (0)

static void complete(Fake& f, int e) {
    std::lock_guard<std::mutex> l(f.mu);
    f.done.insert(e);
}

int main() {
    {   // collectives that complete in time leave the communicator healthy
        Fake f;
        CommWatchdog<FakeOps> wd(FakeOps{&f}, 2.0);
        CHECK(wd.track(1) && wd.track(2) && wd.track(3));
        f.clock = 1.0;
        complete(f, 1);
        complete(f, 2);
        CHECK(wd.poll() == CommState::kHealthy);
        CHECK(wd.in_flight() == 1);
        complete(f, 3);
        f.clock = 10.0;   // long after, but nothing is pending any more
        CHECK(wd.poll() == CommState::kHealthy && wd.in_flight() == 0);
        CHECK(f.aborts == 0 && f.released.size() == 3);
        std::printf("healthy ok\n");
    }
    {   // a collective that never completes (a peer that never joins) is aborted at the deadline
        Fake f;
        CommWatchdog<FakeOps> wd(FakeOps{&f}, 2.0);
        CHECK(wd.track(7));
        f.clock = 1.9;
        CHECK(wd.poll() == CommState::kHealthy);
        f.clock = 2.1;
        CHECK(wd.poll() == CommState::kTimedOut);
        CHECK(f.aborts == 1 && f.released.count(7) == 1 && wd.in_flight() == 0);
        CHECK(wd.poll() == CommState::kTimedOut && f.aborts == 1);   // aborts once, stays aborted
        CHECK(!wd.track(8) && f.released.count(8) == 1);             // nothing more is accepted
        std::printf("timeout ok\n");
    }
    {   // the deadline runs from each collective's own enqueue time, oldest first
        Fake f;
        CommWatchdog<FakeOps> wd(FakeOps{&f}, 2.0);
        CHECK(wd.track(1));
        f.clock = 1.5;
        CHECK(wd.track(2));
        complete(f, 1);
        f.clock = 3.0;     // 1 finished; 2 has run 1.5 s
        CHECK(wd.poll() == CommState::kHealthy && wd.in_flight() == 1);
        f.clock = 3.6;     // 2 has run 2.1 s
        CHECK(wd.poll() == CommState::kTimedOut);
        std::printf("per_collective_deadline ok\n");
    }
    {   // an asynchronous error (a peer failed or left) aborts at once; "in progress" does not
        Fake f;
        CommWatchdog<FakeOps> wd(FakeOps{&f}, 100.0);
        CHECK(wd.track(1));
        f.error = 1;
        CHECK(wd.poll() == CommState::kHealthy && f.aborts == 0);
        f.error = 2;
        CHECK(wd.poll() == CommState::kAsyncError && f.aborts == 1 && f.released.count(1) == 1);
        std::printf("async_error ok\n");
    }
    {   // abort on request (the host learned from a heartbeat that a peer is gone)
        Fake f;
        CommWatchdog<FakeOps> wd(FakeOps{&f}, 100.0);
        CHECK(wd.track(1));
        CHECK(wd.abort() == CommState::kAborted && f.aborts == 1);
        CHECK(wd.abort() == CommState::kAborted && f.aborts == 1);
        CHECK(wd.poll() == CommState::kAborted);
        std::printf("abort_on_request ok\n");
    }
    {   // a polling thread beside a tracking thread: every event is released exactly once and the
        // abort happens exactly once
        Fake f;
        CommWatchdog<FakeOps> wd(FakeOps{&f}, 1.0);
        std::atomic<bool> stop{false};
        std::thread poller([&] {
            while (!stop) wd.poll();
        });
        for (int e = 0; e < 20000; ++e) {
            wd.track(e);
            complete(f, e);
        }
        f.clock = 0.5;
        while (wd.in_flight() > 0) std::this_thread::yield();
        CHECK(wd.state() == CommState::kHealthy && f.released.size() == 20000);
        CHECK(wd.track(20000));
        f.clock = 2.0;
        while (wd.state() == CommState::kHealthy) std::this_thread::yield();
        stop = true;
        poller.join();
        CHECK(wd.state() == CommState::kTimedOut && f.aborts == 1 && f.released.size() == 20001);
        std::printf("threads ok\n");
    }
    return 0;
}
