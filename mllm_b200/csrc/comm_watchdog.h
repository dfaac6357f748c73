// Host-side watchdog of a communicator's collectives (no CUDA or NCCL types in here).
//
// Every collective the library enqueues is tracked by an event recorded right after it on the
// caller's stream.  A poll -- run every few milliseconds by the communicator's watchdog thread,
// or once by mllm_comm_status -- does three things:
//   1. asks the communicator for an asynchronous error (a failed or lost peer, a network error);
//   2. drops the tracked collectives whose events have completed, oldest first;
//   3. compares the age of the oldest one still running against the deadline.
// On an asynchronous error, or when a collective has run longer than the deadline, it aborts the
// communicator once (which ends its kernels on the GPU, so no stream stays blocked on a peer that
// will never answer) and the communicator's state becomes kAsyncError or kTimedOut for good.
//
// The operations it needs come in as a policy type, so the same logic runs against NCCL and the
// CUDA runtime in the library and against fakes in a CPU test:
//   struct Ops {
//       using Event = ...;
//       int  async_error();          // 0: healthy, 1: still initialising, 2: failed
//       bool done(Event e);          // the event has completed
//       void release(Event e);       // the event is no longer tracked (return it to a pool)
//       void abort();                // abort the communicator (called at most once)
//       double now();                // seconds, monotonic
//   };
#pragma once

#include <deque>
#include <mutex>
#include <utility>

namespace mllm_b200 {

enum class CommState : int { kHealthy = 0, kAsyncError = 1, kTimedOut = 2, kAborted = 3 };

template <class Ops>
class CommWatchdog {
public:
    using Event = typename Ops::Event;

    CommWatchdog(Ops ops, double timeout_s) : ops_(std::move(ops)), timeout_s_(timeout_s) {}

    // Starts tracking a collective whose completion `e` marks.  Returns false (and releases the
    // event) if the communicator was aborted already.
    bool track(Event e) {
        std::lock_guard<std::mutex> lock(mu_);
        if (state_ != CommState::kHealthy) {
            ops_.release(e);
            return false;
        }
        pending_.push_back({e, ops_.now()});
        return true;
    }

    // One round of checks (see the file comment).  Returns the state after it.
    CommState poll() {
        std::lock_guard<std::mutex> lock(mu_);
        if (state_ != CommState::kHealthy) return state_;
        if (ops_.async_error() >= 2) return abort_locked(CommState::kAsyncError);
        while (!pending_.empty() && ops_.done(pending_.front().event)) {
            ops_.release(pending_.front().event);
            pending_.pop_front();
        }
        if (!pending_.empty() && ops_.now() - pending_.front().enqueued > timeout_s_)
            return abort_locked(CommState::kTimedOut);
        return state_;
    }

    // Aborts on request (the host learned on its own that a peer is gone).
    CommState abort() {
        std::lock_guard<std::mutex> lock(mu_);
        if (state_ != CommState::kHealthy) return state_;
        return abort_locked(CommState::kAborted);
    }

    CommState state() {
        std::lock_guard<std::mutex> lock(mu_);
        return state_;
    }

    size_t in_flight() {
        std::lock_guard<std::mutex> lock(mu_);
        return pending_.size();
    }

    Ops& ops() { return ops_; }

private:
    struct Pending {
        Event event;
        double enqueued;
    };

    CommState abort_locked(CommState why) {
        state_ = why;
        ops_.abort();
        // the aborted collectives are over as far as the host is concerned
        for (auto& p : pending_) ops_.release(p.event);
        pending_.clear();
        return state_;
    }

    Ops ops_;
    double timeout_s_;
    std::mutex mu_;
    std::deque<Pending> pending_;
    CommState state_ = CommState::kHealthy;
};

}  // namespace mllm_b200
