// Host-side wait with failure detection for the sharded Lloyd loop.
//
// A blocking wait on a stream whose next collective needs a peer that has
// failed never returns.  guarded_wait polls instead: the completion probe
// (an event query), then the peer probe (the communicator's asynchronous
// error, or a failure another rank of the same process has reported), and
// gives up once the wait has made no progress for `limit_s` seconds (no time
// limit when limit_s <= 0: only a failed peer ends the wait).  The caller aborts the communicator on kPeerFailed / kTimedOut, which
// makes the collectives in flight return, and reports an error instead of
// hanging.  Plain host code with injectable probes and clock, so its logic is
// tested without a GPU.
#pragma once

#include <chrono>
#include <thread>

namespace mxk {

enum class Probe { kReady, kPending, kFailed };
enum class WaitResult { kReady, kFailed, kPeerFailed, kTimedOut };

// done(): Probe of the awaited work; peer_failed(): true once a peer is known
// to have failed; now(): seconds on a monotonic clock; pause(): between polls.
template <class Done, class PeerFailed, class Now, class Pause>
WaitResult guarded_wait(Done&& done, PeerFailed&& peer_failed, double limit_s, Now&& now, Pause&& pause) {
    const double start = now();
    for (;;) {
        const Probe p = done();
        if (p == Probe::kReady) return WaitResult::kReady;
        if (p == Probe::kFailed) return WaitResult::kFailed;
        if (peer_failed()) return WaitResult::kPeerFailed;
        if (limit_s > 0.0 && now() - start > limit_s) return WaitResult::kTimedOut;
        pause();
    }
}

inline double monotonic_seconds() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

inline void short_pause() { std::this_thread::sleep_for(std::chrono::microseconds(50)); }

}  // namespace mxk
