// vox_watchdog.h -- the bounded host wait of the tensor-parallel step.
//
// A rank that stops calling (a crashed or stuck process) leaves the other
// ranks' collectives waiting for ever.  Every host wait on a tensor-parallel
// stream therefore polls instead of blocking: it returns as soon as the
// stream is idle, aborts the communicator when the collective library reports
// an asynchronous error, and aborts it when the step has not finished within
// the timeout.  Header-only and free of CUDA/NCCL types so that the logic is
// tested on the host with fakes of the three calls.
#pragma once

#include <chrono>
#include <thread>

namespace vox {

enum WatchdogResult { kWatchdogIdle = 0, kWatchdogAsyncError = 1, kWatchdogTimeout = 2, kWatchdogStreamError = 3 };

// query():        0 = stream idle, 1 = still running, 2 = stream error
// async_error():  true when the communicator reports an asynchronous error
// abort():        aborts the communicator (called at most once)
template <class Query, class AsyncError, class Abort>
WatchdogResult watchdog_wait(Query query, AsyncError async_error, Abort abort, unsigned timeout_ms) {
    using clock = std::chrono::steady_clock;
    const auto t0 = clock::now();
    for (unsigned spin = 0;; ++spin) {
        const int q = query();
        if (q == 0) return kWatchdogIdle;
        if (q != 1) return kWatchdogStreamError;
        if (async_error()) {
            abort();
            return kWatchdogAsyncError;
        }
        const double ms = std::chrono::duration<double, std::milli>(clock::now() - t0).count();
        if (ms > (double)timeout_ms) {
            abort();
            return kWatchdogTimeout;
        }
        if (spin > 64) std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // namespace vox
