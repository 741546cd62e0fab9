// Host check of the tensor-parallel watchdog (voxtral-rust_b200/csrc/vox_watchdog.h)
// with fakes of the stream query, the asynchronous-error poll and the abort.
// Prints one line per scenario: name result abort_calls elapsed_ms.
#include <chrono>
#include <cstdio>

#include "vox_watchdog.h"

using vox::watchdog_wait;

static double now_ms() {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

int main() {
    struct Case { const char* name; int idle_after; int async_after; int stream_error_after; unsigned timeout_ms; };
    // idle_after / async_after / stream_error_after: poll count at which the event happens (-1 never)
    const Case cases[] = {
        {"idle_at_once", 0, -1, -1, 1000},
        {"idle_after_polls", 200, -1, -1, 1000},
        {"async_error", -1, 50, -1, 1000},
        {"rank_stopped_timeout", -1, -1, -1, 300},
        {"stream_error", -1, -1, 10, 1000},
    };
    for (const Case& c : cases) {
        int polls = 0, async_polls = 0, aborts = 0;
        auto query = [&]() {
            const int p = polls++;
            if (c.stream_error_after >= 0 && p >= c.stream_error_after) return 2;
            return (c.idle_after >= 0 && p >= c.idle_after) ? 0 : 1;
        };
        auto async_error = [&]() { return c.async_after >= 0 && async_polls++ >= c.async_after; };
        auto abort = [&]() { ++aborts; };
        const double t0 = now_ms();
        const int r = watchdog_wait(query, async_error, abort, c.timeout_ms);
        std::printf("%s %d %d %.1f\n", c.name, r, aborts, now_ms() - t0);
    }
    return 0;
}
