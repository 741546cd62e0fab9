// vox_host.h -- host-side helpers shared by the C ABI files (vox_capi.cpp,
// vox_tp.cpp): error reporting, the kv.rs ring bookkeeping mirror, device
// allocation and bf16 conversion.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <cstddef>

namespace vox {

// Record a printf-style message for vox_last_error() and return `code`.
int report_errorf(int code, const char* fmt, ...);

// Host mirror of one cache layer: the reference's (len_tokens, pos_offset)
// plus the physical ring start.
struct HostKv {
    size_t len = 0, start = 0, pos_offset = 0;
};

// kv.rs:48-88 append bookkeeping for n tokens.  Returns the ring slot of the
// first new token, or -1 if the result would not fit in `cap` slots.
inline long long host_append(HostKv& s, size_t n, size_t window, size_t cap) {
    if (n == 0) return (long long)((s.start + s.len) % cap);
    HostKv t = s;
    size_t requested = t.len + n;
    size_t drop = requested > window ? requested - window : 0;
    if (drop > 0) {
        size_t keep = t.len > drop ? t.len - drop : 0;
        size_t phys = t.len < drop ? t.len : drop;
        t.start = (t.start + phys) % cap;
        t.len = keep;
        t.pos_offset += drop;
    }
    if (t.len + n > cap) return -1;
    long long slot0 = (long long)((t.start + t.len) % cap);
    t.len += n;
    s = t;
    return slot0;
}

template <class T>
inline cudaError_t dalloc(T** p, size_t n) {
    *p = nullptr;
    if (n == 0) n = 1;
    return cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T));
}

// Round to nearest even (NaN stays NaN).
inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return 0x7FC0;
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}
inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

}  // namespace vox
