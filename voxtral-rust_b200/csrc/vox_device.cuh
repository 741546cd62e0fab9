// vox_device.cuh -- sm_100a device helpers: mbarriers, 1-D bulk (TMA) copies,
// programmatic dependent launch, bounded waits, bf16 unpacking.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "vox_kernels.h"

namespace vox {

// Every spin in these kernels gives up after this long and raises an error
// bit instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

// Make mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// Policy: stream once through L2 (weights are read exactly once per step).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst and src 16-byte aligned, bytes a multiple of 16.  One destination CTA.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Same without an L2 policy (data that later kernels may read again).
__device__ __forceinline__ void bulk_copy_g2s_nohint(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

// Fire-and-forget prefetch of [src, src + bytes) into L2 (16-byte aligned,
// bytes a multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Programmatic dependent launch (no-ops when launched without the attribute).
__device__ __forceinline__ void pdl_wait_prior_grids() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_allow_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" :::);
}

__device__ __forceinline__ void named_barrier_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ uint4 ld_shared_v4(const void* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_addr(p)));
    return v;
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
    return __uint_as_float(static_cast<uint32_t>(h) << 16);
}

__device__ __forceinline__ void raise_error(unsigned* err, unsigned bit) {
    if (err) atomicOr(err, bit);
}

// Bounded wait until a 64-bit counter (written by other GPUs) reaches
// target; false on timeout.
__device__ __forceinline__ bool wait_counter_sys(const unsigned long long* c, unsigned long long target) {
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        unsigned long long v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(c) : "memory");
        if (v >= target) return true;
        if ((it & 63u) == 63u) {
            const uint64_t now = global_timer_ns();
            if (t0 == 0)
                t0 = now;
            else if (now - t0 > kWaitLimitNs)
                return false;
        }
    }
}

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {  // round to nearest even
    const uint32_t u = __float_as_uint(f);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

// v0, v1 as packed bf16 hi parts, hi = bf16(v) rounded to nearest even (the
// same bits as f32_to_bf16_bits for finite v, in one cvt.rn.bf16x2
// instruction), and lo parts, lo = bf16(v - hi) (the subtraction is exact);
// v0 in the low half of each word.
__device__ __forceinline__ void split_bf16x2(float v0, float v1, uint32_t& hi, uint32_t& lo) {
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(v1), "f"(v0));
    const float h0 = __uint_as_float(hi << 16), h1 = __uint_as_float(hi & 0xFFFF0000u);
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(__fsub_rn(v1, h1)), "f"(__fsub_rn(v0, h0)));
}

// Element k of stream b into an X operand in XOP layout (vox_kernels.h):
// v as bf16 hi = bf16(v) and lo = bf16(v - hi).
__device__ __forceinline__ void xop_store(unsigned char* xop, int k, int b, float v) {
    const uint16_t h = f32_to_bf16_bits(v);
    const uint16_t l = f32_to_bf16_bits(v - bf16_bits_to_f32(h));
    const int kk = k & 63;
    uint16_t* base = reinterpret_cast<uint16_t*>(xop + (size_t)(k >> 6) * 2048 + (kk >> 4) * 512 +
                                                 ((kk >> 3) & 1) * 256) + (kk & 7);
    base[b * 8] = h;       // rows 0..7: hi
    base[64 + b * 8] = l;  // rows 8..15 (128 bytes on): lo
}

// State of a cache layer after appending one token (kv.rs:48-88 with n = 1).
__device__ __forceinline__ KvState kv_after_single_append(KvState s, int window, int cap) {
    int requested = s.len + 1;
    int drop = requested > window ? requested - window : 0;
    if (drop > 0) {
        int keep = s.len > drop ? s.len - drop : 0;
        int phys_drop = s.len < drop ? s.len : drop;  // tokens physically present
        s.start = (s.start + phys_drop) % cap;
        s.len = keep;
        s.pos_offset += drop;
    }
    s.len += 1;
    return s;
}

}  // namespace vox
