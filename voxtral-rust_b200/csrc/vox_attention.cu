// vox_attention.cu -- grouped-query decode attention over the KV ring.
//
// Restates attention_gqa_step (crates/voxtral/src/ops.rs:66-132) for one
// query token: for every q head h (kv head h / G), scores over the live
// tokens of the cache, softmax (math.rs:67-88), then the probability-weighted
// sum of V.  Tokens older than seq_len - sliding_window are masked (ops.rs:
// 91-95, 102-105).
//
// B200 layout: one CTA per (kv head, split of the token range).  The CTA
// serves all G query heads of its kv head, so each K/V row is read from HBM
// once per group (the reference reads it G times).  Tiles of 32 tokens are
// double-buffered in shared memory with cp.async; the CTA keeps an
// online-softmax state (running max m, running sum l, unnormalised
// accumulator) per head.  The number of active splits follows the live
// length at run time (at least one tile each), so one captured launch serves
// every step.  Split results go to a scratch buffer and the last CTA of each
// kv head (atomic ticket) merges them: per-split weights exp(m_s - M) / L are
// computed once per head, then every output is a dot product over the splits
// with independent loads.  Merge order is fixed, so results are run-to-run
// deterministic.
//
// The ring is head-major [n_kv, cap, hd]: logical token t of a layer lives
// in slot (start + t) % cap, so sliding-window eviction never moves data.
#include <cuda_runtime.h>
#include <math.h>

#include "vox_device.cuh"

namespace vox {

namespace {

constexpr int kAttnThreads = 128;
constexpr int kTile = 32;
constexpr int kMaxAcc = 4;      // accumulator vectors per thread (G*hd/VEC <= 512)
constexpr int kMaxSplits = 64;  // merge weights kept in shared memory

template <int VEC>
struct VecT;
template <>
struct VecT<1> {
    using T = float;
};
template <>
struct VecT<4> {
    using T = float4;
};

__device__ __forceinline__ float fdot(float acc, const float4& a, const float4& b) {
    acc = fmaf(a.x, b.x, acc);
    acc = fmaf(a.y, b.y, acc);
    acc = fmaf(a.z, b.z, acc);
    acc = fmaf(a.w, b.w, acc);
    return acc;
}
__device__ __forceinline__ float fdot(float acc, const float& a, const float& b) { return fmaf(a, b, acc); }
__device__ __forceinline__ void faxpy(float4& acc, float p, const float4& v) {
    acc.x = fmaf(p, v.x, acc.x);
    acc.y = fmaf(p, v.y, acc.y);
    acc.z = fmaf(p, v.z, acc.z);
    acc.w = fmaf(p, v.w, acc.w);
}
__device__ __forceinline__ void faxpy(float& acc, float p, const float& v) { acc = fmaf(p, v, acc); }
__device__ __forceinline__ void fscale(float4& a, float s) {
    a.x *= s;
    a.y *= s;
    a.z *= s;
    a.w *= s;
}
__device__ __forceinline__ void fscale(float& a, float s) { a *= s; }
__device__ __forceinline__ void fzero(float4& a) { a = make_float4(0.f, 0.f, 0.f, 0.f); }
__device__ __forceinline__ void fzero(float& a) { a = 0.f; }
__device__ __forceinline__ float fget(const float4& a, int i) {
    return i == 0 ? a.x : i == 1 ? a.y : i == 2 ? a.z : a.w;
}
__device__ __forceinline__ float fget(const float& a, int) { return a; }

// 16-byte global -> shared copy; zero-fills when !valid.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(n)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Stage tokens [t0, t0 + kTile) ∩ [.., t_end) of one kv head into smem.
template <int VEC>
__device__ __forceinline__ void load_tile(float* ks, float* vs, const float* kr, const float* vr, int t0,
                                          int t_end, int start, int cap, int hd, int ldk) {
    using T = typename VecT<VEC>::T;
    const int hdv = hd / VEC;
    for (int u = threadIdx.x; u < kTile * hdv; u += kAttnThreads) {
        const int tt = u / hdv, dv = u - tt * hdv;
        const int t = t0 + tt;
        const bool valid = t < t_end;
        int slot = start + (valid ? t : t0);
        if (slot >= cap) slot -= cap;
        const float* sk = kr + (size_t)slot * hd + dv * VEC;
        const float* sv = vr + (size_t)slot * hd + dv * VEC;
        float* dk = ks + tt * ldk + dv * VEC;
        float* dv_ = vs + tt * ldk + dv * VEC;
        if constexpr (VEC == 4) {
            cp_async16(dk, sk, valid);
            cp_async16(dv_, sv, valid);
        } else {
            *dk = valid ? *sk : 0.f;
            *dv_ = valid ? *sv : 0.f;
        }
    }
}

template <int VEC>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(const AttnArgs A) {
    using T = typename VecT<VEC>::T;
    extern __shared__ __align__(16) float sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.x;          // kv head
    const int split = blockIdx.y;
    const int z = blockIdx.z;          // stream
    const int hd = A.hd;
    const int G = A.n_heads / A.n_kv;
    const int hdv = hd / VEC;          // vectors per row
    const int pad = VEC == 4 ? 4 : 1;  // row padding (floats) against bank conflicts
    const int ldk = hd + pad;
    const int tile_f = kTile * ldk;

    float* q_s = sm;                          // [G, hd]
    float* kbuf = q_s + G * hd;               // [2][kTile, ldk]
    float* vbuf = kbuf + 2 * tile_f;          // [2][kTile, ldk]
    float* p_s = vbuf + 2 * tile_f;           // [G, kTile]
    float* m_s = p_s + G * kTile;             // [G] running max
    float* l_s = m_s + G;                     // [G] running sum
    float* a_s = l_s + G;                     // [G] rescale factor of this tile
    float* w_s = a_s + G;                     // [G, kMaxSplits] merge weights
    int* flag_s = reinterpret_cast<int*>(w_s + G * kMaxSplits);

    pdl_allow_dependents();
    pdl_wait_prior_grids();

    const float* q_in = A.q + z * A.q_stride;
    float* out = A.out + z * A.out_stride;
    float* part = A.part + z * A.part_stride;
    unsigned* tickets = A.tickets + (size_t)z * A.n_kv;
    KvState st = A.st[z * A.st_stride];
    if (A.pre_append) st = kv_after_single_append(st, A.kv_window, A.cap);
    const int len = st.len;
    const int mask_start = (A.cfg_window > 0 && len > A.cfg_window) ? len - A.cfg_window : 0;
    const int n_live = len - mask_start;
    int per = (n_live + A.nsplit - 1) / A.nsplit;
    per = ((per + kTile - 1) / kTile) * kTile;
    if (per < kTile) per = kTile;
    const int n_active = (n_live + per - 1) / per;
    float* out_h = out + (size_t)h * G * hd;
    if (n_active == 0) {  // empty cache: the reference returns zeros
        if (split == 0)
            for (int i = tid; i < G * hd; i += kAttnThreads) out_h[i] = 0.f;
        return;
    }
    if (split >= n_active) return;
    const int t_begin = mask_start + split * per;
    const int t_end = min(len, t_begin + per);

    const float* kr = A.k_ring + z * A.ring_stride + (size_t)h * A.cap * hd;
    const float* vr = A.v_ring + z * A.ring_stride + (size_t)h * A.cap * hd;
    load_tile<VEC>(kbuf, vbuf, kr, vr, t_begin, t_end, st.start, A.cap, hd, ldk);
    if constexpr (VEC == 4) cp_async_commit();

    for (int i = tid; i < G * hd; i += kAttnThreads) q_s[i] = q_in[(size_t)h * G * hd + i];
    if (tid < G) {
        m_s[tid] = -INFINITY;
        l_s[tid] = 0.f;
    }
    T acc[kMaxAcc];
#pragma unroll
    for (int j = 0; j < kMaxAcc; ++j) fzero(acc[j]);
    const int n_out = G * hdv;

    int buf = 0;
    for (int t0 = t_begin; t0 < t_end; t0 += kTile, buf ^= 1) {
        const bool has_next = t0 + kTile < t_end;
        if (has_next) {
            load_tile<VEC>(kbuf + (buf ^ 1) * tile_f, vbuf + (buf ^ 1) * tile_f, kr, vr, t0 + kTile, t_end,
                           st.start, A.cap, hd, ldk);
            if constexpr (VEC == 4) cp_async_commit();
        }
        if constexpr (VEC == 4) {
            if (has_next)
                cp_async_wait<1>();
            else
                cp_async_wait<0>();
        }
        __syncthreads();
        const float* k_s = kbuf + buf * tile_f;
        const float* v_s = vbuf + buf * tile_f;
        // Scores: (g, t) pairs; ops.rs:108-113 dot * scale.
        for (int idx = tid; idx < G * kTile; idx += kAttnThreads) {
            const int g = idx / kTile, tt = idx - g * kTile;
            float s = -INFINITY;
            if (t0 + tt < t_end) {
                float d = 0.f;
                const T* qv = reinterpret_cast<const T*>(q_s + g * hd);
                const T* kv = reinterpret_cast<const T*>(k_s + tt * ldk);
                for (int dv = 0; dv < hdv; ++dv) d = fdot(d, qv[dv], kv[dv]);
                s = d * A.scale;
            }
            p_s[idx] = s;
        }
        __syncthreads();
        // Online softmax update, one warp per head.
        for (int g = warp; g < G; g += kAttnThreads / 32) {
            const float s = p_s[g * kTile + lane];
            float mt = s;
#pragma unroll
            for (int o = 16; o; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xFFFFFFFFu, mt, o));
            const float m_old = m_s[g];
            const float m_new = fmaxf(m_old, mt);
            const float p = (s == -INFINITY) ? 0.f : expf(s - m_new);
            float ps = p;
#pragma unroll
            for (int o = 16; o; o >>= 1) ps += __shfl_xor_sync(0xFFFFFFFFu, ps, o);
            p_s[g * kTile + lane] = p;
            if (lane == 0) {
                const float alpha = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
                a_s[g] = alpha;
                l_s[g] = l_s[g] * alpha + ps;
                m_s[g] = m_new;
            }
        }
        __syncthreads();
        // PV (ops.rs:117-128): acc = acc*alpha + sum_t p_t v_t.
#pragma unroll
        for (int j = 0; j < kMaxAcc; ++j) {
            const int o = tid + j * kAttnThreads;
            if (o < n_out) {
                const int g = o / hdv, dv = o - g * hdv;
                fscale(acc[j], a_s[g]);
                const float* pg = p_s + g * kTile;
#pragma unroll 8
                for (int tt = 0; tt < kTile; ++tt)
                    faxpy(acc[j], pg[tt], *reinterpret_cast<const T*>(v_s + tt * ldk + dv * VEC));
            }
        }
        __syncthreads();  // the next iteration refills the other buffer of this pair
    }

    // Split partials: accumulators [n_kv, nsplit, G, hd], then (m, l) pairs
    // [n_kv, nsplit, G, 2], so the merge can read accumulators as vectors.
    const size_t acc_stride = (size_t)G * hd;  // floats per split
    const size_t ml_base = (size_t)A.n_kv * A.nsplit * acc_stride;
    float* pacc = part + ((size_t)h * A.nsplit + split) * acc_stride;
    float* pml = part + ml_base + ((size_t)h * A.nsplit + split) * G * 2;
#pragma unroll
    for (int j = 0; j < kMaxAcc; ++j) {
        const int o = tid + j * kAttnThreads;
        if (o < n_out) *reinterpret_cast<T*>(pacc + (size_t)o * VEC) = acc[j];
    }
    if (tid < G) {
        pml[tid * 2] = m_s[tid];
        pml[tid * 2 + 1] = l_s[tid];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned ticket = atomicAdd(&tickets[h], 1u);
        flag_s[0] = (ticket == (unsigned)(n_active - 1)) ? 1 : 0;
    }
    __syncthreads();
    if (!flag_s[0]) return;
    __threadfence();

    // Last CTA of this kv head: merge weights w_s = exp(m_s - M) / L once per head ...
    const float* bacc = part + (size_t)h * A.nsplit * acc_stride;
    const float* bml = part + ml_base + (size_t)h * A.nsplit * G * 2;
    for (int g = warp; g < G; g += kAttnThreads / 32) {
        float ms[2], ls[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int s = lane + 32 * r;
            ms[r] = s < n_active ? __ldcg(bml + ((size_t)s * G + g) * 2) : -INFINITY;
            ls[r] = s < n_active ? __ldcg(bml + ((size_t)s * G + g) * 2 + 1) : 0.f;
        }
        float M = fmaxf(ms[0], ms[1]);
#pragma unroll
        for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
        float w[2], L = 0.f;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            w[r] = ms[r] == -INFINITY ? 0.f : expf(ms[r] - M);
            L = fmaf(ls[r], w[r], L);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xFFFFFFFFu, L, o);
        const float invL = L > 0.f ? 1.0f / L : 0.f;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int s = lane + 32 * r;
            if (s < n_active) w_s[g * kMaxSplits + s] = w[r] * invL;
        }
    }
    __syncthreads();
    // ... then each output vector is a weighted sum over the splits, loaded
    // eight splits at a time with independent loads.
    const size_t vstride = acc_stride / VEC;
    for (int o = tid; o < n_out; o += kAttnThreads) {
        const int g = o / hdv;
        const T* pv = reinterpret_cast<const T*>(bacc) + o;
        const float* wg = w_s + g * kMaxSplits;
        T sum;
        fzero(sum);
        for (int s0 = 0; s0 < n_active; s0 += 8) {
            T v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (s0 + j < n_active)
                    v[j] = __ldcg(pv + (size_t)(s0 + j) * vstride);
                else
                    fzero(v[j]);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (s0 + j < n_active) faxpy(sum, wg[s0 + j], v[j]);
        }
        *reinterpret_cast<T*>(out_h + (size_t)o * VEC) = sum;
    }
    if (tid == 0) tickets[h] = 0u;
}

}  // namespace

bool attn_supported(int n_heads, int n_kv, int hd) {
    if (n_kv <= 0 || n_heads % n_kv) return false;
    const int G = n_heads / n_kv;
    if (G > kTile * 4) return false;
    const int vec = (hd % 4 == 0) ? 4 : 1;
    return (G * hd / vec) <= kMaxAcc * kAttnThreads;
}

size_t attn_smem_bytes(int n_heads, int n_kv, int hd) {
    const int G = n_heads / n_kv;
    const int pad = (hd % 4 == 0) ? 4 : 1;
    const size_t floats = (size_t)G * hd + 4 * kTile * (hd + pad) + (size_t)G * kTile + 3 * G +
                          (size_t)G * kMaxSplits + 4;
    return floats * 4;
}

int attn_splits_for(int n_kv, int num_sms) {
    int s = (2 * num_sms + n_kv - 1) / n_kv;
    if (s < 1) s = 1;
    if (s > kMaxSplits) s = kMaxSplits;
    return s;
}

cudaError_t attn_prepare(int /*dev*/) {
    cudaError_t e = cudaFuncSetAttribute(attn_split_kernel<4>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(attn_split_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                200 * 1024);
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_kv, a.nsplit, a.n_streams > 1 ? a.n_streams : 1);
    cfg.blockDim = dim3(kAttnThreads, 1, 1);
    cfg.dynamicSmemBytes = attn_smem_bytes(a.n_heads, a.n_kv, a.hd);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    void* args[] = {(void*)&a};
    void* k = (a.hd % 4 == 0) ? (void*)attn_split_kernel<4> : (void*)attn_split_kernel<1>;
    return cudaLaunchKernelExC(&cfg, k, args);
}

}  // namespace vox
