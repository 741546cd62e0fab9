// vox_attention.cu -- grouped-query decode attention over the KV ring.
//
// Restates attention_gqa_step (crates/voxtral/src/ops.rs:66-132) for one
// query token: for every q head h (kv head h / G), scores over the live
// tokens of the cache, softmax (math.rs:67-88), then the probability-weighted
// sum of V.  Tokens older than seq_len - sliding_window are masked (ops.rs:
// 91-95, 102-105).
//
// B200 layout: a persistent grid (every CTA that fits on the SMs) walks one
// work list of chunks: (stream, kv head, chunk of the live token range).
// Chunks have the same number of 32-token tiles across all streams, chosen
// at run time from the live lengths so that every CTA gets about two, which
// keeps streams of very different context lengths balanced and lets one
// captured launch serve every step.  A CTA serves all G query heads of its
// kv head, so each K/V row is read from HBM once per group (the reference
// reads it G times).  Tiles are double-buffered in shared memory with
// cp.async; the CTA keeps an online-softmax state (running max m, running sum
// l, unnormalised accumulator) per head.  Chunk results go to a scratch
// buffer and the last chunk of each (stream, kv head) to finish (atomic
// ticket) merges them: per-chunk weights exp(m_s - M) / L are computed once
// per head, then every output is a dot product over the chunks with
// independent loads.  Merge order is fixed, so results are run-to-run
// deterministic.
//
// The ring is head-major [n_kv, cap, hd]: logical token t of a layer lives
// in slot (start + t) % cap, so sliding-window eviction never moves data.
#include <cuda_runtime.h>
#include <math.h>

#include <mutex>

#include "vox_device.cuh"

namespace vox {

namespace {

constexpr int kAttnThreads = 128;
constexpr int kTile = 32;
constexpr int kMaxAcc = 4;      // accumulator vectors per thread (G*hd/VEC <= 512)
constexpr int kMaxSplits = 64;  // merge weights kept in shared memory
// Most live tokens per kv head for which one stream's attention runs as one
// thread-block cluster per kv head (attn_cluster_kernel).
constexpr int kAttnClusterMaxTokens = 3584;
// Warps of a cluster-attention CTA and K/V ring stages per warp.  A CTA (4
// warps at 136 registers, 17408; 2 stages: 64 KB of K/V slots, the 33 KB merge
// buffer and 8 KB of static state) fits on an SM beside two lean o-proj GEMV
// CTAs (9 warps at 80 registers and a 48 KB ring each): 63488 registers and
// about 205 KB of shared memory, so o-proj streams its weights while attention
// runs.  The second stage lets a warp's first two 8-token groups load before
// the dependency wait: 1.514 vs 1.537 ms per token at context 520-776, 1.577 vs
// 1.621 at 1536 (three stages with 32 KB o-proj rings: 1.519 / 1.617).
constexpr int kClusterWarps = 4;
constexpr int kClusterStages = 2;

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

// Work list shared by every CTA: stream z has items_z chunks of tpi_z tiles
// per kv head; items are numbered stream-major, then kv head, then chunk.
struct AttnPlan {
    int len[8], mask_start[8], start[8], tpi[8], items[8], first[9];
    int firstn[9];  // warp kernel: prefix sums of the chunks that are not a pair's last
};

template <int VEC>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(const AttnArgs A) {
    using T = typename VecT<VEC>::T;
    extern __shared__ __align__(16) float sm[];
    __shared__ AttnPlan plan;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hd = A.hd;
    const int G = A.n_heads / A.n_kv;
    const int hdv = hd / VEC;          // vectors per row
    const int pad = VEC == 4 ? 4 : 1;  // row padding (floats) against bank conflicts
    const int ldk = hd + pad;
    const int tile_f = kTile * ldk;
    const int B = A.n_streams > 1 ? A.n_streams : 1;

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

    // Live range of every stream (ops.rs:91-95) and its share of the work:
    // chunks of equal length across all streams, so long contexts get more
    // CTAs, at most nsplit chunks per (stream, kv head).
    if (tid == 0) {
        long long total_tiles = 0;
        for (int z = 0; z < B; ++z) {
            KvState st = A.st[z * A.st_stride];
            if (A.pre_append) st = kv_after_single_append(st, A.kv_window, A.cap);
            const int len = st.len;
            const int ms = (A.cfg_window > 0 && len > A.cfg_window) ? len - A.cfg_window : 0;
            plan.len[z] = len;
            plan.mask_start[z] = ms;
            plan.start[z] = st.start;
            plan.items[z] = (len - ms + kTile - 1) / kTile;  // live tiles, for now
            total_tiles += (long long)plan.items[z] * A.n_kv;
        }
        const long long slots = 2LL * gridDim.x;
        const int tpi_all = (int)max(1LL, (total_tiles + slots - 1) / slots);
        int first = 0;
        for (int z = 0; z < B; ++z) {
            const int tiles = plan.items[z];
            const int tpi = max(tpi_all, (tiles + A.nsplit - 1) / A.nsplit);
            plan.tpi[z] = tpi;
            plan.items[z] = (tiles + tpi - 1) / tpi;
            plan.first[z] = first;
            first += plan.items[z] * A.n_kv;
        }
        plan.first[B] = first;
    }
    __syncthreads();

    // Streams with nothing to attend to: the reference returns zeros.
    if (blockIdx.x == 0)
        for (int z = 0; z < B; ++z)
            if (plan.items[z] == 0) {
                float* out = A.out + z * A.out_stride;
                for (int i = tid; i < A.n_heads * hd; i += kAttnThreads) {
                    out[i] = 0.f;
                    if (A.xop) xop_store(A.xop, i, z, 0.f);
                }
            }

    const int total = plan.first[B];
    for (int item = blockIdx.x; item < total; item += gridDim.x) {
        __syncthreads();  // shared buffers of the previous item are free
        int z = 0;
        while (z + 1 < B && item >= plan.first[z + 1]) ++z;
        const int n_active = plan.items[z];
        const int local = item - plan.first[z];
        const int h = local / n_active;
        const int split = local - h * n_active;
        const int len = plan.len[z];
        const int per = plan.tpi[z] * kTile;
        const int t_begin = plan.mask_start[z] + split * per;
        const int t_end = min(len, t_begin + per);
        const int ring_start = plan.start[z];

        const float* q_in = A.q + z * A.q_stride;
        float* out_h = A.out + z * A.out_stride + (size_t)h * G * hd;
        float* part = A.part + z * A.part_stride;
        unsigned* tickets = A.tickets + (size_t)z * A.n_kv;
        const float* kr = A.k_ring + z * A.ring_stride + (size_t)h * A.cap * hd;
        const float* vr = A.v_ring + z * A.ring_stride + (size_t)h * A.cap * hd;

        load_tile<VEC>(kbuf, vbuf, kr, vr, t_begin, t_end, ring_start, A.cap, hd, ldk);
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
                               ring_start, A.cap, hd, ldk);
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
        if (!flag_s[0]) continue;
        __threadfence();

        // Last chunk of this (stream, kv head): merge weights w_s = exp(m_s - M) / L
        // once per head ...
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
        // ... then each output vector is a weighted sum over the chunks, loaded
        // eight at a time with independent loads.
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
            if (A.xop)
#pragma unroll
                for (int i = 0; i < VEC; ++i) xop_store(A.xop, h * G * hd + o * VEC + i, z, fget(sum, i));
        }
        if (tid == 0) tickets[h] = 0u;
    }
}

// ---- warp-per-chunk variant for G = 4 or 8 query heads per kv head ----------
// Each warp owns a chunk of tokens of one (stream, kv head) and reads every
// K/V row of it exactly once, straight from HBM into registers: lane l holds
// dims 4l..4l+3 of 32/G consecutive tokens.  The G x (32/G) partial dot
// products are summed across the warp by a transpose-reduce (31 shuffles)
// that leaves lane l with the score of (head l / (32/G), token l % (32/G));
// the online-softmax update then runs on one score per lane, and the PV
// product on the lane's four dims for all G heads.  No shared-memory staging,
// so nothing is re-read per head.
template <int N>
__device__ __forceinline__ void transpose_reduce(float (&v)[N], int lane) {
    // After the step with offset o the lane keeps the half of its values
    // selected by bit o of its lane id; at the end lane l holds value l.
#pragma unroll
    for (int o = 16, n = N; o >= 1; o >>= 1, n >>= 1) {
        const bool up = lane & o;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float keep = up ? v[i + n / 2] : v[i];
            const float send = up ? v[i] : v[i + n / 2];
            v[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, o);
        }
    }
}

__device__ __forceinline__ float dot4(const float4& a, const float4& b) {
    float d = a.x * b.x;
    d = fmaf(a.y, b.y, d);
    d = fmaf(a.z, b.z, d);
    return fmaf(a.w, b.w, d);
}

// Bulk copies of group k of `warp` in chunk [t_begin, t_end) (K rows, then V
// rows, two pieces each at the ring's wrap) into the warp's slot k % D,
// completing on that slot's mbarrier.  Called by lane 0.
template <int G, int D, int NW = kAttnThreads / 32>
__device__ __forceinline__ void attn_issue_group(const AttnArgs& A, int z, int h, int t_begin, int t_end,
                                                 int ring_start, unsigned char* ring_smem, uint64_t (*wbar)[D],
                                                 int warp, int k, int hd) {
    constexpr int TPG = 32 / G;
    const size_t row_bytes = (size_t)hd * 4;
    const uint32_t stage_bytes = (uint32_t)(2 * TPG * row_bytes);
    const float* kbase = A.k_ring + z * A.ring_stride + (size_t)h * A.cap * hd;
    const float* vbase = A.v_ring + z * A.ring_stride + (size_t)h * A.cap * hd;
    const int t0 = t_begin + (warp + NW * k) * TPG;
    const int ntok = min(TPG, t_end - t0);
    int slot0 = ring_start + t0;
    if (slot0 >= A.cap) slot0 -= A.cap;
    const int n1 = min(ntok, A.cap - slot0);
    unsigned char* st = ring_smem + ((size_t)warp * D + k % D) * stage_bytes;
    uint64_t* bar = &wbar[warp][k % D];
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive_expect_tx(bar, (uint32_t)(2 * ntok * row_bytes));
    bulk_copy_g2s_nohint(st, kbase + (size_t)slot0 * hd, (uint32_t)(n1 * row_bytes), bar);
    bulk_copy_g2s_nohint(st + TPG * row_bytes, vbase + (size_t)slot0 * hd, (uint32_t)(n1 * row_bytes), bar);
    if (n1 < ntok) {
        bulk_copy_g2s_nohint(st + n1 * row_bytes, kbase, (uint32_t)((ntok - n1) * row_bytes), bar);
        bulk_copy_g2s_nohint(st + TPG * row_bytes + n1 * row_bytes, vbase, (uint32_t)((ntok - n1) * row_bytes), bar);
    }
}

// One chunk [t_begin, t_end) of kv head h of stream z, run by every warp of
// the CTA: warp w takes groups w, w + NW, ... of the chunk.  Each group's K
// rows and V rows are contiguous in the ring (two pieces at the wrap), so lane
// 0 fetches them with 1-D bulk copies into the warp's own D-stage slot ring;
// all lanes then read their four dims per row.  Leaves each warp's
// accumulators in wacc[warp] and its (m, l) per head in wml[warp]; the caller
// synchronizes before combining them.  warp, lane and hd are the caller's
// (computed once per kernel: passing them keeps the caller's registers);
// pre_issued groups of this warp were already copied by the caller.
template <int G, int D, int NW = kAttnThreads / 32>
__device__ __forceinline__ void attn_chunk_warps(const AttnArgs& A, int z, int h, int t_begin, int t_end,
                                                 int ring_start, unsigned char* ring_smem, uint64_t (*wbar)[D],
                                                 float (*wacc)[G][128], float (*wml)[G][2], uint32_t& phase,
                                                 const int warp, const int lane, const int hd,
                                                 const int pre_issued = 0) {
    constexpr int TPG = 32 / G;
    const unsigned FULL = 0xFFFFFFFFu;
    const bool dim_ok = lane * 4 < hd;
    const int my_g = lane / TPG, my_t = lane % TPG;
    const float* qh = A.q + z * A.q_stride + (size_t)h * G * hd + lane * 4;

    float4 q[G], acc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        q[g] = dim_ok ? *reinterpret_cast<const float4*>(qh + (size_t)g * hd) : make_float4(0.f, 0.f, 0.f, 0.f);
        acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float m_run = -INFINITY, l_run = 0.f;  // of head my_g

    const int n_groups = (t_end - t_begin + TPG - 1) / TPG;
    const int n_my = warp < n_groups ? (n_groups - warp + NW - 1) / NW : 0;
    const size_t row_bytes = (size_t)hd * 4;
    const uint32_t stage_bytes = (uint32_t)(2 * TPG * row_bytes);
    unsigned char* my_ring = ring_smem + (size_t)warp * D * stage_bytes;
    const float* kbase = A.k_ring + z * A.ring_stride + (size_t)h * A.cap * hd;
    const float* vbase = A.v_ring + z * A.ring_stride + (size_t)h * A.cap * hd;
    auto issue = [&](int k) {
        attn_issue_group<G, D, NW>(A, z, h, t_begin, t_end, ring_start, ring_smem, wbar, warp, k, hd);
    };
    if (lane == 0)
        for (int k = pre_issued; k < min(D, n_my); ++k) issue(k);
    __syncwarp();

    for (int k = 0; k < n_my; ++k) {
        const int t0 = t_begin + (warp + NW * k) * TPG;
        const int stg = k % D;
        if (!mbar_wait(&wbar[warp][stg], (phase >> stg) & 1u) && lane == 0) raise_error(A.err, ERR_FULL_WAIT);
        phase ^= 1u << stg;
        const float* ks = reinterpret_cast<const float*>(my_ring + (size_t)stg * stage_bytes) + lane * 4;
        const float* vs = ks + TPG * hd;
        float4 kk[TPG];
#pragma unroll
        for (int j = 0; j < TPG; ++j)
            kk[j] = dim_ok ? *reinterpret_cast<const float4*>(ks + (size_t)j * hd) : make_float4(0.f, 0.f, 0.f, 0.f);
        // ops.rs:108-113: scores q . k * scale (rows past t_end hold stale data
        // and are masked; their sums never mix with live ones)
        float sc[32];
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int j = 0; j < TPG; ++j) sc[g * TPG + j] = dot4(q[g], kk[j]);
        // V rows into registers now, so the slot is refilled while the
        // scores are reduced and the PV product runs
        float4 vv[TPG];
#pragma unroll
        for (int j = 0; j < TPG; ++j)
            vv[j] = (dim_ok && t0 + j < t_end) ? *reinterpret_cast<const float4*>(vs + (size_t)j * hd)
                                               : make_float4(0.f, 0.f, 0.f, 0.f);
        __syncwarp();  // every lane has read this stage before it is refilled
        if (lane == 0 && k + D < n_my) issue(k + D);
        transpose_reduce<32>(sc, lane);
        float s = sc[0] * A.scale;
        if (t0 + my_t >= t_end) s = -INFINITY;
        // online softmax over this group (math.rs:67-88 restated incrementally)
        float gm = s;
#pragma unroll
        for (int o = TPG / 2; o >= 1; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(FULL, gm, o));
        const float m_new = fmaxf(m_run, gm);
        const float p = (s == -INFINITY) ? 0.f : expf(s - m_new);
        float ps = p;
#pragma unroll
        for (int o = TPG / 2; o >= 1; o >>= 1) ps += __shfl_xor_sync(FULL, ps, o);
        const float alpha = (m_run == -INFINITY) ? 0.f : expf(m_run - m_new);
        l_run = l_run * alpha + ps;
        m_run = m_new;
        // PV (ops.rs:117-128) on this lane's dims for every head
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float a = __shfl_sync(FULL, alpha, g * TPG);
            acc[g].x *= a;
            acc[g].y *= a;
            acc[g].z *= a;
            acc[g].w *= a;
#pragma unroll
            for (int j = 0; j < TPG; ++j) {
                const float pj = __shfl_sync(FULL, p, g * TPG + j);
                acc[g].x = fmaf(pj, vv[j].x, acc[g].x);
                acc[g].y = fmaf(pj, vv[j].y, acc[g].y);
                acc[g].z = fmaf(pj, vv[j].z, acc[g].z);
                acc[g].w = fmaf(pj, vv[j].w, acc[g].w);
            }
        }
    }

    // Combine the warps of this chunk in shared memory.
    if (dim_ok)
#pragma unroll
        for (int g = 0; g < G; ++g) *reinterpret_cast<float4*>(&wacc[warp][g][lane * 4]) = acc[g];
    if (my_t == 0) {
        wml[warp][my_g][0] = m_run;
        wml[warp][my_g][1] = l_run;
    }
}

// Warp-per-chunk kernel, D-stage per-warp ring; at most 128 registers, four CTAs per SM.
template <int G, int D>
__global__ void __launch_bounds__(kAttnThreads, 4) attn_warp_kernel(const AttnArgs A) {
    constexpr int TPG = 32 / G;           // tokens per group: G * TPG = 32 scores per step
    constexpr int NW = kAttnThreads / 32; // warps per CTA
    constexpr int HD = 128;               // largest head_dim (4 dims per lane)
    extern __shared__ __align__(128) unsigned char ring_smem[];  // [NW][D][K rows | V rows]
    __shared__ uint64_t wbar[NW][D];
    __shared__ AttnPlan plan;
    __shared__ __align__(16) float wacc[NW][G][HD];  // per-warp accumulators of the chunk
    __shared__ float wml[NW][G][2];                  // per-warp (m, l)
    __shared__ float w_s[G][kMaxSplits];             // merge weights
    __shared__ int flag_s;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hd = A.hd;
    const int B = A.n_streams > 1 ? A.n_streams : 1;
    const unsigned FULL = 0xFFFFFFFFu;

    if (tid < NW * D) mbar_init(&wbar[tid / D][tid % D], 1);
    if (tid == 0) fence_barrier_init();
    pdl_allow_dependents();

    // Work list (same in every CTA): chunks of gpi groups per warp, i.e.
    // NW * gpi * TPG tokens per CTA chunk, at most nsplit chunks per
    // (stream, kv head), about one (several streams) or two chunks per CTA.
    if (tid == 0) {
        long long total_groups = 0;
        for (int z = 0; z < B; ++z) {
            KvState st = A.st[z * A.st_stride];
            if (A.pre_append) st = kv_after_single_append(st, A.kv_window, A.cap);
            const int len = st.len;
            const int ms = (A.cfg_window > 0 && len > A.cfg_window) ? len - A.cfg_window : 0;
            plan.len[z] = len;
            plan.mask_start[z] = ms;
            plan.start[z] = st.start;
            plan.items[z] = (len - ms + TPG - 1) / TPG;  // live groups, for now
            total_groups += (long long)plan.items[z] * A.n_kv;
        }
        // one chunk per warp slot for several streams (8 streams: 2.698 vs 2.738 ms
        // per step with two), two for a single stream
        const long long slots = (B > 1 ? 1LL : 2LL) * gridDim.x * NW;
        const int gpi_all = (int)max(1LL, (total_groups + slots - 1) / slots);
        int first = 0;
        for (int z = 0; z < B; ++z) {
            const int groups = plan.items[z];
            const int gpc = max(gpi_all * NW, (groups + A.nsplit - 1) / A.nsplit);  // groups per chunk
            plan.tpi[z] = gpc;
            plan.items[z] = (groups + gpc - 1) / gpc;
            plan.first[z] = first;
            first += plan.items[z] * A.n_kv;
        }
        plan.first[B] = first;
        // Item order: every (stream, kv head)'s chunks but its last, then all
        // the last chunks.  The last chunks land in the CTAs' final round, so the
        // merge (run by the chunk that finishes last, normally one of these)
        // comes after a CTA's own chunks instead of delaying its next one.
        int fn = 0;
        for (int z = 0; z < B; ++z) {
            plan.firstn[z] = fn;
            fn += (plan.items[z] > 0 ? plan.items[z] - 1 : 0) * A.n_kv;
        }
        plan.firstn[B] = fn;
    }
    // The plan above reads the ring states before the dependency wait: they are
    // written only by the o-proj after this kernel (it commits the layer's
    // append) and by host-ordered copies and kernels that never let their
    // dependents start early, so no kernel still running can change them.  q,
    // the newest K/V row and the output buffer are touched only after the wait.
    __syncthreads();

    // Item i -> (stream z, kv head h, chunk split): every pair's chunks but
    // its last, then the last chunks (see the plan above).
    auto map_item = [&](int item, int& z, int& h, int& split) {
        z = 0;
        if (item < plan.firstn[B]) {  // a chunk other than its pair's last (the pair has >= 2)
            while (z + 1 < B && item >= plan.firstn[z + 1]) ++z;
            const int local = item - plan.firstn[z], per_head = plan.items[z] - 1;
            h = local / per_head;
            split = local - h * per_head;
        } else {  // the last chunk of pair j, pairs in (stream, kv head) order
            int j = item - plan.firstn[B];
            while (plan.items[z] == 0 || j >= A.n_kv) {
                if (plan.items[z] > 0) j -= A.n_kv;
                ++z;
            }
            h = j;
            split = plan.items[z] - 1;
        }
    };
    // Every K/V row but the ones the q|k|v launch just appended (token len - 1
    // of each stream) is final, so each warp copies the first group of this
    // CTA's first chunk now, ahead of the dependency wait, unless that group
    // holds the newest token.
    int pre = 0;
    if ((int)blockIdx.x < plan.first[B]) {
        int z, h, split;
        map_item(blockIdx.x, z, h, split);
        const int per = plan.tpi[z] * TPG;
        const int t_begin = plan.mask_start[z] + split * per;
        const int t_end = min(plan.len[z], t_begin + per);
        const int t0 = t_begin + warp * TPG, ntok = min(TPG, t_end - t0);
        if (ntok > 0 && (t0 + ntok < plan.len[z] || !A.pre_append)) {
            if (lane == 0)
                attn_issue_group<G, D>(A, z, h, t_begin, t_end, plan.start[z], ring_smem, wbar, warp, 0, hd);
            pre = 1;
        }
        __syncwarp();
    }
    pdl_wait_prior_grids();

    if (blockIdx.x == 0)
        for (int z = 0; z < B; ++z)
            if (plan.items[z] == 0) {
                float* out = A.out + z * A.out_stride;
                for (int i = tid; i < A.n_heads * hd; i += kAttnThreads) {
                    out[i] = 0.f;
                    if (A.xop) xop_store(A.xop, i, z, 0.f);
                }
            }

    const int hd4 = hd / 4;
    uint32_t phase = 0;  // parity of the next completion of each of this warp's stages
    const int n_out = G * hd4;  // float4 outputs per (stream, kv head)
    const int total = plan.first[B];
    for (int item = blockIdx.x; item < total; item += gridDim.x) {
        __syncthreads();  // shared partials of the previous chunk are consumed
        int z, h, split;
        map_item(item, z, h, split);
        const int n_active = plan.items[z];
        const int len = plan.len[z];
        const int per = plan.tpi[z] * TPG;
        const int t_begin = plan.mask_start[z] + split * per;
        const int t_end = min(len, t_begin + per);
        const int ring_start = plan.start[z];

        attn_chunk_warps<G, D>(A, z, h, t_begin, t_end, ring_start, ring_smem, wbar, wacc, wml, phase, warp, lane, hd,
                               item == (int)blockIdx.x ? pre : 0);
        __syncthreads();
        const size_t acc_stride = (size_t)G * hd;
        const size_t ml_base = (size_t)A.n_kv * A.nsplit * acc_stride;
        float* part = A.part + z * A.part_stride;
        float* pacc = part + ((size_t)h * A.nsplit + split) * acc_stride;
        float* pml = part + ml_base + ((size_t)h * A.nsplit + split) * G * 2;
        for (int o = tid; o < n_out; o += kAttnThreads) {
            const int g = o / hd4, d = (o - g * hd4) * 4;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < NW; ++w) M = fmaxf(M, wml[w][g][0]);
            float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
            float L = 0.f;
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                const float mw = wml[w][g][0];
                const float e = mw == -INFINITY ? 0.f : expf(mw - M);
                const float4 a = *reinterpret_cast<const float4*>(&wacc[w][g][d]);
                sum.x = fmaf(e, a.x, sum.x);
                sum.y = fmaf(e, a.y, sum.y);
                sum.z = fmaf(e, a.z, sum.z);
                sum.w = fmaf(e, a.w, sum.w);
                L = fmaf(e, wml[w][g][1], L);
            }
            *reinterpret_cast<float4*>(pacc + (size_t)g * hd + d) = sum;
            if (d == 0) {
                pml[g * 2] = M;
                pml[g * 2 + 1] = L;
            }
        }
        __threadfence();
        __syncthreads();
        unsigned* tickets = A.tickets + (size_t)z * A.n_kv;
        if (tid == 0) {
            const unsigned ticket = atomicAdd(&tickets[h], 1u);
            flag_s = (ticket == (unsigned)(n_active - 1)) ? 1 : 0;
        }
        __syncthreads();
        if (!flag_s) continue;
        __threadfence();

        // Last chunk of this (stream, kv head): merge every chunk, fixed order.
        const float* bacc = part + (size_t)h * A.nsplit * acc_stride;
        const float* bml = part + ml_base + (size_t)h * A.nsplit * G * 2;
        for (int g = warp; g < G; g += NW) {
            float ms[2], ls[2];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int sp = lane + 32 * r;
                ms[r] = sp < n_active ? __ldcg(bml + ((size_t)sp * G + g) * 2) : -INFINITY;
                ls[r] = sp < n_active ? __ldcg(bml + ((size_t)sp * G + g) * 2 + 1) : 0.f;
            }
            float M = fmaxf(ms[0], ms[1]);
#pragma unroll
            for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(FULL, M, o));
            float w[2], L = 0.f;
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                w[r] = ms[r] == -INFINITY ? 0.f : expf(ms[r] - M);
                L = fmaf(ls[r], w[r], L);
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(FULL, L, o);
            const float invL = L > 0.f ? 1.0f / L : 0.f;
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int sp = lane + 32 * r;
                if (sp < n_active) w_s[g][sp] = w[r] * invL;
            }
        }
        __syncthreads();
        float* out = A.out + z * A.out_stride + (size_t)h * G * hd;
        for (int o = tid; o < n_out; o += kAttnThreads) {
            const int g = o / hd4, d = (o - g * hd4) * 4;
            const float* pv = bacc + (size_t)g * hd + d;
            float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int s0 = 0; s0 < n_active; s0 += 16) {  // 16 independent loads in flight
                float4 v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    v[j] = s0 + j < n_active ? __ldcg(reinterpret_cast<const float4*>(pv + (size_t)(s0 + j) * acc_stride))
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    if (s0 + j < n_active) {
                        const float wsp = w_s[g][s0 + j];
                        sum.x = fmaf(wsp, v[j].x, sum.x);
                        sum.y = fmaf(wsp, v[j].y, sum.y);
                        sum.z = fmaf(wsp, v[j].z, sum.z);
                        sum.w = fmaf(wsp, v[j].w, sum.w);
                    }
                }
            }
            *reinterpret_cast<float4*>(out + (size_t)g * hd + d) = sum;
            if (A.xop) {
                const int k0 = (h * G + g) * hd + d;
                xop_store(A.xop, k0, z, sum.x);
                xop_store(A.xop, k0 + 1, z, sum.y);
                xop_store(A.xop, k0 + 2, z, sum.z);
                xop_store(A.xop, k0 + 3, z, sum.w);
            }
        }
        if (tid == 0) tickets[h] = 0u;
    }
}

}  // namespace

bool attn_supported(int n_heads, int n_kv, int hd) {
    if (n_kv <= 0 || n_heads % n_kv) return false;
    const int G = n_heads / n_kv;
    if (G > kTile * 4) return false;
    const int vec = (hd % 4 == 0) ? 4 : 1;
    return (G * hd / vec) <= kMaxAcc * kAttnThreads;
}

// ---- cluster variant for one stream and short contexts ----------------------
// One thread-block cluster of CS CTAs per kv head: the CTAs split the head's
// live tokens evenly, run the warp-per-group loop above, combine their warps in
// shared memory, and store the CTA's (m, l, acc) straight into the leader's
// shared memory (st.shared::cluster).  After one cluster barrier the leader
// merges the CS partials in rank order.  No partials in global memory, no
// tickets and no merge loads: the round trips that dominate attention over a
// few hundred tokens are gone.  The context is known on the host, which picks
// this kernel only up to kAttnClusterMaxTokens live tokens.
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
    uint32_t d;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
    return d;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float4 v) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w)
                 : "memory");
}
__device__ __forceinline__ void st_cluster_v2(uint32_t addr, float a, float b) {
    asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 136 registers: 3 warps x 4352 + a GEMV CTA's 17 x 3072 = 65280 <= 65536.
template <int G, int CS>
__global__ void __maxnreg__(136) attn_cluster_kernel(const AttnArgs A) {
    constexpr int TPG = 32 / G;
    constexpr int NW = kClusterWarps;
    constexpr int NT = NW * 32;
    constexpr int HD = 128;
    // [NW][K rows | V rows] slots, then the leader's merge buffer:
    // acc [CS][G][hd] followed by (m, l) [CS][G][2]
    extern __shared__ __align__(128) unsigned char ring_smem[];
    constexpr int D = kClusterStages;
    __shared__ uint64_t wbar[NW][D];
    __shared__ __align__(16) float wacc[NW][G][HD];
    __shared__ float wml[NW][G][2];
    __shared__ int range_s[4];  // t_begin, t_end, ring start, live length
    const int tid = threadIdx.x;
    const int hd = A.hd, hd4 = hd / 4, n_out = G * hd4;
    const uint32_t rank = cluster_rank();
    const int h = blockIdx.x / CS;
    float* macc = reinterpret_cast<float*>(ring_smem + (size_t)NW * D * 2 * TPG * hd * 4);
    float* mml = macc + (size_t)CS * G * hd;

    if (tid < NW * D) mbar_init(&wbar[tid / D][tid % D], 1);
    if (tid == 0) fence_barrier_init();
    // First cluster phase: every CTA of the cluster has started.  Its wait sits
    // just before the first store into the leader's shared memory, so it costs
    // nothing on the path (a CTA may write another's shared memory only once
    // that CTA is running).
    cluster_arrive_relaxed();
    pdl_allow_dependents();
    // The ring state is read before the dependency wait.  In a step graph the
    // only writer is the o-proj launch that commits each layer's append: this
    // step's runs after this kernel, and earlier steps' finished before this
    // graph began (consecutive graph launches are fully ordered).  q and the
    // newest K/V row come from the q|k|v launch just before and are read after
    // the wait.
    if (tid == 0) {
        KvState st = A.st[0];
        if (A.pre_append) st = kv_after_single_append(st, A.kv_window, A.cap);
        const int len = st.len;
        const int ms = (A.cfg_window > 0 && len > A.cfg_window) ? len - A.cfg_window : 0;
        const int groups = (len - ms + TPG - 1) / TPG;
        const int gpc = (groups + CS - 1) / CS;  // groups of this CTA
        const int g0 = min(groups, (int)rank * gpc), g1 = min(groups, g0 + gpc);
        range_s[0] = ms + g0 * TPG;
        range_s[1] = min(len, ms + g1 * TPG);
        range_s[2] = st.start;
        range_s[3] = len;
    }
    __syncthreads();
    // Every K/V row but the one the q|k|v launch just appended (token len - 1,
    // the end of the newest group) is final: a warp whose first group ends
    // before it copies that group now, ahead of the dependency wait.
    int pre = 0;
    for (int k = 0; k < D; ++k) {
        const int warp = tid >> 5, t0 = range_s[0] + (warp + NW * k) * TPG;
        const int ntok = min(TPG, range_s[1] - t0);
        if (pre == k && ntok > 0 && (t0 + ntok < range_s[3] || !A.pre_append)) {
            if ((tid & 31) == 0)
                attn_issue_group<G, D, NW>(A, 0, h, range_s[0], range_s[1], range_s[2], ring_smem, wbar, warp, k, hd);
            pre = k + 1;
        }
        __syncwarp();
    }
    pdl_wait_prior_grids();
    uint32_t phase = 0;
    attn_chunk_warps<G, D, NW>(A, 0, h, range_s[0], range_s[1], range_s[2], ring_smem, wbar, wacc, wml, phase,
                           tid >> 5, tid & 31, hd, pre);
    __syncthreads();

    // This CTA's partial into the leader's buffer, slot `rank`.
    cluster_wait();
    const uint32_t lacc = cluster_map(smem_addr(macc), 0), lml = cluster_map(smem_addr(mml), 0);
    for (int o = tid; o < n_out; o += NT) {
        const int g = o / hd4, d = (o - g * hd4) * 4;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, wml[w][g][0]);
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float mw = wml[w][g][0];
            const float e = mw == -INFINITY ? 0.f : expf(mw - M);
            const float4 a = *reinterpret_cast<const float4*>(&wacc[w][g][d]);
            sum.x = fmaf(e, a.x, sum.x);
            sum.y = fmaf(e, a.y, sum.y);
            sum.z = fmaf(e, a.z, sum.z);
            sum.w = fmaf(e, a.w, sum.w);
            L = fmaf(e, wml[w][g][1], L);
        }
        st_cluster_v4(lacc + (uint32_t)((((size_t)rank * G + g) * hd + d) * 4), sum);
        if (d == 0) st_cluster_v2(lml + (uint32_t)(((size_t)rank * G + g) * 2 * 4), M, L);
    }
    cluster_sync_all();  // every partial has landed in the leader's buffer
    if (rank != 0) return;

    // Merge the CS partials in rank order (the same weights as the global merge).
    float* out = A.out + (size_t)h * G * hd;
    for (int o = tid; o < n_out; o += NT) {
        const int g = o / hd4, d = (o - g * hd4) * 4;
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < CS; ++r) M = fmaxf(M, mml[(r * G + g) * 2]);
        float w[CS], L = 0.f;
#pragma unroll
        for (int r = 0; r < CS; ++r) {
            const float mr = mml[(r * G + g) * 2];
            w[r] = mr == -INFINITY ? 0.f : expf(mr - M);
            L = fmaf(mml[(r * G + g) * 2 + 1], w[r], L);
        }
        const float invL = L > 0.f ? 1.0f / L : 0.f;
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < CS; ++r) {
            const float wr = w[r] * invL;
            const float4 a = *reinterpret_cast<const float4*>(macc + ((size_t)r * G + g) * hd + d);
            sum.x = fmaf(wr, a.x, sum.x);
            sum.y = fmaf(wr, a.y, sum.y);
            sum.z = fmaf(wr, a.z, sum.z);
            sum.w = fmaf(wr, a.w, sum.w);
        }
        *reinterpret_cast<float4*>(out + (size_t)g * hd + d) = sum;
        if (A.xop) {
            const int k0 = (h * G + g) * hd + d;
            xop_store(A.xop, k0, 0, sum.x);
            xop_store(A.xop, k0 + 1, 0, sum.y);
            xop_store(A.xop, k0 + 2, 0, sum.z);
            xop_store(A.xop, k0 + 3, 0, sum.w);
        }
    }
}

size_t attn_smem_bytes(int n_heads, int n_kv, int hd) {
    const int G = n_heads / n_kv;
    const int pad = (hd % 4 == 0) ? 4 : 1;
    const size_t floats = (size_t)G * hd + 4 * kTile * (hd + pad) + (size_t)G * kTile + 3 * G +
                          (size_t)G * kMaxSplits + 4;
    return floats * 4;
}

// Resident CTAs of the persistent attention grid: as many as fit on every SM.
int attn_grid_ctas(int n_heads, int n_kv, int hd) {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    }
    const size_t smem = attn_smem_bytes(n_heads, n_kv, hd) + sizeof(AttnPlan) + 1024;
    int per_sm = (int)((227 * 1024) / smem);
    if (per_sm < 1) per_sm = 1;
    if (per_sm > 4) per_sm = 4;
    return sms * per_sm;
}

// Persistent grid of the warp-per-chunk kernel: four 4-warp CTAs per SM
// (1-stage rings: 32 KB + 10 KB of shared memory, at most 128 registers;
// more warps hide the load latency better than deeper rings per warp).
int attn_warp_grid_ctas() {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    }
    return 4 * sms;
}

int attn_max_splits() { return kMaxSplits; }

int attn_splits_for(int n_kv, int num_sms) {
    int s = (2 * num_sms + n_kv - 1) / n_kv;
    if (s < 1) s = 1;
    if (s > kMaxSplits) s = kMaxSplits;
    return s;
}

cudaError_t attn_prepare(int /*dev*/) {
    cudaError_t e = cudaSuccess;
    for (void* k : {(void*)attn_warp_kernel<4, 1>, (void*)attn_warp_kernel<4, 2>, (void*)attn_warp_kernel<8, 1>,
                    (void*)attn_warp_kernel<8, 2>}) {
        e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
    }
    e = cudaFuncSetAttribute(attn_split_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(attn_split_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                200 * 1024);
}

namespace {
size_t attn_cluster_smem(int G, int hd, int cs) {
    return (size_t)kClusterWarps * kClusterStages * 2 * (32 / G) * hd * 4 + (size_t)cs * G * (hd + 2) * 4;
}
void* attn_cluster_fn(int G, int cs) {
    if (G == 4) return cs == 16 ? (void*)attn_cluster_kernel<4, 16> : (void*)attn_cluster_kernel<4, 8>;
    return cs == 16 ? (void*)attn_cluster_kernel<8, 16> : (void*)attn_cluster_kernel<8, 8>;
}
}  // namespace

int attn_cluster_size(int n_heads, int n_kv, int hd) {
    const int G = n_kv > 0 ? n_heads / n_kv : 0;
    if (n_kv <= 0 || n_heads % n_kv || (G != 4 && G != 8) || hd % 4 || hd <= 0 || hd > 128) return 0;
    // 16 CTAs per kv head where the device can hold every cluster at once
    // (a non-portable size), else the portable 8.  Function attributes belong
    // to a device, so the answer is kept per device (and per shape).
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static int cached[kMaxDevices][2][129] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
    std::lock_guard<std::mutex> lock(mu);
    int& c = cached[dev][G == 8][hd];
    if (c == 0) {
        c = -1;
        for (int cs : {16, 8}) {
            void* k = attn_cluster_fn(G, cs);
            if (cs == 16 && cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
                cudaGetLastError();
                continue;
            }
            if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)attn_cluster_smem(G, 128, cs)) != cudaSuccess) {  // any head_dim
                cudaGetLastError();
                continue;
            }
            // the whole 228 KB for shared memory, so that a GEMV CTA fits beside this one
            if (cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess)
                cudaGetLastError();
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(n_kv * cs, 1, 1);
            cfg.blockDim = dim3(kClusterWarps * 32, 1, 1);
            cfg.dynamicSmemBytes = attn_cluster_smem(G, hd, cs);
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = cs;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) != cudaSuccess) {
                cudaGetLastError();
                continue;
            }
            if (n >= n_kv) {
                c = cs;
                break;
            }
        }
    }
    return c > 0 ? c : 0;
}

int attn_cluster_max_tokens() { return kAttnClusterMaxTokens; }

cudaError_t launch_attention_cluster(const AttnArgs& a, cudaStream_t s, bool pdl) {
    const int cs = attn_cluster_size(a.n_heads, a.n_kv, a.hd);
    if (cs == 0 || a.n_streams > 1) return cudaErrorInvalidValue;
    const int G = a.n_heads / a.n_kv;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_kv * cs, 1, 1);
    cfg.blockDim = dim3(kClusterWarps * 32, 1, 1);
    cfg.dynamicSmemBytes = attn_cluster_smem(G, a.hd, cs);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    void* args[] = {(void*)&a};
    return cudaLaunchKernelExC(&cfg, attn_cluster_fn(G, cs), args);
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl) {
    if (a.n_streams > 8 || a.nsplit < 1 || a.nsplit > kMaxSplits) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    const int B = a.n_streams > 1 ? a.n_streams : 1;
    int grid = attn_grid_ctas(a.n_heads, a.n_kv, a.hd);
    const long long max_items = (long long)B * a.n_kv * a.nsplit;
    if (grid > max_items) grid = (int)max_items;
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(kAttnThreads, 1, 1);
    cfg.dynamicSmemBytes = attn_smem_bytes(a.n_heads, a.n_kv, a.hd);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    void* args[] = {(void*)&a};
    const int G = a.n_heads / a.n_kv;
    void* k = (a.hd % 4 == 0) ? (void*)attn_split_kernel<4> : (void*)attn_split_kernel<1>;
    if (a.hd % 4 == 0 && a.hd <= 128 && (G == 4 || G == 8)) {
        // 1-stage rings: four CTAs (16 warps) per SM
        const int D = 1;
        k = G == 4 ? (D == 1 ? (void*)attn_warp_kernel<4, 1> : (void*)attn_warp_kernel<4, 2>)
                   : (D == 1 ? (void*)attn_warp_kernel<8, 1> : (void*)attn_warp_kernel<8, 2>);
        cfg.dynamicSmemBytes = (size_t)(kAttnThreads / 32) * D * 2 * (32 / G) * a.hd * 4;
        int g2 = attn_warp_grid_ctas();
        if (g2 > max_items) g2 = (int)max_items;
        cfg.gridDim = dim3(g2 > 0 ? g2 : 1, 1, 1);
    }
    return cudaLaunchKernelExC(&cfg, k, args);
}

}  // namespace vox
