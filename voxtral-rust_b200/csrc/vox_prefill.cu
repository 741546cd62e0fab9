// vox_prefill.cu -- batched prompt prefill on the 5th-generation tensor cores.
//
// The reference fills the cache one position at a time (decoder.rs:88-155 per
// token).  Here a pass of T prompt tokens goes through each layer at once:
//
//   * every linear is one dense GEMM  P[t, r] = sum_k W[r, k] X[t, k]  on
//     tcgen05 (M = 128 weight rows, N = 2 tn: the bf16 hi and lo parts of tn
//     tokens' f32 activations, summed in the epilogue), reading the weights
//     pre-tiled for the multi-stream GEMM;
//   * attention is causal over the cache as it was before the pass plus the
//     pass's own keys, each token seeing exactly the window it would see after
//     its own single-token append (kv.rs:48-88, then ops.rs:92-96);
//   * the pass's keys and values enter the ring only after its attention has
//     read them, at the slots T single-token appends would have used, so
//     eviction inside a pass leaves the ring as the token loop would.
//
// X operand layout ("prefill operand"): per token block nb (tn tokens) and K
// block kb (64 elements) one contiguous slab of N = 2 tn rows x 64 bf16 in the
// UMMA canonical K-major layout: K step s (16 elements) at s * N * 32 bytes,
// core matrix (n8, k2) at (k2 * N / 8 + n8) * 128 bytes, row n & 7 at 16-byte
// stride.  Row tt < tn holds hi = bf16(x) of token nb * tn + tt, row tn + tt
// holds lo = bf16(x - hi).  Slab (nb, kb) starts at (nb * kbt + kb) * N * 128.
#include <cuda_runtime.h>
#include <math.h>

#include "vox_device.cuh"
#include "vox_tcgen05.cuh"

namespace vox {

namespace {

constexpr int kPfStages = 4;
constexpr int kPfABytes = 128 * 64 * 2;                // one pre-tiled weight block
constexpr int kPfMaxSlab = 256 * 128;                  // X slab of one K block, N <= 256
constexpr int kPfStageBytes = kPfABytes + kPfMaxSlab;  // 48 KB
constexpr int kPfThreads = 192;                        // w0 producer, w1 MMA, w2..w5 epilogue
constexpr uint32_t kPfTmemCols = 512;                  // two accumulators of up to 256 columns
constexpr unsigned kFull = 0xFFFFFFFFu;

struct PfItem {
    int tile, ks, nb, kb0, kb1;
};

// Item i -> (weight tile, K split, token block), token block fastest: the
// CTAs that run at the same time share weight blocks, which L2 then serves.
__device__ __forceinline__ PfItem pf_item(const PfGemmArgs& A, int i) {
    PfItem it;
    it.nb = i % A.nblocks;
    const int j = i / A.nblocks;
    it.ks = j % A.splits;
    it.tile = j / A.splits;
    it.kb0 = (int)((long long)A.kbt * it.ks / A.splits);
    it.kb1 = (int)((long long)A.kbt * (it.ks + 1) / A.splits);
    return it;
}

__global__ void __launch_bounds__(kPfThreads, 1) pf_gemm_kernel(const __grid_constant__ PfGemmArgs A) {
    extern __shared__ __align__(1024) unsigned char smem[];
    unsigned char* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPfStages * kPfStageBytes);
    uint64_t* empty = full + kPfStages;
    uint64_t* acc_full = empty + kPfStages;  // [2]
    uint64_t* acc_empty = acc_full + 2;      // [2]
    uint32_t* tmem_s = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n = 2 * A.tn;
    const uint32_t slab = (uint32_t)n * 128u;
    const int n_items = A.tiles * A.splits * A.nblocks;

    if (tid == 0) {
        for (int s = 0; s < kPfStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_s)),
                     "r"(kPfTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tmem = *tmem_s;

    if (warp == 0) {
        // ---- producer: weight block + X slab of every K block of every item ----
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = true;
            for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
                const PfItem it = pf_item(A, i);
                for (int kb = it.kb0; kb < it.kb1; ++kb, ++g) {
                    const int slot = (int)(g % kPfStages);
                    if (g >= (uint32_t)kPfStages && !mbar_wait(&empty[slot], ((g / kPfStages) - 1) & 1)) {
                        raise_error(A.err, ERR_EMPTY_WAIT);
                        ok = false;
                        break;
                    }
                    unsigned char* dst = ring + (size_t)slot * kPfStageBytes;
                    mbar_arrive_expect_tx(&full[slot], (uint32_t)kPfABytes + slab);
                    bulk_copy_g2s_nohint(dst, A.wt + ((size_t)it.tile * A.kbt + kb) * kPfABytes, kPfABytes,
                                         &full[slot]);
                    bulk_copy_g2s_nohint(dst + kPfABytes, A.xop + ((size_t)it.nb * A.kbt + kb) * slab, slab,
                                         &full[slot]);
                }
            }
            // no copy may be in flight when the CTA exits
            const uint32_t first = g > (uint32_t)kPfStages ? g - kPfStages : 0u;
            for (uint32_t s = first; s < g; ++s)
                if (!mbar_wait(&full[s % kPfStages], (s / kPfStages) & 1)) raise_error(A.err, ERR_DRAIN_WAIT);
        }
        return;  // the barriers below count warps 1..5 only
    }

    if (warp == 1) {
        // ---- MMA issuer: 4 x (M 128, N n, K 16) per K block ----
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_bf16(128, n);
            const uint32_t b_kstep = (uint32_t)n * 32u, b_lbo = (uint32_t)n * 16u;
            uint32_t g = 0;
            bool ok = true;
            int local = 0;
            for (int i = blockIdx.x; i < n_items; i += gridDim.x, ++local) {
                const PfItem it = pf_item(A, i);
                const int ab = local & 1;
                if (ok && local >= 2 && !mbar_wait(&acc_empty[ab], ((local - 2) >> 1) & 1)) {
                    raise_error(A.err, ERR_FULL_WAIT);
                    ok = false;
                }
                tmem_fence_after();
                const uint32_t d = tmem + (uint32_t)(ab * 256);
                for (int kb = it.kb0; kb < it.kb1 && ok; ++kb, ++g) {
                    const int slot = (int)(g % kPfStages);
                    if (!mbar_wait(&full[slot], (g / kPfStages) & 1)) {
                        raise_error(A.err, ERR_FULL_WAIT);
                        ok = false;
                        break;
                    }
                    tmem_fence_after();
                    const uint32_t a_addr = smem_addr(ring + (size_t)slot * kPfStageBytes);
                    const uint32_t b_addr = a_addr + (uint32_t)kPfABytes;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint64_t ad = umma_desc(a_addr + (uint32_t)j * 4096u, 2048u, 128u);
                        const uint64_t bd = umma_desc(b_addr + (uint32_t)j * b_kstep, b_lbo, 128u);
                        umma_f16(d, ad, bd, idesc, (kb > it.kb0 || j > 0) ? 1u : 0u);
                    }
                    umma_commit(&empty[slot]);  // frees the stage once these MMAs have read it
                }
                umma_commit(&acc_full[ab]);  // accumulator ready for the epilogue
            }
        }
        __syncwarp();
    } else {
        // ---- epilogue warps 2..5: TMEM lanes 32 * (warp % 4) .. + 31 ----
        const int q = warp & 3;
        const int row = q * 32 + lane;
        int local = 0;
        for (int i = blockIdx.x; i < n_items; i += gridDim.x, ++local) {
            const PfItem it = pf_item(A, i);
            const int ab = local & 1;
            if (!mbar_wait(&acc_full[ab], (local >> 1) & 1)) raise_error(A.err, ERR_FULL_WAIT);
            tmem_fence_after();
            const int r = it.tile * 128 + row;
            const bool live = r < A.rows;
            float* out = A.part + (size_t)it.ks * A.T * A.rows + r;
            const int t0 = it.nb * A.tn;
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * 256);
            for (int c = 0; c < A.tn; c += 16) {
                uint32_t hi[16], lo[16];
                tmem_ld16x2(taddr + (uint32_t)c, taddr + (uint32_t)(A.tn + c), hi, lo);
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const int t = t0 + c + u;
                    if (live && t < A.T) out[(size_t)t * A.rows] = __uint_as_float(hi[u]) + __uint_as_float(lo[u]);
                }
            }
            tmem_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[ab]);
        }
    }

    // TMEM is released by the warp that allocated it, after every reader is done.
    tmem_fence_before();
    named_barrier_sync(1, kPfThreads - 32);
    if (warp == 1) {
        tmem_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPfTmemCols)
                     : "memory");
    }
}

// Eight consecutive elements k .. k + 7 of token t into the prefill operand.
__device__ __forceinline__ void pf_store8(unsigned char* xop, int tn, int kbt, int t, int k, const float (&v)[8]) {
    const int nb = t / tn, tt = t - nb * tn, n = 2 * tn;
    const int kb = k >> 6, kk = k & 63;
    const int s = kk >> 4, k2 = (kk >> 3) & 1;
    unsigned char* base = xop + ((size_t)nb * kbt + kb) * (size_t)n * 128 + (size_t)s * n * 32 + (size_t)k2 * n * 16;
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
        const uint16_t h0 = f32_to_bf16_bits(v[j]), h1 = f32_to_bf16_bits(v[j + 1]);
        const uint16_t l0 = f32_to_bf16_bits(v[j] - bf16_bits_to_f32(h0));
        const uint16_t l1 = f32_to_bf16_bits(v[j + 1] - bf16_bits_to_f32(h1));
        hi[j >> 1] = (uint32_t)h0 | ((uint32_t)h1 << 16);
        lo[j >> 1] = (uint32_t)l0 | ((uint32_t)l1 << 16);
    }
    const int lr = tn + tt;
    *reinterpret_cast<uint4*>(base + (tt >> 3) * 128 + (tt & 7) * 16) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(base + (lr >> 3) * 128 + (lr & 7) * 16) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

// Ordered sum of the K-split partials of element e of token t.
__device__ __forceinline__ float pf_sum(const float* part, int splits, int T, int rows, int t, int e) {
    float y = part[(size_t)t * rows + e];
    for (int s = 1; s < splits; ++s) y += part[((size_t)s * T + t) * rows + e];
    return y;
}

// One CTA per token of the padded pass.  The hidden row h[t] becomes either
// the embedding row of the token (plus the adapter row at its position), or
// h[t] + (the GEMM's split sum) (decoder.rs:138-139, 151-152); then RMSNorm
// (math.rs:17-25) times the gain goes into the prefill operand.  Padding
// tokens (t >= T) write zero rows.
__global__ void __launch_bounds__(256) pf_norm_kernel(const __grid_constant__ PfNormArgs A) {
    __shared__ float red[8];
    const int t = blockIdx.x, tid = threadIdx.x;
    const bool live = t < A.T;
    float ss = 0.0f;
    if (live) {
        float* h = A.h + (size_t)t * A.dim;
        if (A.embed) {
            int tok = A.tokens[t];
            if (tok < 0 || tok >= A.vocab) {
                if (tid == 0) raise_error(A.err, ERR_TOKEN_RANGE);
                tok = 0;
            }
            const uint16_t* er = A.embed + (size_t)tok * A.dim;
            const float* ad = A.adapter ? A.adapter + (size_t)((A.pos0 + t) % A.adapter_cap) * A.dim : nullptr;
            for (int e = tid; e < A.dim; e += 256) {
                float v = bf16_bits_to_f32(er[e]);
                if (ad) v = __fadd_rn(ad[e], v);
                h[e] = v;
                ss += __fmul_rn(v, v);
            }
        } else {
            for (int e = tid; e < A.dim; e += 256) {
                const float v = __fadd_rn(h[e], pf_sum(A.part, A.splits, A.T, A.dim, t, e));
                h[e] = v;
                ss += __fmul_rn(v, v);
            }
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();  // also orders this block's h writes before the reads below
    if (!A.xop) return;
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += red[w];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)A.dim), A.eps)));
    const float* h = A.h + (size_t)t * A.dim;
    for (int k8 = tid; k8 < A.dim / 8; k8 += 256) {
        float v[8];
        if (live) {
            const float4 a = *reinterpret_cast<const float4*>(h + k8 * 8);
            const float4 b = *reinterpret_cast<const float4*>(h + k8 * 8 + 4);
            const float4 g0 = __ldg(reinterpret_cast<const float4*>(A.gain + k8 * 8));
            const float4 g1 = __ldg(reinterpret_cast<const float4*>(A.gain + k8 * 8 + 4));
            const float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
            const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(__fmul_rn(x[j], inv), g[j]);  // math.rs:23-24 order
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = 0.0f;
        }
        pf_store8(A.xop, A.tn, A.dim / 64, t, k8 * 8, v);
    }
}

// q|k|v split sums -> RoPE (math.rs:30-65) on q and k at position pos0 + t ->
// q [T, q_dim], the pass's keys and values [T, kv_dim].  One thread per
// (token, element pair).
__global__ void __launch_bounds__(256) pf_qkv_kernel(const __grid_constant__ PfQkvArgs A) {
    const int pairs = (A.q_dim + 2 * A.kv_dim) / 2;
    const long long total = (long long)A.T * pairs;
    const int half = A.head_dim / 2;
    const int rows = A.q_dim + 2 * A.kv_dim;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(e / pairs), r = 2 * (int)(e - (long long)t * pairs);
        const float y0 = pf_sum(A.part, A.splits, A.T, rows, t, r);
        const float y1 = pf_sum(A.part, A.splits, A.T, rows, t, r + 1);
        if (r < A.q_dim + A.kv_dim) {
            const int rr = r < A.q_dim ? r : r - A.q_dim;
            const int d = rr % A.head_dim;
            long long p = A.pos0 + t;
            if (p >= A.max_pos) {
                if (r == 0) raise_error(A.err, ERR_POS_RANGE);
                p = 0;
            }
            const float c = A.rope_cos[p * half + d / 2], sn = A.rope_sin[p * half + d / 2];
            const float o0 = __fsub_rn(__fmul_rn(y0, c), __fmul_rn(y1, sn));
            const float o1 = __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, c));
            float* dst = r < A.q_dim ? A.q + (size_t)t * A.q_dim + rr : A.kc + (size_t)t * A.kv_dim + rr;
            *reinterpret_cast<float2*>(dst) = make_float2(o0, o1);
        } else {
            const int rr = r - A.q_dim - A.kv_dim;
            *reinterpret_cast<float2*>(A.vc + (size_t)t * A.kv_dim + rr) = make_float2(y0, y1);
        }
    }
}

// Causal attention of a pass (ops.rs:66-132 per token).  Logical key j of the
// sequence "cache before the pass, then the pass's tokens": j < len0 is ring
// slot (start0 + j) % cap, j >= len0 is pass token j - len0.  Token t sees
// keys [len0 + t + 1 - n_t, len0 + t] with n_t = min(len0 + t + 1, win).
// Grid (ceil(T / 8), n_kv), 4 warps: warp w takes q head w of the kv head's
// group for 8 tokens; 32-key tiles of K and V staged in shared memory, online
// softmax.  C = head_dim / 32.
constexpr int kPfQB = 8, kPfKT = 32;

template <int C>
__global__ void __launch_bounds__(128) pf_attn_kernel(const __grid_constant__ PfAttnArgs A) {
    extern __shared__ __align__(16) float sm[];
    constexpr int HD = 32 * C, KS = HD + 4;  // padded key rows: conflict-free float4 reads
    float* Ks = sm;                          // [32][KS]
    float* Vs = Ks + kPfKT * KS;             // [32][KS]
    float* Qs = Vs + kPfKT * KS;             // [4][8][HD]
    float* Ps = Qs + 4 * kPfQB * HD;         // [4][8][32]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hk = blockIdx.y, G = A.n_heads / A.n_kv;
    const int t0 = blockIdx.x * kPfQB, nq = min(kPfQB, A.T - t0);
    const int qd = A.n_heads * HD, kvd = A.n_kv * HD;
    const bool active = warp < G;
    const int h = hk * G + warp;  // this warp's q head

    // the queries of the group's heads for these tokens (ops.rs scales the dot)
    for (int e = tid; e < 4 * kPfQB * HD; e += 128) {
        const int w = e / (kPfQB * HD), qi = (e / HD) % kPfQB, d = e % HD;
        Qs[e] = (w < G && qi < nq) ? A.q[(size_t)(t0 + qi) * qd + (size_t)(hk * G + w) * HD + d] : 0.0f;
    }
    auto first_key = [&](int t) {
        const int hi = A.len0 + t;
        const int cnt = min(hi + 1, A.win);
        return hi + 1 - cnt;
    };
    const int j_lo = first_key(t0), j_hi = A.len0 + t0 + nq - 1;

    float o[kPfQB][C], m[kPfQB], l[kPfQB];
#pragma unroll
    for (int qi = 0; qi < kPfQB; ++qi) {
        m[qi] = -INFINITY;
        l[qi] = 0.0f;
#pragma unroll
        for (int c = 0; c < C; ++c) o[qi][c] = 0.0f;
    }
    const float* kr = A.k_ring + (size_t)hk * A.cap * HD;
    const float* vr = A.v_ring + (size_t)hk * A.cap * HD;
    float* P = Ps + warp * kPfQB * 32;

    for (int j0 = j_lo; j0 <= j_hi; j0 += kPfKT) {
        __syncthreads();  // previous tile fully consumed (and Qs written, first time)
        for (int e = tid; e < kPfKT * (HD / 4); e += 128) {
            const int kk = e / (HD / 4), d4 = (e - kk * (HD / 4)) * 4;
            const int j = j0 + kk;
            float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = kv4;
            if (j <= j_hi) {
                const float *ks, *vs;
                if (j < A.len0) {
                    const size_t slot = (size_t)((A.start0 + j) % A.cap);
                    ks = kr + slot * HD;
                    vs = vr + slot * HD;
                } else {
                    ks = A.kc + (size_t)(j - A.len0) * kvd + (size_t)hk * HD;
                    vs = A.vc + (size_t)(j - A.len0) * kvd + (size_t)hk * HD;
                }
                kv4 = *reinterpret_cast<const float4*>(ks + d4);
                vv4 = *reinterpret_cast<const float4*>(vs + d4);
            }
            *reinterpret_cast<float4*>(Ks + kk * KS + d4) = kv4;
            *reinterpret_cast<float4*>(Vs + kk * KS + d4) = vv4;
        }
        __syncthreads();
        if (!active) continue;
        // scores of key j0 + lane for the 8 tokens
        const float* q = Qs + warp * kPfQB * HD;
        float s[kPfQB];
#pragma unroll
        for (int qi = 0; qi < kPfQB; ++qi) s[qi] = 0.0f;
        const float* krow = Ks + lane * KS;
#pragma unroll 4
        for (int d = 0; d < HD; d += 4) {
            const float4 k4 = *reinterpret_cast<const float4*>(krow + d);
#pragma unroll
            for (int qi = 0; qi < kPfQB; ++qi) {
                const float4 q4 = *reinterpret_cast<const float4*>(q + qi * HD + d);
                s[qi] = fmaf(q4.x, k4.x, s[qi]);
                s[qi] = fmaf(q4.y, k4.y, s[qi]);
                s[qi] = fmaf(q4.z, k4.z, s[qi]);
                s[qi] = fmaf(q4.w, k4.w, s[qi]);
            }
        }
        const int j = j0 + lane;
#pragma unroll
        for (int qi = 0; qi < kPfQB; ++qi) {
            const int t = t0 + qi;
            const bool ok = qi < nq && j >= first_key(t) && j <= A.len0 + t;
            float sc = ok ? s[qi] * A.scale : -INFINITY;
            float mt = sc;
#pragma unroll
            for (int off = 16; off; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(kFull, mt, off));
            const float mn = fmaxf(m[qi], mt);
            float p = 0.0f, corr = 1.0f;
            if (mn != -INFINITY) {
                p = ok ? expf(sc - mn) : 0.0f;
                corr = m[qi] == -INFINITY ? 0.0f : expf(m[qi] - mn);
            }
            float ps = p;
#pragma unroll
            for (int off = 16; off; off >>= 1) ps += __shfl_xor_sync(kFull, ps, off);
            l[qi] = l[qi] * corr + ps;
            m[qi] = mn;
#pragma unroll
            for (int c = 0; c < C; ++c) o[qi][c] *= corr;
            P[qi * 32 + lane] = p;
        }
        __syncwarp();
#pragma unroll 4
        for (int kk = 0; kk < kPfKT; kk += 4) {
            float v[4][C];
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int c = 0; c < C; ++c) v[u][c] = Vs[(kk + u) * KS + lane + 32 * c];
#pragma unroll
            for (int qi = 0; qi < kPfQB; ++qi) {
                const float4 p4 = *reinterpret_cast<const float4*>(P + qi * 32 + kk);
#pragma unroll
                for (int c = 0; c < C; ++c) {
                    o[qi][c] = fmaf(p4.x, v[0][c], o[qi][c]);
                    o[qi][c] = fmaf(p4.y, v[1][c], o[qi][c]);
                    o[qi][c] = fmaf(p4.z, v[2][c], o[qi][c]);
                    o[qi][c] = fmaf(p4.w, v[3][c], o[qi][c]);
                }
            }
        }
        __syncwarp();
    }
    if (!active) return;
#pragma unroll
    for (int qi = 0; qi < kPfQB; ++qi) {
        if (qi >= nq) break;
        float* dst = A.out + (size_t)(t0 + qi) * qd + (size_t)h * HD;
        const float inv = l[qi] > 0.0f ? 1.0f / l[qi] : 0.0f;
#pragma unroll
        for (int c = 0; c < C; ++c) dst[lane + 32 * c] = o[qi][c] * inv;
    }
}

// f32 rows [T, K] -> prefill operand (zero rows for padding tokens).  One
// thread per (token, 8 elements).
__global__ void __launch_bounds__(256) pf_split_kernel(const float* __restrict__ src, int T, int Tp, int K,
                                                       unsigned char* xop, int tn) {
    const int k8s = K / 8;
    const long long total = (long long)Tp * k8s;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(e / k8s), k = 8 * (int)(e - (long long)t * k8s);
        float v[8];
        if (t < T) {
            const float4 a = *reinterpret_cast<const float4*>(src + (size_t)t * K + k);
            const float4 b = *reinterpret_cast<const float4*>(src + (size_t)t * K + k + 4);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
            v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = 0.0f;
        }
        pf_store8(xop, tn, K / 64, t, k, v);
    }
}

// w1|w3 split sums (row 2j = gate j, row 2j + 1 = up j) -> SiLU(gate) * up
// (math.rs:4-9, decoder.rs:147-150) -> prefill operand of w2.
__global__ void __launch_bounds__(256) pf_swiglu_kernel(const float* __restrict__ part, int splits, int T, int Tp,
                                                        int hidden, unsigned char* xop, int tn) {
    const int j8s = hidden / 8, rows = 2 * hidden;
    const long long total = (long long)Tp * j8s;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(e / j8s), j0 = 8 * (int)(e - (long long)t * j8s);
        float v[8];
        if (t < T) {
            float y[16];
#pragma unroll
            for (int u = 0; u < 16; u += 4) {
                const float4 a = *reinterpret_cast<const float4*>(part + (size_t)t * rows + 2 * j0 + u);
                y[u] = a.x; y[u + 1] = a.y; y[u + 2] = a.z; y[u + 3] = a.w;
            }
            for (int s = 1; s < splits; ++s) {
                const float* p = part + ((size_t)s * T + t) * rows + 2 * j0;
#pragma unroll
                for (int u = 0; u < 16; u += 4) {
                    const float4 a = *reinterpret_cast<const float4*>(p + u);
                    y[u] += a.x; y[u + 1] += a.y; y[u + 2] += a.z; y[u + 3] += a.w;
                }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float g = y[2 * j], up = y[2 * j + 1];
                v[j] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), up);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = 0.0f;
        }
        pf_store8(xop, tn, hidden / 64, t, j0, v);
    }
}

// The pass's keys and values into the ring at the slots T single-token
// appends use (the live end (start0 + len0 + t) % cap; kv.rs:48-88), only
// the last min(T, cap) tokens (earlier ones would be overwritten), then the
// layer's state after the T appends.
__global__ void __launch_bounds__(256) pf_commit_kernel(const __grid_constant__ PfCommitArgs A) {
    const int c4 = A.kv_dim / 4;
    const int first = A.T > A.cap ? A.T - A.cap : 0;
    const long long total = (long long)(A.T - first) * c4;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int t = first + (int)(e / c4), x = 4 * (int)(e % c4);
        const int hk = x / A.head_dim, d = x - hk * A.head_dim;
        const size_t slot = (size_t)((A.end0 + (long long)t) % A.cap);
        const size_t dst = ((size_t)hk * A.cap + slot) * A.head_dim + d;
        *reinterpret_cast<float4*>(A.k_ring + dst) = *reinterpret_cast<const float4*>(A.kc + (size_t)t * A.kv_dim + x);
        *reinterpret_cast<float4*>(A.v_ring + dst) = *reinterpret_cast<const float4*>(A.vc + (size_t)t * A.kv_dim + x);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) *A.state = A.final_state;
}

int grid_for(long long work, int per_block) {
    long long g = (work + per_block - 1) / per_block;
    if (g < 1) g = 1;
    if (g > 148 * 32) g = 148 * 32;
    return (int)g;
}

}  // namespace

size_t pf_gemm_smem_bytes() { return (size_t)kPfStages * kPfStageBytes + (2 * kPfStages + 4) * 8 + 16; }

cudaError_t pf_prepare() {
    cudaError_t e = cudaFuncSetAttribute(pf_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)pf_gemm_smem_bytes());
    const auto attn_smem = [](int hd) { return (2 * kPfKT * (hd + 4) + 4 * kPfQB * hd + 4 * kPfQB * 32) * 4; };
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(pf_attn_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_smem(32));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(pf_attn_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_smem(64));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(pf_attn_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_smem(128));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(pf_attn_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_smem(256));
    return e;
}

cudaError_t launch_pf_gemm(const PfGemmArgs& a, int grid, cudaStream_t s) {
    if (a.tn < 16 || a.tn > 128 || a.tn % 16 || a.splits < 1 || a.splits > a.kbt || grid < 1)
        return cudaErrorInvalidValue;
    pf_gemm_kernel<<<grid, kPfThreads, pf_gemm_smem_bytes(), s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_pf_norm(const PfNormArgs& a, int Tp, cudaStream_t s) {
    if (a.dim % 64 || (a.xop && a.tn % 16) || (a.embed && !a.tokens)) return cudaErrorInvalidValue;
    pf_norm_kernel<<<Tp, 256, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_pf_qkv(const PfQkvArgs& a, cudaStream_t s) {
    if (a.head_dim % 2 || a.q_dim % 2 || a.kv_dim % 2) return cudaErrorInvalidValue;
    const long long work = (long long)a.T * ((a.q_dim + 2 * a.kv_dim) / 2);
    pf_qkv_kernel<<<grid_for(work, 256), 256, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_pf_attn(const PfAttnArgs& a, cudaStream_t s) {
    const int G = a.n_kv > 0 ? a.n_heads / a.n_kv : 0;
    if (G < 1 || G > 4 || a.n_heads % a.n_kv || a.win < 1) return cudaErrorInvalidValue;
    const int C = a.head_dim / 32;
    if (a.head_dim % 32 || (C != 1 && C != 2 && C != 4 && C != 8)) return cudaErrorInvalidValue;
    const dim3 grid((a.T + kPfQB - 1) / kPfQB, a.n_kv);
    const size_t smem = (size_t)(2 * kPfKT * (a.head_dim + 4) + 4 * kPfQB * a.head_dim + 4 * kPfQB * 32) * 4;
    switch (C) {
        case 1: pf_attn_kernel<1><<<grid, 128, smem, s>>>(a); break;
        case 2: pf_attn_kernel<2><<<grid, 128, smem, s>>>(a); break;
        case 4: pf_attn_kernel<4><<<grid, 128, smem, s>>>(a); break;
        default: pf_attn_kernel<8><<<grid, 128, smem, s>>>(a); break;
    }
    return cudaGetLastError();
}

cudaError_t launch_pf_split(const float* src, int T, int Tp, int K, unsigned char* xop, int tn, cudaStream_t s) {
    if (K % 64 || tn % 16) return cudaErrorInvalidValue;
    pf_split_kernel<<<grid_for((long long)Tp * (K / 8), 256), 256, 0, s>>>(src, T, Tp, K, xop, tn);
    return cudaGetLastError();
}

cudaError_t launch_pf_swiglu(const float* part, int splits, int T, int Tp, int hidden, unsigned char* xop, int tn,
                             cudaStream_t s) {
    if (hidden % 64 || tn % 16) return cudaErrorInvalidValue;
    pf_swiglu_kernel<<<grid_for((long long)Tp * (hidden / 8), 256), 256, 0, s>>>(part, splits, T, Tp, hidden, xop,
                                                                                 tn);
    return cudaGetLastError();
}

cudaError_t launch_pf_commit(const PfCommitArgs& a, cudaStream_t s) {
    if (a.kv_dim % 4 || a.head_dim % 4 || a.cap < 1) return cudaErrorInvalidValue;
    const int first = a.T > a.cap ? a.T - a.cap : 0;
    pf_commit_kernel<<<grid_for((long long)(a.T - first) * (a.kv_dim / 4), 256), 256, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace vox
