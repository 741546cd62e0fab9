// vox_gemv.cu -- batch-1 weight-streaming GEMV for sm_100a.
//
// y[r] = sum_k W[r, k] * x[k] for a row-major weight matrix W [rows, K]
// (bf16 or f32), the reference's `linear` (crates/voxtral/src/ops.rs:11-39)
// for n_rows = 1, fused with what surrounds each linear in
// decoder_layer_forward_step (crates/voxtral/src/decoder.rs:88-155):
//   prologue  RMSNorm of x (math.rs:11-27) or the bf16 embedding row of the
//             step's token;
//   epilogue  store (+bias) | residual add (ops.rs:41-46) | RoPE on q/k
//             (math.rs:30-65) with k/v written into the KV ring slot |
//             SiLU(gate)*up (math.rs:4-9, decoder.rs:147-150) | argmax.
//
// Work split: CTA b owns a contiguous band of rows, hence one contiguous
// byte range of W.  Warp 8 is a producer: one lane streams the band into a
// ring of shared-memory stages with cp.async.bulk (TMA, this CTA only) and
// mbarrier completion.  Warps 0..7 consume: warp w always handles K segment
// (w % nseg) of row pair (w / nseg) of each stage, so its slice of x lives
// in registers for the whole kernel and shared memory carries weights only.
// Each (row, segment) partial sum goes to shared memory and is summed in a
// fixed order, so results are run-to-run deterministic.
//
// Programmatic dependent launch: the producer starts streaming weights (which
// no earlier kernel writes) before griddepcontrol.wait; consumers wait before
// reading x.  Consecutive GEMVs therefore overlap one kernel's tail with the
// next kernel's weight fetch.
#include <cuda_runtime.h>
#include <math.h>

#include "vox_device.cuh"

namespace vox {

namespace {

// Pipeline shape inside a CTA: row pairs per warp per stage.
constexpr int kStageMult = 1;

template <typename WT>
struct Elem;
template <>
struct Elem<uint16_t> {
    static constexpr int kPerChunk = 8;
    __device__ static __forceinline__ void fma_chunk(float& acc0, float& acc1, const uint4& w,
                                                     const float* x) {
        acc0 = fmaf(bf16_lo(w.x), x[0], acc0);
        acc1 = fmaf(bf16_hi(w.x), x[1], acc1);
        acc0 = fmaf(bf16_lo(w.y), x[2], acc0);
        acc1 = fmaf(bf16_hi(w.y), x[3], acc1);
        acc0 = fmaf(bf16_lo(w.z), x[4], acc0);
        acc1 = fmaf(bf16_hi(w.z), x[5], acc1);
        acc0 = fmaf(bf16_lo(w.w), x[6], acc0);
        acc1 = fmaf(bf16_hi(w.w), x[7], acc1);
    }
};
template <>
struct Elem<float> {
    static constexpr int kPerChunk = 4;
    __device__ static __forceinline__ void fma_chunk(float& acc0, float& acc1, const uint4& w,
                                                     const float* x) {
        acc0 = fmaf(__uint_as_float(w.x), x[0], acc0);
        acc1 = fmaf(__uint_as_float(w.y), x[1], acc1);
        acc0 = fmaf(__uint_as_float(w.z), x[2], acc0);
        acc1 = fmaf(__uint_as_float(w.w), x[3], acc1);
    }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// silu(g) * u exactly as the reference orders it: g / (1 + exp(-g)), then * u.
__device__ __forceinline__ float swiglu(float g, float u) {
    float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
    return __fmul_rn(s, u);
}

template <typename WT, int CPT, int EPI, int NW>
__device__ __forceinline__ void gemv_body(const GemvPlan& P, const GemvArgs& A) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int EPC = Elem<WT>::kPerChunk;
    constexpr int kConsumerWarps = NW;

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int K = P.K;
    const int C = K / EPC;                    // 16-byte chunks per row
    const size_t row_bytes = (size_t)K * sizeof(WT);
    const uint32_t stage_bytes = (uint32_t)(P.stage_rows * row_bytes);

    // Row band of this CTA (whole units; paired epilogues never straddle CTAs).
    const int units = P.rows / P.unit;
    const int u0 = (int)((long long)units * blockIdx.x / gridDim.x);
    const int u1 = (int)((long long)units * (blockIdx.x + 1) / gridDim.x);
    const int r0 = u0 * P.unit;
    const int nrows = (u1 - u0) * P.unit;
    const int n_stages_total = (nrows + P.stage_rows - 1) / P.stage_rows;
    const int NS = P.nstages;

    unsigned char* stage_base = smem;
    float* red = reinterpret_cast<float*>(smem + (size_t)NS * stage_bytes);
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(
        smem + (((size_t)NS * stage_bytes + (size_t)P.max_rows_cta * P.nseg * 4 + 15) & ~size_t(15)));
    uint64_t* empty_bar = full_bar + NS;
    float* scratch = reinterpret_cast<float*>(empty_bar + NS);  // 16 floats + 16 ints + 16 floats

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], kConsumerWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();
    pdl_allow_dependents();

    const unsigned char* Wband =
        reinterpret_cast<const unsigned char*>(A.W) + (size_t)r0 * row_bytes;

    if (warp == kConsumerWarps) {
        // ---------------- producer ----------------
        if (lane == 0 && n_stages_total > 0) {
            const uint64_t pol = l2_evict_first_policy();
            bool ok = true;
            int issued = 0;
            for (int s = 0; s < n_stages_total; ++s) {
                const int buf = s % NS;
                if (s >= NS) {
                    if (!mbar_wait(&empty_bar[buf], ((s / NS) - 1) & 1)) {
                        raise_error(A.err, ERR_EMPTY_WAIT);
                        ok = false;
                        break;
                    }
                }
                const int rows_here = min(P.stage_rows, nrows - s * P.stage_rows);
                const uint32_t bytes = (uint32_t)(rows_here * row_bytes);
                mbar_arrive_expect_tx(&full_bar[buf], bytes);
                bulk_copy_g2s(stage_base + (size_t)buf * stage_bytes,
                              Wband + (size_t)s * stage_bytes, bytes, &full_bar[buf], pol);
                ++issued;
            }
            if (ok && A.pf_W && (int)blockIdx.x < A.pf_grid) {
                const int nu = A.pf_rows / A.pf_unit;
                const int v0 = (int)((long long)nu * blockIdx.x / A.pf_grid);
                const int v1 = (int)((long long)nu * (blockIdx.x + 1) / A.pf_grid);
                long long nb = (long long)(v1 - v0) * A.pf_unit * A.pf_row_bytes;
                if (nb > A.pf_max_bytes) nb = A.pf_max_bytes;
                const unsigned char* src =
                    reinterpret_cast<const unsigned char*>(A.pf_W) + (long long)v0 * A.pf_unit * A.pf_row_bytes;
                for (long long o = 0; o + 16 <= nb; o += 16384) {
                    const long long n = nb - o < 16384 ? nb - o : 16384;
                    bulk_prefetch_l2(src + o, (uint32_t)(n & ~15ll));
                }
            }
            if (!ok) {
                // Leave no copy in flight: wait (bounded) for the last issued stages.
                for (int s = max(0, issued - NS); s < issued; ++s)
                    if (!mbar_wait(&full_bar[s % NS], (s / NS) & 1)) raise_error(A.err, ERR_DRAIN_WAIT);
            }
        }
        pdl_wait_prior_grids();
        return;
    }

    // ---------------- consumers ----------------
    const int nseg = P.nseg;
    const int seg = warp % nseg;
    const int tp = warp / nseg;               // first row pair of this warp inside a stage
    const int pair_step = kConsumerWarps / nseg;
    const int segc = C / nseg;
    const int c0 = seg * segc;
    const int vec = blockIdx.y;

    // RMSNorm gains of this warp's K slice do not depend on earlier kernels:
    // fetch them before waiting (small slices only, to bound registers).
    constexpr bool kEarlyGain = CPT <= 4;
    float gr[kEarlyGain ? CPT : 1][EPC];
    if constexpr (kEarlyGain) {
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
            const int cc = lane + 32 * i;
#pragma unroll
            for (int e = 0; e < EPC; ++e)
                gr[i][e] = (A.norm_w && cc < segc) ? A.norm_w[(c0 + cc) * EPC + e] : 0.0f;
        }
    }

    pdl_wait_prior_grids();

    // Tensor-parallel input: wait until every rank's partial sums for this
    // exchange point have arrived (bounded), then x = their sum, in rank order.
    const bool xsum = A.xch && A.xch_in >= 0;
    if (xsum) {
        if (tid == 0) {
            const unsigned long long target = (__ldcg(A.tp_steps) + 1ull) * A.xch_arrivals;
            // Once one wait of the step has expired (a rank stopped), the rest
            // are skipped so that the step ends within one wait limit.
            const bool expired = (*reinterpret_cast<volatile unsigned*>(A.err) & ERR_PEER_WAIT) != 0u;
            if (!expired && !wait_counter_sys(A.xa.counter(A.xch[A.xa.rank], A.xch_in), target))
                raise_error(A.err, ERR_PEER_WAIT);
        }
        named_barrier_sync(1, kConsumerWarps * 32);
    }
    // Input vector: x, or the embedding row of the step's token.
    const float* x = A.x ? A.x + (long long)vec * A.x_stride : nullptr;
    const uint16_t* xe = nullptr;
    const float* xad = nullptr;
    if (A.x_embed) {
        int tok = A.step->tok;
        if (tok < 0 || tok >= A.vocab) {
            if (tid == 0 && blockIdx.x == 0) raise_error(A.err, ERR_TOKEN_RANGE);
            tok = 0;
        }
        xe = A.x_embed + (size_t)tok * K;
        if (A.x_adapter) {
            const long long p = A.step->pos;
            xad = A.x_adapter + (size_t)(p < 0 ? 0 : p % A.adapter_cap) * K;
        }
    }

    // Epilogue inputs that do not depend on this product (the residual row,
    // the position and ring state of the q|k|v epilogue), loaded now so the
    // epilogue, which ends the launch, only stores.  Every producer of these
    // values finished before the dependency wait above.  Thread t's first
    // epilogue row (pair) is t.
    [[maybe_unused]] float pre_res = 0.0f, pre_c = 1.0f, pre_s = 0.0f;
    [[maybe_unused]] long long pre_pos = 0;
    [[maybe_unused]] KvState pre_st{};
    if constexpr (EPI == EPI_RESID) {
        if (tid < nrows) pre_res = A.resid[r0 + tid];
        if (A.kv_commit && blockIdx.x == 0 && tid == 0) pre_st = *A.kv_commit;
    } else if constexpr (EPI == EPI_QKV) {
        pre_pos = A.step->pos;
        pre_st = *A.kv_state;
    }

    // This warp's slice of x in registers: one round trip to L2.
    float xr[CPT][EPC];
#pragma unroll
    for (int i = 0; i < CPT; ++i) {
        const int cc = lane + 32 * i;
#pragma unroll
        for (int e = 0; e < EPC; ++e) xr[i][e] = 0.0f;
        if (cc < segc) {
            const int k0 = (c0 + cc) * EPC;
            if (xe) {
                uint32_t ws[4];
                if constexpr (EPC == 8) {
                    const uint4 w = *reinterpret_cast<const uint4*>(xe + k0);
                    ws[0] = w.x; ws[1] = w.y; ws[2] = w.z; ws[3] = w.w;
                } else {
                    const uint2 w = *reinterpret_cast<const uint2*>(xe + k0);
                    ws[0] = w.x; ws[1] = w.y; ws[2] = 0u; ws[3] = 0u;
                }
#pragma unroll
                for (int e = 0; e < EPC; ++e) xr[i][e] = (e & 1) ? bf16_hi(ws[e >> 1]) : bf16_lo(ws[e >> 1]);
                if (xad) {  // adapter[pos] + tok_embed(token), one f32 add
#pragma unroll
                    for (int e = 0; e < EPC; e += 4) {
                        const float4 a = *reinterpret_cast<const float4*>(xad + k0 + e);
                        xr[i][e] = __fadd_rn(a.x, xr[i][e]);
                        xr[i][e + 1] = __fadd_rn(a.y, xr[i][e + 1]);
                        xr[i][e + 2] = __fadd_rn(a.z, xr[i][e + 2]);
                        xr[i][e + 3] = __fadd_rn(a.w, xr[i][e + 3]);
                    }
                }
            } else if (xsum) {
                unsigned char* own = A.xch[A.xa.rank];
                for (int src = 0; src < A.xa.size; ++src) {
                    const float* sl = A.xa.slot(own, A.xch_in, src);
#pragma unroll
                    for (int e = 0; e < EPC; e += 4) {
                        const float4 v = __ldcg(reinterpret_cast<const float4*>(sl + k0 + e));
                        xr[i][e] += v.x;
                        xr[i][e + 1] += v.y;
                        xr[i][e + 2] += v.z;
                        xr[i][e + 3] += v.w;
                    }
                }
            } else {
#pragma unroll
                for (int e = 0; e < EPC; e += 4) {
                    const float4 v = *reinterpret_cast<const float4*>(x + k0 + e);
                    xr[i][e] = v.x;
                    xr[i][e + 1] = v.y;
                    xr[i][e + 2] = v.z;
                    xr[i][e + 3] = v.w;
                }
            }
        }
    }
    // Stores only after every load of x is issued, so the loads above make one
    // round trip (a store between them could alias them).
    if (A.x_copy_out && blockIdx.x == 0 && tp == 0) {
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
            const int cc = lane + 32 * i;
            if (cc < segc)
#pragma unroll
                for (int e = 0; e < EPC; ++e) A.x_copy_out[(c0 + cc) * EPC + e] = xr[i][e];
        }
    }

    if constexpr (EPI == EPI_QKV) {  // rotation factors of thread t's row pair (needs the position)
        const bool pos_ok = pre_pos >= 0 && pre_pos < A.max_pos;
        const int r = r0 + 2 * tid;
        if (2 * tid < nrows && r < A.q_dim + A.kv_dim) {
            const int rr = r < A.q_dim ? r : r - A.q_dim;
            const int d = rr % A.head_dim, half = A.head_dim / 2;
            pre_c = A.rope_cos[(pos_ok ? pre_pos : 0) * half + d / 2];
            pre_s = A.rope_sin[(pos_ok ? pre_pos : 0) * half + d / 2];
        }
    }

    // RMSNorm (math.rs:22-24) deferred to the epilogue: the dot products use
    // x * g, and each row sum is scaled by inv_rms = 1 / sqrt(sum(x^2) / K + eps)
    // once the partial sums of squares (staged in scratch[32..]) are complete, so
    // the stage loop starts without a CTA-wide reduction.
    if (A.norm_w) {
        // Warps 0..nseg-1 (tp == 0) hold every element of x exactly once.
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < CPT; ++i)
#pragma unroll
            for (int e = 0; e < EPC; ++e) ss = fmaf(xr[i][e], xr[i][e], ss);
        ss = warp_sum(ss);
        if (lane == 0 && tp == 0) scratch[32 + warp] = ss;
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
            const int cc = lane + 32 * i;
#pragma unroll
            for (int e = 0; e < EPC; ++e) {
                float g;
                if constexpr (kEarlyGain)
                    g = gr[i][e];
                else
                    g = cc < segc ? A.norm_w[(c0 + cc) * EPC + e] : 0.0f;
                xr[i][e] = __fmul_rn(xr[i][e], g);
            }
        }
    }

    bool ok = true;
    for (int s = 0; s < n_stages_total; ++s) {
        const int buf = s % NS;
        if (!mbar_wait(&full_bar[buf], (s / NS) & 1)) {
            if (lane == 0) raise_error(A.err, ERR_FULL_WAIT);
            ok = false;
            break;
        }
        for (int pr = tp; pr < P.stage_rows / 2; pr += pair_step) {
        const int ra = s * P.stage_rows + 2 * pr;   // local row index
        if (ra < nrows) {
            const bool has_b = ra + 1 < nrows;
            const unsigned char* rowa = stage_base + (size_t)buf * stage_bytes + (size_t)(2 * pr) * row_bytes;
            const unsigned char* rowb = rowa + row_bytes;
            float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
            for (int i = 0; i < CPT; ++i) {
                const int cc = lane + 32 * i;
                if (cc < segc) {
                    const uint4 wa = ld_shared_v4(rowa + (size_t)(c0 + cc) * 16);
                    Elem<WT>::fma_chunk(a0, a1, wa, xr[i]);
                    if (has_b) {
                        const uint4 wb = ld_shared_v4(rowb + (size_t)(c0 + cc) * 16);
                        Elem<WT>::fma_chunk(b0, b1, wb, xr[i]);
                    }
                }
            }
            const float sa = warp_sum(a0 + a1);
            const float sb = warp_sum(b0 + b1);
            if (lane == 0) {
                red[ra * nseg + seg] = sa;
                if (has_b) red[(ra + 1) * nseg + seg] = sb;
            }
        }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[buf]);
    }
    named_barrier_sync(1, kConsumerWarps * 32);
    if (!ok) return;

    // ---------------- epilogue ----------------
    const int nthr = kConsumerWarps * 32;
    float inv_rms = 1.0f;
    if (A.norm_w) {
        float tot = 0.0f;
        for (int w = 0; w < nseg; ++w) tot += scratch[32 + w];
        inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), A.eps)));
    }
    auto row_sum = [&](int lr) {
        float v = 0.0f;
        for (int q = 0; q < nseg; ++q) v += red[lr * nseg + q];
        return A.norm_w ? __fmul_rn(inv_rms, v) : v;
    };

    if constexpr (EPI == EPI_STORE) {
        float* y = A.y + (long long)vec * A.y_stride;
        for (int lr = tid; lr < nrows; lr += nthr) {
            const int r = r0 + lr;
            float v = row_sum(lr);
            if (A.bias) v = __fadd_rn(A.bias[r], v);
            y[r] = v;
        }
    } else if constexpr (EPI == EPI_RESID) {
        float* y = A.y + (long long)vec * A.y_stride;
        const bool xout = A.xch && A.xch_out >= 0;
        for (int lr = tid; lr < nrows; lr += nthr) {
            const int r = r0 + lr;
            const float v = __fadd_rn(lr == tid ? pre_res : A.resid[r], row_sum(lr));
            y[r] = v;
            if (xout)  // tensor parallel: this rank's partial rows into every rank's slot
                for (int p = 0; p < A.xa.size; ++p) A.xa.slot(A.xch[p], A.xch_out, A.xa.rank)[r] = v;
        }
        if (A.kv_commit && blockIdx.x == 0 && tid == 0)
            *A.kv_commit = kv_after_single_append(pre_st, A.kv_window, A.ring_cap);
        if (xout) {
            named_barrier_sync(1, nthr);  // every row of this CTA is stored
            if (tid == 0) {
                __threadfence_system();
                for (int p = 0; p < A.xa.size; ++p) atomicAdd_system(A.xa.counter(A.xch[p], A.xch_out), 1ull);
            }
        }
    } else if constexpr (EPI == EPI_QKV) {
        const long long pos = pre_pos;
        const bool pos_ok = pos >= 0 && pos < A.max_pos;
        if (!pos_ok && tid == 0 && blockIdx.x == 0) raise_error(A.err, ERR_POS_RANGE);
        const int half = A.head_dim / 2;
        const float* ct = A.rope_cos + (pos_ok ? pos : 0) * half;
        const float* st = A.rope_sin + (pos_ok ? pos : 0) * half;
        const KvState post = kv_after_single_append(pre_st, A.kv_window, A.ring_cap);
        const int slot = (post.start + post.len - 1) % A.ring_cap;
        for (int pp = tid; pp < nrows / 2; pp += nthr) {
            const int r = r0 + 2 * pp;
            const float ya = row_sum(2 * pp), yb = row_sum(2 * pp + 1);
            if (r < A.q_dim + A.kv_dim) {
                // math.rs:58-61: (x0*c - x1*s, x0*s + x1*c), unfused
                const int rr = r < A.q_dim ? r : r - A.q_dim;
                const int d = rr % A.head_dim;
                const float c = pp == tid ? pre_c : ct[d / 2], sn = pp == tid ? pre_s : st[d / 2];
                const float o0 = __fsub_rn(__fmul_rn(ya, c), __fmul_rn(yb, sn));
                const float o1 = __fadd_rn(__fmul_rn(ya, sn), __fmul_rn(yb, c));
                if (r < A.q_dim) {
                    A.y[r] = o0;
                    A.y[r + 1] = o1;
                } else {
                    const int h = rr / A.head_dim;
                    float* dst = A.k_ring + ((size_t)h * A.ring_cap + slot) * A.head_dim + d;
                    dst[0] = o0;
                    dst[1] = o1;
                }
            } else {
                const int rr = r - A.q_dim - A.kv_dim;
                const int h = rr / A.head_dim, d = rr % A.head_dim;
                float* dst = A.v_ring + ((size_t)h * A.ring_cap + slot) * A.head_dim + d;
                dst[0] = ya;
                dst[1] = yb;
            }
        }
    } else if constexpr (EPI == EPI_SWIGLU) {
        float* y = A.y + (long long)vec * A.y_stride;
        for (int pp = tid; pp < nrows / 2; pp += nthr) {
            const int j = (r0 >> 1) + pp;
            y[j] = swiglu(row_sum(2 * pp), row_sum(2 * pp + 1));
        }
    } else if constexpr (EPI == EPI_ARGMAX) {
        float best = -INFINITY;
        int bi = 0x7FFFFFFF;
        for (int lr = tid; lr < nrows; lr += nthr) {
            const int r = r0 + lr;
            const float v = row_sum(lr);
            if (A.y) A.y[r] = v;
            if (v > best || (v == best && r < bi)) {
                best = v;
                bi = r;
            }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xFFFFFFFFu, best, o);
            const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
            if (ov > best || (ov == best && oi < bi)) {
                best = ov;
                bi = oi;
            }
        }
        int* si = reinterpret_cast<int*>(scratch + 16);
        if (lane == 0) {
            scratch[warp] = best;
            si[warp] = bi;
        }
        named_barrier_sync(1, nthr);
        if (tid == 0) {
            for (int w = 1; w < kConsumerWarps; ++w) {
                if (scratch[w] > best || (scratch[w] == best && si[w] < bi)) {
                    best = scratch[w];
                    bi = si[w];
                }
            }
            A.am_part[blockIdx.x].v = best;
            A.am_part[blockIdx.x].i = bi;
        }
    }
}

template <typename WT, int CPT, int EPI, int NW>
__global__ void __launch_bounds__((NW + 1) * 32, NW == 8 ? 2 : 1)
    gemv_kernel(const GemvPlan P, const GemvArgs A) {
    gemv_body<WT, CPT, EPI, NW>(P, A);
}

// 8 consumer warps at <= 80 registers: two such CTAs fit on an SM beside an
// attention CTA (o-proj streams its weights while attention runs).
template <typename WT, int CPT, int EPI, int NW>
__global__ void __maxnreg__(80) gemv_kernel_lean(const GemvPlan P, const GemvArgs A) {
    gemv_body<WT, CPT, EPI, NW>(P, A);
}

template <typename WT, int EPI, int NW>
void* pick_kernel(int cpt) {
    switch (cpt) {
        case 1: return (void*)gemv_kernel<WT, 1, EPI, NW>;
        case 2: return (void*)gemv_kernel<WT, 2, EPI, NW>;
        case 3: return (void*)gemv_kernel<WT, 3, EPI, NW>;
        case 4: return (void*)gemv_kernel<WT, 4, EPI, NW>;
        case 5: return (void*)gemv_kernel<WT, 5, EPI, NW>;
        case 6: return (void*)gemv_kernel<WT, 6, EPI, NW>;
        case 8: return (void*)gemv_kernel<WT, 8, EPI, NW>;
        default: return nullptr;
    }
}

template <typename WT, int NW>
void* pick_epi(int epi, int cpt) {
    switch (epi) {
        case EPI_STORE: return pick_kernel<WT, EPI_STORE, NW>(cpt);
        case EPI_RESID: return pick_kernel<WT, EPI_RESID, NW>(cpt);
        case EPI_QKV: return pick_kernel<WT, EPI_QKV, NW>(cpt);
        case EPI_SWIGLU: return pick_kernel<WT, EPI_SWIGLU, NW>(cpt);
        case EPI_ARGMAX: return pick_kernel<WT, EPI_ARGMAX, NW>(cpt);
    }
    return nullptr;
}

// The lean kernels exist for the launches next to attention: o-proj (after)
// and q|k|v (before), at most 2 chunks per lane.
void* pick_lean(int wsize, int epi, int cpt, int nw) {
    if (wsize != 2 || nw != 8) return nullptr;
    if (epi == EPI_RESID)
        return cpt == 1 ? (void*)gemv_kernel_lean<uint16_t, 1, EPI_RESID, 8>
                        : cpt == 2 ? (void*)gemv_kernel_lean<uint16_t, 2, EPI_RESID, 8> : nullptr;
    if (epi == EPI_QKV)
        return cpt == 1 ? (void*)gemv_kernel_lean<uint16_t, 1, EPI_QKV, 8>
                        : cpt == 2 ? (void*)gemv_kernel_lean<uint16_t, 2, EPI_QKV, 8> : nullptr;
    return nullptr;
}

// bf16 weights have both warp counts; the f32-weight path uses 8.
void* pick(int wsize, int epi, int cpt, int nw) {
    if (wsize == 2) return nw == 16 ? pick_epi<uint16_t, 16>(epi, cpt) : pick_epi<uint16_t, 8>(epi, cpt);
    return nw == 8 ? pick_epi<float, 8>(epi, cpt) : nullptr;
}

int cpt_round(int c) {
    if (c <= 6) return c < 1 ? 1 : c;
    return c <= 8 ? 8 : -1;
}

}  // namespace

bool gemv_supported(int K, int wsize) {
    const int epc = 16 / wsize;
    if (K <= 0 || K % epc) return false;
    const int C = K / epc;
    for (int nseg = 1; nseg <= 8; nseg *= 2)
        if (C % nseg == 0 && cpt_round((C / nseg + 31) / 32) > 0) return true;
    return false;
}

size_t gemv_max_smem() { return 227 * 1024 - 256; }

GemvPlan plan_gemv(int rows, int K, int unit, int wsize, int num_sms, int n_vec, GemvShape shape) {
    GemvPlan p{};
    p.rows = rows;
    p.K = K;
    p.unit = unit;
    p.wsize = wsize;
    p.n_vec = n_vec < 1 ? 1 : n_vec;
    const int epc = 16 / wsize;
    const int C = K / epc;
    // Fewest segments whose per-lane chunk count stays <= 4 (x slice in
    // registers); otherwise the widest split that fits.
    p.nseg = -1;
    p.lean = 0;
    for (int nseg = 1; nseg <= 8; nseg *= 2) {
        if (C % nseg) continue;
        if ((C / nseg + 31) / 32 <= (shape.lean ? 2 : 4)) {
            p.nseg = nseg;
            p.lean = shape.lean && wsize == 2 && shape.warps == 8 ? 1 : 0;
            break;
        }
    }
    if (p.nseg < 0) {
        for (int nseg = 8; nseg >= 1; nseg /= 2)
            if (C % nseg == 0 && cpt_round((C / nseg + 31) / 32) > 0) {
                p.nseg = nseg;
                break;
            }
    }
    if (p.nseg < 0) {
        p.grid = 0;
        return p;
    }
    p.cpt = cpt_round((C / p.nseg + 31) / 32);
    const int warps = shape.warps == 8 ? 8 : 16;
    const int ctas_per_sm = shape.ctas_per_sm == 2 ? 2 : 1;
    p.nw = wsize == 2 ? warps : 8;
    p.stage_rows = 2 * (p.nw / p.nseg) * kStageMult;
    const size_t row_bytes = (size_t)K * wsize;
    size_t stage_bytes = p.stage_rows * row_bytes;
    const int units = rows / unit;
    const int max_grid = num_sms * ctas_per_sm;
    p.grid = units < max_grid ? units : max_grid;
    if (p.grid < 1) p.grid = 1;
    p.max_rows_cta = ((units + p.grid - 1) / p.grid) * unit;
    // Do not reserve stages a CTA can never fill.
    int max_stages_needed = (p.max_rows_cta + p.stage_rows - 1) / p.stage_rows;
    int ns = (int)(shape.ring_bytes / stage_bytes);
    if (ns < 2) ns = 2;
    if (ns > 16) ns = 16;
    if (ns > max_stages_needed) ns = max_stages_needed < 1 ? 1 : max_stages_needed;
    p.nstages = ns;
    size_t red_bytes = ((size_t)p.max_rows_cta * p.nseg * 4 + 15) & ~size_t(15);
    p.smem = (size_t)ns * stage_bytes + red_bytes + 2 * ns * sizeof(uint64_t) + 48 * 4;
    return p;
}

cudaError_t gemv_prepare(int /*dev*/) {
    for (int epi : {EPI_RESID, EPI_QKV})
        for (int c : {1, 2}) {
            cudaError_t e = cudaFuncSetAttribute(pick_lean(2, epi, c, 8), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 227 * 1024);
            if (e != cudaSuccess) return e;
        }
    const int cpts[] = {1, 2, 3, 4, 5, 6, 8};
    for (int ws : {2, 4})
        for (int epi = 0; epi <= EPI_ARGMAX; ++epi)
            for (int c : cpts) {
                for (int nw : {8, 16}) {
                void* k = pick(ws, epi, c, nw);
                if (!k) continue;
                cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     227 * 1024);
                if (e != cudaSuccess) return e;
                }
            }
    return cudaSuccess;
}

cudaError_t launch_gemv(const GemvPlan& p, const GemvArgs& a, int epi, cudaStream_t s, bool pdl) {
    void* k = p.lean ? pick_lean(p.wsize, epi, p.cpt, p.nw) : pick(p.wsize, epi, p.cpt, p.nw);
    if (!k || p.grid < 1) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid, p.n_vec, 1);
    cfg.blockDim = dim3((p.nw + 1) * 32, 1, 1);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    void* args[] = {(void*)&p, (void*)&a};
    return cudaLaunchKernelExC(&cfg, k, args);
}

}  // namespace vox
