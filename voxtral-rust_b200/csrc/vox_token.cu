// vox_token.cu -- one decoder token step as ONE persistent kernel.
//
// Runs, for every layer, decoder_layer_forward_step
// (crates/voxtral/src/decoder.rs:88-155): RMSNorm -> q|k|v -> RoPE -> KV ring
// append -> GQA attention -> o-proj + residual -> RMSNorm -> w1|w3 -> SiLU*up
// -> w2 + residual; then the final RMSNorm, the LM head and the argmax of the
// composed token loop.  The arithmetic of every phase is the same as in the
// separate kernels (vox_gemv.cu, vox_attention.cu); what changes is the
// schedule.
//
// One CTA per SM, launched cooperatively so that all CTAs are resident:
//   * warp 16 (producer): one lane streams this CTA's band of EVERY weight
//     matrix of the step -- wqkv, wo, w1|w3, w2 of each layer, then the LM
//     head -- into a 3 x 48 KB shared-memory ring with cp.async.bulk (TMA,
//     this CTA only).  Weights never depend on activations, so the producer never
//     waits for a phase to finish: HBM keeps streaming across layer and
//     phase boundaries and through the attention phases.
//   * warps 0..15 (consumers): walk the phases.  Between phases they meet at
//     a grid barrier (a monotonic 64-bit counter in global memory; every wait
//     is bounded and aborts the whole step with an error bit if it expires).
//     Activations are read with L2-only loads (ld.global.cg / cp.async.cg),
//     since other SMs wrote them during this launch.
//   * the attention phase of a layer uses warps 0..3: CTA b handles split
//     (b mod splits) of kv head (b / splits); the last CTA of each head merges
//     the splits.  Meanwhile the producer keeps filling the ring with the
//     o-proj and w1|w3 weights.
#include <cuda_runtime.h>
#include <math.h>

#include "vox_device.cuh"

namespace vox {

namespace {

constexpr int kNW = 16;                        // consumer warps
constexpr int kThreads = (kNW + 1) * 32;       // + producer warp
constexpr int kConsumers = kNW * 32;
constexpr uint32_t kSlotBytes = 48 * 1024;
constexpr int kSlots = 3;
constexpr int kMaxSplits = 64;
constexpr int kMaxCpt = 3;  // x slice of at most 3 x 8 floats per lane
constexpr unsigned kAbortMask = ERR_FULL_WAIT | ERR_EMPTY_WAIT | ERR_DRAIN_WAIT | ERR_GRID_WAIT;

struct Layout {
    size_t work_off, bar_off, scratch_off, total;
};

__host__ __device__ inline int band_max_rows(const TokGemv& g, int grid) {
    const int units = g.rows / g.unit;
    return ((units + grid - 1) / grid) * g.unit;
}

__host__ __device__ inline Layout token_layout(const TokenArgs& a, int grid) {
    const int G = a.n_heads / a.n_kv;
    const size_t attn_f = (size_t)kNW * G * a.hd + (size_t)kNW * G * 2 + (size_t)G * kMaxSplits + 8;
    size_t red_f = 0;
    const TokGemv* gs[5] = {&a.g_qkv, &a.g_o, &a.g_w13, &a.g_w2, &a.g_head};
    for (int i = 0; i < 5; ++i) {
        if (i == 4 && a.vocab == 0) continue;
        const size_t r = (size_t)band_max_rows(*gs[i], grid) * gs[i]->nseg;
        if (r > red_f) red_f = r;
    }
    Layout L;
    L.work_off = (size_t)kSlots * kSlotBytes;
    const size_t work = ((attn_f > red_f ? attn_f : red_f) * 4 + 127) & ~size_t(127);
    L.bar_off = L.work_off + work;
    L.scratch_off = L.bar_off + 2 * kSlots * sizeof(uint64_t);
    L.total = L.scratch_off + 64 * 4;
    return L;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

__device__ __forceinline__ bool aborted(const unsigned* err) {
    return (*reinterpret_cast<const volatile unsigned*>(err) & kAbortMask) != 0;
}

__device__ __forceinline__ KvState load_state(const KvState* p) {
    KvState s;
    s.len = __ldcg(&p->len);
    s.start = __ldcg(&p->start);
    s.pos_offset = __ldcg(&p->pos_offset);
    return s;
}

// All consumer threads: every CTA arrives, then waits until the counter
// reaches `target` (bounded; an expired wait or another CTA's abort ends the
// step).  Returns false when the step is aborted.
__device__ bool grid_sync(unsigned long long* bar, unsigned long long target, unsigned* err, int* flag) {
    named_barrier_sync(1, kConsumers);
    if (threadIdx.x == 0) {
        __threadfence();  // this CTA's writes (ordered by the barrier above) before the arrival
        asm volatile("red.relaxed.gpu.global.add.u64 [%0], 1;" ::"l"(bar) : "memory");
        bool ok = !aborted(err);
        uint32_t it = 0;
        uint64_t t0 = 0;
        while (ok) {
            unsigned long long v;
            asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(bar) : "memory");
            if (v >= target) break;
            if ((++it & 127u) == 0) {
                if (aborted(err)) {
                    ok = false;
                    break;
                }
                const uint64_t now = global_timer_ns();
                if (t0 == 0) {
                    t0 = now;
                } else if (now - t0 > kWaitLimitNs) {
                    raise_error(err, ERR_GRID_WAIT);
                    ok = false;
                }
            }
        }
        __threadfence();
        *flag = ok ? 1 : 0;
    }
    named_barrier_sync(1, kConsumers);
    return *flag != 0;
}

__device__ __forceinline__ void tok_band(const TokGemv& P, int& r0, int& nrows) {
    const int units = P.rows / P.unit;
    const int u0 = (int)((long long)units * blockIdx.x / gridDim.x);
    const int u1 = (int)((long long)units * (blockIdx.x + 1) / gridDim.x);
    r0 = u0 * P.unit;
    nrows = (u1 - u0) * P.unit;
}

// ---------------------------------------------------------------------------
// Producer: stream this CTA's band of W into the ring, continuing the global
// stage sequence g.
// ---------------------------------------------------------------------------
// Cursor over this CTA's weight stages in consumer order (per layer: qkv, o,
// w1|w3, w2; then the LM head).  Band geometry is recomputed only when the
// cursor enters a new matrix.
struct Cursor {
    int layer, kind, s, nst, stage_rows, nrows;
    size_t row_bytes;
    const unsigned char* base;
    bool done;
};

__device__ __forceinline__ void cur_next_kind(const TokenArgs& A, Cursor& c) {
    if (c.layer >= A.n_layers) {
        c.done = true;  // the LM head was the last matrix
    } else if (++c.kind == 4) {
        c.kind = 0;
        ++c.layer;
    }
}

// Enter the band of (layer, kind), skipping bands with no rows.
__device__ void cur_enter(const TokenArgs& A, Cursor& c) {
    while (!c.done) {
        const TokGemv* P;
        const uint16_t* W;
        if (c.layer >= A.n_layers) {
            if (!A.vocab) {
                c.done = true;
                return;
            }
            P = &A.g_head;
            W = A.lm_head;
        } else {
            const TokLayer& L = A.layers[c.layer];
            if (c.kind == 0) {
                P = &A.g_qkv; W = L.wqkv;
            } else if (c.kind == 1) {
                P = &A.g_o; W = L.wo;
            } else if (c.kind == 2) {
                P = &A.g_w13; W = L.w13;
            } else {
                P = &A.g_w2; W = L.w2;
            }
        }
        int r0, nrows;
        tok_band(*P, r0, nrows);
        c.row_bytes = (size_t)P->K * 2;
        c.stage_rows = P->stage_rows;
        c.nrows = nrows;
        c.s = 0;
        c.nst = (nrows + P->stage_rows - 1) / P->stage_rows;
        c.base = reinterpret_cast<const unsigned char*>(W) + (size_t)r0 * c.row_bytes;
        if (c.nst > 0) return;
        cur_next_kind(A, c);
    }
}

__device__ __forceinline__ void cur_start(const TokenArgs& A, Cursor& c) {
    c.layer = 0;
    c.kind = 0;
    c.done = false;
    cur_enter(A, c);
}

__device__ __forceinline__ void cur_stage(const Cursor& c, const unsigned char** src, uint32_t* bytes) {
    const int rows_here = min(c.stage_rows, c.nrows - c.s * c.stage_rows);
    *src = c.base + (size_t)c.s * c.stage_rows * c.row_bytes;
    *bytes = (uint32_t)(rows_here * c.row_bytes);
}

__device__ __forceinline__ void cur_advance(const TokenArgs& A, Cursor& c) {
    if (++c.s >= c.nst) {
        cur_next_kind(A, c);
        cur_enter(A, c);
    }
}

// One lane streams every stage of the step into the ring, never waiting for
// a phase to finish: only for a free slot.
__device__ __noinline__ void producer(const TokenArgs& A, unsigned char* ring, uint64_t* full,
                                      uint64_t* empty) {
    const uint64_t pol = l2_evict_first_policy();
    Cursor fill;
    cur_start(A, fill);
    uint32_t g = 0;
    while (!fill.done) {
        const int slot = (int)(g % kSlots);
        if (g >= (uint32_t)kSlots && !mbar_wait(&empty[slot], ((g / kSlots) - 1) & 1)) {
            raise_error(A.err, ERR_EMPTY_WAIT);
            break;
        }
        const unsigned char* src;
        uint32_t bytes;
        cur_stage(fill, &src, &bytes);
        mbar_arrive_expect_tx(&full[slot], bytes);
        bulk_copy_g2s(ring + (size_t)slot * kSlotBytes, src, bytes, &full[slot], pol);
        cur_advance(A, fill);
        ++g;
    }
    // Leave no copy in flight when the CTA exits: wait (bounded) for the last
    // issued stages; on the normal path the consumers already did.
    const uint32_t first = g > (uint32_t)kSlots ? g - kSlots : 0u;
    for (uint32_t st = first; st < g; ++st)
        if (!mbar_wait(&full[st % kSlots], (st / kSlots) & 1)) raise_error(A.err, ERR_DRAIN_WAIT);
}

// ---------------------------------------------------------------------------
// Consumers: one GEMV phase (same math and epilogues as gemv_kernel).
// ---------------------------------------------------------------------------
struct PhaseIO {
    const float* x;          // f32 input (L2 loads) or
    const uint16_t* xe;      // bf16 embedding row
    const float* norm_w;     // RMSNorm gain, or null
    float* x_copy_out;       // CTA 0 stores the raw x here
    float* y;
    const float* resid;
    const TokLayer* L;       // QKV epilogue / state commit
    bool commit;             // o-proj: commit the ring append of layer L
};

template <int CPT, int EPI>
__device__ __forceinline__ void gemv_phase(const TokenArgs& A, const TokGemv& P, const PhaseIO& io,
                                        unsigned char* ring, uint64_t* full, uint64_t* empty, uint32_t* gp,
                                        float* red, float* scratch) {
    constexpr int EPC = 8;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int r0, nrows;
    tok_band(P, r0, nrows);
    const int K = P.K, C = K / EPC;
    const int nseg = P.nseg, seg = warp % nseg, tp = warp / nseg, pair_step = kNW / nseg;
    const int segc = C / nseg, c0 = seg * segc;
    const size_t row_bytes = (size_t)K * 2;

    // x (times the RMSNorm gain when normalising) in registers: one round trip.
    // The 1/rms factor multiplies the row sums in the epilogue instead
    // (y = inv_rms * W (x * g)), so the stage loop starts without waiting
    // for a CTA-wide reduction.
    float xr[CPT][EPC];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < CPT; ++i) {
        const int cc = lane + 32 * i;
#pragma unroll
        for (int e = 0; e < EPC; ++e) xr[i][e] = 0.0f;
        if (cc < segc) {
            const int k0 = (c0 + cc) * EPC;
            if (io.xe) {
                const uint4 w = *reinterpret_cast<const uint4*>(io.xe + k0);
                const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < EPC; ++e) xr[i][e] = (e & 1) ? bf16_hi(ws[e >> 1]) : bf16_lo(ws[e >> 1]);
            } else {
                const float4 a = __ldcg(reinterpret_cast<const float4*>(io.x + k0));
                const float4 b = __ldcg(reinterpret_cast<const float4*>(io.x + k0 + 4));
                xr[i][0] = a.x; xr[i][1] = a.y; xr[i][2] = a.z; xr[i][3] = a.w;
                xr[i][4] = b.x; xr[i][5] = b.y; xr[i][6] = b.z; xr[i][7] = b.w;
            }
            if (io.x_copy_out && blockIdx.x == 0 && tp == 0) {
#pragma unroll
                for (int e = 0; e < EPC; ++e) io.x_copy_out[k0 + e] = xr[i][e];
            }
            if (io.norm_w) {
                const float4 ga = __ldg(reinterpret_cast<const float4*>(io.norm_w + k0));
                const float4 gb = __ldg(reinterpret_cast<const float4*>(io.norm_w + k0 + 4));
                const float gv[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
                for (int e = 0; e < EPC; ++e) {
                    ss = fmaf(xr[i][e], xr[i][e], ss);
                    xr[i][e] = __fmul_rn(xr[i][e], gv[e]);
                }
            }
        }
    }
    float* ssw = scratch + 32;  // per-warp sums of squares (warps with tp == 0)
    if (io.norm_w) {
        ss = warp_sum(ss);
        if (lane == 0 && tp == 0) ssw[warp] = ss;
    }

    uint32_t g = *gp;  // this thread's copy of the global stage counter
    bool ok = true;
    for (int s = 0; s * P.stage_rows < nrows; ++s, ++g) {
        const int slot = (int)(g % kSlots);
        if (ok && !mbar_wait(&full[slot], (g / kSlots) & 1)) {
            if (lane == 0) raise_error(A.err, ERR_FULL_WAIT);
            ok = false;
        }
        if (ok) {
            const unsigned char* stage = ring + (size_t)slot * kSlotBytes;
            for (int pr = tp; pr < P.stage_rows / 2; pr += pair_step) {
                const int ra = s * P.stage_rows + 2 * pr;
                if (ra >= nrows) break;
                const bool has_b = ra + 1 < nrows;
                const unsigned char* rowa = stage + (size_t)(2 * pr) * row_bytes;
                const unsigned char* rowb = rowa + row_bytes;
                float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
                for (int i = 0; i < CPT; ++i) {
                    const int cc = lane + 32 * i;
                    if (cc < segc) {
                        const uint4 wa = ld_shared_v4(rowa + (size_t)(c0 + cc) * 16);
                        a0 = fmaf(bf16_lo(wa.x), xr[i][0], a0);
                        a1 = fmaf(bf16_hi(wa.x), xr[i][1], a1);
                        a0 = fmaf(bf16_lo(wa.y), xr[i][2], a0);
                        a1 = fmaf(bf16_hi(wa.y), xr[i][3], a1);
                        a0 = fmaf(bf16_lo(wa.z), xr[i][4], a0);
                        a1 = fmaf(bf16_hi(wa.z), xr[i][5], a1);
                        a0 = fmaf(bf16_lo(wa.w), xr[i][6], a0);
                        a1 = fmaf(bf16_hi(wa.w), xr[i][7], a1);
                        if (has_b) {
                            const uint4 wb = ld_shared_v4(rowb + (size_t)(c0 + cc) * 16);
                            b0 = fmaf(bf16_lo(wb.x), xr[i][0], b0);
                            b1 = fmaf(bf16_hi(wb.x), xr[i][1], b1);
                            b0 = fmaf(bf16_lo(wb.y), xr[i][2], b0);
                            b1 = fmaf(bf16_hi(wb.y), xr[i][3], b1);
                            b0 = fmaf(bf16_lo(wb.z), xr[i][4], b0);
                            b1 = fmaf(bf16_hi(wb.z), xr[i][5], b1);
                            b0 = fmaf(bf16_lo(wb.w), xr[i][6], b0);
                            b1 = fmaf(bf16_hi(wb.w), xr[i][7], b1);
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
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
    }
    *gp = g;
    // Leave together: a warp whose wait expired marks the CTA, and every warp
    // reads the mark after the barrier, so all return (or all continue).
    int* fail_s = reinterpret_cast<int*>(scratch + 52);
    if (!ok && lane == 0) *fail_s = 1;
    named_barrier_sync(1, kConsumers);
    if (*fail_s) return;

    // math.rs:22: inv_rms = 1 / sqrt(sq_sum / dim + eps) (ssw is ready: barrier above)
    float inv = 1.0f;
    if (io.norm_w) {
        float tot = 0.0f;
        for (int w = 0; w < nseg; ++w) tot += ssw[w];
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), A.eps)));
    }
    auto row_sum = [&](int lr) {
        float v = 0.0f;
        for (int q = 0; q < nseg; ++q) v += red[lr * nseg + q];
        return io.norm_w ? __fmul_rn(inv, v) : v;
    };
    if constexpr (EPI == EPI_RESID) {
        for (int lr = tid; lr < nrows; lr += kConsumers) {
            const int r = r0 + lr;
            io.y[r] = __fadd_rn(__ldcg(io.resid + r), row_sum(lr));
        }
        if (io.commit && blockIdx.x == 0 && tid == 0)
            *io.L->st = kv_after_single_append(load_state(io.L->st), A.kv_window, A.cap);
    } else if constexpr (EPI == EPI_QKV) {
        const long long pos = __ldcg(&A.step->pos);
        const bool pos_ok = pos >= 0 && pos < A.max_pos;
        if (!pos_ok && tid == 0 && blockIdx.x == 0) raise_error(A.err, ERR_POS_RANGE);
        const int half = A.hd / 2;
        const float* ct = A.rope_cos + (pos_ok ? pos : 0) * half;
        const float* st = A.rope_sin + (pos_ok ? pos : 0) * half;
        const KvState post = kv_after_single_append(load_state(io.L->st), A.kv_window, A.cap);
        const int slot = (post.start + post.len - 1) % A.cap;
        for (int pp = tid; pp < nrows / 2; pp += kConsumers) {
            const int r = r0 + 2 * pp;
            const float ya = row_sum(2 * pp), yb = row_sum(2 * pp + 1);
            if (r < A.q_dim + A.kv_dim) {
                // math.rs:58-61: (x0*c - x1*s, x0*s + x1*c), unfused
                const int rr = r < A.q_dim ? r : r - A.q_dim;
                const int d = rr % A.hd;
                const float c = ct[d / 2], sn = st[d / 2];
                const float o0 = __fsub_rn(__fmul_rn(ya, c), __fmul_rn(yb, sn));
                const float o1 = __fadd_rn(__fmul_rn(ya, sn), __fmul_rn(yb, c));
                if (r < A.q_dim) {
                    A.q[r] = o0;
                    A.q[r + 1] = o1;
                } else {
                    float* dst = io.L->k_ring + ((size_t)(rr / A.hd) * A.cap + slot) * A.hd + d;
                    dst[0] = o0;
                    dst[1] = o1;
                }
            } else {
                const int rr = r - A.q_dim - A.kv_dim;
                float* dst = io.L->v_ring + ((size_t)(rr / A.hd) * A.cap + slot) * A.hd + rr % A.hd;
                dst[0] = ya;
                dst[1] = yb;
            }
        }
    } else if constexpr (EPI == EPI_SWIGLU) {
        for (int pp = tid; pp < nrows / 2; pp += kConsumers) {
            const float gv = row_sum(2 * pp), uv = row_sum(2 * pp + 1);
            const float sv = __fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv)));  // math.rs:4-9
            io.y[(r0 >> 1) + pp] = __fmul_rn(sv, uv);                     // decoder.rs:147-150
        }
    } else if constexpr (EPI == EPI_ARGMAX) {
        float best = -INFINITY;
        int bi = 0x7FFFFFFF;
        for (int lr = tid; lr < nrows; lr += kConsumers) {
            const int r = r0 + lr;
            const float v = row_sum(lr);
            io.y[r] = v;
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
        named_barrier_sync(1, kConsumers);
        if (tid == 0) {
            for (int w = 1; w < kNW; ++w)
                if (scratch[w] > best || (scratch[w] == best && si[w] < bi)) {
                    best = scratch[w];
                    bi = si[w];
                }
            A.am_part[blockIdx.x].v = best;
            A.am_part[blockIdx.x].i = bi;
        }
    }
}

template <int EPI>
__device__ void gemv_dispatch(const TokenArgs& A, const TokGemv& P, const PhaseIO& io, unsigned char* ring,
                              uint64_t* full, uint64_t* empty, uint32_t* gp, float* red, float* scratch) {
    switch (P.cpt) {
        case 1: gemv_phase<1, EPI>(A, P, io, ring, full, empty, gp, red, scratch); break;
        case 2: gemv_phase<2, EPI>(A, P, io, ring, full, empty, gp, red, scratch); break;
        default: gemv_phase<3, EPI>(A, P, io, ring, full, empty, gp, red, scratch); break;
    }
}

// ---------------------------------------------------------------------------
// Consumers: attention phase (ops.rs:66-132), threads 0..127.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void attn_sync() { named_barrier_sync(2, kConsumers); }

// Sum of 32 per-lane partial values across the warp, leaving lane l with the
// total of value l (31 shuffles; lane bit o picks the half it keeps).
__device__ __forceinline__ void tok_transpose_reduce(float (&v)[32], int lane) {
#pragma unroll
    for (int o = 16, n = 32; o >= 1; o >>= 1, n >>= 1) {
        const bool up = lane & o;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float keep = up ? v[i + n / 2] : v[i];
            const float send = up ? v[i] : v[i + n / 2];
            v[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, o);
        }
    }
}

// Attention phase, all 16 consumer warps.  Each warp takes 32/G-token groups
// of one kv head (lane l holds dims 4l..4l+3 of q for the G heads); K and V
// rows come from L2 into registers (this launch's QKV phase wrote the new
// token), so the weight ring stays with the producer.  Scores by a
// transpose-reduce (lane l ends with head l/(32/G), token l%(32/G)), online
// softmax per warp, PV on the lane's four dims.  The 16 warps of a CTA
// combine in shared memory into one chunk partial; the last chunk of a kv
// head (atomic ticket) merges the chunks in a fixed order.
template <int G>
__device__ __forceinline__ void attn_phase_warp(const TokenArgs& A, const TokLayer& L, float* work) {
    constexpr int TPG = 32 / G;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hd = A.hd, hd4 = hd / 4;
    const unsigned FULL = 0xFFFFFFFFu;
    float* wacc = work;                              // [kNW][G][hd]
    float* wml = wacc + (size_t)kNW * G * hd;        // [kNW][G][2]
    float* w_s = wml + kNW * G * 2;                  // [G][kMaxSplits]
    int* flag_s = reinterpret_cast<int*>(w_s + G * kMaxSplits);

    const KvState st = kv_after_single_append(load_state(L.st), A.kv_window, A.cap);
    const int len = st.len;
    const int mask_start = (A.cfg_window > 0 && len > A.cfg_window) ? len - A.cfg_window : 0;
    const int n_live = len - mask_start;
    const int groups = (n_live + TPG - 1) / TPG;
    // groups per warp so that every warp of the grid has about one batch, and
    // at most kMaxSplits chunks (of kNW x gpw groups) per kv head
    const long long W = (long long)gridDim.x * kNW;
    int gpw = (int)max(1LL, ((long long)A.n_kv * groups + W - 1) / W);
    while ((groups + kNW * gpw - 1) / (kNW * gpw) > kMaxSplits) ++gpw;
    const int cgroups = kNW * gpw;                   // groups per chunk
    const int n_chunks = (groups + cgroups - 1) / cgroups;
    const bool dim_ok = lane * 4 < hd;
    const int my_g = lane / TPG, my_t = lane % TPG;
    const size_t acc_stride = (size_t)G * hd;
    const size_t ml_base = (size_t)A.n_kv * A.splits * acc_stride;

    if (n_chunks == 0) {  // empty cache: the reference returns zeros
        if (blockIdx.x == 0)
            for (int i = tid; i < A.n_heads * hd; i += kConsumers) A.attn[i] = 0.f;
        return;
    }
    for (int item = blockIdx.x; item < A.n_kv * n_chunks; item += gridDim.x) {
        const int h = item / n_chunks, chunk = item - h * n_chunks;
        const float* kr = L.k_ring + (size_t)h * A.cap * hd + lane * 4;
        const float* vr = L.v_ring + (size_t)h * A.cap * hd + lane * 4;
        const float* qh = A.q + (size_t)h * G * hd + lane * 4;
        float4 q[G], acc[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            q[g] = dim_ok ? __ldcg(reinterpret_cast<const float4*>(qh + (size_t)g * hd)) : make_float4(0.f, 0.f, 0.f, 0.f);
            acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float m_run = -INFINITY, l_run = 0.f;  // of head my_g
        for (int i = 0; i < gpw; ++i) {
            const int grp = chunk * cgroups + warp + kNW * i;
            if (grp >= groups) break;
            const int t0 = mask_start + grp * TPG;
            int slot0 = st.start + t0;
            if (slot0 >= A.cap) slot0 -= A.cap;
            float4 kk[TPG];
#pragma unroll
            for (int j = 0; j < TPG; ++j) {
                int slot = slot0 + j;
                if (slot >= A.cap) slot -= A.cap;
                kk[j] = (dim_ok && t0 + j < len) ? __ldcg(reinterpret_cast<const float4*>(kr + (size_t)slot * hd))
                                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            float sc[32];  // ops.rs:108-113: q . k * scale
#pragma unroll
            for (int g = 0; g < G; ++g)
#pragma unroll
                for (int j = 0; j < TPG; ++j) {
                    float d = q[g].x * kk[j].x;
                    d = fmaf(q[g].y, kk[j].y, d);
                    d = fmaf(q[g].z, kk[j].z, d);
                    sc[g * TPG + j] = fmaf(q[g].w, kk[j].w, d);
                }
            tok_transpose_reduce(sc, lane);
            float4 vv[TPG];
#pragma unroll
            for (int j = 0; j < TPG; ++j) {
                int slot = slot0 + j;
                if (slot >= A.cap) slot -= A.cap;
                vv[j] = (dim_ok && t0 + j < len) ? __ldcg(reinterpret_cast<const float4*>(vr + (size_t)slot * hd))
                                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            float sv = sc[0] * A.scale;
            if (t0 + my_t >= len) sv = -INFINITY;
            float gm = sv;  // online softmax (math.rs:67-88 restated incrementally)
#pragma unroll
            for (int o = TPG / 2; o >= 1; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(FULL, gm, o));
            const float m_new = fmaxf(m_run, gm);
            const float p = (sv == -INFINITY) ? 0.f : expf(sv - m_new);
            float ps = p;
#pragma unroll
            for (int o = TPG / 2; o >= 1; o >>= 1) ps += __shfl_xor_sync(FULL, ps, o);
            const float alpha = (m_run == -INFINITY) ? 0.f : expf(m_run - m_new);
            l_run = l_run * alpha + ps;
            m_run = m_new;
#pragma unroll
            for (int g = 0; g < G; ++g) {  // PV (ops.rs:117-128)
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
        // combine the CTA's warps into one chunk partial
        attn_sync();  // the previous item's readers of the shared partials are done
        if (dim_ok)
#pragma unroll
            for (int g = 0; g < G; ++g) *reinterpret_cast<float4*>(wacc + ((size_t)warp * G + g) * hd + lane * 4) = acc[g];
        if (my_t == 0) {
            wml[(warp * G + my_g) * 2] = m_run;
            wml[(warp * G + my_g) * 2 + 1] = l_run;
        }
        attn_sync();
        float* pacc = A.attn_part + ((size_t)h * A.splits + chunk) * acc_stride;
        float* pml = A.attn_part + ml_base + ((size_t)h * A.splits + chunk) * G * 2;
        for (int o = tid; o < G * hd4; o += kConsumers) {
            const int g = o / hd4, d = (o - g * hd4) * 4;
            float M = -INFINITY;
            for (int w = 0; w < kNW; ++w) M = fmaxf(M, wml[(w * G + g) * 2]);
            float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
            float Ls = 0.f;
            for (int w = 0; w < kNW; ++w) {
                const float mw = wml[(w * G + g) * 2];
                const float e = mw == -INFINITY ? 0.f : expf(mw - M);
                const float4 a = *reinterpret_cast<const float4*>(wacc + ((size_t)w * G + g) * hd + d);
                sum.x = fmaf(e, a.x, sum.x);
                sum.y = fmaf(e, a.y, sum.y);
                sum.z = fmaf(e, a.z, sum.z);
                sum.w = fmaf(e, a.w, sum.w);
                Ls = fmaf(e, wml[(w * G + g) * 2 + 1], Ls);
            }
            *reinterpret_cast<float4*>(pacc + (size_t)g * hd + d) = sum;
            if (d == 0) {
                pml[g * 2] = M;
                pml[g * 2 + 1] = Ls;
            }
        }
        __threadfence();
        attn_sync();
        if (tid == 0) {
            const unsigned ticket = atomicAdd(&A.tickets[h], 1u);
            *flag_s = (ticket == (unsigned)(n_chunks - 1)) ? 1 : 0;
        }
        attn_sync();
        if (!*flag_s) continue;
        __threadfence();
        // last chunk of kv head h: merge weights once per head, then sums
        const float* bacc = A.attn_part + (size_t)h * A.splits * acc_stride;
        const float* bml = A.attn_part + ml_base + (size_t)h * A.splits * G * 2;
        for (int g = warp; g < G; g += kNW) {
            float ms[2], ls[2];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int sp = lane + 32 * r;
                ms[r] = sp < n_chunks ? __ldcg(bml + ((size_t)sp * G + g) * 2) : -INFINITY;
                ls[r] = sp < n_chunks ? __ldcg(bml + ((size_t)sp * G + g) * 2 + 1) : 0.f;
            }
            float M = fmaxf(ms[0], ms[1]);
#pragma unroll
            for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(FULL, M, o));
            float w[2], Lsum = 0.f;
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                w[r] = ms[r] == -INFINITY ? 0.f : expf(ms[r] - M);
                Lsum = fmaf(ls[r], w[r], Lsum);
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) Lsum += __shfl_xor_sync(FULL, Lsum, o);
            const float invL = Lsum > 0.f ? 1.0f / Lsum : 0.f;
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int sp = lane + 32 * r;
                if (sp < n_chunks) w_s[g * kMaxSplits + sp] = w[r] * invL;
            }
        }
        attn_sync();
        float* out = A.attn + (size_t)h * G * hd;
        for (int o = tid; o < G * hd4; o += kConsumers) {
            const int g = o / hd4, d = (o - g * hd4) * 4;
            const float* pv = bacc + (size_t)g * hd + d;
            float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int s0 = 0; s0 < n_chunks; s0 += 16) {
                float4 v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    v[j] = s0 + j < n_chunks ? __ldcg(reinterpret_cast<const float4*>(pv + (size_t)(s0 + j) * acc_stride))
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    if (s0 + j < n_chunks) {
                        const float wj = w_s[g * kMaxSplits + s0 + j];
                        sum.x = fmaf(wj, v[j].x, sum.x);
                        sum.y = fmaf(wj, v[j].y, sum.y);
                        sum.z = fmaf(wj, v[j].z, sum.z);
                        sum.w = fmaf(wj, v[j].w, sum.w);
                    }
                }
            }
            *reinterpret_cast<float4*>(out + (size_t)g * hd + d) = sum;
        }
        if (tid == 0) A.tickets[h] = 0u;
    }
}

__device__ void attn_phase(const TokenArgs& A, const TokLayer& L, float* work) {
    if (A.n_heads == 4 * A.n_kv)
        attn_phase_warp<4>(A, L, work);
    else
        attn_phase_warp<8>(A, L, work);
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
// __grid_constant__: phase functions take the arguments by reference straight
// from the constant parameter bank instead of a per-thread local copy.
__global__ void __launch_bounds__(kThreads, 1) token_step_kernel(const __grid_constant__ TokenArgs A) {
    extern __shared__ __align__(128) unsigned char smem[];
    const Layout Lo = token_layout(A, gridDim.x);
    unsigned char* ring = smem;
    float* work = reinterpret_cast<float*>(smem + Lo.work_off);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Lo.bar_off);
    uint64_t* empty = full + kSlots;
    float* scratch = reinterpret_cast<float*>(smem + Lo.scratch_off);
    int* flag_s = reinterpret_cast<int*>(scratch + 48);
    unsigned long long* base_s = reinterpret_cast<unsigned long long*>(scratch + 50);
    int* fail_s = reinterpret_cast<int*>(scratch + 52);

    const int tid = threadIdx.x, warp = tid >> 5;
    if (tid == 0) {
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kNW);
        }
        fence_barrier_init();
        *base_s = __ldcg(A.bar_base);
        *fail_s = 0;
    }
    __syncthreads();
    uint32_t g_local = 0;  // global stage counter, kept per consumer thread
    uint32_t* g_s = &g_local;

    if (warp == kNW) {
        if ((tid & 31) == 0) producer(A, ring, full, empty);
        return;
    }

    const unsigned long long base = *base_s;
    const unsigned long long G = gridDim.x;
    unsigned long long nbar = 0;
    bool ok = true;
    auto sync = [&]() {
        ++nbar;
        if (ok) ok = grid_sync(A.bar, base + nbar * G, A.err, flag_s);
    };

    for (int l = 0; l < A.n_layers; ++l) {
        const TokLayer* L = A.layers + l;
        PhaseIO io{};
        // 1) RMSNorm -> q|k|v -> RoPE -> ring append (decoder.rs:104-120)
        if (ok) {
            io.norm_w = L->attn_norm;
            io.L = L;
            if (l == 0) {
                int tok = __ldcg(&A.step->tok);
                if (tok < 0 || tok >= A.vocab) {
                    if (tid == 0 && blockIdx.x == 0) raise_error(A.err, ERR_TOKEN_RANGE);
                    tok = 0;
                }
                io.xe = A.embed + (size_t)tok * A.dim;
                io.x_copy_out = A.hid;
            } else {
                io.x = A.hid;
            }
            gemv_dispatch<EPI_QKV>(A, A.g_qkv, io, ring, full, empty, g_s, work, scratch);
        }
        sync();
        // 2) attention over the ring (decoder.rs:121-135)
        if (ok) attn_phase(A, *L, work);
        sync();
        // 3) o-proj + residual (decoder.rs:136-139); commits the append
        if (ok) {
            io = PhaseIO{};
            io.x = A.attn;
            io.y = A.hmid;
            io.resid = A.hid;
            io.L = L;
            io.commit = true;
            gemv_dispatch<EPI_RESID>(A, A.g_o, io, ring, full, empty, g_s, work, scratch);
        }
        sync();
        // 4) RMSNorm -> w1|w3 -> SiLU(gate)*up (decoder.rs:143-150)
        if (ok) {
            io = PhaseIO{};
            io.x = A.hmid;
            io.norm_w = L->ffn_norm;
            io.y = A.act;
            gemv_dispatch<EPI_SWIGLU>(A, A.g_w13, io, ring, full, empty, g_s, work, scratch);
        }
        sync();
        // 5) w2 + residual (decoder.rs:151-152)
        if (ok) {
            io = PhaseIO{};
            io.x = A.act;
            io.y = A.hid;
            io.resid = A.hmid;
            gemv_dispatch<EPI_RESID>(A, A.g_w2, io, ring, full, empty, g_s, work, scratch);
        }
        sync();
    }
    if (A.vocab) {
        if (ok) {
            PhaseIO io{};
            io.x = A.hid;
            io.norm_w = A.final_norm;
            io.y = A.logits;
            gemv_dispatch<EPI_ARGMAX>(A, A.g_head, io, ring, full, empty, g_s, work, scratch);
        }
        sync();
        if (ok && blockIdx.x == 0) {
            // argmax over the per-CTA candidates, lowest index on ties
            const int lane = tid & 31;
            float best = -INFINITY;
            int bi = 0x7FFFFFFF;
            for (int i = tid; i < (int)gridDim.x; i += kConsumers) {
                const float v = __ldcg(&A.am_part[i].v);
                const int idx = __ldcg(&A.am_part[i].i);
                if (v > best || (v == best && idx < bi)) {
                    best = v;
                    bi = idx;
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
            named_barrier_sync(1, kConsumers);
            if (tid == 0) {
                for (int w = 1; w < kNW; ++w)
                    if (scratch[w] > best || (scratch[w] == best && si[w] < bi)) {
                        best = scratch[w];
                        bi = si[w];
                    }
                if (bi == 0x7FFFFFFF) bi = 0;
                StepState* s = A.step;
                s->next_tok = bi;
                if (__ldcg(&s->greedy)) s->tok = bi;
                if (__ldcg(&s->advance)) s->pos = __ldcg(&s->pos) + 1;
                if (A.tok_out) *A.tok_out = bi;
            }
        }
    }
    // Every CTA has read bar_base before the first barrier completed.
    if (blockIdx.x == 0 && tid == 0) *A.bar_base = base + nbar * G;
}

}  // namespace

bool token_plan(int rows, int K, int unit, TokGemv* out) {
    if (K <= 0 || K % 8) return false;
    const int C = K / 8;
    for (int nseg = 1; nseg <= kNW; nseg *= 2) {
        if (C % nseg) continue;
        const int cpt = (C / nseg + 31) / 32;
        const int stage_rows = 2 * (kNW / nseg);
        if (cpt > kMaxCpt || (size_t)stage_rows * K * 2 > kSlotBytes) continue;
        out->rows = rows;
        out->K = K;
        out->unit = unit;
        out->nseg = nseg;
        out->cpt = cpt;
        out->stage_rows = stage_rows;
        return true;
    }
    return false;
}

bool token_kernel_supported(int dim, int hidden, int q_dim, int n_heads, int n_kv, int hd) {
    TokGemv t;
    if (!token_plan(q_dim, dim, 2, &t) || !token_plan(dim, q_dim, 1, &t) || !token_plan(2 * hidden, dim, 2, &t) ||
        !token_plan(dim, hidden, 1, &t))
        return false;
    if (n_kv <= 0 || n_heads % n_kv || hd % 4 || hd > 128) return false;
    const int G = n_heads / n_kv;
    return G == 4 || G == 8;
}

size_t token_smem_bytes(const TokenArgs& a, int grid) { return token_layout(a, grid).total; }

int token_splits(int n_kv, int grid) {
    int s = grid / n_kv;
    if (s < 1) s = 1;
    if (s > kMaxSplits) s = kMaxSplits;
    return s;
}

cudaError_t token_prepare(int /*dev*/) {
    return cudaFuncSetAttribute(token_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

cudaError_t launch_token_step(const TokenArgs& a, int grid, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = token_smem_bytes(a, grid);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {(void*)&a};
    return cudaLaunchKernelExC(&cfg, (void*)token_step_kernel, args);
}

}  // namespace vox
