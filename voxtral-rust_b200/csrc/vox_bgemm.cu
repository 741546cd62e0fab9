// vox_bgemm.cu -- skinny GEMM for multi-stream decode on the 5th-generation
// tensor cores (tcgen05 + TMEM).
//
// Y[b, r] = sum_k W[r, k] * X[b, k] for B <= 8 independent input vectors (the
// reference's `linear`, crates/voxtral/src/ops.rs:11-39, with n_rows = B).
// Weights are read once for all B streams, so the op stays HBM-bound while
// producing B outputs per weight byte.
//
// Layout.  W is pre-tiled once in HBM into 128-row x 64-column bf16 blocks of
// 16 KB, each already in the UMMA canonical K-major no-swizzle layout (8x8
// "core matrices" of 128 bytes: core (m8, k2) of K-step s at
// s*4 KB + (k2*16 + m8)*128, so LBO = 2 KB between K halves and SBO = 128 B
// between 8-row groups).  A work item = one 128-row tile x a range of K
// blocks; its blocks are contiguous, so a producer lane streams them with 1-D
// cp.async.bulk (no tensor map, one destination CTA) into a 4-stage ring.
//
// The B operand is X converted to bf16 twice: hi = bf16(x), lo = bf16(x - hi)
// as columns b and 8 + b of an N = 16 operand, so the product carries ~16
// mantissa bits of the f32 activations; hi and lo are summed in the epilogue.
//
// One lane issues tcgen05.mma (kind::f16, M=128, N=16, K=16, f32 accumulate)
// into a double-buffered TMEM accumulator; tcgen05.commit frees ring stages
// and signals the epilogue warpgroup, which reads the accumulator with
// tcgen05.ld.  Items that split K write partial tiles; the last item of a tile
// (atomic ticket) sums them in split order, so results are deterministic.
#include <cuda_runtime.h>
#include <math.h>

#include "vox_device.cuh"
#include "vox_tcgen05.cuh"

namespace vox {

namespace {

constexpr int kBM = 128;                     // tile rows (UMMA M)
constexpr int kBK = 64;                      // K elements per block
constexpr int kBlockBytes = kBM * kBK * 2;   // 16 KB
constexpr int kStageBlocks = 2;              // blocks per ring stage
constexpr int kStageBytes = kStageBlocks * kBlockBytes;
constexpr int kStages = 4;                   // 128 KB ring in flight per SM
constexpr int kN = 16;                       // UMMA N: 8 streams x (hi, lo)
constexpr int kThreads = 256;                // w0 producer, w1 MMA, w4..w7 epilogue, w1..w7 X prep
constexpr int kWorkers = kThreads - 32;      // every warp but the producer
constexpr uint32_t kTmemCols = 32;           // two 16-column accumulators

constexpr uint32_t kIdesc = umma_idesc_bf16(kBM, kN);

__device__ __forceinline__ uint16_t f2bf(float f) {  // round to nearest even
    const uint32_t u = __float_as_uint(f);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

// Work item i -> (tile, split); a CTA's items keep their split (and so the X
// slab) when the grid is a multiple of the split count.
struct Item {
    int tile, ks, kb0, kb1;
};
__device__ __forceinline__ Item item_of(const BgArgs& A, int i) {
    Item it;
    it.ks = i % A.splits;
    it.tile = i / A.splits;
    it.kb0 = (int)((long long)A.kbt * it.ks / A.splits);
    it.kb1 = (int)((long long)A.kbt * (it.ks + 1) / A.splits);
    return it;
}

constexpr unsigned kFull = 0xFFFFFFFFu;

// Small shared state of the epilogue warpgroup.
constexpr int kMaxSspParts = 64;  // RMSNorm partial sums per stream (dim <= 8192)

struct EpiShared {
    float ssp[kMaxSspParts * 8];  // RMSNorm partial sums of squares, staged
    float inv[8];     // per-stream RMSNorm factor
    float red[4][8];  // per-warp partial sums / maxima
    int redi[4][8];   // per-warp argmax indices
    int flag;         // this item completes its tile
};

// Inputs of a row's epilogue that do not depend on the product: the
// residual row (BG_RESID), the rotation factors and ring slots (BG_QKV), the
// bias (BG_STORE).  The epilogue warps load them while the MMAs of the item
// run, so the last item of a tile (the critical path of the launch) issues
// only stores after its split sum.  Every producer of these values finished
// before this phase started (grid dependency or phase barrier).
struct EpiInputs {
    float a[8], c[8];  // residual or cos (a), sin (c)
    int slot[8];       // ring slot of the appended token per stream
    float s;           // bias or RMSNorm gain of the row
};

__device__ __forceinline__ void bg_epilogue_inputs(const BgArgs& A, int tile, int row, EpiInputs& in) {
    const int r = tile * kBM + row;
    const bool live = r < A.rows;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
        in.a[b] = 0.0f;
        in.c[b] = 0.0f;
        in.slot[b] = 0;
    }
    in.s = 0.0f;
    if (!live) return;
    if (A.epi == BG_STORE) {
        if (A.bias) in.s = A.bias[r];
    } else if (A.epi == BG_RESID) {
#pragma unroll
        for (int b = 0; b < 8; ++b)
            if (b < A.B) in.a[b] = __ldcg(A.resid + (size_t)b * A.y_stride + r);
        in.s = A.xop_out && A.xop_gain ? A.xop_gain[r] : 1.0f;
    } else if (A.epi == BG_QKV) {
        const int half = A.head_dim / 2;
        const bool rope = r < A.q_dim + A.kv_dim, is_q = r < A.q_dim;
        const int rr = is_q ? r : rope ? r - A.q_dim : r - A.q_dim - A.kv_dim;
        const int d = rr % A.head_dim;
        // positions and cache states of the 8 streams in one round trip, then
        // the rotation table rows in a second
        long long pos[8];
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            pos[b] = 0;
            if (b >= A.B) continue;
            if (rope) pos[b] = A.steps[b].pos;
            if (!is_q) {
                const KvState post =
                    kv_after_single_append(A.kv_state[(size_t)b * A.kv_state_stride], A.kv_window, A.ring_cap);
                in.slot[b] = (post.start + post.len - 1) % A.ring_cap;
            }
        }
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            if (!rope || b >= A.B) continue;
            long long p = pos[b];
            if (p < 0 || p >= A.max_pos) {
                if (row == 0) raise_error(A.err, ERR_POS_RANGE);
                p = 0;
            }
            in.a[b] = A.rope_cos[p * half + d / 2];
            in.c[b] = A.rope_sin[p * half + d / 2];
        }
    }
}

// Final values y[b] of row `row` of tile `tile` for every stream, after the
// split sum.  Runs on all 128 threads of the epilogue warpgroup (warp ew);
// rows beyond A.rows hold zeros and store nothing.
__device__ __forceinline__ void bg_epilogue(const BgArgs& A, int tile, int row, int lane, int ew, float (&y)[8],
                                            const EpiInputs& in, EpiShared* es) {
    const int r = tile * kBM + row;
    const bool live = r < A.rows;
    if (A.epi == BG_STORE) {
        if (live) {
#pragma unroll
            for (int b = 0; b < 8; ++b)
                if (b < A.B) A.y[(size_t)b * A.y_stride + r] = A.bias ? __fadd_rn(in.s, y[b]) : y[b];
        }
    } else if (A.epi == BG_QKV) {
        // RoPE pairs (2p, 2p + 1) sit in adjacent lanes (math.rs:58-61, unfused).
        float partner[8];
#pragma unroll
        for (int b = 0; b < 8; ++b) partner[b] = __shfl_xor_sync(kFull, y[b], 1);
        if (!live) return;
        const bool rope = r < A.q_dim + A.kv_dim, is_q = r < A.q_dim;
        const int rr = is_q ? r : rope ? r - A.q_dim : r - A.q_dim - A.kv_dim;
        const int d = rr % A.head_dim, h = rr / A.head_dim;
        const bool odd = d & 1;
        float* const ring = rope ? A.k_ring : A.v_ring;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            if (b >= A.B) continue;
            float o = y[b];
            if (rope) {
                const float c = in.a[b], sn = in.c[b];
                const float ya = odd ? partner[b] : y[b], yb = odd ? y[b] : partner[b];
                o = odd ? __fadd_rn(__fmul_rn(ya, sn), __fmul_rn(yb, c)) : __fsub_rn(__fmul_rn(ya, c), __fmul_rn(yb, sn));
            }
            if (is_q)
                A.y[(size_t)b * A.y_stride + r] = o;
            else
                ring[(size_t)b * A.ring_stride + ((size_t)h * A.ring_cap + in.slot[b]) * A.head_dim + d] = o;
        }
    } else if (A.epi == BG_SWIGLU) {
        // rows 2j (w1) and 2j + 1 (w3): act[j] = silu(gate) * up (decoder.rs:147-150)
        float up[8];
#pragma unroll
        for (int b = 0; b < 8; ++b) up[b] = __shfl_xor_sync(kFull, y[b], 1);
        if (live && !(r & 1)) {
            const int j = r >> 1;
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                if (b >= A.B) continue;
                const float sg = __fdiv_rn(y[b], __fadd_rn(1.0f, expf(-y[b])));
                const float act = __fmul_rn(sg, up[b]);
                A.y[(size_t)b * A.y_stride + j] = act;
                if (A.xop_out) xop_store(A.xop_out, j, b, act);
            }
        }
    } else if (A.epi == BG_RESID) {
        // y = resid + W x (decoder.rs:136-139, 151-152), plus this tile's sums of
        // squares of the new hidden state for the next RMSNorm.
        float sq[8];
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            sq[b] = 0.0f;
            if (live && b < A.B) {
                const float v = __fadd_rn(in.a[b], y[b]);
                A.y[(size_t)b * A.y_stride + r] = v;
                sq[b] = __fmul_rn(v, v);
                if (A.xop_out) xop_store(A.xop_out, r, b, A.xop_gain ? __fmul_rn(v, in.s) : v);
            }
        }
        if (A.ssp_out) {
#pragma unroll
            for (int b = 0; b < 8; ++b)
#pragma unroll
                for (int o = 16; o; o >>= 1) sq[b] += __shfl_xor_sync(kFull, sq[b], o);
            if (lane == 0)
#pragma unroll
                for (int b = 0; b < 8; ++b) es->red[ew][b] = sq[b];
            named_barrier_sync(2, 128);
            if (row < 8) {
                const int b = row;
                A.ssp_out[(size_t)tile * 8 + b] = ((es->red[0][b] + es->red[1][b]) + es->red[2][b]) + es->red[3][b];
            }
            named_barrier_sync(2, 128);
        }
    } else if (A.epi == BG_ARGMAX) {
        // logits (optional) and the tile's best (value, lowest index) per stream
        float best[8];
        int bi[8];
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            best[b] = -INFINITY;
            bi[b] = 0x7FFFFFFF;
            if (live && b < A.B) {
                if (A.y) A.y[(size_t)b * A.y_stride + r] = y[b];
                if (y[b] > best[b]) {
                    best[b] = y[b];
                    bi[b] = r;
                }
            }
        }
#pragma unroll
        for (int b = 0; b < 8; ++b) {
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                const float ov = __shfl_xor_sync(kFull, best[b], o);
                const int oi = __shfl_xor_sync(kFull, bi[b], o);
                if (ov > best[b] || (ov == best[b] && oi < bi[b])) {
                    best[b] = ov;
                    bi[b] = oi;
                }
            }
        }
        if (lane == 0)
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                es->red[ew][b] = best[b];
                es->redi[ew][b] = bi[b];
            }
        named_barrier_sync(2, 128);
        if (row < 8) {
            const int b = row;
            float bv = es->red[0][b];
            int bix = es->redi[0][b];
            for (int w = 1; w < 4; ++w)
                if (es->red[w][b] > bv || (es->red[w][b] == bv && es->redi[w][b] < bix)) {
                    bv = es->red[w][b];
                    bix = es->redi[w][b];
                }
            A.am_part[(size_t)tile * 8 + b].v = bv;
            A.am_part[(size_t)tile * 8 + b].i = bix;
        }
        named_barrier_sync(2, 128);
    }
}

// All worker threads of every CTA: wait until all `n` CTAs have counted
// themselves into `done` (bounded; false when the wait expired).  The
// arrival is made by the caller after its own outputs are written.
__device__ bool wait_all_ctas(unsigned* done, unsigned n, unsigned* err, EpiShared* es) {
    if (threadIdx.x == 32) {
        bool ok = true;
        uint64_t t0 = 0;
        uint32_t it = 0;
        while (true) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(done) : "memory");
            if (v >= n) break;
            if ((++it & 63u) == 0) {
                const uint64_t now = global_timer_ns();
                if (t0 == 0) {
                    t0 = now;
                } else if (now - t0 > kWaitLimitNs) {
                    raise_error(err, ERR_GRID_WAIT);
                    ok = false;
                    break;
                }
            }
        }
        es->flag = ok ? 1 : 0;
    }
    named_barrier_sync(1, kWorkers);
    return es->flag != 0;
}

// One launch runs a chain of up to kBgMaxPhases GEMMs back to back (o-proj,
// w1|w3, w2 and the next layer's q|k|v, or the LM head).  The producer lane
// streams the weights of every phase without a break, since weights never
// depend on earlier phases; the workers of phase p > 0 wait until every CTA
// has finished phase p - 1 (a completion counter in global memory) before
// they read its outputs.  The 128 KB ring holds the next phase's first
// blocks meanwhile, so the wait costs little HBM time.  All CTAs are
// resident together: one CTA per SM, grid <= SM count, and a dependent
// launch cannot start before every CTA of this one has started.
__global__ void __launch_bounds__(kThreads, 1) bgemm_kernel(const __grid_constant__ BgChain C) {
    extern __shared__ __align__(1024) unsigned char smem[];
    unsigned char* ring = smem;                                // kStages x 32 KB
    unsigned char* xs = smem + kStages * kStageBytes;          // X slab: one 512 B slab per K step
    uint64_t* full = reinterpret_cast<uint64_t*>(xs + C.xslab_bytes);
    uint64_t* empty = full + kStages;
    uint64_t* acc_full = empty + kStages;  // [2]
    uint64_t* acc_empty = acc_full + 2;    // [2]
    uint64_t* xbar = acc_empty + 2;        // X operand bulk copy
    uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(xbar + 2);
    EpiShared* es = reinterpret_cast<EpiShared*>(tmem_base_s + 4);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    unsigned* const err = C.ph[0].err;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
        }
        mbar_init(xbar, 1);
        fence_barrier_init();
    }
    if (warp == 1) {  // TMEM accumulators: the whole warp allocates
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(tmem_base_s)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tmem = *tmem_base_s;
    pdl_allow_dependents();
    uint32_t xphase = 0;  // parity of the next X-operand copy (MMA lane only)

    // ---- producer: stream this CTA's weight blocks of every phase ----
    if (warp == 0) {
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            uint32_t g = 0;
            bool ok = true;
            for (int ph = 0; ph < C.n_phases && ok; ++ph) {
                const BgArgs& A = C.ph[ph];
                const int n_items = A.tiles * A.splits;
                for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
                    const Item it = item_of(A, i);
                    const unsigned char* src = A.wt + ((size_t)it.tile * A.kbt + it.kb0) * kBlockBytes;
                    for (int kb = it.kb0; kb < it.kb1; kb += kStageBlocks, ++g) {
                        const int slot = (int)(g % kStages);
                        if (g >= (uint32_t)kStages && !mbar_wait(&empty[slot], ((g / kStages) - 1) & 1)) {
                            raise_error(err, ERR_EMPTY_WAIT);
                            ok = false;
                            break;
                        }
                        const int nb = min(kStageBlocks, it.kb1 - kb);
                        mbar_arrive_expect_tx(&full[slot], (uint32_t)(nb * kBlockBytes));
                        bulk_copy_g2s(ring + (size_t)slot * kStageBytes, src + (size_t)(kb - it.kb0) * kBlockBytes,
                                      (uint32_t)(nb * kBlockBytes), &full[slot], pol);
                    }
                }
            }
            // no copy may be in flight when the CTA exits
            const uint32_t first = g > (uint32_t)kStages ? g - kStages : 0u;
            for (uint32_t s = first; s < g; ++s)
                if (!mbar_wait(&full[s % kStages], (s / kStages) & 1)) raise_error(err, ERR_DRAIN_WAIT);
        }
        // The producer warp takes no part in the rest (its lane 0 streams while
        // the other warps work), so the worker barriers below exclude it.
        pdl_wait_prior_grids();
        return;
    }

    pdl_wait_prior_grids();

    uint32_t g_mma = 0;
    bool mma_ok = true;  // after a wait expires the issuer stops waiting (the result is flagged)
    int local = 0;       // items processed by this CTA, over all phases
    for (int ph = 0; ph < C.n_phases; ++ph) {
        const BgArgs& A = C.ph[ph];
        if (ph > 0) {
            // This CTA's outputs of the previous phase are written (every worker
            // passed its epilogue); count the CTA in, then wait for all others.
            named_barrier_sync(1, kWorkers);
            if (tid == 32) {
                __threadfence();
                atomicAdd(C.done + ph - 1, 1u);
            }
            if (!wait_all_ctas(C.done + ph - 1, gridDim.x, err, es)) mma_ok = false;
        }
        // This launch commits the single-token append of the layer's cache of
        // every stream (the attention launch before it read the old state).
        if (A.kv_commit && blockIdx.x == 0 && tid >= 32 && tid < 32 + A.B) {
            KvState* st = A.kv_commit + (size_t)(tid - 32) * A.kv_state_stride;
            *st = kv_after_single_append(*st, A.kv_window, A.ring_cap);
        }
        // Per-stream RMSNorm factor from the producer's partial sums of squares
        // (math.rs:22: inv = 1 / sqrt(sum / dim + eps)), applied in the X prologue.
        const bool xop = A.xop != nullptr;
        if (A.norm_w && !xop) {
            // all partials loaded at once (one L2 round trip), summed in part order
            const int n = A.ssp_parts * 8;
            for (int e = tid - 32; e < n && e < kMaxSspParts * 8; e += kWorkers) es->ssp[e] = __ldcg(A.ssp + e);
            named_barrier_sync(1, kWorkers);
            if (tid >= 32 && tid < 40) {
                const int b = tid - 32;
                float inv = 1.0f;
                if (b < A.B) {
                    float ss = 0.0f;
                    for (int p = 0; p < A.ssp_parts; ++p) ss += es->ssp[p * 8 + b];
                    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)A.K), A.eps)));
                }
                es->inv[b] = inv;
            }
            named_barrier_sync(1, kWorkers);
        } else if (A.norm_w && warp >= 4) {
            // X operand already holds x * g: the epilogue warpgroup scales the
            // row sums by inv (y = inv * W (x * g)) while the MMAs run
            const int n = A.ssp_parts * 8;
            for (int e = tid - 128; e < n && e < kMaxSspParts * 8; e += 128) es->ssp[e] = __ldcg(A.ssp + e);
            named_barrier_sync(2, 128);
            if (tid >= 128 && tid < 136) {
                const int b = tid - 128;
                float inv = 1.0f;
                if (b < A.B) {
                    float ss = 0.0f;
                    for (int p = 0; p < A.ssp_parts; ++p) ss += es->ssp[p * 8 + b];
                    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)A.K), A.eps)));
                }
                es->inv[b] = inv;
            }
            named_barrier_sync(2, 128);
        }

        const int n_items = A.tiles * A.splits;
        int cur_ks = -1;
        for (int i = blockIdx.x; i < n_items; i += gridDim.x, ++local) {
            const Item it = item_of(A, i);
            const int nkb = it.kb1 - it.kb0;
            // ---- X slab for this split: built by warps 1..7, or copied (XOP) ----
            const bool new_x = it.ks != cur_ks;
            if (new_x && !xop) {
                if (local > 0) {  // the previous item's MMAs read the old slab: wait for their commit
                    const int pb = (local - 1) & 1;
                    if (!mbar_wait(&acc_full[pb], ((local - 1) >> 1) & 1)) raise_error(err, ERR_FULL_WAIT);
                }
                const int kbase = it.kb0 * kBK;
                const int nk8 = nkb * kBK / 8;  // 8-element chunks per stream
                const int n_tasks = 8 * nk8;
                // four chunks per thread per round, all loads issued before any store
                for (int e0 = tid - 32; e0 < n_tasks; e0 += 4 * kWorkers) {
                    float4 xa[4][2];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int e = e0 + u * kWorkers;
                        const int b = e / nk8;
                        const int k = (e - b * nk8) * 8;
                        if (e < n_tasks && b < A.B) {
                            const float* xp = A.x + (size_t)b * A.x_stride + kbase + k;
                            xa[u][0] = __ldcg(reinterpret_cast<const float4*>(xp));
                            xa[u][1] = __ldcg(reinterpret_cast<const float4*>(xp + 4));
                        } else {
                            xa[u][0] = xa[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
                        }
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int e = e0 + u * kWorkers;
                        if (e >= n_tasks) break;
                        const int b = e / nk8;
                        const int k = (e - b * nk8) * 8;
                        uint32_t hi[4] = {0, 0, 0, 0}, lo[4] = {0, 0, 0, 0};
                        if (b < A.B) {
                            float v[8] = {xa[u][0].x, xa[u][0].y, xa[u][0].z, xa[u][0].w,
                                          xa[u][1].x, xa[u][1].y, xa[u][1].z, xa[u][1].w};
                            if (A.norm_w) {  // math.rs:23-24: x * inv * w, in that order
                                const float4 g0 = __ldg(reinterpret_cast<const float4*>(A.norm_w + kbase + k));
                                const float4 g1 = __ldg(reinterpret_cast<const float4*>(A.norm_w + kbase + k + 4));
                                const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
                                const float inv = es->inv[b];
#pragma unroll
                                for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(__fmul_rn(v[j], inv), gv[j]);
                            }
#pragma unroll
                            for (int j = 0; j < 8; j += 2) {
                                const uint16_t h0 = f2bf(v[j]), h1 = f2bf(v[j + 1]);
                                const uint16_t l0 = f2bf(v[j] - bf16_bits_to_f32(h0));
                                const uint16_t l1 = f2bf(v[j + 1] - bf16_bits_to_f32(h1));
                                hi[j >> 1] = (uint32_t)h0 | ((uint32_t)h1 << 16);
                                lo[j >> 1] = (uint32_t)l0 | ((uint32_t)l1 << 16);
                            }
                        }
                        // core (n8, k2) of K-step s at s*512 + (k2*2 + n8)*128 + row*16:
                        // hi parts are rows 0..7 (n8 = 0), lo parts rows 8..15 (n8 = 1)
                        const int s = k / 16, k2 = (k / 8) & 1;
                        unsigned char* base = xs + (size_t)s * 512 + (size_t)k2 * 256;
                        *reinterpret_cast<uint4*>(base + b * 16) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                        *reinterpret_cast<uint4*>(base + 128 + b * 16) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                    }
                }
                // generic-proxy writes must be visible to the tensor core (async proxy)
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                named_barrier_sync(1, kWorkers);
            }
            cur_ks = it.ks;

            const int ab = local & 1;  // accumulator buffer
            // ---- MMA issuer ----
            if (warp == 1 && lane == 0) {
                if (xop && new_x) {
                    // the previous item's MMAs read the old slab: wait for their commit
                    if (local > 0 && !mbar_wait(&acc_full[(local - 1) & 1], ((local - 1) >> 1) & 1))
                        raise_error(err, ERR_FULL_WAIT);
                    const uint32_t xb = (uint32_t)(nkb * 2048);
                    mbar_arrive_expect_tx(xbar, xb);
                    bulk_copy_g2s_nohint(xs, A.xop + (size_t)it.kb0 * 2048, xb, xbar);
                    if (!mbar_wait(xbar, xphase)) {
                        raise_error(err, ERR_FULL_WAIT);
                        mma_ok = false;
                    }
                    xphase ^= 1u;
                }
                if (mma_ok && local >= 2 && !mbar_wait(&acc_empty[ab], ((local - 2) >> 1) & 1)) {
                    raise_error(err, ERR_FULL_WAIT);
                    mma_ok = false;
                }
                tmem_fence_after();
                const uint32_t d = tmem + (uint32_t)(ab * kN);
                const uint32_t xs_addr = smem_addr(xs);
                int kstep = 0;
                for (int kb = it.kb0; kb < it.kb1; kb += kStageBlocks, ++g_mma) {
                    const int slot = (int)(g_mma % kStages);
                    if (!mma_ok) break;
                    if (!mbar_wait(&full[slot], (g_mma / kStages) & 1)) {
                        raise_error(err, ERR_FULL_WAIT);
                        mma_ok = false;
                        break;
                    }
                    tmem_fence_after();
                    const int nb = min(kStageBlocks, it.kb1 - kb);
                    const uint32_t a_addr = smem_addr(ring + (size_t)slot * kStageBytes);
                    for (int j = 0; j < nb * 4; ++j, ++kstep) {
                        const uint64_t ad = umma_desc(a_addr + (uint32_t)j * 4096u, 2048u, 128u);
                        const uint64_t bd = umma_desc(xs_addr + (uint32_t)kstep * 512u, 256u, 128u);
                        umma_f16(d, ad, bd, kIdesc, kstep > 0 ? 1u : 0u);
                    }
                    umma_commit(&empty[slot]);  // frees the stage once these MMAs have read it
                }
                umma_commit(&acc_full[ab]);  // accumulator ready for the epilogue
            }
            __syncwarp();  // warp 1 reconverges before any later barrier

            // ---- epilogue warpgroup: TMEM -> registers -> partial or final rows ----
            if (warp >= 4) {
                const int ew = warp - 4;        // TMEM lanes 32*ew .. 32*ew + 31
                const int row = ew * 32 + lane; // row inside the tile
                EpiInputs in;
                bg_epilogue_inputs(A, it.tile, row, in);
                if (!mbar_wait(&acc_full[ab], (local >> 1) & 1)) raise_error(err, ERR_FULL_WAIT);
                tmem_fence_after();
                uint32_t raw[16];
                tmem_ld16(tmem + ((uint32_t)(ew * 32) << 16) + (uint32_t)(ab * kN), raw);
                tmem_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[ab]);
                float y[8];
#pragma unroll
                for (int b = 0; b < 8; ++b) y[b] = __uint_as_float(raw[b]) + __uint_as_float(raw[8 + b]);

                bool final_item = true;
                if (A.splits > 1) {
                    float* part = A.part + ((size_t)i * kBM + row) * 8;
                    *reinterpret_cast<float4*>(part) = make_float4(y[0], y[1], y[2], y[3]);
                    *reinterpret_cast<float4*>(part + 4) = make_float4(y[4], y[5], y[6], y[7]);
                    __threadfence();
                    named_barrier_sync(2, 128);
                    if (ew == 0 && lane == 0) {
                        const unsigned t = atomicAdd(&A.tickets[it.tile], 1u);
                        es->flag = (t == (unsigned)(A.splits - 1)) ? 1 : 0;
                    }
                    named_barrier_sync(2, 128);
                    final_item = es->flag != 0;
                    named_barrier_sync(2, 128);  // flag read by all before the next item rewrites it
                    if (final_item) {
                        __threadfence();
#pragma unroll
                        for (int b = 0; b < 8; ++b) y[b] = 0.0f;
                        for (int k0 = 0; k0 < A.splits; k0 += 4) {  // four splits' loads in flight
                            float4 pv[4][2];
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                if (k0 + u < A.splits) {
                                    const float* p = A.part + ((size_t)(it.tile * A.splits + k0 + u) * kBM + row) * 8;
                                    pv[u][0] = __ldcg(reinterpret_cast<const float4*>(p));
                                    pv[u][1] = __ldcg(reinterpret_cast<const float4*>(p + 4));
                                } else {
                                    pv[u][0] = pv[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
                                }
                            }
#pragma unroll
                            for (int u = 0; u < 4; ++u) {  // split order, as the partials were made
                                y[0] += pv[u][0].x; y[1] += pv[u][0].y; y[2] += pv[u][0].z; y[3] += pv[u][0].w;
                                y[4] += pv[u][1].x; y[5] += pv[u][1].y; y[6] += pv[u][1].z; y[7] += pv[u][1].w;
                            }
                        }
                        if (ew == 0 && lane == 0) A.tickets[it.tile] = 0u;
                    }
                }
                if (final_item) {
                    if (xop && A.norm_w)
#pragma unroll
                        for (int b = 0; b < 8; ++b) y[b] = __fmul_rn(es->inv[b], y[b]);
                    bg_epilogue(A, it.tile, row, lane, ew, y, in, es);
                }
            }
        }
    }

    // TMEM is released by the warp that allocated it, after every reader is done.
    tmem_fence_before();
    named_barrier_sync(1, kWorkers);
    if (warp == 1) {
        tmem_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                     : "memory");
    }
}

__global__ void tile_weights_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst, int rows,
                                    int K, int tiles) {
    const int kbt = K / kBK;
    const long long total = (long long)tiles * kBM * K;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(e / K), k = (int)(e - (long long)r * K);
        const int t = r / kBM, rr = r - t * kBM;
        const int kb = k / kBK, kk = k - kb * kBK;
        const int s = kk / 16, k2 = (kk / 8) & 1, kin = kk & 7;
        const int m8 = rr / 8, rin = rr & 7;
        const size_t off = ((size_t)t * kbt + kb) * (kBlockBytes / 2) + (size_t)s * 2048 +
                           (size_t)(k2 * 16 + m8) * 64 + rin * 8 + kin;
        dst[off] = r < rows ? src[(size_t)r * K + k] : (uint16_t)0;
    }
}

// Embedding rows of every stream's token (bf16 widened exactly, as
// weights.rs:77-81) into hid [B, dim], with per-128-column sums of squares
// for the first layer's RMSNorm.  Grid (ceil(dim / 128), B), 128 threads.
// Block (0, 0) also zeroes the step's chain completion counters: every chain
// of the previous step has finished when this kernel runs.
__global__ void __launch_bounds__(128) bg_embed_kernel(const uint16_t* __restrict__ embed, int vocab, int dim,
                                                       const StepState* steps, float* hid, float* ssp,
                                                       unsigned char* xop, const float* xop_gain, unsigned* zero,
                                                       int n_zero, unsigned* err) {
    pdl_allow_dependents();
    pdl_wait_prior_grids();
    if (blockIdx.x == 0 && blockIdx.y == 0)
        for (int i = threadIdx.x; i < n_zero; i += blockDim.x) zero[i] = 0u;
    __shared__ float red[4];
    const int b = blockIdx.y, e = blockIdx.x * 128 + threadIdx.x;
    int tok = steps[b].tok;
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) raise_error(err, ERR_TOKEN_RANGE);
        tok = 0;
    }
    float v = 0.0f;
    if (e < dim) {
        v = bf16_bits_to_f32(embed[(size_t)tok * dim + e]);
        hid[(size_t)b * dim + e] = v;
        if (xop) xop_store(xop, e, b, xop_gain ? __fmul_rn(v, xop_gain[e]) : v);
    }
    float sq = __fmul_rn(v, v);
#pragma unroll
    for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(kFull, sq, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x == 0) ssp[(size_t)blockIdx.x * 8 + b] = ((red[0] + red[1]) + red[2]) + red[3];
}

// Per-stream argmax over the LM head's per-tile candidates (lowest index on
// ties), then the step bookkeeping of that stream.  Grid B, 256 threads.
__global__ void __launch_bounds__(256) bg_argmax_final_kernel(const ArgmaxPart* parts, int n_tiles,
                                                              StepState* steps, int32_t* tok_out) {
    pdl_allow_dependents();
    pdl_wait_prior_grids();
    __shared__ float sv[8];
    __shared__ int si[8];
    const int b = blockIdx.x;
    float best = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (int t = threadIdx.x; t < n_tiles; t += blockDim.x) {
        const ArgmaxPart p = parts[(size_t)t * 8 + b];
        if (p.v > best || (p.v == best && p.i < bi)) {
            best = p.v;
            bi = p.i;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, best, o);
        const int oi = __shfl_xor_sync(kFull, bi, o);
        if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = best;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
                best = sv[w];
                bi = si[w];
            }
        if (bi == 0x7FFFFFFF) bi = 0;  // all logits NaN: token 0, as a scan from index 0 keeps
        StepState* st = steps + b;
        st->next_tok = bi;
        if (st->greedy) st->tok = bi;
        if (st->advance) st->pos += 1;
        if (tok_out) tok_out[b] = bi;
    }
}

}  // namespace

cudaError_t launch_bg_embed(const uint16_t* embed, int vocab, int dim, const StepState* steps, int B, float* hid,
                            float* ssp, unsigned char* xop, const float* xop_gain, unsigned* zero, int n_zero,
                            unsigned* err, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((dim + 127) / 128, B, 1);
    cfg.blockDim = dim3(128, 1, 1);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, bg_embed_kernel, embed, vocab, dim, steps, hid, ssp, xop, xop_gain, zero, n_zero,
                              err);
}

cudaError_t launch_bg_argmax_final(const ArgmaxPart* parts, int n_tiles, StepState* steps, int B,
                                   int32_t* tok_out, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(B, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, bg_argmax_final_kernel, parts, n_tiles, steps, tok_out);
}

int bgemm_xslab_bytes(int K, int splits) {
    const int kbt = K / kBK;
    return ((kbt + splits - 1) / splits) * 4 * 512;
}

size_t bgemm_smem_bytes(int xslab_bytes) {
    return (size_t)kStages * kStageBytes + xslab_bytes + (2 * kStages + 6) * 8 + 16 + sizeof(EpiShared);
}

cudaError_t bgemm_prepare(int /*dev*/) {
    return cudaFuncSetAttribute(bgemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

cudaError_t launch_bgemm(const BgChain& c, int grid, cudaStream_t s, bool pdl) {
    if (c.n_phases < 1 || c.n_phases > kBgMaxPhases || (c.n_phases > 1 && !c.done)) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = bgemm_smem_bytes(c.xslab_bytes);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    void* args[] = {(void*)&c};
    return cudaLaunchKernelExC(&cfg, (void*)bgemm_kernel, args);
}

size_t tiled_bytes(int rows, int K) { return (size_t)((rows + kBM - 1) / kBM) * kBM * K * 2; }

cudaError_t launch_tile_weights(const uint16_t* src, uint16_t* dst, int rows, int K, cudaStream_t s) {
    const int tiles = (rows + kBM - 1) / kBM;
    const long long total = (long long)tiles * kBM * K;
    long long g = (total + 255) / 256;
    if (g > 148 * 16) g = 148 * 16;
    tile_weights_kernel<<<(int)g, 256, 0, s>>>(src, dst, rows, K, tiles);
    return cudaGetLastError();
}

}  // namespace vox
