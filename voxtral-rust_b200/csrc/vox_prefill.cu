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
// Wide form (tn = 128, an even number of tiles): tokens are the M = 128 rows
// (the slab's hi and lo halves as two A operands into one accumulator) and
// two weight tiles the N = 2 x 128 columns; a stage is the slab plus two
// weight blocks, 64 KB for twice the products of a 48 KB stage above.
constexpr int kPfWideStages = 3;
constexpr int kPfWideStageBytes = kPfMaxSlab + 2 * kPfABytes;  // 64 KB
constexpr int kPfThreads = 192;                        // w0 producer, w1 MMA, w2..w5 epilogue
constexpr uint32_t kPfTmemCols = 512;                  // two accumulators of up to 256 columns
constexpr unsigned kFull = 0xFFFFFFFFu;

struct PfItem {
    int tile, ks, nb, kb0, kb1;
};

// Item i -> (weight tile, K split, token block), token block fastest: the
// CTAs that run at the same time share weight blocks, which L2 then serves.
// In the wide form `tile` is a pair of weight tiles.
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

// Eight consecutive elements k .. k + 7 of token t into the prefill operand.
__device__ __forceinline__ void pf_store8(unsigned char* xop, int tn, int kbt, int t, int k, const float (&v)[8]) {
    const int nb = t / tn, tt = t - nb * tn, n = 2 * tn;
    const int kb = k >> 6, kk = k & 63;
    const int s = kk >> 4, k2 = (kk >> 3) & 1;
    unsigned char* base = xop + ((size_t)nb * kbt + kb) * (size_t)n * 128 + (size_t)s * n * 32 + (size_t)k2 * n * 16;
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 8; j += 2) split_bf16x2(v[j], v[j + 1], hi[j >> 1], lo[j >> 1]);
    const int lr = tn + tt;
    *reinterpret_cast<uint4*>(base + (tt >> 3) * 128 + (tt & 7) * 16) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(base + (lr >> 3) * 128 + (lr & 7) * 16) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

template <bool WIDE>
__global__ void __launch_bounds__(kPfThreads, 1) pf_gemm_kernel(const __grid_constant__ PfGemmArgs A) {
    constexpr int kStages = WIDE ? kPfWideStages : kPfStages;
    constexpr int kStageBytes = WIDE ? kPfWideStageBytes : kPfStageBytes;
    extern __shared__ __align__(1024) unsigned char smem[];
    unsigned char* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    uint64_t* acc_full = empty + kStages;  // [2]
    uint64_t* acc_empty = acc_full + 2;    // [2]
    uint32_t* tmem_s = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n = 2 * A.tn;
    const uint32_t slab = (uint32_t)n * 128u;
    const int n_items = (WIDE ? A.tiles / 2 : A.tiles) * A.splits * A.nblocks;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
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
                    const int slot = (int)(g % kStages);
                    if (g >= (uint32_t)kStages && !mbar_wait(&empty[slot], ((g / kStages) - 1) & 1)) {
                        raise_error(A.err, ERR_EMPTY_WAIT);
                        ok = false;
                        break;
                    }
                    unsigned char* dst = ring + (size_t)slot * kStageBytes;
                    const unsigned char* xsrc = A.xop + ((size_t)it.nb * A.kbt + kb) * slab;
                    if (WIDE) {  // slab, then the pair's two weight blocks of this K block
                        mbar_arrive_expect_tx(&full[slot], slab + 2u * kPfABytes);
                        bulk_copy_g2s_nohint(dst, xsrc, slab, &full[slot]);
                        for (int w = 0; w < 2; ++w)
                            bulk_copy_g2s_nohint(dst + slab + w * kPfABytes,
                                                 A.wt + ((size_t)(2 * it.tile + w) * A.kbt + kb) * kPfABytes,
                                                 kPfABytes, &full[slot]);
                    } else {
                        mbar_arrive_expect_tx(&full[slot], (uint32_t)kPfABytes + slab);
                        bulk_copy_g2s_nohint(dst, A.wt + ((size_t)it.tile * A.kbt + kb) * kPfABytes, kPfABytes,
                                             &full[slot]);
                        bulk_copy_g2s_nohint(dst + kPfABytes, xsrc, slab, &full[slot]);
                    }
                }
            }
            // no copy may be in flight when the CTA exits
            const uint32_t first = g > (uint32_t)kStages ? g - kStages : 0u;
            for (uint32_t s = first; s < g; ++s)
                if (!mbar_wait(&full[s % kStages], (s / kStages) & 1)) raise_error(A.err, ERR_DRAIN_WAIT);
        }
        return;  // the barriers below count warps 1..5 only
    }

    if (warp == 1) {
        // ---- MMA issuer: 4 x (M 128, N n, K 16) per K block; wide: 4 x 4 x
        // (M 128 tokens, N 128 weight rows, K 16): hi and lo token rows into the
        // same accumulator, the pair's first tile into columns 0..127, the
        // second into 128..255 ----
        if (lane == 0) {
            const uint32_t idesc = WIDE ? umma_idesc_bf16(128, 128) : umma_idesc_bf16(128, n);
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
                    const int slot = (int)(g % kStages);
                    if (!mbar_wait(&full[slot], (g / kStages) & 1)) {
                        raise_error(A.err, ERR_FULL_WAIT);
                        ok = false;
                        break;
                    }
                    tmem_fence_after();
                    const uint32_t s_addr = smem_addr(ring + (size_t)slot * kStageBytes);
                    if (WIDE) {
                        // slab: K step j at j * 8 KB, K halves 4 KB apart, hi token
                        // rows 0..127 then lo rows from 2 KB; weight blocks after it
                        const uint32_t w_addr = s_addr + slab;
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const uint32_t acc = (kb > it.kb0 || j > 0) ? 1u : 0u;
                            const uint64_t ah = umma_desc(s_addr + (uint32_t)j * b_kstep, b_lbo, 128u);
                            const uint64_t al = umma_desc(s_addr + (uint32_t)j * b_kstep + 2048u, b_lbo, 128u);
#pragma unroll
                            for (int w = 0; w < 2; ++w) {
                                const uint64_t bd =
                                    umma_desc(w_addr + (uint32_t)(w * kPfABytes) + (uint32_t)j * 4096u, 2048u, 128u);
                                umma_f16(d + (uint32_t)(w * 128), ah, bd, idesc, acc);
                                umma_f16(d + (uint32_t)(w * 128), al, bd, idesc, 1u);
                            }
                        }
                    } else {
                        const uint32_t b_addr = s_addr + (uint32_t)kPfABytes;
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const uint64_t ad = umma_desc(s_addr + (uint32_t)j * 4096u, 2048u, 128u);
                            const uint64_t bd = umma_desc(b_addr + (uint32_t)j * b_kstep, b_lbo, 128u);
                            umma_f16(d, ad, bd, idesc, (kb > it.kb0 || j > 0) ? 1u : 0u);
                        }
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
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * 256);
            if (WIDE) {
                // lane = token t of the block, columns = weight rows r0 .. r0 + 255:
                // 32 rows per round as float4 stores (rows are a multiple of 64)
                const int t = it.nb * 128 + row, r0 = it.tile * 256;
                for (int c = 0; c < 256; c += 32) {
                    uint32_t a[16], b[16];
                    tmem_ld16x2(taddr + (uint32_t)c, taddr + (uint32_t)(c + 16), a, b);
                    float y[32];
#pragma unroll
                    for (int u = 0; u < 16; ++u) {
                        y[u] = __uint_as_float(a[u]);
                        y[16 + u] = __uint_as_float(b[u]);
                    }
                    const int r = r0 + c;
                    if (t < A.T && r < A.rows) {
                        if (A.act) {
                            // rows 2j (gate) and 2j + 1 (up) are adjacent columns:
                            // SiLU(gate) * up (math.rs:4-9, decoder.rs:147-150), for
                            // hidden units r / 2 .. r / 2 + 15
                            float v[16];
#pragma unroll
                            for (int u = 0; u < 16; ++u) {
                                const float gt = y[2 * u], up = y[2 * u + 1];
                                v[u] = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))), up);
                            }
                            if (A.xop_out) {  // straight into the next GEMM's operand
                                const int kbt_out = A.rows >> 7;  // (rows / 2) / 64 K blocks
#pragma unroll
                                for (int h8 = 0; h8 < 2; ++h8) {
                                    float w8[8];
#pragma unroll
                                    for (int u = 0; u < 8; ++u) w8[u] = v[h8 * 8 + u];
                                    pf_store8(A.xop_out, 128, kbt_out, t, (r >> 1) + h8 * 8, w8);
                                }
                            } else {
                                float* out = A.act + (size_t)t * (A.rows >> 1) + (r >> 1);
#pragma unroll
                                for (int k = 0; k < 16; k += 4)
                                    *reinterpret_cast<float4*>(out + k) = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
                            }
                        } else {
                            float* out = A.part + ((size_t)it.ks * A.T + t) * A.rows + r;
#pragma unroll
                            for (int k = 0; k < 32; k += 4)
                                *reinterpret_cast<float4*>(out + k) = make_float4(y[k], y[k + 1], y[k + 2], y[k + 3]);
                        }
                    }
                }
                tmem_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[ab]);
                continue;
            }
            const int r = it.tile * 128 + row;
            const bool live = r < A.rows;
            const int t0 = it.nb * A.tn;
            if (A.act) {
                // rows 2j (gate) and 2j + 1 (up) sit in adjacent lanes: SiLU(gate) * up
                // (math.rs:4-9, decoder.rs:147-150) straight to act[t, j]
                float* out = A.act + (r >> 1);
                const int hidden = A.rows >> 1;
                for (int c = 0; c < A.tn; c += 16) {
                    uint32_t hi[16], lo[16];
                    tmem_ld16x2(taddr + (uint32_t)c, taddr + (uint32_t)(A.tn + c), hi, lo);
#pragma unroll
                    for (int u = 0; u < 16; ++u) {
                        const int t = t0 + c + u;
                        const float y = __uint_as_float(hi[u]) + __uint_as_float(lo[u]);
                        const float up = __shfl_xor_sync(kFull, y, 1);
                        if (live && !(lane & 1) && t < A.T)
                            out[(size_t)t * hidden] = __fmul_rn(__fdiv_rn(y, __fadd_rn(1.0f, expf(-y))), up);
                    }
                }
            } else {
                float* out = A.part + (size_t)it.ks * A.T * A.rows + r;
                for (int c = 0; c < A.tn; c += 16) {
                    uint32_t hi[16], lo[16];
                    tmem_ld16x2(taddr + (uint32_t)c, taddr + (uint32_t)(A.tn + c), hi, lo);
#pragma unroll
                    for (int u = 0; u < 16; ++u) {
                        const int t = t0 + c + u;
                        if (live && t < A.T)
                            out[(size_t)t * A.rows] = __uint_as_float(hi[u]) + __uint_as_float(lo[u]);
                    }
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

// Operand tiles: 32 tokens x 64 elements staged in shared memory, read from
// row-major f32 rows (consecutive threads on consecutive elements of a row)
// and written to the prefill operand with eight consecutive threads on eight
// consecutive tokens of one 8-element chunk (one 128-byte core-matrix row
// group for hi, one for lo).  Grid (K / 64, ceil(Tp / 32)), 256 threads.
constexpr int kPfTT = 32;

__device__ __forceinline__ void pf_tile_store(const float (*tile)[65], int t0, int Tp, int k0, int kbt,
                                              unsigned char* xop, int tn) {
    const int c = threadIdx.x >> 5, tok = threadIdx.x & 31, t = t0 + tok;
    if (t >= Tp) return;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = tile[tok][c * 8 + j];
    pf_store8(xop, tn, kbt, t, k0 + c * 8, v);
}

// h[t] becomes either the embedding row of the token (plus the adapter row at
// its position), or h[t] + (the GEMM's split sum) (decoder.rs:138-139,
// 151-152); per 512-element chunk of the row its sum of squares goes to
// ssp[t, chunk] (the next RMSNorm's, summed in chunk order).  Grid
// (ceil(dim / 512), T), 128 threads, four elements each.
__global__ void __launch_bounds__(128) pf_resid_kernel(const __grid_constant__ PfNormArgs A) {
    __shared__ float red[4];
    const int t = blockIdx.y, e = blockIdx.x * 512 + threadIdx.x * 4;
    float ss = 0.0f;
    if (e < A.dim) {
        float* h = A.h + (size_t)t * A.dim + e;
        float v[4];
        if (A.embed) {
            int tok = A.tokens[t];
            if (tok < 0 || tok >= A.vocab) {
                if (threadIdx.x == 0) raise_error(A.err, ERR_TOKEN_RANGE);
                tok = 0;
            }
            const uint2 w = *reinterpret_cast<const uint2*>(A.embed + (size_t)tok * A.dim + e);
            v[0] = bf16_lo(w.x); v[1] = bf16_hi(w.x); v[2] = bf16_lo(w.y); v[3] = bf16_hi(w.y);
            if (A.adapter) {
                const float4 a = *reinterpret_cast<const float4*>(
                    A.adapter + (size_t)((A.pos0 + t) % A.adapter_cap) * A.dim + e);
                v[0] = __fadd_rn(a.x, v[0]); v[1] = __fadd_rn(a.y, v[1]);
                v[2] = __fadd_rn(a.z, v[2]); v[3] = __fadd_rn(a.w, v[3]);
            }
        } else {
            const float4 x = *reinterpret_cast<const float4*>(h);
            float4 p = *reinterpret_cast<const float4*>(A.part + (size_t)t * A.dim + e);
            for (int s = 1; s < A.splits; ++s) {
                const float4 q = *reinterpret_cast<const float4*>(A.part + ((size_t)s * A.T + t) * A.dim + e);
                p.x += q.x; p.y += q.y; p.z += q.z; p.w += q.w;
            }
            v[0] = __fadd_rn(x.x, p.x); v[1] = __fadd_rn(x.y, p.y);
            v[2] = __fadd_rn(x.z, p.z); v[3] = __fadd_rn(x.w, p.w);
        }
        *reinterpret_cast<float4*>(h) = make_float4(v[0], v[1], v[2], v[3]);
#pragma unroll
        for (int j = 0; j < 4; ++j) ss += __fmul_rn(v[j], v[j]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0)
        A.ssp[(size_t)t * A.ssp_chunks + blockIdx.x] = ((red[0] + red[1]) + red[2]) + red[3];
}

// RMSNorm (math.rs:17-25: inv = 1 / sqrt(sum / dim + eps), then x * inv * w)
// of the rows pf_resid_kernel wrote, into the prefill operand of the next
// linear; zero rows for padding tokens.
__global__ void __launch_bounds__(256) pf_norm_xop_kernel(const __grid_constant__ PfNormArgs A) {
    __shared__ float tile[kPfTT][65];
    __shared__ float inv_s[kPfTT];
    const int tid = threadIdx.x, k0 = blockIdx.x * 64, t0 = blockIdx.y * kPfTT;
    if (tid < kPfTT) {
        const int t = t0 + tid;
        float inv = 0.0f;
        if (t < A.T) {
            float ss = 0.0f;
            for (int c = 0; c < A.ssp_chunks; ++c) ss += A.ssp[(size_t)t * A.ssp_chunks + c];
            inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)A.dim), A.eps)));
        }
        inv_s[tid] = inv;
    }
    __syncthreads();
    const int k = tid & 63;
    const float g = A.gain[k0 + k];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const int tok = r * 4 + (tid >> 6), t = t0 + tok;
        float v = 0.0f;
        if (t < A.T) v = __fmul_rn(__fmul_rn(A.h[(size_t)t * A.dim + k0 + k], inv_s[tok]), g);
        tile[tok][k] = v;
    }
    __syncthreads();
    pf_tile_store(tile, t0, A.Tp, k0, A.dim / 64, A.xop, A.tn);
}

// q|k|v split sums -> RoPE (math.rs:30-65) on q and k at position pos0 + t ->
// q [T, q_dim], the pass's keys and values [T, kv_dim].  One thread per
// (token, 4 consecutive elements) = two RoPE pairs of one head (q_dim and
// kv_dim are multiples of 64, head_dim of 4); the splits' float4 loads are all
// issued before the sum, which adds them in split order as pf_sum does.
__global__ void __launch_bounds__(256) pf_qkv_kernel(const __grid_constant__ PfQkvArgs A) {
    const int rows = A.q_dim + 2 * A.kv_dim, quads = rows / 4;
    const long long total = (long long)A.T * quads;
    const int half = A.head_dim / 2;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(e / quads), r = 4 * (int)(e - (long long)t * quads);
        float4 p[4];
#pragma unroll
        for (int sp = 0; sp < 4; ++sp)
            if (sp < A.splits) p[sp] = *reinterpret_cast<const float4*>(A.part + ((size_t)sp * A.T + t) * rows + r);
        float4 y = p[0];
#pragma unroll
        for (int sp = 1; sp < 4; ++sp)
            if (sp < A.splits) {
                y.x += p[sp].x; y.y += p[sp].y; y.z += p[sp].z; y.w += p[sp].w;
            }
        for (int sp = 4; sp < A.splits; ++sp) {
            const float4 q = *reinterpret_cast<const float4*>(A.part + ((size_t)sp * A.T + t) * rows + r);
            y.x += q.x; y.y += q.y; y.z += q.z; y.w += q.w;
        }
        if (r < A.q_dim + A.kv_dim) {
            const int rr = r < A.q_dim ? r : r - A.q_dim;
            const int d = rr % A.head_dim;
            long long pos = A.pos0 + t;
            if (pos >= A.max_pos) {
                if (r == 0) raise_error(A.err, ERR_POS_RANGE);
                pos = 0;
            }
            const float2 c = *reinterpret_cast<const float2*>(A.rope_cos + pos * half + d / 2);
            const float2 sn = *reinterpret_cast<const float2*>(A.rope_sin + pos * half + d / 2);
            const float o0 = __fsub_rn(__fmul_rn(y.x, c.x), __fmul_rn(y.y, sn.x));
            const float o1 = __fadd_rn(__fmul_rn(y.x, sn.x), __fmul_rn(y.y, c.x));
            const float o2 = __fsub_rn(__fmul_rn(y.z, c.y), __fmul_rn(y.w, sn.y));
            const float o3 = __fadd_rn(__fmul_rn(y.z, sn.y), __fmul_rn(y.w, c.y));
            float* dst = r < A.q_dim ? A.q + (size_t)t * A.q_dim + rr : A.kc + (size_t)t * A.kv_dim + rr;
            *reinterpret_cast<float4*>(dst) = make_float4(o0, o1, o2, o3);
        } else {
            const int rr = r - A.q_dim - A.kv_dim;
            *reinterpret_cast<float4*>(A.vc + (size_t)t * A.kv_dim + rr) = y;
        }
    }
}

// Causal attention of a pass (ops.rs:66-132 per token), split over the keys.
// Logical key j of the sequence "cache before the pass, then the pass's
// tokens": j < len0 is ring slot (start0 + j) % cap, j >= len0 is pass token
// j - len0.  Token t sees keys [len0 + t + 1 - n_t, len0 + t] with n_t =
// min(len0 + t + 1, win).  A block of 16 tokens covers the union of its
// tokens' ranges, cut into chunks of `kc` keys; CTA (block * cmax + chunk, kv
// head) runs one chunk (CTAs past their block's last chunk exit at once)
// with 8 warps: warp w takes q head w % 4 of the group for tokens
// 8 * (w / 4) .. + 7.  32-key tiles of K and V move into shared memory with
// cp.async, double-buffered; online softmax; the chunk's (o, m, l) per token
// and head go to `part` and pf_attn_merge_kernel combines the chunks in order.
// C = head_dim / 32.
constexpr int kPfQB = 16, kPfKT = 32, kPfAttnThreads = 256;

__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__host__ __device__ constexpr int pf_attn_smem_floats(int hd) {
    return 2 * 2 * kPfKT * (hd + 4) + 4 * kPfQB * hd + 8 * 8 * kPfKT;
}

// First and last logical key of token t of the pass.
__device__ __forceinline__ int pf_first_key(const PfAttnArgs& A, int t) {
    const int hi = A.len0 + t;
    return hi + 1 - min(hi + 1, A.win);
}

// Partial record of (block, chunk, kv head, head in group, token in block):
// o[head_dim] (unnormalised), m, l.
__device__ __forceinline__ float* pf_attn_rec(const PfAttnArgs& A, int qb, int c, int hk, int g, int q) {
    const size_t idx = ((((size_t)qb * A.cmax + c) * A.n_kv + hk) * 4 + g) * A.qb + q;
    return A.part + idx * (size_t)(A.head_dim + 2);
}

template <int C>
__global__ void __launch_bounds__(kPfAttnThreads) pf_attn_kernel(const __grid_constant__ PfAttnArgs A) {
    extern __shared__ __align__(16) float sm[];
    constexpr int HD = 32 * C, KS = HD + 4;  // padded key rows: conflict-free float4 reads
    float* Kst = sm;                         // [2][32][KS]
    float* Vst = Kst + 2 * kPfKT * KS;       // [2][32][KS]
    float* Qs = Vst + 2 * kPfKT * KS;        // [4][16][HD]
    float* Ps = Qs + 4 * kPfQB * HD;         // [8][8][32]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hk = blockIdx.y, G = A.n_heads / A.n_kv;
    const int qblk = blockIdx.x / A.cmax, chunk = blockIdx.x % A.cmax;
    const int g = warp & 3, qb = (warp >> 2) * 8;  // q head in the group, first token of the warp
    const int t0 = qblk * kPfQB, nq = min(kPfQB, A.T - t0);
    const int qd = A.n_heads * HD, kvd = A.n_kv * HD;
    const int b_lo = pf_first_key(A, t0), b_hi = A.len0 + t0 + nq - 1;
    const int j_lo = b_lo + chunk * A.kc;
    if (j_lo > b_hi) return;  // this block has fewer chunks (uniform across the CTA)
    const int j_hi = min(b_hi, j_lo + A.kc - 1);
    const bool active = g < G && qb < nq;

    for (int e = tid; e < 4 * kPfQB * HD; e += kPfAttnThreads) {
        const int w = e / (kPfQB * HD), qi = (e / HD) % kPfQB, d = e % HD;
        Qs[e] = (w < G && qi < nq) ? A.q[(size_t)(t0 + qi) * qd + (size_t)(hk * G + w) * HD + d] : 0.0f;
    }
    const int n_tiles = (j_hi - j_lo) / kPfKT + 1;
    const float* kr = A.k_ring + (size_t)hk * A.cap * HD;
    const float* vr = A.v_ring + (size_t)hk * A.cap * HD;

    auto issue = [&](int tile) {
        const int j0 = j_lo + tile * kPfKT;
        float* ks = Kst + (tile & 1) * kPfKT * KS;
        float* vs = Vst + (tile & 1) * kPfKT * KS;
        for (int e = tid; e < kPfKT * (HD / 4); e += kPfAttnThreads) {
            const int kk = e / (HD / 4), d4 = (e - kk * (HD / 4)) * 4;
            const int j = j0 + kk;
            const float *ksrc = A.kc_in, *vsrc = A.vc_in;  // any valid address when j is past the range
            if (j <= j_hi) {
                if (j < A.len0) {
                    const size_t slot = (size_t)((A.start0 + j) % A.cap);
                    ksrc = kr + slot * HD + d4;
                    vsrc = vr + slot * HD + d4;
                } else {
                    ksrc = A.kc_in + (size_t)(j - A.len0) * kvd + (size_t)hk * HD + d4;
                    vsrc = A.vc_in + (size_t)(j - A.len0) * kvd + (size_t)hk * HD + d4;
                }
            }
            cp_async16(ks + kk * KS + d4, ksrc, j <= j_hi);
            cp_async16(vs + kk * KS + d4, vsrc, j <= j_hi);
        }
        cp_async_commit();
    };

    float o[8][C], m[8], l[8];
#pragma unroll
    for (int qi = 0; qi < 8; ++qi) {
        m[qi] = -INFINITY;
        l[qi] = 0.0f;
#pragma unroll
        for (int c = 0; c < C; ++c) o[qi][c] = 0.0f;
    }
    float* P = Ps + warp * 8 * kPfKT;
    const float* q = Qs + (g * kPfQB + qb) * HD;

    issue(0);
    for (int tile = 0; tile < n_tiles; ++tile) {
        if (tile + 1 < n_tiles) {
            issue(tile + 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();  // this tile (and the queries) visible to every warp
        if (active) {
            const float* krow = Kst + (tile & 1) * kPfKT * KS + lane * KS;
            const float* vs = Vst + (tile & 1) * kPfKT * KS;
            float s[8];
#pragma unroll
            for (int qi = 0; qi < 8; ++qi) s[qi] = 0.0f;
#pragma unroll 4
            for (int d = 0; d < HD; d += 4) {
                const float4 k4 = *reinterpret_cast<const float4*>(krow + d);
#pragma unroll
                for (int qi = 0; qi < 8; ++qi) {
                    const float4 q4 = *reinterpret_cast<const float4*>(q + qi * HD + d);
                    s[qi] = fmaf(q4.x, k4.x, s[qi]);
                    s[qi] = fmaf(q4.y, k4.y, s[qi]);
                    s[qi] = fmaf(q4.z, k4.z, s[qi]);
                    s[qi] = fmaf(q4.w, k4.w, s[qi]);
                }
            }
            const int j = j_lo + tile * kPfKT + lane;
#pragma unroll
            for (int qi = 0; qi < 8; ++qi) {
                const int t = t0 + qb + qi;
                const bool ok = qb + qi < nq && j <= j_hi && j >= pf_first_key(A, t) && j <= A.len0 + t;
                const float sc = ok ? s[qi] * A.scale : -INFINITY;
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
                P[qi * kPfKT + lane] = p;
            }
            __syncwarp();
#pragma unroll 2
            for (int kk = 0; kk < kPfKT; kk += 4) {
                float v[4][C];
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int c = 0; c < C; ++c) v[u][c] = vs[(kk + u) * KS + lane + 32 * c];
#pragma unroll
                for (int qi = 0; qi < 8; ++qi) {
                    const float4 p4 = *reinterpret_cast<const float4*>(P + qi * kPfKT + kk);
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
        __syncthreads();  // every warp done with this stage before the next issue rewrites it
    }
    if (!active) return;
#pragma unroll
    for (int qi = 0; qi < 8; ++qi) {
        if (qb + qi >= nq) break;
        float* rec = pf_attn_rec(A, qblk, chunk, hk, g, qb + qi);
#pragma unroll
        for (int c = 0; c < C; ++c) rec[lane + 32 * c] = o[qi][c];
        if (lane == 0) {
            rec[HD] = m[qi];
            rec[HD + 1] = l[qi];
        }
    }
}

// out[t, head] = (sum_c o_c e^(m_c - M)) / (sum_c l_c e^(m_c - M)) over the
// chunks of the token's block in chunk order (M = max m_c).  Grid (T, n_kv),
// one warp per head of the group, C = head_dim / 32 elements per lane.
template <int C>
__global__ void __launch_bounds__(128) pf_attn_merge_kernel(const __grid_constant__ PfAttnArgs A) {
    constexpr int HD = 32 * C;
    const int t = blockIdx.x, hk = blockIdx.y, g = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = A.n_heads / A.n_kv;
    if (g >= G) return;
    const int qblk = t / A.qb, q = t % A.qb, t0 = qblk * A.qb, nq = min(A.qb, A.T - t0);
    const int b_lo = pf_first_key(A, t0), b_hi = A.len0 + t0 + nq - 1;
    const int nch = (b_hi - b_lo) / A.kc + 1;
    float M = -INFINITY;
    for (int c = 0; c < nch; ++c) M = fmaxf(M, pf_attn_rec(A, qblk, c, hk, g, q)[HD]);
    float L = 0.0f, acc[C];
#pragma unroll
    for (int i = 0; i < C; ++i) acc[i] = 0.0f;
    for (int c = 0; c < nch; ++c) {
        const float* rec = pf_attn_rec(A, qblk, c, hk, g, q);
        const float mc = rec[HD];
        if (mc == -INFINITY) continue;  // no key of this chunk is visible to the token
        const float w = expf(mc - M);
        L += rec[HD + 1] * w;
#pragma unroll
        for (int i = 0; i < C; ++i) acc[i] = fmaf(rec[lane + 32 * i], w, acc[i]);
    }
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
    float* out = A.out + (size_t)t * A.n_heads * HD + (size_t)(hk * G + g) * HD;
#pragma unroll
    for (int i = 0; i < C; ++i) out[lane + 32 * i] = acc[i] * inv;
}

// ---- tensor-core attention of a pass (4 q heads per kv head, head_dim 128) ----
// The same chunks and records as pf_attn_kernel, for blocks of 32 tokens: the
// 32 tokens x 4 q heads of a CTA are the M = 128 rows of two tcgen05 products
// per 64-key tile, S = Q K^T (K = head_dim) and O_tile = P V (K = 64 keys).
// Both operands of each product are f32 values split into bf16 hi and lo
// parts; hi*hi + hi*lo + lo*hi accumulate in f32 in TMEM (about 16 mantissa
// bits per operand; the lo*lo term is below f32 rounding).  Row r = g * 32 +
// tt (q head g of the group, token tt of the block) is TMEM lane r; warps w
// and w + 4 read lane quarter w % 4, warp w < 4 the first half of the row's
// columns and warp w + 4 the second.  Per tile they run the online softmax
// of the reference's attention (ops.rs:66-132, math.rs:67-88, restated
// incrementally: the row maximum is exchanged through shared memory, each
// half keeps its own running sum l under the common correction), write P's
// hi and lo parts for the second product, and add their half of O_tile into
// registers with the correction.  With one chunk per block (cmax == 1) the
// CTA writes the normalised rows itself and no merge runs: as f32 rows, or
// (xop given) straight into the o-proj's prefill operand.
//
// The key / value operands are converted once per layer and pass by
// pf_kv_tiles_kernel into 64 KB tiles on a 64-key grid (kv_base + 64 i), so
// the attention CTAs, which read overlapping key ranges, only bulk-copy them:
// one 64 KB copy per tile into a two-stage ring, the next tile landing while
// this one's products and softmax run.  A CTA's tiles may start before its
// chunk (the grid is global), so keys outside [j_lo, j_hi] are masked like
// keys outside the token's window.  P reuses the stage's K space (the S
// product has finished reading K when the softmax writes P).  Operands in the
// UMMA canonical K-major layout without swizzle (vox_tcgen05.cuh); the bf16
// hi / lo split is one cvt.rn.bf16x2 per pair (split_bf16x2).  Measured per
// 512-token pass: CTAs that each converted their K/V tiles from f32 (staged
// with cp.async) 49 us; with per-thread global loads 91 us.
constexpr int kTcQB = 32, kTcKT = 64, kTcThreads = 256, kTcHD = 128;
constexpr int kTcQBytes = 128 * kTcHD * 2;    // one of Q hi / Q lo (32 KB)
constexpr int kTcKBytes = kTcKT * kTcHD * 2;  // one of K hi / K lo, later P hi / P lo (16 KB)
constexpr int kTcVBytes = kTcHD * kTcKT * 2;  // one of V^T hi / lo (16 KB)
constexpr int kTcTileBytes = 2 * kTcKBytes + 2 * kTcVBytes;  // 64 KB: K hi | K lo | V^T hi | V^T lo
constexpr int kTcSmem = 2 * kTcQBytes + 2 * kTcTileBytes + 2 * 128 * 4 + 64;
static_assert(kTcKBytes == 128 * kTcKT * 2, "P (128 rows x 64 keys) fits the K operand's space");

// Byte offset of element (row, k) of an operand with `rows` rows (a multiple
// of 8) in canonical K-major layout: K step k / 16 at rows * 32 bytes each,
// core matrix ((k / 8) % 2, row / 8), 16 bytes per row, 2 per element.
__device__ __forceinline__ uint32_t kmaj_off(int row, int k, int rows) {
    return (uint32_t)((k >> 4) * rows * 32 + ((k >> 3) & 1) * rows * 16 + (row >> 3) * 128 + (row & 7) * 16 +
                      (k & 7) * 2);
}

// Eight consecutive elements (k % 8 == 0) of one row as bf16 hi and lo.
__device__ __forceinline__ void tc_put8(unsigned char* hi_base, unsigned char* lo_base, uint32_t off,
                                        const float (&v)[8]) {
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 8; j += 2) split_bf16x2(v[j], v[j + 1], hi[j >> 1], lo[j >> 1]);
    *reinterpret_cast<uint4*>(hi_base + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(lo_base + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

__device__ __forceinline__ void ld8(const float* src, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(src);
    const float4 b = *reinterpret_cast<const float4*>(src + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Row of logical key j (cache before the pass, then the pass) of kv head hk.
__device__ __forceinline__ const float* pf_key_row(const PfAttnArgs& A, int hk, int j, const float* ring,
                                                   const float* pass) {
    if (j < A.len0) {
        int slot = A.start0 + j;  // start0 < cap and j < len0 <= cap
        if (slot >= A.cap) slot -= A.cap;
        return ring + ((size_t)hk * A.cap + slot) * kTcHD;
    }
    return pass + (size_t)(j - A.len0) * A.n_kv * kTcHD + (size_t)hk * kTcHD;
}

// Keys and values the pass's attention reads, converted once as the
// tensor-core kernel's B operands: for kv head hk and tile i (keys kv_base +
// 64 i ..), K hi | K lo (64 keys x 128 dims) then V^T hi | V^T lo (128 dims x
// 64 keys); keys past the pass's last are zero.  Grid (kv_tiles, n_kv, 4):
// z = 0, 1 the K rows of keys 32 z .., z = 2, 3 the V^T rows of dims 64 (z - 2) ..
// (64 CTAs per tile-and-head grid took 10.2 us at a 512-token pass).
__global__ void __launch_bounds__(256) pf_kv_tiles_kernel(const __grid_constant__ PfAttnArgs A) {
    const int i = blockIdx.x, hk = blockIdx.y, z = blockIdx.z, tid = threadIdx.x;
    const int j0 = A.kv_base + i * kTcKT, j_last = A.len0 + A.T - 1;
    unsigned char* base = A.kvop + ((size_t)hk * A.kv_tiles + i) * kTcTileBytes;
    // K: key kk, dims d0 .. d0 + 7 (consecutive threads take consecutive keys)
    if (z < 2)
    for (int e = tid; e < (kTcKT / 2) * (kTcHD / 8); e += 256) {
        const int kk = z * 32 + (e & 31), d0 = (e >> 5) * 8, j = j0 + kk;
        float v[8];
        if (j <= j_last) {
            ld8(pf_key_row(A, hk, j, A.k_ring, A.kc_in) + d0, v);
        } else {
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = 0.0f;
        }
        tc_put8(base, base + kTcKBytes, kmaj_off(kk, d0, kTcKT), v);
    }
    // V^T: dim d, keys k0 .. k0 + 7 (consecutive threads take consecutive dims)
    unsigned char* vb = base + 2 * kTcKBytes;
    if (z >= 2)
    for (int e = tid; e < (kTcHD / 2) * (kTcKT / 8); e += 256) {
        const int d = (z - 2) * 64 + (e & 63), k0 = (e >> 6) * 8;
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = j0 + k0 + u;
            v[u] = j <= j_last ? pf_key_row(A, hk, j, A.v_ring, A.vc_in)[d] : 0.0f;
        }
        tc_put8(vb, vb + kTcVBytes, kmaj_off(d, k0, kTcHD), v);
    }
}

__global__ void __launch_bounds__(kTcThreads, 1) pf_attn_tc_kernel(const __grid_constant__ PfAttnArgs A) {
    extern __shared__ __align__(1024) unsigned char tsm[];
    unsigned char* Qh = tsm;
    unsigned char* Ql = Qh + kTcQBytes;
    unsigned char* ring = Ql + kTcQBytes;  // 2 stages of kTcTileBytes
    float* red = reinterpret_cast<float*>(ring + 2 * kTcTileBytes);  // [2][128] half-row maxima, then sums
    uint64_t* bar_s = reinterpret_cast<uint64_t*>(red + 2 * 128);
    uint64_t* bar_o = bar_s + 1;
    uint64_t* bar_f = bar_o + 1;  // [2] a stage's tile landed
    uint32_t* tmem_s = reinterpret_cast<uint32_t*>(bar_f + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hk = blockIdx.y;
    const int qblk = blockIdx.x / A.cmax, chunk = blockIdx.x % A.cmax;
    const int t0 = qblk * kTcQB, nq = min(kTcQB, A.T - t0);
    const int qd = A.n_heads * kTcHD;
    const int b_lo = pf_first_key(A, t0), b_hi = A.len0 + t0 + nq - 1;
    const int j_lo = b_lo + chunk * A.kc;
    if (j_lo > b_hi) return;  // this block has fewer chunks (uniform across the CTA)
    const int j_hi = min(b_hi, j_lo + A.kc - 1);
    const int i_first = (j_lo - A.kv_base) / kTcKT, n_tiles = (j_hi - A.kv_base) / kTcKT - i_first + 1;
    const unsigned char* tiles = A.kvop + ((size_t)hk * A.kv_tiles + i_first) * kTcTileBytes;

    if (tid == 0) {
        mbar_init(bar_s, 1);
        mbar_init(bar_o, 1);
        mbar_init(&bar_f[0], 1);
        mbar_init(&bar_f[1], 1);
        fence_barrier_init();
    }
    __syncthreads();
    auto issue = [&](int k) {  // thread 0: tile k into stage k % 2
        const int st = k & 1;
        mbar_arrive_expect_tx(&bar_f[st], (uint32_t)kTcTileBytes);
        bulk_copy_g2s_nohint(ring + (size_t)st * kTcTileBytes, tiles + (size_t)k * kTcTileBytes,
                             (uint32_t)kTcTileBytes, &bar_f[st]);
    };
    if (tid == 0)
        for (int k = 0; k < min(2, n_tiles); ++k) issue(k);
    if (warp == 0) {
        __syncwarp();  // the allocation is warp-collective
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_s)),
                     "r"(256)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // Q rows (token t0 + tt, q head 4 hk + g) as hi / lo, four rows' loads in
    // flight per thread; consecutive threads take consecutive rows
    for (int e0 = tid; e0 < 128 * (kTcHD / 8); e0 += 4 * kTcThreads) {
        float v[4][8];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int e = e0 + u * kTcThreads, r = e & 127, d0 = (e >> 7) * 8, tt = r & 31, g = r >> 5;
            if (tt < nq) {
                ld8(A.q + (size_t)(t0 + tt) * qd + (size_t)(hk * 4 + g) * kTcHD + d0, v[u]);
            } else {
#pragma unroll
                for (int w = 0; w < 8; ++w) v[u][w] = 0.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int e = e0 + u * kTcThreads, r = e & 127, d0 = (e >> 7) * 8;
            tc_put8(Qh, Ql, kmaj_off(r, d0, 128), v[u]);
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tmem = *tmem_s;
    const uint32_t tS = tmem, tO = tmem + 128;  // S: columns 0..63, O_tile: 128..255

    const int q4 = warp & 3, half = warp >> 2;  // TMEM lane quarter, column half
    const int row = q4 * 32 + lane, tt = lane, g = q4;
    const int t = t0 + tt;
    const int kfirst = max(pf_first_key(A, t), j_lo), klast = min(A.len0 + t, j_hi);
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    float acc[kTcHD / 2];
#pragma unroll
    for (int d = 0; d < kTcHD / 2; ++d) acc[d] = 0.0f;
    float m_run = -INFINITY, l_run = 0.0f;
    constexpr uint32_t idS = umma_idesc_bf16(128, kTcKT), idO = umma_idesc_bf16(128, kTcHD);
    uint32_t phase = 0;

    for (int k = 0; k < n_tiles; ++k) {
        const int j0 = A.kv_base + (i_first + k) * kTcKT;
        unsigned char* Kh = ring + (size_t)(k & 1) * kTcTileBytes;  // K hi, then P hi
        unsigned char* Kl = Kh + kTcKBytes;                           // K lo, then P lo
        unsigned char* Vh = Kl + kTcKBytes;
        unsigned char* Vl = Vh + kTcVBytes;
        if (tid == 0) {
            if (!mbar_wait(&bar_f[k & 1], (uint32_t)(k >> 1) & 1u)) raise_error(A.err, ERR_FULL_WAIT);
            tmem_fence_after();
            const uint32_t qh = smem_addr(Qh), ql = smem_addr(Ql), kh = smem_addr(Kh), kl = smem_addr(Kl);
#pragma unroll
            for (int s = 0; s < kTcHD / 16; ++s) {
                const uint64_t ah = umma_desc(qh + s * 4096u, 2048u, 128u);
                const uint64_t al = umma_desc(ql + s * 4096u, 2048u, 128u);
                const uint64_t bh = umma_desc(kh + s * 2048u, 1024u, 128u);
                const uint64_t bl = umma_desc(kl + s * 2048u, 1024u, 128u);
                umma_f16(tS, ah, bh, idS, s > 0 ? 1u : 0u);
                umma_f16(tS, ah, bl, idS, 1u);
                umma_f16(tS, al, bh, idS, 1u);
            }
            umma_commit(bar_s);
        }
        if (!mbar_wait(bar_s, phase) && lane == 0) raise_error(A.err, ERR_FULL_WAIT);
        tmem_fence_after();
        // this half's 32 scores of the row, masked and scaled
        uint32_t sr[32];
        {
            uint32_t a[16], b[16];
            tmem_ld16x2(tS + lane_base + half * 32, tS + lane_base + half * 32 + 16, a, b);
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                sr[u] = a[u];
                sr[16 + u] = b[u];
            }
        }
        float mt = -INFINITY;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
            const int j = j0 + half * 32 + c;
            const bool ok = tt < nq && j >= kfirst && j <= klast;
            const float sc = ok ? __uint_as_float(sr[c]) * A.scale : -INFINITY;
            sr[c] = __float_as_uint(sc);
            mt = fmaxf(mt, sc);
        }
        red[half * 128 + row] = mt;
        __syncthreads();  // maxima exchanged; every S product done, so K's space takes P
        const float mn = fmaxf(m_run, fmaxf(red[row], red[128 + row]));
        float ps = 0.0f;
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
            float pv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float sc = __uint_as_float(sr[c + u]);
                pv[u] = (mn == -INFINITY || sc == -INFINITY) ? 0.0f : expf(sc - mn);
                ps += pv[u];
            }
            tc_put8(Kh, Kl, kmaj_off(row, half * 32 + c, 128), pv);
        }
        const float corr = mn == -INFINITY ? 1.0f : (m_run == -INFINITY ? 0.0f : expf(m_run - mn));
        l_run = l_run * corr + ps;
        m_run = mn;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tmem_fence_before();
        __syncthreads();  // P written, the scores and the maxima read
        tmem_fence_after();
        if (tid == 0) {
            const uint32_t ph = smem_addr(Kh), pl = smem_addr(Kl), vh = smem_addr(Vh), vl = smem_addr(Vl);
#pragma unroll
            for (int s = 0; s < kTcKT / 16; ++s) {
                const uint64_t ah = umma_desc(ph + s * 4096u, 2048u, 128u);
                const uint64_t al = umma_desc(pl + s * 4096u, 2048u, 128u);
                const uint64_t bh = umma_desc(vh + s * 4096u, 2048u, 128u);
                const uint64_t bl = umma_desc(vl + s * 4096u, 2048u, 128u);
                umma_f16(tO, ah, bh, idO, s > 0 ? 1u : 0u);
                umma_f16(tO, ah, bl, idO, 1u);
                umma_f16(tO, al, bh, idO, 1u);
            }
            umma_commit(bar_o);
        }
        if (!mbar_wait(bar_o, phase) && lane == 0) raise_error(A.err, ERR_FULL_WAIT);
        tmem_fence_after();
#pragma unroll
        for (int c = 0; c < kTcHD / 2; c += 32) {
            uint32_t a[16], b[16];
            const uint32_t ta = tO + lane_base + half * 64 + c;
            tmem_ld16x2(ta, ta + 16, a, b);
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                acc[c + u] = fmaf(acc[c + u], corr, __uint_as_float(a[u]));
                acc[c + 16 + u] = fmaf(acc[c + 16 + u], corr, __uint_as_float(b[u]));
            }
        }
        phase ^= 1u;
        tmem_fence_before();
        __syncthreads();  // this stage's products are read and TMEM is free for the next tile
        tmem_fence_after();
        if (tid == 0 && k + 2 < n_tiles) issue(k + 2);
    }
    // the two halves' sums under the same corrections add to the row's l
    red[half * 128 + row] = l_run;
    __syncthreads();
    if (tt < nq && A.cmax == 1) {
        // one chunk per block: the normalised row itself, as the merge of a
        // single record computes it (weight e^0 = 1, then times 1 / l)
        const float L = red[row] + red[128 + row], inv = L > 0.0f ? 1.0f / L : 0.0f;
        if (A.xop) {  // straight into the o-proj's operand (64 dims = one K block)
            const int k0 = (hk * 4 + g) * kTcHD + half * 64;
#pragma unroll
            for (int d = 0; d < kTcHD / 2; d += 8) {
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = acc[d + u] * inv;
                pf_store8(A.xop, A.xop_tn, qd / 64, t, k0 + d, v);
            }
        } else {
            float* out = A.out + (size_t)t * A.n_heads * kTcHD + (size_t)(hk * 4 + g) * kTcHD + half * 64;
#pragma unroll
            for (int d = 0; d < kTcHD / 2; d += 4)
                *reinterpret_cast<float4*>(out + d) =
                    make_float4(acc[d] * inv, acc[d + 1] * inv, acc[d + 2] * inv, acc[d + 3] * inv);
        }
    } else if (tt < nq) {
        float* rec = pf_attn_rec(A, qblk, chunk, hk, g, tt);
        // records are head_dim + 2 floats: 8-byte, not 16-byte, aligned
#pragma unroll
        for (int d = 0; d < kTcHD / 2; d += 2)
            *reinterpret_cast<float2*>(rec + half * 64 + d) = make_float2(acc[d], acc[d + 1]);
        if (half == 0) {
            rec[kTcHD] = m_run;
            rec[kTcHD + 1] = red[row] + red[128 + row];
        }
    }
    tmem_fence_before();
    __syncthreads();
    if (warp == 0) {
        tmem_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");
    }
}

// f32 rows [T, K] -> prefill operand (zero rows for padding tokens), through
// a shared-memory tile (see pf_tile_store).
__global__ void __launch_bounds__(256) pf_split_kernel(const float* __restrict__ src, int T, int Tp, int K,
                                                       unsigned char* xop, int tn) {
    __shared__ float tile[kPfTT][65];
    const int tid = threadIdx.x, k0 = blockIdx.x * 64, t0 = blockIdx.y * kPfTT, k = tid & 63;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const int tok = r * 4 + (tid >> 6), t = t0 + tok;
        tile[tok][k] = t < T ? src[(size_t)t * K + k0 + k] : 0.0f;
    }
    __syncthreads();
    pf_tile_store(tile, t0, Tp, k0, K / 64, xop, tn);
}

// w1|w3 split sums (row 2j = gate j, row 2j + 1 = up j) -> SiLU(gate) * up
// (math.rs:4-9, decoder.rs:147-150) -> prefill operand of w2, through a
// shared-memory tile (see pf_tile_store).
__global__ void __launch_bounds__(256) pf_swiglu_kernel(const float* __restrict__ part, int splits, int T, int Tp,
                                                        int hidden, unsigned char* xop, int tn) {
    __shared__ float tile[kPfTT][65];
    const int tid = threadIdx.x, j0 = blockIdx.x * 64, t0 = blockIdx.y * kPfTT, jj = tid & 63;
    const int rows = 2 * hidden;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const int tok = r * 4 + (tid >> 6), t = t0 + tok;
        float v = 0.0f;
        if (t < T) {
            float2 y = *reinterpret_cast<const float2*>(part + (size_t)t * rows + 2 * (j0 + jj));
            for (int s = 1; s < splits; ++s) {
                const float2 q = *reinterpret_cast<const float2*>(part + ((size_t)s * T + t) * rows + 2 * (j0 + jj));
                y.x += q.x;
                y.y += q.y;
            }
            v = __fmul_rn(__fdiv_rn(y.x, __fadd_rn(1.0f, expf(-y.x))), y.y);
        }
        tile[tok][jj] = v;
    }
    __syncthreads();
    pf_tile_store(tile, t0, Tp, j0, hidden / 64, xop, tn);
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

size_t pf_gemm_smem_bytes(bool wide) {
    return wide ? (size_t)kPfWideStages * kPfWideStageBytes + (2 * kPfWideStages + 4) * 8 + 16
                : (size_t)kPfStages * kPfStageBytes + (2 * kPfStages + 4) * 8 + 16;
}

bool pf_gemm_wide_ok(int rows, int tn) { return tn == 128 && rows % 256 == 0; }

cudaError_t pf_prepare() {
    cudaError_t e = cudaFuncSetAttribute(pf_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)pf_gemm_smem_bytes(false));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(pf_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)pf_gemm_smem_bytes(true));
    const auto attn_smem = [](int hd) { return pf_attn_smem_floats(hd) * 4; };
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(pf_attn_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_smem(32));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(pf_attn_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_smem(64));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(pf_attn_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_smem(128));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(pf_attn_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_smem(256));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(pf_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
    return e;
}

cudaError_t launch_pf_gemm(const PfGemmArgs& a, int grid, bool wide, cudaStream_t s) {
    if (a.tn < 16 || a.tn > 128 || a.tn % 16 || a.splits < 1 || a.splits > a.kbt || grid < 1 ||
        (a.act && (a.splits != 1 || a.rows % 2)) || (wide && (!pf_gemm_wide_ok(a.rows, a.tn) || a.tiles % 2)) ||
        (a.xop_out && (!wide || !a.act || a.xop_out == a.xop)))
        return cudaErrorInvalidValue;
    if (wide)
        pf_gemm_kernel<true><<<grid, kPfThreads, pf_gemm_smem_bytes(true), s>>>(a);
    else
        pf_gemm_kernel<false><<<grid, kPfThreads, pf_gemm_smem_bytes(false), s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_pf_resid(const PfNormArgs& a, cudaStream_t s) {
    if (a.dim % 64 || !a.ssp || a.ssp_chunks != (a.dim + 511) / 512 || (a.embed && !a.tokens))
        return cudaErrorInvalidValue;
    pf_resid_kernel<<<dim3(a.ssp_chunks, a.T), 128, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_pf_norm_xop(const PfNormArgs& a, cudaStream_t s) {
    if (a.dim % 64 || a.tn % 16 || a.Tp % 16 || !a.xop || !a.ssp) return cudaErrorInvalidValue;
    pf_norm_xop_kernel<<<dim3(a.dim / 64, (a.Tp + kPfTT - 1) / kPfTT), 256, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_pf_qkv(const PfQkvArgs& a, cudaStream_t s) {
    if (a.head_dim % 4 || a.q_dim % 64 || a.kv_dim % 64 || a.splits < 1) return cudaErrorInvalidValue;
    const long long work = (long long)a.T * ((a.q_dim + 2 * a.kv_dim) / 4);
    pf_qkv_kernel<<<grid_for(work, 256), 256, 0, s>>>(a);
    return cudaGetLastError();
}

int pf_attn_cmax(int T, int len0, int win, int kc, int qb) {
    int worst = 0;
    for (int t0 = 0; t0 < T; t0 += qb) {
        const int nq = T - t0 < qb ? T - t0 : qb;
        const int hi0 = len0 + t0, lo = hi0 + 1 - (hi0 + 1 < win ? hi0 + 1 : win);
        const int n = (len0 + t0 + nq - 1 - lo) / kc + 1;
        worst = n > worst ? n : worst;
    }
    return worst;
}

size_t pf_attn_part_floats(int T, int n_kv, int head_dim, int cmax, int qb) {
    return (size_t)((T + qb - 1) / qb) * cmax * n_kv * 4 * qb * (head_dim + 2);
}

cudaError_t launch_pf_attn(const PfAttnArgs& a, cudaStream_t s) {
    const int G = a.n_kv > 0 ? a.n_heads / a.n_kv : 0;
    if (G < 1 || G > 4 || a.n_heads % a.n_kv || a.win < 1 || a.kc < kPfKT || a.kc % kPfKT || a.cmax < 1 ||
        !a.part || a.qb != kPfQB)
        return cudaErrorInvalidValue;
    const int C = a.head_dim / 32;
    if (a.head_dim % 32 || (C != 1 && C != 2 && C != 4 && C != 8)) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)(((a.T + kPfQB - 1) / kPfQB) * a.cmax), a.n_kv);
    const size_t smem = (size_t)pf_attn_smem_floats(a.head_dim) * 4;
    switch (C) {
        case 1: pf_attn_kernel<1><<<grid, kPfAttnThreads, smem, s>>>(a); break;
        case 2: pf_attn_kernel<2><<<grid, kPfAttnThreads, smem, s>>>(a); break;
        case 4: pf_attn_kernel<4><<<grid, kPfAttnThreads, smem, s>>>(a); break;
        default: pf_attn_kernel<8><<<grid, kPfAttnThreads, smem, s>>>(a); break;
    }
    return cudaGetLastError();
}

bool pf_attn_tc_supported(int n_heads, int n_kv, int head_dim) {
    return n_kv > 0 && n_heads == 4 * n_kv && head_dim == kTcHD;
}

cudaError_t launch_pf_attn_tc(const PfAttnArgs& a, cudaStream_t s) {
    if (!pf_attn_tc_supported(a.n_heads, a.n_kv, a.head_dim) || a.win < 1 || a.kc < kTcKT || a.kc % kTcKT ||
        a.cmax < 1 || !a.part || a.qb != kTcQB || !a.kvop || a.kv_base % kTcKT ||
        a.kv_base > a.len0 + 1 - (a.len0 + 1 < a.win ? a.len0 + 1 : a.win) ||
        a.kv_base + a.kv_tiles * kTcKT < a.len0 + a.T ||
        (a.xop && (a.cmax != 1 || a.xop_tn < 16 || a.xop_tn > 128 || a.xop_tn % 16)))
        return cudaErrorInvalidValue;
    const dim3 grid((unsigned)(((a.T + kTcQB - 1) / kTcQB) * a.cmax), a.n_kv);
    pf_attn_tc_kernel<<<grid, kTcThreads, kTcSmem, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_pf_kv_tiles(const PfAttnArgs& a, cudaStream_t s) {
    if (!pf_attn_tc_supported(a.n_heads, a.n_kv, a.head_dim) || !a.kvop || a.kv_tiles < 1 || a.kv_base < 0 ||
        a.kv_base % kTcKT || a.kv_base + a.kv_tiles * kTcKT < a.len0 + a.T)
        return cudaErrorInvalidValue;
    pf_kv_tiles_kernel<<<dim3(a.kv_tiles, a.n_kv, 4), 256, 0, s>>>(a);
    return cudaGetLastError();
}

size_t pf_kv_tile_bytes() { return (size_t)kTcTileBytes; }

cudaError_t launch_pf_attn_merge(const PfAttnArgs& a, cudaStream_t s) {
    if (a.qb < 1) return cudaErrorInvalidValue;
    const dim3 grid(a.T, a.n_kv);
    switch (a.head_dim / 32) {
        case 1: pf_attn_merge_kernel<1><<<grid, 128, 0, s>>>(a); break;
        case 2: pf_attn_merge_kernel<2><<<grid, 128, 0, s>>>(a); break;
        case 4: pf_attn_merge_kernel<4><<<grid, 128, 0, s>>>(a); break;
        case 8: pf_attn_merge_kernel<8><<<grid, 128, 0, s>>>(a); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_pf_split(const float* src, int T, int Tp, int K, unsigned char* xop, int tn, cudaStream_t s) {
    if (K % 64 || tn % 16 || Tp % 16) return cudaErrorInvalidValue;
    pf_split_kernel<<<dim3(K / 64, (Tp + kPfTT - 1) / kPfTT), 256, 0, s>>>(src, T, Tp, K, xop, tn);
    return cudaGetLastError();
}

cudaError_t launch_pf_swiglu(const float* part, int splits, int T, int Tp, int hidden, unsigned char* xop, int tn,
                             cudaStream_t s) {
    if (hidden % 64 || tn % 16 || Tp % 16) return cudaErrorInvalidValue;
    pf_swiglu_kernel<<<dim3(hidden / 64, (Tp + kPfTT - 1) / kPfTT), 256, 0, s>>>(part, splits, T, Tp, hidden,
                                                                                 xop, tn);
    return cudaGetLastError();
}

cudaError_t launch_pf_commit(const PfCommitArgs& a, cudaStream_t s) {
    if (a.kv_dim % 4 || a.head_dim % 4 || a.cap < 1) return cudaErrorInvalidValue;
    const int first = a.T > a.cap ? a.T - a.cap : 0;
    pf_commit_kernel<<<grid_for((long long)(a.T - first) * (a.kv_dim / 4), 256), 256, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace vox
