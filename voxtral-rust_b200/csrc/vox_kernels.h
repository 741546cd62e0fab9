// vox_kernels.h -- internal interface between the host library (vox_capi.cpp)
// and the sm_100a kernels (*.cu).  Plain structs of device pointers and
// sizes; no torch types anywhere.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace vox {

// Ring bookkeeping of one cache layer, mirrored on the device.
//   len        = len_tokens (kv.rs:6)
//   start      = physical ring slot of logical token 0
//   pos_offset = pos_offset (kv.rs:7)
struct KvState {
    int32_t len;
    int32_t start;
    int64_t pos_offset;
};

// Per-step inputs of the token loop, resident on the device so that one
// captured CUDA graph serves every step.
struct StepState {
    int64_t pos;       // absolute position of the token being decoded
    int32_t tok;       // input token id
    int32_t next_tok;  // argmax written by the last kernel of the step
    int32_t greedy;    // 1: next_tok becomes tok for the following step
    int32_t advance;   // 1: pos += 1 at the end of the step
    int32_t pad[2];
};

struct ArgmaxPart {
    float v;
    int32_t i;
};

// Error bits written to the context's device error word.
enum : unsigned {
    ERR_FULL_WAIT = 1u,      // consumer waited too long for a weight stage
    ERR_EMPTY_WAIT = 2u,     // producer waited too long for a free stage
    ERR_DRAIN_WAIT = 4u,     // producer could not drain its copies
    ERR_POS_RANGE = 8u,      // position beyond the RoPE table
    ERR_TOKEN_RANGE = 16u,   // token id outside the vocabulary
    ERR_GRID_WAIT = 64u,     // a grid-wide wait (token kernel, GEMM chain) expired
    ERR_PEER_WAIT = 128u,    // a wait for another GPU's data expired (tensor-parallel exchange)
};

// Tensor-parallel exchange area of one rank (device memory, shared with the
// other ranks through CUDA IPC): [points][size][dim] f32 receive slots (slot
// (k, r) holds rank r's partial sums for exchange point k), then [points]
// arrival counters, then [size] argmax keys and the key arrival counter.
// Counters only grow: point k has received step s's data once it reaches
// (s + 1) * arrivals-per-step.
struct XchArea {
    int rank, size, points, dim;
    __host__ __device__ size_t slot_floats() const { return (size_t)points * size * dim; }
    __host__ __device__ size_t bytes() const { return slot_floats() * 4 + ((size_t)points + size + 1) * 8; }
    __host__ __device__ float* slot(unsigned char* base, int point, int src) const {
        return reinterpret_cast<float*>(base) + ((size_t)point * size + src) * dim;
    }
    __host__ __device__ unsigned long long* counter(unsigned char* base, int point) const {
        return reinterpret_cast<unsigned long long*>(base + slot_floats() * 4) + point;
    }
    __host__ __device__ unsigned long long* keys(unsigned char* base) const {
        return reinterpret_cast<unsigned long long*>(base + slot_floats() * 4) + points;
    }
    __host__ __device__ unsigned long long* key_counter(unsigned char* base) const { return keys(base) + size; }
};

enum : int { EPI_STORE = 0, EPI_RESID = 1, EPI_QKV = 2, EPI_SWIGLU = 3, EPI_ARGMAX = 4 };

// Launch plan of one weight-streaming GEMV (y = W x, W row-major [rows, K]).
struct GemvPlan {
    int rows, K, unit;      // unit: rows per indivisible work item (2 for paired epilogues)
    int wsize;              // bytes per weight element (2 bf16, 4 f32)
    int nseg;               // K segments per row (one warp each)
    int cpt;                // 16-byte chunks per lane per segment (template parameter)
    int stage_rows;         // rows per pipeline stage
    int nstages;            // pipeline depth
    int nw;                 // consumer warps per CTA (8 or 16)
    int grid;               // CTAs
    int max_rows_cta;       // most rows any CTA owns
    int n_vec;              // independent input vectors (gridDim.y)
    size_t smem;            // dynamic shared memory bytes
    int lean;               // 1: the <= 80-register kernel (o-proj beside attention)
};

struct GemvArgs {
    const void* W;
    // input vector x [K] (f32), or the bf16 embedding row of step->tok
    const float* x;
    long long x_stride;         // between input vectors (gridDim.y)
    const uint16_t* x_embed;
    int vocab;
    // non-null with x_embed: x = adapter row + embedding row, the streaming
    // decoder input (adapter ring [adapter_cap, K] f32, row = pos mod cap)
    const float* x_adapter;
    int adapter_cap;
    const StepState* step;
    const float* norm_w;        // non-null: RMSNorm(x) with this gain first
    float eps;
    float* x_copy_out;          // non-null: CTA 0 stores the raw x here
    // outputs
    float* y;
    long long y_stride;
    const float* resid;
    const float* bias;
    // QKV epilogue: RoPE on q and k, k/v into the ring slot of the new token
    int q_dim, kv_dim, head_dim;
    const float* rope_cos;      // [max_pos, head_dim/2]
    const float* rope_sin;
    int max_pos;
    float* k_ring;              // [n_kv, cap, head_dim]
    float* v_ring;
    int ring_cap;
    int kv_window;
    const KvState* kv_state;    // state before this step's append
    // O-proj: commit this step's single-token append to the layer state
    KvState* kv_commit;
    // LM head
    ArgmaxPart* am_part;
    unsigned* err;
    // Tensor-parallel exchange over peer memory (null xch: off).  xch[p] is
    // rank p's exchange area (a peer mapping for p != rank).
    unsigned char* const* xch;
    XchArea xa;
    int xch_out;                      // >= 0: rows also go to slot (xch_out, rank) of every rank
    int xch_in;                       // >= 0: x = sum over ranks of this rank's slots (xch_in, *)
    unsigned long long xch_arrivals;  // arrivals per step at point xch_in (size x producer grid)
    const unsigned long long* tp_steps;  // steps this rank has completed
    // Next weight launch (non-null pf_W): once this CTA's producer has issued
    // its last copy it prefetches into L2 the first pf_max_bytes of the band
    // the same-index CTA of that launch streams.
    const void* pf_W;
    long long pf_row_bytes;
    int pf_rows, pf_unit, pf_grid;
    int pf_max_bytes;
};

struct AttnArgs {
    const float* q;             // [n_heads, hd]
    const float* k_ring;        // [n_kv, cap, hd]
    const float* v_ring;
    int n_heads, n_kv, hd, cap;
    int cfg_window;             // DecoderConfig.sliding_window (masking); 0 = none
    const KvState* st;
    int pre_append;             // 1: st is the state before a single-token append
    int kv_window;              // cache window used to evict (pre_append only)
    int nsplit;
    float* part;                // accumulators [n_kv, nsplit, G, hd], then (m, l) [n_kv, nsplit, G, 2]
    unsigned* tickets;          // [n_kv], zero between launches
    float* out;                 // [n_heads, hd]
    float scale;
    unsigned* err;
    // Independent streams (gridDim.z; 0 counts as 1): stream z reads and
    // writes every pointer above advanced by z times its stride, and uses
    // tickets + z * n_kv.
    int n_streams;
    long long q_stride, ring_stride, out_stride, part_stride, st_stride;
    // non-null: the output also goes to this X operand of the next GEMM
    // (XOP layout, stream z in row z; see XOP_BYTES below)
    unsigned char* xop;
};

// X operand of the multi-stream GEMM in global memory ("XOP" layout): for a
// vector set of width K (8 streams), K / 64 blocks of 2 KB, each the bf16
// hi/lo image the tensor core reads from shared memory: element k of stream b
// at block k / 64, K-step (k % 64) / 16, half (k / 8) % 2, then hi in rows
// 0..7 and lo in rows 8..15 (row b), element k % 8.  A producer kernel writes
// its outputs there directly, so the GEMM loads its slice with one bulk copy.
inline size_t xop_bytes(int K) { return (size_t)(K / 64) * 2048; }

// Record a failure for vox_last_error() and return `code` (host side).
int report_error(int code, const char* msg);

// ---- multi-stream skinny GEMM on tcgen05 (bf16 weights, B <= 8 streams) ----
enum : int { BG_STORE = 0, BG_QKV = 1, BG_RESID = 2, BG_SWIGLU = 3, BG_ARGMAX = 4 };

struct BgArgs {
    const unsigned char* wt;    // weights pre-tiled into 128 x 64 UMMA blocks (launch_tile_weights)
    int rows, K;                // logical weight shape [rows, K]
    int tiles, kbt;             // 128-row tiles, 64-wide K blocks per tile
    int splits;                 // K splits per tile
    int B;                      // active streams (<= 8)
    int xslab_bytes;            // shared bytes of one split's X operand
    const float* x;             // [B, x_stride] f32 inputs (X operand built in the kernel), or
    const unsigned char* xop;   // the X operand already in XOP layout (one bulk copy per split)
    long long x_stride;
    const float* norm_w;        // non-null: apply RMSNorm with this gain to x
    const float* ssp;           // RMSNorm partial sums of squares [ssp_parts, 8] of x
    int ssp_parts;
    float eps;
    int epi;
    float* y;                   // [B, y_stride]
    long long y_stride;
    const float* bias;
    const float* resid;
    float* ssp_out;             // BG_RESID: per-tile sums of squares of y [tiles, 8]
    unsigned char* xop_out;     // BG_RESID / BG_SWIGLU: also write y (times xop_gain) in XOP layout
    const float* xop_gain;      // per-element gain for xop_out (the next RMSNorm's); null = 1
    int q_dim, kv_dim, head_dim;
    const float* rope_cos;
    const float* rope_sin;
    int max_pos;
    const StepState* steps;     // per stream
    KvState* kv_state;
    long long kv_state_stride;
    float* k_ring;
    float* v_ring;
    long long ring_stride;      // floats between streams' rings
    int ring_cap, kv_window;
    KvState* kv_commit;         // non-null: commit one single-token append per stream
    ArgmaxPart* am_part;        // [tiles, 8]
    float* part;                // split-K partial tiles [tiles * splits, 128, 8]
    unsigned* tickets;          // [tiles], zero between launches
    unsigned* err;
};

// A chain of GEMMs run by one persistent launch, phase after phase; phase p
// reads what phase p - 1 wrote (see vox_bgemm.cu).
constexpr int kBgMaxPhases = 4;
struct BgChain {
    int n_phases;
    int xslab_bytes;            // largest X operand of any phase
    unsigned* done;             // [n_phases - 1] CTA completion counters, zero at launch
    BgArgs ph[kBgMaxPhases];
};

// K blocks (of 64) one split may cover: its X operand (2 KB per block) sits
// next to the 128 KB weight ring in the 227 KB of one CTA.
constexpr int kBgMaxBlocksPerSplit = 40;
size_t bgemm_smem_bytes(int xslab_bytes);
int bgemm_xslab_bytes(int K, int splits);
cudaError_t bgemm_prepare(int dev);
// grid <= number of SMs when n_phases > 1 (all CTAs must be resident together).
cudaError_t launch_bgemm(const BgChain& c, int grid, cudaStream_t s, bool pdl);
size_t tiled_bytes(int rows, int K);
cudaError_t launch_bg_embed(const uint16_t* embed, int vocab, int dim, const StepState* steps, int B, float* hid,
                            float* ssp, unsigned char* xop, const float* xop_gain, unsigned* zero, int n_zero,
                            unsigned* err, cudaStream_t s, bool pdl);
cudaError_t launch_bg_argmax_final(const ArgmaxPart* parts, int n_tiles, StepState* steps, int B,
                                   int32_t* tok_out, cudaStream_t s, bool pdl);
cudaError_t launch_tile_weights(const uint16_t* src, uint16_t* dst, int rows, int K, cudaStream_t s);

// ---- batched prompt prefill (vox_prefill.cu) ----
// Prefill operand: per token block (tn tokens) and 64-wide K block one slab of
// 2 tn rows (bf16 hi rows, then lo rows) x 64 in UMMA canonical K-major layout.
inline size_t pf_xop_bytes(int t_pad, int K) { return (size_t)t_pad * 2 * K * 2; }

struct PfGemmArgs {
    const unsigned char* wt;    // weights pre-tiled into 128 x 64 UMMA blocks (launch_tile_weights)
    const unsigned char* xop;   // prefill operand of the pass
    float* part;                // [splits, T, rows] K-split partial products, or
    float* act;                 // non-null (splits 1, w1|w3 rows interleaved): SiLU(gate) * up [T, rows / 2]
    unsigned char* xop_out;     // wide form with act: SiLU(gate) * up as the next GEMM's prefill operand
                                //   (a buffer other than xop) instead of act
    int rows, kbt, tiles;       // weight shape: rows, 64-wide K blocks, 128-row tiles (even in the wide form)
    int tn, nblocks, T;         // tokens per block (16..128, multiple of 16), blocks, live tokens
    int splits;                 // K splits (<= kbt)
    unsigned* err;
};

struct PfNormArgs {
    float* h;                   // [T, dim] hidden rows, updated in place
    float* ssp;                 // [T, ssp_chunks] sums of squares per 512-element chunk
    int ssp_chunks;             // ceil(dim / 512)
    int Tp;                     // padded tokens (operand rows)
    const float* part;          // residual mode: [splits, T, dim] partials added to h
    int splits;
    const uint16_t* embed;      // embedding mode: rows of the token ids (bf16), h overwritten
    const int32_t* tokens;      // [T]
    int vocab;
    const float* adapter;       // embedding mode, nullable: adapter ring [adapter_cap, dim]
    int adapter_cap;
    long long pos0;             // position of token 0 of the pass
    const float* gain;          // RMSNorm gain of the next linear
    float eps;
    unsigned char* xop;         // nullable: prefill operand of the next linear
    int tn;
    int T, dim;
    unsigned* err;
};

struct PfQkvArgs {
    const float* part;          // [splits, T, q_dim + 2 kv_dim]
    int splits, T;
    int q_dim, kv_dim, head_dim;
    const float* rope_cos;
    const float* rope_sin;
    int max_pos;
    long long pos0;
    float* q;                   // [T, q_dim]
    float* kc;                  // [T, kv_dim] the pass's keys (RoPE applied)
    float* vc;                  // [T, kv_dim] the pass's values
    unsigned* err;
};

struct PfAttnArgs {
    const float* q;             // [T, n_heads * head_dim]
    const float* kc_in;         // [T, n_kv * head_dim] the pass's keys
    const float* vc_in;
    const float* k_ring;        // layer ring [n_kv, cap, head_dim]
    const float* v_ring;
    int T, n_heads, n_kv, head_dim, cap;
    int len0, start0;           // the layer's cache before the pass
    int win;                    // keys a token sees: min(cache window, attention window)
    int qb;                     // tokens per block: 16 (CUDA-core kernel) or 32 (tensor-core kernel)
    int kc, cmax;               // keys per chunk (multiple of 32, or 64 for tensor cores), most chunks of any block
    unsigned* err;
    float* part;                // chunk partials, pf_attn_part_floats
    float scale;
    float* out;                 // [T, n_heads * head_dim]
    unsigned char* xop;         // tensor-core kernel, cmax 1: non-null = write the rows as the next
    int xop_tn;                 //   GEMM's prefill operand (tokens per block) instead of `out`
    unsigned char* kvop;        // tensor-core kernel: K / V operand tiles (pf_kv_tiles_kernel), kv_tiles
    int kv_base, kv_tiles;      //   of pf_kv_tile_bytes() per kv head from key kv_base (a multiple of 64,
                                //   at most the pass's first key) through the pass's last key
};

struct PfCommitArgs {
    const float* kc;
    const float* vc;
    float* k_ring;
    float* v_ring;
    int T, kv_dim, head_dim, cap;
    long long end0;             // (start0 + len0) % cap before the pass
    KvState* state;
    KvState final_state;        // state after T single-token appends
};

size_t pf_gemm_smem_bytes(bool wide);
// The wide form (tokens as the M = 128 rows, two weight tiles as N = 256)
// takes full 128-token blocks and a multiple of 256 weight rows.
bool pf_gemm_wide_ok(int rows, int tn);
cudaError_t pf_prepare();
cudaError_t launch_pf_gemm(const PfGemmArgs& a, int grid, bool wide, cudaStream_t s);
// The hidden rows (embedding + adapter, or residual + split sums) and their
// sums of squares; then RMSNorm x gain into the operand (Tp = padded tokens,
// blocks x tn, a multiple of 16).
cudaError_t launch_pf_resid(const PfNormArgs& a, cudaStream_t s);
cudaError_t launch_pf_norm_xop(const PfNormArgs& a, cudaStream_t s);
cudaError_t launch_pf_qkv(const PfQkvArgs& a, cudaStream_t s);
int pf_attn_cmax(int T, int len0, int win, int kc, int qb);
size_t pf_attn_part_floats(int T, int n_kv, int head_dim, int cmax, int qb);
// Tensor-core variant (4 q heads per kv head, head_dim 128; qb 32, kc a multiple of 64).
bool pf_attn_tc_supported(int n_heads, int n_kv, int head_dim);
cudaError_t launch_pf_attn_tc(const PfAttnArgs& a, cudaStream_t s);
// The pass's keys and values as the tensor-core attention's operand tiles.
cudaError_t launch_pf_kv_tiles(const PfAttnArgs& a, cudaStream_t s);
size_t pf_kv_tile_bytes();
cudaError_t launch_pf_attn(const PfAttnArgs& a, cudaStream_t s);
cudaError_t launch_pf_attn_merge(const PfAttnArgs& a, cudaStream_t s);
cudaError_t launch_pf_split(const float* src, int T, int Tp, int K, unsigned char* xop, int tn, cudaStream_t s);
cudaError_t launch_pf_swiglu(const float* part, int splits, int T, int Tp, int hidden, unsigned char* xop, int tn,
                             cudaStream_t s);
cudaError_t launch_pf_commit(const PfCommitArgs& a, cudaStream_t s);

// ---- launchers (return the launch error) ----
// Launch shape of a weight-streaming GEMV: consumer warps per CTA (8 or 16,
// plus one producer warp), CTAs per SM (1 or 2) and shared-memory ring bytes
// per CTA.  Measured on the 26-layer single-GPU step (256 steps, context
// 520-776): two 8-warp CTAs per SM with 72-88 KB rings beat one 16-warp CTA
// with a 160 KB ring (1.566 vs 1.571 ms per token, w1|w3 alone 5.75 vs 5.68
// TB/s; 64 KB rings lose): a CTA of the next launch can start streaming on an
// SM while the other CTA of this launch is still in its tail, and an attention
// CTA fits beside one GEMV CTA.  The o-proj launch, which follows attention,
// uses the lean shape: the 80-register kernel with K cut into 8 segments (at
// most 2 chunks per lane, no spills) and a 48 KB ring, so two o-proj CTAs fit
// beside a cluster-attention CTA with its two-stage K/V ring and stream their
// weights while attention runs (with a 72 KB ring beside one-stage attention:
// 1.559 vs 1.574 ms per token, context 520-776; the same shape for q|k|v,
// before attention, measured 1.619 vs 1.567).  Tensor-parallel o-proj
// and w2 keep the wide shape, whose fewer CTAs mean fewer peer arrivals per
// exchange.
struct GemvShape {
    int warps;
    int ctas_per_sm;
    size_t ring_bytes;
    int lean;
};
constexpr GemvShape kGemvPaired{8, 2, 80 * 1024, 0};
constexpr GemvShape kGemvLean{8, 2, 48 * 1024, 1};
constexpr GemvShape kGemvWide{16, 1, 160 * 1024, 0};
GemvPlan plan_gemv(int rows, int K, int unit, int wsize, int num_sms, int n_vec, GemvShape shape = kGemvWide);
bool gemv_supported(int K, int wsize);
// L2 prefetch of the next weight launch by each GEMV CTA's producer, bytes per
// CTA.  The launches of a step stream back to back, and the next launch's CTAs
// only find room on an SM once this launch's CTAs leave, all at about the same
// time; bytes prefetched into L2 during the tail keep HBM busy across the
// boundary.  Measured on the 26-layer step (context 520-776), ms per token:
// none 1.569, 16 KB 1.546, 24 KB 1.538, 32 KB 1.537, 40 KB 1.542, 48 KB 1.552,
// 56 KB 1.564, 80 KB 1.588, 160 KB 1.580 (larger prefetches slow the tail of
// the launch that issues them).
constexpr int kGemvPrefetchBytes = 32 * 1024;

inline void gemv_set_prefetch(GemvArgs& a, const void* W, const GemvPlan& p, int wsize) {
    a.pf_W = W;
    a.pf_row_bytes = (long long)p.K * wsize;
    a.pf_rows = p.rows;
    a.pf_unit = p.unit;
    a.pf_grid = p.grid;
    a.pf_max_bytes = kGemvPrefetchBytes;
}

size_t gemv_max_smem();
cudaError_t gemv_prepare(int dev);   // raise per-kernel smem limits once per device
cudaError_t launch_gemv(const GemvPlan& p, const GemvArgs& a, int epi, cudaStream_t s, bool pdl);

int attn_splits_for(int n_kv, int num_sms);
int attn_max_splits();  // most chunks per (stream, kv head) a launch may use
bool attn_supported(int n_heads, int n_kv, int hd);
size_t attn_smem_bytes(int n_heads, int n_kv, int hd);
cudaError_t attn_prepare(int dev);
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl);
// One stream, short context: one thread-block cluster per kv head merging in
// distributed shared memory.  attn_cluster_size is 16 or 8 CTAs per kv head,
// or 0 when this shape or device cannot run it; the host uses it for at most
// attn_cluster_max_tokens() live tokens.  It reads the ring state before its
// grid-dependency wait, so no kernel that may still run when it starts may
// write a.st (true in the step graphs, where only a later o-proj commits it).
int attn_cluster_size(int n_heads, int n_kv, int hd);
int attn_cluster_max_tokens();
cudaError_t launch_attention_cluster(const AttnArgs& a, cudaStream_t s, bool pdl);

cudaError_t launch_argmax_final(const ArgmaxPart* parts, int n, StepState* step, int32_t* tok_out,
                                cudaStream_t s, bool pdl);
// Tensor-parallel argmax: this rank's best (value, index + index_offset) as
// an order-preserving 64-bit key (max-reduced across ranks), then the step
// bookkeeping from the reduced key.
cudaError_t launch_tp_argmax_key(const ArgmaxPart* parts, int n, long long index_offset, unsigned long long* key,
                                 cudaStream_t s, bool pdl);
cudaError_t launch_tp_argmax_apply(const unsigned long long* key, StepState* step, int32_t* tok_out, cudaStream_t s);
// Same over peer memory in one launch: this rank's key to every rank, wait
// for all keys, take the max, apply it, count the step in tp_steps.
cudaError_t launch_tp_argmax_xch(const ArgmaxPart* parts, int n, long long index_offset, unsigned char* const* xch,
                                 XchArea xa, unsigned long long* tp_steps, StepState* step, int32_t* tok_out,
                                 unsigned* err, cudaStream_t s, bool pdl);
cudaError_t launch_kv_scatter(const float* src_k, const float* src_v, float* k_ring, float* v_ring,
                              int n_kv, int hd, int cap, int slot0, int n_tokens, cudaStream_t s);
cudaError_t launch_kv_gather(const float* k_ring, const float* v_ring, float* dst_k, float* dst_v,
                             int n_kv, int hd, int cap, int start, int len, cudaStream_t s);
// Fill rows of a matrix from the counter-based generator.  Element (r, c) of
// the logical tensor `tensor_id` ([rows, cols]) lands at
// dst[(r * row_mul + row_add) * cols + c]; wsize 2 = bf16, 4 = f32.
cudaError_t launch_gen_matrix(void* dst, int wsize, uint64_t seed, uint64_t tensor_id, float std,
                              long long rows, long long cols, int row_mul, int row_add,
                              cudaStream_t s);
// Same for a [rows, cols] block whose element (0, 0) is (row0, col0) of a
// tensor with full_cols columns (tensor-parallel shards).
cudaError_t launch_gen_matrix_part(void* dst, int wsize, uint64_t seed, uint64_t tensor_id, float std,
                                   long long rows, long long cols, int row_mul, int row_add, long long row0,
                                   long long col0, long long full_cols, cudaStream_t s);
cudaError_t launch_fill_f32(float* dst, float v, long long n, cudaStream_t s);
// Fill tokens 0..len-1 of a ring (start slot 0) from the generator: K from
// tensor id_k, V from id_v, each [len, n_kv, hd] token-major, bf16-rounded.
cudaError_t launch_kv_fill_random(float* kr, float* vr, int n_kv, int hd, int cap, int len, uint64_t seed,
                                  uint64_t id_k, uint64_t id_v, float stdv, cudaStream_t s);
cudaError_t launch_rmsnorm_rows(float* out, const float* in, const float* w, long long n_rows,
                                int dim, float eps, cudaStream_t s);
cudaError_t launch_rope_table(float* data, const float* cos_t, const float* sin_t, long long seq_len,
                              int n_heads, int hd, cudaStream_t s);
cudaError_t launch_silu(float* x, long long n, cudaStream_t s);
cudaError_t launch_softmax(float* x, long long n, cudaStream_t s);
cudaError_t launch_add(float* dst, const float* src, long long n, cudaStream_t s);

}  // namespace vox
