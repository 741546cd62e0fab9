// vox_capi.cpp -- host side of the C ABI declared in include/vox_decoder.h.
//
// Owns device memory, the CUDA stream, the rolling-cache bookkeeping (the
// exact integer arithmetic of crates/voxtral/src/kv.rs:48-88, mirrored on the
// device), kernel launch plans and the captured CUDA graph of a token step.
// Every compute step runs on the GPU; this file only validates, copies and
// launches.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/vox_decoder.h"
#include "vox_host.h"
#include "vox_internal.h"
#include "vox_kernels.h"

using namespace vox;

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define CUDA_TRY(expr)                                                                   \
    do {                                                                                 \
        cudaError_t e_ = (expr);                                                         \
        if (e_ != cudaSuccess)                                                           \
            return fail(e_ == cudaErrorMemoryAllocation ? VOX_ERR_OOM : VOX_ERR_CUDA,     \
                        "%s failed: %s", #expr, cudaGetErrorString(e_));                  \
    } while (0)

#define TRY(expr)                  \
    do {                           \
        int rc_ = (expr);          \
        if (rc_ != VOX_OK) return rc_; \
    } while (0)

struct LayerDev {
    void* wqkv = nullptr;   // [q_dim + 2 kv_dim, dim]: wq rows, wk rows, wv rows
    void* wo = nullptr;     // [dim, q_dim]
    void* w13 = nullptr;    // [2 hidden, dim]: row 2j = w1[j], row 2j+1 = w3[j]
    void* w2 = nullptr;     // [dim, hidden]
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
    bool ready = false;
    // The same matrices pre-tiled for the tensor-core multi-stream GEMM
    // (launch_tile_weights); rebuilt after every upload.
    unsigned char *wqkv_t = nullptr, *wo_t = nullptr, *w13_t = nullptr, *w2_t = nullptr;
    bool tiled = false;
};

// Launch shape of one multi-stream GEMM (vox_bgemm.cu).
struct BgPlan {
    int rows = 0, K = 0, tiles = 0, kbt = 0, splits = 1, grid = 1, xslab = 0;
};

// Device buffers of the multi-stream step, sized for 8 streams.
struct BatchBufs {
    bool ready = false;
    float *hid = nullptr, *hmid = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr, *logits = nullptr;
    float* ssp = nullptr;        // RMSNorm partial sums [dim tiles, 8]
    float* part = nullptr;       // split-K partial tiles
    float* attn_part = nullptr;  // attention split partials, all streams
    ArgmaxPart* am = nullptr;    // [vocab tiles, 8]
    unsigned* tickets = nullptr;       // GEMM tiles
    unsigned* attn_tickets = nullptr;  // [8, n_kv]
    StepState* steps = nullptr;        // [8]
    int32_t* tok_out = nullptr;        // [8]
    StepState* h_steps = nullptr;      // pinned [8]
    int32_t* h_tok = nullptr;          // pinned token history
    size_t h_tok_cap = 0;
    BgPlan p_qkv, p_o, p_w13, p_w2, p_head;         // one GEMM per launch
    BgPlan c_qkv, c_o, c_w13, c_w2, c_head;         // phases of the per-layer chains
    unsigned* done = nullptr;  // chain completion counters [n_layers + 1][kBgMaxPhases]
    int n_done = 0;
    // X operands in XOP layout, written by the producing kernel: hid * attn_norm
    // (q|k|v, LM head), attention output (o-proj), hmid * ffn_norm (w1|w3), act (w2)
    unsigned char *xop_a = nullptr, *xop_o = nullptr, *xop_f = nullptr, *xop_h = nullptr;
};

// Device buffers of the batched prefill (vox_prefill.cu), sized for one pass
// of up to kPrefillPass tokens; `part` grows with the largest split plan.
constexpr int kPrefillPass = 512;
struct PrefillBufs {
    bool ready = false;
    float *h = nullptr, *q = nullptr, *kc = nullptr, *vc = nullptr, *attn = nullptr, *part = nullptr;
    size_t part_floats = 0;
    float* ssp = nullptr;        // [kPrefillPass, ceil(dim / 512)] RMSNorm partial sums
    float* attn_part = nullptr;  // attention chunk partials
    size_t attn_part_floats = 0;
    float* kvop = nullptr;       // K / V operand tiles of the tensor-core attention
    size_t kvop_floats = 0;
    unsigned char* xop = nullptr;
    unsigned char* xop2 = nullptr;  // second operand buffer: the w2 operand written by the w1|w3 epilogue
    int32_t* tokens = nullptr;    // [kPrefillPass]
    int32_t* h_tokens = nullptr;  // pinned staging
};

// Launch shape of one prefill GEMM: the K split count that minimises the
// busiest CTA's work over tiles x token blocks x splits items, at least 4 K
// blocks per split, ties to fewer splits.  An item costs its K blocks (48 KB
// of operands each) plus its epilogue: a 128-row x tn-token f32 tile written
// and read back once by the consumer, about 3 K blocks' worth at tn = 128.
//
// The wide form (full 128-token blocks, rows a multiple of 256; only where the
// caller allows it) takes a pair of tiles per item: a K block moves 64 KB for
// twice the products, and the epilogue's 256-row tile costs about 4 of them.
// Measured at 512 tokens: the w1|w3 GEMM (one split, SwiGLU epilogue) 92 vs
// 97 us, the prefill 1.5 % faster; the split-K GEMMs slower (q|k|v 42 vs 35,
// o-proj 31 vs 24, w2 52 vs 45 us: half the items need more splits, and a
// lane's partial row is stored along one token), so they stay narrow.
struct PfPlan {
    int rows = 0, K = 0, tiles = 0, kbt = 0, splits = 1, grid = 1;
    bool wide = false;
};
PfPlan make_pfplan(int rows, int K, int nblocks, int tn, int num_sms, bool allow_wide = false) {
    PfPlan p;
    p.rows = rows;
    p.K = K;
    p.tiles = (rows + 127) / 128;
    p.kbt = K / 64;
    p.wide = allow_wide && pf_gemm_wide_ok(rows, tn);
    const long long base = (long long)(p.wide ? p.tiles / 2 : p.tiles) * nblocks;
    long long best = -1;
    for (int s = 1; s <= 16 && s <= p.kbt; ++s) {
        if (s > 1 && p.kbt / s < 4) break;
        const long long items = base * s;
        const long long grid = std::min<long long>(items, num_sms);
        const long long epi = p.wide ? 4 : (3 * tn + 127) / 128;
        const long long cost = ((items + grid - 1) / grid) * ((p.kbt + s - 1) / s + epi);
        if (best < 0 || cost < best) {
            best = cost;
            p.splits = s;
            p.grid = (int)grid;
        }
    }
    return p;
}

// K splits and grid of a multi-stream GEMM launched on its own: one CTA per
// SM (the 128 KB weight ring fills it), the split count that minimises the
// busiest CTA's K blocks (items per CTA x blocks per item), at most
// kBgMaxBlocksPerSplit K blocks per split so the split's X operand fits in
// shared memory.  The grid is a multiple of the split count, so a CTA keeps
// its split (and X operand) across items.
BgPlan make_bgplan(int rows, int K, int num_sms) {
    BgPlan p;
    p.rows = rows;
    p.K = K;
    p.tiles = (rows + 127) / 128;
    p.kbt = K / 64;
    long long best = -1;
    for (int s = 1; s <= p.kbt && s <= 64; ++s) {
        const int per = (p.kbt + s - 1) / s;
        if (per > kBgMaxBlocksPerSplit) continue;
        int grid = num_sms - num_sms % s;
        if (grid < s) grid = s;
        const long long items = (long long)p.tiles * s;
        if (grid > items) grid = (int)items;
        const long long cost = ((items + grid - 1) / grid) * per;
        if (best < 0 || cost < best) {
            best = cost;
            p.splits = s;
            p.grid = grid;
        }
    }
    p.xslab = bgemm_xslab_bytes(K, p.splits);
    return p;
}

// Plan of one phase of a persistent GEMM chain: the grid is fixed (one CTA
// per SM); the split count minimises the busiest CTA's K blocks, ties going
// to fewer splits.  A CTA whose items change split rebuilds its X operand,
// which costs about one K block.
BgPlan make_chain_plan(int rows, int K, int grid) {
    BgPlan p;
    p.rows = rows;
    p.K = K;
    p.tiles = (rows + 127) / 128;
    p.kbt = K / 64;
    p.grid = grid;
    long long best = -1;
    for (int s = 1; s <= p.kbt && s <= 64; ++s) {
        const int per = (p.kbt + s - 1) / s;
        if (per > kBgMaxBlocksPerSplit) continue;
        const long long items = (long long)p.tiles * s;
        const long long rounds = (items + grid - 1) / grid;
        long long cost = rounds * per;
        if (rounds > 1 && grid % s) cost += rounds;  // X operand rebuilt between items
        if (best < 0 || cost < best) {
            best = cost;
            p.splits = s;
        }
    }
    p.xslab = bgemm_xslab_bytes(K, p.splits);
    return p;
}

BgChain chain_of(const BgArgs& a, const BgPlan& p) {
    BgChain c{};
    c.n_phases = 1;
    c.xslab_bytes = p.xslab;
    c.ph[0] = a;
    return c;
}

}  // namespace

int vox::report_error(int code, const char* msg) { return fail(code, "%s", msg); }

int vox::report_errorf(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

struct vox_ctx {
    vox_decoder_config cfg{};
    vox_ctx_options opt{};
    int dev = 0, num_sms = 148, wsize = 2;
    size_t q_dim = 0, kv_dim = 0, qkv_rows = 0;
    cudaStream_t stream = nullptr;
    std::vector<LayerDev> layers;
    uint16_t* embed = nullptr;
    void* lm_head = nullptr;
    float* final_norm = nullptr;
    bool embed_ready = false, head_ready = false;
    float* rope_cos = nullptr;
    float* rope_sin = nullptr;
    int max_pos = 0;
    float *hid = nullptr, *hmid = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr,
          *logits = nullptr;
    ArgmaxPart* am_part = nullptr;
    float* attn_part = nullptr;
    unsigned* tickets = nullptr;
    int nsplit = 1;
    StepState* step = nullptr;
    int32_t* tok_out = nullptr;
    unsigned* err = nullptr;
    StepState* h_steps = nullptr;  // pinned, one slot per queued step
    size_t h_steps_cap = 0;
    int32_t* h_tok = nullptr;      // pinned
    unsigned* h_err = nullptr;     // pinned
    cudaEvent_t ev[16] = {};
    std::vector<vox_kv*> caches;   // caches created from this context, still alive
    uint64_t launches = 0;
    GemvPlan p_qkv{}, p_o{}, p_w13{}, p_w2{}, p_head{};
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    // multi-stream path
    unsigned char* head_t = nullptr;
    bool head_tiled = false;
    BatchBufs bb;
    PrefillBufs pf;
};

// A rolling cache of one stream, or of n_streams independent streams laid
// out stream-major so that stream s is itself a single-stream cache (a view).
struct vox_kv {
    vox_ctx* ctx = nullptr;
    size_t n_layers = 0, n_kv = 0, hd = 0, window = 0, cap = 0;
    size_t n_streams = 1;
    float* k = nullptr;          // [n_streams, n_layers, n_kv, cap, hd]
    float* v = nullptr;
    KvState* dstate = nullptr;   // [n_streams, n_layers]
    std::vector<HostKv> hs_store;  // owner: host mirror [n_streams, n_layers]
    HostKv* hs = nullptr;          // [n_layers] of this cache (stream 0 of an owner)
    vox_kv* parent = nullptr;      // set on a stream view
    std::vector<vox_kv*> views;    // owner: views by stream, created on demand
    cudaGraphExec_t step_graph = nullptr;
    uint64_t graph_kernels = 0;
    cudaGraphExec_t step_graph_short = nullptr;  // same step, cluster attention (short contexts)
    uint64_t graph_kernels_short = 0;
    cudaGraphExec_t batch_graph = nullptr;  // multi-stream step over all streams
    uint64_t batch_kernels = 0;
    size_t layer_elems() const { return n_kv * cap * hd; }
    size_t stream_elems() const { return n_layers * layer_elems(); }
};

namespace {

int check_device_errors(vox_ctx* c) {
    CUDA_TRY(cudaMemcpyAsync(c->h_err, c->err, sizeof(unsigned), cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    unsigned bits = *c->h_err;
    if (bits) {
        CUDA_TRY(cudaMemsetAsync(c->err, 0, sizeof(unsigned), c->stream));
        if (bits & (ERR_FULL_WAIT | ERR_EMPTY_WAIT | ERR_DRAIN_WAIT | ERR_GRID_WAIT)) {
            // An aborted step leaves barrier counters and tickets half-advanced.
            CUDA_TRY(cudaMemsetAsync(c->tickets, 0, c->cfg.n_kv_heads * sizeof(unsigned), c->stream));
            if (c->bb.ready) {
                size_t tiles = 0;
                for (const BgPlan* p : {&c->bb.p_qkv, &c->bb.p_o, &c->bb.p_w13, &c->bb.p_w2, &c->bb.p_head})
                    tiles = std::max(tiles, (size_t)p->tiles);
                CUDA_TRY(cudaMemsetAsync(c->bb.tickets, 0, tiles * sizeof(unsigned), c->stream));
                CUDA_TRY(cudaMemsetAsync(c->bb.done, 0, (size_t)c->bb.n_done * sizeof(unsigned), c->stream));
                CUDA_TRY(cudaMemsetAsync(c->bb.attn_tickets, 0, 8 * c->cfg.n_kv_heads * sizeof(unsigned), c->stream));
            }
        }
        CUDA_TRY(cudaStreamSynchronize(c->stream));
        if (bits & (ERR_FULL_WAIT | ERR_EMPTY_WAIT | ERR_DRAIN_WAIT | ERR_GRID_WAIT))
            return fail(VOX_ERR_DEVICE_TIMEOUT, "a bounded wait inside a kernel expired (bits 0x%x)", bits);
        if (bits & ERR_POS_RANGE) return fail(VOX_ERR_RANGE, "position beyond the RoPE table");
        if (bits & ERR_TOKEN_RANGE) return fail(VOX_ERR_RANGE, "token id outside the vocabulary");
        return fail(VOX_ERR_CUDA, "device error bits 0x%x", bits);
    }
    return VOX_OK;
}

int ensure_scratch(vox_ctx* c, size_t bytes) {
    if (bytes <= c->scratch_bytes) return VOX_OK;
    if (c->scratch) {
        CUDA_TRY(cudaStreamSynchronize(c->stream));
        cudaFree(c->scratch);
        c->scratch = nullptr;
        c->scratch_bytes = 0;
    }
    size_t b = 1 << 20;
    while (b < bytes) b <<= 1;
    CUDA_TRY(cudaMalloc(&c->scratch, b));
    c->scratch_bytes = b;
    return VOX_OK;
}

int validate_cfg(const vox_decoder_config* c) {
    if (!c) return fail(VOX_ERR_INVALID_ARG, "config is null");
    // decoder.rs:22-41, same order and messages.
    if (c->dim == 0) return fail(VOX_ERR_CONFIG, "dim must be > 0");
    if (c->hidden_dim == 0) return fail(VOX_ERR_CONFIG, "hidden_dim must be > 0");
    if (c->n_heads == 0) return fail(VOX_ERR_CONFIG, "n_heads must be > 0");
    if (c->n_kv_heads == 0) return fail(VOX_ERR_CONFIG, "n_kv_heads must be > 0");
    if (c->head_dim == 0) return fail(VOX_ERR_CONFIG, "head_dim must be > 0");
    if (c->n_heads % c->n_kv_heads != 0)
        return fail(VOX_ERR_CONFIG, "n_heads must be divisible by n_kv_heads");
    if (c->n_heads * c->head_dim < c->dim) return fail(VOX_ERR_CONFIG, "n_heads * head_dim must cover dim");
    if (c->sliding_window == 0)
        return fail(VOX_ERR_CONFIG, "sliding_window must be > 0 for rolling attention cache");
    return VOX_OK;
}

// Shapes the kernels need beyond the reference's own checks.
int check_kernel_shapes(const vox_decoder_config* c, int wsize) {
    const size_t q_dim = c->n_heads * c->head_dim;
    if (c->head_dim % 2) return fail(VOX_ERR_UNSUPPORTED, "head_dim must be even (interleaved RoPE pairs)");
    if (c->dim > (1u << 30) || c->hidden_dim > (1u << 30))
        return fail(VOX_ERR_UNSUPPORTED, "dimensions too large");
    if (!gemv_supported((int)c->dim, wsize) || !gemv_supported((int)q_dim, wsize) ||
        !gemv_supported((int)c->hidden_dim, wsize))
        return fail(VOX_ERR_UNSUPPORTED,
                    "dim, n_heads*head_dim and hidden_dim must be multiples of %d elements and at most %d",
                    16 / wsize, wsize == 2 ? 16384 : 8192);
    if (!attn_supported((int)c->n_heads, (int)c->n_kv_heads, (int)c->head_dim))
        return fail(VOX_ERR_UNSUPPORTED, "attention shape (group %zu x head_dim %zu) too large",
                    c->n_heads / c->n_kv_heads, c->head_dim);
    return VOX_OK;
}

int check_matrix_len(size_t got, size_t want, const char* name) {
    if (got != want) return fail(VOX_ERR_SHAPE, "%s shape mismatch", name);
    return VOX_OK;
}

// decoder.rs:58-84, generic over slice flavours.
template <class WS>
int validate_weights(const vox_decoder_config* cfg, const WS* w) {
    if (!w) return fail(VOX_ERR_INVALID_ARG, "weights are null");
    const size_t q_dim = cfg->n_heads * cfg->head_dim, kv_dim = cfg->n_kv_heads * cfg->head_dim;
    TRY(check_matrix_len(w->attention_norm.len, cfg->dim, "attention_norm"));
    TRY(check_matrix_len(w->wq.len, q_dim * cfg->dim, "wq"));
    TRY(check_matrix_len(w->wk.len, kv_dim * cfg->dim, "wk"));
    TRY(check_matrix_len(w->wv.len, kv_dim * cfg->dim, "wv"));
    TRY(check_matrix_len(w->wo.len, cfg->dim * q_dim, "wo"));
    TRY(check_matrix_len(w->ffn_norm.len, cfg->dim, "ffn_norm"));
    TRY(check_matrix_len(w->w1.len, cfg->hidden_dim * cfg->dim, "w1"));
    TRY(check_matrix_len(w->w2.len, cfg->dim * cfg->hidden_dim, "w2"));
    TRY(check_matrix_len(w->w3.len, cfg->hidden_dim * cfg->dim, "w3"));
    const void* ptrs[] = {w->attention_norm.ptr, w->wq.ptr, w->wk.ptr, w->wv.ptr, w->wo.ptr,
                          w->ffn_norm.ptr, w->w1.ptr, w->w2.ptr, w->w3.ptr};
    for (const void* p : ptrs)
        if (!p) return fail(VOX_ERR_INVALID_ARG, "a weight pointer is null");
    return VOX_OK;
}

// Convert a host matrix into the context's weight dtype.
std::vector<unsigned char> to_wdtype(const float* src, size_t n, int wsize) {
    std::vector<unsigned char> out(n * wsize);
    if (wsize == 4) {
        std::memcpy(out.data(), src, n * 4);
    } else {
        uint16_t* o = reinterpret_cast<uint16_t*>(out.data());
        for (size_t i = 0; i < n; ++i) o[i] = f32_to_bf16(src[i]);
    }
    return out;
}
std::vector<unsigned char> to_wdtype(const uint16_t* src, size_t n, int wsize) {
    std::vector<unsigned char> out(n * wsize);
    if (wsize == 2) {
        std::memcpy(out.data(), src, n * 2);
    } else {
        float* o = reinterpret_cast<float*>(out.data());
        for (size_t i = 0; i < n; ++i) o[i] = bf16_to_f32(src[i]);
    }
    return out;
}

int alloc_layer(vox_ctx* c, LayerDev& L) {
    if (L.wqkv) return VOX_OK;
    const size_t dim = c->cfg.dim, hid = c->cfg.hidden_dim;
    CUDA_TRY(cudaMalloc(&L.wqkv, c->qkv_rows * dim * c->wsize));
    CUDA_TRY(cudaMalloc(&L.wo, dim * c->q_dim * c->wsize));
    CUDA_TRY(cudaMalloc(&L.w13, 2 * hid * dim * c->wsize));
    CUDA_TRY(cudaMalloc(&L.w2, dim * hid * c->wsize));
    CUDA_TRY(dalloc(&L.attn_norm, dim));
    CUDA_TRY(dalloc(&L.ffn_norm, dim));
    return VOX_OK;
}

template <class WS>
int upload_layer(vox_ctx* c, size_t layer, const WS* w) {
    if (!c) return fail(VOX_ERR_INVALID_ARG, "context is null");
    if (layer >= c->layers.size()) return fail(VOX_ERR_INVALID_ARG, "layer %zu out of range", layer);
    TRY(validate_weights(&c->cfg, w));
    CUDA_TRY(cudaSetDevice(c->dev));
    LayerDev& L = c->layers[layer];
    TRY(alloc_layer(c, L));
    const size_t dim = c->cfg.dim, hid = c->cfg.hidden_dim, ws = c->wsize;
    auto put = [&](void* dst, const auto& slice) -> int {
        auto bytes = to_wdtype(slice.ptr, slice.len, (int)ws);
        CUDA_TRY(cudaMemcpy(dst, bytes.data(), bytes.size(), cudaMemcpyHostToDevice));
        return VOX_OK;
    };
    unsigned char* qkv = static_cast<unsigned char*>(L.wqkv);
    TRY(put(qkv, w->wq));
    TRY(put(qkv + c->q_dim * dim * ws, w->wk));
    TRY(put(qkv + (c->q_dim + c->kv_dim) * dim * ws, w->wv));
    TRY(put(L.wo, w->wo));
    TRY(put(L.w2, w->w2));
    // w1 -> even rows, w3 -> odd rows of w13.
    const size_t row = dim * ws;
    {
        auto b1 = to_wdtype(w->w1.ptr, w->w1.len, (int)ws);
        auto b3 = to_wdtype(w->w3.ptr, w->w3.len, (int)ws);
        CUDA_TRY(cudaMemcpy2D(L.w13, 2 * row, b1.data(), row, row, hid, cudaMemcpyHostToDevice));
        CUDA_TRY(cudaMemcpy2D(static_cast<unsigned char*>(L.w13) + row, 2 * row, b3.data(), row, row,
                              hid, cudaMemcpyHostToDevice));
    }
    CUDA_TRY(cudaMemcpy(L.attn_norm, w->attention_norm.ptr, dim * 4, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(L.ffn_norm, w->ffn_norm.ptr, dim * 4, cudaMemcpyHostToDevice));
    L.ready = true;
    L.tiled = false;
    return VOX_OK;
}

cudaError_t record_launch(vox_ctx* c, cudaError_t e) {
    if (e == cudaSuccess) ++c->launches;
    return e;
}

GemvArgs base_args(vox_ctx* c) {
    GemvArgs a{};
    a.step = c->step;
    a.eps = c->cfg.norm_eps;
    a.err = c->err;
    return a;
}

void set_prefetch(GemvArgs& a, const void* W, const GemvPlan& p, int wsize) {
    gemv_set_prefetch(a, W, p, wsize);
}

// Enqueue one decoder layer (decoder.rs:88-155) as five kernels.  With
// from_embed the input is the embedding row of the step's token, plus the
// row of `adapter` (an [adapter_cap, dim] ring) at the step's position when
// given: the streaming decoder input.
int enqueue_layer(vox_ctx* c, vox_kv* kv, size_t l, bool from_embed, bool pdl, bool short_attn = false,
                  const float* adapter = nullptr, int adapter_cap = 0) {
    const LayerDev& L = c->layers[l];
    float* kr = kv->k + l * kv->layer_elems();
    float* vr = kv->v + l * kv->layer_elems();
    KvState* st = kv->dstate + l;
    const int cap = (int)kv->cap, win = (int)kv->window;

    // 1) RMSNorm -> q|k|v -> RoPE -> k, v into the ring slot.
    GemvArgs a = base_args(c);
    a.W = L.wqkv;
    if (from_embed) {
        a.x_embed = c->embed;
        a.vocab = (int)c->opt.vocab;
        a.x_adapter = adapter;
        a.adapter_cap = adapter_cap;
        a.x_copy_out = c->hid;
    } else {
        a.x = c->hid;
    }
    a.norm_w = L.attn_norm;
    a.y = c->q;
    a.q_dim = (int)c->q_dim;
    a.kv_dim = (int)c->kv_dim;
    a.head_dim = (int)c->cfg.head_dim;
    a.rope_cos = c->rope_cos;
    a.rope_sin = c->rope_sin;
    a.max_pos = c->max_pos;
    a.k_ring = kr;
    a.v_ring = vr;
    a.ring_cap = cap;
    a.kv_window = win;
    a.kv_state = st;
    set_prefetch(a, L.wo, c->p_o, c->wsize);
    CUDA_TRY(record_launch(c, launch_gemv(c->p_qkv, a, EPI_QKV, c->stream, pdl)));

    // 2) attention over the ring (ops.rs:66-132).
    AttnArgs at{};
    at.q = c->q;
    at.k_ring = kr;
    at.v_ring = vr;
    at.n_heads = (int)c->cfg.n_heads;
    at.n_kv = (int)c->cfg.n_kv_heads;
    at.hd = (int)c->cfg.head_dim;
    at.cap = cap;
    at.cfg_window = (int)c->cfg.sliding_window;
    at.st = st;
    at.pre_append = 1;
    at.kv_window = win;
    at.nsplit = c->nsplit;
    at.part = c->attn_part;
    at.tickets = c->tickets;
    at.out = c->attn;
    at.scale = 1.0f / sqrtf((float)c->cfg.head_dim);
    at.err = c->err;
    CUDA_TRY(record_launch(c, short_attn ? launch_attention_cluster(at, c->stream, pdl)
                                         : launch_attention(at, c->stream, pdl)));

    // 3) o-proj + residual (decoder.rs:136-139); commits the append.
    a = base_args(c);
    a.W = L.wo;
    a.x = c->attn;
    a.y = c->hmid;
    a.resid = c->hid;
    a.kv_commit = st;
    a.kv_window = win;
    a.ring_cap = cap;
    set_prefetch(a, L.w13, c->p_w13, c->wsize);
    CUDA_TRY(record_launch(c, launch_gemv(c->p_o, a, EPI_RESID, c->stream, pdl)));

    // 4) RMSNorm -> w1|w3 -> SiLU(gate)*up (decoder.rs:143-150).
    a = base_args(c);
    a.W = L.w13;
    a.x = c->hmid;
    a.norm_w = L.ffn_norm;
    a.y = c->act;
    set_prefetch(a, L.w2, c->p_w2, c->wsize);
    CUDA_TRY(record_launch(c, launch_gemv(c->p_w13, a, EPI_SWIGLU, c->stream, pdl)));

    // 5) w2 + residual (decoder.rs:151-152).
    a = base_args(c);
    a.W = L.w2;
    a.x = c->act;
    a.y = c->hid;
    a.resid = c->hmid;
    if (l + 1 < c->layers.size())
        set_prefetch(a, c->layers[l + 1].wqkv, c->p_qkv, c->wsize);
    else if (c->lm_head)
        set_prefetch(a, c->lm_head, c->p_head, c->wsize);
    CUDA_TRY(record_launch(c, launch_gemv(c->p_w2, a, EPI_RESID, c->stream, pdl)));
    return VOX_OK;
}

// Final RMSNorm -> LM head -> argmax.
int enqueue_head(vox_ctx* c, bool pdl) {
    GemvArgs a = base_args(c);
    a.W = c->lm_head;
    a.x = c->hid;
    a.norm_w = c->final_norm;
    a.y = c->logits;
    a.am_part = c->am_part;
    CUDA_TRY(record_launch(c, launch_gemv(c->p_head, a, EPI_ARGMAX, c->stream, pdl)));
    CUDA_TRY(record_launch(c, launch_argmax_final(c->am_part, c->p_head.grid, c->step, c->tok_out,
                                                  c->stream, pdl)));
    return VOX_OK;
}

// ---- multi-stream step (tensor-core GEMMs, vox_bgemm.cu) ----------------------
int batch_supported(vox_ctx* c) {
    if (c->wsize != 2) return fail(VOX_ERR_UNSUPPORTED, "the multi-stream step needs bf16 weights");
    const vox_decoder_config& g = c->cfg;
    if (g.dim % 64 || c->q_dim % 64 || g.hidden_dim % 64)
        return fail(VOX_ERR_UNSUPPORTED, "the multi-stream step needs dim, n_heads*head_dim and hidden_dim "
                                         "to be multiples of 64");
    if (g.dim > 8192) return fail(VOX_ERR_UNSUPPORTED, "the multi-stream step needs dim <= 8192");
    return VOX_OK;
}

int tile_into(vox_ctx* c, unsigned char** dst, const void* src, int rows, int K) {
    if (!*dst) CUDA_TRY(cudaMalloc(dst, tiled_bytes(rows, K)));
    CUDA_TRY(record_launch(c, launch_tile_weights(static_cast<const uint16_t*>(src),
                                                  reinterpret_cast<uint16_t*>(*dst), rows, K, c->stream)));
    return VOX_OK;
}

// (Re)tile the layer matrices whose tiled copy is stale (enqueued only).
int tile_layers(vox_ctx* c) {
    const int dim = (int)c->cfg.dim, hid = (int)c->cfg.hidden_dim, qd = (int)c->q_dim, kvd = (int)c->kv_dim;
    for (auto& L : c->layers) {
        if (L.tiled) continue;
        TRY(tile_into(c, &L.wqkv_t, L.wqkv, qd + 2 * kvd, dim));
        TRY(tile_into(c, &L.wo_t, L.wo, dim, qd));
        TRY(tile_into(c, &L.w13_t, L.w13, 2 * hid, dim));
        TRY(tile_into(c, &L.w2_t, L.w2, dim, hid));
        L.tiled = true;
    }
    return VOX_OK;
}

// Allocate the multi-stream buffers once and (re)tile stale weights.
int ensure_batch(vox_ctx* c) {
    TRY(batch_supported(c));
    if (c->opt.vocab == 0 || !c->head_ready || !c->embed_ready)
        return fail(VOX_ERR_NOT_READY, "the multi-stream path needs the embedding and LM head");
    for (size_t l = 0; l < c->layers.size(); ++l)
        if (!c->layers[l].ready) return fail(VOX_ERR_NOT_READY, "layer %zu weights not uploaded", l);
    BatchBufs& b = c->bb;
    const int dim = (int)c->cfg.dim, hid = (int)c->cfg.hidden_dim, qd = (int)c->q_dim;
    const int vocab = (int)c->opt.vocab;
    if (!b.ready) {
        b.p_qkv = make_bgplan((int)c->qkv_rows, dim, c->num_sms);
        b.p_o = make_bgplan(dim, qd, c->num_sms);
        b.p_w13 = make_bgplan(2 * hid, dim, c->num_sms);
        b.p_w2 = make_bgplan(dim, hid, c->num_sms);
        b.p_head = make_bgplan(vocab, dim, c->num_sms);
        b.c_qkv = make_chain_plan((int)c->qkv_rows, dim, c->num_sms);
        b.c_o = make_chain_plan(dim, qd, c->num_sms);
        b.c_w13 = make_chain_plan(2 * hid, dim, c->num_sms);
        b.c_w2 = make_chain_plan(dim, hid, c->num_sms);
        b.c_head = make_chain_plan(vocab, dim, c->num_sms);
        b.n_done = (int)(c->layers.size() + 1) * kBgMaxPhases;
        CUDA_TRY(dalloc(&b.done, (size_t)b.n_done));
        CUDA_TRY(cudaMemset(b.done, 0, (size_t)b.n_done * sizeof(unsigned)));
        size_t part = 0, tiles = 0;
        for (const BgPlan* p : {&b.p_qkv, &b.p_o, &b.p_w13, &b.p_w2, &b.p_head, &b.c_qkv, &b.c_o, &b.c_w13,
                                &b.c_w2, &b.c_head}) {
            part = std::max(part, (size_t)p->tiles * p->splits * 128 * 8);
            tiles = std::max(tiles, (size_t)p->tiles);
        }
        const size_t nkv = c->cfg.n_kv_heads, hd = c->cfg.head_dim, G = c->cfg.n_heads / nkv;
        const size_t ns = (size_t)attn_max_splits();
        CUDA_TRY(dalloc(&b.hid, 8 * (size_t)dim));
        CUDA_TRY(dalloc(&b.hmid, 8 * (size_t)dim));
        CUDA_TRY(dalloc(&b.q, 8 * (size_t)qd));
        CUDA_TRY(dalloc(&b.attn, 8 * (size_t)qd));
        CUDA_TRY(dalloc(&b.act, 8 * (size_t)hid));
        CUDA_TRY(dalloc(&b.logits, 8 * (size_t)vocab));
        CUDA_TRY(dalloc(&b.ssp, 8 * (size_t)((dim + 127) / 128)));
        CUDA_TRY(dalloc(&b.part, part));
        CUDA_TRY(dalloc(&b.attn_part, 8 * nkv * ns * G * (hd + 2)));
        CUDA_TRY(dalloc(&b.am, 8 * (size_t)b.p_head.tiles));
        CUDA_TRY(dalloc(&b.tickets, tiles));
        CUDA_TRY(cudaMemset(b.tickets, 0, tiles * sizeof(unsigned)));
        CUDA_TRY(dalloc(&b.attn_tickets, 8 * nkv));
        CUDA_TRY(cudaMemset(b.attn_tickets, 0, 8 * nkv * sizeof(unsigned)));
        CUDA_TRY(cudaMemset(b.hid, 0, 8 * (size_t)dim * 4));
        CUDA_TRY(cudaMemset(b.hmid, 0, 8 * (size_t)dim * 4));
        CUDA_TRY(cudaMemset(b.attn, 0, 8 * (size_t)qd * 4));
        CUDA_TRY(cudaMemset(b.act, 0, 8 * (size_t)hid * 4));
        CUDA_TRY(cudaMemset(b.ssp, 0, 8 * (size_t)((dim + 127) / 128) * 4));
        CUDA_TRY(dalloc(&b.xop_a, xop_bytes(dim)));
        CUDA_TRY(dalloc(&b.xop_o, xop_bytes(qd)));
        CUDA_TRY(dalloc(&b.xop_f, xop_bytes(dim)));
        CUDA_TRY(dalloc(&b.xop_h, xop_bytes(hid)));
        for (unsigned char* x : {b.xop_a, b.xop_f}) CUDA_TRY(cudaMemset(x, 0, xop_bytes(dim)));
        CUDA_TRY(cudaMemset(b.xop_o, 0, xop_bytes(qd)));
        CUDA_TRY(cudaMemset(b.xop_h, 0, xop_bytes(hid)));
        CUDA_TRY(dalloc(&b.steps, 8));
        CUDA_TRY(cudaMemset(b.steps, 0, 8 * sizeof(StepState)));
        CUDA_TRY(dalloc(&b.tok_out, 8));
        CUDA_TRY(cudaMallocHost(&b.h_steps, 8 * sizeof(StepState)));
        b.ready = true;
    }
    TRY(tile_layers(c));
    if (!c->head_tiled) {
        TRY(tile_into(c, &c->head_t, c->lm_head, vocab, dim));
        c->head_tiled = true;
    }
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    return VOX_OK;
}

// ---- batched prefill (tensor-core GEMMs, vox_prefill.cu) ------------------------
// Shapes the batched prefill handles: bf16 weights, every K a multiple of 64,
// at most 4 q heads per kv head, head_dim 32, 64, 128 or 256.
bool prefill_batched_supported(const vox_ctx* c) {
    const vox_decoder_config& g = c->cfg;
    if (c->wsize != 2 || c->opt.vocab == 0) return false;
    if (g.dim % 64 || c->q_dim % 64 || g.hidden_dim % 64) return false;
    const size_t G = g.n_heads / g.n_kv_heads;
    if (G < 1 || G > 4) return false;
    return g.head_dim == 32 || g.head_dim == 64 || g.head_dim == 128 || g.head_dim == 256;
}

int ensure_prefill(vox_ctx* c) {
    PrefillBufs& f = c->pf;
    if (f.ready) return VOX_OK;
    const size_t T = kPrefillPass, dim = c->cfg.dim, qd = c->q_dim, kvd = c->kv_dim, hid = c->cfg.hidden_dim;
    const size_t kmax = std::max(std::max(dim, qd), hid);
    CUDA_TRY(dalloc(&f.h, T * dim));
    CUDA_TRY(dalloc(&f.q, T * qd));
    CUDA_TRY(dalloc(&f.kc, T * kvd));
    CUDA_TRY(dalloc(&f.vc, T * kvd));
    CUDA_TRY(dalloc(&f.attn, T * qd));
    CUDA_TRY(cudaMalloc(&f.xop, pf_xop_bytes((int)T, (int)kmax)));
    CUDA_TRY(cudaMalloc(&f.xop2, pf_xop_bytes((int)T, (int)kmax)));
    CUDA_TRY(dalloc(&f.tokens, T));
    CUDA_TRY(dalloc(&f.ssp, T * ((dim + 511) / 512)));
    CUDA_TRY(cudaMallocHost(&f.h_tokens, T * sizeof(int32_t)));
    f.ready = true;
    return VOX_OK;
}

// Grow-only device scratch (the stream is drained before a buffer is replaced).
int ensure_scratch(vox_ctx* c, float** buf, size_t* have, size_t floats) {
    if (floats <= *have) return VOX_OK;
    if (*buf) {
        CUDA_TRY(cudaStreamSynchronize(c->stream));
        cudaFree(*buf);
        *buf = nullptr;
        *have = 0;
    }
    CUDA_TRY(dalloc(buf, floats));
    *have = floats;
    return VOX_OK;
}

// Hidden rows of the pass (embedding or residual) and their RMSNorm into the
// prefill operand of the next linear.
int enqueue_pf_norm(vox_ctx* c, PfNormArgs a) {
    a.h = c->pf.h;
    a.ssp = c->pf.ssp;
    a.ssp_chunks = ((int)c->cfg.dim + 511) / 512;
    a.dim = (int)c->cfg.dim;
    a.eps = c->cfg.norm_eps;
    a.xop = c->pf.xop;
    a.err = c->err;
    CUDA_TRY(record_launch(c, launch_pf_resid(a, c->stream)));
    CUDA_TRY(record_launch(c, launch_pf_norm_xop(a, c->stream)));
    return VOX_OK;
}

int enqueue_pf_gemm(vox_ctx* c, const PfPlan& p, const unsigned char* wt, int tn, int nblocks, int T,
                    float* act = nullptr, unsigned char* xop_out = nullptr, const unsigned char* xop = nullptr) {
    PfGemmArgs a{};
    a.wt = wt;
    a.xop = xop ? xop : c->pf.xop;
    a.part = c->pf.part;
    a.act = act;
    a.xop_out = xop_out;
    a.rows = p.rows;
    a.kbt = p.kbt;
    a.tiles = p.tiles;
    a.tn = tn;
    a.nblocks = nblocks;
    a.T = T;
    a.splits = p.splits;
    a.err = c->err;
    CUDA_TRY(record_launch(c, launch_pf_gemm(a, p.grid, p.wide, c->stream)));
    return VOX_OK;
}

// Prefill of tokens[0..n) at positions pos0.. through every layer, one pass
// of up to kPrefillPass tokens at a time (decoder.rs:88-155 for each token,
// kv.rs:48-88 appends in token order).  With `adapter` the first layer's
// input of position p is adapter[p mod adapter_cap] + widen(embed[token]).
// The last layer's attention output, o-proj and FFN feed only the logits,
// which a prefill discards, so they are not computed.  Synchronises once.
int prefill_batched(vox_ctx* c, vox_kv* kv, const int32_t* tokens, size_t n, size_t pos0, const float* adapter,
                    int adapter_cap) {
    TRY(tile_layers(c));
    TRY(ensure_prefill(c));
    PrefillBufs& f = c->pf;
    const vox_decoder_config& g = c->cfg;
    const int dim = (int)g.dim, qd = (int)c->q_dim, kvd = (int)c->kv_dim, hid = (int)g.hidden_dim;
    const int rows_qkv = qd + 2 * kvd;
    const size_t nl = c->layers.size();
    int win = (int)kv->window;
    if (g.sliding_window > 0) win = std::min(win, (int)g.sliding_window);
    for (size_t i0 = 0; i0 < n; i0 += kPrefillPass) {
        const int T = (int)std::min<size_t>(kPrefillPass, n - i0);
        const int tn = T >= 128 ? 128 : (T + 15) / 16 * 16;
        const int nblocks = (T + tn - 1) / tn, Tp = nblocks * tn;
        const PfPlan pq = make_pfplan(rows_qkv, dim, nblocks, tn, c->num_sms);
        const PfPlan po = make_pfplan(dim, qd, nblocks, tn, c->num_sms);
        const PfPlan p13 = make_pfplan(2 * hid, dim, nblocks, tn, c->num_sms, true);
        const PfPlan p2 = make_pfplan(dim, hid, nblocks, tn, c->num_sms);
        size_t part = 0;
        for (const PfPlan* p : {&pq, &po, &p13, &p2}) part = std::max(part, (size_t)p->splits * T * p->rows);
        TRY(ensure_scratch(c, &f.part, &f.part_floats, part));
        // the staging buffer is reused: the previous pass's copy must be done
        CUDA_TRY(cudaStreamSynchronize(c->stream));
        std::memcpy(f.h_tokens, tokens + i0, (size_t)T * sizeof(int32_t));
        CUDA_TRY(cudaMemcpyAsync(f.tokens, f.h_tokens, (size_t)T * sizeof(int32_t), cudaMemcpyHostToDevice,
                                 c->stream));
        const long long p0 = (long long)(pos0 + i0);

        PfNormArgs na{};
        na.embed = c->embed;
        na.tokens = f.tokens;
        na.vocab = (int)c->opt.vocab;
        na.adapter = adapter;
        na.adapter_cap = adapter_cap;
        na.pos0 = p0;
        na.gain = c->layers[0].attn_norm;
        na.tn = tn;
        na.T = T;
        na.Tp = Tp;
        TRY(enqueue_pf_norm(c, na));

        for (size_t l = 0; l < nl; ++l) {
            const LayerDev& L = c->layers[l];
            const bool last = l + 1 == nl;
            float* kr = kv->k + l * kv->layer_elems();
            float* vr = kv->v + l * kv->layer_elems();
            // 1) q|k|v for every token, RoPE at its position
            TRY(enqueue_pf_gemm(c, pq, L.wqkv_t, tn, nblocks, T));
            PfQkvArgs qa{};
            qa.part = f.part;
            qa.splits = pq.splits;
            qa.T = T;
            qa.q_dim = qd;
            qa.kv_dim = kvd;
            qa.head_dim = (int)g.head_dim;
            qa.rope_cos = c->rope_cos;
            qa.rope_sin = c->rope_sin;
            qa.max_pos = c->max_pos;
            qa.pos0 = p0;
            qa.q = f.q;
            qa.kc = f.kc;
            qa.vc = f.vc;
            qa.err = c->err;
            CUDA_TRY(record_launch(c, launch_pf_qkv(qa, c->stream)));
            HostKv& hs = kv->hs[l];
            // 2) causal attention over the cache before the pass + the pass
            if (!last) {
                PfAttnArgs aa{};
                aa.q = f.q;
                aa.kc_in = f.kc;
                aa.vc_in = f.vc;
                aa.k_ring = kr;
                aa.v_ring = vr;
                aa.T = T;
                aa.n_heads = (int)g.n_heads;
                aa.n_kv = (int)g.n_kv_heads;
                aa.head_dim = (int)g.head_dim;
                aa.cap = (int)kv->cap;
                aa.len0 = (int)hs.len;
                aa.start0 = (int)hs.start;
                aa.win = win;
                // tensor-core blocks of 32 tokens (4 q heads per kv head, head_dim
                // 128), else CUDA-core blocks of 16; chunks of >= 128 keys.  The
                // tensor-core kernel takes one chunk per block when the blocks x kv
                // heads fill 3/4 of the SMs (prompts of 512 / 4096 tokens: 6.90 /
                // 76.7 ms against 7.48-7.73 / 83.7-87.1 ms with 2, 4 or 8 chunks per
                // block, which also need the merge), else enough
                // chunks to cover the SMs (at most 8); the CUDA-core kernel about 8.
                const bool tc = pf_attn_tc_supported(aa.n_heads, aa.n_kv, aa.head_dim);
                aa.qb = tc ? 32 : 16;
                const int span = std::min((int)hs.len + T, win) + aa.qb - 1, kt = tc ? 64 : 32;
                const int units = (T + aa.qb - 1) / aa.qb * aa.n_kv, sms = c->num_sms;
                const int per = !tc ? 8 : 4 * units >= 3 * sms ? 1 : std::min(8, (sms + units - 1) / units);
                aa.kc = std::max(128, ((span + per - 1) / per + kt - 1) / kt * kt);
                aa.cmax = pf_attn_cmax(T, aa.len0, win, aa.kc, aa.qb);
                aa.err = c->err;
                TRY(ensure_scratch(c, &f.attn_part, &f.attn_part_floats,
                                   pf_attn_part_floats(T, aa.n_kv, aa.head_dim, aa.cmax, aa.qb)));
                aa.part = f.attn_part;
                aa.scale = 1.0f / sqrtf((float)g.head_dim);
                aa.out = f.attn;
                // the tensor-core kernel with a single chunk per block writes the
                // normalised rows straight into the o-proj's operand (the q|k|v
                // GEMM that read the operand buffer before has finished)
                const bool direct = tc && aa.cmax == 1;
                if (direct) {
                    aa.xop = f.xop;
                    aa.xop_tn = tn;
                }
                if (tc) {
                    // the keys and values it reads, once, as 64-key operand tiles
                    // from the pass's first visible key rounded down to 64
                    const int first = aa.len0 + 1 - std::min(aa.len0 + 1, win);
                    aa.kv_base = first / 64 * 64;
                    aa.kv_tiles = (aa.len0 + T - 1 - aa.kv_base) / 64 + 1;
                    TRY(ensure_scratch(c, &f.kvop, &f.kvop_floats,
                                       (size_t)aa.n_kv * aa.kv_tiles * pf_kv_tile_bytes() / sizeof(float)));
                    aa.kvop = reinterpret_cast<unsigned char*>(f.kvop);
                    CUDA_TRY(record_launch(c, launch_pf_kv_tiles(aa, c->stream)));
                }
                CUDA_TRY(record_launch(c, tc ? launch_pf_attn_tc(aa, c->stream) : launch_pf_attn(aa, c->stream)));
                if (!direct) {
                    CUDA_TRY(record_launch(c, launch_pf_attn_merge(aa, c->stream)));
                    CUDA_TRY(record_launch(c, launch_pf_split(f.attn, T, Tp, qd, f.xop, tn, c->stream)));
                }
            }
            // 3) the pass's keys and values into the ring, state after T appends
            PfCommitArgs ca{};
            ca.kc = f.kc;
            ca.vc = f.vc;
            ca.k_ring = kr;
            ca.v_ring = vr;
            ca.T = T;
            ca.kv_dim = kvd;
            ca.head_dim = (int)g.head_dim;
            ca.cap = (int)kv->cap;
            ca.end0 = (long long)((hs.start + hs.len) % kv->cap);
            ca.state = kv->dstate + l;
            for (int t = 0; t < T; ++t) host_append(hs, 1, kv->window, kv->cap);
            ca.final_state.len = (int32_t)hs.len;
            ca.final_state.start = (int32_t)hs.start;
            ca.final_state.pos_offset = (int64_t)hs.pos_offset;
            CUDA_TRY(record_launch(c, launch_pf_commit(ca, c->stream)));
            if (last) break;
            // 4) o-proj + residual, RMSNorm -> w1|w3 -> SwiGLU -> w2 + residual
            TRY(enqueue_pf_gemm(c, po, L.wo_t, tn, nblocks, T));
            na = PfNormArgs{};
            na.part = f.part;
            na.splits = po.splits;
            na.gain = L.ffn_norm;
            na.tn = tn;
            na.T = T;
            na.Tp = Tp;
            TRY(enqueue_pf_norm(c, na));
            const unsigned char* w2_xop = f.xop;
            if (p13.splits == 1 && p13.wide) {
                // SwiGLU in the GEMM epilogue straight into the w2 operand, a second
                // buffer (other CTAs still read the w1|w3 operand from the first)
                TRY(enqueue_pf_gemm(c, p13, L.w13_t, tn, nblocks, T, f.part, f.xop2));
                w2_xop = f.xop2;
            } else if (p13.splits == 1) {  // SwiGLU in the GEMM epilogue, then the w2 operand
                TRY(enqueue_pf_gemm(c, p13, L.w13_t, tn, nblocks, T, f.part));
                CUDA_TRY(record_launch(c, launch_pf_split(f.part, T, Tp, hid, f.xop, tn, c->stream)));
            } else {
                TRY(enqueue_pf_gemm(c, p13, L.w13_t, tn, nblocks, T));
                CUDA_TRY(record_launch(c, launch_pf_swiglu(f.part, p13.splits, T, Tp, hid, f.xop, tn, c->stream)));
            }
            TRY(enqueue_pf_gemm(c, p2, L.w2_t, tn, nblocks, T, nullptr, nullptr, w2_xop));
            na.splits = p2.splits;
            na.gain = c->layers[l + 1].attn_norm;
            TRY(enqueue_pf_norm(c, na));
        }
    }
    return check_device_errors(c);
}

BgArgs bg_args(vox_ctx* c, const BgPlan& p, const unsigned char* wt, int B, int epi) {
    BgArgs a{};
    a.wt = wt;
    a.rows = p.rows;
    a.K = p.K;
    a.tiles = p.tiles;
    a.kbt = p.kbt;
    a.splits = p.splits;
    a.B = B;
    a.xslab_bytes = p.xslab;
    a.eps = c->cfg.norm_eps;
    a.epi = epi;
    a.part = c->bb.part;
    a.tickets = c->bb.tickets;
    a.err = c->err;
    a.ssp_parts = (int)((c->cfg.dim + 127) / 128);
    return a;
}

// One token for each of the B streams of `kv`: embed, 26 x (QKV + RoPE + ring
// append, attention, o-proj + residual + append commit, w1|w3 + SwiGLU, w2 +
// residual), final RMSNorm + LM head + per-stream argmax.  The GEMMs read
// each weight once for all streams.
int enqueue_batch_step(vox_ctx* c, vox_kv* kv, bool pdl) {
    BatchBufs& bb = c->bb;
    const int B = (int)kv->n_streams;
    const int dim = (int)c->cfg.dim, hid = (int)c->cfg.hidden_dim, qd = (int)c->q_dim;
    const long long ring_stride = (long long)kv->stream_elems();
    const int cap = (int)kv->cap, win = (int)kv->window;
    const int nkv = (int)c->cfg.n_kv_heads, hd = (int)c->cfg.head_dim, G = (int)(c->cfg.n_heads / nkv);
    const int nsplit = attn_max_splits();  // chunks per (stream, kv head) at most
    CUDA_TRY(record_launch(c, launch_bg_embed(c->embed, (int)c->opt.vocab, dim, bb.steps, B, bb.hid, bb.ssp,
                                              bb.xop_a, c->layers[0].attn_norm, bb.done, bb.n_done, c->err,
                                              c->stream, pdl)));
    const int L = (int)c->layers.size();
    // VOX_STEP_PERSISTENT: o-proj, w1|w3, w2 and the next q|k|v (or the LM
    // head) run as one persistent chain launch; otherwise (and by default,
    // about 3% faster on B200) one launch per GEMM.
    const bool chained = c->opt.step_mode == VOX_STEP_PERSISTENT;
    const BgPlan& P_qkv = chained ? bb.c_qkv : bb.p_qkv;
    const BgPlan& P_o = chained ? bb.c_o : bb.p_o;
    const BgPlan& P_w13 = chained ? bb.c_w13 : bb.p_w13;
    const BgPlan& P_w2 = chained ? bb.c_w2 : bb.p_w2;
    const BgPlan& P_head = chained ? bb.c_head : bb.p_head;
    auto launch_chain = [&](BgChain& ch, const BgPlan* const* plans) -> int {
        if (chained) {
            ch.xslab_bytes = 0;
            for (int p = 0; p < ch.n_phases; ++p) ch.xslab_bytes = std::max(ch.xslab_bytes, ch.ph[p].xslab_bytes);
            CUDA_TRY(record_launch(c, launch_bgemm(ch, c->num_sms, c->stream, pdl)));
            return VOX_OK;
        }
        for (int p = 0; p < ch.n_phases; ++p)
            CUDA_TRY(record_launch(c, launch_bgemm(chain_of(ch.ph[p], *plans[p]), plans[p]->grid, c->stream, pdl)));
        return VOX_OK;
    };
    auto qkv_args = [&](int l) {
        const LayerDev& Ld = c->layers[l];
        BgArgs a = bg_args(c, P_qkv, Ld.wqkv_t, B, BG_QKV);
        a.xop = bb.xop_a;  // hid * attn_norm, written by the embedding or the previous w2
        a.norm_w = Ld.attn_norm;
        a.ssp = bb.ssp;
        a.y = bb.q;
        a.y_stride = qd;
        a.q_dim = qd;
        a.kv_dim = (int)c->kv_dim;
        a.head_dim = hd;
        a.rope_cos = c->rope_cos;
        a.rope_sin = c->rope_sin;
        a.max_pos = c->max_pos;
        a.steps = bb.steps;
        a.kv_state = kv->dstate + l;
        a.kv_state_stride = (long long)kv->n_layers;
        a.k_ring = kv->k + (size_t)l * kv->layer_elems();
        a.v_ring = kv->v + (size_t)l * kv->layer_elems();
        a.ring_stride = ring_stride;
        a.ring_cap = cap;
        a.kv_window = win;
        return a;
    };
    // chain 0: q|k|v of layer 0
    {
        BgChain ch = chain_of(qkv_args(0), P_qkv);
        ch.done = bb.done;
        const BgPlan* plans[1] = {&P_qkv};
        TRY(launch_chain(ch, plans));
    }
    for (int l = 0; l < L; ++l) {
        const LayerDev& Ld = c->layers[l];
        float* kr = kv->k + (size_t)l * kv->layer_elems();
        float* vr = kv->v + (size_t)l * kv->layer_elems();
        KvState* st = kv->dstate + l;

        AttnArgs at{};
        at.q = bb.q;
        at.k_ring = kr;
        at.v_ring = vr;
        at.n_heads = (int)c->cfg.n_heads;
        at.n_kv = nkv;
        at.hd = hd;
        at.cap = cap;
        at.cfg_window = (int)c->cfg.sliding_window;
        at.st = st;
        at.pre_append = 1;
        at.kv_window = win;
        at.nsplit = nsplit;
        at.part = bb.attn_part;
        at.tickets = bb.attn_tickets;
        at.out = bb.attn;
        at.scale = 1.0f / sqrtf((float)hd);
        at.err = c->err;
        at.n_streams = B;
        at.q_stride = qd;
        at.ring_stride = ring_stride;
        at.out_stride = qd;
        at.part_stride = (long long)nkv * nsplit * G * (hd + 2);
        at.st_stride = (long long)kv->n_layers;
        at.xop = bb.xop_o;
        CUDA_TRY(record_launch(c, launch_attention(at, c->stream, pdl)));

        // chain l + 1: o-proj + residual (commits the append), w1|w3 + SwiGLU,
        // w2 + residual, then layer l + 1's q|k|v or the LM head.
        BgChain ch{};
        ch.n_phases = 4;
        ch.done = bb.done + (size_t)(l + 1) * kBgMaxPhases;
        BgArgs a = bg_args(c, P_o, Ld.wo_t, B, BG_RESID);
        a.xop = bb.xop_o;
        a.y = bb.hmid;
        a.y_stride = dim;
        a.resid = bb.hid;
        a.ssp_out = bb.ssp;
        a.xop_out = bb.xop_f;
        a.xop_gain = Ld.ffn_norm;
        a.kv_commit = st;
        a.kv_state_stride = (long long)kv->n_layers;
        a.kv_window = win;
        a.ring_cap = cap;
        ch.ph[0] = a;

        a = bg_args(c, P_w13, Ld.w13_t, B, BG_SWIGLU);
        a.xop = bb.xop_f;
        a.norm_w = Ld.ffn_norm;
        a.ssp = bb.ssp;
        a.y = bb.act;
        a.y_stride = hid;
        a.xop_out = bb.xop_h;
        ch.ph[1] = a;

        a = bg_args(c, P_w2, Ld.w2_t, B, BG_RESID);
        a.xop = bb.xop_h;
        a.y = bb.hid;
        a.y_stride = dim;
        a.resid = bb.hmid;
        a.ssp_out = bb.ssp;
        a.xop_out = bb.xop_a;  // the next q|k|v's (or the LM head's) operand
        a.xop_gain = l + 1 < L ? c->layers[l + 1].attn_norm : c->final_norm;
        ch.ph[2] = a;

        if (l + 1 < L) {
            ch.ph[3] = qkv_args(l + 1);
        } else {
            a = bg_args(c, P_head, c->head_t, B, BG_ARGMAX);
            a.xop = bb.xop_a;
            a.norm_w = c->final_norm;
            a.ssp = bb.ssp;
            a.y = bb.logits;
            a.y_stride = (long long)c->opt.vocab;
            a.am_part = bb.am;
            ch.ph[3] = a;
        }
        const BgPlan* plans[4] = {&P_o, &P_w13, &P_w2, l + 1 < L ? &P_qkv : &P_head};
        TRY(launch_chain(ch, plans));
    }
    CUDA_TRY(record_launch(c, launch_bg_argmax_final(bb.am, P_head.tiles, bb.steps, B, bb.tok_out, c->stream,
                                                     pdl)));
    return VOX_OK;
}

int build_batch_graph(vox_ctx* c, vox_kv* kv) {
    if (kv->batch_graph) return VOX_OK;
    const uint64_t before = c->launches;
    CUDA_TRY(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_batch_step(c, kv, true);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(c->stream, &g);
    if (rc != VOX_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    CUDA_TRY(e);
    e = cudaGraphInstantiate(&kv->batch_graph, g, 0);
    cudaGraphDestroy(g);
    CUDA_TRY(e);
    kv->batch_kernels = c->launches - before;
    c->launches = before;
    return VOX_OK;
}

int model_ready(vox_ctx* c, vox_kv* kv) {
    if (!c || !kv) return fail(VOX_ERR_INVALID_ARG, "null context or cache");
    if (kv->ctx != c) return fail(VOX_ERR_INVALID_ARG, "cache belongs to another context");
    if (c->opt.vocab == 0) return fail(VOX_ERR_NOT_READY, "context was created without a vocabulary");
    if (!c->embed_ready || !c->head_ready) return fail(VOX_ERR_NOT_READY, "embedding or LM head not uploaded");
    for (size_t l = 0; l < c->layers.size(); ++l)
        if (!c->layers[l].ready) return fail(VOX_ERR_NOT_READY, "layer %zu weights not uploaded", l);
    if (kv->n_layers != c->layers.size())
        return fail(VOX_ERR_SHAPE, "cache has %zu layers, model has %zu", kv->n_layers, c->layers.size());
    if (kv->n_kv != c->cfg.n_kv_heads || kv->hd != c->cfg.head_dim)
        return fail(VOX_ERR_SHAPE, "cache head shape does not match the decoder config");
    return VOX_OK;
}

// One token step as a CUDA graph.  Single-stream steps get two graphs when
// the shape allows: attention as one cluster per kv head (contexts up to
// attn_cluster_max_tokens()) or the persistent split-K kernel; launch_graph
// picks one per step from the context length the host already knows.
static int capture_step(vox_ctx* c, vox_kv* kv, bool short_attn, cudaGraphExec_t* out, uint64_t* kernels,
                        const float* adapter = nullptr, int adapter_cap = 0) {
    const uint64_t before = c->launches;
    CUDA_TRY(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    int rc = VOX_OK;
    for (size_t l = 0; l < c->layers.size() && rc == VOX_OK; ++l)
        rc = enqueue_layer(c, kv, l, l == 0, true, short_attn, adapter, adapter_cap);
    if (rc == VOX_OK) rc = enqueue_head(c, true);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(c->stream, &g);
    if (rc != VOX_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    CUDA_TRY(e);
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    CUDA_TRY(e);
    *kernels = c->launches - before;
    c->launches = before;
    return VOX_OK;
}

int build_step_graph(vox_ctx* c, vox_kv* kv) {
    if (kv->step_graph) return VOX_OK;
    TRY(capture_step(c, kv, false, &kv->step_graph, &kv->graph_kernels));
    if (attn_cluster_size((int)c->cfg.n_heads, (int)c->cfg.n_kv_heads, (int)c->cfg.head_dim) > 0)
        TRY(capture_step(c, kv, true, &kv->step_graph_short, &kv->graph_kernels_short));
    return VOX_OK;
}

int ensure_host_steps(vox_ctx* c, size_t n) {
    if (n <= c->h_steps_cap) return VOX_OK;
    if (c->h_steps) {
        CUDA_TRY(cudaStreamSynchronize(c->stream));
        cudaFreeHost(c->h_steps);
        c->h_steps = nullptr;
    }
    size_t cap = 1024;
    while (cap < n) cap <<= 1;
    CUDA_TRY(cudaMallocHost(&c->h_steps, cap * sizeof(StepState)));
    c->h_steps_cap = cap;
    return VOX_OK;
}

// Live tokens the attention of every layer reads after `steps` more
// single-token appends (kv.rs:48-88 eviction, then the config's window mask).
size_t live_tokens_after(const vox_ctx* c, const vox_kv* kv, size_t steps) {
    size_t n = 0;
    for (size_t l = 0; l < kv->n_layers; ++l) n = std::max(n, kv->hs[l].len);
    n = std::min(n + steps, kv->window);
    if (c->cfg.sliding_window > 0) n = std::min(n, (size_t)c->cfg.sliding_window);
    return n;
}

// `live` = live tokens of this step's attention (after its append).
int launch_graph(vox_ctx* c, vox_kv* kv, size_t live) {
    const bool use_short = kv->step_graph_short && live <= (size_t)attn_cluster_max_tokens();
    CUDA_TRY(cudaGraphLaunch(use_short ? kv->step_graph_short : kv->step_graph, c->stream));
    c->launches += use_short ? kv->graph_kernels_short : kv->graph_kernels;
    return VOX_OK;
}

void mirror_single_append_all(vox_kv* kv) {
    for (size_t l = 0; l < kv->n_layers; ++l) host_append(kv->hs[l], 1, kv->window, kv->cap);
}

int upload_state(vox_kv* kv, size_t layer) {
    KvState d{};
    d.len = (int32_t)kv->hs[layer].len;
    d.start = (int32_t)kv->hs[layer].start;
    d.pos_offset = (int64_t)kv->hs[layer].pos_offset;
    CUDA_TRY(cudaMemcpyAsync(kv->dstate + layer, &d, sizeof d, cudaMemcpyHostToDevice, kv->ctx->stream));
    CUDA_TRY(cudaStreamSynchronize(kv->ctx->stream));
    return VOX_OK;
}

}  // namespace

namespace {

// Upload n floats, run `fn` on the device copy, download back into `io`.
template <class F>
int inplace_op(vox_ctx* c, float* io, size_t n, F fn) {
    if (!c || (!io && n)) return fail(VOX_ERR_INVALID_ARG, "null argument");
    if (n == 0) return VOX_OK;
    CUDA_TRY(cudaSetDevice(c->dev));
    TRY(ensure_scratch(c, n * 4));
    float* d = static_cast<float*>(c->scratch);
    CUDA_TRY(cudaMemcpyAsync(d, io, n * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(record_launch(c, fn(d)));
    CUDA_TRY(cudaMemcpyAsync(io, d, n * 4, cudaMemcpyDeviceToHost, c->stream));
    return check_device_errors(c);
}

}  // namespace

// ============================================================================
// C ABI
// ============================================================================
extern "C" {

const char* vox_last_error(void) { return g_err.c_str(); }
int vox_abi_version(void) { return VOX_ABI_VERSION; }

int vox_config_validate(const vox_decoder_config* cfg) { return validate_cfg(cfg); }

int vox_layer_weights_validate_f32(const vox_decoder_config* cfg, const vox_layer_weights_f32* w) {
    TRY(validate_cfg(cfg));
    return validate_weights(cfg, w);
}
int vox_layer_weights_validate_bf16(const vox_decoder_config* cfg, const vox_layer_weights_bf16* w) {
    TRY(validate_cfg(cfg));
    return validate_weights(cfg, w);
}

void vox_ctx_destroy(vox_ctx* c) {
    if (!c) return;
    cudaSetDevice(c->dev);
    if (c->stream) cudaStreamSynchronize(c->stream);
    while (!c->caches.empty()) vox_kv_destroy(c->caches.back());
    for (auto& L : c->layers) {
        cudaFree(L.wqkv_t);
        cudaFree(L.wo_t);
        cudaFree(L.w13_t);
        cudaFree(L.w2_t);
        cudaFree(L.wqkv);
        cudaFree(L.wo);
        cudaFree(L.w13);
        cudaFree(L.w2);
        cudaFree(L.attn_norm);
        cudaFree(L.ffn_norm);
    }
    void* ptrs[] = {c->embed, c->lm_head, c->final_norm, c->rope_cos, c->rope_sin, c->hid, c->hmid,
                    c->q, c->attn, c->act, c->logits, c->am_part, c->attn_part, c->tickets, c->step,
                    c->tok_out, c->err, c->scratch};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    {
        BatchBufs& b = c->bb;
        void* bp[] = {c->head_t, b.hid, b.hmid, b.q, b.attn, b.act, b.logits, b.ssp, b.part, b.attn_part, b.am,
                      b.tickets, b.attn_tickets, b.steps, b.tok_out, b.done, b.xop_a, b.xop_o, b.xop_f, b.xop_h};
        for (void* p : bp)
            if (p) cudaFree(p);
        if (b.h_steps) cudaFreeHost(b.h_steps);
        if (b.h_tok) cudaFreeHost(b.h_tok);
    }
    {
        PrefillBufs& f = c->pf;
        void* fp[] = {f.h, f.q, f.kc, f.vc, f.attn, f.part, f.xop, f.xop2, f.tokens, f.ssp, f.attn_part, f.kvop};
        for (void* p : fp)
            if (p) cudaFree(p);
        if (f.h_tokens) cudaFreeHost(f.h_tokens);
    }
    if (c->h_steps) cudaFreeHost(c->h_steps);
    if (c->h_tok) cudaFreeHost(c->h_tok);
    if (c->h_err) cudaFreeHost(c->h_err);
    for (auto& e : c->ev)
        if (e) cudaEventDestroy(e);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

int vox_ctx_create(const vox_decoder_config* cfg, const vox_ctx_options* opt, vox_ctx** out) {
    if (!out) return fail(VOX_ERR_INVALID_ARG, "out is null");
    *out = nullptr;
    TRY(validate_cfg(cfg));
    vox_ctx_options o{};
    if (opt) o = *opt;
    if (o.n_layers == 0) o.n_layers = 1;
    if (o.max_positions == 0) o.max_positions = 32768;
    if (o.step_mode < VOX_STEP_AUTO || o.step_mode > VOX_STEP_PERSISTENT)
        return fail(VOX_ERR_INVALID_ARG, "unknown step mode %d", o.step_mode);
    if (o.weight_dtype != VOX_WEIGHTS_BF16 && o.weight_dtype != VOX_WEIGHTS_F32)
        return fail(VOX_ERR_INVALID_ARG, "unknown weight dtype %d", o.weight_dtype);
    const int wsize = o.weight_dtype == VOX_WEIGHTS_F32 ? 4 : 2;
    TRY(check_kernel_shapes(cfg, wsize));
    if (o.vocab > (size_t)INT32_MAX) return fail(VOX_ERR_UNSUPPORTED, "vocab too large");
    if (o.max_positions > (size_t)(1 << 24))
        return fail(VOX_ERR_UNSUPPORTED, "max_positions above 2^24 (positions are exact f32)");

    int ndev = 0;
    CUDA_TRY(cudaGetDeviceCount(&ndev));
    if (o.device < 0 || o.device >= ndev) return fail(VOX_ERR_INVALID_ARG, "device %d not present", o.device);
    CUDA_TRY(cudaSetDevice(o.device));
    cudaDeviceProp prop;
    CUDA_TRY(cudaGetDeviceProperties(&prop, o.device));
    if (prop.major != 10)
        return fail(VOX_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", o.device,
                    prop.major, prop.minor);

    vox_ctx* c = new vox_ctx();
    c->cfg = *cfg;
    c->opt = o;
    c->dev = o.device;
    c->num_sms = prop.multiProcessorCount;
    c->wsize = wsize;
    c->q_dim = cfg->n_heads * cfg->head_dim;
    c->kv_dim = cfg->n_kv_heads * cfg->head_dim;
    c->qkv_rows = c->q_dim + 2 * c->kv_dim;
    c->layers.resize(o.n_layers);
    c->max_pos = (int)o.max_positions;

    auto bail = [&](int rc) {
        vox_ctx_destroy(c);
        return rc;
    };
#define CTX_TRY(expr)                                                                        \
    do {                                                                                     \
        cudaError_t e_ = (expr);                                                             \
        if (e_ != cudaSuccess)                                                               \
            return bail(fail(e_ == cudaErrorMemoryAllocation ? VOX_ERR_OOM : VOX_ERR_CUDA,    \
                             "%s failed: %s", #expr, cudaGetErrorString(e_)));                \
    } while (0)

    CTX_TRY(gemv_prepare(c->dev));
    CTX_TRY(attn_prepare(c->dev));
    CTX_TRY(bgemm_prepare(c->dev));
    CTX_TRY(pf_prepare());
    CTX_TRY(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    for (auto& e : c->ev) CTX_TRY(cudaEventCreate(&e));

    const size_t dim = cfg->dim, hid = cfg->hidden_dim, hd = cfg->head_dim;
    // Launch plans.
    const int dimi = (int)dim, hidi = (int)hid;
    c->p_qkv = plan_gemv((int)c->qkv_rows, dimi, 2, wsize, c->num_sms, 1, kGemvPaired);
    c->p_o = plan_gemv(dimi, (int)c->q_dim, 1, wsize, c->num_sms, 1, kGemvLean);
    c->p_w13 = plan_gemv(2 * hidi, dimi, 2, wsize, c->num_sms, 1, kGemvPaired);
    c->p_w2 = plan_gemv(dimi, hidi, 1, wsize, c->num_sms, 1, kGemvPaired);
    if (o.vocab) c->p_head = plan_gemv((int)o.vocab, dimi, 1, wsize, c->num_sms, 1, kGemvPaired);
    for (const GemvPlan* p : {&c->p_qkv, &c->p_o, &c->p_w13, &c->p_w2})
        if (p->grid < 1 || p->smem > gemv_max_smem())
            return bail(fail(VOX_ERR_UNSUPPORTED, "no GEMV plan for rows %d x K %d", p->rows, p->K));
    if (o.vocab && (c->p_head.grid < 1 || c->p_head.smem > gemv_max_smem()))
        return bail(fail(VOX_ERR_UNSUPPORTED, "no LM-head plan for vocab %zu", (size_t)o.vocab));
    c->nsplit = attn_max_splits();

    // Activations and scratch.
    CTX_TRY(dalloc(&c->hid, dim));
    CTX_TRY(dalloc(&c->hmid, dim));
    CTX_TRY(dalloc(&c->q, c->q_dim));
    CTX_TRY(dalloc(&c->attn, c->q_dim));
    CTX_TRY(dalloc(&c->act, hid));
    CTX_TRY(dalloc(&c->logits, o.vocab));
    CTX_TRY(dalloc(&c->am_part, (size_t)c->num_sms));
    const size_t G = cfg->n_heads / cfg->n_kv_heads;
    CTX_TRY(dalloc(&c->attn_part, cfg->n_kv_heads * c->nsplit * G * (hd + 2)));
    CTX_TRY(dalloc(&c->tickets, cfg->n_kv_heads));
    CTX_TRY(cudaMemset(c->tickets, 0, cfg->n_kv_heads * sizeof(unsigned)));
    CTX_TRY(dalloc(&c->step, 1));
    CTX_TRY(cudaMemset(c->step, 0, sizeof(StepState)));
    CTX_TRY(dalloc(&c->tok_out, 1));
    CTX_TRY(dalloc(&c->err, 1));
    CTX_TRY(cudaMemset(c->err, 0, sizeof(unsigned)));
    CTX_TRY(cudaMallocHost(&c->h_tok, sizeof(int32_t)));
    CTX_TRY(cudaMallocHost(&c->h_err, sizeof(unsigned)));
    if (ensure_host_steps(c, 1024) != VOX_OK) return bail(VOX_ERR_OOM);

    // RoPE table: inv_freq = theta^(-(2p)/hd), angle = pos * inv_freq,
    // (sin, cos) of angle, all in f32 with libm as math.rs:52-56 does.
    {
        const size_t half = hd / 2, n = (size_t)c->max_pos * half;
        std::vector<float> ct(n), st(n), inv(half);
        for (size_t p = 0; p < half; ++p)
            inv[p] = powf(cfg->rope_theta, -((float)(2 * p)) / (float)hd);
        for (size_t pos = 0; pos < (size_t)c->max_pos; ++pos)
            for (size_t p = 0; p < half; ++p) {
                const float angle = (float)pos * inv[p];
                st[pos * half + p] = sinf(angle);
                ct[pos * half + p] = cosf(angle);
            }
        CTX_TRY(dalloc(&c->rope_cos, n));
        CTX_TRY(dalloc(&c->rope_sin, n));
        CTX_TRY(cudaMemcpy(c->rope_cos, ct.data(), n * 4, cudaMemcpyHostToDevice));
        CTX_TRY(cudaMemcpy(c->rope_sin, st.data(), n * 4, cudaMemcpyHostToDevice));
    }
#undef CTX_TRY
    *out = c;
    return VOX_OK;
}

int vox_ctx_upload_layer_f32(vox_ctx* c, size_t layer, const vox_layer_weights_f32* w) {
    return upload_layer(c, layer, w);
}
int vox_ctx_upload_layer_bf16(vox_ctx* c, size_t layer, const vox_layer_weights_bf16* w) {
    return upload_layer(c, layer, w);
}

int vox_ctx_upload_embed_bf16(vox_ctx* c, const uint16_t* embed, size_t len) {
    if (!c || !embed) return fail(VOX_ERR_INVALID_ARG, "null argument");
    if (c->opt.vocab == 0) return fail(VOX_ERR_NOT_READY, "context was created without a vocabulary");
    if (len != c->opt.vocab * c->cfg.dim) return fail(VOX_ERR_SHAPE, "embed shape mismatch");
    CUDA_TRY(cudaSetDevice(c->dev));
    if (!c->embed) CUDA_TRY(dalloc(&c->embed, len));
    CUDA_TRY(cudaMemcpy(c->embed, embed, len * 2, cudaMemcpyHostToDevice));
    c->embed_ready = true;
    return VOX_OK;
}

int vox_ctx_upload_lm_head_bf16(vox_ctx* c, const uint16_t* head, size_t len) {
    if (!c || !head) return fail(VOX_ERR_INVALID_ARG, "null argument");
    if (c->opt.vocab == 0) return fail(VOX_ERR_NOT_READY, "context was created without a vocabulary");
    if (len != c->opt.vocab * c->cfg.dim) return fail(VOX_ERR_SHAPE, "lm_head shape mismatch");
    CUDA_TRY(cudaSetDevice(c->dev));
    if (!c->lm_head) CUDA_TRY(cudaMalloc(&c->lm_head, len * c->wsize));
    auto bytes = to_wdtype(head, len, c->wsize);
    CUDA_TRY(cudaMemcpy(c->lm_head, bytes.data(), bytes.size(), cudaMemcpyHostToDevice));
    if (!c->final_norm) {
        CUDA_TRY(dalloc(&c->final_norm, c->cfg.dim));
        CUDA_TRY(launch_fill_f32(c->final_norm, 1.0f, (long long)c->cfg.dim, c->stream));
        CUDA_TRY(cudaStreamSynchronize(c->stream));
    }
    c->head_ready = true;
    c->head_tiled = false;
    return VOX_OK;
}

int vox_ctx_upload_final_norm(vox_ctx* c, const float* gain, size_t len) {
    if (!c || !gain) return fail(VOX_ERR_INVALID_ARG, "null argument");
    if (len != c->cfg.dim) return fail(VOX_ERR_SHAPE, "final_norm shape mismatch");
    CUDA_TRY(cudaSetDevice(c->dev));
    if (!c->final_norm) CUDA_TRY(dalloc(&c->final_norm, c->cfg.dim));
    CUDA_TRY(cudaMemcpy(c->final_norm, gain, len * 4, cudaMemcpyHostToDevice));
    return VOX_OK;
}

int vox_ctx_init_random(vox_ctx* c, uint64_t seed, float stdv) {
    if (!c) return fail(VOX_ERR_INVALID_ARG, "context is null");
    CUDA_TRY(cudaSetDevice(c->dev));
    const long long dim = (long long)c->cfg.dim, hid = (long long)c->cfg.hidden_dim;
    const long long qd = (long long)c->q_dim, kvd = (long long)c->kv_dim;
    const int ws = c->wsize;
    cudaStream_t s = c->stream;
    for (size_t l = 0; l < c->layers.size(); ++l) {
        LayerDev& L = c->layers[l];
        TRY(alloc_layer(c, L));
        const uint64_t b = 16 * (uint64_t)l;
        CUDA_TRY(launch_gen_matrix(L.wqkv, ws, seed, b + 1, stdv, qd, dim, 1, 0, s));
        CUDA_TRY(launch_gen_matrix(L.wqkv, ws, seed, b + 2, stdv, kvd, dim, 1, (int)qd, s));
        CUDA_TRY(launch_gen_matrix(L.wqkv, ws, seed, b + 3, stdv, kvd, dim, 1, (int)(qd + kvd), s));
        CUDA_TRY(launch_gen_matrix(L.wo, ws, seed, b + 4, stdv, dim, qd, 1, 0, s));
        CUDA_TRY(launch_gen_matrix(L.w13, ws, seed, b + 5, stdv, hid, dim, 2, 0, s));
        CUDA_TRY(launch_gen_matrix(L.w2, ws, seed, b + 6, stdv, dim, hid, 1, 0, s));
        CUDA_TRY(launch_gen_matrix(L.w13, ws, seed, b + 7, stdv, hid, dim, 2, 1, s));
        CUDA_TRY(launch_fill_f32(L.attn_norm, 1.0f, dim, s));
        CUDA_TRY(launch_fill_f32(L.ffn_norm, 1.0f, dim, s));
        L.ready = true;
        L.tiled = false;
    }
    if (c->opt.vocab) {
        const long long V = (long long)c->opt.vocab;
        if (!c->embed) CUDA_TRY(dalloc(&c->embed, (size_t)(V * dim)));
        if (!c->lm_head) CUDA_TRY(cudaMalloc(&c->lm_head, (size_t)(V * dim) * ws));
        if (!c->final_norm) CUDA_TRY(dalloc(&c->final_norm, (size_t)dim));
        CUDA_TRY(launch_gen_matrix(c->embed, 2, seed, 1000000, stdv, V, dim, 1, 0, s));
        CUDA_TRY(launch_gen_matrix(c->lm_head, ws, seed, 1000001, stdv, V, dim, 1, 0, s));
        CUDA_TRY(launch_fill_f32(c->final_norm, 1.0f, dim, s));
        c->embed_ready = c->head_ready = true;
        c->head_tiled = false;
    }
    CUDA_TRY(cudaStreamSynchronize(s));
    return VOX_OK;
}

int vox_ctx_download_matrix(vox_ctx* c, size_t layer, int which, void* out, size_t out_bytes) {
    if (!c || !out) return fail(VOX_ERR_INVALID_ARG, "null argument");
    CUDA_TRY(cudaSetDevice(c->dev));
    const size_t dim = c->cfg.dim, hid = c->cfg.hidden_dim, ws = c->wsize;
    if (which >= 7) {
        if (!c->embed_ready || !c->head_ready) return fail(VOX_ERR_NOT_READY, "no embedding / LM head");
        const size_t n = c->opt.vocab * dim;
        const size_t es = which == 7 ? 2 : ws;
        if (out_bytes < n * es) return fail(VOX_ERR_SHAPE, "output buffer too small");
        CUDA_TRY(cudaMemcpy(out, which == 7 ? (void*)c->embed : c->lm_head, n * es, cudaMemcpyDeviceToHost));
        return VOX_OK;
    }
    if (layer >= c->layers.size() || !c->layers[layer].ready)
        return fail(VOX_ERR_NOT_READY, "layer %zu not uploaded", layer);
    const LayerDev& L = c->layers[layer];
    const unsigned char* qkv = static_cast<const unsigned char*>(L.wqkv);
    const void* src = nullptr;
    size_t n = 0;
    switch (which) {
        case 0: src = qkv; n = c->q_dim * dim; break;
        case 1: src = qkv + c->q_dim * dim * ws; n = c->kv_dim * dim; break;
        case 2: src = qkv + (c->q_dim + c->kv_dim) * dim * ws; n = c->kv_dim * dim; break;
        case 3: src = L.wo; n = dim * c->q_dim; break;
        case 5: src = L.w2; n = dim * hid; break;
        case 4:
        case 6: {
            n = hid * dim;
            if (out_bytes < n * ws) return fail(VOX_ERR_SHAPE, "output buffer too small");
            const size_t row = dim * ws;
            CUDA_TRY(cudaMemcpy2D(out, row, static_cast<const unsigned char*>(L.w13) + (which == 6 ? row : 0),
                                  2 * row, row, hid, cudaMemcpyDeviceToHost));
            return VOX_OK;
        }
        default: return fail(VOX_ERR_INVALID_ARG, "unknown matrix %d", which);
    }
    if (out_bytes < n * ws) return fail(VOX_ERR_SHAPE, "output buffer too small");
    CUDA_TRY(cudaMemcpy(out, src, n * ws, cudaMemcpyDeviceToHost));
    return VOX_OK;
}

void* vox_ctx_stream(vox_ctx* c) { return c ? (void*)c->stream : nullptr; }

int vox_ctx_synchronize(vox_ctx* c) {
    if (!c) return fail(VOX_ERR_INVALID_ARG, "context is null");
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    return check_device_errors(c);
}

int vox_ctx_record_event(vox_ctx* c, int slot) {
    if (!c || slot < 0 || slot >= 16) return fail(VOX_ERR_INVALID_ARG, "bad event slot");
    CUDA_TRY(cudaEventRecord(c->ev[slot], c->stream));
    return VOX_OK;
}

int vox_ctx_event_elapsed_ms(vox_ctx* c, int a, int b, float* ms) {
    if (!c || !ms || a < 0 || a >= 16 || b < 0 || b >= 16) return fail(VOX_ERR_INVALID_ARG, "bad event slot");
    CUDA_TRY(cudaEventSynchronize(c->ev[b]));
    CUDA_TRY(cudaEventElapsedTime(ms, c->ev[a], c->ev[b]));
    return VOX_OK;
}

uint64_t vox_ctx_kernel_launches(vox_ctx* c) { return c ? c->launches : 0; }

// ---- KV cache ----------------------------------------------------------------
static int create_cache(vox_ctx* c, size_t n_streams, size_t n_layers, size_t n_kv, size_t hd, size_t window,
                        size_t cap, vox_kv** out) {
    if (!c || !out) return fail(VOX_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    if (n_layers == 0 || n_kv == 0 || hd == 0 || window == 0)
        return fail(VOX_ERR_INVALID_ARG, "n_layers, n_kv_heads, head_dim and sliding_window must be > 0");
    if (n_streams == 0 || n_streams > 8) return fail(VOX_ERR_UNSUPPORTED, "n_streams must be 1..8");
    if (cap < window) return fail(VOX_ERR_INVALID_ARG, "capacity below the window");
    if (cap > (size_t)INT32_MAX / 2) return fail(VOX_ERR_UNSUPPORTED, "capacity too large");
    CUDA_TRY(cudaSetDevice(c->dev));
    vox_kv* kv = new vox_kv();
    kv->ctx = c;
    kv->n_layers = n_layers;
    kv->n_kv = n_kv;
    kv->hd = hd;
    kv->window = window;
    kv->cap = cap;
    kv->n_streams = n_streams;
    kv->hs_store.assign(n_streams * n_layers, HostKv{});
    kv->hs = kv->hs_store.data();
    kv->views.assign(n_streams, nullptr);
    cudaError_t e = dalloc(&kv->k, n_streams * kv->stream_elems());
    if (e == cudaSuccess) e = dalloc(&kv->v, n_streams * kv->stream_elems());
    if (e == cudaSuccess) e = dalloc(&kv->dstate, n_streams * n_layers);
    if (e == cudaSuccess) e = cudaMemset(kv->dstate, 0, n_streams * n_layers * sizeof(KvState));
    if (e != cudaSuccess) {
        vox_kv_destroy(kv);
        return fail(e == cudaErrorMemoryAllocation ? VOX_ERR_OOM : VOX_ERR_CUDA, "cache allocation: %s",
                    cudaGetErrorString(e));
    }
    c->caches.push_back(kv);
    *out = kv;
    return VOX_OK;
}

// Single-stream entry points take a one-stream cache or a stream view.
static int single_stream(const vox_kv* kv) {
    if (kv->n_streams != 1 && !kv->parent)
        return fail(VOX_ERR_INVALID_ARG, "cache holds %zu streams: pass a stream view (vox_kv_stream)",
                    kv->n_streams);
    return VOX_OK;
}

static void release_graphs(vox_kv* kv) {
    if (kv->step_graph) cudaGraphExecDestroy(kv->step_graph);
    if (kv->step_graph_short) cudaGraphExecDestroy(kv->step_graph_short);
    if (kv->batch_graph) cudaGraphExecDestroy(kv->batch_graph);
    kv->step_graph = kv->step_graph_short = kv->batch_graph = nullptr;
}

int vox_kv_create_ex(vox_ctx* c, size_t n_layers, size_t n_kv, size_t hd, size_t window, size_t cap,
                     vox_kv** out) {
    return create_cache(c, 1, n_layers, n_kv, hd, window, cap, out);
}

int vox_kv_create(vox_ctx* c, size_t n_layers, size_t n_kv, size_t hd, size_t window, vox_kv** out) {
    return create_cache(c, 1, n_layers, n_kv, hd, window, window, out);
}

int vox_kv_create_streams(vox_ctx* c, size_t n_streams, size_t n_layers, size_t n_kv, size_t hd, size_t window,
                          vox_kv** out) {
    return create_cache(c, n_streams, n_layers, n_kv, hd, window, window, out);
}

int vox_kv_n_streams(const vox_kv* kv, size_t* out) {
    if (!kv || !out) return fail(VOX_ERR_INVALID_ARG, "bad argument");
    *out = kv->parent ? 1 : kv->n_streams;
    return VOX_OK;
}

int vox_kv_stream(vox_kv* kv, size_t stream, vox_kv** out) {
    if (!kv || !out) return fail(VOX_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    if (kv->parent) return fail(VOX_ERR_INVALID_ARG, "already a stream view");
    if (stream >= kv->n_streams) return fail(VOX_ERR_INVALID_ARG, "stream %zu out of range", stream);
    if (kv->n_streams == 1) {
        *out = kv;
        return VOX_OK;
    }
    if (!kv->views[stream]) {
        vox_kv* w = new vox_kv();
        w->ctx = kv->ctx;
        w->n_layers = kv->n_layers;
        w->n_kv = kv->n_kv;
        w->hd = kv->hd;
        w->window = kv->window;
        w->cap = kv->cap;
        w->n_streams = 1;
        w->k = kv->k + stream * kv->stream_elems();
        w->v = kv->v + stream * kv->stream_elems();
        w->dstate = kv->dstate + stream * kv->n_layers;
        w->hs = kv->hs_store.data() + stream * kv->n_layers;
        w->parent = kv;
        kv->views[stream] = w;
    }
    *out = kv->views[stream];
    return VOX_OK;
}

void vox_kv_destroy(vox_kv* kv) {
    if (!kv || kv->parent) return;  // views live as long as their cache
    vox_ctx* c = kv->ctx;
    cudaSetDevice(c->dev);
    cudaStreamSynchronize(c->stream);
    for (size_t i = 0; i < c->caches.size(); ++i)
        if (c->caches[i] == kv) {
            c->caches.erase(c->caches.begin() + (long)i);
            break;
        }
    for (vox_kv* w : kv->views)
        if (w) {
            release_graphs(w);
            delete w;
        }
    release_graphs(kv);
    cudaFree(kv->k);
    cudaFree(kv->v);
    cudaFree(kv->dstate);
    delete kv;
}

int vox_kv_reset(vox_kv* kv) {
    if (!kv) return fail(VOX_ERR_INVALID_ARG, "cache is null");
    CUDA_TRY(cudaSetDevice(kv->ctx->dev));
    CUDA_TRY(cudaStreamSynchronize(kv->ctx->stream));
    const size_t n = (kv->parent ? 1 : kv->n_streams) * kv->n_layers;
    for (size_t i = 0; i < n; ++i) kv->hs[i] = HostKv{};
    CUDA_TRY(cudaMemset(kv->dstate, 0, n * sizeof(KvState)));
    return VOX_OK;
}

int vox_kv_fill_random(vox_kv* kv, size_t n_tokens, uint64_t seed, uint64_t tensor_id, float stdv) {
    if (!kv) return fail(VOX_ERR_INVALID_ARG, "cache is null");
    TRY(single_stream(kv));
    if (n_tokens > kv->window) return fail(VOX_ERR_INVALID_ARG, "%zu tokens exceed the window %zu", n_tokens, kv->window);
    vox_ctx* c = kv->ctx;
    CUDA_TRY(cudaSetDevice(c->dev));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    std::vector<KvState> d(kv->n_layers);
    for (size_t l = 0; l < kv->n_layers; ++l) {
        CUDA_TRY(record_launch(c, launch_kv_fill_random(kv->k + l * kv->layer_elems(), kv->v + l * kv->layer_elems(),
                                                        (int)kv->n_kv, (int)kv->hd, (int)kv->cap, (int)n_tokens,
                                                        seed, tensor_id + 2 * l, tensor_id + 2 * l + 1, stdv,
                                                        c->stream)));
        kv->hs[l] = HostKv{n_tokens, 0, 0};
        d[l].len = (int32_t)n_tokens;
        d[l].start = 0;
        d[l].pos_offset = 0;
    }
    CUDA_TRY(cudaMemcpyAsync(kv->dstate, d.data(), d.size() * sizeof(KvState), cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    return VOX_OK;
}

int vox_kv_append_layer(vox_kv* kv, size_t layer, const float* k_new, const float* v_new, size_t n) {
    if (!kv) return fail(VOX_ERR_INVALID_ARG, "cache is null");
    TRY(single_stream(kv));
    if (layer >= kv->n_layers) return fail(VOX_ERR_INVALID_ARG, "layer %zu out of range", layer);
    if (n == 0) return VOX_OK;  // kv.rs:55-57
    if (!k_new || !v_new) return fail(VOX_ERR_INVALID_ARG, "null k/v");
    vox_ctx* c = kv->ctx;
    CUDA_TRY(cudaSetDevice(c->dev));
    HostKv s = kv->hs[layer];
    const long long slot0 = host_append(s, n, kv->window, kv->cap);
    if (slot0 < 0)
        return fail(VOX_ERR_UNSUPPORTED, "append of %zu tokens exceeds the ring capacity %zu", n, kv->cap);
    const size_t elems = n * kv->n_kv * kv->hd;
    TRY(ensure_scratch(c, 2 * elems * 4));
    float* sk = static_cast<float*>(c->scratch);
    float* sv = sk + elems;
    CUDA_TRY(cudaMemcpyAsync(sk, k_new, elems * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaMemcpyAsync(sv, v_new, elems * 4, cudaMemcpyHostToDevice, c->stream));
    // Only the last `cap` tokens can survive; skip the rest.
    size_t skip = n > kv->cap ? n - kv->cap : 0;
    CUDA_TRY(record_launch(c, launch_kv_scatter(sk + skip * kv->n_kv * kv->hd, sv + skip * kv->n_kv * kv->hd,
                                                kv->k + layer * kv->layer_elems(),
                                                kv->v + layer * kv->layer_elems(), (int)kv->n_kv,
                                                (int)kv->hd, (int)kv->cap, (int)((slot0 + skip) % kv->cap),
                                                (int)(n - skip), c->stream)));
    kv->hs[layer] = s;
    return upload_state(kv, layer);
}

int vox_kv_layer_len_tokens(const vox_kv* kv, size_t layer, size_t* out) {
    if (!kv || !out || layer >= kv->n_layers) return fail(VOX_ERR_INVALID_ARG, "bad argument");
    TRY(single_stream(kv));
    *out = kv->hs[layer].len;
    return VOX_OK;
}

int vox_kv_layer_pos_offset(const vox_kv* kv, size_t layer, size_t* out) {
    if (!kv || !out || layer >= kv->n_layers) return fail(VOX_ERR_INVALID_ARG, "bad argument");
    TRY(single_stream(kv));
    *out = kv->hs[layer].pos_offset;
    return VOX_OK;
}

int vox_kv_layer_device_state(const vox_kv* kv, size_t layer, int64_t out[3]) {
    if (!kv || !out || layer >= kv->n_layers) return fail(VOX_ERR_INVALID_ARG, "bad argument");
    TRY(single_stream(kv));
    vox_ctx* c = kv->ctx;
    CUDA_TRY(cudaSetDevice(c->dev));
    KvState d{};
    CUDA_TRY(cudaMemcpyAsync(&d, kv->dstate + layer, sizeof d, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    out[0] = d.len;
    out[1] = d.start;
    out[2] = d.pos_offset;
    return VOX_OK;
}

int vox_kv_layer_tensors(const vox_kv* kv, size_t layer, float* keys, float* values, size_t cap_elems) {
    if (!kv || layer >= kv->n_layers) return fail(VOX_ERR_INVALID_ARG, "bad argument");
    TRY(single_stream(kv));
    vox_ctx* c = kv->ctx;
    const HostKv& s = kv->hs[layer];
    const size_t elems = s.len * kv->n_kv * kv->hd;
    if (elems == 0) return VOX_OK;
    if (!keys || !values || cap_elems < elems)
        return fail(VOX_ERR_SHAPE, "buffers hold %zu elements, need %zu", cap_elems, elems);
    CUDA_TRY(cudaSetDevice(c->dev));
    TRY(ensure_scratch(c, 2 * elems * 4));
    float* dk = static_cast<float*>(c->scratch);
    float* dv = dk + elems;
    CUDA_TRY(record_launch(c, launch_kv_gather(kv->k + layer * kv->layer_elems(), kv->v + layer * kv->layer_elems(),
                                               dk, dv, (int)kv->n_kv, (int)kv->hd, (int)kv->cap, (int)s.start,
                                               (int)s.len, c->stream)));
    CUDA_TRY(cudaMemcpyAsync(keys, dk, elems * 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaMemcpyAsync(values, dv, elems * 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    return VOX_OK;
}

// ---- decoder layer step --------------------------------------------------------
int vox_decoder_layer_forward_step(vox_ctx* c, size_t layer, vox_kv* kv, const float* hidden,
                                   size_t hidden_len, size_t pos, float* out, size_t out_len) {
    if (!c || !kv) return fail(VOX_ERR_INVALID_ARG, "null context or cache");
    TRY(single_stream(kv));
    TRY(validate_cfg(&c->cfg));                                    // decoder.rs:96
    if (layer >= c->layers.size() || !c->layers[layer].ready)      // decoder.rs:97
        return fail(VOX_ERR_NOT_READY, "layer %zu weights not uploaded", layer);
    if (hidden_len != c->cfg.dim || !hidden) return fail(VOX_ERR_SHAPE, "hidden size mismatch");  // :98
    if (out_len != c->cfg.dim || !out) return fail(VOX_ERR_SHAPE, "output size mismatch");
    if (kv->ctx != c) return fail(VOX_ERR_INVALID_ARG, "cache belongs to another context");
    if (layer >= kv->n_layers) return fail(VOX_ERR_INVALID_ARG, "layer %zu beyond the cache", layer);
    if (kv->n_kv != c->cfg.n_kv_heads || kv->hd != c->cfg.head_dim)
        return fail(VOX_ERR_SHAPE, "cache head shape does not match the decoder config");
    if (pos >= (size_t)c->max_pos) return fail(VOX_ERR_RANGE, "position %zu beyond max_positions %d", pos, c->max_pos);
    CUDA_TRY(cudaSetDevice(c->dev));
    StepState* hs = c->h_steps;
    CUDA_TRY(cudaStreamSynchronize(c->stream));  // the pinned slot is reused below
    std::memset(hs, 0, sizeof(StepState));
    hs->pos = (int64_t)pos;
    CUDA_TRY(cudaMemcpyAsync(c->step, hs, sizeof(StepState), cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaMemcpyAsync(c->hid, hidden, c->cfg.dim * 4, cudaMemcpyHostToDevice, c->stream));
    TRY(enqueue_layer(c, kv, layer, false, true));
    CUDA_TRY(cudaMemcpyAsync(out, c->hid, c->cfg.dim * 4, cudaMemcpyDeviceToHost, c->stream));
    TRY(check_device_errors(c));
    host_append(kv->hs[layer], 1, kv->window, kv->cap);
    return VOX_OK;
}

// ---- token loop --------------------------------------------------------------------
int vox_model_step(vox_ctx* c, vox_kv* kv, int32_t token, size_t pos, int32_t* next_token, float* logits) {
    TRY(model_ready(c, kv));
    TRY(single_stream(kv));
    if (token < 0 || (size_t)token >= c->opt.vocab) return fail(VOX_ERR_RANGE, "token %d outside the vocabulary", token);
    if (pos >= (size_t)c->max_pos) return fail(VOX_ERR_RANGE, "position %zu beyond max_positions %d", pos, c->max_pos);
    CUDA_TRY(cudaSetDevice(c->dev));
    TRY(build_step_graph(c, kv));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    StepState* hs = c->h_steps;
    std::memset(hs, 0, sizeof(StepState));
    hs->pos = (int64_t)pos;
    hs->tok = token;
    CUDA_TRY(cudaMemcpyAsync(c->step, hs, sizeof(StepState), cudaMemcpyHostToDevice, c->stream));
    TRY(launch_graph(c, kv, live_tokens_after(c, kv, 1)));
    CUDA_TRY(cudaMemcpyAsync(c->h_tok, c->tok_out, 4, cudaMemcpyDeviceToHost, c->stream));
    if (logits)
        CUDA_TRY(cudaMemcpyAsync(logits, c->logits, c->opt.vocab * 4, cudaMemcpyDeviceToHost, c->stream));
    TRY(check_device_errors(c));
    mirror_single_append_all(kv);
    if (next_token) *next_token = *c->h_tok;
    return VOX_OK;
}

static int prefill_checks(vox_ctx* c, vox_kv* kv, const int32_t* tokens, size_t n, size_t pos0) {
    TRY(model_ready(c, kv));
    TRY(single_stream(kv));
    if (n == 0) return VOX_OK;
    if (!tokens) return fail(VOX_ERR_INVALID_ARG, "tokens is null");
    if (pos0 + n > (size_t)c->max_pos) return fail(VOX_ERR_RANGE, "positions beyond max_positions %d", c->max_pos);
    for (size_t i = 0; i < n; ++i)
        if (tokens[i] < 0 || (size_t)tokens[i] >= c->opt.vocab)
            return fail(VOX_ERR_RANGE, "token %d outside the vocabulary", tokens[i]);
    return VOX_OK;
}

int vox_model_prefill(vox_ctx* c, vox_kv* kv, const int32_t* tokens, size_t n, size_t pos0) {
    TRY(prefill_checks(c, kv, tokens, n, pos0));
    if (n < 2 || !prefill_batched_supported(c)) return vox_model_prefill_steps(c, kv, tokens, n, pos0);
    CUDA_TRY(cudaSetDevice(c->dev));
    return prefill_batched(c, kv, tokens, n, pos0, nullptr, 0);
}

int vox_model_prefill_steps(vox_ctx* c, vox_kv* kv, const int32_t* tokens, size_t n, size_t pos0) {
    TRY(prefill_checks(c, kv, tokens, n, pos0));
    if (n == 0) return VOX_OK;
    CUDA_TRY(cudaSetDevice(c->dev));
    TRY(build_step_graph(c, kv));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    TRY(ensure_host_steps(c, n));
    for (size_t i = 0; i < n; ++i) {
        StepState* hs = c->h_steps + i;
        std::memset(hs, 0, sizeof(StepState));
        hs->pos = (int64_t)(pos0 + i);
        hs->tok = tokens[i];
        CUDA_TRY(cudaMemcpyAsync(c->step, hs, sizeof(StepState), cudaMemcpyHostToDevice, c->stream));
        TRY(launch_graph(c, kv, live_tokens_after(c, kv, i + 1)));
    }
    TRY(check_device_errors(c));
    for (size_t i = 0; i < n; ++i) mirror_single_append_all(kv);
    return VOX_OK;
}

int vox_model_generate(vox_ctx* c, vox_kv* kv, int32_t token, size_t pos, size_t n_steps, int32_t* tokens_out) {
    TRY(model_ready(c, kv));
    TRY(single_stream(kv));
    if (n_steps == 0) return VOX_OK;
    if (token < 0 || (size_t)token >= c->opt.vocab) return fail(VOX_ERR_RANGE, "token %d outside the vocabulary", token);
    if (pos + n_steps > (size_t)c->max_pos) return fail(VOX_ERR_RANGE, "positions beyond max_positions %d", c->max_pos);
    CUDA_TRY(cudaSetDevice(c->dev));
    TRY(build_step_graph(c, kv));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    TRY(ensure_host_steps(c, n_steps + 1));
    StepState* hs = c->h_steps;
    std::memset(hs, 0, sizeof(StepState));
    hs->pos = (int64_t)pos;
    hs->tok = token;
    hs->greedy = 1;
    hs->advance = 1;
    CUDA_TRY(cudaMemcpyAsync(c->step, hs, sizeof(StepState), cudaMemcpyHostToDevice, c->stream));
    int32_t* tok_hist = reinterpret_cast<int32_t*>(c->h_steps + 1);  // pinned staging for the ids
    for (size_t i = 0; i < n_steps; ++i) {
        TRY(launch_graph(c, kv, live_tokens_after(c, kv, i + 1)));
        if (tokens_out)
            CUDA_TRY(cudaMemcpyAsync(tok_hist + i, c->tok_out, 4, cudaMemcpyDeviceToHost, c->stream));
    }
    TRY(check_device_errors(c));
    for (size_t i = 0; i < n_steps; ++i) mirror_single_append_all(kv);
    if (tokens_out) std::memcpy(tokens_out, tok_hist, n_steps * 4);
    return VOX_OK;
}

// ---- multi-stream token loop -----------------------------------------------------
static int batch_ready(vox_ctx* c, vox_kv* kv) {
    TRY(model_ready(c, kv));
    if (kv->parent) return fail(VOX_ERR_INVALID_ARG, "pass the multi-stream cache, not a stream view");
    TRY(ensure_batch(c));
    TRY(build_batch_graph(c, kv));
    return VOX_OK;
}

static int check_stream_inputs(vox_ctx* c, const vox_kv* kv, const int32_t* tokens, const size_t* positions,
                               size_t n_steps) {
    if (!tokens || !positions) return fail(VOX_ERR_INVALID_ARG, "tokens or positions is null");
    for (size_t s = 0; s < kv->n_streams; ++s) {
        if (tokens[s] < 0 || (size_t)tokens[s] >= c->opt.vocab)
            return fail(VOX_ERR_RANGE, "stream %zu: token %d outside the vocabulary", s, tokens[s]);
        if (positions[s] + n_steps > (size_t)c->max_pos)
            return fail(VOX_ERR_RANGE, "stream %zu: positions beyond max_positions %d", s, c->max_pos);
    }
    return VOX_OK;
}

static int upload_batch_steps(vox_ctx* c, const vox_kv* kv, const int32_t* tokens, const size_t* positions,
                              int greedy) {
    StepState* hs = c->bb.h_steps;
    std::memset(hs, 0, 8 * sizeof(StepState));
    for (size_t s = 0; s < kv->n_streams; ++s) {
        hs[s].pos = (int64_t)positions[s];
        hs[s].tok = tokens[s];
        hs[s].greedy = greedy;
        hs[s].advance = greedy;
    }
    CUDA_TRY(cudaMemcpyAsync(c->bb.steps, hs, kv->n_streams * sizeof(StepState), cudaMemcpyHostToDevice,
                             c->stream));
    return VOX_OK;
}

static void mirror_batch_appends(vox_kv* kv, size_t n_steps) {
    for (HostKv& h : kv->hs_store)
        for (size_t i = 0; i < n_steps; ++i) host_append(h, 1, kv->window, kv->cap);
}

int vox_model_step_batch(vox_ctx* c, vox_kv* kv, const int32_t* tokens, const size_t* positions,
                         int32_t* next_tokens, float* logits) {
    TRY(batch_ready(c, kv));
    TRY(check_stream_inputs(c, kv, tokens, positions, 1));
    CUDA_TRY(cudaStreamSynchronize(c->stream));  // the pinned step slots are reused below
    TRY(upload_batch_steps(c, kv, tokens, positions, 0));
    CUDA_TRY(cudaGraphLaunch(kv->batch_graph, c->stream));
    c->launches += kv->batch_kernels;
    if (next_tokens)
        CUDA_TRY(cudaMemcpyAsync(next_tokens, c->bb.tok_out, kv->n_streams * 4, cudaMemcpyDeviceToHost, c->stream));
    if (logits)
        CUDA_TRY(cudaMemcpyAsync(logits, c->bb.logits, kv->n_streams * c->opt.vocab * 4, cudaMemcpyDeviceToHost,
                                 c->stream));
    TRY(check_device_errors(c));
    mirror_batch_appends(kv, 1);
    return VOX_OK;
}

int vox_model_generate_batch(vox_ctx* c, vox_kv* kv, const int32_t* tokens, const size_t* positions,
                             size_t n_steps, int32_t* tokens_out) {
    TRY(batch_ready(c, kv));
    if (n_steps == 0) return VOX_OK;
    TRY(check_stream_inputs(c, kv, tokens, positions, n_steps));
    BatchBufs& bb = c->bb;
    const size_t B = kv->n_streams;
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    if (tokens_out && n_steps * B > bb.h_tok_cap) {
        if (bb.h_tok) cudaFreeHost(bb.h_tok);
        bb.h_tok = nullptr;
        bb.h_tok_cap = 0;
        size_t cap = 1024;
        while (cap < n_steps * B) cap <<= 1;
        CUDA_TRY(cudaMallocHost(&bb.h_tok, cap * 4));
        bb.h_tok_cap = cap;
    }
    TRY(upload_batch_steps(c, kv, tokens, positions, 1));
    for (size_t i = 0; i < n_steps; ++i) {
        CUDA_TRY(cudaGraphLaunch(kv->batch_graph, c->stream));
        c->launches += kv->batch_kernels;
        if (tokens_out)
            CUDA_TRY(cudaMemcpyAsync(bb.h_tok + i * B, bb.tok_out, B * 4, cudaMemcpyDeviceToHost, c->stream));
    }
    TRY(check_device_errors(c));
    mirror_batch_appends(kv, n_steps);
    if (tokens_out) std::memcpy(tokens_out, bb.h_tok, n_steps * B * 4);
    return VOX_OK;
}

// ---- profiling hook ----------------------------------------------------------------
int vox_profile_gemv(vox_ctx* c, int which, size_t n, float* avg_ms, uint64_t* bytes_per_launch) {
    if (!c || !avg_ms || n == 0) return fail(VOX_ERR_INVALID_ARG, "bad argument");
    if (which < 1 || which > 4) return fail(VOX_ERR_INVALID_ARG, "which must be 1..4");
    for (size_t l = 0; l < c->layers.size(); ++l)
        if (!c->layers[l].ready) return fail(VOX_ERR_NOT_READY, "layer %zu weights not uploaded", l);
    if (which == 4 && (!c->head_ready || !c->opt.vocab)) return fail(VOX_ERR_NOT_READY, "no LM head");
    CUDA_TRY(cudaSetDevice(c->dev));
    const GemvPlan* plan = which == 1 ? &c->p_o : which == 2 ? &c->p_w13 : which == 3 ? &c->p_w2 : &c->p_head;
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    CUDA_TRY(cudaEventRecord(c->ev[14], c->stream));
    for (size_t i = 0; i < n; ++i) {
        const LayerDev& L = c->layers[i % c->layers.size()];
        GemvArgs a = base_args(c);
        int epi = EPI_RESID;
        if (which == 1) {
            a.W = L.wo; a.x = c->attn; a.y = c->hmid; a.resid = c->hid;
        } else if (which == 2) {
            a.W = L.w13; a.x = c->hmid; a.norm_w = L.ffn_norm; a.y = c->act; epi = EPI_SWIGLU;
        } else if (which == 3) {
            a.W = L.w2; a.x = c->act; a.y = c->hmid; a.resid = c->hmid;
        } else {
            a.W = c->lm_head; a.x = c->hid; a.norm_w = c->final_norm; a.y = c->logits;
            a.am_part = c->am_part; epi = EPI_ARGMAX;
        }
        CUDA_TRY(record_launch(c, launch_gemv(*plan, a, epi, c->stream, true)));
    }
    CUDA_TRY(cudaEventRecord(c->ev[15], c->stream));
    CUDA_TRY(cudaEventSynchronize(c->ev[15]));
    float ms = 0.f;
    CUDA_TRY(cudaEventElapsedTime(&ms, c->ev[14], c->ev[15]));
    *avg_ms = ms / (float)n;
    if (bytes_per_launch) *bytes_per_launch = (uint64_t)plan->rows * (uint64_t)plan->K * (uint64_t)c->wsize;
    return check_device_errors(c);
}

int vox_profile_bgemm(vox_ctx* c, int which, size_t n_streams, size_t n, float* avg_ms, uint64_t* bytes_per_launch) {
    if (!c || !avg_ms || n == 0) return fail(VOX_ERR_INVALID_ARG, "bad argument");
    if (which < 1 || which > 6) return fail(VOX_ERR_INVALID_ARG, "which must be 1..6");
    if (n_streams < 1 || n_streams > 8) return fail(VOX_ERR_INVALID_ARG, "n_streams must be 1..8");
    for (size_t l = 0; l < c->layers.size(); ++l)
        if (!c->layers[l].ready) return fail(VOX_ERR_NOT_READY, "layer %zu weights not uploaded", l);
    CUDA_TRY(cudaSetDevice(c->dev));
    TRY(ensure_batch(c));
    BatchBufs& bb = c->bb;
    const int B = (int)n_streams, dim = (int)c->cfg.dim, hid = (int)c->cfg.hidden_dim, qd = (int)c->q_dim;
    const BgPlan& p = which == 1 ? bb.p_o : which == 2 ? bb.p_w13 : which == 3 ? bb.p_w2 : which == 4 ? bb.p_head
                                                                                                      : bb.p_qkv;
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    CUDA_TRY(cudaEventRecord(c->ev[14], c->stream));
    for (size_t i = 0; i < n && which == 6; ++i) {  // o-proj, w1|w3, w2, q|k|v as one chain launch
        const LayerDev& L = c->layers[i % c->layers.size()];
        BgChain ch{};
        ch.n_phases = 4;
        ch.done = bb.done;
        BgArgs a = bg_args(c, bb.c_o, L.wo_t, B, BG_RESID);
        a.x = bb.attn; a.x_stride = qd; a.y = bb.hmid; a.y_stride = dim; a.resid = bb.hid; a.ssp_out = bb.ssp;
        ch.ph[0] = a;
        a = bg_args(c, bb.c_w13, L.w13_t, B, BG_SWIGLU);
        a.x = bb.hmid; a.x_stride = dim; a.norm_w = L.ffn_norm; a.ssp = bb.ssp; a.y = bb.act; a.y_stride = hid;
        ch.ph[1] = a;
        a = bg_args(c, bb.c_w2, L.w2_t, B, BG_RESID);
        a.x = bb.act; a.x_stride = hid; a.y = bb.hid; a.y_stride = dim; a.resid = bb.hmid; a.ssp_out = bb.ssp;
        ch.ph[2] = a;
        a = bg_args(c, bb.c_qkv, L.wqkv_t, B, BG_STORE);
        a.x = bb.hid; a.x_stride = dim; a.y = bb.act; a.y_stride = (long long)c->qkv_rows;
        ch.ph[3] = a;
        for (int p = 0; p < 4; ++p) ch.xslab_bytes = std::max(ch.xslab_bytes, ch.ph[p].xslab_bytes);
        CUDA_TRY(cudaMemsetAsync(bb.done, 0, kBgMaxPhases * sizeof(unsigned), c->stream));
        CUDA_TRY(record_launch(c, launch_bgemm(ch, c->num_sms, c->stream, true)));
    }
    for (size_t i = 0; i < n && which != 6; ++i) {
        const LayerDev& L = c->layers[i % c->layers.size()];
        BgArgs a;
        if (which == 1) {
            a = bg_args(c, p, L.wo_t, B, BG_RESID);
            a.x = bb.attn; a.x_stride = qd; a.y = bb.hmid; a.y_stride = dim; a.resid = bb.hid; a.ssp_out = bb.ssp;
        } else if (which == 2) {
            a = bg_args(c, p, L.w13_t, B, BG_SWIGLU);
            a.x = bb.hmid; a.x_stride = dim; a.norm_w = L.ffn_norm; a.ssp = bb.ssp; a.y = bb.act; a.y_stride = hid;
        } else if (which == 3) {
            a = bg_args(c, p, L.w2_t, B, BG_RESID);
            a.x = bb.act; a.x_stride = hid; a.y = bb.hmid; a.y_stride = dim; a.resid = bb.hmid; a.ssp_out = bb.ssp;
        } else if (which == 4) {
            a = bg_args(c, p, c->head_t, B, BG_ARGMAX);
            a.x = bb.hid; a.x_stride = dim; a.norm_w = c->final_norm; a.ssp = bb.ssp; a.y = bb.logits;
            a.y_stride = (long long)c->opt.vocab; a.am_part = bb.am;
        } else {
            a = bg_args(c, p, L.wqkv_t, B, BG_STORE);
            a.x = bb.hid; a.x_stride = dim; a.y = bb.act; a.y_stride = (long long)c->qkv_rows;
        }
        CUDA_TRY(record_launch(c, launch_bgemm(chain_of(a, p), p.grid, c->stream, true)));
    }
    CUDA_TRY(cudaEventRecord(c->ev[15], c->stream));
    CUDA_TRY(cudaEventSynchronize(c->ev[15]));
    float ms = 0.f;
    CUDA_TRY(cudaEventElapsedTime(&ms, c->ev[14], c->ev[15]));
    *avg_ms = ms / (float)n;
    if (bytes_per_launch)
        *bytes_per_launch = which == 6 ? (uint64_t)(dim * qd + 2 * hid * dim + dim * hid + c->qkv_rows * dim) * 2u
                                       : (uint64_t)p.rows * (uint64_t)p.K * 2u;
    return check_device_errors(c);
}

// ---- op-level entry points ----------------------------------------------------------
static int linear_impl(vox_ctx* c, const float* input, size_t n_rows, size_t in_dim, const void* weight,
                       int wsize, size_t out_dim, const float* bias, float* out) {
    if (!c || !input || !weight || !out) return fail(VOX_ERR_INVALID_ARG, "null argument");
    if (n_rows == 0 || out_dim == 0) return VOX_OK;
    if (!gemv_supported((int)in_dim, wsize) || in_dim > (1u << 30) || out_dim > (1u << 30) || n_rows > 65535)
        return fail(VOX_ERR_UNSUPPORTED, "linear: in_dim %zu must be a multiple of %d and at most %d", in_dim,
                    16 / wsize, wsize == 2 ? 16384 : 8192);
    CUDA_TRY(cudaSetDevice(c->dev));
    GemvPlan p = plan_gemv((int)out_dim, (int)in_dim, 1, wsize, c->num_sms, (int)n_rows);
    if (p.grid < 1 || p.smem > gemv_max_smem()) return fail(VOX_ERR_UNSUPPORTED, "no plan for this linear");
    const size_t wb = (out_dim * in_dim * wsize + 255) & ~size_t(255);
    const size_t xb = (n_rows * in_dim * 4 + 255) & ~size_t(255);
    const size_t yb = (n_rows * out_dim * 4 + 255) & ~size_t(255);
    const size_t bb = (out_dim * 4 + 255) & ~size_t(255);
    TRY(ensure_scratch(c, wb + xb + yb + bb));
    unsigned char* base = static_cast<unsigned char*>(c->scratch);
    void* dW = base;
    float* dx = reinterpret_cast<float*>(base + wb);
    float* dy = reinterpret_cast<float*>(base + wb + xb);
    float* db = reinterpret_cast<float*>(base + wb + xb + yb);
    CUDA_TRY(cudaMemcpyAsync(dW, weight, out_dim * in_dim * wsize, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaMemcpyAsync(dx, input, n_rows * in_dim * 4, cudaMemcpyHostToDevice, c->stream));
    if (bias) CUDA_TRY(cudaMemcpyAsync(db, bias, out_dim * 4, cudaMemcpyHostToDevice, c->stream));
    GemvArgs a = base_args(c);
    a.W = dW;
    a.x = dx;
    a.x_stride = (long long)in_dim;
    a.y = dy;
    a.y_stride = (long long)out_dim;
    a.bias = bias ? db : nullptr;
    CUDA_TRY(record_launch(c, launch_gemv(p, a, EPI_STORE, c->stream, false)));
    CUDA_TRY(cudaMemcpyAsync(out, dy, n_rows * out_dim * 4, cudaMemcpyDeviceToHost, c->stream));
    return check_device_errors(c);
}

int vox_linear_f32(vox_ctx* c, const float* input, size_t n_rows, size_t in_dim, const float* weight,
                   size_t out_dim, const float* bias, float* out) {
    return linear_impl(c, input, n_rows, in_dim, weight, 4, out_dim, bias, out);
}

int vox_linear_bf16(vox_ctx* c, const float* input, size_t n_rows, size_t in_dim, const uint16_t* weight,
                    size_t out_dim, const float* bias, float* out) {
    return linear_impl(c, input, n_rows, in_dim, weight, 2, out_dim, bias, out);
}

// K splits per 128-row tile of the tensor-core skinny GEMM: enough items to
// cover every SM once, and few enough K blocks per split that the split's X
// operand fits next to the weight ring.
static int bgemm_splits(int tiles, int kbt, int num_sms) {
    int s = (num_sms + tiles - 1) / tiles;
    const int min_s = (kbt + kBgMaxBlocksPerSplit - 1) / kBgMaxBlocksPerSplit;
    if (s < min_s) s = min_s;
    if (s > kbt) s = kbt;
    return s < 1 ? 1 : s;
}

int vox_linear_batched_bf16(vox_ctx* c, const float* input, size_t n_rows, size_t in_dim, const uint16_t* weight,
                            size_t out_dim, const float* bias, float* out) {
    if (!c || !input || !weight || !out) return fail(VOX_ERR_INVALID_ARG, "null argument");
    if (n_rows == 0 || out_dim == 0) return VOX_OK;
    if (n_rows > 8) return fail(VOX_ERR_UNSUPPORTED, "linear_batched: at most 8 rows, got %zu", n_rows);
    if (in_dim == 0 || in_dim % 64 || in_dim > (1u << 20) || out_dim > (1u << 26))
        return fail(VOX_ERR_UNSUPPORTED, "linear_batched: in_dim %zu must be a positive multiple of 64", in_dim);
    CUDA_TRY(cudaSetDevice(c->dev));
    const int rows = (int)out_dim, K = (int)in_dim;
    const int tiles = (rows + 127) / 128, kbt = K / 64;
    const int splits = bgemm_splits(tiles, kbt, c->num_sms);
    const int items = tiles * splits;
    int grid = c->num_sms - c->num_sms % splits;
    if (grid < 1) grid = splits;
    if (grid > items) grid = items;
    auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
    const size_t wb = al(out_dim * in_dim * 2), tb = al(tiled_bytes(rows, K));
    const size_t xb = al(n_rows * in_dim * 4), yb = al(n_rows * out_dim * 4), bb = al(out_dim * 4);
    const size_t pb = al((size_t)items * 128 * 8 * 4), kb = al((size_t)tiles * 4);
    TRY(ensure_scratch(c, wb + tb + xb + yb + bb + pb + kb));
    unsigned char* p = static_cast<unsigned char*>(c->scratch);
    uint16_t* dW = reinterpret_cast<uint16_t*>(p);
    unsigned char* dT = p + wb;
    float* dx = reinterpret_cast<float*>(p + wb + tb);
    float* dy = reinterpret_cast<float*>(p + wb + tb + xb);
    float* db = reinterpret_cast<float*>(p + wb + tb + xb + yb);
    float* dpart = reinterpret_cast<float*>(p + wb + tb + xb + yb + bb);
    unsigned* dtick = reinterpret_cast<unsigned*>(p + wb + tb + xb + yb + bb + pb);
    CUDA_TRY(cudaMemcpyAsync(dW, weight, out_dim * in_dim * 2, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaMemcpyAsync(dx, input, n_rows * in_dim * 4, cudaMemcpyHostToDevice, c->stream));
    if (bias) CUDA_TRY(cudaMemcpyAsync(db, bias, out_dim * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaMemsetAsync(dtick, 0, (size_t)tiles * 4, c->stream));
    CUDA_TRY(record_launch(c, launch_tile_weights(dW, reinterpret_cast<uint16_t*>(dT), rows, K, c->stream)));
    BgArgs a{};
    a.wt = dT;
    a.rows = rows;
    a.K = K;
    a.tiles = tiles;
    a.kbt = kbt;
    a.splits = splits;
    a.B = (int)n_rows;
    a.xslab_bytes = bgemm_xslab_bytes(K, splits);
    a.x = dx;
    a.x_stride = (long long)in_dim;
    a.epi = BG_STORE;
    a.y = dy;
    a.y_stride = (long long)out_dim;
    a.bias = bias ? db : nullptr;
    a.part = dpart;
    a.tickets = dtick;
    a.err = c->err;
    BgPlan pl{};
    pl.xslab = a.xslab_bytes;
    CUDA_TRY(record_launch(c, launch_bgemm(chain_of(a, pl), grid, c->stream, false)));
    CUDA_TRY(cudaMemcpyAsync(out, dy, n_rows * out_dim * 4, cudaMemcpyDeviceToHost, c->stream));
    return check_device_errors(c);
}

int vox_silu_inplace(vox_ctx* c, float* x, size_t n) {
    return inplace_op(c, x, n, [&](float* d) { return launch_silu(d, (long long)n, c->stream); });
}

int vox_softmax_inplace(vox_ctx* c, float* x, size_t n) {
    return inplace_op(c, x, n, [&](float* d) { return launch_softmax(d, (long long)n, c->stream); });
}

int vox_add_inplace(vox_ctx* c, float* dst, const float* src, size_t n) {
    if (!c || ((!dst || !src) && n)) return fail(VOX_ERR_INVALID_ARG, "null argument");
    if (n == 0) return VOX_OK;
    CUDA_TRY(cudaSetDevice(c->dev));
    TRY(ensure_scratch(c, 2 * n * 4 + 256));
    float* dd = static_cast<float*>(c->scratch);
    float* ds = dd + ((n + 63) & ~size_t(63));
    CUDA_TRY(cudaMemcpyAsync(dd, dst, n * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaMemcpyAsync(ds, src, n * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(record_launch(c, launch_add(dd, ds, (long long)n, c->stream)));
    CUDA_TRY(cudaMemcpyAsync(dst, dd, n * 4, cudaMemcpyDeviceToHost, c->stream));
    return check_device_errors(c);
}

int vox_rms_norm_rows(vox_ctx* c, float* out, const float* input, const float* weight, size_t n_elems,
                      size_t dim, float eps) {
    if (!c || ((!out || !input || !weight) && n_elems)) return fail(VOX_ERR_INVALID_ARG, "null argument");
    if (dim == 0) return fail(VOX_ERR_INVALID_ARG, "dim must be > 0");
    const size_t rows = n_elems / dim;  // math.rs:17 chunks_exact: a ragged tail is left untouched
    if (rows == 0) return VOX_OK;
    if (rows > 0x7FFFFFFF) return fail(VOX_ERR_UNSUPPORTED, "too many rows");
    CUDA_TRY(cudaSetDevice(c->dev));
    const size_t n = rows * dim, nb = (n * 4 + 255) & ~size_t(255), wb = (dim * 4 + 255) & ~size_t(255);
    TRY(ensure_scratch(c, 2 * nb + wb));
    unsigned char* base = static_cast<unsigned char*>(c->scratch);
    float* din = reinterpret_cast<float*>(base);
    float* dout = reinterpret_cast<float*>(base + nb);
    float* dw = reinterpret_cast<float*>(base + 2 * nb);
    CUDA_TRY(cudaMemcpyAsync(din, input, n * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaMemcpyAsync(dw, weight, dim * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(record_launch(c, launch_rmsnorm_rows(dout, din, dw, (long long)rows, (int)dim, eps, c->stream)));
    CUDA_TRY(cudaMemcpyAsync(out, dout, n * 4, cudaMemcpyDeviceToHost, c->stream));
    return check_device_errors(c);
}

int vox_rope_interleaved_inplace(vox_ctx* c, float* data, size_t seq_len, size_t n_heads, size_t hd,
                                 size_t pos_offset, float theta) {
    if (!c) return fail(VOX_ERR_INVALID_ARG, "context is null");
    if (hd % 2) return fail(VOX_ERR_INVALID_ARG, "head_dim must be even");  // math.rs:39
    const size_t n = seq_len * n_heads * hd;
    if (n == 0) return VOX_OK;
    if (!data) return fail(VOX_ERR_INVALID_ARG, "data is null");
    CUDA_TRY(cudaSetDevice(c->dev));
    // Angle table in f32 with libm (math.rs:52-56); the rotation runs on the GPU.
    const size_t half = hd / 2;
    std::vector<float> ct(seq_len * half), st(seq_len * half), inv(half);
    for (size_t p = 0; p < half; ++p) inv[p] = powf(theta, -((float)(2 * p)) / (float)hd);
    for (size_t t = 0; t < seq_len; ++t) {
        const float posf = (float)(pos_offset + t);
        for (size_t p = 0; p < half; ++p) {
            const float angle = posf * inv[p];
            st[t * half + p] = sinf(angle);
            ct[t * half + p] = cosf(angle);
        }
    }
    const size_t db = (n * 4 + 255) & ~size_t(255), tb = (seq_len * half * 4 + 255) & ~size_t(255);
    TRY(ensure_scratch(c, db + 2 * tb));
    unsigned char* base = static_cast<unsigned char*>(c->scratch);
    float* dd = reinterpret_cast<float*>(base);
    float* dc = reinterpret_cast<float*>(base + db);
    float* ds = reinterpret_cast<float*>(base + db + tb);
    CUDA_TRY(cudaMemcpyAsync(dd, data, n * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaMemcpyAsync(dc, ct.data(), seq_len * half * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaMemcpyAsync(ds, st.data(), seq_len * half * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(record_launch(c, launch_rope_table(dd, dc, ds, (long long)seq_len, (int)n_heads, (int)hd, c->stream)));
    CUDA_TRY(cudaMemcpyAsync(data, dd, n * 4, cudaMemcpyDeviceToHost, c->stream));
    return check_device_errors(c);
}

int vox_attention_gqa_step(vox_ctx* c, const float* q, const float* keys, const float* values,
                           const vox_attention_shape* sh, float* out) {
    if (!c || !sh || !q || !out) return fail(VOX_ERR_INVALID_ARG, "null argument");
    if (sh->n_heads == 0 || sh->n_kv_heads == 0 || sh->head_dim == 0)
        return fail(VOX_ERR_INVALID_ARG, "n_heads, n_kv_heads and head_dim must be > 0");
    if (sh->n_heads % sh->n_kv_heads) return fail(VOX_ERR_INVALID_ARG, "n_heads must be divisible by n_kv_heads");
    if (!attn_supported((int)sh->n_heads, (int)sh->n_kv_heads, (int)sh->head_dim))
        return fail(VOX_ERR_UNSUPPORTED, "attention shape not supported");
    if (sh->seq_len > (size_t)INT32_MAX / 2) return fail(VOX_ERR_UNSUPPORTED, "seq_len too large");
    if (sh->seq_len && (!keys || !values)) return fail(VOX_ERR_INVALID_ARG, "null keys/values");
    CUDA_TRY(cudaSetDevice(c->dev));
    const size_t nh = sh->n_heads, nkv = sh->n_kv_heads, hd = sh->head_dim, L = sh->seq_len;
    const size_t G = nh / nkv;
    const int nsplit = attn_splits_for((int)nkv, c->num_sms);
    auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
    const size_t kvb = al(L * nkv * hd * 4), qb = al(nh * hd * 4), pb = al(nkv * nsplit * G * (hd + 2) * 4),
                 tb = al(nkv * 4), sb = al(sizeof(KvState));
    TRY(ensure_scratch(c, 4 * kvb + 2 * qb + pb + tb + sb));
    unsigned char* base = static_cast<unsigned char*>(c->scratch);
    float* stage_k = reinterpret_cast<float*>(base);
    float* stage_v = reinterpret_cast<float*>(base + kvb);
    float* ring_k = reinterpret_cast<float*>(base + 2 * kvb);
    float* ring_v = reinterpret_cast<float*>(base + 3 * kvb);
    float* dq = reinterpret_cast<float*>(base + 4 * kvb);
    float* dout = reinterpret_cast<float*>(base + 4 * kvb + qb);
    float* dpart = reinterpret_cast<float*>(base + 4 * kvb + 2 * qb);
    unsigned* dtick = reinterpret_cast<unsigned*>(base + 4 * kvb + 2 * qb + pb);
    KvState* dst = reinterpret_cast<KvState*>(base + 4 * kvb + 2 * qb + pb + tb);
    if (L) {
        CUDA_TRY(cudaMemcpyAsync(stage_k, keys, L * nkv * hd * 4, cudaMemcpyHostToDevice, c->stream));
        CUDA_TRY(cudaMemcpyAsync(stage_v, values, L * nkv * hd * 4, cudaMemcpyHostToDevice, c->stream));
        CUDA_TRY(record_launch(c, launch_kv_scatter(stage_k, stage_v, ring_k, ring_v, (int)nkv, (int)hd, (int)L, 0,
                                                    (int)L, c->stream)));
    }
    CUDA_TRY(cudaMemcpyAsync(dq, q, nh * hd * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaMemsetAsync(dtick, 0, nkv * 4, c->stream));
    KvState* hst = reinterpret_cast<KvState*>(c->h_steps);
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    hst->len = (int32_t)L;
    hst->start = 0;
    hst->pos_offset = 0;
    CUDA_TRY(cudaMemcpyAsync(dst, hst, sizeof(KvState), cudaMemcpyHostToDevice, c->stream));
    AttnArgs at{};
    at.q = dq;
    at.k_ring = ring_k;
    at.v_ring = ring_v;
    at.n_heads = (int)nh;
    at.n_kv = (int)nkv;
    at.hd = (int)hd;
    at.cap = L ? (int)L : 1;
    at.cfg_window = (int)sh->sliding_window;
    at.st = dst;
    at.pre_append = 0;
    at.nsplit = nsplit;
    at.part = dpart;
    at.tickets = dtick;
    at.out = dout;
    at.scale = 1.0f / sqrtf((float)hd);  // ops.rs:89
    at.err = c->err;
    CUDA_TRY(record_launch(c, launch_attention(at, c->stream, false)));
    CUDA_TRY(cudaMemcpyAsync(out, dout, nh * hd * 4, cudaMemcpyDeviceToHost, c->stream));
    return check_device_errors(c);
}

}  // extern "C"

// ---- interface for the other host files (vox_internal.h) -------------------------
namespace vox {

int ctx_info(const vox_ctx* c, CtxInfo* out) {
    if (!c || !out) return fail(VOX_ERR_INVALID_ARG, "null context");
    out->device = c->dev;
    out->stream = c->stream;
    out->cfg = c->cfg;
    out->weight_dtype = c->wsize == 4 ? VOX_WEIGHTS_F32 : VOX_WEIGHTS_BF16;
    out->dim = c->cfg.dim;
    out->vocab = c->opt.vocab;
    out->n_layers = c->layers.size();
    out->max_pos = c->max_pos;
    return VOX_OK;
}

int ctx_model_ready(vox_ctx* c, vox_kv* kv) {
    TRY(model_ready(c, kv));
    return single_stream(kv);
}

void release_step_graphs(StepGraphs* g) {
    if (!g) return;
    if (g->full) cudaGraphExecDestroy(g->full);
    if (g->short_attn) cudaGraphExecDestroy(g->short_attn);
    *g = StepGraphs{};
}

int capture_adapter_graphs(vox_ctx* c, vox_kv* kv, const float* adapter, int adapter_cap, StepGraphs* g) {
    TRY(ctx_model_ready(c, kv));
    if (!adapter || adapter_cap <= 0) return fail(VOX_ERR_INVALID_ARG, "adapter ring missing");
    CUDA_TRY(cudaSetDevice(c->dev));
    release_step_graphs(g);
    TRY(capture_step(c, kv, false, &g->full, &g->k_full, adapter, adapter_cap));
    if (attn_cluster_size((int)c->cfg.n_heads, (int)c->cfg.n_kv_heads, (int)c->cfg.head_dim) > 0)
        TRY(capture_step(c, kv, true, &g->short_attn, &g->k_short, adapter, adapter_cap));
    g->adapter = adapter;
    g->adapter_cap = adapter_cap;
    return VOX_OK;
}

int run_step_graphs(vox_ctx* c, vox_kv* kv, const StepGraphs& g, const int32_t* fixed, size_t n_fixed,
                    size_t pos0, int32_t greedy_tok, size_t n_greedy, int32_t* tokens_out) {
    TRY(ctx_model_ready(c, kv));
    if (!g.full) return fail(VOX_ERR_INVALID_ARG, "step graphs not captured");
    if (n_fixed + n_greedy == 0) return VOX_OK;
    if (n_fixed && !fixed) return fail(VOX_ERR_INVALID_ARG, "tokens are null");
    if (pos0 + n_fixed + n_greedy > (size_t)c->max_pos)
        return fail(VOX_ERR_RANGE, "positions beyond max_positions %d", c->max_pos);
    for (size_t i = 0; i < n_fixed; ++i)
        if (fixed[i] < 0 || (size_t)fixed[i] >= c->opt.vocab)
            return fail(VOX_ERR_RANGE, "token %d outside the vocabulary", fixed[i]);
    if (n_greedy && (greedy_tok < 0 || (size_t)greedy_tok >= c->opt.vocab))
        return fail(VOX_ERR_RANGE, "token %d outside the vocabulary", greedy_tok);
    CUDA_TRY(cudaSetDevice(c->dev));
    if (n_fixed >= 2 && prefill_batched_supported(c)) {  // the cache's mirror follows inside
        TRY(prefill_batched(c, kv, fixed, n_fixed, pos0, g.adapter, g.adapter_cap));
        pos0 += n_fixed;
        fixed = nullptr;
        n_fixed = 0;
        if (n_greedy == 0) return VOX_OK;
    }
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    TRY(ensure_host_steps(c, n_fixed + 1 + n_greedy));
    auto launch = [&](size_t live) -> int {
        const bool use_short = g.short_attn && live <= (size_t)attn_cluster_max_tokens();
        CUDA_TRY(cudaGraphLaunch(use_short ? g.short_attn : g.full, c->stream));
        c->launches += use_short ? g.k_short : g.k_full;
        return VOX_OK;
    };
    for (size_t i = 0; i < n_fixed; ++i) {
        StepState* hs = c->h_steps + i;
        std::memset(hs, 0, sizeof(StepState));
        hs->pos = (int64_t)(pos0 + i);
        hs->tok = fixed[i];
        CUDA_TRY(cudaMemcpyAsync(c->step, hs, sizeof(StepState), cudaMemcpyHostToDevice, c->stream));
        TRY(launch(live_tokens_after(c, kv, i + 1)));
    }
    int32_t* tok_hist = reinterpret_cast<int32_t*>(c->h_steps + n_fixed + 1);
    if (n_greedy) {
        StepState* hs = c->h_steps + n_fixed;
        std::memset(hs, 0, sizeof(StepState));
        hs->pos = (int64_t)(pos0 + n_fixed);
        hs->tok = greedy_tok;
        hs->greedy = 1;
        hs->advance = 1;
        CUDA_TRY(cudaMemcpyAsync(c->step, hs, sizeof(StepState), cudaMemcpyHostToDevice, c->stream));
        for (size_t i = 0; i < n_greedy; ++i) {
            TRY(launch(live_tokens_after(c, kv, n_fixed + i + 1)));
            CUDA_TRY(cudaMemcpyAsync(tok_hist + i, c->tok_out, 4, cudaMemcpyDeviceToHost, c->stream));
        }
    }
    TRY(check_device_errors(c));
    for (size_t i = 0; i < n_fixed + n_greedy; ++i) mirror_single_append_all(kv);
    if (tokens_out && n_greedy) std::memcpy(tokens_out, tok_hist, n_greedy * 4);
    return VOX_OK;
}

}  // namespace vox
