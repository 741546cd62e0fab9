// vox_tp.cpp -- tensor-parallel single-stream decoding (one process per GPU).
//
// Each of tp_size ranks holds one shard of every layer:
//   q|k|v rows of its q heads and kv heads (column-parallel: n_heads / tp and
//   n_kv_heads / tp heads per rank), the matching columns of wo (row-parallel),
//   w1|w3 rows hidden / tp (column-parallel), the matching columns of w2
//   (row-parallel), and vocab / tp rows of the LM head.
// The cache holds the rank's kv heads only.  After o-proj and after w2 the
// 3072-wide f32 partial sums are all-reduced with NCCL (sum) inside the
// step's CUDA graph; rank 0 adds the residual before the reduction, so the
// reduced vector is residual + sum of partials on every rank.  The LM head's
// argmax is one 64-bit all-reduce (max) of an order-preserving (value,
// index) key.  Embedding, RMSNorms and residual stream are replicated.
//
// After vox_tp_connect_peers the exchange runs over NVLink peer memory
// instead, fused into the GEMVs: the o-proj / w2 epilogue stores its rows
// into a receive slot of every rank and bumps each rank's arrival counter
// (system-scope fence + atomic); the next GEMV's prologue waits (bounded) for
// all ranks' arrivals and sums the slots in rank order, so every rank holds
// bit-identical activations, while its producer warp already streams
// weights.  The argmax keys travel the same way in one kernel.  The areas
// are mapped with CUDA IPC (one process per GPU).
//
// The per-rank kernels are the single-stream ones (vox_gemv.cu,
// vox_attention.cu) run on the local shapes.  NCCL is loaded at run time
// (dlopen of libnccl.so.2), so the library itself does not depend on it.
#include <dlfcn.h>
#include <math.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "../../include/vox_decoder.h"
#include "vox_host.h"
#include "vox_kernels.h"
#include "vox_watchdog.h"

using namespace vox;

#define TP_CUDA(expr)                                                                               \
    do {                                                                                            \
        cudaError_t e_ = (expr);                                                                    \
        if (e_ != cudaSuccess)                                                                      \
            return report_errorf(e_ == cudaErrorMemoryAllocation ? VOX_ERR_OOM : VOX_ERR_CUDA,     \
                                 "%s failed: %s", #expr, cudaGetErrorString(e_));                  \
    } while (0)

#define TP_TRY(expr)                   \
    do {                               \
        int rc_ = (expr);              \
        if (rc_ != VOX_OK) return rc_; \
    } while (0)

namespace {

struct NcclApi {
    bool ok = false;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    // watchdog (optional symbols): poll for asynchronous errors, abort a stuck communicator
    ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
};

int nccl(const NcclApi** out) {
    static NcclApi api;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (h) {
            api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
            api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
            api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
            api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
            api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
            api.comm_get_async_error =
                reinterpret_cast<decltype(api.comm_get_async_error)>(dlsym(h, "ncclCommGetAsyncError"));
            api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(dlsym(h, "ncclCommAbort"));
            api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.comm_destroy &&
                     api.error_string;
        }
    }
    if (!api.ok) return report_errorf(VOX_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
    *out = &api;
    return VOX_OK;
}

#define TP_NCCL(api, expr)                                                                          \
    do {                                                                                            \
        ncclResult_t r_ = (expr);                                                                   \
        if (r_ != ncclSuccess)                                                                      \
            return report_errorf(VOX_ERR_CUDA, "%s failed: %s", #expr, (api)->error_string(r_));    \
    } while (0)

struct TpLayer {
    uint16_t* wqkv = nullptr;  // [q_l + 2 kv_l, dim]
    uint16_t* wo = nullptr;    // [dim, q_l]
    uint16_t* w13 = nullptr;   // [2 hid_l, dim], rows interleaved w1 / w3
    uint16_t* w2 = nullptr;    // [dim, hid_l]
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
    bool ready = false;
};

}  // namespace

struct vox_tp {
    vox_decoder_config cfg{};
    vox_ctx_options opt{};
    vox_tp_shard sh{};
    int dev = 0, num_sms = 148;
    cudaStream_t stream = nullptr;
    ncclComm_t comm = nullptr;
    const NcclApi* api = nullptr;
    std::vector<TpLayer> layers;
    uint16_t* embed = nullptr;  // [vocab, dim], replicated
    uint16_t* head = nullptr;   // [vocab_l, dim]
    float* final_norm = nullptr;
    bool embed_ready = false, head_ready = false;
    float *rope_cos = nullptr, *rope_sin = nullptr;
    int max_pos = 0;
    float *hid = nullptr, *hmid = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr, *logits = nullptr,
          *zeros = nullptr;
    ArgmaxPart* am_part = nullptr;
    float* attn_part = nullptr;
    unsigned* tickets = nullptr;
    int nsplit = 1;
    StepState* step = nullptr;
    int32_t* tok_out = nullptr;
    unsigned* err = nullptr;
    unsigned long long* key = nullptr;
    // cache of this rank's kv heads
    size_t window = 0, cap = 0;
    float *k = nullptr, *v = nullptr;  // [n_layers, kv_l heads, cap, hd]
    KvState* dstate = nullptr;
    std::vector<HostKv> hs;
    GemvPlan p_qkv{}, p_o{}, p_w13{}, p_w2{}, p_head{};
    cudaGraphExec_t graph = nullptr;
    cudaGraphExec_t graph_short = nullptr;  // same step, cluster attention (short contexts)
    uint64_t graph_kernels = 0, launches = 0;
    StepState* h_steps = nullptr;  // pinned
    size_t h_steps_cap = 0;
    int32_t* h_tok = nullptr;       // pinned
    unsigned* h_err = nullptr;      // pinned
    cudaEvent_t ev[8] = {};
    // exchange over peer memory (after vox_tp_connect_peers); NCCL otherwise
    XchArea xa{};
    unsigned char* xch_own = nullptr;           // this rank's exchange area (IPC-exported)
    std::vector<unsigned char*> peer_maps;      // opened IPC mappings of the other ranks' areas
    unsigned char** xch_ptrs = nullptr;         // device array [size]: every rank's area
    unsigned long long* tp_steps = nullptr;     // steps completed (device)
    bool p2p = false;
    // watchdog: every host wait on the stream is bounded by timeout_ms; a
    // step that does not finish in time (a rank stopped) aborts the NCCL
    // communicator and leaves the context broken (every later call fails)
    unsigned timeout_ms = 30000;
    bool broken = false;
    size_t layer_elems() const { return sh.n_kv_heads * cap * cfg.head_dim; }
};

namespace {

// Wait for the stream with the watchdog (vox_watchdog.h): poll, abort the
// communicator on an asynchronous NCCL error or after timeout_ms.
int tp_wait(vox_tp* t) {
    cudaError_t stream_err = cudaSuccess;
    ncclResult_t async_err = ncclSuccess;
    auto query = [&]() {
        stream_err = cudaStreamQuery(t->stream);
        return stream_err == cudaSuccess ? 0 : stream_err == cudaErrorNotReady ? 1 : 2;
    };
    auto async_error = [&]() {
        if (!t->comm || !t->api || !t->api->comm_get_async_error) return false;
        ncclResult_t ar = ncclSuccess;
        if (t->api->comm_get_async_error(t->comm, &ar) != ncclSuccess) return false;
        async_err = ar;
        return ar != ncclSuccess && ar != ncclInProgress;
    };
    auto abort = [&]() {
        t->broken = true;
        if (t->comm && t->api && t->api->comm_abort) t->api->comm_abort(t->comm);
        if (t->api && t->api->comm_abort) t->comm = nullptr;
    };
    switch (watchdog_wait(query, async_error, abort, t->timeout_ms)) {
        case kWatchdogIdle:
            return VOX_OK;
        case kWatchdogAsyncError:
            return report_errorf(VOX_ERR_CUDA, "NCCL reported an asynchronous error (%s); communicator aborted",
                                 t->api->error_string(async_err));
        case kWatchdogTimeout:
            return report_errorf(VOX_ERR_DEVICE_TIMEOUT,
                                 "tensor-parallel step not finished after %u ms (a rank stopped?); the context is "
                                 "no longer usable", t->timeout_ms);
        default:
            return report_errorf(VOX_ERR_CUDA, "tensor-parallel stream failed: %s", cudaGetErrorString(stream_err));
    }
}

int check_errors(vox_tp* t) {
    TP_CUDA(cudaMemcpyAsync(t->h_err, t->err, sizeof(unsigned), cudaMemcpyDeviceToHost, t->stream));
    TP_TRY(tp_wait(t));
    const unsigned bits = *t->h_err;
    if (!bits) return VOX_OK;
    TP_CUDA(cudaMemsetAsync(t->err, 0, sizeof(unsigned), t->stream));
    TP_CUDA(cudaMemsetAsync(t->tickets, 0, t->sh.n_kv_heads * sizeof(unsigned), t->stream));
    TP_TRY(tp_wait(t));
    if (bits & ERR_PEER_WAIT) t->broken = true;  // the ranks' exchange counters no longer agree
    if (bits & (ERR_FULL_WAIT | ERR_EMPTY_WAIT | ERR_DRAIN_WAIT | ERR_PEER_WAIT))
        return report_errorf(VOX_ERR_DEVICE_TIMEOUT, "a bounded wait inside a kernel expired (bits 0x%x)", bits);
    if (bits & ERR_POS_RANGE) return report_errorf(VOX_ERR_RANGE, "position beyond the RoPE table");
    if (bits & ERR_TOKEN_RANGE) return report_errorf(VOX_ERR_RANGE, "token id outside the vocabulary");
    return report_errorf(VOX_ERR_CUDA, "device error bits 0x%x", bits);
}

GemvArgs base(vox_tp* t) {
    GemvArgs a{};
    a.step = t->step;
    a.eps = t->cfg.norm_eps;
    a.err = t->err;
    a.xch_out = a.xch_in = -1;
    if (t->p2p) {
        a.xch = t->xch_ptrs;
        a.xa = t->xa;
        a.tp_steps = t->tp_steps;
    }
    return a;
}

// Exchange points: 2l after layer l's o-proj, 2l + 1 after its w2.
int point_after_o(size_t l) { return (int)(2 * l); }
int point_after_w2(size_t l) { return (int)(2 * l + 1); }

// One layer (decoder.rs:88-155) on this rank's shard, two all-reduces.
int enqueue_layer(vox_tp* t, size_t l, bool short_attn) {
    const TpLayer& L = t->layers[l];
    const vox_tp_shard& s = t->sh;
    float* kr = t->k + l * t->layer_elems();
    float* vr = t->v + l * t->layer_elems();
    KvState* st = t->dstate + l;
    const int cap = (int)t->cap, win = (int)t->window, hd = (int)t->cfg.head_dim;
    const size_t dim = t->cfg.dim;

    GemvArgs a = base(t);
    a.W = L.wqkv;
    if (l == 0) {
        a.x_embed = t->embed;
        a.vocab = (int)s.vocab;
        a.x_copy_out = t->hid;
    } else if (t->p2p) {  // x = sum of the ranks' w2 partials of layer l - 1
        a.xch_in = point_after_w2(l - 1);
        a.xch_arrivals = (unsigned long long)s.size * t->p_w2.grid;
        a.x_copy_out = t->hid;
    } else {
        a.x = t->hid;
    }
    a.norm_w = L.attn_norm;
    a.y = t->q;
    a.q_dim = (int)(s.n_heads * hd);
    a.kv_dim = (int)(s.n_kv_heads * hd);
    a.head_dim = hd;
    a.rope_cos = t->rope_cos;
    a.rope_sin = t->rope_sin;
    a.max_pos = t->max_pos;
    a.k_ring = kr;
    a.v_ring = vr;
    a.ring_cap = cap;
    a.kv_window = win;
    a.kv_state = st;
    gemv_set_prefetch(a, L.wo, t->p_o, 2);
    TP_CUDA(launch_gemv(t->p_qkv, a, EPI_QKV, t->stream, true));

    AttnArgs at{};
    at.q = t->q;
    at.k_ring = kr;
    at.v_ring = vr;
    at.n_heads = (int)s.n_heads;
    at.n_kv = (int)s.n_kv_heads;
    at.hd = hd;
    at.cap = cap;
    at.cfg_window = (int)t->cfg.sliding_window;
    at.st = st;
    at.pre_append = 1;
    at.kv_window = win;
    at.nsplit = t->nsplit;
    at.part = t->attn_part;
    at.tickets = t->tickets;
    at.out = t->attn;
    at.scale = 1.0f / sqrtf((float)hd);
    at.err = t->err;
    TP_CUDA(short_attn ? launch_attention_cluster(at, t->stream, true) : launch_attention(at, t->stream, true));

    // o-proj partial (+ residual on rank 0), commit of the append, all-reduce
    a = base(t);
    a.W = L.wo;
    a.x = t->attn;
    a.y = t->hmid;
    a.resid = s.rank == 0 ? t->hid : t->zeros;
    a.kv_commit = st;
    a.kv_window = win;
    a.ring_cap = cap;
    if (t->p2p) a.xch_out = point_after_o(l);
    gemv_set_prefetch(a, L.w13, t->p_w13, 2);
    TP_CUDA(launch_gemv(t->p_o, a, EPI_RESID, t->stream, true));
    if (!t->p2p)
        TP_NCCL(t->api, t->api->all_reduce(t->hmid, t->hmid, dim, ncclFloat32, ncclSum, t->comm, t->stream));

    a = base(t);
    a.W = L.w13;
    if (t->p2p) {
        a.xch_in = point_after_o(l);
        a.xch_arrivals = (unsigned long long)s.size * t->p_o.grid;
        a.x_copy_out = t->hmid;  // the reduced vector, for w2's residual
    } else {
        a.x = t->hmid;
    }
    a.norm_w = L.ffn_norm;
    a.y = t->act;
    gemv_set_prefetch(a, L.w2, t->p_w2, 2);
    TP_CUDA(launch_gemv(t->p_w13, a, EPI_SWIGLU, t->stream, true));

    a = base(t);
    a.W = L.w2;
    a.x = t->act;
    a.y = t->hid;
    a.resid = s.rank == 0 ? t->hmid : t->zeros;
    if (t->p2p) a.xch_out = point_after_w2(l);
    if (l + 1 < t->layers.size())
        gemv_set_prefetch(a, t->layers[l + 1].wqkv, t->p_qkv, 2);
    else if (t->head)
        gemv_set_prefetch(a, t->head, t->p_head, 2);
    TP_CUDA(launch_gemv(t->p_w2, a, EPI_RESID, t->stream, true));
    if (!t->p2p)
        TP_NCCL(t->api, t->api->all_reduce(t->hid, t->hid, dim, ncclFloat32, ncclSum, t->comm, t->stream));
    return VOX_OK;
}

int enqueue_head(vox_tp* t) {
    GemvArgs a = base(t);
    a.W = t->head;
    if (t->p2p) {
        a.xch_in = point_after_w2(t->layers.size() - 1);
        a.xch_arrivals = (unsigned long long)t->sh.size * t->p_w2.grid;
    } else {
        a.x = t->hid;
    }
    a.norm_w = t->final_norm;
    a.y = t->logits;
    a.am_part = t->am_part;
    TP_CUDA(launch_gemv(t->p_head, a, EPI_ARGMAX, t->stream, true));
    if (t->p2p) {
        TP_CUDA(launch_tp_argmax_xch(t->am_part, t->p_head.grid, (long long)t->sh.vocab_begin, t->xch_ptrs, t->xa,
                                     t->tp_steps, t->step, t->tok_out, t->err, t->stream, true));
        return VOX_OK;
    }
    TP_CUDA(launch_tp_argmax_key(t->am_part, t->p_head.grid, (long long)t->sh.vocab_begin, t->key, t->stream, true));
    TP_NCCL(t->api, t->api->all_reduce(t->key, t->key, 1, ncclUint64, ncclMax, t->comm, t->stream));
    TP_CUDA(launch_tp_argmax_apply(t->key, t->step, t->tok_out, t->stream));
    return VOX_OK;
}

// The step as a CUDA graph.  As on one GPU, a second graph runs attention as
// one thread-block cluster per local kv head for contexts up to
// attn_cluster_max_tokens(); every rank decodes the same tokens, so every rank
// picks the same graph and the collectives stay in step.
int capture_step(vox_tp* t, bool short_attn, cudaGraphExec_t* out) {
    TP_CUDA(cudaStreamBeginCapture(t->stream, cudaStreamCaptureModeThreadLocal));
    int rc = VOX_OK;
    for (size_t l = 0; l < t->layers.size() && rc == VOX_OK; ++l) rc = enqueue_layer(t, l, short_attn);
    if (rc == VOX_OK) rc = enqueue_head(t);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(t->stream, &g);
    if (rc != VOX_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    TP_CUDA(e);
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    TP_CUDA(e);
    return VOX_OK;
}

int build_graph(vox_tp* t) {
    if (t->graph) return VOX_OK;
    TP_TRY(capture_step(t, false, &t->graph));
    if (attn_cluster_size((int)t->sh.n_heads, (int)t->sh.n_kv_heads, (int)t->cfg.head_dim) > 0)
        TP_TRY(capture_step(t, true, &t->graph_short));
    t->graph_kernels = t->layers.size() * 5 + (t->p2p ? 2 : 3);
    return VOX_OK;
}

void release_graphs(vox_tp* t) {
    if (t->graph) cudaGraphExecDestroy(t->graph);
    if (t->graph_short) cudaGraphExecDestroy(t->graph_short);
    t->graph = t->graph_short = nullptr;
}

int ready(vox_tp* t) {
    if (!t) return report_errorf(VOX_ERR_INVALID_ARG, "tensor-parallel context is null");
    if (t->broken)
        return report_errorf(VOX_ERR_DEVICE_TIMEOUT, "a previous step timed out (a rank stopped); destroy this context");
    if (!t->embed_ready || !t->head_ready) return report_errorf(VOX_ERR_NOT_READY, "embedding or LM head not uploaded");
    for (size_t l = 0; l < t->layers.size(); ++l)
        if (!t->layers[l].ready) return report_errorf(VOX_ERR_NOT_READY, "layer %zu weights not uploaded", l);
    TP_CUDA(cudaSetDevice(t->dev));
    return build_graph(t);
}

int ensure_host_steps(vox_tp* t, size_t n) {
    if (n <= t->h_steps_cap) return VOX_OK;
    if (t->h_steps) {
        TP_CUDA(cudaStreamSynchronize(t->stream));
        cudaFreeHost(t->h_steps);
        t->h_steps = nullptr;
        t->h_steps_cap = 0;
    }
    size_t c = 1024;
    while (c < n) c <<= 1;
    TP_CUDA(cudaMallocHost(&t->h_steps, c * sizeof(StepState)));
    t->h_steps_cap = c;
    return VOX_OK;
}

// `steps` = this step's index + 1 in the current call: the attention reads
// the cache after that many more appends.
int launch_step(vox_tp* t, size_t steps) {
    size_t live = 0;
    for (const HostKv& h : t->hs) live = std::max(live, h.len);
    live = std::min(live + steps, t->window);
    if (t->cfg.sliding_window > 0) live = std::min(live, (size_t)t->cfg.sliding_window);
    const bool use_short = t->graph_short && live <= (size_t)attn_cluster_max_tokens();
    TP_CUDA(cudaGraphLaunch(use_short ? t->graph_short : t->graph, t->stream));
    t->launches += t->graph_kernels;
    return VOX_OK;
}

void mirror(vox_tp* t, size_t n_steps) {
    for (HostKv& h : t->hs)
        for (size_t i = 0; i < n_steps; ++i) host_append(h, 1, t->window, t->cap);
}

int alloc_layer(vox_tp* t, TpLayer& L) {
    if (L.wqkv) return VOX_OK;
    const vox_tp_shard& s = t->sh;
    const size_t dim = t->cfg.dim, hd = t->cfg.head_dim;
    const size_t q_l = s.n_heads * hd, kv_l = s.n_kv_heads * hd;
    TP_CUDA(dalloc(&L.wqkv, (q_l + 2 * kv_l) * dim));
    TP_CUDA(dalloc(&L.wo, dim * q_l));
    TP_CUDA(dalloc(&L.w13, 2 * s.hidden * dim));
    TP_CUDA(dalloc(&L.w2, dim * s.hidden));
    TP_CUDA(dalloc(&L.attn_norm, dim));
    TP_CUDA(dalloc(&L.ffn_norm, dim));
    return VOX_OK;
}

}  // namespace

extern "C" {

int vox_tp_shard_of(const vox_decoder_config* cfg, size_t vocab, int tp_rank, int tp_size, vox_tp_shard* out) {
    if (!cfg || !out) return report_errorf(VOX_ERR_INVALID_ARG, "null argument");
    const int v = vox_config_validate(cfg);
    if (v != VOX_OK) return v;
    if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size)
        return report_errorf(VOX_ERR_INVALID_ARG, "rank %d of %d", tp_rank, tp_size);
    const size_t T = (size_t)tp_size;
    if (cfg->n_kv_heads % T || cfg->n_heads % T || cfg->hidden_dim % T || vocab % T)
        return report_errorf(VOX_ERR_UNSUPPORTED,
                             "tensor parallel %d needs n_kv_heads, n_heads, hidden_dim and vocab divisible by it",
                             tp_size);
    vox_tp_shard s{};
    s.rank = tp_rank;
    s.size = tp_size;
    s.n_heads = cfg->n_heads / T;
    s.n_kv_heads = cfg->n_kv_heads / T;
    s.hidden = cfg->hidden_dim / T;
    s.vocab = vocab;
    s.vocab_local = vocab / T;
    // whole kv groups stay together: q heads [r*nh, (r+1)*nh) attend to kv heads [r*nkv, (r+1)*nkv)
    s.q_head_begin = (size_t)tp_rank * s.n_heads;
    s.kv_head_begin = (size_t)tp_rank * s.n_kv_heads;
    s.hidden_begin = (size_t)tp_rank * s.hidden;
    s.vocab_begin = (size_t)tp_rank * s.vocab_local;
    *out = s;
    return VOX_OK;
}

int vox_tp_unique_id(unsigned char id[128]) {
    if (!id) return report_errorf(VOX_ERR_INVALID_ARG, "id is null");
    const NcclApi* api = nullptr;
    TP_TRY(nccl(&api));
    ncclUniqueId u;
    TP_NCCL(api, api->get_unique_id(&u));
    static_assert(sizeof(u.internal) == 128, "NCCL unique id size");
    memcpy(id, u.internal, 128);
    return VOX_OK;
}

void vox_tp_destroy(vox_tp* t) {
    if (!t) return;
    cudaSetDevice(t->dev);
    if (t->stream) {
        const unsigned keep = t->timeout_ms;
        if (tp_wait(t) != VOX_OK) cudaGetLastError();  // bounded: aborts a stuck communicator
        t->timeout_ms = keep;
        cudaStreamSynchronize(t->stream);
    }
    release_graphs(t);  // they hold NCCL calls: release before the communicator
    if (t->comm && t->api) t->api->comm_destroy(t->comm);
    for (unsigned char* m : t->peer_maps)
        if (m) cudaIpcCloseMemHandle(m);
    if (t->xch_ptrs) cudaFree(t->xch_ptrs);
    if (t->xch_own) cudaFree(t->xch_own);
    if (t->tp_steps) cudaFree(t->tp_steps);
    for (auto& L : t->layers) {
        void* p[] = {L.wqkv, L.wo, L.w13, L.w2, L.attn_norm, L.ffn_norm};
        for (void* q : p)
            if (q) cudaFree(q);
    }
    void* p[] = {t->embed, t->head, t->final_norm, t->rope_cos, t->rope_sin, t->hid, t->hmid, t->q, t->attn,
                 t->act, t->logits, t->zeros, t->am_part, t->attn_part, t->tickets, t->step, t->tok_out, t->err,
                 t->key, t->k, t->v, t->dstate};
    for (void* q : p)
        if (q) cudaFree(q);
    if (t->h_steps) cudaFreeHost(t->h_steps);
    if (t->h_tok) cudaFreeHost(t->h_tok);
    if (t->h_err) cudaFreeHost(t->h_err);
    for (auto& e : t->ev)
        if (e) cudaEventDestroy(e);
    if (t->stream) cudaStreamDestroy(t->stream);
    delete t;
}

int vox_tp_create(const vox_decoder_config* cfg, const vox_ctx_options* opt, int tp_rank, int tp_size,
                  const unsigned char id[128], vox_tp** out) {
    if (!out || !id) return report_errorf(VOX_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    vox_ctx_options o{};
    if (opt) o = *opt;
    if (o.n_layers == 0) o.n_layers = 1;
    if (o.max_positions == 0) o.max_positions = 32768;
    if (o.vocab == 0) return report_errorf(VOX_ERR_INVALID_ARG, "tensor-parallel decoding needs a vocabulary");
    if (o.weight_dtype != VOX_WEIGHTS_BF16)
        return report_errorf(VOX_ERR_UNSUPPORTED, "tensor-parallel decoding holds bf16 weights");
    if (o.vocab > (size_t)INT32_MAX || o.max_positions > (size_t)(1 << 24))
        return report_errorf(VOX_ERR_UNSUPPORTED, "vocab or max_positions too large");
    vox_tp_shard sh{};
    TP_TRY(vox_tp_shard_of(cfg, o.vocab, tp_rank, tp_size, &sh));
    const size_t dim = cfg->dim, hd = cfg->head_dim;
    const size_t q_l = sh.n_heads * hd, kv_l = sh.n_kv_heads * hd;
    if (hd % 2 || !gemv_supported((int)dim, 2) || !gemv_supported((int)q_l, 2) || !gemv_supported((int)sh.hidden, 2) ||
        !attn_supported((int)sh.n_heads, (int)sh.n_kv_heads, (int)hd))
        return report_errorf(VOX_ERR_UNSUPPORTED, "shard shapes not supported by the kernels");
    const NcclApi* api = nullptr;
    TP_TRY(nccl(&api));

    int ndev = 0;
    TP_CUDA(cudaGetDeviceCount(&ndev));
    if (o.device < 0 || o.device >= ndev) return report_errorf(VOX_ERR_INVALID_ARG, "device %d not present", o.device);
    TP_CUDA(cudaSetDevice(o.device));
    cudaDeviceProp prop;
    TP_CUDA(cudaGetDeviceProperties(&prop, o.device));
    if (prop.major != 10)
        return report_errorf(VOX_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", o.device,
                             prop.major, prop.minor);

    vox_tp* t = new vox_tp();
    t->cfg = *cfg;
    t->opt = o;
    t->sh = sh;
    t->dev = o.device;
    t->num_sms = prop.multiProcessorCount;
    t->api = api;
    t->max_pos = (int)o.max_positions;
    t->window = cfg->sliding_window;
    t->cap = cfg->sliding_window;
    t->layers.resize(o.n_layers);
    t->hs.assign(o.n_layers, HostKv{});
    auto bail = [&](int rc) {
        vox_tp_destroy(t);
        return rc;
    };
#define CREATE_TRY(expr)                                                                                 \
    do {                                                                                                 \
        cudaError_t e_ = (expr);                                                                         \
        if (e_ != cudaSuccess)                                                                           \
            return bail(report_errorf(e_ == cudaErrorMemoryAllocation ? VOX_ERR_OOM : VOX_ERR_CUDA,      \
                                      "%s failed: %s", #expr, cudaGetErrorString(e_)));                  \
    } while (0)
    CREATE_TRY(gemv_prepare(t->dev));
    CREATE_TRY(attn_prepare(t->dev));
    CREATE_TRY(cudaStreamCreateWithFlags(&t->stream, cudaStreamNonBlocking));
    for (auto& e : t->ev) CREATE_TRY(cudaEventCreate(&e));
    const int dimi = (int)dim, hidi = (int)sh.hidden;
    // o-proj and w2 end in the peer exchange: the wide shape (fewer CTAs, fewer
    // arrivals per exchange); q|k|v and w1|w3 in the paired shape (TP 2:
    // 1.719 vs 1.752-1.766 ms per token).
    t->p_qkv = plan_gemv((int)(q_l + 2 * kv_l), dimi, 2, 2, t->num_sms, 1, kGemvPaired);
    t->p_o = plan_gemv(dimi, (int)q_l, 1, 2, t->num_sms, 1);
    t->p_w13 = plan_gemv(2 * hidi, dimi, 2, 2, t->num_sms, 1, kGemvPaired);
    t->p_w2 = plan_gemv(dimi, hidi, 1, 2, t->num_sms, 1);
    t->p_head = plan_gemv((int)sh.vocab_local, dimi, 1, 2, t->num_sms, 1);
    for (const GemvPlan* p : {&t->p_qkv, &t->p_o, &t->p_w13, &t->p_w2, &t->p_head})
        if (p->grid < 1 || p->smem > gemv_max_smem())
            return bail(report_errorf(VOX_ERR_UNSUPPORTED, "no GEMV plan for a shard shape"));
    const size_t G = sh.n_heads / sh.n_kv_heads;
    t->nsplit = attn_max_splits();
    CREATE_TRY(dalloc(&t->hid, dim));
    CREATE_TRY(dalloc(&t->hmid, dim));
    CREATE_TRY(dalloc(&t->zeros, dim));
    CREATE_TRY(cudaMemset(t->zeros, 0, dim * 4));
    CREATE_TRY(dalloc(&t->q, q_l));
    CREATE_TRY(dalloc(&t->attn, q_l));
    CREATE_TRY(dalloc(&t->act, sh.hidden));
    CREATE_TRY(dalloc(&t->logits, sh.vocab_local));
    CREATE_TRY(dalloc(&t->am_part, (size_t)t->num_sms));
    CREATE_TRY(dalloc(&t->attn_part, sh.n_kv_heads * t->nsplit * G * (hd + 2)));
    CREATE_TRY(dalloc(&t->tickets, sh.n_kv_heads));
    CREATE_TRY(cudaMemset(t->tickets, 0, sh.n_kv_heads * sizeof(unsigned)));
    CREATE_TRY(dalloc(&t->step, 1));
    CREATE_TRY(cudaMemset(t->step, 0, sizeof(StepState)));
    CREATE_TRY(dalloc(&t->tok_out, 1));
    CREATE_TRY(dalloc(&t->err, 1));
    CREATE_TRY(cudaMemset(t->err, 0, sizeof(unsigned)));
    CREATE_TRY(dalloc(&t->key, 1));
    CREATE_TRY(dalloc(&t->k, o.n_layers * t->layer_elems()));
    CREATE_TRY(dalloc(&t->v, o.n_layers * t->layer_elems()));
    CREATE_TRY(dalloc(&t->dstate, o.n_layers));
    CREATE_TRY(cudaMemset(t->dstate, 0, o.n_layers * sizeof(KvState)));
    t->xa.rank = tp_rank;
    t->xa.size = tp_size;
    t->xa.points = (int)(2 * o.n_layers);
    t->xa.dim = (int)dim;
    CREATE_TRY(cudaMalloc(&t->xch_own, t->xa.bytes()));
    CREATE_TRY(cudaMemset(t->xch_own, 0, t->xa.bytes()));
    CREATE_TRY(dalloc(&t->tp_steps, 1));
    CREATE_TRY(cudaMemset(t->tp_steps, 0, sizeof(unsigned long long)));
    CREATE_TRY(cudaMallocHost(&t->h_tok, 4));
    CREATE_TRY(cudaMallocHost(&t->h_err, sizeof(unsigned)));
    if (ensure_host_steps(t, 1024) != VOX_OK) return bail(VOX_ERR_OOM);
    {
        // RoPE table (math.rs:52-56), as the single-device context builds it
        const size_t half = hd / 2, n = (size_t)t->max_pos * half;
        std::vector<float> ct(n), stb(n), inv(half);
        for (size_t p = 0; p < half; ++p) inv[p] = powf(cfg->rope_theta, -((float)(2 * p)) / (float)hd);
        for (size_t pos = 0; pos < (size_t)t->max_pos; ++pos)
            for (size_t p = 0; p < half; ++p) {
                const float angle = (float)pos * inv[p];
                stb[pos * half + p] = sinf(angle);
                ct[pos * half + p] = cosf(angle);
            }
        CREATE_TRY(dalloc(&t->rope_cos, n));
        CREATE_TRY(dalloc(&t->rope_sin, n));
        CREATE_TRY(cudaMemcpy(t->rope_cos, ct.data(), n * 4, cudaMemcpyHostToDevice));
        CREATE_TRY(cudaMemcpy(t->rope_sin, stb.data(), n * 4, cudaMemcpyHostToDevice));
    }
#undef CREATE_TRY
    ncclUniqueId u;
    memcpy(u.internal, id, 128);
    const ncclResult_t r = api->comm_init_rank(&t->comm, tp_size, u, tp_rank);
    if (r != ncclSuccess) {
        t->comm = nullptr;
        return bail(report_errorf(VOX_ERR_CUDA, "ncclCommInitRank failed: %s", api->error_string(r)));
    }
    *out = t;
    return VOX_OK;
}

int vox_tp_ipc_handle(vox_tp* t, unsigned char out[64]) {
    if (!t || !out) return report_errorf(VOX_ERR_INVALID_ARG, "null argument");
    TP_CUDA(cudaSetDevice(t->dev));
    cudaIpcMemHandle_t h;
    TP_CUDA(cudaIpcGetMemHandle(&h, t->xch_own));
    static_assert(sizeof(h) == 64, "CUDA IPC handle size");
    memcpy(out, &h, 64);
    return VOX_OK;
}

int vox_tp_connect_peers(vox_tp* t, const unsigned char* handles) {
    if (!t || !handles) return report_errorf(VOX_ERR_INVALID_ARG, "null argument");
    if (t->p2p) return VOX_OK;
    TP_CUDA(cudaSetDevice(t->dev));
    TP_CUDA(cudaStreamSynchronize(t->stream));
    const int T = t->sh.size;
    std::vector<unsigned char*> ptrs(T, nullptr);
    for (int p = 0; p < T; ++p) {
        if (p == t->sh.rank) {
            ptrs[p] = t->xch_own;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, handles + (size_t)p * 64, 64);
        void* m = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&m, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (unsigned char* q : t->peer_maps) cudaIpcCloseMemHandle(q);
            t->peer_maps.clear();
            return report_errorf(VOX_ERR_CUDA, "mapping rank %d's exchange area failed: %s", p, cudaGetErrorString(e));
        }
        ptrs[p] = static_cast<unsigned char*>(m);
        t->peer_maps.push_back(ptrs[p]);
    }
    TP_CUDA(dalloc(&t->xch_ptrs, (size_t)T));
    TP_CUDA(cudaMemcpy(t->xch_ptrs, ptrs.data(), T * sizeof(unsigned char*), cudaMemcpyHostToDevice));
    release_graphs(t);  // the next step is captured again with the peer-memory exchange
    t->p2p = true;
    return VOX_OK;
}

int vox_tp_init_random(vox_tp* t, uint64_t seed, float stdv) {
    if (!t) return report_errorf(VOX_ERR_INVALID_ARG, "tensor-parallel context is null");
    TP_CUDA(cudaSetDevice(t->dev));
    const vox_tp_shard& s = t->sh;
    const long long dim = (long long)t->cfg.dim, hd = (long long)t->cfg.head_dim;
    const long long q_full = (long long)t->cfg.n_heads * hd, kv_full = (long long)t->cfg.n_kv_heads * hd;
    const long long hid_full = (long long)t->cfg.hidden_dim;
    const long long q_l = (long long)s.n_heads * hd, kv_l = (long long)s.n_kv_heads * hd, hid_l = (long long)s.hidden;
    const long long q0 = (long long)s.q_head_begin * hd, kv0 = (long long)s.kv_head_begin * hd;
    const long long h0 = (long long)s.hidden_begin;
    cudaStream_t st = t->stream;
    for (size_t l = 0; l < t->layers.size(); ++l) {
        TpLayer& L = t->layers[l];
        TP_TRY(alloc_layer(t, L));
        const uint64_t b = 16 * (uint64_t)l;  // tensor ids of the single-device generator
        // q|k|v: rows of this rank's heads (column-parallel)
        TP_CUDA(launch_gen_matrix_part(L.wqkv, 2, seed, b + 1, stdv, q_l, dim, 1, 0, q0, 0, dim, st));
        TP_CUDA(launch_gen_matrix_part(L.wqkv, 2, seed, b + 2, stdv, kv_l, dim, 1, (int)q_l, kv0, 0, dim, st));
        TP_CUDA(launch_gen_matrix_part(L.wqkv, 2, seed, b + 3, stdv, kv_l, dim, 1, (int)(q_l + kv_l), kv0, 0, dim, st));
        // wo [dim, q_full]: columns of this rank's q heads (row-parallel)
        TP_CUDA(launch_gen_matrix_part(L.wo, 2, seed, b + 4, stdv, dim, q_l, 1, 0, 0, q0, q_full, st));
        // w1 / w3 rows interleaved; w2 [dim, hidden]: matching columns
        TP_CUDA(launch_gen_matrix_part(L.w13, 2, seed, b + 5, stdv, hid_l, dim, 2, 0, h0, 0, dim, st));
        TP_CUDA(launch_gen_matrix_part(L.w13, 2, seed, b + 7, stdv, hid_l, dim, 2, 1, h0, 0, dim, st));
        TP_CUDA(launch_gen_matrix_part(L.w2, 2, seed, b + 6, stdv, dim, hid_l, 1, 0, 0, h0, hid_full, st));
        TP_CUDA(launch_fill_f32(L.attn_norm, 1.0f, dim, st));
        TP_CUDA(launch_fill_f32(L.ffn_norm, 1.0f, dim, st));
        L.ready = true;
    }
    (void)kv_full;
    const long long V = (long long)s.vocab, Vl = (long long)s.vocab_local;
    if (!t->embed) TP_CUDA(dalloc(&t->embed, (size_t)(V * dim)));
    if (!t->head) TP_CUDA(dalloc(&t->head, (size_t)(Vl * dim)));
    if (!t->final_norm) TP_CUDA(dalloc(&t->final_norm, (size_t)dim));
    TP_CUDA(launch_gen_matrix(t->embed, 2, seed, 1000000, stdv, V, dim, 1, 0, st));
    TP_CUDA(launch_gen_matrix_part(t->head, 2, seed, 1000001, stdv, Vl, dim, 1, 0, (long long)s.vocab_begin, 0, dim, st));
    TP_CUDA(launch_fill_f32(t->final_norm, 1.0f, dim, st));
    t->embed_ready = t->head_ready = true;
    TP_CUDA(cudaStreamSynchronize(st));
    return VOX_OK;
}

int vox_tp_upload_layer_bf16(vox_tp* t, size_t layer, const vox_layer_weights_bf16* w) {
    if (!t) return report_errorf(VOX_ERR_INVALID_ARG, "tensor-parallel context is null");
    if (layer >= t->layers.size()) return report_errorf(VOX_ERR_INVALID_ARG, "layer %zu out of range", layer);
    TP_TRY(vox_layer_weights_validate_bf16(&t->cfg, w));
    TP_CUDA(cudaSetDevice(t->dev));
    TpLayer& L = t->layers[layer];
    TP_TRY(alloc_layer(t, L));
    const vox_tp_shard& s = t->sh;
    const size_t dim = t->cfg.dim, hd = t->cfg.head_dim;
    const size_t q_l = s.n_heads * hd, kv_l = s.n_kv_heads * hd;
    const size_t q0 = s.q_head_begin * hd, kv0 = s.kv_head_begin * hd;
    const size_t q_full = t->cfg.n_heads * hd, hid_full = t->cfg.hidden_dim;
    const size_t row = dim * 2;
    // row blocks of the column-parallel matrices
    TP_CUDA(cudaMemcpy(L.wqkv, w->wq.ptr + q0 * dim, q_l * row, cudaMemcpyHostToDevice));
    TP_CUDA(cudaMemcpy(L.wqkv + q_l * dim, w->wk.ptr + kv0 * dim, kv_l * row, cudaMemcpyHostToDevice));
    TP_CUDA(cudaMemcpy(L.wqkv + (q_l + kv_l) * dim, w->wv.ptr + kv0 * dim, kv_l * row, cudaMemcpyHostToDevice));
    TP_CUDA(cudaMemcpy2D(L.w13, 2 * row, w->w1.ptr + s.hidden_begin * dim, row, row, s.hidden, cudaMemcpyHostToDevice));
    TP_CUDA(cudaMemcpy2D(L.w13 + dim, 2 * row, w->w3.ptr + s.hidden_begin * dim, row, row, s.hidden,
                         cudaMemcpyHostToDevice));
    // column blocks of the row-parallel matrices
    TP_CUDA(cudaMemcpy2D(L.wo, q_l * 2, w->wo.ptr + q0, q_full * 2, q_l * 2, dim, cudaMemcpyHostToDevice));
    TP_CUDA(cudaMemcpy2D(L.w2, s.hidden * 2, w->w2.ptr + s.hidden_begin, hid_full * 2, s.hidden * 2, dim,
                         cudaMemcpyHostToDevice));
    TP_CUDA(cudaMemcpy(L.attn_norm, w->attention_norm.ptr, dim * 4, cudaMemcpyHostToDevice));
    TP_CUDA(cudaMemcpy(L.ffn_norm, w->ffn_norm.ptr, dim * 4, cudaMemcpyHostToDevice));
    L.ready = true;
    return VOX_OK;
}

int vox_tp_upload_embed_bf16(vox_tp* t, const uint16_t* embed, size_t len) {
    if (!t || !embed) return report_errorf(VOX_ERR_INVALID_ARG, "null argument");
    if (len != t->sh.vocab * t->cfg.dim) return report_errorf(VOX_ERR_SHAPE, "embed shape mismatch");
    TP_CUDA(cudaSetDevice(t->dev));
    if (!t->embed) TP_CUDA(dalloc(&t->embed, len));
    TP_CUDA(cudaMemcpy(t->embed, embed, len * 2, cudaMemcpyHostToDevice));
    t->embed_ready = true;
    return VOX_OK;
}

int vox_tp_upload_lm_head_bf16(vox_tp* t, const uint16_t* head, size_t len, const float* final_norm) {
    if (!t || !head) return report_errorf(VOX_ERR_INVALID_ARG, "null argument");
    if (len != t->sh.vocab * t->cfg.dim) return report_errorf(VOX_ERR_SHAPE, "lm_head shape mismatch");
    TP_CUDA(cudaSetDevice(t->dev));
    const size_t dim = t->cfg.dim;
    if (!t->head) TP_CUDA(dalloc(&t->head, t->sh.vocab_local * dim));
    TP_CUDA(cudaMemcpy(t->head, head + t->sh.vocab_begin * dim, t->sh.vocab_local * dim * 2, cudaMemcpyHostToDevice));
    if (!t->final_norm) TP_CUDA(dalloc(&t->final_norm, dim));
    if (final_norm) {
        TP_CUDA(cudaMemcpy(t->final_norm, final_norm, dim * 4, cudaMemcpyHostToDevice));
    } else {
        TP_CUDA(launch_fill_f32(t->final_norm, 1.0f, (long long)dim, t->stream));
        TP_CUDA(cudaStreamSynchronize(t->stream));
    }
    t->head_ready = true;
    return VOX_OK;
}

int vox_tp_step(vox_tp* t, int32_t token, size_t pos, int32_t* next_token, float* logits_local) {
    TP_TRY(ready(t));
    if (token < 0 || (size_t)token >= t->sh.vocab) return report_errorf(VOX_ERR_RANGE, "token %d outside the vocabulary", token);
    if (pos >= (size_t)t->max_pos) return report_errorf(VOX_ERR_RANGE, "position %zu beyond max_positions", pos);
    TP_TRY(tp_wait(t));
    StepState* hs = t->h_steps;
    memset(hs, 0, sizeof(StepState));
    hs->pos = (int64_t)pos;
    hs->tok = token;
    TP_CUDA(cudaMemcpyAsync(t->step, hs, sizeof(StepState), cudaMemcpyHostToDevice, t->stream));
    TP_TRY(launch_step(t, 1));
    TP_CUDA(cudaMemcpyAsync(t->h_tok, t->tok_out, 4, cudaMemcpyDeviceToHost, t->stream));
    if (logits_local)
        TP_CUDA(cudaMemcpyAsync(logits_local, t->logits, t->sh.vocab_local * 4, cudaMemcpyDeviceToHost, t->stream));
    TP_TRY(check_errors(t));
    mirror(t, 1);
    if (next_token) *next_token = *t->h_tok;
    return VOX_OK;
}

int vox_tp_prefill(vox_tp* t, const int32_t* tokens, size_t n, size_t pos0) {
    TP_TRY(ready(t));
    if (n == 0) return VOX_OK;
    if (!tokens) return report_errorf(VOX_ERR_INVALID_ARG, "tokens is null");
    if (pos0 + n > (size_t)t->max_pos) return report_errorf(VOX_ERR_RANGE, "positions beyond max_positions");
    for (size_t i = 0; i < n; ++i)
        if (tokens[i] < 0 || (size_t)tokens[i] >= t->sh.vocab)
            return report_errorf(VOX_ERR_RANGE, "token %d outside the vocabulary", tokens[i]);
    TP_TRY(tp_wait(t));
    TP_TRY(ensure_host_steps(t, n));
    for (size_t i = 0; i < n; ++i) {
        StepState* hs = t->h_steps + i;
        memset(hs, 0, sizeof(StepState));
        hs->pos = (int64_t)(pos0 + i);
        hs->tok = tokens[i];
        TP_CUDA(cudaMemcpyAsync(t->step, hs, sizeof(StepState), cudaMemcpyHostToDevice, t->stream));
        TP_TRY(launch_step(t, i + 1));
    }
    TP_TRY(check_errors(t));
    mirror(t, n);
    return VOX_OK;
}

int vox_tp_generate(vox_tp* t, int32_t token, size_t pos, size_t n_steps, int32_t* tokens_out) {
    TP_TRY(ready(t));
    if (n_steps == 0) return VOX_OK;
    if (token < 0 || (size_t)token >= t->sh.vocab) return report_errorf(VOX_ERR_RANGE, "token %d outside the vocabulary", token);
    if (pos + n_steps > (size_t)t->max_pos) return report_errorf(VOX_ERR_RANGE, "positions beyond max_positions");
    TP_TRY(tp_wait(t));
    TP_TRY(ensure_host_steps(t, n_steps + 1));
    StepState* hs = t->h_steps;
    memset(hs, 0, sizeof(StepState));
    hs->pos = (int64_t)pos;
    hs->tok = token;
    hs->greedy = 1;
    hs->advance = 1;
    TP_CUDA(cudaMemcpyAsync(t->step, hs, sizeof(StepState), cudaMemcpyHostToDevice, t->stream));
    int32_t* hist = reinterpret_cast<int32_t*>(t->h_steps + 1);
    for (size_t i = 0; i < n_steps; ++i) {
        TP_TRY(launch_step(t, i + 1));
        if (tokens_out) TP_CUDA(cudaMemcpyAsync(hist + i, t->tok_out, 4, cudaMemcpyDeviceToHost, t->stream));
    }
    TP_TRY(check_errors(t));
    mirror(t, n_steps);
    if (tokens_out) memcpy(tokens_out, hist, n_steps * 4);
    return VOX_OK;
}

int vox_tp_kv_state(const vox_tp* t, size_t layer, int64_t out[3]) {
    if (!t || !out || layer >= t->layers.size()) return report_errorf(VOX_ERR_INVALID_ARG, "bad argument");
    TP_CUDA(cudaSetDevice(t->dev));
    KvState d{};
    TP_CUDA(cudaMemcpyAsync(&d, t->dstate + layer, sizeof d, cudaMemcpyDeviceToHost, t->stream));
    TP_CUDA(cudaStreamSynchronize(t->stream));
    out[0] = d.len;
    out[1] = d.start;
    out[2] = d.pos_offset;
    return VOX_OK;
}

int vox_tp_set_timeout_ms(vox_tp* t, unsigned timeout_ms) {
    if (!t || timeout_ms == 0) return report_errorf(VOX_ERR_INVALID_ARG, "null context or zero timeout");
    t->timeout_ms = timeout_ms;
    return VOX_OK;
}

int vox_tp_reset(vox_tp* t) {
    if (!t) return report_errorf(VOX_ERR_INVALID_ARG, "tensor-parallel context is null");
    TP_CUDA(cudaSetDevice(t->dev));
    TP_CUDA(cudaStreamSynchronize(t->stream));
    TP_CUDA(cudaMemsetAsync(t->dstate, 0, t->layers.size() * sizeof(KvState), t->stream));
    TP_CUDA(cudaStreamSynchronize(t->stream));
    for (HostKv& h : t->hs) h = HostKv{};
    return VOX_OK;
}

int vox_tp_record_event(vox_tp* t, int slot) {
    if (!t || slot < 0 || slot >= 8) return report_errorf(VOX_ERR_INVALID_ARG, "bad event slot");
    TP_CUDA(cudaEventRecord(t->ev[slot], t->stream));
    return VOX_OK;
}

int vox_tp_event_elapsed_ms(vox_tp* t, int a, int b, float* ms) {
    if (!t || !ms || a < 0 || a >= 8 || b < 0 || b >= 8) return report_errorf(VOX_ERR_INVALID_ARG, "bad event slot");
    TP_CUDA(cudaEventSynchronize(t->ev[b]));
    TP_CUDA(cudaEventElapsedTime(ms, t->ev[a], t->ev[b]));
    return VOX_OK;
}

uint64_t vox_tp_kernel_launches(const vox_tp* t) { return t ? t->launches : 0; }

}  // extern "C"
