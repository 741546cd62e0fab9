// vox_stream.cpp -- the streaming decode driver: the caller of the token loop.
//
// Restates the reference's streaming schedule (crates/voxtral/src/stream.rs,
// the integer helpers; crates/voxtral/src/pipeline.rs, PipelineState) and
// wires it to the device token loop the way the design document describes
// (docs/plans/2026-02-11-voxtral-rust-design.md:40-46): with a prompt of L ids
// ([BOS] + [STREAMING_PAD] * (left_pad + delay)), decoding starts once L
// adapter positions exist; positions 0..L-2 are prefilled, position L-1
// yields the first token, and every later position p feeds
// adapter[p] + tok_embed(previous token).  Prompt positions feed
// adapter[p] + tok_embed(prompt[p]) the same way.
//
// Adapter rows live in a device ring of `adapter_capacity` positions; a push
// copies rows there on the context's stream, so a decode enqueued earlier
// reads its rows before a later push can overwrite them.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "../../include/vox_decoder.h"
#include "vox_host.h"
#include "vox_internal.h"

using namespace vox;

// ---- stream.rs -----------------------------------------------------------------

extern "C" void vox_stream_prompt_config_default(vox_stream_prompt_config* out) {
    if (!out) return;
    out->left_pad_tokens = 32;   // stream.rs:11-19
    out->delay_tokens = 6;       // 480 ms at 12.5 Hz
    out->eos_extra_tokens = 10;
}

extern "C" size_t vox_stream_right_pad_tokens(const vox_stream_prompt_config* c) {
    return c ? c->delay_tokens + 1 + c->eos_extra_tokens : 0;  // stream.rs:21-25
}

extern "C" size_t vox_stream_build_prompt_ids(uint32_t bos_id, uint32_t streaming_pad_id,
                                              const vox_stream_prompt_config* c, uint32_t* out, size_t cap) {
    if (!c) return 0;
    const size_t n = 1 + c->left_pad_tokens + c->delay_tokens;  // stream.rs:26-34
    for (size_t i = 0; out && i < n && i < cap; ++i) out[i] = i == 0 ? bos_id : streaming_pad_id;
    return n;
}

extern "C" int vox_stream_decode_ready(size_t total_adapter_tokens, size_t prompt_len) {
    return total_adapter_tokens >= prompt_len;  // stream.rs:36-38
}

extern "C" size_t vox_stream_decodable_token_budget(size_t total_adapter_tokens, size_t prompt_len) {
    // stream.rs:47-53: first token at position L-1, then one per position L..N-1.
    return total_adapter_tokens < prompt_len ? 0 : total_adapter_tokens - prompt_len + 1;
}

extern "C" size_t vox_stream_finish_zero_padding_samples(size_t consumed_samples, size_t samples_per_token,
                                                         const vox_stream_prompt_config* c) {
    if (!c || samples_per_token == 0) return 0;  // the reference debug_asserts samples_per_token > 0
    const size_t rem = consumed_samples % samples_per_token;  // stream.rs:60-69
    const size_t align = rem == 0 ? 0 : samples_per_token - rem;
    return align + vox_stream_right_pad_tokens(c) * samples_per_token;
}

// ---- pipeline.rs -----------------------------------------------------------------

struct vox_pipeline {
    vox_pipeline_config cfg{};
    std::vector<uint32_t> prompt;       // PipelineState::prompt_ids
    size_t adapter_tokens_total = 0;
    size_t generated_tokens = 0;
    bool finished = false;
    // device side (null ctx: planner only, as the reference's PipelineState)
    vox_ctx* ctx = nullptr;
    vox_kv* kv = nullptr;
    size_t dim = 0, cap = 0;
    float* adapter = nullptr;           // [cap, dim] ring, row = position mod cap
    StepGraphs graphs;
    int32_t last_token = 0;
};

namespace {

size_t decodable_now(const vox_pipeline* p) {
    // pipeline.rs:68-71 (saturating_sub)
    const size_t total = vox_stream_decodable_token_budget(p->adapter_tokens_total, p->prompt.size());
    return total > p->generated_tokens ? total - p->generated_tokens : 0;
}

// First adapter position not yet handed to a decode launch.
size_t next_unenqueued_position(const vox_pipeline* p) {
    return p->generated_tokens == 0 ? 0 : p->prompt.size() - 1 + p->generated_tokens;
}

}  // namespace

extern "C" int vox_pipeline_create(vox_ctx* ctx, vox_kv* kv, const vox_pipeline_config* cfg,
                                   size_t adapter_capacity, vox_pipeline** out) {
    if (!cfg || !out) return report_errorf(VOX_ERR_INVALID_ARG, "null config or output");
    *out = nullptr;
    auto* p = new vox_pipeline();
    p->cfg = *cfg;
    const size_t n = vox_stream_build_prompt_ids(cfg->bos_id, cfg->streaming_pad_id, &cfg->prompt, nullptr, 0);
    p->prompt.resize(n);
    vox_stream_build_prompt_ids(cfg->bos_id, cfg->streaming_pad_id, &cfg->prompt, p->prompt.data(), n);
    if (ctx || kv) {
        CtxInfo info{};
        int rc = ctx_info(ctx, &info);
        if (rc == VOX_OK) rc = ctx_model_ready(ctx, kv);
        if (rc != VOX_OK) {
            delete p;
            return rc;
        }
        if ((size_t)cfg->bos_id >= info.vocab || (size_t)cfg->streaming_pad_id >= info.vocab) {
            delete p;
            return report_errorf(VOX_ERR_RANGE, "prompt ids outside the vocabulary of %zu", info.vocab);
        }
        if (adapter_capacity < n || adapter_capacity > (size_t)1 << 24) {
            delete p;
            return report_errorf(VOX_ERR_INVALID_ARG, "adapter_capacity must be in [prompt length %zu, 2^24]", n);
        }
        p->ctx = ctx;
        p->kv = kv;
        p->dim = info.dim;
        p->cap = adapter_capacity;
        if (cudaSetDevice(info.device) != cudaSuccess ||
            cudaMalloc(&p->adapter, adapter_capacity * info.dim * sizeof(float)) != cudaSuccess) {
            delete p;
            return report_errorf(VOX_ERR_OOM, "cannot allocate the %zu-position adapter ring", adapter_capacity);
        }
        rc = capture_adapter_graphs(ctx, kv, p->adapter, (int)adapter_capacity, &p->graphs);
        if (rc != VOX_OK) {
            cudaFree(p->adapter);
            delete p;
            return rc;
        }
    }
    *out = p;
    return VOX_OK;
}

extern "C" void vox_pipeline_destroy(vox_pipeline* p) {
    if (!p) return;
    if (p->ctx) {
        CtxInfo info{};
        if (ctx_info(p->ctx, &info) == VOX_OK) {
            cudaSetDevice(info.device);
            cudaStreamSynchronize(info.stream);
        }
    }
    release_step_graphs(&p->graphs);
    if (p->adapter) cudaFree(p->adapter);
    delete p;
}

extern "C" size_t vox_pipeline_prompt_ids(const vox_pipeline* p, uint32_t* out, size_t cap) {
    if (!p) return 0;
    for (size_t i = 0; out && i < p->prompt.size() && i < cap; ++i) out[i] = p->prompt[i];
    return p->prompt.size();
}

extern "C" size_t vox_pipeline_adapter_tokens_total(const vox_pipeline* p) { return p ? p->adapter_tokens_total : 0; }
extern "C" size_t vox_pipeline_generated_tokens(const vox_pipeline* p) { return p ? p->generated_tokens : 0; }
extern "C" size_t vox_pipeline_decodable_now(const vox_pipeline* p) { return p ? decodable_now(p) : 0; }
extern "C" int vox_pipeline_is_finished(const vox_pipeline* p) { return p && p->finished; }

extern "C" int vox_pipeline_push_adapter_tokens(vox_pipeline* p, const float* rows, size_t n_tokens) {
    if (!p) return report_errorf(VOX_ERR_INVALID_ARG, "null pipeline");
    if (n_tokens == 0) return VOX_OK;  // pipeline.rs:62-64
    if (p->ctx) {
        if (!rows) return report_errorf(VOX_ERR_INVALID_ARG, "adapter rows are null");
        const size_t pending = p->adapter_tokens_total + n_tokens - next_unenqueued_position(p);
        if (pending > p->cap)
            return report_errorf(VOX_ERR_RANGE,
                                 "adapter ring of %zu positions full (%zu not yet decoded): decode before pushing more",
                                 p->cap, pending - n_tokens);
        CtxInfo info{};
        int rc = ctx_info(p->ctx, &info);
        if (rc != VOX_OK) return rc;
        if (cudaSetDevice(info.device) != cudaSuccess) return report_errorf(VOX_ERR_CUDA, "cudaSetDevice failed");
        size_t done = 0;
        while (done < n_tokens) {  // at most two pieces: the ring wraps once
            const size_t slot = (p->adapter_tokens_total + done) % p->cap;
            const size_t n = std::min(n_tokens - done, p->cap - slot);
            cudaError_t e = cudaMemcpyAsync(p->adapter + slot * p->dim, rows + done * p->dim,
                                            n * p->dim * sizeof(float), cudaMemcpyHostToDevice, info.stream);
            if (e != cudaSuccess) return report_errorf(VOX_ERR_CUDA, "adapter upload failed: %s", cudaGetErrorString(e));
            done += n;
        }
    }
    p->adapter_tokens_total += n_tokens;
    return VOX_OK;
}

extern "C" int vox_pipeline_mark_decoded(vox_pipeline* p, size_t n_tokens) {
    if (!p) return report_errorf(VOX_ERR_INVALID_ARG, "null pipeline");
    if (p->ctx) return report_errorf(VOX_ERR_INVALID_ARG, "a pipeline with a context marks its own tokens (vox_pipeline_decode)");
    if (n_tokens > decodable_now(p))  // pipeline.rs:74 debug_assert
        return report_errorf(VOX_ERR_INVALID_ARG, "mark_decoded(%zu) beyond decodable_now %zu", n_tokens, decodable_now(p));
    p->generated_tokens += n_tokens;
    return VOX_OK;
}

extern "C" int vox_pipeline_decode(vox_pipeline* p, size_t max_tokens, int32_t* tokens_out, size_t* n_out) {
    if (!p || !n_out) return report_errorf(VOX_ERR_INVALID_ARG, "null pipeline or output count");
    *n_out = 0;
    if (!p->ctx) return report_errorf(VOX_ERR_NOT_READY, "pipeline has no context (planner only)");
    const size_t n = std::min(max_tokens, decodable_now(p));
    if (n == 0) return VOX_OK;
    if (!tokens_out) return report_errorf(VOX_ERR_INVALID_ARG, "tokens_out is null");
    const size_t L = p->prompt.size();
    std::vector<int32_t> fixed;
    size_t pos0;
    int32_t first;
    if (p->generated_tokens == 0) {  // prefill 0..L-2, first token from position L-1
        fixed.assign(p->prompt.begin(), p->prompt.end() - 1);
        first = (int32_t)p->prompt[L - 1];
        pos0 = 0;
    } else {
        first = p->last_token;
        pos0 = L - 1 + p->generated_tokens;
    }
    int rc = run_step_graphs(p->ctx, p->kv, p->graphs, fixed.data(), fixed.size(), pos0, first, n, tokens_out);
    if (rc != VOX_OK) return rc;
    p->generated_tokens += n;  // pipeline.rs:73-76
    p->last_token = tokens_out[n - 1];
    *n_out = n;
    return VOX_OK;
}

extern "C" size_t vox_pipeline_finish_padding_samples(vox_pipeline* p, size_t consumed_audio_samples) {
    if (!p) return 0;
    p->finished = true;  // pipeline.rs:78-85
    return vox_stream_finish_zero_padding_samples(consumed_audio_samples, p->cfg.samples_per_token, &p->cfg.prompt);
}
