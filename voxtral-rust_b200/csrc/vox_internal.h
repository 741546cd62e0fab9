// vox_internal.h -- what the host files beside vox_capi.cpp (the streaming
// pipeline, the weight loader) need from a context: its shape, a model
// readiness check, and step graphs whose first input is the embedding row
// plus an adapter row.  vox_ctx and vox_kv stay opaque here.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/vox_decoder.h"

namespace vox {

struct CtxInfo {
    int device;
    cudaStream_t stream;
    vox_decoder_config cfg;
    size_t dim, vocab, n_layers;
    int max_pos;
    int weight_dtype;  // vox_weight_dtype
};

int ctx_info(const vox_ctx* c, CtxInfo* out);

// The checks of vox_model_step: weights present, cache shaped like the
// model, a single-stream cache.
int ctx_model_ready(vox_ctx* c, vox_kv* kv);

// One token step captured as CUDA graphs (a cluster-attention variant for
// short contexts when the shape has one), with the first layer's input
// x = adapter[pos mod adapter_cap] + widen(embed[token]).
struct StepGraphs {
    cudaGraphExec_t full = nullptr, short_attn = nullptr;
    uint64_t k_full = 0, k_short = 0;
    const float* adapter = nullptr;  // the ring the graphs read
    int adapter_cap = 0;
};
int capture_adapter_graphs(vox_ctx* c, vox_kv* kv, const float* adapter, int adapter_cap, StepGraphs* g);
void release_step_graphs(StepGraphs* g);

// n_fixed steps with the given tokens at positions pos0.. (outputs dropped;
// a batched tensor-core prefill when the shape allows and n_fixed >= 2), then n_greedy greedy steps starting from greedy_tok at pos0 + n_fixed, each
// step's argmax feeding the next; tokens_out[n_greedy] (nullable).  One
// synchronisation at the end; the cache's host mirror follows the appends.
int run_step_graphs(vox_ctx* c, vox_kv* kv, const StepGraphs& g, const int32_t* fixed, size_t n_fixed,
                    size_t pos0, int32_t greedy_tok, size_t n_greedy, int32_t* tokens_out);

}  // namespace vox
