/*
 * vox_decoder.h -- C ABI of the B200 (sm_100a) decoder-token-loop library.
 *
 * This is the drop-in boundary for the decoder path of voxtral-rust
 * (crates/voxtral/src/{decoder,kv,ops,math}.rs).  Every entry point names the
 * reference item it replaces.  Conventions:
 *   - every function returns an int status (VOX_OK == 0); on failure
 *     vox_last_error() returns a thread-local message for the last failure
 *     on the calling thread (the reference returns anyhow::Error);
 *   - host buffers are borrowed for the duration of the call only; the
 *     library copies what it keeps (weights are copied to device memory);
 *   - a vox_ctx owns one CUDA device and one CUDA stream.  A context and the
 *     caches made from it are single-thread-affine, the same discipline as
 *     the reference's `&mut RollingKvCache`.
 *
 * Numerics: activations, KV cache and accumulation are f32.  Weight
 * matrices are held as bf16 by default (VOX_WEIGHTS_BF16); bf16 weights
 * widened to f32 are exactly the f32 weights the reference would use
 * (weights.rs:77-81).  VOX_WEIGHTS_F32 keeps f32 weights for callers whose
 * weights are not bf16-representable.
 */
#ifndef VOX_DECODER_H
#define VOX_DECODER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VOX_ABI_VERSION 1

typedef enum vox_status {
    VOX_OK = 0,
    VOX_ERR_INVALID_ARG = 1,    /* null pointer, index out of range */
    VOX_ERR_CONFIG = 2,         /* DecoderConfig::validate failed (decoder.rs:22-41) */
    VOX_ERR_SHAPE = 3,          /* length mismatch (decoder.rs:58-84, :98) */
    VOX_ERR_UNSUPPORTED = 4,    /* shape the kernels do not handle (message says which) */
    VOX_ERR_CUDA = 5,           /* CUDA runtime error (message has the CUDA string) */
    VOX_ERR_OOM = 6,            /* device or pinned allocation failed */
    VOX_ERR_NOT_READY = 7,      /* weights needed by the call were never uploaded */
    VOX_ERR_DEVICE_TIMEOUT = 8, /* a bounded wait inside a kernel expired */
    VOX_ERR_RANGE = 9,          /* position beyond the RoPE table, token outside the vocab */
    VOX_ERR_IO = 10,            /* a file could not be opened or mapped */
    VOX_ERR_FORMAT = 11         /* malformed file (safetensors header, tekken.json) or unsupported dtype */
} vox_status;

typedef enum vox_weight_dtype { VOX_WEIGHTS_BF16 = 0, VOX_WEIGHTS_F32 = 1 } vox_weight_dtype;

/* DecoderConfig (decoder.rs:10-19), field for field. */
typedef struct vox_decoder_config {
    size_t dim;
    size_t hidden_dim;
    size_t n_heads;
    size_t n_kv_heads;
    size_t head_dim;
    size_t sliding_window;
    float norm_eps;
    float rope_theta;
} vox_decoder_config;

/* Options of a context.  Zero-initialise and set what you need; zero means
 * "default" for every field. */
typedef struct vox_ctx_options {
    int device;               /* CUDA device ordinal */
    size_t n_layers;          /* layers whose weights the context holds (default 1) */
    size_t vocab;             /* vocabulary for the token loop; 0 = no embedding / LM head */
    size_t max_positions;     /* RoPE table length; positions must stay below it (default 32768) */
    int weight_dtype;         /* vox_weight_dtype */
    int step_mode;            /* vox_step_mode: how vox_model_* run a token step */
} vox_ctx_options;

/* How the multi-stream step (vox_model_step_batch / _generate_batch) runs its
 * GEMMs; single-stream steps always run five kernels per layer (QKV + RoPE +
 * ring append, attention, o-proj, w1|w3 + SwiGLU, w2) plus LM head and argmax,
 * captured in a CUDA graph.  VOX_STEP_PERSISTENT runs o-proj, w1|w3, w2 and the
 * next q|k|v as one persistent launch per layer; VOX_STEP_AUTO and
 * VOX_STEP_LAYERS launch every GEMM on its own (the faster choice on B200). */
typedef enum vox_step_mode { VOX_STEP_AUTO = 0, VOX_STEP_LAYERS = 1, VOX_STEP_PERSISTENT = 2 } vox_step_mode;

typedef struct vox_f32_slice { const float* ptr; size_t len; } vox_f32_slice;
typedef struct vox_bf16_slice { const uint16_t* ptr; size_t len; } vox_bf16_slice;

/* DecoderLayerWeights (decoder.rs:45-55), f32 flavour: the reference's own
 * struct.  Matrices are row-major [out, in] as in the reference. */
typedef struct vox_layer_weights_f32 {
    vox_f32_slice attention_norm, wq, wk, wv, wo, ffn_norm, w1, w2, w3;
} vox_layer_weights_f32;

/* Same tensors with matrices given as bf16 bit patterns. */
typedef struct vox_layer_weights_bf16 {
    vox_f32_slice attention_norm;
    vox_bf16_slice wq, wk, wv, wo;
    vox_f32_slice ffn_norm;
    vox_bf16_slice w1, w2, w3;
} vox_layer_weights_bf16;

/* AttentionShape (ops.rs:49-56). sliding_window 0 = no window. */
typedef struct vox_attention_shape {
    size_t n_heads;
    size_t head_dim;
    size_t seq_len;
    size_t n_kv_heads;
    size_t sliding_window;
} vox_attention_shape;

typedef struct vox_ctx vox_ctx;
typedef struct vox_kv vox_kv;

/* ---- errors and config --------------------------------------------------- */
const char* vox_last_error(void);
int vox_abi_version(void);
/* DecoderConfig::validate (decoder.rs:22-41); same checks, same order. */
int vox_config_validate(const vox_decoder_config* cfg);
/* DecoderLayerWeights::validate (decoder.rs:58-84). */
int vox_layer_weights_validate_f32(const vox_decoder_config* cfg, const vox_layer_weights_f32* w);
int vox_layer_weights_validate_bf16(const vox_decoder_config* cfg, const vox_layer_weights_bf16* w);

/* ---- context and weights ------------------------------------------------- */
int vox_ctx_create(const vox_decoder_config* cfg, const vox_ctx_options* opt, vox_ctx** out);
/* Also destroys every cache still attached to the context; their handles
 * become invalid.  Destroy caches first if you keep handles to them. */
void vox_ctx_destroy(vox_ctx* ctx);
/* Copy one layer's weights to the device (caller keeps ownership).  With
 * VOX_WEIGHTS_BF16 the f32 upload rounds matrices to bf16, nearest-even. */
int vox_ctx_upload_layer_f32(vox_ctx* ctx, size_t layer, const vox_layer_weights_f32* w);
int vox_ctx_upload_layer_bf16(vox_ctx* ctx, size_t layer, const vox_layer_weights_bf16* w);
/* Token loop tensors (no reference counterpart: the reference stops at one
 * layer step).  embed and lm_head are [vocab, dim] bf16; final_norm [dim]. */
int vox_ctx_upload_embed_bf16(vox_ctx* ctx, const uint16_t* embed, size_t len);
int vox_ctx_upload_lm_head_bf16(vox_ctx* ctx, const uint16_t* lm_head, size_t len);
int vox_ctx_upload_final_norm(vox_ctx* ctx, const float* gain, size_t len);
/* Fill every weight on the device from the library's counter-based
 * generator (bit-identical to the oracle's): matrices ~N(0, std^2) rounded
 * to the weight dtype, norm gains 1.0. */
int vox_ctx_init_random(vox_ctx* ctx, uint64_t seed, float std);
/* Copy a stored matrix back in reference layout (for checks).
 * which: 0 wq 1 wk 2 wv 3 wo 4 w1 5 w2 6 w3 7 embed 8 lm_head.  Output is
 * bf16 bits (uint16) or f32 according to the context's weight dtype. */
int vox_ctx_download_matrix(vox_ctx* ctx, size_t layer, int which, void* out, size_t out_bytes);
/* The context's CUDA stream (cudaStream_t) and a synchronise helper. */
void* vox_ctx_stream(vox_ctx* ctx);
int vox_ctx_synchronize(vox_ctx* ctx);
/* CUDA-event timing on the context's stream (slots 0..15). */
int vox_ctx_record_event(vox_ctx* ctx, int slot);
int vox_ctx_event_elapsed_ms(vox_ctx* ctx, int slot_a, int slot_b, float* ms);
/* Kernel launches issued by the library since the context was created. */
uint64_t vox_ctx_kernel_launches(vox_ctx* ctx);

/* ---- rolling KV cache (kv.rs) --------------------------------------------- */
/* RollingKvCache::new (kv.rs:33-46).  Device ring of `sliding_window` tokens
 * per layer; eviction is index arithmetic, not a copy. */
int vox_kv_create(vox_ctx* ctx, size_t n_layers, size_t n_kv_heads, size_t head_dim,
                  size_t sliding_window, vox_kv** out);
/* Same with a ring larger than the window, for callers that append more
 * than `sliding_window` tokens in one call (kv.rs:64-74 keeps them all). */
int vox_kv_create_ex(vox_ctx* ctx, size_t n_layers, size_t n_kv_heads, size_t head_dim,
                     size_t sliding_window, size_t capacity_tokens, vox_kv** out);
void vox_kv_destroy(vox_kv* kv);
/* RollingKvCache::append_layer (kv.rs:48-88); k_new/v_new are host
 * [n_new, n_kv_heads, head_dim] f32. */
int vox_kv_append_layer(vox_kv* kv, size_t layer, const float* k_new, const float* v_new,
                        size_t n_new_tokens);
/* layer_len_tokens (kv.rs:90), layer_pos_offset (kv.rs:94). */
int vox_kv_layer_len_tokens(const vox_kv* kv, size_t layer, size_t* out);
int vox_kv_layer_pos_offset(const vox_kv* kv, size_t layer, size_t* out);
/* layer_tensors (kv.rs:98-101): copies the layer's K and V to host in the
 * reference's logical order [len_tokens, n_kv_heads, head_dim].  Each
 * buffer must hold at least len_tokens*n_kv_heads*head_dim floats
 * (capacity given in elements). */
int vox_kv_layer_tensors(const vox_kv* kv, size_t layer, float* keys, float* values,
                         size_t capacity_elems);
/* Device-side ring bookkeeping of a layer, for index checks:
 * out[0] = len_tokens, out[1] = physical start slot, out[2] = pos_offset. */
int vox_kv_layer_device_state(const vox_kv* kv, size_t layer, int64_t out[3]);
/* Forget every token (all layers back to len 0, pos_offset 0). */
int vox_kv_reset(vox_kv* kv);

/* ---- multi-stream caches -------------------------------------------------- */
/* n_streams (1..8) independent RollingKvCaches (kv.rs:33-46) in one
 * allocation, for the multi-stream step (vox_model_step_batch).  Each stream
 * has its own ring, length and pos_offset. */
int vox_kv_create_streams(vox_ctx* ctx, size_t n_streams, size_t n_layers, size_t n_kv_heads,
                          size_t head_dim, size_t sliding_window, vox_kv** out);
/* Number of streams of a cache (1 for a single-stream cache or a view). */
int vox_kv_n_streams(const vox_kv* kv, size_t* out);
/* A handle to stream `stream` of a multi-stream cache that every
 * single-stream entry point accepts (append, observers, layer step,
 * vox_model_step).  It shares the cache's memory, lives until the cache is
 * destroyed (vox_kv_destroy on a view does nothing) and is the cache itself
 * when it holds one stream.  Single-stream entry points reject a
 * multi-stream cache with VOX_ERR_INVALID_ARG. */
int vox_kv_stream(vox_kv* kv, size_t stream, vox_kv** out);
/* Replace the contents of every layer of a single-stream cache (or view)
 * with n_tokens tokens from the library's counter-based generator:
 * layer l's keys are tensor tensor_id + 2l and its values tensor
 * tensor_id + 2l + 1, each [n_tokens, n_kv_heads, head_dim] token-major,
 * ~N(0, std^2) rounded to bf16.  len_tokens = n_tokens, pos_offset = 0;
 * n_tokens <= sliding_window. */
int vox_kv_fill_random(vox_kv* kv, size_t n_tokens, uint64_t seed, uint64_t tensor_id, float std);
/* ---- decoder step (decoder.rs:88-155) -------------------------------------- */
/* decoder_layer_forward_step: hidden [dim] f32 in, out [dim] f32 (the
 * reference returns a new Vec; here the caller owns `out`).  Appends one
 * token to `layer_idx` of the cache. */
int vox_decoder_layer_forward_step(vox_ctx* ctx, size_t layer_idx, vox_kv* kv,
                                   const float* hidden, size_t hidden_len, size_t pos,
                                   float* out, size_t out_len);

/* ---- composed token loop (no reference counterpart, see header text) ----- */
/* One token through embed -> all layers -> final RMSNorm -> LM head ->
 * argmax (lowest index wins ties).  Runs as one CUDA graph.  logits_out
 * (nullable) receives [vocab] f32. */
int vox_model_step(vox_ctx* ctx, vox_kv* kv, int32_t token, size_t pos, int32_t* next_token,
                   float* logits_out);
/* Greedy decode of n_steps tokens starting from `token` at `pos`, entirely
 * on the device (each step's argmax feeds the next).  tokens_out [n_steps]. */
int vox_model_generate(vox_ctx* ctx, vox_kv* kv, int32_t token, size_t pos, size_t n_steps,
                       int32_t* tokens_out);
/* Prefill of n tokens at positions pos0.. (logits discarded): the cache ends
 * as n single-token steps (decoder.rs:88-155, kv.rs:48-88) leave it, within
 * float tolerance.  With bf16 weights (every K a multiple of 64, at most 4 q
 * heads per kv head, head_dim 32/64/128/256) and n >= 2, passes of up to 512
 * tokens run each layer at once: dense tensor-core GEMMs over all the pass's
 * tokens, causal attention over the cache plus the pass, keys and values
 * appended at the slots the token loop would use.  Otherwise, as
 * vox_model_prefill_steps. */
int vox_model_prefill(vox_ctx* ctx, vox_kv* kv, const int32_t* tokens, size_t n, size_t pos0);
/* The same prefill as n sequential token steps (one CUDA graph launch each). */
int vox_model_prefill_steps(vox_ctx* ctx, vox_kv* kv, const int32_t* tokens, size_t n, size_t pos0);

/* One token for every stream of a multi-stream cache (bf16 weights): the
 * step of vox_model_step, with every linear on the tensor cores reading each
 * weight once for all streams.  tokens[s], positions[s] per stream;
 * next_tokens [n_streams] and logits_out [n_streams, vocab] are nullable.
 * Runs as one CUDA graph. */
int vox_model_step_batch(vox_ctx* ctx, vox_kv* kv, const int32_t* tokens, const size_t* positions,
                         int32_t* next_tokens, float* logits_out);
/* Greedy decode of n_steps tokens for every stream on the device.
 * tokens_out [n_steps, n_streams] (nullable). */
int vox_model_generate_batch(vox_ctx* ctx, vox_kv* kv, const int32_t* tokens, const size_t* positions,
                             size_t n_steps, int32_t* tokens_out);
/* ---- tensor-parallel single stream (no reference counterpart) -------------------- */
/* One process per GPU; tp_size ranks share each layer: rank r holds the q|k|v
 * rows of q heads [r*n_heads/T, (r+1)*n_heads/T) and of the kv heads they
 * attend to, the matching columns of wo, w1|w3 rows [r*hidden/T, ...) and the
 * matching columns of w2, and LM-head rows [r*vocab/T, ...).  The residual
 * stream is all-reduced (NCCL, sum) after o-proj and after w2; the greedy
 * token is an all-reduce (max) of (value, index) keys.  n_heads, n_kv_heads,
 * hidden_dim and vocab must divide by tp_size; bf16 weights. */
typedef struct vox_tp vox_tp;
typedef struct vox_tp_shard {
    int rank, size;
    size_t n_heads, n_kv_heads, hidden;   /* local counts */
    size_t vocab, vocab_local;
    size_t q_head_begin, kv_head_begin, hidden_begin, vocab_begin;
} vox_tp_shard;
/* The shard a rank holds (host only; validates like vox_config_validate). */
int vox_tp_shard_of(const vox_decoder_config* cfg, size_t vocab, int tp_rank, int tp_size, vox_tp_shard* out);
/* NCCL unique id: made by one rank, passed to every rank's vox_tp_create. */
int vox_tp_unique_id(unsigned char id[128]);
/* Collective over all ranks (each blocks until all have joined).  opt: device,
 * n_layers, vocab (required), max_positions; weight_dtype must be bf16.  The
 * context owns a rolling cache of window cfg->sliding_window for its kv heads. */
int vox_tp_create(const vox_decoder_config* cfg, const vox_ctx_options* opt, int tp_rank, int tp_size,
                  const unsigned char id[128], vox_tp** out);
/* Peer-memory exchange (replaces the NCCL all-reduces with stores into the
 * other GPUs' memory, fused into the GEMVs): every rank exports the CUDA IPC
 * handle of its exchange area, the host gathers all of them in rank order
 * ([tp_size][64] bytes) and every rank connects.  Collective; call between
 * steps on all ranks, or never (NCCL stays in use). */
int vox_tp_ipc_handle(vox_tp* tp, unsigned char out[64]);
int vox_tp_connect_peers(vox_tp* tp, const unsigned char* handles);
/* Releases the captured graph, then the NCCL communicator, then memory. */
void vox_tp_destroy(vox_tp* tp);
/* This rank's shards of the weights vox_ctx_init_random makes (same generator,
 * same tensor ids, so the ranks together hold exactly those weights). */
int vox_tp_init_random(vox_tp* tp, uint64_t seed, float std);
/* Full (unsharded) tensors in; each rank copies its shard. */
int vox_tp_upload_layer_bf16(vox_tp* tp, size_t layer, const vox_layer_weights_bf16* w);
int vox_tp_upload_embed_bf16(vox_tp* tp, const uint16_t* embed, size_t len);
int vox_tp_upload_lm_head_bf16(vox_tp* tp, const uint16_t* lm_head, size_t len, const float* final_norm);
/* Collective token steps (every rank calls them with the same arguments).
 * logits_local (nullable) receives this rank's [vocab/T] slice of the logits. */
int vox_tp_step(vox_tp* tp, int32_t token, size_t pos, int32_t* next_token, float* logits_local);
int vox_tp_prefill(vox_tp* tp, const int32_t* tokens, size_t n, size_t pos0);
int vox_tp_generate(vox_tp* tp, int32_t token, size_t pos, size_t n_steps, int32_t* tokens_out);
/* Device ring state of a layer: len_tokens, start slot, pos_offset. */
int vox_tp_kv_state(const vox_tp* tp, size_t layer, int64_t out[3]);
/* Forget every cached token (all layers back to len 0, pos_offset 0); local,
 * call it on every rank between the same two steps. */
int vox_tp_reset(vox_tp* tp);
/* Watchdog bound (default 30000 ms) on every wait of a step: a step that does
 * not finish in time (another rank stopped calling) returns
 * VOX_ERR_DEVICE_TIMEOUT after aborting the NCCL communicator (asynchronous
 * NCCL errors abort it at once); with the peer-memory exchange the kernels'
 * own bounded waits (2 s) end the step.  The context is then unusable: every
 * later step fails; destroy it. */
int vox_tp_set_timeout_ms(vox_tp* tp, unsigned timeout_ms);
int vox_tp_record_event(vox_tp* tp, int slot);  /* slots 0..7 */
int vox_tp_event_elapsed_ms(vox_tp* tp, int slot_a, int slot_b, float* ms);
uint64_t vox_tp_kernel_launches(const vox_tp* tp);
/* ---- streaming decode driver (stream.rs, pipeline.rs) ---------------------------- */
/* StreamPromptConfig (stream.rs:4-9). */
typedef struct vox_stream_prompt_config {
    size_t left_pad_tokens;
    size_t delay_tokens;
    size_t eos_extra_tokens;
} vox_stream_prompt_config;
/* StreamPromptConfig::default (stream.rs:11-19): 32 / 6 / 10. */
void vox_stream_prompt_config_default(vox_stream_prompt_config* out);
/* StreamPromptConfig::right_pad_tokens (stream.rs:21-25). */
size_t vox_stream_right_pad_tokens(const vox_stream_prompt_config* cfg);
/* build_prompt_ids (stream.rs:26-34): [bos] + [pad] * (left_pad + delay).
 * Returns the prompt length and writes at most cap ids (out nullable). */
size_t vox_stream_build_prompt_ids(uint32_t bos_id, uint32_t streaming_pad_id,
                                   const vox_stream_prompt_config* cfg, uint32_t* out, size_t cap);
/* decode_ready (stream.rs:36-38) and decodable_token_budget (stream.rs:47-53). */
int vox_stream_decode_ready(size_t total_adapter_tokens, size_t prompt_len);
size_t vox_stream_decodable_token_budget(size_t total_adapter_tokens, size_t prompt_len);
/* finish_zero_padding_samples (stream.rs:60-69); 0 if samples_per_token is 0. */
size_t vox_stream_finish_zero_padding_samples(size_t consumed_samples, size_t samples_per_token,
                                              const vox_stream_prompt_config* cfg);

/* PipelineConfig (pipeline.rs:12-18). */
typedef struct vox_pipeline_config {
    uint32_t bos_id;
    uint32_t streaming_pad_id;
    size_t samples_per_token;
    vox_stream_prompt_config prompt;
} vox_pipeline_config;
/* PipelineState (pipeline.rs:28-90) driving the token loop.  With ctx and kv
 * NULL it is the reference's planner only (push / decodable_now /
 * mark_decoded / finish_padding_samples).  With a context and a
 * single-stream cache it also decodes on the device: adapter rows pushed
 * with vox_pipeline_push_adapter_tokens go to a device ring of
 * adapter_capacity positions (>= the prompt length), and
 * vox_pipeline_decode runs the schedule of the design document
 * (docs/plans/2026-02-11-voxtral-rust-design.md:40-46): with a prompt of L
 * ids, positions 0..L-2 are prefilled with adapter[p] + tok_embed(prompt[p]),
 * position L-1 yields the first token, and every later position p feeds
 * adapter[p] + tok_embed(previous token), greedy, on the device.  Destroy a
 * pipeline before its cache and context. */
typedef struct vox_pipeline vox_pipeline;
int vox_pipeline_create(vox_ctx* ctx, vox_kv* kv, const vox_pipeline_config* cfg, size_t adapter_capacity,
                        vox_pipeline** out);
void vox_pipeline_destroy(vox_pipeline* p);
/* PipelineState::prompt_ids: returns the length, writes at most cap ids. */
size_t vox_pipeline_prompt_ids(const vox_pipeline* p, uint32_t* out, size_t cap);
size_t vox_pipeline_adapter_tokens_total(const vox_pipeline* p);   /* pipeline.rs:54 */
size_t vox_pipeline_generated_tokens(const vox_pipeline* p);       /* pipeline.rs:58 */
size_t vox_pipeline_decodable_now(const vox_pipeline* p);          /* pipeline.rs:68-71 */
int vox_pipeline_is_finished(const vox_pipeline* p);               /* pipeline.rs:87 */
/* push_adapter_tokens (pipeline.rs:62-67).  rows [n_tokens, dim] f32 host
 * memory (NULL allowed for a planner-only pipeline).  VOX_ERR_RANGE if the
 * ring would overwrite positions not yet handed to vox_pipeline_decode. */
int vox_pipeline_push_adapter_tokens(vox_pipeline* p, const float* rows, size_t n_tokens);
/* mark_decoded (pipeline.rs:73-76), planner-only pipelines: a pipeline with a
 * context counts the tokens vox_pipeline_decode produces itself.
 * VOX_ERR_INVALID_ARG when n_tokens > decodable_now (the reference's
 * debug_assert). */
int vox_pipeline_mark_decoded(vox_pipeline* p, size_t n_tokens);
/* Decode min(max_tokens, decodable_now) tokens on the device (the first call
 * also prefills the prompt); tokens_out receives them, *n_out their count. */
int vox_pipeline_decode(vox_pipeline* p, size_t max_tokens, int32_t* tokens_out, size_t* n_out);
/* finish_padding_samples (pipeline.rs:78-85): marks the pipeline finished and
 * returns the zero samples to append. */
size_t vox_pipeline_finish_padding_samples(vox_pipeline* p, size_t consumed_audio_samples);

/* ---- safetensors checkpoints (weights.rs) --------------------------------------- */
/* WeightStore (weights.rs:16-42): a read-only memory map of a .safetensors
 * file whose header is validated at open (8-byte little-endian length <= 1e8,
 * JSON {name: {dtype, shape, data_offsets}} + optional "__metadata__",
 * tensors packed back to back covering the data section exactly, each of
 * numel * element-size bytes).  VOX_ERR_IO if the file cannot be read,
 * VOX_ERR_FORMAT if it is not valid safetensors. */
typedef struct vox_weights vox_weights;
typedef enum vox_tensor_dtype {
    VOX_DT_BOOL = 0, VOX_DT_U8, VOX_DT_I8, VOX_DT_F8_E5M2, VOX_DT_F8_E4M3, VOX_DT_I16, VOX_DT_U16,
    VOX_DT_F16, VOX_DT_BF16, VOX_DT_I32, VOX_DT_U32, VOX_DT_F32, VOX_DT_F64, VOX_DT_I64, VOX_DT_U64
} vox_tensor_dtype;
int vox_weights_open(const char* path, vox_weights** out);
void vox_weights_close(vox_weights* w);
/* names (weights.rs:44-47): count, then the i-th name (in data-offset order;
 * the reference's order is unspecified).  NULL when i is out of range. */
size_t vox_weights_count(const vox_weights* w);
const char* vox_weights_name(const vox_weights* w, size_t i);
/* dtype (vox_tensor_dtype), rank and up to shape_cap dims of a tensor. */
int vox_weights_info(const vox_weights* w, const char* name, int* dtype, size_t* shape, size_t shape_cap,
                     size_t* ndim);
/* tensor_f32 (weights.rs:49-93): F32 copied, BF16 widened exactly
 * (bits << 16); any other dtype is VOX_ERR_FORMAT ("unsupported dtype").
 * *n_elems receives the element count; out NULL is a size query. */
int vox_weights_tensor_f32(const vox_weights* w, const char* name, float* out, size_t cap_elems,
                           size_t* n_elems);
/* Load a decoder checkpoint into a context (copies to the device; the file
 * can be closed afterwards).  Tensor names, as in the reference's checkpoint
 * (e2e_model_env.rs:23-32 checks the first two):
 *   layers.{l}.attention.{wq,wk,wv,wo}.weight, layers.{l}.attention_norm.weight,
 *   layers.{l}.feed_forward.{w1,w2,w3}.weight, layers.{l}.ffn_norm.weight
 *   for l < n_layers; with a vocabulary also VOX_CKPT_EMBED, VOX_CKPT_FINAL_NORM
 *   and VOX_CKPT_LM_HEAD (absent = the LM head is tied to the embedding,
 *   params.rs tied_embeddings).  BF16 or F32 tensors; matrices are rounded to
 *   the context's weight dtype (nearest even), norms kept in f32.  Shapes are
 *   checked by element count against the context's config.  The reference
 *   parses ada_rms_norm_t_cond (params.rs:24-27) but its decoder never applies
 *   it; neither does this loader (a caller can fold a fixed modulation into
 *   ffn_norm through vox_ctx_upload_layer_*). */
#define VOX_CKPT_EMBED "mm_streams_embeddings.embedding_module.tok_embeddings.weight"
#define VOX_CKPT_LM_HEAD "output.weight"
#define VOX_CKPT_FINAL_NORM "norm.weight"
int vox_ctx_load_checkpoint(vox_ctx* ctx, const vox_weights* w);

/* ---- Tekken tokenizer decode (tokenizer.rs) ------------------------------------- */
/* TekkenTokenizer (tokenizer.rs:26-214): ids -> bytes -> text after the token
 * loop's argmax.  Functions returning int without a status return 1 for the
 * reference's Some and 0 for None. */
typedef struct vox_tekken vox_tekken;
/* TekkenAudioConfig (tokenizer.rs:17-23). */
typedef struct vox_tekken_audio_config {
    uint32_t sampling_rate;
    float frame_rate;
    size_t transcription_delay_ms;
    size_t streaming_n_left_pad_tokens;
} vox_tekken_audio_config;
/* from_json_str (tokenizer.rs:72-130) / from_path (:132-137): VOX_ERR_FORMAT
 * for malformed JSON, missing or mistyped fields, default_vocab_size 0 or
 * invalid base64 (standard alphabet, canonical padding); VOX_ERR_IO if the
 * file cannot be read. */
int vox_tekken_from_json(const char* json, size_t len, vox_tekken** out);
int vox_tekken_from_path(const char* path, vox_tekken** out);
void vox_tekken_destroy(vox_tekken* t);
size_t vox_tekken_default_vocab_size(const vox_tekken* t);      /* tokenizer.rs:139 */
size_t vox_tekken_special_token_count(const vox_tekken* t);     /* tokenizer.rs:143 */
/* special_id (tokenizer.rs:147); bos "<s>", eos "</s>", "[STREAMING_PAD]". */
int vox_tekken_special_id(const vox_tekken* t, const char* text, uint32_t* id);
int vox_tekken_audio(const vox_tekken* t, vox_tekken_audio_config* out);     /* tokenizer.rs:163 */
/* transcription_delay_tokens (tokenizer.rs:167-171): round(ms / 1000 * frame_rate). */
int vox_tekken_transcription_delay_tokens(const vox_tekken* t, size_t* out);
/* default_prompt_ids (tokenizer.rs:173-184): [bos] + [pad] * (left pad + delay);
 * *len = length, at most cap ids written. */
int vox_tekken_default_prompt_ids(const vox_tekken* t, uint32_t* out, size_t cap, size_t* len);
/* decode_token_bytes (tokenizer.rs:186-203): None for ids beyond the vocab,
 * control specials and vocab ids without bytes.  *bytes stays valid while
 * the tokenizer lives. */
int vox_tekken_decode_token_bytes(const vox_tekken* t, uint32_t token_id, const uint8_t** bytes, size_t* len);
/* decode_to_utf8_lossy (tokenizer.rs:204-213): concatenated bytes decoded as
 * UTF-8 with each maximal invalid subpart replaced by U+FFFD.  Returns the
 * text's byte length; writes at most cap - 1 bytes plus a NUL (out nullable). */
size_t vox_tekken_decode_to_utf8_lossy(const vox_tekken* t, const uint32_t* ids, size_t n, char* out, size_t cap);

/* ---- encoder front end on the GPU (mel.rs, conv.rs) -------------------------------- */
/* MelCtx (mel.rs:114-272): incremental log-mel frames [frames, 128] of 16 kHz
 * audio (periodic Hann 400, hop 160, 201-bin DFT, Slaney mel filters, log10
 * clamp), computed on `device`.  The internal buffer starts with
 * 200 + left_pad_samples zeros, as MelCtx::new does. */
typedef struct vox_mel vox_mel;
int vox_mel_create(int device, size_t left_pad_samples, vox_mel** out);
void vox_mel_destroy(vox_mel* m);
size_t vox_mel_left_pad_samples(const vox_mel* m);                  /* mel.rs:154 */
/* feed (mel.rs:159-166): append samples, compute every complete frame;
 * *new_frames (nullable) receives how many. */
int vox_mel_feed(vox_mel* m, const float* samples, size_t n, size_t* new_frames);
/* finish (mel.rs:170-202): right_pad_samples zeros, a 200-sample reflection,
 * the remaining frames, then the last frame dropped. */
int vox_mel_finish(vox_mel* m, size_t right_pad_samples);
size_t vox_mel_frames(const vox_mel* m);
/* data (mel.rs:206): frames [first, first + n) copied to out [n, 128]. */
int vox_mel_data(vox_mel* m, size_t first_frame, size_t n_frames, float* out);

/* ConvStemState (conv.rs:134-347) with ConvStemWeights (conv.rs:80-87):
 * conv0 (mel_bins -> dim, kernel 3, stride 1) and conv1 (dim -> dim, kernel 3,
 * stride 2), causal, GELU (tanh form) after each, on `device`.  Weights are
 * [dim, cin, 3] f32 host arrays (copied). */
typedef struct vox_conv_stem vox_conv_stem;
int vox_conv_stem_create(int device, size_t mel_bins, size_t dim, const float* conv0_weight,
                         const float* conv0_bias, const float* conv1_weight, const float* conv1_bias,
                         vox_conv_stem** out);
void vox_conv_stem_destroy(vox_conv_stem* s);
/* process (conv.rs:163-334): mel_new [n_new, mel_bins] host; out [*n_out, dim]
 * host with room for out_cap_rows rows (n_new / 2 + 1 always suffice). */
int vox_conv_stem_process(vox_conv_stem* s, const float* mel_new, size_t n_new, float* out,
                          size_t out_cap_rows, size_t* n_out);
/* causal_conv1d_colmajor (conv.rs:28-73) for kernel 3, stride 1 or 2, with
 * gelu_inplace (conv.rs:11-19) after it when apply_gelu; input [cin, length]
 * and output [cout, vox_conv_out_len(length, 3, stride)] column-major host
 * arrays; bias nullable. */
size_t vox_conv_out_len(size_t length, size_t kernel, size_t stride);
int vox_causal_conv1d_gelu(int device, const float* input, const float* weight, const float* bias, size_t cin,
                           size_t cout, size_t length, size_t stride, int apply_gelu, float* output);
/* Kernel launches issued by a mel context and a conv stem (either nullable). */
uint64_t vox_encoder_kernel_launches(const vox_mel* m, const vox_conv_stem* s);

/* ---- profiling hook (no reference counterpart) --------------------------------- */
/* Times one of the step's weight-streaming GEMVs on its own: n_launches
 * back-to-back launches (cycling over the layers, so every launch streams a
 * different matrix from HBM) with programmatic dependent launch, bracketed by
 * CUDA events on the context's stream.  which: 1 o-proj, 2 w1|w3 (SwiGLU),
 * 3 w2, 4 LM head.  Writes activations only (no cache state changes).
 * avg_ms = mean duration per launch; bytes_per_launch = weight bytes each
 * launch streams. */
int vox_profile_gemv(vox_ctx* ctx, int which, size_t n_launches, float* avg_ms,
                     uint64_t* bytes_per_launch);

/* Same for the multi-stream tensor-core GEMM with n_streams input vectors
 * (needs the embedding and LM head): which 1 o-proj, 2 w1|w3 (SwiGLU),
 * 3 w2, 4 LM head, 5 q|k|v (plain store), 6 o-proj + w1|w3 + w2 + q|k|v as
 * one persistent launch (bytes_per_launch counts all four). */
int vox_profile_bgemm(vox_ctx* ctx, int which, size_t n_streams, size_t n_launches, float* avg_ms,
                      uint64_t* bytes_per_launch);
/* ---- op-level entry points (host buffers) ------------------------------------ */
/* linear (ops.rs:11-39): out[n_rows, out_dim] = input[n_rows, in_dim] * W^T + bias. */
int vox_linear_f32(vox_ctx* ctx, const float* input, size_t n_rows, size_t in_dim,
                   const float* weight, size_t out_dim, const float* bias, float* out);
int vox_linear_bf16(vox_ctx* ctx, const float* input, size_t n_rows, size_t in_dim,
                    const uint16_t* weight, size_t out_dim, const float* bias, float* out);
/* linear (ops.rs:11-39) with bf16 weights for up to 8 input rows at once, on
 * the tensor cores (tcgen05, f32 accumulation; each f32 input is carried as a
 * bf16 hi + lo pair).  in_dim a multiple of 64.  The weights are streamed
 * once for all rows: the multi-stream decode shape. */
int vox_linear_batched_bf16(vox_ctx* ctx, const float* input, size_t n_rows, size_t in_dim,
                            const uint16_t* weight, size_t out_dim, const float* bias, float* out);
/* add_inplace (ops.rs:41-46). */
int vox_add_inplace(vox_ctx* ctx, float* dst, const float* src, size_t n);
/* attention_gqa_step (ops.rs:66-132): q [n_heads, head_dim]; keys/values
 * [seq_len, n_kv_heads, head_dim]; out [n_heads, head_dim]. */
int vox_attention_gqa_step(vox_ctx* ctx, const float* query, const float* keys,
                           const float* values, const vox_attention_shape* shape, float* out);
/* rms_norm_rows (math.rs:11-27). */
int vox_rms_norm_rows(vox_ctx* ctx, float* out, const float* input, const float* weight,
                      size_t n_elems, size_t dim, float eps);
/* rope_interleaved_inplace (math.rs:30-65): data [seq_len, n_heads, head_dim]. */
int vox_rope_interleaved_inplace(vox_ctx* ctx, float* data, size_t seq_len, size_t n_heads,
                                 size_t head_dim, size_t pos_offset, float theta);
/* silu_inplace (math.rs:4-9), softmax_inplace (math.rs:67-88). */
int vox_silu_inplace(vox_ctx* ctx, float* x, size_t n);
int vox_softmax_inplace(vox_ctx* ctx, float* x, size_t n);

/* ---- allocation-free attention (no counterpart in the reference) ---------------- */
/* attention_gqa_step for callers that must not allocate device memory (memory
 * owned by a pool or arena, a fixed memory budget, an allocation-free decode
 * path).  Same math as vox_attention_gqa_step, but every pointer is DEVICE
 * memory the caller owns: query [n_heads, head_dim], keys and values
 * head-major [n_kv_heads, seq_len, head_dim] (this library's cache layout),
 * out [n_heads, head_dim].  Runs on the calling thread's current device, on
 * `stream` (a cudaStream_t, 0 = default stream), and returns without
 * synchronising.  It calls no cudaMalloc/cudaFree: its split-K working memory
 * is a fixed 1 MiB device array inside the library, reserved on every GPU
 * that loads it until the process exits.  Shapes whose per-split data
 * (n_heads * (head_dim + 2) * 4 bytes) cannot fit are rejected with
 * VOX_ERR_UNSUPPORTED.  The first call on a device performs a one-time
 * set-up (looks up the array's device address, sets a kernel attribute), so
 * make that first call before any stream capture.  All calls on a device
 * share the array: calls that can overlap on the GPU (other streams, other
 * threads) race and must be serialised by the caller.  The array's device
 * address is looked up once per device: do not use this entry point on a
 * device after resetting it (cudaDeviceReset).  Errors are reported for the
 * arguments and for the launch only: the call returns before the kernel
 * runs, so a bounded wait that expires inside the kernel (the output is then
 * incomplete) is not reported; use vox_attention_gqa_step where that status
 * is needed.  A CUDA error already pending on the calling thread is reported
 * as VOX_ERR_CUDA and nothing is launched. */
int vox_attention_gqa_step_noalloc(const float* d_query, const float* d_keys,
                                   const float* d_values, const vox_attention_shape* shape,
                                   float* d_out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* VOX_DECODER_H */
