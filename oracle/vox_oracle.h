/*
 * vox_oracle.h -- CPU oracle for the voxtral-rust decoder token loop.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * crate's CPU kernels (crates/voxtral/src/{math,ops,kv,decoder}.rs).  It is
 * the checker the CUDA library is compared against; nothing in the product
 * path links, loads or calls it.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg use it.
 *
 * Exactness rules followed throughout (they mirror what rustc emits for the
 * reference): f32 arithmetic, the same loop order for every reduction, no
 * FMA contraction and no fast-math (the Makefile passes -ffp-contract=off),
 * and libm expf/powf/sinf/cosf for Rust's f32::exp/powf/sin_cos.
 *
 * Parity pin: the reference is Rust and no Rust toolchain exists in this
 * build environment, so the crate cannot be run to produce outputs.  The
 * oracle is pinned to the reference's own unit tests (their inputs and
 * expected values are committed as fixtures under tests/golden/).
 */
#ifndef VOX_ORACLE_H
#define VOX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* DecoderConfig, decoder.rs:10-19 (usize fields as size_t). */
typedef struct vo_config {
    size_t dim;
    size_t hidden_dim;
    size_t n_heads;
    size_t n_kv_heads;
    size_t head_dim;
    size_t sliding_window;
    float norm_eps;
    float rope_theta;
} vo_config;

/* Error codes returned by the oracle's fallible functions (0 = Ok). */
enum {
    VO_OK = 0,
    VO_ERR_DIM = 1,          /* "dim must be > 0" */
    VO_ERR_HIDDEN_DIM = 2,   /* "hidden_dim must be > 0" */
    VO_ERR_N_HEADS = 3,      /* "n_heads must be > 0" */
    VO_ERR_N_KV_HEADS = 4,   /* "n_kv_heads must be > 0" */
    VO_ERR_HEAD_DIM = 5,     /* "head_dim must be > 0" */
    VO_ERR_GQA_DIVISIBLE = 6,/* "n_heads must be divisible by n_kv_heads" */
    VO_ERR_COVER_DIM = 7,    /* "n_heads * head_dim must cover dim" */
    VO_ERR_WINDOW = 8,       /* "sliding_window must be > 0 ..." */
    VO_ERR_HIDDEN_LEN = 9,   /* "hidden size mismatch" */
    VO_ERR_WEIGHT_SHAPE = 10,/* "<tensor> shape mismatch" */
    VO_ERR_ARG = 11          /* bad argument to a composed (non-reference) helper */
};

void vo_set_threads(int n);
int vo_get_threads(void);

/* ---- math.rs ---------------------------------------------------------- */
void vo_silu_inplace(float* x, size_t n);
void vo_rms_norm_rows(float* out, const float* in, const float* weight,
                      size_t n_elems, size_t dim, float eps);
void vo_rope_interleaved_inplace(float* data, size_t seq_len, size_t n_heads,
                                 size_t head_dim, size_t pos_offset, float theta);
void vo_softmax_inplace(float* x, size_t n);

/* ---- ops.rs ----------------------------------------------------------- */
void vo_linear(const float* input, size_t n_rows, size_t in_dim,
               const float* weight, size_t out_dim, const float* bias,
               float* out);
/* Same as vo_linear with weight[o*in+i] = f32(bf16 bits << 16) (weights.rs:77-81). */
void vo_linear_bf16(const float* input, size_t n_rows, size_t in_dim,
                    const uint16_t* weight, size_t out_dim, const float* bias,
                    float* out);
void vo_add_inplace(float* dst, const float* src, size_t n);
void vo_attention_gqa_step(const float* query, const float* keys,
                           const float* values, size_t n_heads,
                           size_t head_dim, size_t seq_len, size_t n_kv_heads,
                           size_t sliding_window, float* out);

/* ---- kv.rs ------------------------------------------------------------ */
typedef struct vo_kv vo_kv;
vo_kv* vo_kv_new(size_t n_layers, size_t n_kv_heads, size_t head_dim,
                 size_t sliding_window);
void vo_kv_free(vo_kv* kv);
vo_kv* vo_kv_clone(const vo_kv* kv);
void vo_kv_append_layer(vo_kv* kv, size_t layer, const float* k_new,
                        const float* v_new, size_t n_new_tokens);
size_t vo_kv_layer_len_tokens(const vo_kv* kv, size_t layer);
size_t vo_kv_layer_pos_offset(const vo_kv* kv, size_t layer);
const float* vo_kv_layer_keys(const vo_kv* kv, size_t layer);
const float* vo_kv_layer_values(const vo_kv* kv, size_t layer);
/* Overwrite a layer's logical contents (used to pre-fill a context). */
int vo_kv_layer_set(vo_kv* kv, size_t layer, const float* keys,
                    const float* values, size_t len_tokens, size_t pos_offset);

/* ---- decoder.rs ------------------------------------------------------- */
typedef struct vo_layer_weights {
    /* Exactly one of the f32 / bf16 pointers of each matrix is used: the
     * bf16 ones when `bf16` is non-zero.  Norm gains are always f32. */
    int bf16;
    const float* attention_norm;
    const float* ffn_norm;
    const float *wq, *wk, *wv, *wo, *w1, *w2, *w3;
    const uint16_t *wq_h, *wk_h, *wv_h, *wo_h, *w1_h, *w2_h, *w3_h;
} vo_layer_weights;

int vo_config_validate(const vo_config* cfg);
int vo_decoder_layer_forward_step(const vo_config* cfg, size_t layer_idx,
                                  const vo_layer_weights* w, vo_kv* cache,
                                  const float* hidden, size_t hidden_len,
                                  size_t pos, float* out);

/* ---- composed token loop (not in the reference: it has one layer step) */
typedef struct vo_model {
    vo_config cfg;
    size_t n_layers;
    size_t vocab;
    const vo_layer_weights* layers; /* n_layers entries */
    const uint16_t* embed;          /* [vocab, dim] bf16 */
    const float* final_norm;        /* [dim] */
    const uint16_t* lm_head;        /* [vocab, dim] bf16 */
} vo_model;

int vo_model_step(const vo_model* m, vo_kv* cache, int32_t token, size_t pos,
                  float* logits_out, int32_t* argmax_out);
/* Streaming input: x = adapter_row + widen(embed[token]) (design doc :40-46). */
int vo_model_step_adapter(const vo_model* m, vo_kv* cache, int32_t token,
                          const float* adapter_row, size_t pos,
                          float* logits_out, int32_t* argmax_out);

/* ---- streaming schedule (stream.rs, pipeline.rs) ------------------------ */
typedef struct vo_stream_prompt_config {   /* StreamPromptConfig (stream.rs:4-9) */
    size_t left_pad_tokens;
    size_t delay_tokens;
    size_t eos_extra_tokens;
} vo_stream_prompt_config;

size_t vo_stream_right_pad_tokens(const vo_stream_prompt_config* c);
size_t vo_stream_build_prompt_ids(uint32_t bos_id, uint32_t pad_id,
                                  const vo_stream_prompt_config* c,
                                  uint32_t* out, size_t cap);
int vo_stream_decode_ready(size_t total_adapter_tokens, size_t prompt_len);
size_t vo_stream_decodable_token_budget(size_t total_adapter_tokens, size_t prompt_len);
size_t vo_stream_finish_zero_padding_samples(size_t consumed_samples, size_t samples_per_token,
                                             const vo_stream_prompt_config* c);

typedef struct vo_pipeline {               /* PipelineState (pipeline.rs:28-35) */
    uint32_t bos_id, streaming_pad_id;
    size_t samples_per_token;
    vo_stream_prompt_config prompt;
    size_t prompt_len;
    size_t adapter_tokens_total;
    size_t generated_tokens;
    int finished;
} vo_pipeline;

void vo_pipeline_init(vo_pipeline* p, uint32_t bos_id, uint32_t pad_id, size_t samples_per_token,
                      const vo_stream_prompt_config* prompt);
void vo_pipeline_push_adapter_tokens(vo_pipeline* p, size_t n_tokens);
size_t vo_pipeline_decodable_now(const vo_pipeline* p);
int vo_pipeline_mark_decoded(vo_pipeline* p, size_t n_tokens);
size_t vo_pipeline_finish_padding_samples(vo_pipeline* p, size_t consumed_audio_samples);

/* ---- seeded synthetic data (counter-based, bit-exact on any IEEE target) */
void vo_gen_normal_f32(uint64_t seed, uint64_t tensor_id, float std_scale,
                       uint64_t first, size_t n, float* out);
void vo_gen_normal_bf16(uint64_t seed, uint64_t tensor_id, float std_scale,
                        uint64_t first, size_t n, uint16_t* out);
void vo_gen_uniform_ids(uint64_t seed, uint64_t tensor_id, uint32_t bound,
                        uint64_t first, size_t n, int32_t* out);
uint16_t vo_f32_to_bf16_rne(float f);

/* ---- encoder front end (mel.rs, conv.rs; vox_oracle_encoder.c) ---------- */
typedef struct vo_mel vo_mel;
void vo_mel_build_filters(float* filters);          /* [128, 201] */
void vo_mel_build_dft(float* cos_t, float* sin_t);  /* [201, 400] each */
void vo_mel_build_window(float* w);                 /* [400] */
vo_mel* vo_mel_new(size_t left_pad_samples);
void vo_mel_free(vo_mel* m);
size_t vo_mel_left_pad_samples(const vo_mel* m);
size_t vo_mel_feed(vo_mel* m, const float* x, size_t n);
void vo_mel_finish(vo_mel* m, size_t right_pad_samples);
size_t vo_mel_frames(const vo_mel* m);
const float* vo_mel_data(const vo_mel* m);          /* [frames, 128] */

void vo_gelu_inplace(float* x, size_t n);
size_t vo_conv_out_len(size_t length, size_t kernel, size_t stride);
void vo_causal_conv1d_colmajor(float* output, const float* input, const float* weight, const float* bias,
                               size_t cin, size_t cout, size_t length, size_t kernel, size_t stride);
typedef struct vo_conv_stem vo_conv_stem;
vo_conv_stem* vo_conv_stem_new(size_t mel_bins, size_t dim);
void vo_conv_stem_free(vo_conv_stem* s);
size_t vo_conv_stem_process(vo_conv_stem* s, const float* w0, const float* b0, const float* w1, const float* b1,
                            const float* mel_new, size_t n_new, float* out);

#ifdef __cplusplus
}
#endif
#endif
