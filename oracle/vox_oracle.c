/*
 * vox_oracle.c -- CPU oracle for the voxtral-rust decoder token loop.
 *
 * TEST INFRASTRUCTURE ONLY (see vox_oracle.h).  Every function restates one
 * function of the reference crate and cites it as path:line relative to the
 * reference repository root.  Compile with -ffp-contract=off and without
 * -ffast-math so that each f32 operation rounds exactly once, in the order
 * the Rust source writes it.
 *
 * Threading: vo_linear may split the OUTPUT rows across OpenMP threads.  Each
 * output element is still one sequential sum in input order, so results are
 * bit-identical to the single-threaded loop (the reference itself is
 * single-threaded; rayon is declared in its Cargo.toml but never used).
 */
#include "vox_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 1;

void vo_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int vo_get_threads(void) { return g_threads; }

static inline float bf16_to_f32(uint16_t h) {
    /* weights.rs:77-81: f32::from_bits((bits as u32) << 16) */
    union { uint32_t u; float f; } c;
    c.u = ((uint32_t)h) << 16;
    return c.f;
}

uint16_t vo_f32_to_bf16_rne(float f) {
    union { uint32_t u; float f; } c;
    c.f = f;
    if ((c.u & 0x7F800000u) == 0x7F800000u && (c.u & 0x007FFFFFu)) return 0x7FC0;
    uint32_t u = c.u + 0x7FFFu + ((c.u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* ======================================================================
 * math.rs
 * ====================================================================== */

/* math.rs:4-9  silu_inplace: v = t / (1 + exp(-t)) */
void vo_silu_inplace(float* x, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        float t = x[i];
        x[i] = t / (1.0f + expf(-t));
    }
}

/* math.rs:11-27  rms_norm_rows: per row, sq_sum sequential, then
 * inv = 1 / sqrt(sq/dim + eps); out = x * inv * w (left to right). */
void vo_rms_norm_rows(float* out, const float* in, const float* weight,
                      size_t n_elems, size_t dim, float eps) {
    for (size_t r = 0; r + dim <= n_elems; r += dim) {
        const float* x = in + r;
        float* y = out + r;
        float sq_sum = 0.0f;
        for (size_t i = 0; i < dim; ++i) sq_sum += x[i] * x[i];
        float inv_rms = 1.0f / sqrtf(sq_sum / (float)dim + eps);
        for (size_t i = 0; i < dim; ++i) y[i] = x[i] * inv_rms * weight[i];
    }
}

/* math.rs:30-65  rope_interleaved_inplace (GPT-J pairs (2p, 2p+1)).
 * inv_freq = theta.powf(-(2p as f32) / (head_dim as f32)); angle = pos*inv;
 * (sin, cos) = angle.sin_cos(). */
void vo_rope_interleaved_inplace(float* data, size_t seq_len, size_t n_heads,
                                 size_t head_dim, size_t pos_offset, float theta) {
    size_t row_stride = n_heads * head_dim;
    for (size_t t = 0; t < seq_len; ++t) {
        float pos = (float)(pos_offset + t);
        float* row = data + t * row_stride;
        for (size_t h = 0; h < n_heads; ++h) {
            float* head = row + h * head_dim;
            for (size_t pair = 0; pair < head_dim / 2; ++pair) {
                size_t i0 = 2 * pair, i1 = i0 + 1;
                float inv_freq = powf(theta, -((float)i0) / (float)head_dim);
                float angle = pos * inv_freq;
                float s = sinf(angle), c = cosf(angle);
                float x0 = head[i0], x1 = head[i1];
                head[i0] = x0 * c - x1 * s;
                head[i1] = x0 * s + x1 * c;
            }
        }
    }
}

/* math.rs:67-88  softmax_inplace: max (strict >), exp(x-max) summed in
 * order, divide only when sum > 0. */
void vo_softmax_inplace(float* x, size_t n) {
    if (n == 0) return;
    float max_v = x[0];
    for (size_t i = 1; i < n; ++i)
        if (x[i] > max_v) max_v = x[i];
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        x[i] = expf(x[i] - max_v);
        sum += x[i];
    }
    if (sum > 0.0f)
        for (size_t i = 0; i < n; ++i) x[i] /= sum;
}

/* ======================================================================
 * ops.rs
 * ====================================================================== */

/* ops.rs:11-39  linear: y[r,o] = (bias[o] or 0) + sum_i x[r,i]*W[o,i],
 * accumulated sequentially in i. */
void vo_linear(const float* input, size_t n_rows, size_t in_dim,
               const float* weight, size_t out_dim, const float* bias,
               float* out) {
    for (size_t r = 0; r < n_rows; ++r) {
        const float* x = input + r * in_dim;
        float* y = out + r * out_dim;
        long long n_out = (long long)out_dim;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && out_dim >= 64)
        for (long long o = 0; o < n_out; ++o) {
            const float* w = weight + (size_t)o * in_dim;
            float sum = bias ? bias[o] : 0.0f;
            for (size_t i = 0; i < in_dim; ++i) sum += x[i] * w[i];
            y[o] = sum;
        }
    }
}

void vo_linear_bf16(const float* input, size_t n_rows, size_t in_dim,
                    const uint16_t* weight, size_t out_dim, const float* bias,
                    float* out) {
    for (size_t r = 0; r < n_rows; ++r) {
        const float* x = input + r * in_dim;
        float* y = out + r * out_dim;
        long long n_out = (long long)out_dim;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && out_dim >= 64)
        for (long long o = 0; o < n_out; ++o) {
            const uint16_t* w = weight + (size_t)o * in_dim;
            float sum = bias ? bias[o] : 0.0f;
            for (size_t i = 0; i < in_dim; ++i) sum += x[i] * bf16_to_f32(w[i]);
            y[o] = sum;
        }
    }
}

/* ops.rs:41-46 */
void vo_add_inplace(float* dst, const float* src, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] += src[i];
}

/* ops.rs:66-132  attention_gqa_step.  One query token; keys/values are
 * token-major [seq_len, n_kv_heads, head_dim].  kv head = h / (n_heads /
 * n_kv_heads).  Tokens t < seq_len - window (window != 0) score -inf.
 * scores = dot * (1/sqrt(head_dim)); softmax; PV skips exact-zero weights. */
static void attention_one_head(const float* q, const float* keys,
                               const float* values, size_t head_dim,
                               size_t seq_len, size_t n_kv_heads, size_t kv_h,
                               size_t start, float scale, float* scores,
                               float* out_h) {
    for (size_t t = 0; t < seq_len; ++t) {
        if (t < start) {
            scores[t] = -INFINITY;
            continue;
        }
        const float* k = keys + (t * n_kv_heads + kv_h) * head_dim;
        float dot = 0.0f;
        for (size_t i = 0; i < head_dim; ++i) dot += q[i] * k[i];
        scores[t] = dot * scale;
    }
    vo_softmax_inplace(scores, seq_len);
    for (size_t i = 0; i < head_dim; ++i) out_h[i] = 0.0f;
    for (size_t t = 0; t < seq_len; ++t) {
        float a = scores[t];
        if (a == 0.0f) continue;
        const float* v = values + (t * n_kv_heads + kv_h) * head_dim;
        for (size_t i = 0; i < head_dim; ++i) out_h[i] += a * v[i];
    }
}

void vo_attention_gqa_step(const float* query, const float* keys,
                           const float* values, size_t n_heads,
                           size_t head_dim, size_t seq_len, size_t n_kv_heads,
                           size_t sliding_window, float* out) {
    size_t kv_group = n_heads / n_kv_heads;
    float scale = 1.0f / sqrtf((float)head_dim);
    size_t start = 0;
    if (sliding_window != 0 && seq_len > sliding_window) start = seq_len - sliding_window;
    long long nh = (long long)n_heads;
#pragma omp parallel num_threads(g_threads) if (g_threads > 1 && seq_len * head_dim >= 4096)
    {
        float* scores = (float*)malloc((seq_len ? seq_len : 1) * sizeof(float));
#pragma omp for schedule(static)
        for (long long h = 0; h < nh; ++h) {
            attention_one_head(query + (size_t)h * head_dim, keys, values, head_dim,
                               seq_len, n_kv_heads, (size_t)h / kv_group, start,
                               scale, scores, out + (size_t)h * head_dim);
        }
        free(scores);
    }
}

/* ======================================================================
 * kv.rs
 * ====================================================================== */

typedef struct vo_layer_kv {
    float* keys;
    float* values;
    size_t len_tokens;
    size_t pos_offset;
    size_t cap_tokens; /* allocation bookkeeping only (Vec capacity) */
} vo_layer_kv;

struct vo_kv {
    size_t n_layers, n_kv_heads, head_dim, sliding_window;
    vo_layer_kv* layers;
};

/* kv.rs:33-46 RollingKvCache::new */
vo_kv* vo_kv_new(size_t n_layers, size_t n_kv_heads, size_t head_dim,
                 size_t sliding_window) {
    vo_kv* kv = (vo_kv*)calloc(1, sizeof(vo_kv));
    kv->n_layers = n_layers;
    kv->n_kv_heads = n_kv_heads;
    kv->head_dim = head_dim;
    kv->sliding_window = sliding_window;
    kv->layers = (vo_layer_kv*)calloc(n_layers ? n_layers : 1, sizeof(vo_layer_kv));
    return kv;
}

void vo_kv_free(vo_kv* kv) {
    if (!kv) return;
    for (size_t l = 0; l < kv->n_layers; ++l) {
        free(kv->layers[l].keys);
        free(kv->layers[l].values);
    }
    free(kv->layers);
    free(kv);
}

vo_kv* vo_kv_clone(const vo_kv* src) {
    vo_kv* kv = vo_kv_new(src->n_layers, src->n_kv_heads, src->head_dim, src->sliding_window);
    size_t stride = src->n_kv_heads * src->head_dim;
    for (size_t l = 0; l < src->n_layers; ++l) {
        const vo_layer_kv* s = &src->layers[l];
        vo_layer_kv* d = &kv->layers[l];
        d->len_tokens = s->len_tokens;
        d->pos_offset = s->pos_offset;
        d->cap_tokens = s->len_tokens;
        size_t bytes = s->len_tokens * stride * sizeof(float);
        d->keys = (float*)malloc(bytes ? bytes : 4);
        d->values = (float*)malloc(bytes ? bytes : 4);
        if (bytes) {
            memcpy(d->keys, s->keys, bytes);
            memcpy(d->values, s->values, bytes);
        }
    }
    return kv;
}

static void layer_reserve(vo_layer_kv* c, size_t tokens, size_t stride) {
    if (tokens <= c->cap_tokens) return;
    size_t cap = c->cap_tokens ? c->cap_tokens : 4;
    while (cap < tokens) cap *= 2;
    c->keys = (float*)realloc(c->keys, cap * stride * sizeof(float));
    c->values = (float*)realloc(c->values, cap * stride * sizeof(float));
    c->cap_tokens = cap;
}

/* kv.rs:48-88 append_layer.
 * drop = (len + n) saturating_sub window.  When drop > 0: keep = len
 * saturating_sub drop; keep == 0 clears the layer, otherwise the oldest
 * `drop` tokens are drained (memmove of the kept tail to the front);
 * pos_offset += drop in both cases.  Then the new tokens are appended. */
void vo_kv_append_layer(vo_kv* kv, size_t layer, const float* k_new,
                        const float* v_new, size_t n_new_tokens) {
    if (n_new_tokens == 0) return;
    size_t stride = kv->n_kv_heads * kv->head_dim;
    vo_layer_kv* c = &kv->layers[layer];
    size_t requested = c->len_tokens + n_new_tokens;
    size_t drop = requested > kv->sliding_window ? requested - kv->sliding_window : 0;
    if (drop > 0) {
        size_t keep = c->len_tokens > drop ? c->len_tokens - drop : 0;
        if (keep == 0) {
            c->len_tokens = 0;
        } else {
            memmove(c->keys, c->keys + drop * stride, keep * stride * sizeof(float));
            memmove(c->values, c->values + drop * stride, keep * stride * sizeof(float));
            c->len_tokens = keep;
        }
        c->pos_offset += drop;
    }
    layer_reserve(c, c->len_tokens + n_new_tokens, stride);
    memcpy(c->keys + c->len_tokens * stride, k_new, n_new_tokens * stride * sizeof(float));
    memcpy(c->values + c->len_tokens * stride, v_new, n_new_tokens * stride * sizeof(float));
    c->len_tokens += n_new_tokens;
}

/* kv.rs:90-101 observers */
size_t vo_kv_layer_len_tokens(const vo_kv* kv, size_t layer) { return kv->layers[layer].len_tokens; }
size_t vo_kv_layer_pos_offset(const vo_kv* kv, size_t layer) { return kv->layers[layer].pos_offset; }
const float* vo_kv_layer_keys(const vo_kv* kv, size_t layer) { return kv->layers[layer].keys; }
const float* vo_kv_layer_values(const vo_kv* kv, size_t layer) { return kv->layers[layer].values; }

int vo_kv_layer_set(vo_kv* kv, size_t layer, const float* keys,
                    const float* values, size_t len_tokens, size_t pos_offset) {
    if (layer >= kv->n_layers) return VO_ERR_ARG;
    size_t stride = kv->n_kv_heads * kv->head_dim;
    vo_layer_kv* c = &kv->layers[layer];
    layer_reserve(c, len_tokens, stride);
    if (len_tokens) {
        memcpy(c->keys, keys, len_tokens * stride * sizeof(float));
        memcpy(c->values, values, len_tokens * stride * sizeof(float));
    }
    c->len_tokens = len_tokens;
    c->pos_offset = pos_offset;
    return VO_OK;
}

/* ======================================================================
 * decoder.rs
 * ====================================================================== */

/* decoder.rs:22-41 DecoderConfig::validate (same check order). */
int vo_config_validate(const vo_config* c) {
    if (c->dim == 0) return VO_ERR_DIM;
    if (c->hidden_dim == 0) return VO_ERR_HIDDEN_DIM;
    if (c->n_heads == 0) return VO_ERR_N_HEADS;
    if (c->n_kv_heads == 0) return VO_ERR_N_KV_HEADS;
    if (c->head_dim == 0) return VO_ERR_HEAD_DIM;
    if (c->n_heads % c->n_kv_heads != 0) return VO_ERR_GQA_DIVISIBLE;
    if (c->n_heads * c->head_dim < c->dim) return VO_ERR_COVER_DIM;
    if (c->sliding_window == 0) return VO_ERR_WINDOW;
    return VO_OK;
}

static void lin(const vo_layer_weights* w, const float* f, const uint16_t* h,
                const float* x, size_t in_dim, size_t out_dim, float* y) {
    if (w->bf16)
        vo_linear_bf16(x, 1, in_dim, h, out_dim, NULL, y);
    else
        vo_linear(x, 1, in_dim, f, out_dim, NULL, y);
}

/* decoder.rs:88-155 decoder_layer_forward_step.  Weight lengths are the
 * caller's responsibility here (decoder.rs:58-84 checks Vec lengths, which
 * raw pointers do not carry). */
int vo_decoder_layer_forward_step(const vo_config* cfg, size_t layer_idx,
                                  const vo_layer_weights* w, vo_kv* cache,
                                  const float* hidden, size_t hidden_len,
                                  size_t pos, float* out) {
    int rc = vo_config_validate(cfg);
    if (rc) return rc;
    if (hidden_len != cfg->dim) return VO_ERR_HIDDEN_LEN;
    size_t dim = cfg->dim, hd = cfg->head_dim;
    size_t q_dim = cfg->n_heads * hd, kv_dim = cfg->n_kv_heads * hd;

    float* x_norm = (float*)malloc(dim * sizeof(float));
    float* q = (float*)malloc(q_dim * sizeof(float));
    float* k = (float*)malloc(kv_dim * sizeof(float));
    float* v = (float*)malloc(kv_dim * sizeof(float));
    float* attn = (float*)malloc(q_dim * sizeof(float));
    float* attn_proj = (float*)malloc(dim * sizeof(float));
    float* h = (float*)malloc(dim * sizeof(float));
    float* h_norm = (float*)malloc(dim * sizeof(float));
    float* gate = (float*)malloc(cfg->hidden_dim * sizeof(float));
    float* up = (float*)malloc(cfg->hidden_dim * sizeof(float));
    float* down = (float*)malloc(dim * sizeof(float));

    /* 1) attention branch: decoder.rs:104-139 */
    vo_rms_norm_rows(x_norm, hidden, w->attention_norm, dim, dim, cfg->norm_eps);
    lin(w, w->wq, w->wq_h, x_norm, dim, q_dim, q);
    lin(w, w->wk, w->wk_h, x_norm, dim, kv_dim, k);
    lin(w, w->wv, w->wv_h, x_norm, dim, kv_dim, v);
    vo_rope_interleaved_inplace(q, 1, cfg->n_heads, hd, pos, cfg->rope_theta);
    vo_rope_interleaved_inplace(k, 1, cfg->n_kv_heads, hd, pos, cfg->rope_theta);
    vo_kv_append_layer(cache, layer_idx, k, v, 1);
    size_t seq_len = vo_kv_layer_len_tokens(cache, layer_idx);
    vo_attention_gqa_step(q, vo_kv_layer_keys(cache, layer_idx),
                          vo_kv_layer_values(cache, layer_idx), cfg->n_heads, hd,
                          seq_len, cfg->n_kv_heads, cfg->sliding_window, attn);
    lin(w, w->wo, w->wo_h, attn, q_dim, dim, attn_proj);
    memcpy(h, hidden, dim * sizeof(float));
    vo_add_inplace(h, attn_proj, dim);

    /* 2) FFN branch: decoder.rs:141-154 */
    vo_rms_norm_rows(h_norm, h, w->ffn_norm, dim, dim, cfg->norm_eps);
    lin(w, w->w1, w->w1_h, h_norm, dim, cfg->hidden_dim, gate);
    lin(w, w->w3, w->w3_h, h_norm, dim, cfg->hidden_dim, up);
    vo_silu_inplace(gate, cfg->hidden_dim);
    for (size_t i = 0; i < cfg->hidden_dim; ++i) gate[i] *= up[i];
    lin(w, w->w2, w->w2_h, gate, cfg->hidden_dim, dim, down);
    vo_add_inplace(h, down, dim);
    memcpy(out, h, dim * sizeof(float));

    free(x_norm); free(q); free(k); free(v); free(attn); free(attn_proj);
    free(h); free(h_norm); free(gate); free(up); free(down);
    return VO_OK;
}

/* ======================================================================
 * Composed token loop.  The reference has one layer step only; the full
 * step is composed as: x = widen(embed[token]); 26 x layer step at the
 * absolute position; final RMSNorm (gain final_norm, eps norm_eps);
 * logits = linear(x, lm_head); argmax with the lowest index winning ties.
 * ====================================================================== */
/* Layers, final norm, LM head and argmax from the input vector x (consumed). */
static int model_forward(const vo_model* m, vo_kv* cache, float* x, size_t pos,
                         float* logits_out, int32_t* argmax_out) {
    const vo_config* cfg = &m->cfg;
    size_t dim = cfg->dim;
    float* y = (float*)malloc(dim * sizeof(float));
    for (size_t l = 0; l < m->n_layers; ++l) {
        int rc = vo_decoder_layer_forward_step(cfg, l, &m->layers[l], cache, x, dim, pos, y);
        if (rc) { free(x); free(y); return rc; }
        float* t = x; x = y; y = t;
    }
    vo_rms_norm_rows(y, x, m->final_norm, dim, dim, cfg->norm_eps);
    float* logits = logits_out ? logits_out : (float*)malloc(m->vocab * sizeof(float));
    vo_linear_bf16(y, 1, dim, m->lm_head, m->vocab, NULL, logits);
    if (argmax_out) {
        size_t best = 0;
        for (size_t i = 1; i < m->vocab; ++i)
            if (logits[i] > logits[best]) best = i;
        *argmax_out = (int32_t)best;
    }
    if (!logits_out) free(logits);
    free(x); free(y);
    return VO_OK;
}

int vo_model_step(const vo_model* m, vo_kv* cache, int32_t token, size_t pos,
                  float* logits_out, int32_t* argmax_out) {
    size_t dim = m->cfg.dim;
    if (token < 0 || (size_t)token >= m->vocab) return VO_ERR_ARG;
    float* x = (float*)malloc(dim * sizeof(float));
    for (size_t i = 0; i < dim; ++i) x[i] = bf16_to_f32(m->embed[(size_t)token * dim + i]);
    return model_forward(m, cache, x, pos, logits_out, argmax_out);
}

/* Streaming input (docs/plans/2026-02-11-voxtral-rust-design.md:40-46): the
 * decoder input at an adapter position is adapter[pos] + tok_embed(token),
 * one f32 addition per element. */
int vo_model_step_adapter(const vo_model* m, vo_kv* cache, int32_t token,
                          const float* adapter_row, size_t pos,
                          float* logits_out, int32_t* argmax_out) {
    size_t dim = m->cfg.dim;
    if (token < 0 || (size_t)token >= m->vocab || !adapter_row) return VO_ERR_ARG;
    float* x = (float*)malloc(dim * sizeof(float));
    for (size_t i = 0; i < dim; ++i)
        x[i] = adapter_row[i] + bf16_to_f32(m->embed[(size_t)token * dim + i]);
    return model_forward(m, cache, x, pos, logits_out, argmax_out);
}

/* ======================================================================
 * stream.rs / pipeline.rs: the streaming schedule (integer bookkeeping).
 * ====================================================================== */

/* StreamPromptConfig::right_pad_tokens (stream.rs:21-25). */
size_t vo_stream_right_pad_tokens(const vo_stream_prompt_config* c) {
    return c->delay_tokens + 1 + c->eos_extra_tokens;
}

/* build_prompt_ids (stream.rs:26-34): [bos] + [pad] * (left_pad + delay).
 * Returns the prompt length; writes at most cap ids. */
size_t vo_stream_build_prompt_ids(uint32_t bos_id, uint32_t pad_id,
                                  const vo_stream_prompt_config* c,
                                  uint32_t* out, size_t cap) {
    size_t n = 1 + c->left_pad_tokens + c->delay_tokens;
    for (size_t i = 0; i < n && i < cap; ++i) out[i] = i == 0 ? bos_id : pad_id;
    return n;
}

/* decode_ready (stream.rs:36-38). */
int vo_stream_decode_ready(size_t total_adapter_tokens, size_t prompt_len) {
    return total_adapter_tokens >= prompt_len;
}

/* decodable_token_budget (stream.rs:47-53): N - L + 1 when N >= L, else 0. */
size_t vo_stream_decodable_token_budget(size_t total_adapter_tokens, size_t prompt_len) {
    return total_adapter_tokens < prompt_len ? 0 : total_adapter_tokens - prompt_len + 1;
}

/* finish_zero_padding_samples (stream.rs:60-69): align to the token
 * boundary, then (delay + 1 + eos_extra) token steps of zeros. */
size_t vo_stream_finish_zero_padding_samples(size_t consumed_samples, size_t samples_per_token,
                                             const vo_stream_prompt_config* c) {
    if (samples_per_token == 0) return 0;
    size_t rem = consumed_samples % samples_per_token;
    size_t align = rem == 0 ? 0 : samples_per_token - rem;
    return align + vo_stream_right_pad_tokens(c) * samples_per_token;
}

/* PipelineState (pipeline.rs:28-90). */
void vo_pipeline_init(vo_pipeline* p, uint32_t bos_id, uint32_t pad_id, size_t samples_per_token,
                      const vo_stream_prompt_config* prompt) {
    p->bos_id = bos_id;
    p->streaming_pad_id = pad_id;
    p->samples_per_token = samples_per_token;
    p->prompt = *prompt;
    p->prompt_len = 1 + prompt->left_pad_tokens + prompt->delay_tokens;
    p->adapter_tokens_total = 0;
    p->generated_tokens = 0;
    p->finished = 0;
}

void vo_pipeline_push_adapter_tokens(vo_pipeline* p, size_t n_tokens) {
    p->adapter_tokens_total += n_tokens;  /* pipeline.rs:62-67 */
}

size_t vo_pipeline_decodable_now(const vo_pipeline* p) {
    size_t total = vo_stream_decodable_token_budget(p->adapter_tokens_total, p->prompt_len);
    return total > p->generated_tokens ? total - p->generated_tokens : 0;  /* saturating_sub */
}

/* pipeline.rs:73-76; the reference debug_asserts n <= decodable_now. */
int vo_pipeline_mark_decoded(vo_pipeline* p, size_t n_tokens) {
    if (n_tokens > vo_pipeline_decodable_now(p)) return VO_ERR_ARG;
    p->generated_tokens += n_tokens;
    return VO_OK;
}

size_t vo_pipeline_finish_padding_samples(vo_pipeline* p, size_t consumed_audio_samples) {
    p->finished = 1;
    return vo_stream_finish_zero_padding_samples(consumed_audio_samples, p->samples_per_token, &p->prompt);
}

/* ======================================================================
 * Seeded synthetic data.  Counter-based so that any element can be made
 * independently (and identically on the GPU):
 *   key   = mix(seed ^ mix(tensor_id + C1))
 *   h_j   = mix(key + (3e + j) * C2),  j = 0, 1, 2
 *   s     = sum of the twelve 16-bit fields of h_0..h_2
 *   z     = (2s + 12 - 12*65536) * 2^-17   (exact; Irwin-Hall(12), mean 0, var ~1)
 *   value = z * std (one f32 rounding), bf16 by round-to-nearest-even.
 * Uniform ids: (top 32 bits of h_0) * bound >> 32.
 * ====================================================================== */
static inline uint64_t mix64(uint64_t z) {
    z ^= z >> 30;
    z *= 0xBF58476D1CE4E5B9ULL;
    z ^= z >> 27;
    z *= 0x94D049BB133111EBULL;
    z ^= z >> 31;
    return z;
}

static inline uint64_t gen_key(uint64_t seed, uint64_t tensor_id) {
    return mix64(seed ^ mix64(tensor_id + 0x632BE59BD9B4E019ULL));
}

static inline float gen_z(uint64_t key, uint64_t e) {
    uint32_t s = 0;
    for (int j = 0; j < 3; ++j) {
        uint64_t h = mix64(key + (3 * e + (uint64_t)j) * 0x9E3779B97F4A7C15ULL);
        s += (uint32_t)(h & 0xFFFF) + (uint32_t)((h >> 16) & 0xFFFF) +
             (uint32_t)((h >> 32) & 0xFFFF) + (uint32_t)(h >> 48);
    }
    int32_t c = (int32_t)(2 * s + 12) - 786432;
    return (float)c * (1.0f / 131072.0f);
}

void vo_gen_normal_f32(uint64_t seed, uint64_t tensor_id, float std_scale,
                       uint64_t first, size_t n, float* out) {
    uint64_t key = gen_key(seed, tensor_id);
    long long nn = (long long)n;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && n > 65536)
    for (long long i = 0; i < nn; ++i) out[i] = gen_z(key, first + (uint64_t)i) * std_scale;
}

void vo_gen_normal_bf16(uint64_t seed, uint64_t tensor_id, float std_scale,
                        uint64_t first, size_t n, uint16_t* out) {
    uint64_t key = gen_key(seed, tensor_id);
    long long nn = (long long)n;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && n > 65536)
    for (long long i = 0; i < nn; ++i)
        out[i] = vo_f32_to_bf16_rne(gen_z(key, first + (uint64_t)i) * std_scale);
}

void vo_gen_uniform_ids(uint64_t seed, uint64_t tensor_id, uint32_t bound,
                        uint64_t first, size_t n, int32_t* out) {
    uint64_t key = gen_key(seed, tensor_id);
    for (size_t i = 0; i < n; ++i) {
        uint64_t h = mix64(key + (3 * (first + i)) * 0x9E3779B97F4A7C15ULL);
        out[i] = (int32_t)(((h >> 32) * (uint64_t)bound) >> 32);
    }
}
