/*
 * vox_oracle_encoder.c -- CPU restatement of the reference's encoder front
 * end: the incremental log-mel spectrogram (crates/voxtral/src/mel.rs:15-275)
 * and the causal conv stem (crates/voxtral/src/conv.rs:11-360).
 *
 * TEST INFRASTRUCTURE ONLY (the oracle): used by tests/ and bench.py's CPU
 * baseline as the checker, never by the product library.
 *
 * f32 throughout, the reference's loop order, no FMA contraction
 * (-ffp-contract=off), libm logf/expf/cosf/sinf/log10f/tanhf as rustc's f32
 * methods call them.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "vox_oracle.h"

/* constants.rs:4-14 */
#define SR 16000
#define MEL_BINS 128
#define HOP 160
#define WIN 400
#define NFFT 400
#define NFREQ (NFFT / 2 + 1)
#define LOG_MEL_MAX 1.5f
static const float kPi = 3.14159265358979323846f; /* std::f32::consts::PI */

/* mel.rs:15-27 (Slaney scale) */
static float hertz_to_mel(float freq) {
    const float min_log_hz = 1000.0f, min_log_mel = 15.0f, logstep = 0.06875178f;
    float mels = 3.0f * freq / 200.0f;
    if (freq >= min_log_hz) mels = min_log_mel + logf(freq / min_log_hz) * logstep;
    return mels;
}

/* mel.rs:30-40 */
static float mel_to_hertz(float mels) {
    const float min_log_hz = 1000.0f, min_log_mel = 15.0f, logstep = 0.06875178f;
    float freq = 200.0f * mels / 3.0f;
    if (mels >= min_log_mel) freq = min_log_hz * expf(logstep * (mels - min_log_mel));
    return freq;
}

/* mel.rs:42-81: filters [MEL_BINS, NFREQ] */
void vo_mel_build_filters(float* filters) {
    float fft_freqs[NFREQ], filter_freqs[MEL_BINS + 2], filter_diff[MEL_BINS + 1];
    for (int f = 0; f < NFREQ; ++f) fft_freqs[f] = (float)f * (float)SR / (float)NFFT;
    const float mel_min = hertz_to_mel(0.0f), mel_max = hertz_to_mel((float)SR / 2.0f);
    for (int i = 0; i < MEL_BINS + 2; ++i)
        filter_freqs[i] = mel_to_hertz(mel_min + (mel_max - mel_min) * (float)i / (float)(MEL_BINS + 1));
    for (int i = 0; i < MEL_BINS + 1; ++i) {
        filter_diff[i] = filter_freqs[i + 1] - filter_freqs[i];
        if (filter_diff[i] == 0.0f) filter_diff[i] = 1e-6f;
    }
    for (int m = 0; m < MEL_BINS; ++m) {
        const float denom = filter_freqs[m + 2] - filter_freqs[m];
        const float enorm = 2.0f / denom;
        for (int f = 0; f < NFREQ; ++f) {
            const float down = (fft_freqs[f] - filter_freqs[m]) / filter_diff[m];
            const float up = (filter_freqs[m + 2] - fft_freqs[f]) / filter_diff[m + 1];
            float val = down < up ? down : up; /* f32::min (no NaNs here) */
            if (val < 0.0f) val = 0.0f;
            filters[m * NFREQ + f] = val * enorm;
        }
    }
}

/* mel.rs:83-96: cos/sin [NFREQ, NFFT] */
void vo_mel_build_dft(float* cos_t, float* sin_t) {
    for (int k = 0; k < NFREQ; ++k)
        for (int n = 0; n < NFFT; ++n) {
            const float angle = 2.0f * kPi * (float)k * (float)n / (float)NFFT;
            cos_t[k * NFFT + n] = cosf(angle);
            sin_t[k * NFFT + n] = sinf(angle);
        }
}

/* mel.rs:98-106: periodic Hann */
void vo_mel_build_window(float* w) {
    for (int i = 0; i < WIN; ++i) {
        const float angle = 2.0f * kPi * (float)i / (float)WIN;
        w[i] = 0.5f * (1.0f - cosf(angle));
    }
}

struct vo_mel {
    float filters[MEL_BINS * NFREQ];
    float dft_cos[NFREQ * NFFT], dft_sin[NFREQ * NFFT];
    float window[WIN];
    float* samples;
    size_t n_samples, cap_samples;
    float* mel;
    size_t n_frames, cap_frames;
    size_t left_pad;
    int finished;
};

static void push_samples(vo_mel* m, const float* x, size_t n, int zeros) {
    if (m->n_samples + n > m->cap_samples) {
        size_t c = m->cap_samples ? m->cap_samples : 1024;
        while (c < m->n_samples + n) c *= 2;
        m->samples = (float*)realloc(m->samples, c * sizeof(float));
        m->cap_samples = c;
    }
    for (size_t i = 0; i < n; ++i) m->samples[m->n_samples + i] = zeros ? 0.0f : x[i];
    m->n_samples += n;
}

/* mel.rs:130-151 MelCtx::new */
vo_mel* vo_mel_new(size_t left_pad_samples) {
    vo_mel* m = (vo_mel*)calloc(1, sizeof(vo_mel));
    vo_mel_build_filters(m->filters);
    vo_mel_build_dft(m->dft_cos, m->dft_sin);
    vo_mel_build_window(m->window);
    m->left_pad = NFFT / 2 + left_pad_samples;
    push_samples(m, NULL, m->left_pad, 1);
    return m;
}

void vo_mel_free(vo_mel* m) {
    if (!m) return;
    free(m->samples);
    free(m->mel);
    free(m);
}

size_t vo_mel_left_pad_samples(const vo_mel* m) { return m->left_pad; }

/* mel.rs:210-271 compute_available */
static size_t compute_available(vo_mel* m) {
    size_t new_frames = 0;
    float windowed[NFFT], power[NFREQ];
    for (;;) {
        const size_t t = m->n_frames, start = t * HOP, end = start + WIN;
        if (end > m->n_samples) break;
        if (m->cap_frames < t + 1) {
            size_t c = m->cap_frames ? m->cap_frames * 2 : 64;
            m->mel = (float*)realloc(m->mel, c * MEL_BINS * sizeof(float));
            m->cap_frames = c;
        }
        for (int i = 0; i < NFFT; ++i) windowed[i] = m->samples[start + i] * m->window[i];
        for (int k = 0; k < NFREQ; ++k) {
            float re = 0.0f, im = 0.0f;
            const float* cr = m->dft_cos + k * NFFT;
            const float* sr = m->dft_sin + k * NFFT;
            for (int n = 0; n < NFFT; ++n) {
                re += windowed[n] * cr[n];
                im += windowed[n] * sr[n];
            }
            power[k] = re * re + im * im;
        }
        float* row = m->mel + t * MEL_BINS;
        for (int b = 0; b < MEL_BINS; ++b) {
            const float* filt = m->filters + b * NFREQ;
            float sum = 0.0f;
            for (int k = 0; k < NFREQ; ++k) sum += filt[k] * power[k];
            if (sum < 1e-10f) sum = 1e-10f;
            float val = log10f(sum);
            const float min_val = LOG_MEL_MAX - 8.0f;
            if (val < min_val) val = min_val;
            row[b] = (val + 4.0f) / 4.0f;
        }
        m->n_frames += 1;
        new_frames += 1;
    }
    return new_frames;
}

/* mel.rs:159-166 feed */
size_t vo_mel_feed(vo_mel* m, const float* x, size_t n) {
    if (n == 0) return 0;
    push_samples(m, x, n, 0);
    return compute_available(m);
}

/* mel.rs:170-202 finish */
void vo_mel_finish(vo_mel* m, size_t right_pad_samples) {
    if (m->finished) return;
    if (right_pad_samples > 0) push_samples(m, NULL, right_pad_samples, 1);
    const size_t reflect_len = NFFT / 2;
    const size_t real_end = m->n_samples > right_pad_samples ? m->n_samples - right_pad_samples : 0;
    for (size_t i = 0; i < reflect_len; ++i) {
        const long long src = (long long)real_end - 2 - (long long)i;
        float v = 0.0f;
        if (src >= 0 && (size_t)src < m->n_samples) v = m->samples[src];
        push_samples(m, &v, 1, 0);
    }
    compute_available(m);
    if (m->n_frames > 0) m->n_frames -= 1; /* vLLM convention: drop the last frame */
    m->finished = 1;
}

size_t vo_mel_frames(const vo_mel* m) { return m->n_frames; }
const float* vo_mel_data(const vo_mel* m) { return m->mel; }

/* ---- conv.rs ------------------------------------------------------------ */

/* conv.rs:11-19 gelu_inplace */
void vo_gelu_inplace(float* x, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        const float val = x[i];
        const float x3 = val * val * val;
        const float inner = 0.7978846f * (val + 0.044715f * x3);
        x[i] = 0.5f * val * (1.0f + tanhf(inner));
    }
}

/* conv.rs:29-34: ceil((len - kernel + (kernel - stride)) / stride + 1), clamped at 0 */
size_t vo_conv_out_len(size_t length, size_t kernel, size_t stride) {
    const size_t padding_total = kernel - stride;
    const float n_frames = ((float)length - (float)kernel + (float)padding_total) / (float)stride + 1.0f;
    const float c = ceilf(n_frames);
    return c > 0.0f ? (size_t)c : 0;
}

/* conv.rs:28-73 causal_conv1d_colmajor */
void vo_causal_conv1d_colmajor(float* output, const float* input, const float* weight, const float* bias,
                               size_t cin, size_t cout, size_t length, size_t kernel, size_t stride) {
    const size_t out_len = vo_conv_out_len(length, kernel, stride);
    if (out_len == 0) return;
    const long long left_pad = (long long)(kernel - stride);
    for (size_t oc = 0; oc < cout; ++oc) {
        const float b = bias ? bias[oc] : 0.0f;
        for (size_t ol = 0; ol < out_len; ++ol) {
            float sum = b;
            const long long base = (long long)(ol * stride) - left_pad;
            for (size_t ic = 0; ic < cin; ++ic) {
                const float* in_row = input + ic * length;
                const size_t wb = oc * cin * kernel + ic * kernel;
                for (size_t k = 0; k < kernel; ++k) {
                    const long long il = base + (long long)k;
                    if (il >= 0 && (size_t)il < length) sum += in_row[il] * weight[wb + k];
                }
            }
            output[oc * out_len + ol] = sum;
        }
    }
}

struct vo_conv_stem {
    size_t mel_bins, dim;
    float* mel_tail;       /* [mel_bins, 2] */
    float* conv0_tail;     /* [dim, 2] */
    float* conv0_residual; /* [dim] */
    size_t residual_count;
    int initialized;
};

vo_conv_stem* vo_conv_stem_new(size_t mel_bins, size_t dim) {
    vo_conv_stem* s = (vo_conv_stem*)calloc(1, sizeof(vo_conv_stem));
    s->mel_bins = mel_bins;
    s->dim = dim;
    s->mel_tail = (float*)calloc(mel_bins * 2, sizeof(float));
    s->conv0_tail = (float*)calloc(dim * 2, sizeof(float));
    s->conv0_residual = (float*)calloc(dim, sizeof(float));
    return s;
}

void vo_conv_stem_free(vo_conv_stem* s) {
    if (!s) return;
    free(s->mel_tail);
    free(s->conv0_tail);
    free(s->conv0_residual);
    free(s);
}

/* conv.rs:336-347 update_mel_tail */
static void update_mel_tail(vo_conv_stem* s, const float* mel_new, size_t n_new) {
    const size_t ts = n_new > 2 ? n_new - 2 : 0, tc = n_new < 2 ? n_new : 2;
    memset(s->mel_tail, 0, s->mel_bins * 2 * sizeof(float));
    for (size_t f = 0; f < tc; ++f)
        for (size_t m = 0; m < s->mel_bins; ++m) s->mel_tail[m * 2 + (2 - tc + f)] = mel_new[(ts + f) * s->mel_bins + m];
}

/* conv.rs:163-334 ConvStemState::process.  out must hold (n_new_mel / 2 + 2) * dim
 * floats; returns the number of new positions (rows of out, row-major [n, dim]). */
size_t vo_conv_stem_process(vo_conv_stem* s, const float* w0, const float* b0, const float* w1, const float* b1,
                            const float* mel_new, size_t n_new, float* out) {
    if (n_new == 0) return 0;
    const size_t M = s->mel_bins, D = s->dim;
    const int is_first = !s->initialized;
    float* conv0_new;
    size_t conv0_len;
    if (is_first) {
        float* conv_in = (float*)malloc(M * n_new * sizeof(float));
        for (size_t t = 0; t < n_new; ++t)
            for (size_t c = 0; c < M; ++c) conv_in[c * n_new + t] = mel_new[t * M + c];
        conv0_new = (float*)malloc(D * n_new * sizeof(float));
        vo_causal_conv1d_colmajor(conv0_new, conv_in, w0, b0, M, D, n_new, 3, 1);
        vo_gelu_inplace(conv0_new, D * n_new);
        update_mel_tail(s, mel_new, n_new);
        s->initialized = 1;
        conv0_len = n_new;
        free(conv_in);
    } else {
        const size_t pl = 2 + n_new;
        float* conv_in = (float*)calloc(M * pl, sizeof(float));
        for (size_t m = 0; m < M; ++m) {
            conv_in[m * pl] = s->mel_tail[m * 2];
            conv_in[m * pl + 1] = s->mel_tail[m * 2 + 1];
            for (size_t f = 0; f < n_new; ++f) conv_in[m * pl + 2 + f] = mel_new[f * M + m];
        }
        float* full = (float*)malloc(D * pl * sizeof(float));
        vo_causal_conv1d_colmajor(full, conv_in, w0, b0, M, D, pl, 3, 1);
        vo_gelu_inplace(full, D * pl);
        conv0_new = (float*)malloc(D * n_new * sizeof(float));
        for (size_t d = 0; d < D; ++d) memcpy(conv0_new + d * n_new, full + d * pl + 2, n_new * sizeof(float));
        update_mel_tail(s, mel_new, n_new);
        conv0_len = n_new;
        free(conv_in);
        free(full);
    }
    /* stride alignment for conv1 (conv.rs:227-272) */
    const size_t prev_res = s->residual_count, total = prev_res + conv0_len;
    const size_t new_res = total & 1, from_new = conv0_len - new_res, feed_total = prev_res + from_new;
    if (feed_total == 0) {
        if (new_res == 1)
            for (size_t d = 0; d < D; ++d) s->conv0_residual[d] = conv0_new[d * conv0_len + conv0_len - 1];
        s->residual_count = new_res;
        free(conv0_new);
        return 0;
    }
    float* feed = (float*)calloc(D * feed_total, sizeof(float));
    size_t fpos = 0;
    if (prev_res == 1) {
        for (size_t d = 0; d < D; ++d) feed[d * feed_total] = s->conv0_residual[d];
        fpos = 1;
    }
    for (size_t d = 0; d < D; ++d) memcpy(feed + d * feed_total + fpos, conv0_new + d * conv0_len, from_new * sizeof(float));
    if (new_res == 1)
        for (size_t d = 0; d < D; ++d) s->conv0_residual[d] = conv0_new[d * conv0_len + conv0_len - 1];
    s->residual_count = new_res;
    free(conv0_new);
    /* conv1 (conv.rs:274-318) */
    float* c1_in;
    size_t c1_len, discard;
    if (is_first) {
        for (size_t d = 0; d < D; ++d) {
            s->conv0_tail[d * 2] = feed[d * feed_total + feed_total - 2];
            s->conv0_tail[d * 2 + 1] = feed[d * feed_total + feed_total - 1];
        }
        c1_in = feed;
        c1_len = feed_total;
        discard = 0;
    } else {
        c1_len = 2 + feed_total;
        c1_in = (float*)calloc(D * c1_len, sizeof(float));
        for (size_t d = 0; d < D; ++d) {
            c1_in[d * c1_len] = s->conv0_tail[d * 2];
            c1_in[d * c1_len + 1] = s->conv0_tail[d * 2 + 1];
            memcpy(c1_in + d * c1_len + 2, feed + d * feed_total, feed_total * sizeof(float));
        }
        for (size_t d = 0; d < D; ++d) {
            s->conv0_tail[d * 2] = feed[d * feed_total + feed_total - 2];
            s->conv0_tail[d * 2 + 1] = feed[d * feed_total + feed_total - 1];
        }
        discard = 1;
        free(feed);
    }
    const size_t c1_out_len = c1_len / 2;
    float* c1_out = (float*)malloc(D * c1_out_len * sizeof(float));
    vo_causal_conv1d_colmajor(c1_out, c1_in, w1, b1, D, D, c1_len, 3, 2);
    vo_gelu_inplace(c1_out, D * c1_out_len);
    free(c1_in);
    const size_t n_out = c1_out_len > discard ? c1_out_len - discard : 0;
    for (size_t si = 0; si < n_out; ++si)
        for (size_t d = 0; d < D; ++d) out[si * D + d] = c1_out[d * c1_out_len + discard + si];
    free(c1_out);
    return n_out;
}
