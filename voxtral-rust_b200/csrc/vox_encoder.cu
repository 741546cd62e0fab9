// vox_encoder.cu -- the encoder front end on the GPU: the incremental log-mel
// spectrogram (MelCtx, crates/voxtral/src/mel.rs:114-272) and the causal conv
// stem (ConvStemState, crates/voxtral/src/conv.rs:134-347), the producers of
// the adapter rows the streaming decoder consumes.
//
// Log-mel: one CTA per frame.  The frame's 400 windowed samples go to shared
// memory; thread k < 201 forms the DFT bin's real and imaginary sums over
// n = 0..399 in the reference's order, reading the cosine and sine tables
// transposed ([n][k], so a warp's loads are contiguous); thread b < 128 forms
// the mel band's sum over k in order, then the log10 clamp.  Products and
// sums are separately rounded (no FMA), so the power spectrum and the band
// sums equal the reference's bit for bit; only log10f may differ in the last
// place.  The tables are computed once on the host with the same f32 formulas
// as mel.rs:42-106.
//
// Conv stem: the reference's chunk bookkeeping (mel tail, conv0 residual for
// the stride-2 alignment, conv0 tail) runs on the host over device buffers.
// Each causal convolution of the stem is two kernels: the sum over input
// channels split into ranges across CTAs (a chunk has only a few output
// positions, so the split is what spreads the 19.7 MB weight read of conv1
// over the SMs), then a fixed-order reduction of the ranges with the bias and
// the tanh-approximated GELU (conv.rs:11-19).  Weights are transposed to
// [ic][k][oc] at upload so a warp's weight loads are contiguous.  The
// op-level call (vox_causal_conv1d_gelu) keeps the reference's own order: one
// thread per output channel sums bias + in[ic][t] * w[oc][ic][k] over ic then
// k as conv.rs:60-68 does, bit-identical; tanhf may differ in the last place.
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <vector>

#include "../../include/vox_decoder.h"
#include "vox_device.cuh"
#include "vox_host.h"

using namespace vox;

namespace {

constexpr int kSr = 16000, kMelBins = 128, kHop = 160, kWin = 400, kNfft = 400, kNfreq = kNfft / 2 + 1;
constexpr float kLogMelMax = 1.5f;
constexpr float kPi = 3.14159265358979323846f;  // std::f32::consts::PI

// ---- host tables (mel.rs:15-106) ----
float hertz_to_mel(float freq) {
    const float min_log_hz = 1000.0f, min_log_mel = 15.0f, logstep = 0.06875178f;
    float mels = 3.0f * freq / 200.0f;
    if (freq >= min_log_hz) mels = min_log_mel + std::log(freq / min_log_hz) * logstep;
    return mels;
}
float mel_to_hertz(float mels) {
    const float min_log_hz = 1000.0f, min_log_mel = 15.0f, logstep = 0.06875178f;
    float freq = 200.0f * mels / 3.0f;
    if (mels >= min_log_mel) freq = min_log_hz * std::exp(logstep * (mels - min_log_mel));
    return freq;
}
void build_tables(std::vector<float>& filt_t, std::vector<float>& cos_t, std::vector<float>& sin_t,
                  std::vector<float>& window) {
    float fft_freqs[kNfreq], ff[kMelBins + 2], fd[kMelBins + 1];
    for (int f = 0; f < kNfreq; ++f) fft_freqs[f] = (float)f * (float)kSr / (float)kNfft;
    const float mel_min = hertz_to_mel(0.0f), mel_max = hertz_to_mel((float)kSr / 2.0f);
    for (int i = 0; i < kMelBins + 2; ++i)
        ff[i] = mel_to_hertz(mel_min + (mel_max - mel_min) * (float)i / (float)(kMelBins + 1));
    for (int i = 0; i < kMelBins + 1; ++i) {
        fd[i] = ff[i + 1] - ff[i];
        if (fd[i] == 0.0f) fd[i] = 1e-6f;
    }
    filt_t.assign((size_t)kNfreq * kMelBins, 0.0f);  // [k][m]
    for (int m = 0; m < kMelBins; ++m) {
        const float enorm = 2.0f / (ff[m + 2] - ff[m]);
        for (int f = 0; f < kNfreq; ++f) {
            const float down = (fft_freqs[f] - ff[m]) / fd[m];
            const float up = (ff[m + 2] - fft_freqs[f]) / fd[m + 1];
            float v = down < up ? down : up;
            if (v < 0.0f) v = 0.0f;
            filt_t[(size_t)f * kMelBins + m] = v * enorm;
        }
    }
    cos_t.assign((size_t)kNfft * kNfreq, 0.0f);  // [n][k]
    sin_t.assign((size_t)kNfft * kNfreq, 0.0f);
    for (int k = 0; k < kNfreq; ++k)
        for (int n = 0; n < kNfft; ++n) {
            const float angle = 2.0f * kPi * (float)k * (float)n / (float)kNfft;
            cos_t[(size_t)n * kNfreq + k] = std::cos(angle);
            sin_t[(size_t)n * kNfreq + k] = std::sin(angle);
        }
    window.assign(kWin, 0.0f);
    for (int i = 0; i < kWin; ++i) window[i] = 0.5f * (1.0f - std::cos(2.0f * kPi * (float)i / (float)kWin));
}

// ---- kernels ----
// samples: the window starting at frame f0's first sample; frame j starts at j * 160.
__global__ void __launch_bounds__(256) log_mel_kernel(const float* __restrict__ samples,
                                                      const float* __restrict__ window,
                                                      const float* __restrict__ cos_t,
                                                      const float* __restrict__ sin_t,
                                                      const float* __restrict__ filt_t, float* __restrict__ mel_out) {
    __shared__ float wnd[kNfft];
    __shared__ float power[kNfreq];
    const int j = blockIdx.x, tid = threadIdx.x;
    const float* x = samples + (size_t)j * kHop;
    for (int i = tid; i < kNfft; i += blockDim.x) wnd[i] = __fmul_rn(x[i], window[i]);
    __syncthreads();
    if (tid < kNfreq) {
        float re = 0.0f, im = 0.0f;
#pragma unroll 16  // table loads run ahead; the sums keep their order
        for (int n = 0; n < kNfft; ++n) {
            const float w = wnd[n];
            re = __fadd_rn(re, __fmul_rn(w, cos_t[n * kNfreq + tid]));
            im = __fadd_rn(im, __fmul_rn(w, sin_t[n * kNfreq + tid]));
        }
        power[tid] = __fadd_rn(__fmul_rn(re, re), __fmul_rn(im, im));
    }
    __syncthreads();
    if (tid < kMelBins) {
        float sum = 0.0f;
#pragma unroll 8
        for (int k = 0; k < kNfreq; ++k) sum = __fadd_rn(sum, __fmul_rn(filt_t[k * kMelBins + tid], power[k]));
        if (sum < 1e-10f) sum = 1e-10f;
        float val = log10f(sum);
        const float min_val = kLogMelMax - 8.0f;
        if (val < min_val) val = min_val;
        mel_out[(size_t)j * kMelBins + tid] = __fdiv_rn(__fadd_rn(val, 4.0f), 4.0f);
    }
}

constexpr int kConvPT = 4;  // output positions per thread

// out[oc][ol] (col-major [cout, out_len]) = gelu(bias[oc] + sum_ic sum_k in[ic][ol*stride - (3-stride) + k] * w).
// wt: weights transposed to [cin][3][cout].
__global__ void __launch_bounds__(128) causal_conv3_gelu_kernel(const float* __restrict__ in, int length,
                                                                const float* __restrict__ wt,
                                                                const float* __restrict__ bias, int cin, int cout,
                                                                int stride, int out_len, float* __restrict__ out,
                                                                int gelu) {
    const int oc = blockIdx.x * blockDim.x + threadIdx.x;
    const int ol0 = blockIdx.y * kConvPT;
    if (oc >= cout) return;
    const int left_pad = 3 - stride;
    float sum[kConvPT];
    const float b = bias ? bias[oc] : 0.0f;
#pragma unroll
    for (int p = 0; p < kConvPT; ++p) sum[p] = b;
    for (int ic = 0; ic < cin; ++ic) {
        const float* row = in + (size_t)ic * length;
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const float w = wt[((size_t)ic * 3 + k) * cout + oc];
#pragma unroll
            for (int p = 0; p < kConvPT; ++p) {
                const int il = (ol0 + p) * stride - left_pad + k;
                if (ol0 + p < out_len && il >= 0 && il < length) sum[p] = __fadd_rn(sum[p], __fmul_rn(__ldg(row + il), w));
            }
        }
    }
#pragma unroll
    for (int p = 0; p < kConvPT; ++p) {
        if (ol0 + p >= out_len) break;
        float v = sum[p];
        if (gelu) {  // conv.rs:11-19
            const float x3 = __fmul_rn(__fmul_rn(v, v), v);
            const float inner = __fmul_rn(0.7978846f, __fadd_rn(v, __fmul_rn(0.044715f, x3)));
            v = __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(inner)));
        }
        out[(size_t)oc * out_len + ol0 + p] = v;
    }
}

// The conv stem's form of the same convolution: the sum over input channels is
// split into `gridDim.y` contiguous ranges so that a streaming chunk (a few
// output positions) still spreads the weight read over every SM; part[s] holds
// split s's sums [cout, out_len] (bias not included).  conv_reduce_gelu_kernel
// adds the splits in order, then the bias, then the GELU: deterministic, and
// equal to the sequential sum within float rounding.
__global__ void __launch_bounds__(128) conv3_split_kernel(const float* __restrict__ in, int length,
                                                          const float* __restrict__ wt, int cin, int cout, int stride,
                                                          int out_len, int splits, float* __restrict__ part) {
    const int oc = blockIdx.x * blockDim.x + threadIdx.x;
    const int s = blockIdx.y;
    const int ol0 = blockIdx.z * kConvPT;
    if (oc >= cout) return;
    const int ic0 = (int)((long long)cin * s / splits), ic1 = (int)((long long)cin * (s + 1) / splits);
    const int left_pad = 3 - stride;
    float sum[kConvPT];
#pragma unroll
    for (int p = 0; p < kConvPT; ++p) sum[p] = 0.0f;
    int ic = ic0;
    for (; ic + 4 <= ic1; ic += 4) {  // four channels' weights in flight per thread
        float w[4][3];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int k = 0; k < 3; ++k) w[u][k] = __ldg(wt + ((size_t)(ic + u) * 3 + k) * cout + oc);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float* row = in + (size_t)(ic + u) * length;
#pragma unroll
            for (int k = 0; k < 3; ++k)
#pragma unroll
                for (int p = 0; p < kConvPT; ++p) {
                    const int il = (ol0 + p) * stride - left_pad + k;
                    if (ol0 + p < out_len && il >= 0 && il < length) sum[p] = fmaf(__ldg(row + il), w[u][k], sum[p]);
                }
        }
    }
    for (; ic < ic1; ++ic) {
        const float* row = in + (size_t)ic * length;
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const float w = __ldg(wt + ((size_t)ic * 3 + k) * cout + oc);
#pragma unroll
            for (int p = 0; p < kConvPT; ++p) {
                const int il = (ol0 + p) * stride - left_pad + k;
                if (ol0 + p < out_len && il >= 0 && il < length) sum[p] = fmaf(__ldg(row + il), w, sum[p]);
            }
        }
    }
    float* dst = part + ((size_t)s * cout + oc) * out_len;
#pragma unroll
    for (int p = 0; p < kConvPT; ++p)
        if (ol0 + p < out_len) dst[ol0 + p] = sum[p];
}

// out[oc][t] = gelu(bias[oc] + sum over splits of part[s][oc][t]), splits in order.
__global__ void conv_reduce_gelu_kernel(const float* __restrict__ part, int splits, const float* __restrict__ bias,
                                        int cout, int out_len, float* __restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long n = (long long)cout * out_len;
    if (i >= n) return;
    float v = part[i];
    for (int s = 1; s < splits; ++s) v += part[(size_t)s * n + i];
    v = __fadd_rn(bias[i / out_len], v);
    const float x3 = __fmul_rn(__fmul_rn(v, v), v);
    const float inner = __fmul_rn(0.7978846f, __fadd_rn(v, __fmul_rn(0.044715f, x3)));
    out[i] = __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(inner)));
}

// dst[d * dst_len + dst_off + j] = src[d * src_len + src_off + j] for j < n, d < rows.
__global__ void copy_cols_kernel(float* __restrict__ dst, int dst_len, int dst_off, const float* __restrict__ src,
                                 int src_len, int src_off, int n, int rows) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)rows * n) return;
    const int d = (int)(i / n), j = (int)(i % n);
    dst[(size_t)d * dst_len + dst_off + j] = src[(size_t)d * src_len + src_off + j];
}

// Col-major [rows, len] columns col0.. -> row-major [n, rows].
__global__ void cols_to_rows_kernel(float* __restrict__ dst, const float* __restrict__ src, int len, int col0, int n,
                                    int rows) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)rows * n) return;
    const int t = (int)(i / rows), d = (int)(i % rows);
    dst[i] = src[(size_t)d * len + col0 + t];
}

size_t conv_out_len(size_t length, size_t kernel, size_t stride) {  // conv.rs:35-37, in f32 as the reference
    const size_t padding_total = kernel - stride;
    const float n_frames = ((float)length - (float)kernel + (float)padding_total) / (float)stride + 1.0f;
    const float c = std::ceil(n_frames);
    return c > 0.0f ? (size_t)c : 0;
}

#define ENC_CUDA(expr)                                                                              \
    do {                                                                                            \
        cudaError_t e_ = (expr);                                                                    \
        if (e_ != cudaSuccess)                                                                      \
            return report_errorf(e_ == cudaErrorMemoryAllocation ? VOX_ERR_OOM : VOX_ERR_CUDA,     \
                                 "%s failed: %s", #expr, cudaGetErrorString(e_));                  \
    } while (0)
#define ENC_TRY(expr)                  \
    do {                               \
        int rc_ = (expr);              \
        if (rc_ != VOX_OK) return rc_; \
    } while (0)

// A growable device buffer of floats.
struct DBuf {
    float* p = nullptr;
    size_t cap = 0;
    int reserve(size_t n, cudaStream_t s) {
        if (n <= cap) return VOX_OK;
        size_t c = cap ? cap : 4096;
        while (c < n) c *= 2;
        float* q = nullptr;
        ENC_CUDA(cudaMalloc(&q, c * sizeof(float)));
        if (p) {
            ENC_CUDA(cudaMemcpyAsync(q, p, cap * sizeof(float), cudaMemcpyDeviceToDevice, s));
            ENC_CUDA(cudaStreamSynchronize(s));
            cudaFree(p);
        }
        p = q;
        cap = c;
        return VOX_OK;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
    }
};

// Split count of the conv stem's convolutions: enough CTAs for two per SM,
// at least 8 input channels per split.
int conv_splits(size_t cin, size_t cout, size_t out_len, int num_sms) {
    const long long base = (long long)((cout + 127) / 128) * (long long)((out_len + kConvPT - 1) / kConvPT);
    long long want = (2LL * num_sms + base - 1) / base;
    const long long most = (long long)(cin / 8) > 0 ? (long long)(cin / 8) : 1;
    if (want > most) want = most;
    if (want > 64) want = 64;
    return want < 1 ? 1 : (int)want;
}

// conv + bias + GELU into out [cout, out_len]; part: room for splits x cout x out_len floats.
int launch_conv(const float* in, size_t length, const float* wt, const float* bias, size_t cin, size_t cout,
                size_t stride, size_t out_len, float* out, float* part, int splits, cudaStream_t s) {
    if (out_len == 0) return VOX_OK;
    dim3 grid((unsigned)((cout + 127) / 128), (unsigned)splits, (unsigned)((out_len + kConvPT - 1) / kConvPT));
    conv3_split_kernel<<<grid, 128, 0, s>>>(in, (int)length, wt, (int)cin, (int)cout, (int)stride, (int)out_len,
                                            splits, part);
    ENC_CUDA(cudaGetLastError());
    const long long n = (long long)cout * (long long)out_len;
    conv_reduce_gelu_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(part, splits, bias, (int)cout, (int)out_len,
                                                                        out);
    ENC_CUDA(cudaGetLastError());
    return VOX_OK;
}

int launch_copy_cols(float* dst, size_t dst_len, size_t dst_off, const float* src, size_t src_len, size_t src_off,
                     size_t n, size_t rows, cudaStream_t s) {
    if (n == 0 || rows == 0) return VOX_OK;
    const long long total = (long long)rows * (long long)n;
    copy_cols_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(dst, (int)dst_len, (int)dst_off, src,
                                                                     (int)src_len, (int)src_off, (int)n, (int)rows);
    ENC_CUDA(cudaGetLastError());
    return VOX_OK;
}

}  // namespace

// ---- MelCtx ---------------------------------------------------------------------

struct vox_mel {
    int dev = 0;
    cudaStream_t stream = nullptr;
    float *window = nullptr, *cos_t = nullptr, *sin_t = nullptr, *filt_t = nullptr;
    std::vector<float> samples;  // host history from sample index `base` on
    size_t base = 0;             // absolute index of samples[0]
    size_t n_samples = 0;        // absolute sample count (the reference's samples.len())
    size_t left_pad = 0;
    size_t n_frames = 0;
    bool finished = false;
    DBuf d_samples, d_mel;       // frame window upload; mel rows [frames, 128]
    uint64_t launches = 0;
};

namespace {

// mel.rs:210-271: every frame whose 400 samples are present, on the GPU.
int mel_compute_available(vox_mel* m, size_t* new_frames) {
    *new_frames = 0;
    if (m->n_samples < kWin) return VOX_OK;
    const size_t total = (m->n_samples - kWin) / kHop + 1;  // frames t with t*160 + 400 <= len
    if (total <= m->n_frames) return VOX_OK;
    const size_t f0 = m->n_frames, nf = total - f0;
    const size_t s0 = f0 * kHop, s1 = (total - 1) * kHop + kWin;
    ENC_TRY(m->d_samples.reserve(s1 - s0, m->stream));
    ENC_TRY(m->d_mel.reserve(total * kMelBins, m->stream));
    ENC_CUDA(cudaMemcpyAsync(m->d_samples.p, m->samples.data() + (s0 - m->base), (s1 - s0) * sizeof(float),
                             cudaMemcpyHostToDevice, m->stream));
    log_mel_kernel<<<(unsigned)nf, 256, 0, m->stream>>>(m->d_samples.p, m->window, m->cos_t, m->sin_t, m->filt_t,
                                                        m->d_mel.p + f0 * kMelBins);
    ENC_CUDA(cudaGetLastError());
    ++m->launches;
    ENC_CUDA(cudaStreamSynchronize(m->stream));  // the host window is reused by the next feed
    m->n_frames = total;
    *new_frames = nf;
    // keep what later frames or the end-of-stream reflection can still read
    size_t keep_from = m->n_frames * kHop;
    if (m->n_samples >= 202 && m->n_samples - 202 < keep_from) keep_from = m->n_samples - 202;
    if (keep_from > m->base) {
        m->samples.erase(m->samples.begin(), m->samples.begin() + (keep_from - m->base));
        m->base = keep_from;
    }
    return VOX_OK;
}

}  // namespace

extern "C" int vox_mel_create(int device, size_t left_pad_samples, vox_mel** out) {
    if (!out) return report_errorf(VOX_ERR_INVALID_ARG, "null output");
    *out = nullptr;
    ENC_CUDA(cudaSetDevice(device));
    auto* m = new vox_mel();
    m->dev = device;
    std::vector<float> filt, cs, sn, win;
    build_tables(filt, cs, sn, win);
    auto fail = [&](int rc) {
        vox_mel_destroy(m);
        return rc;
    };
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&m->window, win.size() * 4) != cudaSuccess || cudaMalloc(&m->cos_t, cs.size() * 4) != cudaSuccess ||
        cudaMalloc(&m->sin_t, sn.size() * 4) != cudaSuccess || cudaMalloc(&m->filt_t, filt.size() * 4) != cudaSuccess)
        return fail(report_errorf(VOX_ERR_OOM, "cannot allocate the log-mel tables"));
    if (cudaMemcpy(m->window, win.data(), win.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(m->cos_t, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(m->sin_t, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(m->filt_t, filt.data(), filt.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return fail(report_errorf(VOX_ERR_CUDA, "cannot upload the log-mel tables"));
    m->left_pad = kNfft / 2 + left_pad_samples;  // mel.rs:130-151
    m->samples.assign(m->left_pad, 0.0f);
    m->n_samples = m->left_pad;
    *out = m;
    return VOX_OK;
}

extern "C" void vox_mel_destroy(vox_mel* m) {
    if (!m) return;
    cudaSetDevice(m->dev);
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (float* p : {m->window, m->cos_t, m->sin_t, m->filt_t})
        if (p) cudaFree(p);
    m->d_samples.release();
    m->d_mel.release();
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

extern "C" size_t vox_mel_left_pad_samples(const vox_mel* m) { return m ? m->left_pad : 0; }

extern "C" int vox_mel_feed(vox_mel* m, const float* x, size_t n, size_t* new_frames) {
    if (!m || (!x && n)) return report_errorf(VOX_ERR_INVALID_ARG, "null mel context or samples");
    if (new_frames) *new_frames = 0;
    if (n == 0) return VOX_OK;  // mel.rs:160-162
    ENC_CUDA(cudaSetDevice(m->dev));
    m->samples.insert(m->samples.end(), x, x + n);
    m->n_samples += n;
    size_t nf = 0;
    ENC_TRY(mel_compute_available(m, &nf));
    if (new_frames) *new_frames = nf;
    return VOX_OK;
}

extern "C" int vox_mel_finish(vox_mel* m, size_t right_pad_samples) {
    if (!m) return report_errorf(VOX_ERR_INVALID_ARG, "null mel context");
    if (m->finished) return VOX_OK;  // mel.rs:170-173
    ENC_CUDA(cudaSetDevice(m->dev));
    m->samples.insert(m->samples.end(), right_pad_samples, 0.0f);
    m->n_samples += right_pad_samples;
    const size_t real_end = m->n_samples > right_pad_samples ? m->n_samples - right_pad_samples : 0;
    for (size_t i = 0; i < kNfft / 2; ++i) {  // 200-sample reflection (mel.rs:184-191)
        const long long src = (long long)real_end - 2 - (long long)i;
        float v = 0.0f;
        if (src >= 0 && (size_t)src < m->n_samples && (size_t)src >= m->base) v = m->samples[(size_t)src - m->base];
        m->samples.push_back(v);
        ++m->n_samples;
    }
    size_t nf = 0;
    ENC_TRY(mel_compute_available(m, &nf));
    if (m->n_frames > 0) --m->n_frames;  // mel.rs:195-199: drop the last frame
    m->finished = true;
    return VOX_OK;
}

extern "C" size_t vox_mel_frames(const vox_mel* m) { return m ? m->n_frames : 0; }

extern "C" int vox_mel_data(vox_mel* m, size_t first_frame, size_t n_frames, float* out) {
    if (!m || (!out && n_frames)) return report_errorf(VOX_ERR_INVALID_ARG, "null mel context or output");
    if (first_frame + n_frames > m->n_frames)
        return report_errorf(VOX_ERR_INVALID_ARG, "frames [%zu, %zu) beyond the %zu computed", first_frame,
                             first_frame + n_frames, m->n_frames);
    if (n_frames == 0) return VOX_OK;
    ENC_CUDA(cudaSetDevice(m->dev));
    ENC_CUDA(cudaMemcpyAsync(out, m->d_mel.p + first_frame * kMelBins, n_frames * kMelBins * sizeof(float),
                             cudaMemcpyDeviceToHost, m->stream));
    ENC_CUDA(cudaStreamSynchronize(m->stream));
    return VOX_OK;
}

// ---- ConvStemState ------------------------------------------------------------------

struct vox_conv_stem {
    int dev = 0;
    cudaStream_t stream = nullptr;
    size_t mel_bins = 0, dim = 0;
    float *w0t = nullptr, *b0 = nullptr, *w1t = nullptr, *b1 = nullptr;  // weights [cin][3][dim]
    std::vector<float> mel_tail;   // [mel_bins, 2] col-major (host: it comes from the host input)
    float* conv0_tail = nullptr;   // [dim, 2] device
    float* residual = nullptr;     // [dim] device
    size_t residual_count = 0;
    bool initialized = false;
    DBuf conv_in, conv0, feed, c1_in, c1_out, rows, part;
    std::vector<float> h_in;
    int num_sms = 148;
    uint64_t launches = 0;
};

namespace {

// [cout, cin, 3] -> [cin][3][cout]
std::vector<float> transpose_w(const float* w, size_t cout, size_t cin) {
    std::vector<float> t(cout * cin * 3);
    for (size_t oc = 0; oc < cout; ++oc)
        for (size_t ic = 0; ic < cin; ++ic)
            for (size_t k = 0; k < 3; ++k) t[(ic * 3 + k) * cout + oc] = w[(oc * cin + ic) * 3 + k];
    return t;
}

}  // namespace

extern "C" int vox_conv_stem_create(int device, size_t mel_bins, size_t dim, const float* conv0_weight,
                                    const float* conv0_bias, const float* conv1_weight, const float* conv1_bias,
                                    vox_conv_stem** out) {
    if (!out || !conv0_weight || !conv0_bias || !conv1_weight || !conv1_bias)
        return report_errorf(VOX_ERR_INVALID_ARG, "null weights or output");
    *out = nullptr;
    if (mel_bins == 0 || dim == 0 || mel_bins > 65536 || dim > 65536)
        return report_errorf(VOX_ERR_INVALID_ARG, "mel_bins and dim must be in [1, 65536]");
    ENC_CUDA(cudaSetDevice(device));
    auto* s = new vox_conv_stem();
    s->dev = device;
    if (cudaDeviceGetAttribute(&s->num_sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || s->num_sms <= 0)
        s->num_sms = 148;
    s->mel_bins = mel_bins;
    s->dim = dim;
    s->mel_tail.assign(mel_bins * 2, 0.0f);
    const auto w0 = transpose_w(conv0_weight, dim, mel_bins), w1 = transpose_w(conv1_weight, dim, dim);
    auto fail = [&](int rc) {
        vox_conv_stem_destroy(s);
        return rc;
    };
    if (cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&s->w0t, w0.size() * 4) != cudaSuccess || cudaMalloc(&s->w1t, w1.size() * 4) != cudaSuccess ||
        cudaMalloc(&s->b0, dim * 4) != cudaSuccess || cudaMalloc(&s->b1, dim * 4) != cudaSuccess ||
        cudaMalloc(&s->conv0_tail, dim * 2 * 4) != cudaSuccess || cudaMalloc(&s->residual, dim * 4) != cudaSuccess)
        return fail(report_errorf(VOX_ERR_OOM, "cannot allocate the conv stem"));
    if (cudaMemcpy(s->w0t, w0.data(), w0.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(s->w1t, w1.data(), w1.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(s->b0, conv0_bias, dim * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(s->b1, conv1_bias, dim * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(s->conv0_tail, 0, dim * 2 * 4) != cudaSuccess || cudaMemset(s->residual, 0, dim * 4) != cudaSuccess)
        return fail(report_errorf(VOX_ERR_CUDA, "cannot upload the conv stem weights"));
    *out = s;
    return VOX_OK;
}

extern "C" void vox_conv_stem_destroy(vox_conv_stem* s) {
    if (!s) return;
    cudaSetDevice(s->dev);
    if (s->stream) cudaStreamSynchronize(s->stream);
    for (float* p : {s->w0t, s->b0, s->w1t, s->b1, s->conv0_tail, s->residual})
        if (p) cudaFree(p);
    for (DBuf* b : {&s->conv_in, &s->conv0, &s->feed, &s->c1_in, &s->c1_out, &s->rows, &s->part}) b->release();
    if (s->stream) cudaStreamDestroy(s->stream);
    delete s;
}

// ConvStemState::process (conv.rs:163-334).  mel_new: host [n_new, mel_bins];
// out: host [*n_out, dim] with room for (n_new / 2 + 1) rows.
extern "C" int vox_conv_stem_process(vox_conv_stem* s, const float* mel_new, size_t n_new, float* out,
                                     size_t out_cap_rows, size_t* n_out) {
    if (!s || !n_out || (!mel_new && n_new)) return report_errorf(VOX_ERR_INVALID_ARG, "null argument");
    *n_out = 0;
    if (n_new == 0) return VOX_OK;
    if (n_new > (1u << 24)) return report_errorf(VOX_ERR_INVALID_ARG, "too many mel frames in one call");
    ENC_CUDA(cudaSetDevice(s->dev));
    const size_t M = s->mel_bins, D = s->dim;
    cudaStream_t st = s->stream;
    const bool is_first = !s->initialized;
    // conv0 input, col-major [M, L]: the 2 tail frames (after the first call), then the new frames
    const size_t L = is_first ? n_new : 2 + n_new, pre = is_first ? 0 : 2;
    s->h_in.assign(M * L, 0.0f);
    for (size_t m = 0; m < M; ++m) {
        if (!is_first) {
            s->h_in[m * L] = s->mel_tail[m * 2];
            s->h_in[m * L + 1] = s->mel_tail[m * 2 + 1];
        }
        for (size_t f = 0; f < n_new; ++f) s->h_in[m * L + pre + f] = mel_new[f * M + m];
    }
    {  // update_mel_tail (conv.rs:336-347)
        const size_t ts = n_new > 2 ? n_new - 2 : 0, tc = n_new < 2 ? n_new : 2;
        std::fill(s->mel_tail.begin(), s->mel_tail.end(), 0.0f);
        for (size_t f = 0; f < tc; ++f)
            for (size_t m = 0; m < M; ++m) s->mel_tail[m * 2 + (2 - tc + f)] = mel_new[(ts + f) * M + m];
    }
    s->initialized = true;
    ENC_TRY(s->conv_in.reserve(M * L, st));
    ENC_TRY(s->conv0.reserve(D * L, st));
    ENC_CUDA(cudaMemcpyAsync(s->conv_in.p, s->h_in.data(), M * L * 4, cudaMemcpyHostToDevice, st));
    {  // stride 1: out_len = L
        const int sp = conv_splits(M, D, L, s->num_sms);
        ENC_TRY(s->part.reserve((size_t)sp * D * L, st));
        ENC_TRY(launch_conv(s->conv_in.p, L, s->w0t, s->b0, M, D, 1, L, s->conv0.p, s->part.p, sp, st));
        s->launches += 2;
    }
    const size_t c0_len = n_new;  // new conv0 columns start at column `pre`

    // stride alignment for conv1 (conv.rs:227-272)
    const size_t prev_res = s->residual_count, total = prev_res + c0_len;
    const size_t new_res = total & 1, from_new = c0_len - new_res, feed_total = prev_res + from_new;
    if (feed_total == 0) {
        if (new_res == 1) ENC_TRY(launch_copy_cols(s->residual, 1, 0, s->conv0.p, L, pre + c0_len - 1, 1, D, st));
        s->residual_count = new_res;
        ENC_CUDA(cudaStreamSynchronize(st));
        return VOX_OK;
    }
    // conv1 input, col-major [D, c1_len]: (tail,) residual, new conv0 columns
    const size_t c1_pre = is_first ? 0 : 2, c1_len = c1_pre + feed_total;
    ENC_TRY(s->c1_in.reserve(D * c1_len, st));
    if (!is_first) ENC_TRY(launch_copy_cols(s->c1_in.p, c1_len, 0, s->conv0_tail, 2, 0, 2, D, st));
    if (prev_res == 1) ENC_TRY(launch_copy_cols(s->c1_in.p, c1_len, c1_pre, s->residual, 1, 0, 1, D, st));
    ENC_TRY(launch_copy_cols(s->c1_in.p, c1_len, c1_pre + prev_res, s->conv0.p, L, pre, from_new, D, st));
    if (new_res == 1) ENC_TRY(launch_copy_cols(s->residual, 1, 0, s->conv0.p, L, pre + c0_len - 1, 1, D, st));
    s->residual_count = new_res;
    // the last two fed columns are the next call's conv1 context (conv.rs:281-303)
    ENC_TRY(launch_copy_cols(s->conv0_tail, 2, 0, s->c1_in.p, c1_len, c1_len - 2, 2, D, st));
    const size_t c1_out_len = c1_len / 2, discard = is_first ? 0 : 1;
    ENC_TRY(s->c1_out.reserve(D * c1_out_len, st));
    {
        const int sp = conv_splits(D, D, c1_out_len, s->num_sms);
        ENC_TRY(s->part.reserve((size_t)sp * D * c1_out_len, st));
        ENC_TRY(launch_conv(s->c1_in.p, c1_len, s->w1t, s->b1, D, D, 2, c1_out_len, s->c1_out.p, s->part.p, sp, st));
        s->launches += 2;
    }
    const size_t n = c1_out_len > discard ? c1_out_len - discard : 0;
    if (n > out_cap_rows) return report_errorf(VOX_ERR_SHAPE, "output holds %zu of %zu positions", out_cap_rows, n);
    if (n) {
        ENC_TRY(s->rows.reserve(D * n, st));
        const long long tot = (long long)D * (long long)n;
        cols_to_rows_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, st>>>(s->rows.p, s->c1_out.p, (int)c1_out_len,
                                                                           (int)discard, (int)n, (int)D);
        ENC_CUDA(cudaGetLastError());
        ENC_CUDA(cudaMemcpyAsync(out, s->rows.p, D * n * 4, cudaMemcpyDeviceToHost, st));
    }
    ENC_CUDA(cudaStreamSynchronize(st));
    *n_out = n;
    return VOX_OK;
}

// ---- op level (conv.rs:11-73) ---------------------------------------------------------

extern "C" size_t vox_conv_out_len(size_t length, size_t kernel, size_t stride) {
    if (kernel < stride || stride == 0) return 0;
    return conv_out_len(length, kernel, stride);
}

extern "C" int vox_causal_conv1d_gelu(int device, const float* input, const float* weight, const float* bias,
                                      size_t cin, size_t cout, size_t length, size_t stride, int apply_gelu,
                                      float* output) {
    if (!input || !weight || !output) return report_errorf(VOX_ERR_INVALID_ARG, "null argument");
    if (stride != 1 && stride != 2) return report_errorf(VOX_ERR_UNSUPPORTED, "kernel 3 with stride 1 or 2 only");
    if (cin == 0 || cout == 0 || cin > 65536 || cout > 65536 || length > (1u << 24))
        return report_errorf(VOX_ERR_INVALID_ARG, "bad convolution shape");
    const size_t out_len = conv_out_len(length, 3, stride);
    if (out_len == 0) return VOX_OK;
    ENC_CUDA(cudaSetDevice(device));
    const auto wt = transpose_w(weight, cout, cin);
    float *din = nullptr, *dw = nullptr, *db = nullptr, *dout = nullptr;
    auto cleanup = [&]() {
        for (float* p : {din, dw, db, dout})
            if (p) cudaFree(p);
    };
    if (cudaMalloc(&din, cin * length * 4) != cudaSuccess || cudaMalloc(&dw, wt.size() * 4) != cudaSuccess ||
        cudaMalloc(&dout, cout * out_len * 4) != cudaSuccess || (bias && cudaMalloc(&db, cout * 4) != cudaSuccess)) {
        cleanup();
        return report_errorf(VOX_ERR_OOM, "cannot allocate the convolution buffers");
    }
    int rc = VOX_OK;
    if (cudaMemcpy(din, input, cin * length * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dw, wt.data(), wt.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        (bias && cudaMemcpy(db, bias, cout * 4, cudaMemcpyHostToDevice) != cudaSuccess)) {
        rc = report_errorf(VOX_ERR_CUDA, "convolution upload failed");
    } else {
        dim3 grid((unsigned)((cout + 127) / 128), (unsigned)((out_len + kConvPT - 1) / kConvPT));
        causal_conv3_gelu_kernel<<<grid, 128>>>(din, (int)length, dw, db, (int)cin, (int)cout, (int)stride,
                                                (int)out_len, dout, apply_gelu ? 1 : 0);
        cudaError_t e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaMemcpy(output, dout, cout * out_len * 4, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) rc = report_errorf(VOX_ERR_CUDA, "convolution failed: %s", cudaGetErrorString(e));
    }
    cleanup();
    return rc;
}

extern "C" uint64_t vox_encoder_kernel_launches(const vox_mel* m, const vox_conv_stem* s) {
    return (m ? m->launches : 0) + (s ? s->launches : 0);
}
