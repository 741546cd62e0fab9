// vox_misc.cu -- small kernels around the token loop: final argmax, KV ring
// scatter/gather, seeded weight generation, and the op-level element-wise
// kernels (RMSNorm rows, RoPE, SiLU, softmax, add).
#include <cuda_runtime.h>
#include <math.h>

#include "vox_device.cuh"

namespace vox {

namespace {

// ---- final argmax over the LM head's per-CTA candidates ----------------------
__global__ void __launch_bounds__(256) argmax_final_kernel(const ArgmaxPart* parts, int n,
                                                          StepState* step, int32_t* tok_out) {
    pdl_allow_dependents();
    pdl_wait_prior_grids();
    __shared__ float sv[8];
    __shared__ int si[8];
    float best = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = parts[i].v;
        const int idx = parts[i].i;
        if (v > best || (v == best && idx < bi)) {
            best = v;
            bi = idx;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, best, o);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = best;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
                best = sv[w];
                bi = si[w];
            }
        if (bi == 0x7FFFFFFF) bi = 0;  // all logits NaN: token 0, as a scan from index 0 keeps
        step->next_tok = bi;
        if (step->greedy) step->tok = bi;
        if (step->advance) step->pos += 1;
        if (tok_out) *tok_out = bi;
    }
}

// ---- tensor-parallel argmax: one (value, index) key per rank --------------------
// Order-preserving key: a larger key is a larger value, or the same value at a
// lower global index; 0 means "no finite candidate" (all NaN).
__device__ __forceinline__ unsigned long long tp_argmax_key(float best, int bi, long long index_offset) {
    if (bi == 0x7FFFFFFF) return 0ull;
    if (best == 0.0f) best = 0.0f;  // -0 and +0 compare equal: same key
    const uint32_t u = __float_as_uint(best);
    const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    const uint32_t gi = (uint32_t)(index_offset + bi);
    return ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - gi);
}

__device__ __forceinline__ void tp_apply_key(unsigned long long k, StepState* step, int32_t* tok_out) {
    const int idx = k == 0ull ? 0 : (int)(0xFFFFFFFFu - (uint32_t)k);  // all NaN: token 0
    step->next_tok = idx;
    if (step->greedy) step->tok = idx;
    if (step->advance) step->pos += 1;
    if (tok_out) *tok_out = idx;
}

__global__ void __launch_bounds__(256) tp_argmax_key_kernel(const ArgmaxPart* parts, int n, long long index_offset,
                                                           unsigned long long* key) {
    pdl_allow_dependents();
    pdl_wait_prior_grids();
    __shared__ float sv[8];
    __shared__ int si[8];
    float best = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = parts[i].v;
        const int idx = parts[i].i;
        if (v > best || (v == best && idx < bi)) {
            best = v;
            bi = idx;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, best, o);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = best;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
                best = sv[w];
                bi = si[w];
            }
        *key = tp_argmax_key(best, bi, index_offset);
    }
}

// One block: the rank's best candidate, exchanged with every rank through
// peer memory, then the global argmax and the step bookkeeping.
__global__ void __launch_bounds__(256) tp_argmax_xch_kernel(const ArgmaxPart* parts, int n, long long index_offset,
                                                           unsigned char* const* xch, XchArea xa,
                                                           unsigned long long* tp_steps, StepState* step,
                                                           int32_t* tok_out, unsigned* err) {
    pdl_allow_dependents();
    pdl_wait_prior_grids();
    __shared__ float sv[8];
    __shared__ int si[8];
    float best = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = parts[i].v;
        const int idx = parts[i].i;
        if (v > best || (v == best && idx < bi)) {
            best = v;
            bi = idx;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, best, o);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = best;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
                best = sv[w];
                bi = si[w];
            }
        const unsigned long long mine = tp_argmax_key(best, bi, index_offset);
        for (int p = 0; p < xa.size; ++p) xa.keys(xch[p])[xa.rank] = mine;
        __threadfence_system();
        for (int p = 0; p < xa.size; ++p) atomicAdd_system(xa.key_counter(xch[p]), 1ull);
        unsigned char* own = xch[xa.rank];
        const unsigned long long done = *reinterpret_cast<volatile unsigned long long*>(tp_steps);
        unsigned long long k = 0ull;
        const bool expired = (*reinterpret_cast<volatile unsigned*>(err) & ERR_PEER_WAIT) != 0u;
        if (!expired && wait_counter_sys(xa.key_counter(own), (done + 1ull) * (unsigned long long)xa.size)) {
            for (int r = 0; r < xa.size; ++r) {
                const unsigned long long kr = __ldcg(xa.keys(own) + r);
                if (kr > k) k = kr;
            }
        } else {
            raise_error(err, ERR_PEER_WAIT);
        }
        tp_apply_key(k, step, tok_out);
        *tp_steps = done + 1ull;
    }
}

__global__ void tp_argmax_apply_kernel(const unsigned long long* key, StepState* step, int32_t* tok_out) {
    pdl_allow_dependents();
    pdl_wait_prior_grids();
    if (threadIdx.x == 0) tp_apply_key(*key, step, tok_out);
}

// ---- KV ring scatter / gather -------------------------------------------------
// src is token-major [n, n_kv, hd] (the reference's layout); ring head-major.
__global__ void kv_scatter_kernel(const float* __restrict__ sk, const float* __restrict__ sv,
                                  float* __restrict__ kr, float* __restrict__ vr, int n_kv, int hd,
                                  int cap, int slot0, long long total) {
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int d = (int)(e % hd);
        const long long th = e / hd;
        const int h = (int)(th % n_kv);
        const long long t = th / n_kv;
        const long long slot = (slot0 + t) % cap;
        const size_t dst = ((size_t)h * cap + slot) * hd + d;
        kr[dst] = sk[e];
        vr[dst] = sv[e];
    }
}

__global__ void kv_gather_kernel(const float* __restrict__ kr, const float* __restrict__ vr,
                                 float* __restrict__ dk, float* __restrict__ dv, int n_kv, int hd,
                                 int cap, int start, long long total) {
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int d = (int)(e % hd);
        const long long th = e / hd;
        const int h = (int)(th % n_kv);
        const long long t = th / n_kv;
        const long long slot = (start + t) % cap;
        const size_t src = ((size_t)h * cap + slot) * hd + d;
        dk[e] = kr[src];
        dv[e] = vr[src];
    }
}

// ---- seeded generator (same definition as the oracle's) -----------------------
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z ^= z >> 30;
    z *= 0xBF58476D1CE4E5B9ull;
    z ^= z >> 27;
    z *= 0x94D049BB133111EBull;
    z ^= z >> 31;
    return z;
}

__device__ __forceinline__ float gen_z(uint64_t key, uint64_t e) {
    uint32_t s = 0;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const uint64_t h = mix64(key + (3 * e + (uint64_t)j) * 0x9E3779B97F4A7C15ull);
        s += (uint32_t)(h & 0xFFFF) + (uint32_t)((h >> 16) & 0xFFFF) +
             (uint32_t)((h >> 32) & 0xFFFF) + (uint32_t)(h >> 48);
    }
    const int32_t c = (int32_t)(2 * s + 12) - 786432;
    return __fmul_rn((float)c, 1.0f / 131072.0f);
}

__device__ __forceinline__ uint16_t f32_to_bf16_rne(float f) {
    const uint32_t u = __float_as_uint(f);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return 0x7FC0;
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

// Element (r, c) of a [rows, cols] block of the logical tensor, whose
// top-left element is (row0, col0) of a tensor with full_cols columns; the
// generator is indexed by the logical element.
__global__ void gen_matrix_kernel(void* dst, int wsize, uint64_t key, float stdv, long long rows,
                                  long long cols, int row_mul, int row_add, long long row0, long long col0,
                                  long long full_cols) {
    const long long total = rows * cols;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const long long r = e / cols, c = e - r * cols;
        const size_t o = (size_t)(r * row_mul + row_add) * cols + c;
        const uint64_t le = (uint64_t)((row0 + r) * full_cols + col0 + c);
        const float v = __fmul_rn(gen_z(key, le), stdv);
        if (wsize == 2)
            reinterpret_cast<uint16_t*>(dst)[o] = f32_to_bf16_rne(v);
        else
            reinterpret_cast<float*>(dst)[o] = v;
    }
}

// Random cache contents: logical token t of kv head h, element d, is element
// (t * n_kv + h) * hd + d of the generator's tensor (the reference's
// token-major layout), rounded to bf16 and stored widened in the ring slot t.
__global__ void kv_fill_random_kernel(float* __restrict__ kr, float* __restrict__ vr, int n_kv, int hd, int cap,
                                      long long total, uint64_t key_k, uint64_t key_v, float stdv) {
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int d = (int)(e % hd);
        const long long th = e / hd;
        const int h = (int)(th % n_kv);
        const long long t = th / n_kv;
        const size_t dst = ((size_t)h * cap + t) * hd + d;
        kr[dst] = bf16_bits_to_f32(f32_to_bf16_rne(__fmul_rn(gen_z(key_k, (uint64_t)e), stdv)));
        vr[dst] = bf16_bits_to_f32(f32_to_bf16_rne(__fmul_rn(gen_z(key_v, (uint64_t)e), stdv)));
    }
}

__global__ void fill_kernel(float* dst, float v, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        dst[i] = v;
}

// ---- op-level element-wise kernels ----------------------------------------------
// rms_norm_rows (math.rs:11-27): one CTA per row.
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(float* out, const float* in,
                                                          const float* w, int dim, float eps) {
    __shared__ float red[8];
    const float* x = in + (size_t)blockIdx.x * dim;
    float* y = out + (size_t)blockIdx.x * dim;
    float ss = 0.f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)dim), eps)));
    for (int i = threadIdx.x; i < dim; i += blockDim.x) y[i] = __fmul_rn(__fmul_rn(x[i], inv), w[i]);
}

// rope_interleaved_inplace (math.rs:30-65) with a [seq_len, hd/2] cos/sin table.
__global__ void rope_table_kernel(float* data, const float* ct, const float* st, long long seq_len,
                                  int n_heads, int hd) {
    const int half = hd / 2;
    const long long total = seq_len * n_heads * half;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int p = (int)(e % half);
        const long long th = e / half;
        const long long t = th / n_heads;
        float* x = data + th * hd + 2 * p;
        const float c = ct[t * half + p], s = st[t * half + p];
        const float x0 = x[0], x1 = x[1];
        x[0] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        x[1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
}

// silu_inplace (math.rs:4-9)
__global__ void silu_kernel(float* x, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const float t = x[i];
        x[i] = __fdiv_rn(t, __fadd_rn(1.0f, expf(-t)));
    }
}

// softmax_inplace (math.rs:67-88): one CTA; max, exp-sum, divide if sum > 0.
__global__ void __launch_bounds__(1024) softmax_kernel(float* x, long long n) {
    __shared__ float red[32];
    __shared__ float bc;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    float m = -INFINITY;
    for (long long i = tid; i < n; i += blockDim.x) m = fmaxf(m, x[i]);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (tid == 0) {
        float t = red[0];
        for (int i = 1; i < nw; ++i) t = fmaxf(t, red[i]);
        bc = t;
    }
    __syncthreads();
    const float mx = bc;
    float s = 0.f;
    for (long long i = tid; i < n; i += blockDim.x) {
        const float e = expf(x[i] - mx);
        x[i] = e;
        s += e;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    __syncthreads();
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
        for (int i = 0; i < nw; ++i) t += red[i];
        bc = t;
    }
    __syncthreads();
    const float sum = bc;
    if (sum > 0.f)
        for (long long i = tid; i < n; i += blockDim.x) x[i] = __fdiv_rn(x[i], sum);
}

__global__ void add_kernel(float* dst, const float* src, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        dst[i] = __fadd_rn(dst[i], src[i]);
}

inline int grid_for(long long n, int block) {
    long long g = (n + block - 1) / block;
    if (g > 148 * 8) g = 148 * 8;
    return g < 1 ? 1 : (int)g;
}

uint64_t host_mix64(uint64_t z) {
    z ^= z >> 30;
    z *= 0xBF58476D1CE4E5B9ull;
    z ^= z >> 27;
    z *= 0x94D049BB133111EBull;
    z ^= z >> 31;
    return z;
}

}  // namespace

cudaError_t launch_argmax_final(const ArgmaxPart* parts, int n, StepState* step, int32_t* tok_out,
                                cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, argmax_final_kernel, parts, n, step, tok_out);
}

cudaError_t launch_tp_argmax_key(const ArgmaxPart* parts, int n, long long index_offset, unsigned long long* key,
                                 cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, tp_argmax_key_kernel, parts, n, index_offset, key);
}

cudaError_t launch_tp_argmax_xch(const ArgmaxPart* parts, int n, long long index_offset, unsigned char* const* xch,
                                 XchArea xa, unsigned long long* tp_steps, StepState* step, int32_t* tok_out,
                                 unsigned* err, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, tp_argmax_xch_kernel, parts, n, index_offset, xch, xa, tp_steps, step, tok_out,
                              err);
}

cudaError_t launch_tp_argmax_apply(const unsigned long long* key, StepState* step, int32_t* tok_out, cudaStream_t s) {
    tp_argmax_apply_kernel<<<1, 32, 0, s>>>(key, step, tok_out);
    return cudaGetLastError();
}

cudaError_t launch_kv_scatter(const float* sk, const float* sv, float* kr, float* vr, int n_kv, int hd,
                              int cap, int slot0, int n_tokens, cudaStream_t s) {
    const long long total = (long long)n_tokens * n_kv * hd;
    if (total == 0) return cudaSuccess;
    kv_scatter_kernel<<<grid_for(total, 256), 256, 0, s>>>(sk, sv, kr, vr, n_kv, hd, cap, slot0, total);
    return cudaGetLastError();
}

cudaError_t launch_kv_gather(const float* kr, const float* vr, float* dk, float* dv, int n_kv, int hd,
                             int cap, int start, int len, cudaStream_t s) {
    const long long total = (long long)len * n_kv * hd;
    if (total == 0) return cudaSuccess;
    kv_gather_kernel<<<grid_for(total, 256), 256, 0, s>>>(kr, vr, dk, dv, n_kv, hd, cap, start, total);
    return cudaGetLastError();
}

cudaError_t launch_gen_matrix(void* dst, int wsize, uint64_t seed, uint64_t tensor_id, float stdv,
                              long long rows, long long cols, int row_mul, int row_add,
                              cudaStream_t s) {
    return launch_gen_matrix_part(dst, wsize, seed, tensor_id, stdv, rows, cols, row_mul, row_add, 0, 0, cols, s);
}

cudaError_t launch_gen_matrix_part(void* dst, int wsize, uint64_t seed, uint64_t tensor_id, float stdv,
                                   long long rows, long long cols, int row_mul, int row_add, long long row0,
                                   long long col0, long long full_cols, cudaStream_t s) {
    const uint64_t key = host_mix64(seed ^ host_mix64(tensor_id + 0x632BE59BD9B4E019ull));
    const long long total = rows * cols;
    if (total == 0) return cudaSuccess;
    gen_matrix_kernel<<<grid_for(total, 256), 256, 0, s>>>(dst, wsize, key, stdv, rows, cols, row_mul,
                                                           row_add, row0, col0, full_cols);
    return cudaGetLastError();
}

cudaError_t launch_kv_fill_random(float* kr, float* vr, int n_kv, int hd, int cap, int len, uint64_t seed,
                                  uint64_t id_k, uint64_t id_v, float stdv, cudaStream_t s) {
    const long long total = (long long)len * n_kv * hd;
    if (total == 0) return cudaSuccess;
    const uint64_t kk = host_mix64(seed ^ host_mix64(id_k + 0x632BE59BD9B4E019ull));
    const uint64_t kvv = host_mix64(seed ^ host_mix64(id_v + 0x632BE59BD9B4E019ull));
    kv_fill_random_kernel<<<grid_for(total, 256), 256, 0, s>>>(kr, vr, n_kv, hd, cap, total, kk, kvv, stdv);
    return cudaGetLastError();
}

cudaError_t launch_fill_f32(float* dst, float v, long long n, cudaStream_t s) {
    fill_kernel<<<grid_for(n, 256), 256, 0, s>>>(dst, v, n);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm_rows(float* out, const float* in, const float* w, long long n_rows, int dim,
                                float eps, cudaStream_t s) {
    if (n_rows == 0) return cudaSuccess;
    rmsnorm_rows_kernel<<<(unsigned)n_rows, 256, 0, s>>>(out, in, w, dim, eps);
    return cudaGetLastError();
}

cudaError_t launch_rope_table(float* data, const float* ct, const float* st, long long seq_len,
                              int n_heads, int hd, cudaStream_t s) {
    const long long total = seq_len * n_heads * (hd / 2);
    if (total == 0) return cudaSuccess;
    rope_table_kernel<<<grid_for(total, 256), 256, 0, s>>>(data, ct, st, seq_len, n_heads, hd);
    return cudaGetLastError();
}

cudaError_t launch_silu(float* x, long long n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    silu_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, n);
    return cudaGetLastError();
}

cudaError_t launch_softmax(float* x, long long n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    softmax_kernel<<<1, 1024, 0, s>>>(x, n);
    return cudaGetLastError();
}

cudaError_t launch_add(float* dst, const float* src, long long n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    add_kernel<<<grid_for(n, 256), 256, 0, s>>>(dst, src, n);
    return cudaGetLastError();
}

}  // namespace vox
