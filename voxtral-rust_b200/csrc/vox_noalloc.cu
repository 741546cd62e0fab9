// vox_noalloc.cu -- decode attention for callers that cannot allocate.
//
// Some hosts of this library may not call cudaMalloc at all: an inference
// server whose memory is owned by a pool or arena it hands out itself, a
// process running under a fixed device-memory budget, or code that must not
// allocate on its decode path.  vox_attention_gqa_step_noalloc serves them:
// the caller passes device buffers for the inputs and the output, and the
// split-K working memory (per-split partial results, per-head tickets, the
// token-range descriptor) lives in one file-scope device array of fixed size
// instead of being allocated.
//
// The array is reserved once per GPU that loads the library and stays
// reserved until the process exits.  Every call on a device uses the same
// array: calls whose kernels can overlap on the GPU (different streams, or
// different host threads) race on it and must be serialised by the caller.
// The array's device address is looked up once per device; a caller that
// resets a device (cudaDeviceReset) must not call this entry point on it
// afterwards.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/vox_decoder.h"
#include "vox_device.cuh"

namespace vox {

namespace {

// Fixed scratch: a 256-byte descriptor block (the token-range state at 0, the
// device error word at kErrOffset), the tickets, then the partials.
constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;  // 1 MiB per device
static __device__ __align__(256) unsigned char g_attn_scratch[kNoAllocScratchBytes];

constexpr size_t kErrOffset = 64;
constexpr size_t kTicketOffset = 256;
constexpr int kMaxDevices = 64;

struct DeviceSetup {
    bool ready = false;
    unsigned char* scratch = nullptr;  // device address of g_attn_scratch
    int num_sms = 0;
};

std::mutex g_setup_mutex;
DeviceSetup g_setup[kMaxDevices];

size_t round256(size_t b) { return (b + 255) & ~size_t(255); }

// Writes the token-range descriptor (len = seq_len, start 0) and clears the
// error word and the tickets: the previous call leaves its values behind.
__global__ void noalloc_prepare_kernel(int seq_len, int n_kv) {
    KvState* st = reinterpret_cast<KvState*>(g_attn_scratch);
    unsigned* tickets = reinterpret_cast<unsigned*>(g_attn_scratch + kTicketOffset);
    if (threadIdx.x == 0) {
        st->len = seq_len;
        st->start = 0;
        st->pos_offset = 0;
        *reinterpret_cast<unsigned*>(g_attn_scratch + kErrOffset) = 0u;
    }
    for (int i = threadIdx.x; i < n_kv; i += blockDim.x) tickets[i] = 0u;
}

// Once per device, with that device current: resolve the array's device
// address (the host-side name is only a stand-in), read the SM count and
// raise the attention kernel's shared-memory limit.
int setup_device(int dev, DeviceSetup** out) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    DeviceSetup& s = g_setup[dev];
    if (!s.ready) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess) return report_error(VOX_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed");
        e = cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return report_error(VOX_ERR_CUDA, "cannot read the SM count");
        e = attn_prepare(dev);
        if (e != cudaSuccess) return report_error(VOX_ERR_CUDA, "cannot set the attention smem limit");
        s.scratch = static_cast<unsigned char*>(p);
        s.ready = true;
    }
    *out = &s;
    return VOX_OK;
}

}  // namespace

}  // namespace vox

using namespace vox;

extern "C" int vox_attention_gqa_step_noalloc(const float* d_query, const float* d_keys,
                                              const float* d_values, const vox_attention_shape* sh,
                                              float* d_out, void* stream) {
    if (!sh || !d_query || !d_out) return report_error(VOX_ERR_INVALID_ARG, "null argument");
    if (sh->n_heads == 0 || sh->n_kv_heads == 0 || sh->head_dim == 0)
        return report_error(VOX_ERR_INVALID_ARG, "n_heads, n_kv_heads and head_dim must be > 0");
    if (sh->n_heads % sh->n_kv_heads)
        return report_error(VOX_ERR_INVALID_ARG, "n_heads must be divisible by n_kv_heads");
    if (sh->seq_len && (!d_keys || !d_values)) return report_error(VOX_ERR_INVALID_ARG, "null keys/values");
    if (sh->n_heads > 4096 || sh->head_dim > 4096 || sh->seq_len > (size_t)INT32_MAX / 2 ||
        !attn_supported((int)sh->n_heads, (int)sh->n_kv_heads, (int)sh->head_dim))
        return report_error(VOX_ERR_UNSUPPORTED, "attention shape not supported");

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return report_error(VOX_ERR_CUDA, "no usable current CUDA device");
    DeviceSetup* s = nullptr;
    int rc = setup_device(dev, &s);
    if (rc != VOX_OK) return rc;

    const size_t nh = sh->n_heads, nkv = sh->n_kv_heads, hd = sh->head_dim;
    const size_t G = nh / nkv;
    const size_t part_off = kTicketOffset + round256(nkv * sizeof(unsigned));
    const size_t per_split = nkv * G * (hd + 2) * sizeof(float);
    // Use as many splits as the kernel wants, down to what the array holds.
    int nsplit = attn_splits_for((int)nkv, s->num_sms);
    while (nsplit > 1 && part_off + (size_t)nsplit * per_split > kNoAllocScratchBytes) --nsplit;
    if (part_off + (size_t)nsplit * per_split > kNoAllocScratchBytes)
        return report_error(VOX_ERR_UNSUPPORTED,
                            "attention needs more than the 1 MiB no-alloc scratch "
                            "(n_heads * (head_dim + 2) * 4 bytes per split must fit)");

    // An error left by earlier work of the caller is reported as such (and
    // left in place for the caller), not mistaken for a launch failure here.
    if (cudaPeekAtLastError() != cudaSuccess)
        return report_error(VOX_ERR_CUDA, "an earlier CUDA error is pending on this thread; nothing was launched");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    noalloc_prepare_kernel<<<1, 64, 0, st>>>((int)sh->seq_len, (int)nkv);
    if (cudaGetLastError() != cudaSuccess) return report_error(VOX_ERR_CUDA, "prepare launch failed");

    AttnArgs at{};
    at.q = d_query;
    at.k_ring = d_keys;
    at.v_ring = d_values;
    at.n_heads = (int)nh;
    at.n_kv = (int)nkv;
    at.hd = (int)hd;
    at.cap = sh->seq_len ? (int)sh->seq_len : 1;
    at.cfg_window = (int)sh->sliding_window;
    at.st = reinterpret_cast<const KvState*>(s->scratch);
    at.pre_append = 0;
    at.nsplit = nsplit;
    at.part = reinterpret_cast<float*>(s->scratch + part_off);
    at.tickets = reinterpret_cast<unsigned*>(s->scratch + kTicketOffset);
    at.out = d_out;
    at.scale = 1.0f / sqrtf((float)hd);  // ops.rs:89
    // A bounded wait that expires inside the kernel sets a bit here; the call
    // returns before the kernel runs, so it cannot report it (see the header).
    at.err = reinterpret_cast<unsigned*>(s->scratch + kErrOffset);
    if (launch_attention(at, st, false) != cudaSuccess) {
        (void)cudaGetLastError();
        return report_error(VOX_ERR_CUDA, "attention launch failed");
    }
    return VOX_OK;
}
