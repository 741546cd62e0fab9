// vox_weights.cpp -- safetensors checkpoints: WeightStore (weights.rs:16-93)
// and the upload of a decoder checkpoint into a context.
//
// The file is memory-mapped read-only (weights.rs:37-42).  Its header is
// parsed and validated once at open time, with the rules of the safetensors
// format the reference reads through the `safetensors` crate (0.4.5,
// Cargo.lock:847-848): an 8-byte little-endian header length (at most
// 100,000,000), a JSON object of {name: {dtype, shape, data_offsets}} plus an
// optional "__metadata__" map, tensors packed back to back from offset 0 in
// offset order, each exactly numel * element size bytes, the last one ending
// at the end of the file.  tensor_f32 (weights.rs:49-93) copies F32 data and
// widens BF16 by bits << 16; other dtypes are refused.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/vox_decoder.h"
#include "vox_host.h"
#include "vox_internal.h"
#include "vox_json.h"

using namespace vox;

namespace {

struct DtypeInfo {
    const char* name;
    size_t size;
};
// Order = vox_tensor_dtype.
const DtypeInfo kDtypes[] = {{"BOOL", 1}, {"U8", 1},   {"I8", 1},   {"F8_E5M2", 1}, {"F8_E4M3", 1},
                             {"I16", 2},  {"U16", 2},  {"F16", 2},  {"BF16", 2},    {"I32", 4},
                             {"U32", 4},  {"F32", 4},  {"F64", 8},  {"I64", 8},     {"U64", 8}};
constexpr int kNumDtypes = sizeof(kDtypes) / sizeof(kDtypes[0]);
constexpr uint64_t kMaxHeader = 100000000ull;

struct TensorEntry {
    std::string name;
    int dtype = 0;
    std::vector<size_t> shape;
    size_t begin = 0, end = 0;  // relative to the data section
};

}  // namespace

struct vox_weights {
    void* map = nullptr;
    size_t map_len = 0;
    const unsigned char* data = nullptr;  // start of the data section
    size_t data_len = 0;
    std::vector<TensorEntry> tensors;     // in offset order
    const TensorEntry* find(const char* name) const {
        for (const auto& t : tensors)
            if (t.name == name) return &t;
        return nullptr;
    }
};

namespace {

int parse_header(vox_weights* w, const unsigned char* base, size_t len) {
    if (len < 8) return report_errorf(VOX_ERR_FORMAT, "safetensors: file shorter than the 8-byte header length");
    uint64_t n = 0;
    for (int i = 7; i >= 0; --i) n = (n << 8) | base[i];
    if (n > kMaxHeader) return report_errorf(VOX_ERR_FORMAT, "safetensors: header of %llu bytes is too large",
                                             (unsigned long long)n);
    if (n > len - 8) return report_errorf(VOX_ERR_FORMAT, "safetensors: header length %llu beyond the file",
                                          (unsigned long long)n);
    const char* h = reinterpret_cast<const char*>(base + 8);
    if (n == 0 || h[0] != '{') return report_errorf(VOX_ERR_FORMAT, "safetensors: header does not start with '{'");
    Json root;
    std::string err;
    JsonParser jp(h, (size_t)n);
    if (!jp.parse(&root, &err) || root.kind != Json::Object)
        return report_errorf(VOX_ERR_FORMAT, "safetensors: invalid header JSON (%s)", err.c_str());
    w->data = base + 8 + n;
    w->data_len = len - 8 - (size_t)n;
    for (const auto& kv : root.obj) {
        if (kv.first == "__metadata__") {
            if (kv.second.kind != Json::Object && kv.second.kind != Json::Null)
                return report_errorf(VOX_ERR_FORMAT, "safetensors: __metadata__ is not a map");
            for (const auto& m : kv.second.obj)
                if (m.second.kind != Json::String)
                    return report_errorf(VOX_ERR_FORMAT, "safetensors: __metadata__ values must be strings");
            continue;
        }
        const Json& t = kv.second;
        const Json* dt = t.get("dtype");
        const Json* sh = t.get("shape");
        const Json* off = t.get("data_offsets");
        if (t.kind != Json::Object || !dt || dt->kind != Json::String || !sh || sh->kind != Json::Array || !off ||
            off->kind != Json::Array || off->arr.size() != 2)
            return report_errorf(VOX_ERR_FORMAT, "safetensors: malformed entry for %s", kv.first.c_str());
        TensorEntry e;
        e.name = kv.first;
        e.dtype = -1;
        for (int d = 0; d < kNumDtypes; ++d)
            if (dt->str == kDtypes[d].name) e.dtype = d;
        if (e.dtype < 0)
            return report_errorf(VOX_ERR_FORMAT, "safetensors: unknown dtype %s for %s", dt->str.c_str(),
                                 kv.first.c_str());
        size_t numel = 1;
        for (const Json& d : sh->arr) {
            if (d.kind != Json::Number || !d.is_int || d.i64 < 0)
                return report_errorf(VOX_ERR_FORMAT, "safetensors: bad shape for %s", kv.first.c_str());
            const size_t v = (size_t)d.i64;
            if (v && numel > SIZE_MAX / v) return report_errorf(VOX_ERR_FORMAT, "safetensors: shape overflow");
            numel *= v;
            e.shape.push_back(v);
        }
        for (const Json& o : off->arr)
            if (o.kind != Json::Number || !o.is_int || o.i64 < 0)
                return report_errorf(VOX_ERR_FORMAT, "safetensors: bad data_offsets for %s", kv.first.c_str());
        e.begin = (size_t)off->arr[0].i64;
        e.end = (size_t)off->arr[1].i64;
        if (e.end < e.begin || numel > SIZE_MAX / kDtypes[e.dtype].size ||
            e.end - e.begin != numel * kDtypes[e.dtype].size)
            return report_errorf(VOX_ERR_FORMAT, "safetensors: %s holds %zu bytes, its shape and dtype need %zu",
                                 kv.first.c_str(), e.end - e.begin, numel * kDtypes[e.dtype].size);
        w->tensors.push_back(std::move(e));
    }
    std::sort(w->tensors.begin(), w->tensors.end(),
              [](const TensorEntry& a, const TensorEntry& b) { return a.begin < b.begin || (a.begin == b.begin && a.end < b.end); });
    size_t at = 0;
    for (const auto& e : w->tensors) {
        if (e.begin != at) return report_errorf(VOX_ERR_FORMAT, "safetensors: invalid offset for %s", e.name.c_str());
        at = e.end;
    }
    if (at != w->data_len)
        return report_errorf(VOX_ERR_FORMAT, "safetensors: tensors cover %zu of %zu data bytes", at, w->data_len);
    return VOX_OK;
}

}  // namespace

extern "C" int vox_weights_open(const char* path, vox_weights** out) {
    if (!path || !out) return report_errorf(VOX_ERR_INVALID_ARG, "null path or output");
    *out = nullptr;
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return report_errorf(VOX_ERR_IO, "cannot open %s", path);
    struct stat stt;
    if (fstat(fd, &stt) != 0) {
        close(fd);
        return report_errorf(VOX_ERR_IO, "cannot stat %s", path);
    }
    auto* w = new vox_weights();
    w->map_len = (size_t)stt.st_size;
    if (w->map_len) {
        w->map = mmap(nullptr, w->map_len, PROT_READ, MAP_PRIVATE, fd, 0);
        if (w->map == MAP_FAILED) {
            close(fd);
            delete w;
            return report_errorf(VOX_ERR_IO, "cannot map %s", path);
        }
    }
    close(fd);
    const int rc = parse_header(w, static_cast<const unsigned char*>(w->map), w->map_len);
    if (rc != VOX_OK) {
        vox_weights_close(w);
        return rc;
    }
    *out = w;
    return VOX_OK;
}

extern "C" void vox_weights_close(vox_weights* w) {
    if (!w) return;
    if (w->map && w->map != MAP_FAILED) munmap(w->map, w->map_len);
    delete w;
}

extern "C" size_t vox_weights_count(const vox_weights* w) { return w ? w->tensors.size() : 0; }

extern "C" const char* vox_weights_name(const vox_weights* w, size_t i) {
    return w && i < w->tensors.size() ? w->tensors[i].name.c_str() : nullptr;
}

extern "C" int vox_weights_info(const vox_weights* w, const char* name, int* dtype, size_t* shape, size_t shape_cap,
                                size_t* ndim) {
    if (!w || !name) return report_errorf(VOX_ERR_INVALID_ARG, "null weights or name");
    const TensorEntry* e = w->find(name);
    if (!e) return report_errorf(VOX_ERR_INVALID_ARG, "tensor %s not found", name);
    if (dtype) *dtype = e->dtype;
    if (ndim) *ndim = e->shape.size();
    for (size_t i = 0; shape && i < e->shape.size() && i < shape_cap; ++i) shape[i] = e->shape[i];
    return VOX_OK;
}

extern "C" int vox_weights_tensor_f32(const vox_weights* w, const char* name, float* out, size_t cap_elems,
                                      size_t* n_elems) {
    if (!w || !name) return report_errorf(VOX_ERR_INVALID_ARG, "null weights or name");
    const TensorEntry* e = w->find(name);
    if (!e) return report_errorf(VOX_ERR_INVALID_ARG, "tensor %s not found", name);
    const unsigned char* raw = w->data + e->begin;
    const size_t bytes = e->end - e->begin;
    size_t n;
    if (e->dtype == VOX_DT_F32) {
        n = bytes / 4;
    } else if (e->dtype == VOX_DT_BF16) {
        n = bytes / 2;
    } else {  // weights.rs:84-89
        return report_errorf(VOX_ERR_FORMAT, "unsupported dtype for %s: %s", name, kDtypes[e->dtype].name);
    }
    if (n_elems) *n_elems = n;
    if (!out) return VOX_OK;  // size query
    if (cap_elems < n) return report_errorf(VOX_ERR_SHAPE, "output holds %zu of %zu elements of %s", cap_elems, n, name);
    if (e->dtype == VOX_DT_F32) {
        std::memcpy(out, raw, n * 4);  // little-endian host, as from_le_bytes
    } else {
        for (size_t i = 0; i < n; ++i) {
            const uint32_t bits = (uint32_t)raw[2 * i] | ((uint32_t)raw[2 * i + 1] << 8);
            out[i] = bf16_to_f32((uint16_t)bits);  // f32::from_bits(bits << 16), weights.rs:77-81
        }
    }
    return VOX_OK;
}

// ---- decoder checkpoint -> context ------------------------------------------------

namespace {

// A tensor as bf16 bits: BF16 copied, F32 rounded to nearest even (what the
// bf16 upload of an f32 matrix does).
int tensor_bf16(const vox_weights* w, const std::string& name, size_t want, std::vector<uint16_t>* out) {
    const TensorEntry* e = w->find(name.c_str());
    if (!e) return report_errorf(VOX_ERR_INVALID_ARG, "checkpoint has no tensor %s", name.c_str());
    if (e->dtype != VOX_DT_BF16 && e->dtype != VOX_DT_F32)
        return report_errorf(VOX_ERR_FORMAT, "unsupported dtype for %s: %s", name.c_str(), kDtypes[e->dtype].name);
    const size_t n = (e->end - e->begin) / kDtypes[e->dtype].size;
    if (n != want) return report_errorf(VOX_ERR_SHAPE, "%s shape mismatch (%zu elements, want %zu)", name.c_str(), n, want);
    out->resize(n);
    const unsigned char* raw = w->data + e->begin;
    if (e->dtype == VOX_DT_BF16) {
        std::memcpy(out->data(), raw, n * 2);
    } else {
        for (size_t i = 0; i < n; ++i) {
            float f;
            std::memcpy(&f, raw + 4 * i, 4);
            (*out)[i] = f32_to_bf16(f);
        }
    }
    return VOX_OK;
}

int tensor_f32(const vox_weights* w, const std::string& name, size_t want, std::vector<float>* out) {
    size_t n = 0;
    int rc = vox_weights_tensor_f32(w, name.c_str(), nullptr, 0, &n);
    if (rc != VOX_OK) return rc;
    if (n != want) return report_errorf(VOX_ERR_SHAPE, "%s shape mismatch (%zu elements, want %zu)", name.c_str(), n, want);
    out->resize(n);
    return vox_weights_tensor_f32(w, name.c_str(), out->data(), n, &n);
}

}  // namespace

extern "C" int vox_ctx_load_checkpoint(vox_ctx* ctx, const vox_weights* w) {
    if (!ctx || !w) return report_errorf(VOX_ERR_INVALID_ARG, "null context or weights");
    CtxInfo info{};
    int rc = ctx_info(ctx, &info);
    if (rc != VOX_OK) return rc;
    const vox_decoder_config& c = info.cfg;
    const size_t dim = c.dim, hid = c.hidden_dim, q = c.n_heads * c.head_dim, kv = c.n_kv_heads * c.head_dim;
    for (size_t l = 0; l < info.n_layers; ++l) {
        const std::string p = "layers." + std::to_string(l) + ".";
        std::vector<float> an, fn;
        if ((rc = tensor_f32(w, p + "attention_norm.weight", dim, &an)) != VOX_OK) return rc;
        if ((rc = tensor_f32(w, p + "ffn_norm.weight", dim, &fn)) != VOX_OK) return rc;
        if (info.weight_dtype == VOX_WEIGHTS_F32) {
            std::vector<float> m[7];
            const char* names[7] = {"attention.wq", "attention.wk", "attention.wv", "attention.wo",
                                    "feed_forward.w1", "feed_forward.w2", "feed_forward.w3"};
            const size_t sizes[7] = {q * dim, kv * dim, kv * dim, dim * q, hid * dim, dim * hid, hid * dim};
            for (int i = 0; i < 7; ++i)
                if ((rc = tensor_f32(w, p + names[i] + ".weight", sizes[i], &m[i])) != VOX_OK) return rc;
            vox_layer_weights_f32 lw{{an.data(), an.size()}, {m[0].data(), m[0].size()}, {m[1].data(), m[1].size()},
                                     {m[2].data(), m[2].size()}, {m[3].data(), m[3].size()}, {fn.data(), fn.size()},
                                     {m[4].data(), m[4].size()}, {m[5].data(), m[5].size()}, {m[6].data(), m[6].size()}};
            if ((rc = vox_ctx_upload_layer_f32(ctx, l, &lw)) != VOX_OK) return rc;
        } else {
            std::vector<uint16_t> m[7];
            const char* names[7] = {"attention.wq", "attention.wk", "attention.wv", "attention.wo",
                                    "feed_forward.w1", "feed_forward.w2", "feed_forward.w3"};
            const size_t sizes[7] = {q * dim, kv * dim, kv * dim, dim * q, hid * dim, dim * hid, hid * dim};
            for (int i = 0; i < 7; ++i)
                if ((rc = tensor_bf16(w, p + names[i] + ".weight", sizes[i], &m[i])) != VOX_OK) return rc;
            vox_layer_weights_bf16 lw{{an.data(), an.size()}, {m[0].data(), m[0].size()}, {m[1].data(), m[1].size()},
                                      {m[2].data(), m[2].size()}, {m[3].data(), m[3].size()}, {fn.data(), fn.size()},
                                      {m[4].data(), m[4].size()}, {m[5].data(), m[5].size()}, {m[6].data(), m[6].size()}};
            if ((rc = vox_ctx_upload_layer_bf16(ctx, l, &lw)) != VOX_OK) return rc;
        }
    }
    if (info.vocab == 0) return VOX_OK;
    std::vector<uint16_t> emb;
    if ((rc = tensor_bf16(w, VOX_CKPT_EMBED, info.vocab * dim, &emb)) != VOX_OK) return rc;
    if ((rc = vox_ctx_upload_embed_bf16(ctx, emb.data(), emb.size())) != VOX_OK) return rc;
    if (w->find(VOX_CKPT_LM_HEAD)) {  // untied head; otherwise tied to the embedding (params.rs:152)
        std::vector<uint16_t> head;
        if ((rc = tensor_bf16(w, VOX_CKPT_LM_HEAD, info.vocab * dim, &head)) != VOX_OK) return rc;
        if ((rc = vox_ctx_upload_lm_head_bf16(ctx, head.data(), head.size())) != VOX_OK) return rc;
    } else {
        if ((rc = vox_ctx_upload_lm_head_bf16(ctx, emb.data(), emb.size())) != VOX_OK) return rc;
    }
    std::vector<float> fnorm;
    if ((rc = tensor_f32(w, VOX_CKPT_FINAL_NORM, dim, &fnorm)) != VOX_OK) return rc;
    return vox_ctx_upload_final_norm(ctx, fnorm.data(), fnorm.size());
}
