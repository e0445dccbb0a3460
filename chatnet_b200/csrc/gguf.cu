// gguf.cu -- host side: GGUF files into HBM.
//
//   cn_gguf_open     GgufReader.Load (Gguf/GgufReader.cs:34-75) + the mapping of
//                    MemoryMappedWeights (Memory/MemoryMappedWeights.cs:23-40):
//                    magic, version 2 or 3, metadata key/values, tensor
//                    descriptors, the data section at the next multiple of
//                    general.alignment (default 32); the file is mapped
//                    read-only and tensor bytes are read in place
//   cn_gguf_llama_config   GgufReader.ExtractModelConfig (GgufReader.cs:80-176) for
//                    the fields a Llama decoder needs
//   cn_gguf_upload   one tensor, byte for byte, onto the device (cn_tensor_upload)
//   cn_llama_create_from_gguf   LlamaWeights.ResolveAll (Models/Llama/LlamaWeights.cs:
//                    78-145) in cn_llama_create order, output.weight falling back to
//                    token_embd.weight, then cn_llama_create
//
// Byte sizes follow GgufTensorInfo.ByteSize (Gguf/GgufTensorInfo.cs:30-114)
// through cn_byte_size.  Errors map as the reader's exceptions do: a bad magic,
// version or truncated header is CN_ERR_INVALID_ARG, a missing tensor
// CN_ERR_NOT_FOUND, an architecture without a Llama decoder CN_ERR_UNSUPPORTED.
#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <new>
#include <string>
#include <unordered_map>
#include <vector>

#include "cn_common.cuh"
#include "cn_internal.h"

namespace {

// GGUF metadata value types (GgufConstants.cs)
enum : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7,
    kStr = 8, kArr = 9, kU64 = 10, kI64 = 11, kF64 = 12
};
constexpr uint32_t kMagic = 0x46554747u;  // "GGUF", little-endian
constexpr int kDefaultAlignment = 32;

struct Value {
    uint32_t type = 0;
    int64_t i = 0;       // integer and bool types
    double f = 0.0;      // float types
    std::string s;       // strings
    uint32_t arr_type = 0;
    uint64_t arr_len = 0;
};

struct Tensor {
    std::string name;
    int type = 0;
    int n_dims = 0;
    uint64_t dims[4] = {1, 1, 1, 1};
    uint64_t offset = 0;  // from the start of the data section
    uint64_t bytes = 0;
};

// Little-endian cursor over the mapped file; any read past the end marks it bad.
struct Cursor {
    const uint8_t* p;
    uint64_t size, pos = 0;
    bool bad = false;
    bool take(void* dst, uint64_t n) {
        if (bad || n > size - pos) {
            bad = true;
            return false;
        }
        memcpy(dst, p + pos, n);
        pos += n;
        return true;
    }
    template <typename T>
    T get() {
        T v{};
        take(&v, sizeof(T));
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (bad || n > size - pos) {
            bad = true;
            return std::string();
        }
        std::string s(reinterpret_cast<const char*>(p + pos), n);
        pos += n;
        return s;
    }
};

bool read_scalar(Cursor& c, uint32_t type, Value& v) {
    v.type = type;
    switch (type) {
        case kU8: v.i = c.get<uint8_t>(); break;
        case kI8: v.i = c.get<int8_t>(); break;
        case kU16: v.i = c.get<uint16_t>(); break;
        case kI16: v.i = c.get<int16_t>(); break;
        case kU32: v.i = c.get<uint32_t>(); break;
        case kI32: v.i = c.get<int32_t>(); break;
        case kF32: v.f = c.get<float>(); break;
        case kBool: v.i = c.get<uint8_t>() != 0; break;
        case kStr: v.s = c.str(); break;
        case kU64: v.i = (int64_t)c.get<uint64_t>(); break;
        case kI64: v.i = c.get<int64_t>(); break;
        case kF64: v.f = c.get<double>(); break;
        default: return false;
    }
    return !c.bad;
}

bool read_value(Cursor& c, uint32_t type, Value& v) {
    if (type != kArr) return read_scalar(c, type, v);
    // arrays (GgufReader.ReadArray): element type, length, elements; only the
    // element type and length are kept (string arrays: the vocabulary)
    v.type = kArr;
    v.arr_type = c.get<uint32_t>();
    v.arr_len = c.get<uint64_t>();
    for (uint64_t i = 0; i < v.arr_len && !c.bad; i++) {
        Value e;
        if (!read_value(c, v.arr_type, e)) return false;
    }
    return !c.bad;
}

}  // namespace

struct cn_gguf {
    int fd = -1;
    void* map = nullptr;
    uint64_t size = 0;
    uint32_t version = 0;
    int alignment = kDefaultAlignment;
    uint64_t data_off = 0;
    std::unordered_map<std::string, Value> meta;
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, int> index;
};

namespace cn {

static void gguf_free(cn_gguf* g) {
    if (!g) return;
    if (g->map && g->map != MAP_FAILED) munmap(g->map, g->size);
    if (g->fd >= 0) close(g->fd);
    delete g;
}

static const Value* meta_get(const cn_gguf* g, const std::string& key) {
    auto it = g->meta.find(key);
    return it == g->meta.end() ? nullptr : &it->second;
}

static bool is_int(const Value* v) {
    return v && (v->type == kU8 || v->type == kI8 || v->type == kU16 || v->type == kI16 || v->type == kU32 ||
                 v->type == kI32 || v->type == kU64 || v->type == kI64 || v->type == kBool);
}

// GgufMetadata.GetInt32 semantics (Gguf/GgufMetadata.cs:53-63): only int32,
// uint32, int64 and uint64 values count (other integer widths give the
// default), and the value is cast to a 32-bit int the way C#'s unchecked
// (int) cast does -- the low 32 bits, so a uint32 0xFFFFFFFF reads as -1.
static int64_t meta_int(const cn_gguf* g, const std::string& key, int64_t def) {
    const Value* v = meta_get(g, key);
    if (!v || !(v->type == kU32 || v->type == kI32 || v->type == kU64 || v->type == kI64)) return def;
    return (int64_t)(int32_t)(uint32_t)(uint64_t)v->i;
}

// One key's part of ExtractModelConfig.GetArchFloat (Gguf/GgufReader.cs:93-108):
// a float, a double, a uint32 or an int32 value, in that order of type tests;
// any other type (other integer widths, bool) does not count.
static bool meta_float(const cn_gguf* g, const std::string& key, double* out) {
    const Value* v = meta_get(g, key);
    if (!v) return false;
    if (v->type == kF32 || v->type == kF64) {
        *out = v->f;
        return true;
    }
    if (v->type == kU32) {
        *out = (double)(uint32_t)(uint64_t)v->i;
        return true;
    }
    if (v->type == kI32) {
        *out = (double)(int32_t)v->i;
        return true;
    }
    return false;
}

}  // namespace cn

using namespace cn;

extern "C" {

int cn_gguf_open(const char* path, cn_gguf** out) {
    CN_CHECK(path && out, CN_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    cn_gguf* g = new (std::nothrow) cn_gguf();
    CN_CHECK(g, CN_ERR_OOM, "host allocation failed");
    g->fd = open(path, O_RDONLY);
    if (g->fd < 0) {
        gguf_free(g);
        return set_error(CN_ERR_NOT_FOUND, "cannot open GGUF file %s", path);
    }
    struct stat st;
    if (fstat(g->fd, &st) != 0 || st.st_size < 24) {
        gguf_free(g);
        return set_error(CN_ERR_INVALID_ARG, "%s: not a GGUF file (too short)", path);
    }
    g->size = (uint64_t)st.st_size;
    g->map = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (g->map == MAP_FAILED) {
        g->map = nullptr;
        gguf_free(g);
        return set_error(CN_ERR_INVALID_ARG, "%s: mmap failed", path);
    }
    Cursor c{static_cast<const uint8_t*>(g->map), g->size};
    const uint32_t magic = c.get<uint32_t>();
    if (magic != kMagic) {
        gguf_free(g);
        return set_error(CN_ERR_INVALID_ARG, "Invalid GGUF magic: 0x%08X, expected 0x%08X", magic, kMagic);
    }
    g->version = c.get<uint32_t>();
    if (g->version < 2 || g->version > 3) {
        const uint32_t v = g->version;
        gguf_free(g);
        return set_error(CN_ERR_INVALID_ARG, "Unsupported GGUF version: %u", v);
    }
    const uint64_t n_tensors = c.get<uint64_t>();
    const uint64_t n_kv = c.get<uint64_t>();
    for (uint64_t i = 0; i < n_kv && !c.bad; i++) {
        std::string key = c.str();
        const uint32_t type = c.get<uint32_t>();
        Value v;
        if (!read_value(c, type, v)) {
            gguf_free(g);
            return set_error(CN_ERR_INVALID_ARG, "%s: bad metadata value (key '%s', type %u)", path, key.c_str(),
                             type);
        }
        g->meta[key] = v;
    }
    g->alignment = (int)meta_int(g, "general.alignment", kDefaultAlignment);
    if (g->alignment <= 0 || (g->alignment & (g->alignment - 1)) != 0) g->alignment = kDefaultAlignment;
    for (uint64_t i = 0; i < n_tensors && !c.bad; i++) {
        Tensor t;
        t.name = c.str();
        const uint32_t nd = c.get<uint32_t>();
        if (nd > 4) {
            gguf_free(g);
            return set_error(CN_ERR_INVALID_ARG, "%s: tensor '%s' has %u dimensions", path, t.name.c_str(), nd);
        }
        t.n_dims = (int)nd;
        uint64_t elems = nd ? 1 : 0;
        bool overflow = false;
        for (uint32_t d = 0; d < nd; d++) {
            t.dims[d] = c.get<uint64_t>();
            overflow |= __builtin_mul_overflow(elems, t.dims[d], &elems);
        }
        // no real tensor comes near 2^56 elements; past that the byte size
        // (up to 4 bytes per element) could wrap around
        if (overflow || elems >= (1ull << 56)) {
            const std::string name = t.name;
            gguf_free(g);
            return set_error(CN_ERR_INVALID_ARG, "%s: tensor '%s' has too many elements", path, name.c_str());
        }
        t.type = (int)c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
        t.bytes = cn_byte_size(t.type, elems);
        g->index[t.name] = (int)g->tensors.size();
        g->tensors.push_back(t);
    }
    if (c.bad) {
        gguf_free(g);
        return set_error(CN_ERR_INVALID_ARG, "%s: truncated GGUF header", path);
    }
    const uint64_t mask = (uint64_t)g->alignment - 1;
    g->data_off = (c.pos + mask) & ~mask;
    for (const Tensor& t : g->tensors) {
        if (t.bytes == 0 && t.n_dims > 0 && t.type != CN_TYPE_F32) continue;  // a type without a byte size
        uint64_t start = 0;
        if (__builtin_add_overflow(g->data_off, t.offset, &start) || start > g->size ||
            t.bytes > g->size - start) {
            const std::string name = t.name;
            gguf_free(g);
            return set_error(CN_ERR_INVALID_ARG, "%s: tensor '%s' runs past the end of the file", path,
                             name.c_str());
        }
    }
    *out = g;
    return CN_OK;
}

int cn_gguf_close(cn_gguf* g) {
    gguf_free(g);
    return CN_OK;
}

int cn_gguf_tensor_count(const cn_gguf* g, int* n) {
    CN_CHECK(g && n, CN_ERR_INVALID_ARG, "null argument");
    *n = (int)g->tensors.size();
    return CN_OK;
}

int cn_gguf_tensor_info(const cn_gguf* g, int i, const char** name, int* type, int* n_dims, uint64_t* dims,
                        uint64_t* bytes, uint64_t* file_offset) {
    CN_CHECK(g, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK(i >= 0 && i < (int)g->tensors.size(), CN_ERR_INVALID_ARG, "tensor index %d out of range", i);
    const Tensor& t = g->tensors[i];
    if (name) *name = t.name.c_str();
    if (type) *type = t.type;
    if (n_dims) *n_dims = t.n_dims;
    if (dims)
        for (int d = 0; d < 4; d++) dims[d] = t.dims[d];
    if (bytes) *bytes = t.bytes;
    if (file_offset) *file_offset = g->data_off + t.offset;
    return CN_OK;
}

int cn_gguf_find(const cn_gguf* g, const char* name, int* index) {
    CN_CHECK(g && name && index, CN_ERR_INVALID_ARG, "null argument");
    auto it = g->index.find(name);
    CN_CHECK(it != g->index.end(), CN_ERR_NOT_FOUND, "Tensor not found: %s", name);
    *index = it->second;
    return CN_OK;
}

int cn_gguf_get_int(const cn_gguf* g, const char* key, int64_t* out) {
    CN_CHECK(g && key && out, CN_ERR_INVALID_ARG, "null argument");
    const Value* v = meta_get(g, key);
    CN_CHECK(v, CN_ERR_NOT_FOUND, "metadata key not found: %s", key);
    CN_CHECK(is_int(v), CN_ERR_INVALID_ARG, "metadata key %s is not an integer", key);
    *out = v->i;
    return CN_OK;
}

int cn_gguf_get_float(const cn_gguf* g, const char* key, double* out) {
    CN_CHECK(g && key && out, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK(meta_get(g, key), CN_ERR_NOT_FOUND, "metadata key not found: %s", key);
    CN_CHECK(meta_float(g, key, out), CN_ERR_INVALID_ARG, "metadata key %s is not a number", key);
    return CN_OK;
}

int cn_gguf_get_string(const cn_gguf* g, const char* key, const char** out) {
    CN_CHECK(g && key && out, CN_ERR_INVALID_ARG, "null argument");
    const Value* v = meta_get(g, key);
    CN_CHECK(v, CN_ERR_NOT_FOUND, "metadata key not found: %s", key);
    CN_CHECK(v->type == kStr, CN_ERR_INVALID_ARG, "metadata key %s is not a string", key);
    *out = v->s.c_str();
    return CN_OK;
}

int cn_gguf_llama_config(const cn_gguf* g, cn_llama_config* cfg) {
    CN_CHECK(g && cfg, CN_ERR_INVALID_ARG, "null argument");
    const Value* av = meta_get(g, "general.architecture");
    const std::string arch = av && av->type == kStr ? av->s : std::string("llama");
    // ModelFactory.DetectArchitecture (Models/ModelFactory.cs:23-39): these have
    // their own decoders in the reference; anything unknown is run as Llama
    for (const char* other : {"qwen2", "qwen", "mistral", "gemma", "gemma2", "phi2", "phi3", "phi"})
        CN_CHECK(arch != other, CN_ERR_UNSUPPORTED, "architecture '%s' has no Llama decoder here", arch.c_str());
    auto arch_int = [&](const char* suffix, int64_t def) {
        const int64_t v = meta_int(g, arch + "." + suffix, -1);
        return v >= 0 ? v : meta_int(g, suffix, def);
    };
    auto arch_float = [&](const char* suffix, double def) {
        double v;
        if (meta_float(g, arch + "." + suffix, &v) || meta_float(g, suffix, &v)) return v;
        return def;
    };
    cn_llama_config c = {};
    c.n_heads = (int)arch_int("attention.head_count", 32);
    c.n_kv_heads = (int)arch_int("attention.head_count_kv", c.n_heads);
    c.dim = (int)arch_int("embedding_length", 2048);
    c.n_layers = (int)arch_int("block_count", 22);
    c.hidden_dim = (int)arch_int("feed_forward_length", 5632);
    c.ctx_len = (int)arch_int("context_length", 2048);
    c.rope_base = (float)arch_float("rope.freq_base", 10000.0);
    c.rms_eps = (float)arch_float("attention.layer_norm_rms_epsilon", 1e-5);
    const int64_t key_len = arch_int("attention.key_length", -1);
    c.head_dim = key_len > 0 ? (int)key_len : (c.n_heads > 0 ? c.dim / c.n_heads : 0);
    // vocabulary: the token array's length, else <arch>.vocab_size, else 32000
    const Value* tok = meta_get(g, "tokenizer.ggml.tokens");
    c.vocab = tok && tok->type == kArr && tok->arr_type == kStr ? (int)tok->arr_len : (int)arch_int("vocab_size", 32000);
    c.kv_dtype = CN_KV_F32;
    c.max_batch = 1;
    *cfg = c;
    return CN_OK;
}

// [rows, cols] of a GGUF tensor: cols = ne[0] (innermost), rows = the rest.
static void tensor_shape(const Tensor& t, int64_t* rows, int64_t* cols) {
    *cols = (int64_t)t.dims[0];
    int64_t r = 1;
    for (int d = 1; d < t.n_dims; d++) r *= (int64_t)t.dims[d];
    *rows = t.n_dims > 0 ? r : 0;
}

int cn_gguf_upload(cn_ctx* ctx, const cn_gguf* g, const char* name, cn_tensor** out) {
    CN_CHECK(ctx && g && name && out, CN_ERR_INVALID_ARG, "null argument");
    int idx = 0;
    int rc = cn_gguf_find(g, name, &idx);
    if (rc) return rc;
    const Tensor& t = g->tensors[idx];
    CN_CHECK(type_supported(t.type), CN_ERR_UNSUPPORTED, "tensor %s: ggml type %d not supported", name, t.type);
    int64_t rows, cols;
    tensor_shape(t, &rows, &cols);
    const uint8_t* src = static_cast<const uint8_t*>(g->map) + g->data_off + t.offset;
    return cn_tensor_upload(ctx, src, t.bytes, t.type, rows, cols, out);
}

// Region of tensor `name` ([rows, cols]) that tensor-parallel rank r of
// `size` holds: rows of q/k/v/gate/up/lm_head (heads, FFN rows, vocabulary),
// columns of O/down (their input), everything else whole.
static void shard_region(const char* name, int64_t rows, int64_t cols, int r, int size, int64_t* row0,
                         int64_t* nrows, int64_t* col0, int64_t* ncols) {
    *row0 = 0;
    *nrows = rows;
    *col0 = 0;
    *ncols = cols;
    const std::string n(name);
    if (size <= 1 || n == "token_embd.weight" || n.size() >= 11 && n.compare(n.size() - 11, 11, "norm.weight") == 0)
        return;
    if (n.find(".attn_output.") != std::string::npos || n.find(".ffn_down.") != std::string::npos) {
        *ncols = cols / size;
        *col0 = (int64_t)r * *ncols;
        return;
    }
    *nrows = rows / size;
    *row0 = (int64_t)r * *nrows;
}

static int create_from_gguf(cn_ctx* ctx, const cn_gguf* g, cn_tp* tp, int max_batch, int kv_dtype, cn_llama** out,
                            cn_tensor** tensors_out, int n_tensors_out) {
    CN_CHECK(ctx && g && out && tensors_out, CN_ERR_INVALID_ARG, "null argument");
    cn_llama_config c;
    int rc = cn_gguf_llama_config(g, &c);
    if (rc) return rc;
    c.max_batch = max_batch;
    c.kv_dtype = kv_dtype;
    const int n = CN_LLAMA_TENSORS(c.n_layers);
    CN_CHECK(n_tensors_out >= n, CN_ERR_INVALID_ARG, "tensors_out holds %d, the model needs %d", n_tensors_out, n);
    static const char* kLayer[9] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                                    "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};
    std::vector<std::string> names;
    names.push_back("token_embd.weight");
    names.push_back("output.weight");
    names.push_back("output_norm.weight");
    for (int l = 0; l < c.n_layers; l++)
        for (const char* k : kLayer) names.push_back("blk." + std::to_string(l) + "." + k + ".weight");
    std::vector<cn_tensor*> ts(n, nullptr);
    auto release = [&]() {
        for (int i = 0; i < n; i++)
            if (ts[i] && !(i == 1 && ts[1] == ts[0])) cn_tensor_free(ts[i]);
    };
    const int size = tp ? tp->size : 1, rank = tp ? tp->rank : 0;
    if (size > 1)
        CN_CHECK(c.n_kv_heads % size == 0 && c.hidden_dim % size == 0 && c.vocab % size == 0 &&
                     c.dim % (256 * size) == 0 && c.hidden_dim % (256 * size) == 0,
                 CN_ERR_INVALID_ARG,
                 "the model does not shard over %d ranks (kv heads, hidden_dim and vocab must divide, and O/down "
                 "inputs must split into whole 256-weight blocks)", size);
    for (int i = 0; i < n; i++) {
        int idx;
        const bool tied = i == 1 && cn_gguf_find(g, names[i].c_str(), &idx) != CN_OK;
        if (tied && size == 1) {
            ts[1] = ts[0];  // tied lm_head (LlamaWeights.cs:89-98)
            continue;
        }
        // a tied lm_head under tensor parallelism: this rank's vocabulary rows of token_embd
        const char* nm = tied ? "token_embd.weight" : names[i].c_str();
        if (size == 1) {
            rc = cn_gguf_upload(ctx, g, nm, &ts[i]);
        } else {
            if ((rc = cn_gguf_find(g, nm, &idx))) {
                release();
                return rc;
            }
            const Tensor& t = g->tensors[idx];
            if (!type_supported(t.type)) {
                release();
                return set_error(CN_ERR_UNSUPPORTED, "tensor %s: ggml type %d not supported", nm, t.type);
            }
            int64_t rows, cols, r0, nr, c0, nc;
            tensor_shape(t, &rows, &cols);
            shard_region(names[i].c_str(), rows, cols, rank, size, &r0, &nr, &c0, &nc);
            const uint8_t* src = static_cast<const uint8_t*>(g->map) + g->data_off + t.offset;
            rc = cn_tensor_upload_slice(ctx, src, t.bytes, t.type, rows, cols, r0, nr, c0, nc, &ts[i]);
        }
        if (rc) {
            release();
            return rc;
        }
    }
    rc = tp ? cn_llama_create_tp(ctx, &c, ts.data(), n, tp, out) : cn_llama_create(ctx, &c, ts.data(), n, out);
    if (rc) {
        release();
        return rc;
    }
    for (int i = 0; i < n; i++) tensors_out[i] = ts[i];
    return CN_OK;
}

int cn_llama_create_from_gguf(cn_ctx* ctx, const cn_gguf* g, int max_batch, int kv_dtype, cn_llama** out,
                              cn_tensor** tensors_out, int n_tensors_out) {
    return create_from_gguf(ctx, g, nullptr, max_batch, kv_dtype, out, tensors_out, n_tensors_out);
}

int cn_llama_create_from_gguf_tp(cn_ctx* ctx, const cn_gguf* g, cn_tp* tp, int max_batch, int kv_dtype,
                                 cn_llama** out, cn_tensor** tensors_out, int n_tensors_out) {
    CN_CHECK(tp, CN_ERR_INVALID_ARG, "null tensor-parallel group");
    return create_from_gguf(ctx, g, tp, max_batch, kv_dtype, out, tensors_out, n_tensors_out);
}

}  // extern "C"
