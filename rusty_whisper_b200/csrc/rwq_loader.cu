// rwq_loader.cu -- whisper model files into the library's weights: the
// legacy ggml container (reference model.rs:145-275, `load_model`) and
// GGUF v2/v3 (gguf.rs:156-300, `gguf::load`), told apart by their magic
// like `load_model` does.
//
// What the reference's loader produces, this one produces too: the 11
// hyper-parameters, the mel filterbank, the byte-level vocabulary padded
// with "[_extra_token_<i>]" up to n_vocab, and every tensor under its
// whisper.cpp name -- f32 as is, f16 widened to f32, quantized blocks kept
// verbatim.  2-D quantized tensors are the matmul weights: their raw ggml
// blocks go to the GPU unchanged through `rwq_qtensor_new` the first time
// `rwq_model_qtensor` asks for them.  Quantized tensors of other ranks are
// dequantized (on the GPU, with the bit-exact dequant kernel) when
// `rwq_model_dense` asks for them, as the reference does at load time.
// Parsing itself touches no GPU.
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>
#include <cuda_runtime.h>
#include "rwq.h"
#include "rwq_common.cuh"
#include "rwq_internal.h"

struct rwq_model {
    struct Tensor {
        std::string name;
        int dtype = 0;           // 0 f32, 1 f16, else a ggml block type
        int ndims = 0;
        int64_t shape[3] = {1, 1, 1};   // row-major, last dimension fastest
        int64_t n_elems = 1;
        std::vector<uint8_t> raw;       // quantized blocks, verbatim
        std::vector<float> dense;       // f32 / f16 tensors, or dequantized on demand
        bool dense_ready = false;
        rwq_qtensor* q = nullptr;       // device weight (2-D quantized), on demand
    };
    int32_t hp[11] = {0};
    std::vector<float> mel;
    int64_t n_mel = 0, n_fft_bins = 0;
    std::vector<std::string> vocab;
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, int64_t> index;   // later tensors of a name win, like a map insert
    std::mutex mu;
    ~rwq_model() {
        for (auto& t : tensors)
            if (t.q) rwq_qtensor_free(t.q);
    }
};

namespace {

constexpr uint32_t GGML_MAGIC = 0x67676d6cu;   // "ggml"
constexpr uint32_t GGUF_MAGIC = 0x46554747u;   // "GGUF"

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    rwq::set_last_error(buf);
    return code;
}

// f16 bits -> f32, exactly (model.rs:68-86): normals, subnormals, inf, NaN.
float f16_to_f32(uint16_t h) {
    const uint32_t sign = uint32_t(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {   // subnormal: normalise
            int e = -1;
            do {
                man <<= 1;
                ++e;
            } while (!(man & 0x400u));
            bits = sign | (uint32_t(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// Little-endian cursor over the whole file with bounds checks.
struct Cursor {
    const uint8_t* p;
    size_t n, pos = 0;
    const char* what;   // "gguf" or "ggml"
    bool ok = true;
    bool have(size_t k) const { return ok && pos + k <= n && pos + k >= pos; }
    const uint8_t* take(size_t k) {
        if (!have(k)) {
            ok = false;
            return nullptr;
        }
        const uint8_t* r = p + pos;
        pos += k;
        return r;
    }
    uint32_t u32() {
        const uint8_t* b = take(4);
        return b ? uint32_t(b[0]) | uint32_t(b[1]) << 8 | uint32_t(b[2]) << 16 | uint32_t(b[3]) << 24 : 0u;
    }
    int32_t i32() { return int32_t(u32()); }
    uint64_t u64() {
        const uint64_t lo = u32(), hi = u32();
        return lo | (hi << 32);
    }
};

int truncated(const Cursor& c) { return fail(RWQ_ERR_ARG, "%s: truncated file", c.what); }

int quant_bytes(int dtype) { return rwq::block_bytes(dtype); }   // -1 if unsupported

void pad_vocab(rwq_model* m) {
    for (int64_t i = int64_t(m->vocab.size()); i < int64_t(m->hp[0]); ++i)
        m->vocab.push_back("[_extra_token_" + std::to_string(i) + "]");
}

// Decode one tensor's payload (dtype + element count known) from `data`.
int fill_tensor(rwq_model::Tensor& t, const uint8_t* data, const char* what) {
    if (t.dtype == 0) {
        t.dense.resize(size_t(t.n_elems));
        std::memcpy(t.dense.data(), data, size_t(t.n_elems) * 4);
        t.dense_ready = true;
    } else if (t.dtype == 1) {
        t.dense.resize(size_t(t.n_elems));
        for (int64_t i = 0; i < t.n_elems; ++i)
            t.dense[size_t(i)] = f16_to_f32(uint16_t(data[2 * i] | (data[2 * i + 1] << 8)));
        t.dense_ready = true;
    } else {
        const int bb = quant_bytes(t.dtype);
        t.raw.assign(data, data + size_t(t.n_elems / rwq::QK) * size_t(bb));
    }
    (void)what;
    return RWQ_OK;
}

// Bytes of a tensor's payload, or a negative status.
int64_t payload_bytes(const rwq_model::Tensor& t, const char* what) {
    if (t.dtype == 0) return t.n_elems * 4;
    if (t.dtype == 1) return t.n_elems * 2;
    const int bb = quant_bytes(t.dtype);
    if (bb < 0) return fail(RWQ_ERR_DTYPE, "%s: tensor '%s': unsupported dtype %d", what, t.name.c_str(), t.dtype);
    if (t.n_elems % rwq::QK)
        return fail(RWQ_ERR_SHAPE, "%s: tensor '%s': %lld elements not divisible by block size", what,
                    t.name.c_str(), (long long)t.n_elems);
    return t.n_elems / rwq::QK * bb;
}

void add_tensor(rwq_model* m, rwq_model::Tensor&& t) {
    m->index[t.name] = int64_t(m->tensors.size());
    m->tensors.push_back(std::move(t));
}

// ---------------------------------------------------------- legacy ggml
int load_ggml(Cursor& c, rwq_model* m) {
    for (int i = 0; i < 11; ++i) m->hp[i] = c.i32();
    const int32_t n_mel = c.i32(), n_bins = c.i32();
    if (!c.ok) return truncated(c);
    if (n_mel < 0 || n_bins < 0) return fail(RWQ_ERR_ARG, "ggml: bad mel filter shape %d x %d", n_mel, n_bins);
    const size_t nf = size_t(n_mel) * size_t(n_bins);
    const uint8_t* fb = c.take(nf * 4);
    if (!fb) return truncated(c);
    m->mel.resize(nf);
    std::memcpy(m->mel.data(), fb, nf * 4);
    m->n_mel = n_mel;
    m->n_fft_bins = n_bins;

    const int32_t n_tokens = c.i32();
    if (!c.ok) return truncated(c);
    for (int32_t i = 0; i < n_tokens; ++i) {
        const int32_t len = c.i32();
        const uint8_t* w = len >= 0 ? c.take(size_t(len)) : nullptr;
        if (!w) return len < 0 ? fail(RWQ_ERR_ARG, "ggml: negative token length") : truncated(c);
        m->vocab.emplace_back(reinterpret_cast<const char*>(w), size_t(len));
    }
    pad_vocab(m);

    // Tensors until the end of the file (a header that does not fit in
    // what is left ends the list, as an EOF on its first field does).
    while (c.have(4)) {
        rwq_model::Tensor t;
        const int32_t n_dims = c.i32(), name_len = c.i32();
        t.dtype = c.i32();
        if (!c.ok) return truncated(c);
        if (n_dims < 0 || n_dims > 3) return fail(RWQ_ERR_SHAPE, "ggml: tensor with %d dims", n_dims);
        int64_t dims[3] = {1, 1, 1};   // ggml order: fastest first
        for (int d = 0; d < n_dims; ++d) dims[d] = c.i32();
        if (name_len < 0) return fail(RWQ_ERR_ARG, "ggml: negative tensor name length");
        const uint8_t* nm = c.take(size_t(name_len));
        if (!nm) return truncated(c);
        t.name.assign(reinterpret_cast<const char*>(nm), size_t(name_len));
        t.ndims = n_dims;
        t.n_elems = dims[0] * dims[1] * dims[2];
        for (int d = 0; d < 3; ++d)
            if (dims[d] < 0) return fail(RWQ_ERR_SHAPE, "ggml: tensor '%s': negative dimension", t.name.c_str());
        const int shown = n_dims > 0 ? n_dims : 1;
        for (int d = 0; d < shown; ++d) t.shape[d] = dims[shown - 1 - d];   // reversed: row-major
        for (int d = shown; d < 3; ++d) t.shape[d] = 1;
        if (t.ndims == 0) t.ndims = 1;
        const int64_t nbytes = payload_bytes(t, "ggml");
        if (nbytes < 0) return int(nbytes);
        const uint8_t* data = c.take(size_t(nbytes));
        if (!data) return truncated(c);
        fill_tensor(t, data, "ggml");
        add_tensor(m, std::move(t));
    }
    return RWQ_OK;
}

// ------------------------------------------------------------------ GGUF
struct Value {
    enum Kind { INT, STRINGS, OTHER } kind = OTHER;
    int64_t i = 0;
    std::vector<std::string> s;
};

// One metadata value of type `t` (gguf.rs `Parser::value`): the integer
// types become integers, strings and string arrays are kept, f32/f64 and
// other arrays are skipped, anything else is an error.
int read_value(Cursor& c, uint32_t t, Value& v, int depth) {
    if (depth > 8) return fail(RWQ_ERR_ARG, "gguf: nested arrays too deep");
    switch (t) {
        case 0: case 1: {   // u8, i8 (taken as unsigned, as the reference does)
            const uint8_t* b = c.take(1);
            if (!b) return truncated(c);
            v.kind = Value::INT;
            v.i = b[0];
            return RWQ_OK;
        }
        case 2: case 3: {   // u16, i16 (sign-extended)
            const uint8_t* b = c.take(2);
            if (!b) return truncated(c);
            v.kind = Value::INT;
            v.i = int16_t(uint16_t(b[0] | (b[1] << 8)));
            return RWQ_OK;
        }
        case 4: v.kind = Value::INT; v.i = c.u32(); break;            // u32
        case 5: v.kind = Value::INT; v.i = c.i32(); break;            // i32
        case 6: if (!c.take(4)) return truncated(c); v.kind = Value::OTHER; return RWQ_OK;   // f32
        case 7: {   // bool
            const uint8_t* b = c.take(1);
            if (!b) return truncated(c);
            v.kind = Value::INT;
            v.i = b[0];
            return RWQ_OK;
        }
        case 8: {   // string
            const uint64_t len = c.u64();
            const uint8_t* b = c.ok ? c.take(size_t(len)) : nullptr;
            if (!b) return truncated(c);
            v.kind = Value::STRINGS;
            v.s.assign(1, std::string(reinterpret_cast<const char*>(b), size_t(len)));
            return RWQ_OK;
        }
        case 9: {   // array
            const uint32_t et = c.u32();
            const uint64_t n = c.u64();
            if (!c.ok) return truncated(c);
            if (et == 8) {
                v.kind = Value::STRINGS;
                v.s.clear();
                for (uint64_t k = 0; k < n; ++k) {
                    const uint64_t len = c.u64();
                    const uint8_t* b = c.ok ? c.take(size_t(len)) : nullptr;
                    if (!b) return truncated(c);
                    v.s.emplace_back(reinterpret_cast<const char*>(b), size_t(len));
                }
            } else {
                for (uint64_t k = 0; k < n; ++k) {
                    Value e;
                    const int rc = read_value(c, et, e, depth + 1);
                    if (rc) return rc;
                }
                v.kind = Value::OTHER;
            }
            return RWQ_OK;
        }
        case 10: case 11: v.kind = Value::INT; v.i = int64_t(c.u64()); break;   // u64, i64
        case 12: if (!c.take(8)) return truncated(c); v.kind = Value::OTHER; return RWQ_OK;   // f64
        default: return fail(RWQ_ERR_ARG, "gguf: unknown metadata type %u", t);
    }
    return c.ok ? RWQ_OK : truncated(c);
}

const char* const HPARAM_KEYS[11] = {
    "whisper.n_vocab",     "whisper.n_audio_ctx",  "whisper.n_audio_state", "whisper.n_audio_head",
    "whisper.n_audio_layer", "whisper.n_text_ctx", "whisper.n_text_state",  "whisper.n_text_head",
    "whisper.n_text_layer", "whisper.n_mels",      "whisper.ftype"};

int load_gguf(Cursor& c, rwq_model* m) {
    const uint32_t version = c.u32();
    const uint64_t n_tensors = c.u64(), n_kv = c.u64();
    if (!c.ok) return truncated(c);
    if (version < 2 || version > 3) return fail(RWQ_ERR_ARG, "gguf: unsupported version %u", version);
    std::unordered_map<std::string, int64_t> ints;
    std::vector<std::string> tokens;
    uint64_t alignment = 32;
    for (uint64_t k = 0; k < n_kv; ++k) {
        const uint64_t klen = c.u64();
        const uint8_t* kb = c.ok ? c.take(size_t(klen)) : nullptr;
        if (!kb) return truncated(c);
        const std::string key(reinterpret_cast<const char*>(kb), size_t(klen));
        const uint32_t t = c.u32();
        if (!c.ok) return truncated(c);
        Value v;
        const int rc = read_value(c, t, v, 0);
        if (rc) return rc;
        if (v.kind == Value::INT) {
            if (key == "general.alignment") alignment = uint64_t(v.i);
            ints[key] = v.i;
        } else if (v.kind == Value::STRINGS) {
            if (key == "tokenizer.ggml.tokens") {
                tokens = std::move(v.s);
            } else if (key == "general.architecture" && (v.s.empty() || v.s[0] != "whisper")) {
                return fail(RWQ_ERR_ARG, "gguf: general.architecture is not \"whisper\"");
            }
        }
    }
    if (alignment == 0) return fail(RWQ_ERR_ARG, "gguf: general.alignment is 0");
    for (int i = 0; i < 11; ++i) {
        auto it = ints.find(HPARAM_KEYS[i]);
        if (it == ints.end()) return fail(RWQ_ERR_ARG, "gguf: missing metadata key %s", HPARAM_KEYS[i]);
        m->hp[i] = int32_t(it->second);
    }

    struct Info {
        rwq_model::Tensor t;
        uint64_t offset;
    };
    std::vector<Info> infos;
    for (uint64_t k = 0; k < n_tensors; ++k) {
        Info in;
        const uint64_t nlen = c.u64();
        const uint8_t* nb = c.ok ? c.take(size_t(nlen)) : nullptr;
        if (!nb) return truncated(c);
        in.t.name.assign(reinterpret_cast<const char*>(nb), size_t(nlen));
        const uint32_t n_dims = c.u32();
        if (!c.ok) return truncated(c);
        if (n_dims > 3) return fail(RWQ_ERR_SHAPE, "gguf: tensor '%s' has %u dims", in.t.name.c_str(), n_dims);
        uint64_t ne[3] = {1, 1, 1};
        for (uint32_t d = 0; d < n_dims; ++d) ne[d] = c.u64();
        in.t.dtype = int32_t(c.u32());
        in.offset = c.u64();
        if (!c.ok) return truncated(c);
        in.t.ndims = n_dims ? int(n_dims) : 1;
        in.t.n_elems = 1;
        for (uint32_t d = 0; d < n_dims; ++d) {
            if (ne[d] > (uint64_t(1) << 40)) return fail(RWQ_ERR_SHAPE, "gguf: tensor '%s' too large", in.t.name.c_str());
            in.t.shape[d] = int64_t(ne[n_dims - 1 - d]);   // reversed: row-major
            in.t.n_elems *= int64_t(ne[d]);
        }
        infos.push_back(std::move(in));
    }
    tokens.swap(m->vocab);
    pad_vocab(m);

    // The data section starts at the next multiple of the alignment,
    // counted from the start of the file.
    const uint64_t data_start = (uint64_t(c.pos) + alignment - 1) / alignment * alignment;
    for (auto& in : infos) {
        const int64_t nbytes = payload_bytes(in.t, "gguf");
        if (nbytes < 0) return int(nbytes);
        const uint64_t start = data_start + in.offset;
        if (start < data_start || start > c.n || uint64_t(nbytes) > c.n - start)
            return fail(RWQ_ERR_ARG, "gguf: tensor '%s' out of bounds", in.t.name.c_str());
        fill_tensor(in.t, c.p + start, "gguf");
        if (in.t.name == "whisper.mel_filters") {
            if (!in.t.dense_ready)
                return fail(RWQ_ERR_DTYPE, "gguf: whisper.mel_filters must be f32 or f16");
            m->mel = in.t.dense;
            m->n_mel = in.t.ndims >= 2 ? in.t.shape[0] : 1;
            m->n_fft_bins = in.t.ndims >= 2 ? in.t.shape[1] : in.t.shape[0];
        } else {
            add_tensor(m, std::move(in.t));
        }
    }
    return RWQ_OK;
}

const rwq_model::Tensor* tensor_at(const rwq_model* m, int64_t i) {
    if (!m || i < 0 || i >= int64_t(m->tensors.size())) return nullptr;
    return &m->tensors[size_t(i)];
}

}  // namespace

extern "C" {

int rwq_model_load(const char* path, rwq_model** out) {
    if (!out) return fail(RWQ_ERR_ARG, "out is null");
    *out = nullptr;
    if (!path) return fail(RWQ_ERR_ARG, "path is null");
    FILE* f = std::fopen(path, "rb");
    if (!f) return fail(RWQ_ERR_ARG, "cannot open %s", path);
    std::vector<uint8_t> buf;
    uint8_t chunk[1 << 16];
    size_t got;
    while ((got = std::fread(chunk, 1, sizeof chunk, f)) > 0) buf.insert(buf.end(), chunk, chunk + got);
    const bool err = std::ferror(f) != 0;
    std::fclose(f);
    if (err) return fail(RWQ_ERR_ARG, "read error on %s", path);
    return rwq_model_load_memory(buf.data(), buf.size(), out);
}

int rwq_model_load_memory(const uint8_t* data, size_t len, rwq_model** out) {
    if (!out) return fail(RWQ_ERR_ARG, "out is null");
    *out = nullptr;
    if (!data && len) return fail(RWQ_ERR_ARG, "data is null");
    Cursor c{data, len};
    c.what = "model";
    const uint32_t magic = c.u32();
    if (!c.ok) return fail(RWQ_ERR_ARG, "model file shorter than its magic");
    std::unique_ptr<rwq_model> m(new rwq_model);
    int rc;
    if (magic == GGUF_MAGIC) {
        c.what = "gguf";
        rc = load_gguf(c, m.get());
    } else if (magic == GGML_MAGIC) {
        c.what = "ggml";
        rc = load_ggml(c, m.get());
    } else {
        return fail(RWQ_ERR_ARG, "bad magic %#x, expected 'ggml' (%#x) or 'GGUF' (%#x)", magic, GGML_MAGIC,
                    GGUF_MAGIC);
    }
    if (rc) return rc;
    *out = m.release();
    return RWQ_OK;
}

int rwq_model_free(rwq_model* m) {
    delete m;
    return RWQ_OK;
}

int rwq_model_hparams(const rwq_model* m, int32_t* out11) {
    if (!m || !out11) return fail(RWQ_ERR_ARG, "null argument");
    std::memcpy(out11, m->hp, sizeof m->hp);
    return RWQ_OK;
}

int rwq_model_mel_filters(const rwq_model* m, const float** data, int64_t* n_mel, int64_t* n_fft_bins) {
    if (!m || !data || !n_mel || !n_fft_bins) return fail(RWQ_ERR_ARG, "null argument");
    *data = m->mel.empty() ? nullptr : m->mel.data();
    *n_mel = m->n_mel;
    *n_fft_bins = m->n_fft_bins;
    return RWQ_OK;
}

int rwq_model_vocab_size(const rwq_model* m, int64_t* n) {
    if (!m || !n) return fail(RWQ_ERR_ARG, "null argument");
    *n = int64_t(m->vocab.size());
    return RWQ_OK;
}

int rwq_model_token(const rwq_model* m, int64_t id, const char** bytes, int64_t* len) {
    if (!m || !bytes || !len) return fail(RWQ_ERR_ARG, "null argument");
    if (id < 0 || id >= int64_t(m->vocab.size()))
        return fail(RWQ_ERR_ARG, "token id %lld out of range [0, %zu)", (long long)id, m->vocab.size());
    *bytes = m->vocab[size_t(id)].data();
    *len = int64_t(m->vocab[size_t(id)].size());
    return RWQ_OK;
}

int rwq_model_n_tensors(const rwq_model* m, int64_t* n) {
    if (!m || !n) return fail(RWQ_ERR_ARG, "null argument");
    *n = int64_t(m->tensors.size());
    return RWQ_OK;
}

int rwq_model_find(const rwq_model* m, const char* name, int64_t* index) {
    if (!m || !name || !index) return fail(RWQ_ERR_ARG, "null argument");
    auto it = m->index.find(name);
    if (it == m->index.end()) return fail(RWQ_ERR_ARG, "no tensor named '%s'", name);
    *index = it->second;
    return RWQ_OK;
}

int rwq_model_tensor(const rwq_model* m, int64_t i, const char** name, int* dtype, int* ndims, int64_t* shape3) {
    const rwq_model::Tensor* t = tensor_at(m, i);
    if (!t) return fail(RWQ_ERR_ARG, "tensor index %lld out of range", (long long)i);
    if (name) *name = t->name.c_str();
    if (dtype) *dtype = t->dtype;
    if (ndims) *ndims = t->ndims;
    if (shape3)
        for (int d = 0; d < 3; ++d) shape3[d] = t->shape[d];
    return RWQ_OK;
}

int rwq_model_tensor_raw(const rwq_model* m, int64_t i, const uint8_t** data, size_t* len) {
    const rwq_model::Tensor* t = tensor_at(m, i);
    if (!t) return fail(RWQ_ERR_ARG, "tensor index %lld out of range", (long long)i);
    if (!data || !len) return fail(RWQ_ERR_ARG, "null argument");
    if (t->dtype == 0 || t->dtype == 1) return fail(RWQ_ERR_DTYPE, "tensor '%s' is not quantized", t->name.c_str());
    *data = t->raw.data();
    *len = t->raw.size();
    return RWQ_OK;
}

int rwq_model_qtensor(rwq_model* m, int64_t i, rwq_qtensor** out) {
    if (!out) return fail(RWQ_ERR_ARG, "out is null");
    *out = nullptr;
    if (!tensor_at(m, i)) return fail(RWQ_ERR_ARG, "tensor index %lld out of range", (long long)i);
    std::lock_guard<std::mutex> g(m->mu);
    rwq_model::Tensor& t = m->tensors[size_t(i)];
    if (t.dtype == 0 || t.dtype == 1 || t.ndims != 2)
        return fail(RWQ_ERR_DTYPE, "tensor '%s' is not a 2-D quantized weight", t.name.c_str());
    if (!t.q) {
        const int rc = rwq_qtensor_new(t.raw.data(), t.raw.size(), t.dtype, t.shape[0], t.shape[1], &t.q);
        if (rc) return rc;
    }
    *out = t.q;
    return RWQ_OK;
}

int rwq_model_dense(rwq_model* m, int64_t i, const float** data, int64_t* n) {
    if (!data || !n) return fail(RWQ_ERR_ARG, "null argument");
    if (!tensor_at(m, i)) return fail(RWQ_ERR_ARG, "tensor index %lld out of range", (long long)i);
    std::lock_guard<std::mutex> g(m->mu);
    rwq_model::Tensor& t = m->tensors[size_t(i)];
    if (!t.dense_ready) {
        if (t.ndims == 2)
            return fail(RWQ_ERR_DTYPE, "tensor '%s' is a quantized matmul weight (use rwq_model_qtensor)",
                        t.name.c_str());
        // Other quantized tensors become f32 (quant.rs `to_dense`), one
        // 32-element block per row of the bit-exact dequant kernel.
        const int64_t rows = t.n_elems / rwq::QK;
        rwq_qtensor* q = nullptr;
        int rc = rwq_qtensor_new(t.raw.data(), t.raw.size(), t.dtype, rows, rwq::QK, &q);
        if (rc) return rc;
        float* dev = nullptr;
        cudaError_t e = cudaMalloc(&dev, size_t(t.n_elems) * 4);
        if (e == cudaSuccess) {
            rc = rwq_dequant_rows_dev(q, nullptr, rows, dev, nullptr);
            if (!rc) {
                t.dense.resize(size_t(t.n_elems));
                e = cudaMemcpy(t.dense.data(), dev, size_t(t.n_elems) * 4, cudaMemcpyDeviceToHost);
            }
            cudaFree(dev);
        }
        rwq_qtensor_free(q);
        if (rc) return rc;
        if (e != cudaSuccess) return fail(RWQ_ERR_CUDA, "dequantize '%s': %s", t.name.c_str(), cudaGetErrorString(e));
        t.dense_ready = true;
    }
    *data = t.dense.data();
    *n = t.n_elems;
    return RWQ_OK;
}

}  // extern "C"
