// gguf_file.cpp -- see gguf_file.hpp.
#include "gguf_file.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <limits>

namespace hesa_gguf {

namespace {

constexpr uint32_t kMagic = 0x46554747u;        // "GGUF", little-endian
constexpr uint64_t kMaxCount = uint64_t(1) << 32;
constexpr int kMaxDepth = 8;

bool read_bytes(const uint8_t* d, size_t n, size_t& off, void* out, size_t len) {
    if (off > n || len > n - off) return false;
    std::memcpy(out, d + off, len);
    off += len;
    return true;
}

template <typename T>
bool read_pod(const uint8_t* d, size_t n, size_t& off, T& out) {
    return read_bytes(d, n, off, &out, sizeof(T));
}

bool read_str(const uint8_t* d, size_t n, size_t& off, std::string& out) {
    uint64_t len = 0;
    if (!read_pod(d, n, off, len)) return false;
    if (off > n || len > n - off) return false;
    out.assign(reinterpret_cast<const char*>(d + off), static_cast<size_t>(len));
    off += static_cast<size_t>(len);
    return true;
}

size_t scalar_size(ValueType t) {
    switch (t) {
        case ValueType::U8: case ValueType::I8: case ValueType::BOOL: return 1;
        case ValueType::U16: case ValueType::I16: return 2;
        case ValueType::U32: case ValueType::I32: case ValueType::F32: return 4;
        case ValueType::U64: case ValueType::I64: case ValueType::F64: return 8;
        default: return 0;
    }
}

bool known_type(uint32_t t) { return t <= static_cast<uint32_t>(ValueType::F64); }

}  // namespace

bool Value::is_int() const {
    switch (type) {
        case ValueType::U8: case ValueType::I8: case ValueType::U16: case ValueType::I16: case ValueType::U32:
        case ValueType::I32: case ValueType::U64: case ValueType::I64: case ValueType::BOOL: return true;
        default: return false;
    }
}

bool Value::is_float() const { return type == ValueType::F32 || type == ValueType::F64; }

void type_block(uint32_t type, int64_t& elems, int64_t& bytes) {
    // the public GGUF block layouts (ggml); the byte sizes of the five types
    // the CUDA backend runs match src/model/gguf_loader.cpp:26-35
    struct B { uint32_t t; int64_t e, b; };
    static const B table[] = {
        {F32, 1, 4},     {F16, 1, 2},     {BF16, 1, 2},    {Q4_0, 32, 18},  {Q4_1, 32, 20},
        {Q5_0, 32, 22},  {Q5_1, 32, 24},  {Q8_0, 32, 34},  {Q8_1, 32, 36},  {Q2_K, 256, 84},
        {Q3_K, 256, 110}, {Q4_K, 256, 144}, {Q5_K, 256, 176}, {Q6_K, 256, 210}, {Q8_K, 256, 292},
        {I8, 1, 1},      {I16, 1, 2},     {I32, 1, 4},     {I64, 1, 8},     {F64, 1, 8},
    };
    for (const B& e : table)
        if (e.t == type) {
            elems = e.e;
            bytes = e.b;
            return;
        }
    elems = bytes = 0;
}

File::~File() {
    if (map_) munmap(map_, size_);
    if (fd_ >= 0) close(fd_);
}

int File::fail(int code, const std::string& what) {
    error_ = what;
    return code;
}

int File::open(const std::string& path) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) return fail(kFileNotFound, "cannot open " + path);
    struct stat st;
    if (fstat(fd_, &st) != 0 || st.st_size < 0) return fail(kFileNotFound, "cannot stat " + path);
    const size_t n = static_cast<size_t>(st.st_size);
    if (n < 24) return fail(kInvalidFormat, "file shorter than a GGUF header");
    void* m = mmap(nullptr, n, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (m == MAP_FAILED) return fail(kOutOfMemory, "mmap failed");
    map_ = m;
    return parse(static_cast<const uint8_t*>(m), n);
}

int File::read_value(size_t& off, ValueType t, Value& v, int depth) {
    const uint8_t* d = data_;
    const size_t n = size_;
    v.type = t;
    switch (t) {
        case ValueType::U8: { uint8_t x; if (!read_pod(d, n, off, x)) break; v.i = x; v.u = x; return kOk; }
        case ValueType::I8: { int8_t x; if (!read_pod(d, n, off, x)) break; v.i = x; return kOk; }
        case ValueType::U16: { uint16_t x; if (!read_pod(d, n, off, x)) break; v.i = x; v.u = x; return kOk; }
        case ValueType::I16: { int16_t x; if (!read_pod(d, n, off, x)) break; v.i = x; return kOk; }
        case ValueType::U32: { uint32_t x; if (!read_pod(d, n, off, x)) break; v.i = x; v.u = x; return kOk; }
        case ValueType::I32: { int32_t x; if (!read_pod(d, n, off, x)) break; v.i = x; return kOk; }
        case ValueType::U64: {
            uint64_t x;
            if (!read_pod(d, n, off, x)) break;
            v.u = x;
            v.i = x > static_cast<uint64_t>(std::numeric_limits<int64_t>::max()) ? std::numeric_limits<int64_t>::max()
                                                                                  : static_cast<int64_t>(x);
            return kOk;
        }
        case ValueType::I64: { int64_t x; if (!read_pod(d, n, off, x)) break; v.i = x; return kOk; }
        case ValueType::F32: { float x; if (!read_pod(d, n, off, x)) break; v.f = x; return kOk; }
        case ValueType::F64: { double x; if (!read_pod(d, n, off, x)) break; v.f = x; return kOk; }
        case ValueType::BOOL: {
            uint8_t x;
            if (!read_pod(d, n, off, x) || x > 1) break;
            v.i = x;
            return kOk;
        }
        case ValueType::STRING: if (!read_str(d, n, off, v.s)) break; return kOk;
        case ValueType::ARRAY: {
            uint32_t et = 0;
            uint64_t cnt = 0;
            if (!read_pod(d, n, off, et) || !read_pod(d, n, off, cnt)) break;
            if (!known_type(et) || cnt > kMaxCount || depth >= kMaxDepth)
                return fail(kInvalidFormat, "bad array header");
            v.elem = static_cast<ValueType>(et);
            v.count = cnt;
            const size_t es = scalar_size(v.elem);
            // every element takes at least es bytes (8 for a string's or an
            // array's length): the count must fit the rest of the file
            if (off > n || cnt > (n - off) / (es ? es : 8)) break;
            if (es) {
                if (v.elem == ValueType::F32 || v.elem == ValueType::F64) v.floats.reserve(cnt);
                else v.ints.reserve(cnt);
            }
            for (uint64_t i = 0; i < cnt; ++i) {
                Value e;
                const int rc = read_value(off, v.elem, e, depth + 1);
                if (rc != kOk) return rc;
                if (e.is_float()) v.floats.push_back(e.f);
                else if (e.is_int()) v.ints.push_back(e.i);
                else if (v.elem == ValueType::STRING) v.strings.push_back(std::move(e.s));
                // nested arrays: the length is kept, the contents are not
            }
            return kOk;
        }
        default: return fail(kInvalidFormat, "unknown metadata value type");
    }
    return fail(kInvalidFormat, "metadata value runs past the end of the file");
}

int File::parse(const uint8_t* data, size_t size) {
    data_ = data;
    size_ = size;
    kv_.clear();
    tensors_.clear();
    by_name_.clear();
    size_t off = 0;
    uint32_t magic = 0;
    uint64_t n_tensors = 0, n_kv = 0;
    if (!read_pod(data_, size_, off, magic) || magic != kMagic) return fail(kInvalidFormat, "not a GGUF file");
    if (!read_pod(data_, size_, off, version_) || (version_ != 2 && version_ != 3))
        return fail(kInvalidFormat, "unsupported GGUF version");
    if (!read_pod(data_, size_, off, n_tensors) || !read_pod(data_, size_, off, n_kv))
        return fail(kInvalidFormat, "truncated header");
    // every key and every tensor info takes at least 8 + 4 bytes
    if (n_kv > size_ / 12 || n_tensors > size_ / 12) return fail(kInvalidFormat, "implausible counts");

    for (uint64_t i = 0; i < n_kv; ++i) {
        std::string key;
        uint32_t t = 0;
        if (!read_str(data_, size_, off, key) || !read_pod(data_, size_, off, t))
            return fail(kInvalidFormat, "truncated metadata key");
        if (!known_type(t)) return fail(kInvalidFormat, "unknown type of key " + key);
        Value v;
        const int rc = read_value(off, static_cast<ValueType>(t), v, 0);
        if (rc != kOk) return fail(rc, error_ + " (key " + key + ")");
        kv_[key] = std::move(v);
    }

    alignment_ = 32;
    if (const Value* a = find("general.alignment")) {
        if (!a->is_int() || a->i <= 0 || (a->i & (a->i - 1)) != 0 || a->i > (1 << 20))
            return fail(kInvalidFormat, "general.alignment is not a power of two");
        alignment_ = static_cast<uint64_t>(a->i);
    }

    tensors_.reserve(static_cast<size_t>(n_tensors));
    for (uint64_t i = 0; i < n_tensors; ++i) {
        TensorInfo ti;
        if (!read_str(data_, size_, off, ti.name) || !read_pod(data_, size_, off, ti.n_dims))
            return fail(kInvalidFormat, "truncated tensor info");
        if (ti.n_dims < 1 || ti.n_dims > 4) return fail(kInvalidFormat, "tensor " + ti.name + ": bad dimension count");
        for (uint32_t dd = 0; dd < ti.n_dims; ++dd) {
            uint64_t x = 0;
            if (!read_pod(data_, size_, off, x)) return fail(kInvalidFormat, "truncated tensor dims");
            if (x == 0 || x > (uint64_t(1) << 40)) return fail(kInvalidFormat, "tensor " + ti.name + ": bad dimension");
            ti.ne[dd] = static_cast<int64_t>(x);
        }
        if (!read_pod(data_, size_, off, ti.type) || !read_pod(data_, size_, off, ti.offset))
            return fail(kInvalidFormat, "truncated tensor info");
        // element count without overflow (each factor <= 2^40, the product <= 2^62)
        long double prod = 1.0L;
        for (int dd = 0; dd < 4; ++dd) prod *= static_cast<long double>(ti.ne[dd]);
        if (prod > static_cast<long double>(int64_t(1) << 62)) return fail(kInvalidFormat, "tensor too large");
        int64_t be = 0, bb = 0;
        type_block(ti.type, be, bb);
        if (be > 0) {
            if (ti.ne[0] % be != 0) return fail(kInvalidFormat, "tensor " + ti.name + ": rows are not whole blocks");
            ti.bytes = static_cast<uint64_t>(ti.nelements() / be * bb);
        }
        if (by_name_.count(ti.name)) return fail(kInvalidFormat, "duplicate tensor " + ti.name);
        by_name_[ti.name] = tensors_.size();
        tensors_.push_back(std::move(ti));
    }

    const uint64_t end = off;
    data_offset_ = (end + alignment_ - 1) / alignment_ * alignment_;
    if (data_offset_ > size_ && !tensors_.empty()) return fail(kInvalidFormat, "no tensor data section");
    const uint64_t avail = size_ >= data_offset_ ? size_ - data_offset_ : 0;
    for (TensorInfo& ti : tensors_) {
        if (ti.offset % alignment_ != 0) return fail(kInvalidFormat, "tensor " + ti.name + ": misaligned offset");
        if (ti.bytes == 0) continue;   // a type this reader does not size: no pointer
        if (ti.offset > avail || ti.bytes > avail - ti.offset)
            return fail(kInvalidFormat, "tensor " + ti.name + ": data past the end of the file");
        ti.data = data_ + data_offset_ + ti.offset;
    }
    error_.clear();
    return kOk;
}

const Value* File::find(const std::string& key) const {
    auto it = kv_.find(key);
    return it == kv_.end() ? nullptr : &it->second;
}

int64_t File::get_int(const std::string& key, int64_t def) const {
    const Value* v = find(key);
    if (!v) return def;
    if (v->is_int()) return v->i;
    if (v->is_float()) return static_cast<int64_t>(v->f);
    return def;
}

double File::get_float(const std::string& key, double def) const {
    const Value* v = find(key);
    if (!v) return def;
    if (v->is_float()) return v->f;
    if (v->is_int()) return static_cast<double>(v->i);
    return def;
}

std::string File::get_string(const std::string& key) const {
    const Value* v = find(key);
    return v && v->type == ValueType::STRING ? v->s : std::string();
}

const TensorInfo* File::tensor(const std::string& name) const {
    auto it = by_name_.find(name);
    return it == by_name_.end() ? nullptr : &tensors_[it->second];
}

int File::llama_shape(LlamaShape& out) const {
    out = LlamaShape{};
    out.arch = get_string("general.architecture");
    if (out.arch.empty()) return kInvalidFormat;
    const std::string a = out.arch + ".";
    out.n_layer = get_int(a + "block_count", 0);
    out.d_model = get_int(a + "embedding_length", 0);
    out.d_ff = get_int(a + "feed_forward_length", 0);
    out.n_head = get_int(a + "attention.head_count", 0);
    out.n_kv_head = get_int(a + "attention.head_count_kv", out.n_head);
    out.context = get_int(a + "context_length", 0);
    out.rms_eps = static_cast<float>(get_float(a + "attention.layer_norm_rms_epsilon", 1e-5));
    out.rope_base = static_cast<float>(get_float(a + "rope.freq_base", 10000.0));
    if (const TensorInfo* t = tensor("token_embd.weight")) out.vocab = t->rows();
    if (!out.vocab) {
        if (const Value* v = find("tokenizer.ggml.tokens")) out.vocab = static_cast<int64_t>(v->count);
    }
    if (out.n_layer <= 0 || out.d_model <= 0 || out.d_ff <= 0 || out.n_head <= 0 || out.n_kv_head <= 0 ||
        out.vocab <= 0 || out.d_model % out.n_head != 0 || out.n_head % out.n_kv_head != 0)
        return kInvalidFormat;
    return kOk;
}

}  // namespace hesa_gguf
