// gguf_file.hpp -- a bounds-checked reader of GGUF v2/v3 model files.
//
// The repair of the reference's GGUFReader (src/model/gguf_loader.cpp:
// 138-272), written anew so that real GGUF files reach the CUDA backend:
//   * every metadata value type of the format is decoded, ARRAY (of any
//     element type, nested arrays included), UINT8/INT8/UINT16/INT16 and
//     BOOL among them -- the reference skips 4 bytes for the types it does
//     not know (gguf_loader.cpp:184-187), which desynchronises the parse at
//     the first tokenizer array;
//   * the tensor infos follow the metadata directly (the reference aligns
//     before reading them, gguf_loader.cpp:249); only the tensor data starts
//     at a multiple of `general.alignment` (default 32);
//   * `<arch>.attention.layer_norm_rms_epsilon` is a float (the reference
//     reads it as an integer, gguf_loader.cpp:230);
//   * every read is checked against the file size, every tensor's bytes
//     against the data section, and dimension products against overflow:
//     a truncated or corrupt file is INVALID_FORMAT, never a wild read;
//   * block sizes of the quantized types follow the public format (Q3_K is
//     110 bytes per 256 weights; gguf_loader.cpp:32 says 112).
// The file is memory-mapped read-only; tensor bytes are returned as
// pointers into the mapping. Plain C++17 + POSIX, no CUDA, no reference
// headers: error values are those of hesa::Error (include/hesa/result.hpp:
// 14-30).
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace hesa_gguf {

// hesa::Error values (include/hesa/result.hpp:14-30)
enum Status : int { kOk = 0, kOutOfMemory = 1, kInvalidArgument = 2, kTensorNotFound = 5, kFileNotFound = 7,
                    kInvalidFormat = 8 };

enum class ValueType : uint32_t {
    U8 = 0, I8 = 1, U16 = 2, I16 = 3, U32 = 4, I32 = 5, F32 = 6, BOOL = 7, STRING = 8, ARRAY = 9,
    U64 = 10, I64 = 11, F64 = 12
};

// One metadata value. Integers (and BOOL) are in `i` (U64 values above
// INT64_MAX also in `u`), floats in `f`, strings in `s`. An ARRAY keeps its
// element type and length, and its elements when they are numbers or strings
// (nested arrays keep their length only).
struct Value {
    ValueType type = ValueType::U8;
    int64_t i = 0;
    uint64_t u = 0;
    double f = 0.0;
    std::string s;
    ValueType elem = ValueType::U8;
    uint64_t count = 0;
    std::vector<int64_t> ints;
    std::vector<double> floats;
    std::vector<std::string> strings;

    bool is_int() const;
    bool is_float() const;
};

// ggml tensor types (the ids of src/model/gguf_loader.hpp:15-45)
enum TensorType : uint32_t {
    F32 = 0, F16 = 1, Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, Q8_1 = 9, Q2_K = 10, Q3_K = 11,
    Q4_K = 12, Q5_K = 13, Q6_K = 14, Q8_K = 15, I8 = 24, I16 = 25, I32 = 26, I64 = 27, F64 = 28, BF16 = 30
};

// Elements and bytes of one block of a tensor type (0, 0 if unknown).
void type_block(uint32_t type, int64_t& elems, int64_t& bytes);

struct TensorInfo {
    std::string name;
    uint32_t n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};   // GGUF order: ne[0] is the contiguous (row) dimension
    uint32_t type = 0;
    uint64_t offset = 0;            // from the start of the data section
    uint64_t bytes = 0;             // 0 for a type this reader does not size
    const uint8_t* data = nullptr;  // into the mapping (null for an unsized type)

    int64_t nelements() const { return ne[0] * ne[1] * ne[2] * ne[3]; }
    // row-major view: rows = ne[1] * ne[2] * ne[3], cols = ne[0]
    int64_t rows() const { return ne[1] * ne[2] * ne[3]; }
    int64_t cols() const { return ne[0]; }
};

// The shape of a Llama-style decoder, read from `<arch>.*` keys.
struct LlamaShape {
    std::string arch;
    int64_t n_layer = 0, d_model = 0, n_head = 0, n_kv_head = 0, d_ff = 0, vocab = 0, context = 0;
    float rms_eps = 1e-5f;
    float rope_base = 10000.0f;
};

class File {
public:
    File() = default;
    ~File();
    File(const File&) = delete;
    File& operator=(const File&) = delete;

    // Map and parse `path`; kOk or a hesa::Error value (message in error()).
    int open(const std::string& path);
    // Parse a file already in memory (not copied; must outlive this object).
    int parse(const uint8_t* data, size_t size);

    uint32_t version() const { return version_; }
    uint64_t alignment() const { return alignment_; }
    uint64_t data_offset() const { return data_offset_; }
    size_t size() const { return size_; }
    const std::string& error() const { return error_; }

    const std::map<std::string, Value>& metadata() const { return kv_; }
    const Value* find(const std::string& key) const;
    int64_t get_int(const std::string& key, int64_t def) const;
    double get_float(const std::string& key, double def) const;
    std::string get_string(const std::string& key) const;

    const std::vector<TensorInfo>& tensors() const { return tensors_; }
    const TensorInfo* tensor(const std::string& name) const;

    // kOk and the decoder shape, or kInvalidFormat when a key it needs is missing.
    int llama_shape(LlamaShape& out) const;

private:
    int fail(int code, const std::string& what);
    int read_value(size_t& off, ValueType t, Value& v, int depth);

    const uint8_t* data_ = nullptr;
    size_t size_ = 0;
    void* map_ = nullptr;
    int fd_ = -1;
    uint32_t version_ = 0;
    uint64_t alignment_ = 32;
    uint64_t data_offset_ = 0;
    std::map<std::string, Value> kv_;
    std::vector<TensorInfo> tensors_;
    std::map<std::string, size_t> by_name_;
    std::string error_;
};

}  // namespace hesa_gguf
