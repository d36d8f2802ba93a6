// device_model.hpp -- GGUF weights resident in GPU memory, and a decode
// session that runs a Llama-style decoder straight from them.
//
// The reference keeps every tensor in host memory: Model::load copies the
// packed rows of each GGUF tensor into a host std::vector
// (src/model/gguf_loader.cpp:291-316) and Tensor::Impl::device_ptr is never
// set (src/tensor/tensor.cpp:63-77); its design puts weights on the compute
// device at load (docs/architecture.md:453-485). DeviceModel does that for
// the CUDA backend: one device allocation, every tensor copied once (through
// pinned staging buffers, asynchronously on the caller's stream), the Q, K, V
// rows of each layer and its gate and up rows placed back to back so the
// decode step runs each group as one matvec. Device pointers are plain
// (void*), for hesa_cuda_* calls and for device-resident TensorViews
// (CudaBackend::device_view).
#pragma once

#include "gguf_file.hpp"

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace hesa_gguf {

struct DeviceTensor {
    std::string name;
    void* ptr = nullptr;     // device
    uint64_t bytes = 0;
    uint32_t type = 0;       // ggml type id
    int64_t rows = 0, cols = 0;   // row-major [rows, cols]: cols = GGUF ne[0]
};

class DeviceModel {
public:
    DeviceModel() = default;
    ~DeviceModel();
    DeviceModel(const DeviceModel&) = delete;
    DeviceModel& operator=(const DeviceModel&) = delete;

    // Copy every tensor of `f` with a known size to GPU `device` (made current)
    // on `stream` (a cudaStream_t); returns when the copies are done. kOk or a
    // hesa::Error value (message in error()).
    int upload(const File& f, int device, void* stream);

    const DeviceTensor* find(const std::string& name) const;
    const std::vector<DeviceTensor>& tensors() const { return t_; }
    size_t bytes() const { return bytes_; }
    int device() const { return device_; }
    const std::string& error() const { return error_; }

private:
    int fail(int code, const std::string& what);
    void release();

    void* base_ = nullptr;
    size_t bytes_ = 0;
    int device_ = 0;
    std::vector<DeviceTensor> t_;
    std::map<std::string, size_t> idx_;
    std::string error_;
};

// One token at a time through the decoder of a DeviceModel (GGUF tensor
// names "token_embd", "blk.N.attn_norm|attn_q|attn_k|attn_v|attn_output|
// ffn_norm|ffn_gate|ffn_up|ffn_down", "output_norm", "output" -- the LM head
// falls back to token_embd when the file ties them) with an fp16 KV ring of
// `ctx` slots, via hesa_cuda_embed + hesa_cuda_decode_step. Every projection
// and the LM head must share one of the quantized types the kernels run
// (Q4_0, Q8_0, Q4_K, Q5_K, Q6_K); norms are F32.
class DecodeSession {
public:
    DecodeSession() = default;
    ~DecodeSession();
    DecodeSession(const DecodeSession&) = delete;
    DecodeSession& operator=(const DecodeSession&) = delete;

    int init(const File& f, const DeviceModel& m, int32_t ctx, void* stream);
    // Enqueue one token at position pos; *logits_dev <- the device logits
    // [vocab] (valid once the stream reaches them).
    int step(int32_t token, int32_t pos, const float** logits_dev);
    // The device scalars the step reads (write them yourself to replay a
    // captured graph of enqueue_step() at new tokens and positions).
    int32_t* token_dev() const { return tok_pos_; }
    int32_t* pos_dev() const { return tok_pos_ ? tok_pos_ + 1 : nullptr; }
    int enqueue_step();   // the step with the device token and position as they are
    int64_t vocab() const { return shape_.vocab; }
    const LlamaShape& shape() const { return shape_; }
    const std::string& error() const { return error_; }

private:
    int fail(int code, const std::string& what);
    void release();

    LlamaShape shape_;
    int qtype_ = 0, emb_qtype_ = 0;
    int32_t ctx_ = 0, rope_rows_ = 0;
    void* stream_ = nullptr;
    std::vector<unsigned char> model_;    // hesa_cuda_model
    std::vector<unsigned char> layers_;   // hesa_cuda_layer[n_layer]
    const void* emb_ = nullptr;
    const void* w_out_ = nullptr;
    const float* out_norm_ = nullptr;
    void* kv_ = nullptr;          // every layer's K and V caches
    float* rope_ = nullptr;
    float* x_ = nullptr;
    float* logits_ = nullptr;
    void* ws_ = nullptr;
    size_t ws_bytes_ = 0;
    int32_t* tok_pos_ = nullptr;  // device [token, position]
    int32_t* host_tp_ = nullptr;  // pinned [token, position]
    std::string error_;
};

}  // namespace hesa_gguf
