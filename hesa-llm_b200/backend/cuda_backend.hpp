// cuda_backend.hpp -- hesa::Backend implementation for NVIDIA B200 (sm_100a).
//
// The drop-in for the CUDA slot of hesa-llm: src/backend/backend.cpp:32-37
// constructs `CudaBackend(cfg)` when HESA_HAS_CUDA is defined, and
// CMakeLists.txt:99-100 compiles src/backend/cuda_backend.cpp. This class is
// that backend. It implements the interface of include/hesa/backend.hpp:28-65
// and reaches the GPU only through the C ABI of include/hesa_cuda.h.
//
// Operands may live in device or host memory (checked per pointer):
//   * device-resident views -- weights uploaded once by hesa_gguf::DeviceModel
//     (backend/device_model.hpp) from a GGUF file, activations and outputs in
//     device buffers -- are used in place, with no copy and no host wait;
//   * host views (Tensors of the reference own host memory,
//     src/tensor/tensor.cpp:63-77, where device_ptr is never set): weight
//     views of a quantized dtype are uploaded once and cached by (host
//     pointer, bytes), which assumes the bytes do not change while cached
//     (GGUF weights are immutable after Model::load; free_tensor or forget()
//     drops a copy); activations and outputs travel through pinned staging
//     buffers on every call, on the backend's own stream.
// Calls are asynchronous on that stream except where a host result is
// produced (matmul writes a host `out`); synchronize() joins.
#pragma once

#include "hesa/backend.hpp"

#include <cstddef>
#include <cstdint>
#include <map>
#include <utility>

namespace hesa {

class CudaBackend final : public Backend {
public:
    explicit CudaBackend(DeviceConfig cfg);
    ~CudaBackend() override;

    CudaBackend(const CudaBackend&) = delete;
    CudaBackend& operator=(const CudaBackend&) = delete;

    BackendType type() const override { return BackendType::CUDA; }
    const char* name() const override { return "CUDA (B200 sm_100a)"; }
    bool supports(Dtype dt) const override;
    size_t device_memory() const override;
    size_t device_memory_used() const override;

    Result<Tensor> alloc_tensor(Dtype dtype, std::span<const int64_t> shape) override;
    Result<void> free_tensor(Tensor& tensor) override;

    // out = scale * a @ b with a = W [n_out, k] (Q4_0/Q8_0/Q4_K/Q5_K/Q6_K or
    // F32), b = [k, batch] F32 (any byte strides, e.g. a transposed [batch, k]
    // view), out = [n_out, batch] F32 (any byte strides).
    // The other ops follow the CPU backend (src/backend/cpu_backend.cpp:162-294)
    // on contiguous F32 views: add, mul, silu element-wise; softmax and
    // rms_norm over rows of the last dimension; rope on [n_tokens, n_heads,
    // n_dims] with one position per token (rotate-half); attention on
    // q [n_q, heads, d], k, v [n_k, heads, d], no mask, scale 1/sqrt(d) unless
    // given. Unlike the CPU backend, attention overwrites `out` (the CPU
    // version adds to whatever it holds). quantize packs [rows, k] F32 into
    // Q4_0/Q4_K/Q5_K/Q6_K rows; Q8_0 is INVALID_FORMAT because its packed rows
    // do not fit a Tensor of one byte per element.
    Result<void> matmul(TensorView a, TensorView b, TensorView out, float scale = 1.0f) override;
    Result<void> add(TensorView a, TensorView b, TensorView out) override;
    Result<void> mul(TensorView a, TensorView b, TensorView out) override;
    Result<void> softmax(TensorView in, TensorView out, int axis = -1) override;
    Result<void> rms_norm(TensorView in, TensorView weight, TensorView out, float eps = 1e-6f) override;
    Result<void> rope(TensorView in_out, std::span<const int32_t> positions, float freq_base,
                      int n_dims) override;
    Result<void> silu(TensorView in, TensorView out) override;
    Result<void> scaled_dot_product_attention(TensorView q, TensorView k, TensorView v, TensorView out,
                                              TensorView mask = {}, float scale = 0.0f) override;
    Result<Tensor> quantize(TensorView src, Dtype target_dtype) override;
    Result<void> synchronize() override;
    Result<void> copy_tensor(const Tensor& src, Tensor& dst) override;

    // Views on device memory (the GGUF weights of a hesa_gguf::DeviceModel,
    // or device activations): matmul takes them without any host copy. A
    // quantized weight view is [rows, cols]; an activation view [k, batch]
    // over `batch` device rows of k floats (ld floats apart); an output view
    // [n_out, batch] likewise. With device-resident a, b and out, matmul is
    // asynchronous on stream() and returns without waiting.
    static TensorView device_view(const void* ptr, Dtype dtype, int64_t rows, int64_t cols);
    static TensorView device_columns(float* ptr, int64_t k, int64_t batch, int64_t ld);
    // GGUF tensor type id -> Dtype (false when the Dtype enum has no such type)
    static bool dtype_of_gguf(uint32_t type, Dtype& out);

    int device_id() const { return device_; }
    void* stream() const { return stream_; }
    // number of weight uploads kept on the device (test hook)
    size_t cached_weights() const { return weights_.size(); }
    // drop the device copies made from host bytes at `host`
    void forget(const void* host);

private:
    struct DevBuf {
        void* ptr = nullptr;
        size_t bytes = 0;
    };
    Result<void> ensure(DevBuf& b, size_t bytes);
    Result<void> ensure_host(DevBuf& b, size_t bytes);
    Result<const void*> device_weights(const void* host, size_t bytes);
    Result<void> activate() const;
    // contiguous F32 view -> device scratch buffer `slot` (returns the device pointer)
    Result<float*> upload(const TensorView& v, int slot);
    // device scratch buffer `slot` -> contiguous F32 view, then synchronize
    Result<void> download(int slot, TensorView& v);

    int device_ = 0;
    size_t memory_limit_ = 0;
    void* stream_ = nullptr;
    std::map<std::pair<const void*, size_t>, DevBuf> weights_;
    size_t weight_bytes_ = 0;
    DevBuf d_x_, d_y_, d_ws_, h_x_, h_y_;
    DevBuf scratch_[6];   // device operands of the element-wise and attention ops
    size_t ws_zeroed_ = 0;
};

}  // namespace hesa
