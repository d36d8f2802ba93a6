// cuda_backend.cpp -- hesa::Backend for B200 on top of the hesa_cuda C ABI.
// See cuda_backend.hpp for the ownership model.
#include "cuda_backend.hpp"

#include "hesa_cuda.h"

#include <cuda_runtime.h>

#include <cstring>

namespace hesa {

namespace {

// GGUF type id of a quantized hesa::Dtype (include/hesa/tensor.hpp:18-33 ->
// src/model/gguf_loader.hpp:15-45), 0 for F32, -1 if this backend has no kernel.
int qtype_of(Dtype dt) {
    switch (dt) {
        case Dtype::Q4_0: return HESA_CUDA_Q4_0;
        case Dtype::Q8_0: return HESA_CUDA_Q8_0;
        case Dtype::Q4_K: return HESA_CUDA_Q4_K;
        case Dtype::Q5_K: return HESA_CUDA_Q5_K;
        case Dtype::Q6_K: return HESA_CUDA_Q6_K;
        case Dtype::F32: return 0;
        default: return -1;
    }
}

Result<void> from_abi(int rc) {
    if (rc == 0) return ok();
    return error(static_cast<Error>(rc));
}

Result<void> from_cuda(cudaError_t e) {
    if (e == cudaSuccess) return ok();
    return error(Error::CUDA_ERROR);
}

template <typename T>
Result<T> fail_as(Error e) {
    return std::unexpected{make_error_code(e)};
}

float load_f32(const TensorView& v, int64_t i, int64_t j) {
    const auto st = v.byte_strides();
    const auto* base = static_cast<const uint8_t*>(v.data());
    float f;
    std::memcpy(&f, base + static_cast<size_t>(i) * st[0] + static_cast<size_t>(j) * st[1], sizeof(float));
    return f;
}

void store_f32(TensorView& v, int64_t i, int64_t j, float f) {
    const auto st = v.byte_strides();
    auto* base = static_cast<uint8_t*>(v.data());
    std::memcpy(base + static_cast<size_t>(i) * st[0] + static_cast<size_t>(j) * st[1], &f, sizeof(float));
}

}  // namespace

CudaBackend::CudaBackend(DeviceConfig cfg) : device_(cfg.device_id), memory_limit_(cfg.memory_limit) {
    if (cudaSetDevice(device_) == cudaSuccess) {
        cudaStream_t s = nullptr;
        if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) == cudaSuccess) stream_ = s;
    }
}

CudaBackend::~CudaBackend() {
    if (cudaSetDevice(device_) != cudaSuccess) return;
    if (stream_) cudaStreamSynchronize(static_cast<cudaStream_t>(stream_));
    for (auto& kv : weights_) cudaFree(kv.second.ptr);
    for (DevBuf* b : {&d_x_, &d_y_, &d_ws_})
        if (b->ptr) cudaFree(b->ptr);
    for (DevBuf* b : {&h_x_, &h_y_})
        if (b->ptr) cudaFreeHost(b->ptr);
    if (stream_) cudaStreamDestroy(static_cast<cudaStream_t>(stream_));
}

Result<void> CudaBackend::activate() const {
    if (!stream_) return error(Error::BACKEND_NOT_AVAILABLE);
    return from_cuda(cudaSetDevice(device_));
}

bool CudaBackend::supports(Dtype dt) const { return qtype_of(dt) >= 0; }

size_t CudaBackend::device_memory() const {
    size_t free_b = 0, total = 0;
    if (cudaSetDevice(device_) != cudaSuccess || cudaMemGetInfo(&free_b, &total) != cudaSuccess) return 0;
    return memory_limit_ ? std::min(memory_limit_, total) : total;
}

size_t CudaBackend::device_memory_used() const {
    return weight_bytes_ + d_x_.bytes + d_y_.bytes + d_ws_.bytes;
}

Result<void> CudaBackend::ensure(DevBuf& b, size_t bytes) {
    if (b.bytes >= bytes && b.ptr) return ok();
    if (b.ptr) cudaFree(b.ptr);
    b = DevBuf{};
    if (memory_limit_ && device_memory_used() + bytes > memory_limit_) return error(Error::OUT_OF_MEMORY);
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return error(Error::OUT_OF_MEMORY);
    b.ptr = p;
    b.bytes = bytes;
    return ok();
}

Result<void> CudaBackend::ensure_host(DevBuf& b, size_t bytes) {
    if (b.bytes >= bytes && b.ptr) return ok();
    if (b.ptr) cudaFreeHost(b.ptr);
    b = DevBuf{};
    void* p = nullptr;
    if (cudaMallocHost(&p, bytes) != cudaSuccess) return error(Error::OUT_OF_MEMORY);
    b.ptr = p;
    b.bytes = bytes;
    return ok();
}

Result<const void*> CudaBackend::device_weights(const void* host, size_t bytes) {
    const auto key = std::make_pair(host, bytes);
    auto it = weights_.find(key);
    if (it != weights_.end()) return static_cast<const void*>(it->second.ptr);
    if (memory_limit_ && device_memory_used() + bytes > memory_limit_) return fail_as<const void*>(Error::OUT_OF_MEMORY);
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return fail_as<const void*>(Error::OUT_OF_MEMORY);
    if (cudaMemcpyAsync(p, host, bytes, cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream_)) != cudaSuccess) {
        cudaFree(p);
        return fail_as<const void*>(Error::CUDA_ERROR);
    }
    weights_[key] = DevBuf{p, bytes};
    weight_bytes_ += bytes;
    return static_cast<const void*>(p);
}

Result<Tensor> CudaBackend::alloc_tensor(Dtype dtype, std::span<const int64_t> shape) {
    Tensor t(dtype, shape, this);
    if (t.nelements() == 0) return fail_as<Tensor>(Error::INVALID_ARGUMENT);
    return std::move(t);
}

Result<void> CudaBackend::free_tensor(Tensor& tensor) {
    // evict any device copy made from this tensor's bytes
    for (auto it = weights_.begin(); it != weights_.end();) {
        if (it->first.first == tensor.data()) {
            cudaFree(it->second.ptr);
            weight_bytes_ -= it->second.bytes;
            it = weights_.erase(it);
        } else {
            ++it;
        }
    }
    tensor = Tensor{};
    return ok();
}

Result<void> CudaBackend::matmul(TensorView a, TensorView b, TensorView out, float scale) {
    HESA_CHECK(activate());
    if (a.ndim() != 2 || b.ndim() != 2 || out.ndim() != 2) return error(Error::SHAPE_MISMATCH);
    if (b.dtype() != Dtype::F32 || out.dtype() != Dtype::F32) return error(Error::INVALID_ARGUMENT);
    const int qt = qtype_of(a.dtype());
    if (qt < 0) return error(Error::BACKEND_NOT_AVAILABLE);
    const int64_t M = a.shape()[0], K = a.shape()[1], N = b.shape()[1];
    if (b.shape()[0] != K || out.shape()[0] != M || out.shape()[1] != N || M <= 0 || K <= 0 || N <= 0)
        return error(Error::SHAPE_MISMATCH);
    cudaStream_t s = static_cast<cudaStream_t>(stream_);

    // weights: packed GGUF rows (byte strides of quantized views are not
    // meaningful, dtype_size is 1), or a row-major F32 matrix
    size_t wbytes;
    if (qt > 0) {
        wbytes = hesa_cuda_row_bytes(qt, K) * static_cast<size_t>(M);
        if (wbytes == 0) return error(Error::SHAPE_MISMATCH);
    } else {
        const auto st = a.byte_strides();
        if (st[1] != sizeof(float) || st[0] != static_cast<size_t>(K) * sizeof(float))
            return error(Error::INVALID_ARGUMENT);
        wbytes = static_cast<size_t>(M) * K * sizeof(float);
    }
    auto dw = device_weights(a.data(), wbytes);
    if (!dw) return std::unexpected{dw.error()};

    // activations: b[k, j] -> x[j*K + k]
    const size_t xbytes = static_cast<size_t>(N) * K * sizeof(float);
    const size_t ybytes = static_cast<size_t>(N) * M * sizeof(float);
    HESA_CHECK(ensure_host(h_x_, xbytes));
    HESA_CHECK(ensure_host(h_y_, ybytes));
    HESA_CHECK(ensure(d_x_, xbytes));
    HESA_CHECK(ensure(d_y_, ybytes));
    HESA_CHECK(from_cuda(cudaStreamSynchronize(s)));  // staging buffers are free
    float* hx = static_cast<float*>(h_x_.ptr);
    for (int64_t j = 0; j < N; ++j)
        for (int64_t k = 0; k < K; ++k) hx[j * K + k] = load_f32(b, k, j);
    HESA_CHECK(from_cuda(cudaMemcpyAsync(d_x_.ptr, hx, xbytes, cudaMemcpyHostToDevice, s)));

    if (qt > 0) {
        const size_t ws = hesa_cuda_qmatvec_workspace_size(qt, M, K, N);
        if (d_ws_.bytes < ws) {
            HESA_CHECK(ensure(d_ws_, ws));
            HESA_CHECK(from_cuda(cudaMemsetAsync(d_ws_.ptr, 0, d_ws_.bytes, s)));
        }
        HESA_CHECK(from_abi(hesa_cuda_qmatvec(qt, *dw, M, K, static_cast<const float*>(d_x_.ptr), K, N,
                                              static_cast<float*>(d_y_.ptr), M, scale, d_ws_.ptr, d_ws_.bytes, s)));
    } else {
        HESA_CHECK(from_abi(hesa_cuda_matmul_f32(static_cast<const float*>(*dw), M, K,
                                                 static_cast<const float*>(d_x_.ptr), K, N,
                                                 static_cast<float*>(d_y_.ptr), M, scale, s)));
    }
    HESA_CHECK(from_cuda(cudaMemcpyAsync(h_y_.ptr, d_y_.ptr, ybytes, cudaMemcpyDeviceToHost, s)));
    HESA_CHECK(from_cuda(cudaStreamSynchronize(s)));
    const float* hy = static_cast<const float*>(h_y_.ptr);
    for (int64_t j = 0; j < N; ++j)
        for (int64_t i = 0; i < M; ++i) store_f32(out, i, j, hy[j * M + i]);
    return ok();
}

Result<void> CudaBackend::add(TensorView, TensorView, TensorView) { return error(Error::BACKEND_NOT_AVAILABLE); }
Result<void> CudaBackend::mul(TensorView, TensorView, TensorView) { return error(Error::BACKEND_NOT_AVAILABLE); }
Result<void> CudaBackend::softmax(TensorView, TensorView, int) { return error(Error::BACKEND_NOT_AVAILABLE); }
Result<void> CudaBackend::rms_norm(TensorView, TensorView, TensorView, float) {
    return error(Error::BACKEND_NOT_AVAILABLE);
}
Result<void> CudaBackend::rope(TensorView, std::span<const int32_t>, float, int) {
    return error(Error::BACKEND_NOT_AVAILABLE);
}
Result<void> CudaBackend::silu(TensorView, TensorView) { return error(Error::BACKEND_NOT_AVAILABLE); }
Result<void> CudaBackend::scaled_dot_product_attention(TensorView, TensorView, TensorView, TensorView, TensorView,
                                                       float) {
    return error(Error::BACKEND_NOT_AVAILABLE);
}

Result<Tensor> CudaBackend::quantize(TensorView, Dtype) { return fail_as<Tensor>(Error::BACKEND_NOT_AVAILABLE); }

Result<void> CudaBackend::synchronize() {
    HESA_CHECK(activate());
    return from_cuda(cudaStreamSynchronize(static_cast<cudaStream_t>(stream_)));
}

Result<void> CudaBackend::copy_tensor(const Tensor& src, Tensor& dst) {
    // host tensors (src/tensor/tensor.cpp:63-77): copy bytes and drop any
    // device copy of the destination, whose contents change
    std::memcpy(dst.data(), src.data(), std::min(src.nbytes(), dst.nbytes()));
    for (auto it = weights_.begin(); it != weights_.end();) {
        if (it->first.first == dst.data()) {
            cudaFree(it->second.ptr);
            weight_bytes_ -= it->second.bytes;
            it = weights_.erase(it);
        } else {
            ++it;
        }
    }
    return ok();
}

}  // namespace hesa
