// cuda_backend.cpp -- hesa::Backend for B200 on top of the hesa_cuda C ABI.
// See cuda_backend.hpp for the ownership model.
#include "cuda_backend.hpp"

#include "hesa_cuda.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

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

// true when v is F32 and laid out row-major without gaps (the CPU backend's
// element-wise kernels read data() as a flat array)
bool contiguous_f32(const TensorView& v) {
    if (v.dtype() != Dtype::F32 || v.data() == nullptr) return false;
    const auto st = v.byte_strides();
    size_t expect = sizeof(float);
    for (size_t d = v.ndim(); d-- > 0;) {
        if (v.shape()[d] > 1 && st[d] != expect) return false;
        expect *= static_cast<size_t>(v.shape()[d]);
    }
    return true;
}

// true when p points into device (or managed) memory of any device
bool on_device(const void* p) {
    if (!p) return false;
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();   // a plain host pointer: not an error to keep
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
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
    for (DevBuf& b : scratch_)
        if (b.ptr) cudaFree(b.ptr);
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
    size_t n = weight_bytes_ + d_x_.bytes + d_y_.bytes + d_ws_.bytes;
    for (const DevBuf& b : scratch_) n += b.bytes;
    return n;
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

void CudaBackend::forget(const void* host) {
    for (auto it = weights_.begin(); it != weights_.end();) {
        if (it->first.first == host) {
            cudaFree(it->second.ptr);
            weight_bytes_ -= it->second.bytes;
            it = weights_.erase(it);
        } else {
            ++it;
        }
    }
}

Result<void> CudaBackend::free_tensor(Tensor& tensor) {
    // evict any device copy made from this tensor's bytes
    forget(tensor.data());
    tensor = Tensor{};
    return ok();
}

TensorView CudaBackend::device_view(const void* ptr, Dtype dtype, int64_t rows, int64_t cols) {
    const size_t es = dtype_size(dtype);
    const size_t st[2] = {static_cast<size_t>(cols) * es, es};
    return TensorView(ptr, dtype, Shape{rows, cols}, std::span<const size_t>(st, 2));
}

TensorView CudaBackend::device_columns(float* ptr, int64_t k, int64_t batch, int64_t ld) {
    // [k, batch] with element (i, j) at ptr[j * ld + i]
    const size_t st[2] = {sizeof(float), static_cast<size_t>(ld) * sizeof(float)};
    return TensorView(static_cast<void*>(ptr), Dtype::F32, Shape{k, batch}, std::span<const size_t>(st, 2));
}

bool CudaBackend::dtype_of_gguf(uint32_t type, Dtype& out) {
    switch (type) {
        case 0: out = Dtype::F32; return true;
        case 1: out = Dtype::F16; return true;
        case 30: out = Dtype::BF16; return true;
        case 24: out = Dtype::I8; return true;
        case 2: out = Dtype::Q4_0; return true;
        case 3: out = Dtype::Q4_1; return true;
        case 6: out = Dtype::Q5_0; return true;
        case 7: out = Dtype::Q5_1; return true;
        case 8: out = Dtype::Q8_0; return true;
        case 10: out = Dtype::Q2_K; return true;
        case 11: out = Dtype::Q3_K; return true;
        case 12: out = Dtype::Q4_K; return true;
        case 13: out = Dtype::Q5_K; return true;
        case 14: out = Dtype::Q6_K; return true;
        default: return false;
    }
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
    // device-resident weights are used in place; host weights are uploaded once
    const void* dev_w = nullptr;
    if (on_device(a.data())) {
        dev_w = a.data();
    } else {
        auto dw = device_weights(a.data(), wbytes);
        if (!dw) return std::unexpected{dw.error()};
        dev_w = *dw;
    }

    // device-resident activations and outputs: no staging, no host wait. The
    // C ABI wants batch rows of x (k floats, ldx apart) and of y (n_out, ldy
    // apart), i.e. b and out as column views over device rows.
    if (on_device(b.data()) && on_device(out.data())) {
        const auto bs = b.byte_strides();
        const auto os = out.byte_strides();
        if (bs[0] != sizeof(float) || os[0] != sizeof(float)) return error(Error::INVALID_ARGUMENT);
        const int64_t ldx = N > 1 ? static_cast<int64_t>(bs[1] / sizeof(float)) : K;
        const int64_t ldy = N > 1 ? static_cast<int64_t>(os[1] / sizeof(float)) : M;
        if ((N > 1 && (bs[1] % sizeof(float) || os[1] % sizeof(float))) || ldx < K || ldy < M)
            return error(Error::INVALID_ARGUMENT);
        if (qt > 0) {
            const size_t ws = hesa_cuda_qmatvec_workspace_size(qt, M, K, N);
            if (d_ws_.bytes < ws) {
                HESA_CHECK(ensure(d_ws_, ws));
                HESA_CHECK(from_cuda(cudaMemsetAsync(d_ws_.ptr, 0, d_ws_.bytes, s)));
            }
            return from_abi(hesa_cuda_qmatvec(qt, dev_w, M, K, static_cast<const float*>(b.data()), ldx, N,
                                              static_cast<float*>(out.data()), ldy, scale, d_ws_.ptr, d_ws_.bytes,
                                              s));
        }
        return from_abi(hesa_cuda_matmul_f32(static_cast<const float*>(dev_w), M, K,
                                             static_cast<const float*>(b.data()), ldx, N,
                                             static_cast<float*>(out.data()), ldy, scale, s));
    }
    if (on_device(b.data()) || on_device(out.data())) return error(Error::INVALID_ARGUMENT);   // mixed

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
        HESA_CHECK(from_abi(hesa_cuda_qmatvec(qt, dev_w, M, K, static_cast<const float*>(d_x_.ptr), K, N,
                                              static_cast<float*>(d_y_.ptr), M, scale, d_ws_.ptr, d_ws_.bytes, s)));
    } else {
        HESA_CHECK(from_abi(hesa_cuda_matmul_f32(static_cast<const float*>(dev_w), M, K,
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

Result<float*> CudaBackend::upload(const TensorView& v, int slot) {
    if (!contiguous_f32(v)) return fail_as<float*>(Error::INVALID_ARGUMENT);
    const size_t bytes = static_cast<size_t>(v.nelements()) * sizeof(float);
    auto r = ensure(scratch_[slot], bytes > 0 ? bytes : sizeof(float));
    if (!r) return std::unexpected{r.error()};
    if (bytes && cudaMemcpyAsync(scratch_[slot].ptr, v.data(), bytes, cudaMemcpyHostToDevice,
                                 static_cast<cudaStream_t>(stream_)) != cudaSuccess)
        return fail_as<float*>(Error::CUDA_ERROR);
    return static_cast<float*>(scratch_[slot].ptr);
}

Result<void> CudaBackend::download(int slot, TensorView& v) {
    if (!contiguous_f32(v)) return error(Error::INVALID_ARGUMENT);
    const size_t bytes = static_cast<size_t>(v.nelements()) * sizeof(float);
    cudaStream_t s = static_cast<cudaStream_t>(stream_);
    if (bytes) HESA_CHECK(from_cuda(cudaMemcpyAsync(v.data(), scratch_[slot].ptr, bytes, cudaMemcpyDeviceToHost, s)));
    return from_cuda(cudaStreamSynchronize(s));
}

Result<void> CudaBackend::add(TensorView a, TensorView b, TensorView out) {
    HESA_CHECK(activate());
    if (a.nelements() != b.nelements() || a.nelements() != out.nelements()) return error(Error::SHAPE_MISMATCH);
    if (a.nelements() == 0) return ok();
    auto da = upload(a, 0);
    if (!da) return std::unexpected{da.error()};
    auto db = upload(b, 1);
    if (!db) return std::unexpected{db.error()};
    HESA_CHECK(from_abi(hesa_cuda_add(*da, *db, *da, a.nelements(), stream_)));
    return download(0, out);
}

Result<void> CudaBackend::mul(TensorView a, TensorView b, TensorView out) {
    HESA_CHECK(activate());
    if (a.nelements() != b.nelements() || a.nelements() != out.nelements()) return error(Error::SHAPE_MISMATCH);
    if (a.nelements() == 0) return ok();
    auto da = upload(a, 0);
    if (!da) return std::unexpected{da.error()};
    auto db = upload(b, 1);
    if (!db) return std::unexpected{db.error()};
    HESA_CHECK(from_abi(hesa_cuda_mul(*da, *db, *da, a.nelements(), stream_)));
    return download(0, out);
}

Result<void> CudaBackend::silu(TensorView in, TensorView out) {
    HESA_CHECK(activate());
    if (in.nelements() != out.nelements()) return error(Error::SHAPE_MISMATCH);
    if (in.nelements() == 0) return ok();
    auto d = upload(in, 0);
    if (!d) return std::unexpected{d.error()};
    HESA_CHECK(from_abi(hesa_cuda_silu_mul(*d, nullptr, *d, in.nelements(), stream_)));
    return download(0, out);
}

Result<void> CudaBackend::softmax(TensorView in, TensorView out, int axis) {
    HESA_CHECK(activate());
    if (in.ndim() == 0 || in.nelements() != out.nelements()) return error(Error::SHAPE_MISMATCH);
    if (axis != -1 && axis != static_cast<int>(in.ndim()) - 1) return error(Error::BACKEND_NOT_AVAILABLE);
    if (in.nelements() == 0) return ok();
    const int64_t n = in.shape()[in.ndim() - 1];
    auto d = upload(in, 0);
    if (!d) return std::unexpected{d.error()};
    HESA_CHECK(from_abi(hesa_cuda_softmax(*d, *d, in.nelements() / n, n, stream_)));
    return download(0, out);
}

Result<void> CudaBackend::rms_norm(TensorView in, TensorView weight, TensorView out, float eps) {
    HESA_CHECK(activate());
    if (in.ndim() == 0 || in.nelements() != out.nelements()) return error(Error::SHAPE_MISMATCH);
    const int64_t n = in.shape()[in.ndim() - 1];
    if (static_cast<int64_t>(weight.nelements()) != n) return error(Error::SHAPE_MISMATCH);
    if (in.nelements() == 0) return ok();
    auto d = upload(in, 0);
    if (!d) return std::unexpected{d.error()};
    auto dw = upload(weight, 1);
    if (!dw) return std::unexpected{dw.error()};
    auto r = ensure(scratch_[2], static_cast<size_t>(in.nelements()) * sizeof(float));
    if (!r) return r;
    HESA_CHECK(from_abi(hesa_cuda_rms_norm(*d, *dw, static_cast<float*>(scratch_[2].ptr), in.nelements() / n, n,
                                           eps, stream_)));
    return download(2, out);
}

Result<void> CudaBackend::rope(TensorView in_out, std::span<const int32_t> positions, float freq_base, int n_dims) {
    HESA_CHECK(activate());
    if (in_out.ndim() < 3 || n_dims <= 0 || (n_dims & 1) || in_out.shape()[2] != n_dims)
        return error(Error::SHAPE_MISMATCH);
    const int64_t n_tokens = in_out.shape()[0], n_heads = in_out.shape()[1];
    if (!positions.empty() && static_cast<int64_t>(positions.size()) < n_tokens) return error(Error::SHAPE_MISMATCH);
    int32_t max_pos = 0;
    for (int64_t t = 0; t < n_tokens; ++t) {
        const int32_t p = positions.empty() ? static_cast<int32_t>(t) : positions[t];
        if (p < 0) return error(Error::INVALID_ARGUMENT);
        max_pos = std::max(max_pos, p);
    }
    // angle table rows 0 .. max_pos, with the CPU backend's own float formulas
    std::vector<float> table(static_cast<size_t>(max_pos + 1) * n_dims);
    HESA_CHECK(from_abi(hesa_cuda_rope_table(table.data(), max_pos + 1, n_dims, freq_base)));
    auto r = ensure(scratch_[3], table.size() * sizeof(float));
    if (!r) return r;
    cudaStream_t s = static_cast<cudaStream_t>(stream_);
    HESA_CHECK(from_cuda(cudaMemcpyAsync(scratch_[3].ptr, table.data(), table.size() * sizeof(float),
                                         cudaMemcpyHostToDevice, s)));
    auto d = upload(in_out, 0);
    if (!d) return std::unexpected{d.error()};
    for (int64_t t = 0; t < n_tokens; ++t) {
        const int32_t p = positions.empty() ? static_cast<int32_t>(t) : positions[t];
        HESA_CHECK(from_abi(hesa_cuda_rope(*d + t * n_heads * n_dims, n_heads, n_dims,
                                           static_cast<const float*>(scratch_[3].ptr), max_pos + 1, nullptr, p,
                                           stream_)));
    }
    return download(0, in_out);   // waits, so `table` outlives the copy
}

Result<void> CudaBackend::scaled_dot_product_attention(TensorView q, TensorView k, TensorView v, TensorView out,
                                                       TensorView mask, float scale) {
    HESA_CHECK(activate());
    if (mask.data() != nullptr) return error(Error::BACKEND_NOT_AVAILABLE);   // the CPU backend ignores it too
    if (q.ndim() != 3 || k.ndim() != 3 || v.ndim() != 3 || out.ndim() != 3) return error(Error::SHAPE_MISMATCH);
    const int64_t n_q = q.shape()[0], n_heads = q.shape()[1], d = q.shape()[2], n_k = k.shape()[0];
    if (k.shape()[1] != n_heads || k.shape()[2] != d || v.shape()[0] != n_k || v.shape()[1] != n_heads ||
        v.shape()[2] != d || out.shape()[0] != n_q || out.shape()[1] != n_heads || out.shape()[2] != d)
        return error(Error::SHAPE_MISMATCH);
    if (!contiguous_f32(q) || !contiguous_f32(k) || !contiguous_f32(v) || !contiguous_f32(out))
        return error(Error::INVALID_ARGUMENT);
    const float sc = scale > 0.0f ? scale : 1.0f / std::sqrt(static_cast<float>(d));
    // per head: scores = sc * Q_h K_h^T (matmul with a = K_h [n_k, d]),
    // softmax over keys, out_h = P V_h (matmul with a = V_h^T [d, n_k])
    const float* hq = static_cast<const float*>(q.data());
    const float* hk = static_cast<const float*>(k.data());
    const float* hv = static_cast<const float*>(v.data());
    float* ho = static_cast<float*>(out.data());
    std::vector<float> qh(static_cast<size_t>(n_q) * d), kh(static_cast<size_t>(n_k) * d),
        vt(static_cast<size_t>(d) * n_k), oh(static_cast<size_t>(n_q) * d);
    const size_t bq = qh.size() * 4, bk = kh.size() * 4, bs = static_cast<size_t>(n_q) * n_k * 4;
    for (int slot : {0, 1, 2, 4})
        if (auto r = ensure(scratch_[slot], slot == 0 ? bq : slot == 1 ? bk : slot == 2 ? bs : bq); !r) return r;
    if (auto r = ensure(scratch_[5], bk); !r) return r;
    cudaStream_t s = static_cast<cudaStream_t>(stream_);
    float* dq = static_cast<float*>(scratch_[0].ptr);
    float* dk = static_cast<float*>(scratch_[1].ptr);
    float* ds = static_cast<float*>(scratch_[2].ptr);
    float* dout = static_cast<float*>(scratch_[4].ptr);
    float* dvt = static_cast<float*>(scratch_[5].ptr);
    for (int64_t h = 0; h < n_heads; ++h) {
        for (int64_t i = 0; i < n_q; ++i)
            std::memcpy(&qh[i * d], hq + (i * n_heads + h) * d, d * 4);
        for (int64_t j = 0; j < n_k; ++j) {
            std::memcpy(&kh[j * d], hk + (j * n_heads + h) * d, d * 4);
            for (int64_t e = 0; e < d; ++e) vt[e * n_k + j] = hv[(j * n_heads + h) * d + e];
        }
        HESA_CHECK(from_cuda(cudaMemcpyAsync(dq, qh.data(), bq, cudaMemcpyHostToDevice, s)));
        HESA_CHECK(from_cuda(cudaMemcpyAsync(dk, kh.data(), bk, cudaMemcpyHostToDevice, s)));
        HESA_CHECK(from_cuda(cudaMemcpyAsync(dvt, vt.data(), bk, cudaMemcpyHostToDevice, s)));
        HESA_CHECK(from_abi(hesa_cuda_matmul_f32(dk, n_k, d, dq, d, n_q, ds, n_k, sc, stream_)));
        HESA_CHECK(from_abi(hesa_cuda_softmax(ds, ds, n_q, n_k, stream_)));
        HESA_CHECK(from_abi(hesa_cuda_matmul_f32(dvt, d, n_k, ds, n_k, n_q, dout, d, 1.0f, stream_)));
        HESA_CHECK(from_cuda(cudaMemcpyAsync(oh.data(), dout, bq, cudaMemcpyDeviceToHost, s)));
        HESA_CHECK(from_cuda(cudaStreamSynchronize(s)));   // host staging is reused by the next head
        for (int64_t i = 0; i < n_q; ++i) std::memcpy(ho + (i * n_heads + h) * d, &oh[i * d], d * 4);
    }
    return ok();
}

Result<Tensor> CudaBackend::quantize(TensorView src, Dtype target_dtype) {
    auto a = activate();
    if (!a) return std::unexpected{a.error()};
    const int qt = qtype_of(target_dtype);
    if (qt <= 0) return fail_as<Tensor>(Error::BACKEND_NOT_AVAILABLE);
    if (src.ndim() != 2 || !contiguous_f32(src)) return fail_as<Tensor>(Error::INVALID_ARGUMENT);
    const int64_t rows = src.shape()[0], k = src.shape()[1];
    const size_t rb = hesa_cuda_row_bytes(qt, k);
    if (rb == 0) return fail_as<Tensor>(Error::SHAPE_MISMATCH);
    // a quantized Tensor holds one byte per element (dtype_size 1,
    // src/tensor/tensor.cpp:28-37): enough for the packed rows of every type
    // but Q8_0, whose 34-byte blocks of 32 need 17/16 bytes per element (the
    // reference loader truncates Q8_0 rows to that size, gguf_loader.cpp:305-309)
    if (rb * static_cast<size_t>(rows) > static_cast<size_t>(rows * k)) return fail_as<Tensor>(Error::INVALID_FORMAT);
    auto d = upload(src, 0);
    if (!d) return std::unexpected{d.error()};
    if (auto r = ensure(scratch_[1], rb * rows); !r) return std::unexpected{r.error()};
    if (const int rc = hesa_cuda_quantize(qt, *d, rows, k, k, scratch_[1].ptr, stream_); rc != 0)
        return fail_as<Tensor>(static_cast<Error>(rc));
    // the packed rows go at the start of the Tensor, as Model::load puts them
    const int64_t shape[2] = {rows, k};
    Tensor t(target_dtype, std::span<const int64_t>(shape, 2), this);
    if (t.nbytes() < rb * rows) return fail_as<Tensor>(Error::INTERNAL_ERROR);
    cudaStream_t s = static_cast<cudaStream_t>(stream_);
    if (cudaMemcpyAsync(t.data(), scratch_[1].ptr, rb * rows, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return fail_as<Tensor>(Error::CUDA_ERROR);
    return std::move(t);
}

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
