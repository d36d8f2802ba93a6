/*
 * hesa_cuda.h -- C ABI of the B200 (sm_100a) CUDA backend for hesa-llm's
 * decode hot path: GGUF block-quantized weight x fp32 activation matvec with
 * fused dequantization.
 *
 * Conventions shared by every entry point:
 *   - Pointers are device pointers unless a parameter says "host". The
 *     library never allocates or frees device memory on these paths; the
 *     caller owns every buffer, including the workspace.
 *   - Weights W are row-major [n_out, k]: each row is k/block_elems packed
 *     GGUF blocks, rows back to back (the layout Model::load produces after
 *     reversing the GGUF dims, src/model/gguf_loader.cpp:291-316). W must be
 *     16-byte aligned.
 *   - qtype is the GGUF/ggml type id (src/model/gguf_loader.hpp:15-45):
 *     Q4_0 = 2, Q8_0 = 8, Q4_K = 12, Q5_K = 13, Q6_K = 14.
 *   - Return value: 0 on success, else a hesa::Error value
 *     (include/hesa/result.hpp:14-30): INVALID_ARGUMENT = 2,
 *     BACKEND_NOT_AVAILABLE = 3, SHAPE_MISMATCH = 6, INVALID_FORMAT = 8,
 *     CUDA_ERROR = 9, INTERNAL_ERROR = 14. Nothing throws across the ABI.
 *   - Calls are asynchronous on `stream` (a cudaStream_t; NULL is the legacy
 *     default stream).
 */
#ifndef HESA_CUDA_H
#define HESA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define HESA_CUDA_API __attribute__((visibility("default")))
#else
#define HESA_CUDA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum hesa_cuda_qtype {
    HESA_CUDA_Q4_0 = 2,
    HESA_CUDA_Q8_0 = 8,
    HESA_CUDA_Q4_K = 12,
    HESA_CUDA_Q5_K = 13,
    HESA_CUDA_Q6_K = 14
};

enum hesa_cuda_status {
    HESA_CUDA_OK = 0,
    HESA_CUDA_INVALID_ARGUMENT = 2,
    HESA_CUDA_BACKEND_NOT_AVAILABLE = 3,
    HESA_CUDA_SHAPE_MISMATCH = 6,
    HESA_CUDA_INVALID_FORMAT = 8,
    HESA_CUDA_ERROR = 9,
    HESA_CUDA_INTERNAL_ERROR = 14
};

/* Library version and the device architecture the kernels were built for
 * ("sm_100a"). */
HESA_CUDA_API const char* hesa_cuda_version(void);

/* Bytes of one packed row of k weights of qtype (0 if k is not a multiple of
 * the block size or qtype is unsupported). Mirrors gguf_type_size
 * (src/model/gguf_loader.cpp:19-38) for one row. */
HESA_CUDA_API size_t hesa_cuda_row_bytes(int qtype, int64_t k);

/* Device workspace the matvec needs for n_out x k at this batch, in bytes
 * (cross-warp partial sums and arrival counters). The workspace must be
 * zero-filled once before its first use; every successful call leaves it
 * zero-filled again, so it can be reused by later calls on the same stream.
 * After a call that reports HESA_CUDA_ERROR, zero it again. */
HESA_CUDA_API size_t hesa_cuda_qmatvec_workspace_size(int qtype, int64_t n_out, int64_t k, int64_t batch);

/* y[b*ldy + n] = scale * sum_k deq(W[n,k]) * x[b*ldx + k]
 * for n < n_out, b < batch. fp32 activations and outputs.
 *
 * Replaces, for quantized `a`, hesa::Backend::matmul(TensorView a,
 * TensorView b, TensorView out, float scale) (include/hesa/backend.hpp:43-44)
 * whose CPU semantics are cpu_matmul_f32 (src/backend/cpu_backend.cpp:24-41):
 * a = W [n_out, k], b = x^T [k, batch], out = y^T [n_out, batch].
 * batch >= 8 runs on the tensor-core tile path; smaller batches on CUDA cores.
 * x and y must be 16-byte aligned with ldx, ldy multiples of 4. */
HESA_CUDA_API int hesa_cuda_qmatvec(int qtype, const void* w, int64_t n_out, int64_t k,
                                    const float* x, int64_t ldx, int64_t batch,
                                    float* y, int64_t ldy, float scale,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* out[r*ldo + i] = deq(W[r, i]) for r < n_rows, i < k: the exact fp32 value
 * of every weight, bit-identical to the GGUF definition ((d*sc)*q - dmin*m
 * with each operation rounded separately). Used for embedding-row lookups
 * and as the bit-exactness check of the decoders. Replaces nothing in the
 * reference (it has no dequantizer; CPU_Backend::quantize is a stub,
 * src/backend/cpu_backend.cpp:296-302). */
HESA_CUDA_API int hesa_cuda_dequantize(int qtype, const void* w, int64_t n_rows, int64_t k,
                                       float* out, int64_t ldo, void* stream);

/* Sticky device-side status of the kernels' bounded waits: 0 when no wait
 * has ever timed out in this process, else a nonzero code naming the wait.
 * Reading synchronizes `stream`. hesa_cuda_clear_device_status resets it. */
HESA_CUDA_API int hesa_cuda_device_status(void* stream, int* status_out);
HESA_CUDA_API int hesa_cuda_clear_device_status(void* stream);

/* Last error message recorded on this host thread ("" if none). */
HESA_CUDA_API const char* hesa_cuda_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
