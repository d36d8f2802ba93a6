// abi.cu -- the extern "C" entry points declared in include/hesa_cuda.h.
//
// Validation happens here, on the host, before anything is launched: bad
// qtype, shape, stride, alignment or null pointer return an error code and
// launch nothing. CUDA errors map to HESA_CUDA_ERROR with the message kept
// per host thread.
#include "../../include/hesa_cuda.h"
#include "qmatvec.h"
#include "qtypes.cuh"

#include <string>

namespace {

thread_local std::string t_last_error;

int fail(int code, const char* what) {
    t_last_error = what;
    return code;
}

int cuda_fail(cudaError_t e, const char* where) {
    t_last_error = std::string(where) + ": " + cudaGetErrorString(e);
    return HESA_CUDA_ERROR;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

const char* hesa_cuda_version(void) { return "hesa-b200 0.1 sm_100a"; }

const char* hesa_cuda_last_error(void) { return t_last_error.c_str(); }

size_t hesa_cuda_row_bytes(int qtype, int64_t k) {
    const int be = hesa_cuda::block_elems(qtype);
    if (be == 0 || k <= 0 || k % be != 0) return 0;
    return static_cast<size_t>(k / be) * static_cast<size_t>(hesa_cuda::block_bytes(qtype));
}

size_t hesa_cuda_qmatvec_workspace_size(int qtype, int64_t n_out, int64_t k, int64_t batch) {
    (void)batch;
    if (!hesa_cuda::qtype_supported(qtype) || n_out <= 0 || k <= 0) return 0;
    return hesa_cuda::qmv_workspace_bytes(static_cast<int>(n_out));
}

int hesa_cuda_qmatvec(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, int64_t ldx,
                      int64_t batch, float* y, int64_t ldy, float scale, void* workspace,
                      size_t workspace_bytes, void* stream) {
    if (!hesa_cuda::qtype_supported(qtype)) return fail(HESA_CUDA_BACKEND_NOT_AVAILABLE, "unsupported qtype");
    if (!w || !x || !y) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (n_out <= 0 || k <= 0 || batch <= 0) return fail(HESA_CUDA_SHAPE_MISMATCH, "non-positive dimension");
    if (n_out >= (int64_t(1) << 31) || k >= (int64_t(1) << 31))
        return fail(HESA_CUDA_SHAPE_MISMATCH, "dimension too large");
    if (k % hesa_cuda::block_elems(qtype) != 0)
        return fail(HESA_CUDA_SHAPE_MISMATCH, "k is not a multiple of the block size");
    if (ldx < k || (batch > 1 && ldy < n_out)) return fail(HESA_CUDA_SHAPE_MISMATCH, "leading dimension too small");
    if (!aligned16(w)) return fail(HESA_CUDA_INVALID_ARGUMENT, "weights must be 16-byte aligned");
    if (!aligned16(x) || !aligned16(y) || (ldx & 3) || (batch > 1 && (ldy & 3)))
        return fail(HESA_CUDA_INVALID_ARGUMENT, "x / y must be 16-byte aligned with ldx, ldy multiples of 4");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    if (hesa_cuda::qmv_stream_eligible(w, n_out, k)) {
        const size_t need = hesa_cuda::qmv_workspace_bytes(static_cast<int>(n_out));
        if (!workspace || workspace_bytes < need) return fail(HESA_CUDA_INVALID_ARGUMENT, "workspace too small");
        if (!aligned16(workspace)) return fail(HESA_CUDA_INVALID_ARGUMENT, "workspace must be 16-byte aligned");
        for (int64_t b = 0; b < batch; ++b) {
            e = hesa_cuda::qmv_stream(qtype, w, n_out, k, x + b * ldx, y + b * ldy, scale, workspace, s, 0);
            if (e != cudaSuccess) return cuda_fail(e, "qmatvec stream kernel");
        }
    } else {
        e = hesa_cuda::qmv_rowwise(qtype, w, n_out, k, x, ldx, batch, y, ldy, scale, s);
        if (e != cudaSuccess) return cuda_fail(e, "qmatvec rowwise kernel");
    }
    return HESA_CUDA_OK;
}

int hesa_cuda_dequantize(int qtype, const void* w, int64_t n_rows, int64_t k, float* out, int64_t ldo,
                         void* stream) {
    if (!hesa_cuda::qtype_supported(qtype)) return fail(HESA_CUDA_BACKEND_NOT_AVAILABLE, "unsupported qtype");
    if (!w || !out) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (n_rows <= 0 || k <= 0 || k % hesa_cuda::block_elems(qtype) != 0 || ldo < k)
        return fail(HESA_CUDA_SHAPE_MISMATCH, "bad shape");
    cudaError_t e = hesa_cuda::dequantize(qtype, w, n_rows, k, out, ldo, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "dequantize kernel");
    return HESA_CUDA_OK;
}

int hesa_cuda_device_status(void* stream, int* status_out) {
    if (!status_out) return fail(HESA_CUDA_INVALID_ARGUMENT, "null status pointer");
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "synchronize");
    int v = 0;
    e = hesa_cuda::read_device_status(&v);
    if (e != cudaSuccess) return cuda_fail(e, "read device status");
    *status_out = v;
    return HESA_CUDA_OK;
}

int hesa_cuda_clear_device_status(void* stream) {
    cudaError_t e = hesa_cuda::clear_device_status(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "clear device status");
    return HESA_CUDA_OK;
}

}  // extern "C"
