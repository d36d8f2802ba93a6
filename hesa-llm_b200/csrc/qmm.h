// qmm.h -- host launcher of the batched tensor-core matmul (qmm.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace hesa_cuda {

// Q4_K / Q5_K weights, k a multiple of 256, batch >= 2, W 16-byte aligned.
bool qmm_eligible(int qtype, const void* w, int64_t n_out, int64_t k, int64_t batch);
// Workspace bytes (zero-filled before first use; left zero-filled on success),
// 0 for a type the kernel does not take.
size_t qmm_workspace_bytes(int qtype, int64_t n_out, int64_t k, int64_t batch);
// y[b * ldy + i] = scale * sum_k deq(W[i, k]) x[b * ldx + k] for b < batch:
// two launches per 16 activation rows (staging, then the matmul).
cudaError_t qmm(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, int64_t ldx, int64_t batch,
                float* y, int64_t ldy, float scale, void* workspace, cudaStream_t stream);

// The same on the 5th-generation tensor cores (tcgen05 / TMEM / TMA,
// qmm_tc.cu): one launch per 16 activation rows.
bool qmm_tc_eligible(int qtype, const void* w, int64_t n_out, int64_t k, int64_t batch);
size_t qmm_tc_workspace_bytes(int qtype, int64_t n_out, int64_t k, int64_t batch);
cudaError_t qmm_tc(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, int64_t ldx, int64_t batch,
                   float* y, int64_t ldy, float scale, void* workspace, cudaStream_t stream);

}  // namespace hesa_cuda
