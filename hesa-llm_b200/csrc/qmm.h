// qmm.h -- host launcher of the batched tensor-core matmul (qmm_tc.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace hesa_cuda {

// Batched matvec on the 5th-generation tensor cores (tcgen05 / TMEM / TMA,
// qmm_tc.cu): y[b * ldy + i] = scale * sum_k deq(W[i, k]) x[b * ldx + k] for
// b < batch, one launch per 16 activation rows. Q4_K / Q5_K weights, k a
// multiple of 256, batch >= 2, W 16-byte aligned. Workspace: zero-filled
// before first use; its counters are left at zero on success.
bool qmm_tc_eligible(int qtype, const void* w, int64_t n_out, int64_t k, int64_t batch);
size_t qmm_tc_workspace_bytes(int qtype, int64_t n_out, int64_t k, int64_t batch);
cudaError_t qmm_tc(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, int64_t ldx, int64_t batch,
                   float* y, int64_t ldy, float scale, void* workspace, cudaStream_t stream);

// The same for Q8_0 / Q4_0 weights (qmm_tc_blk.cu): one tcgen05 MMA per 32-weight
// block, the fp16 block scales applied in fp32 afterwards; one launch per 8
// activation rows.
bool qmm_blk_eligible(int qtype, const void* w, int64_t n_out, int64_t k, int64_t batch);
size_t qmm_blk_workspace_bytes(int qtype, int64_t n_out, int64_t k, int64_t batch);
cudaError_t qmm_blk(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, int64_t ldx, int64_t batch,
                    float* y, int64_t ldy, float scale, void* workspace, cudaStream_t stream);

}  // namespace hesa_cuda
