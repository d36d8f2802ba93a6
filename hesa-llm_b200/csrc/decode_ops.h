// decode_ops.h -- host launchers of the decode-step kernels (decode_ops.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "peer_sync.cuh"

namespace hesa_cuda {

cudaError_t matmul_f32(const float* a, int64_t n_out, int64_t k, const float* x, int64_t ldx, int64_t batch,
                       float* y, int64_t ldy, float scale, cudaStream_t s);
cudaError_t rms_norm(const float* in, const float* w, float* out, int64_t n_rows, int64_t n, float eps,
                     cudaStream_t s);
cudaError_t silu_mul(const float* g, const float* u, float* o, int64_t n, cudaStream_t s);
cudaError_t binary(const float* a, const float* b, float* o, int64_t n, int op /*0 add, 1 mul*/,
                   cudaStream_t s);
cudaError_t softmax(const float* in, float* out, int64_t n_rows, int64_t n, cudaStream_t s);
cudaError_t rope(float* data, int64_t n_heads, int64_t head_dim, const float* table, int32_t table_rows,
                 const int32_t* pos_dev, int32_t pos_host, cudaStream_t s);
cudaError_t kv_store(const float* k, const float* v, void* kc, void* vc, int64_t row_elems, int64_t ctx,
                     const int32_t* pos_dev, int32_t pos_host, cudaStream_t s);
// rope(q) in place, rope(k), then k and v as fp16 into slot *pos_dev % ctx.
cudaError_t rope_kv(float* q, const float* k, const float* v, void* kc, void* vc, int64_t n_head, int64_t n_kv_head,
                    int64_t head_dim, const float* table, int32_t table_rows, int64_t ctx, const int32_t* pos_dev,
                    cudaStream_t s);
int attention_splits(int64_t ctx);
size_t attention_workspace_bytes(int64_t n_head, int64_t head_dim, int64_t ctx);
cudaError_t attention(const float* q, const void* kc, const void* vc, float* out, int64_t n_head,
                      int64_t n_kv_head, int64_t head_dim, int64_t ctx, const int32_t* pos_dev, int32_t pos_host,
                      void* workspace, cudaStream_t s);
// rope_kv followed by attention in one launch (the decode step's form): q and
// k_new unrotated, this token's k and v written to slot *pos_dev % ctx; a
// position outside the rope table records device status 3 and computes
// nothing.
cudaError_t attention_rope(const float* q, const float* k_new, const float* v_new, void* kc, void* vc, float* out,
                           int64_t n_head, int64_t n_kv_head, int64_t head_dim, const float* table,
                           int32_t table_rows, int64_t ctx, const int32_t* pos_dev, void* workspace,
                           cudaStream_t s);
// attention_rope of this rank's heads in a head-sharded decode step: element
// h * head_dim + d of its output is element peer_off + h * head_dim + d of the
// tagged vector at peer_out[p] on every rank p (tag (*ll_count << 12) | ll_lo;
// element order as peer_sync.cuh).
cudaError_t attention_rope_shard(const float* q, const float* k_new, const float* v_new, void* kc, void* vc,
                                 float* out, int64_t n_head, int64_t n_kv_head, int64_t head_dim, const float* table,
                                 int32_t table_rows, int64_t ctx, const int32_t* pos_dev, void* workspace,
                                 uint64_t* const* peer_out, int64_t peer_off, int peer_world,
                                 const uint32_t* ll_count, uint32_t ll_lo, cudaStream_t s);

}  // namespace hesa_cuda
