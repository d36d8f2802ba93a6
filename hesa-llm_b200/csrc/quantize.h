// quantize.h -- host-side launcher of the GGUF block quantizer (quantize.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace hesa_cuda {

// dst (packed rows, n_rows * row_bytes(qtype, k)) <- blocks of src [n_rows, k]
// (row stride ld floats), deterministic round-to-nearest.
cudaError_t quantize(int qtype, const float* src, int64_t n_rows, int64_t k, int64_t ld, void* dst,
                     cudaStream_t stream);

}  // namespace hesa_cuda
