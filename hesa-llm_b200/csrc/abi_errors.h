// abi_errors.h -- the C ABI's per-thread error message (abi.cu), for entry
// points defined in other files.
#pragma once

#include <cuda_runtime.h>

namespace hesa_cuda {

// Keep `what` as this host thread's last error message; return `code`.
int record_error(int code, const char* what);
// "<where>: <CUDA error string>"; returns HESA_CUDA_ERROR.
int record_cuda_error(cudaError_t e, const char* where);

}  // namespace hesa_cuda
