// ref_shim.cpp -- extern "C" entry points over hesa-llm's own CPU kernels.
//
// TEST INFRASTRUCTURE ONLY. Compiled (by oracle/build.py) together with the
// reference's src/backend/cpu_backend.cpp and src/tensor/tensor.cpp into
// oracle/_ref/libhesa_ref.so, so the tests can pin the oracle against the
// reference's own arithmetic and bench.py can time the reference's CPU path.
// Nothing here reimplements a kernel: every function forwards to hesa::*.
#include "hesa/backend.hpp"

#include <cstdint>
#include <thread>
#include <vector>

extern "C" {

// hesa::cpu_matmul_f32 (src/backend/cpu_backend.cpp:24-41): C = scale * A @ B.
void ref_cpu_matmul_f32(const float* a, const float* b, float* out,
                        int M, int N, int K, float scale) {
    hesa::cpu_matmul_f32(a, b, out, M, N, K, scale);
}

// The reference's matmul applied as a matvec over row slices from n_threads
// host threads: rows [i0, i1) of A go to thread t. Each call is the
// reference's own scalar kernel on a contiguous row range, so per-row results
// are identical to one single-threaded call.
void ref_cpu_matvec_mt(const float* a, const float* x, float* y,
                       int M, int K, float scale, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads == 1) {
        hesa::cpu_matmul_f32(a, x, y, M, 1, K, scale);
        return;
    }
    std::vector<std::thread> pool;
    pool.reserve(static_cast<size_t>(n_threads));
    for (int t = 0; t < n_threads; ++t) {
        const int i0 = static_cast<int>(static_cast<int64_t>(M) * t / n_threads);
        const int i1 = static_cast<int>(static_cast<int64_t>(M) * (t + 1) / n_threads);
        if (i1 <= i0) continue;
        pool.emplace_back([=] {
            hesa::cpu_matmul_f32(a + static_cast<int64_t>(i0) * K, x, y + i0, i1 - i0, 1, K, scale);
        });
    }
    for (auto& th : pool) th.join();
}

void ref_cpu_rms_norm_f32(const float* in, const float* w, float* out,
                          size_t n_rows, size_t row_size, float eps) {
    hesa::cpu_rms_norm_f32(in, w, out, n_rows, row_size, eps);
}

void ref_cpu_silu_f32(const float* in, float* out, size_t n) {
    hesa::cpu_silu_f32(in, out, n);
}

void ref_cpu_softmax_f32(const float* in, float* out, size_t n_rows, size_t row_size) {
    hesa::cpu_softmax_f32(in, out, n_rows, row_size);
}

void ref_cpu_rope_f32(float* data, const int32_t* positions, size_t n_tokens,
                      size_t n_heads, size_t head_dim, float freq_base) {
    hesa::cpu_rope_f32(data, positions, n_tokens, n_heads, head_dim, freq_base);
}

}  // extern "C"
