// test_cuda_backend.cpp -- hesa::CudaBackend against hesa-llm's own CPU_Backend.
//
// Built by tests/test_cuda_backend_gpu.py together with the reference's
// Tensor and CPU_Backend sources (src/tensor/tensor.cpp,
// src/backend/cpu_backend.cpp) and the oracle's C quantizer. Every op of the
// Backend interface (include/hesa/backend.hpp:38-64) runs on both backends on
// the same seeded inputs:
//   * matmul of quantized weights: CudaBackend on the packed GGUF rows,
//     CPU_Backend on the same rows dequantized to F32; rel-L2 <= 1e-5
//   * matmul F32, softmax, rms_norm, silu, attention: rel-L2 <= 1e-5
//   * add, mul, rope: bit-exact
//   * quantize: byte-exact against the oracle's quantizer (the CPU backend
//     returns BACKEND_NOT_AVAILABLE for it, cpu_backend.cpp:296-302); Q8_0
//     rows do not fit a one-byte-per-element Tensor and are refused
// plus the weight cache, shape checks and error codes.
// Prints one line per check and exits non-zero when any fails.
#include "backend/cuda_backend.hpp"
#include "backend/cpu_backend.hpp"
#include "hesa_oracle.h"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

using namespace hesa;

namespace {

int g_failed = 0;

void report(const std::string& name, bool pass, const std::string& detail = {}) {
    std::printf("%s %s%s%s\n", pass ? "PASS" : "FAIL", name.c_str(), detail.empty() ? "" : ": ", detail.c_str());
    if (!pass) ++g_failed;
}

std::vector<float> gaussian(size_t n, float sigma, unsigned seed) {
    std::mt19937 rng(seed);
    std::normal_distribution<float> d(0.0f, sigma);
    std::vector<float> v(n);
    for (auto& x : v) x = d(rng);
    return v;
}

double rel_l2(const float* a, const float* b, size_t n) {
    double num = 0, den = 0;
    for (size_t i = 0; i < n; ++i) {
        const double e = double(a[i]) - double(b[i]);
        num += e * e;
        den += double(b[i]) * double(b[i]);
    }
    return den > 0 ? std::sqrt(num / den) : std::sqrt(num);
}

bool bit_equal(const float* a, const float* b, size_t n) { return std::memcmp(a, b, n * sizeof(float)) == 0; }

std::string fmt(double v) {
    char buf[32];
    std::snprintf(buf, sizeof buf, "%.3e", v);
    return buf;
}

TensorView f32(std::vector<float>& v, Shape s) { return TensorView(v.data(), Dtype::F32, s); }

Dtype dtype_of(int qt) {
    switch (qt) {
        case 2: return Dtype::Q4_0;
        case 8: return Dtype::Q8_0;
        case 12: return Dtype::Q4_K;
        case 13: return Dtype::Q5_K;
        default: return Dtype::Q6_K;
    }
}

const char* qname(int qt) {
    switch (qt) {
        case 2: return "Q4_0";
        case 8: return "Q8_0";
        case 12: return "Q4_K";
        case 13: return "Q5_K";
        default: return "Q6_K";
    }
}

// packed rows of W [n_out, k] and their F32 dequantization
struct QWeights {
    std::vector<uint8_t> packed;
    std::vector<float> deq;
};

QWeights make_weights(int qt, int64_t n_out, int64_t k, unsigned seed) {
    QWeights w;
    const size_t rb = oracle_row_bytes(qt, k);
    const auto src = gaussian(size_t(n_out * k), 0.02f, seed);
    w.packed.resize(rb * n_out);
    w.deq.resize(size_t(n_out * k));
    for (int64_t r = 0; r < n_out; ++r) {
        oracle_quantize_row(qt, &src[size_t(r * k)], &w.packed[rb * r], k);
        oracle_dequantize_row(qt, &w.packed[rb * r], &w.deq[size_t(r * k)], k);
    }
    return w;
}

void test_matmul_quantized(CudaBackend& gpu, CPU_Backend& cpu) {
    const int64_t n_out = 300, k = 512;
    for (int qt : {2, 8, 12, 13, 14}) {
        QWeights w = make_weights(qt, n_out, k, 100 + qt);
        // the packed rows as the reference's Model::load leaves them: a
        // quantized [n_out, k] view whose data() is the packed bytes
        TensorView wq(w.packed.data(), dtype_of(qt), Shape{n_out, k});
        TensorView wf(w.deq.data(), Dtype::F32, Shape{n_out, k});
        for (int64_t batch : {1, 3}) {
            // activations [batch, k] as the model holds them, passed as the
            // transposed [k, batch] view the matmul contract takes
            auto x = gaussian(size_t(batch * k), 1.0f, 7 + unsigned(batch));
            Tensor xt(Dtype::F32, Shape{batch, k});
            std::memcpy(xt.data(), x.data(), x.size() * 4);
            TensorView xv = xt.transpose(0, 1);
            // the CPU backend reads b as a contiguous [k, batch] array
            // (cpu_backend.cpp:146-160), so it gets an explicit transpose
            std::vector<float> xkb(x.size());
            for (int64_t j = 0; j < batch; ++j)
                for (int64_t i = 0; i < k; ++i) xkb[size_t(i * batch + j)] = x[size_t(j * k + i)];
            std::vector<float> got(size_t(n_out * batch)), want(got.size());
            auto rg = gpu.matmul(wq, xv, f32(got, Shape{n_out, batch}), 0.5f);
            auto rc = cpu.matmul(wf, f32(xkb, Shape{k, batch}), f32(want, Shape{n_out, batch}), 0.5f);
            const std::string name = std::string("matmul ") + qname(qt) + " batch " + std::to_string(batch);
            if (!rg || !rc) {
                report(name, false, "call failed");
                continue;
            }
            const double e = rel_l2(got.data(), want.data(), got.size());
            report(name, e <= 1e-5, "rel-L2 " + fmt(e));
        }
    }
}

void test_matmul_f32(CudaBackend& gpu, CPU_Backend& cpu) {
    const int64_t n_out = 96, k = 200, batch = 2;
    auto a = gaussian(size_t(n_out * k), 0.05f, 31);
    auto x = gaussian(size_t(k * batch), 1.0f, 32);
    std::vector<float> got(size_t(n_out * batch)), want(got.size());
    auto rg = gpu.matmul(f32(a, Shape{n_out, k}), f32(x, Shape{k, batch}), f32(got, Shape{n_out, batch}));
    auto rc = cpu.matmul(f32(a, Shape{n_out, k}), f32(x, Shape{k, batch}), f32(want, Shape{n_out, batch}));
    const double e = rel_l2(got.data(), want.data(), got.size());
    report("matmul F32", rg && rc && e <= 1e-5, "rel-L2 " + fmt(e));
}

void test_elementwise(CudaBackend& gpu, CPU_Backend& cpu) {
    const int64_t n = 3 * 1000 + 7;
    auto a = gaussian(size_t(n), 2.0f, 41), b = gaussian(size_t(n), 2.0f, 42);
    std::vector<float> got(static_cast<size_t>(n)), want(static_cast<size_t>(n));
    const Shape s{3, 1002};   // 3006 elements
    std::vector<float> a3(a.begin(), a.begin() + 3006), b3(b.begin(), b.begin() + 3006), g3(3006), w3(3006);

    auto r1 = gpu.add(f32(a3, s), f32(b3, s), f32(g3, s));
    cpu.add(f32(a3, s), f32(b3, s), f32(w3, s));
    report("add", r1.has_value() && bit_equal(g3.data(), w3.data(), 3006));

    auto r2 = gpu.mul(f32(a3, s), f32(b3, s), f32(g3, s));
    cpu.mul(f32(a3, s), f32(b3, s), f32(w3, s));
    report("mul", r2.has_value() && bit_equal(g3.data(), w3.data(), 3006));

    auto r3 = gpu.silu(f32(a, Shape{n}), f32(got, Shape{n}));
    cpu.silu(f32(a, Shape{n}), f32(want, Shape{n}));
    const double es = rel_l2(got.data(), want.data(), got.size());
    report("silu", r3.has_value() && es <= 1e-5, "rel-L2 " + fmt(es));

    auto r4 = gpu.softmax(f32(a3, s), f32(g3, s));
    cpu.softmax(f32(a3, s), f32(w3, s));
    const double ex = rel_l2(g3.data(), w3.data(), 3006);
    report("softmax", r4.has_value() && ex <= 1e-5, "rel-L2 " + fmt(ex));

    auto wn = gaussian(1002, 1.0f, 43);
    auto r5 = gpu.rms_norm(f32(a3, s), f32(wn, Shape{1002}), f32(g3, s), 1e-6f);
    cpu.rms_norm(f32(a3, s), f32(wn, Shape{1002}), f32(w3, s), 1e-6f);
    const double er = rel_l2(g3.data(), w3.data(), 3006);
    report("rms_norm", r5.has_value() && er <= 1e-5, "rel-L2 " + fmt(er));

    // empty tensors are a no-op, as on the CPU
    std::vector<float> none;
    report("add empty", gpu.add(f32(none, Shape{0}), f32(none, Shape{0}), f32(none, Shape{0})).has_value());
}

void test_rope(CudaBackend& gpu, CPU_Backend& cpu) {
    const int64_t n_tokens = 5, n_heads = 4, hd = 128;
    auto x = gaussian(size_t(n_tokens * n_heads * hd), 1.0f, 51);
    auto y = x;
    const std::vector<int32_t> pos = {0, 1, 17, 1000, 4095};
    const Shape s{n_tokens, n_heads, hd};
    auto rg = gpu.rope(f32(x, s), pos, 10000.0f, int(hd));
    cpu.rope(f32(y, s), pos, 10000.0f, int(hd));
    report("rope positions", rg.has_value() && bit_equal(x.data(), y.data(), x.size()));

    auto x2 = gaussian(size_t(3 * 2 * 64), 1.0f, 52);
    auto y2 = x2;
    const Shape s2{3, 2, 64};
    auto rg2 = gpu.rope(f32(x2, s2), {}, 500000.0f, 64);
    cpu.rope(f32(y2, s2), {}, 500000.0f, 64);
    report("rope default positions", rg2.has_value() && bit_equal(x2.data(), y2.data(), x2.size()));

    auto r3 = gpu.rope(f32(x2, s2), {}, 10000.0f, 32);
    report("rope n_dims != head_dim rejected", !r3 && r3.error() == make_error_code(Error::SHAPE_MISMATCH));
}

void test_attention(CudaBackend& gpu, CPU_Backend& cpu) {
    struct Case {
        int64_t n_q, n_k, heads, d;
        float scale;
    };
    for (Case c : {Case{1, 37, 4, 64, 0.0f}, Case{6, 200, 2, 128, 0.0f}, Case{3, 9, 3, 32, 0.25f}}) {
        auto q = gaussian(size_t(c.n_q * c.heads * c.d), 1.0f, 61);
        auto kk = gaussian(size_t(c.n_k * c.heads * c.d), 1.0f, 62);
        auto v = gaussian(size_t(c.n_k * c.heads * c.d), 1.0f, 63);
        std::vector<float> got(q.size(), 123.0f), want(q.size(), 0.0f);   // the CPU version accumulates into out
        const Shape sq{c.n_q, c.heads, c.d}, sk{c.n_k, c.heads, c.d};
        auto rg = gpu.scaled_dot_product_attention(f32(q, sq), f32(kk, sk), f32(v, sk), f32(got, sq), {}, c.scale);
        cpu.scaled_dot_product_attention(f32(q, sq), f32(kk, sk), f32(v, sk), f32(want, sq), {}, c.scale);
        const double e = rel_l2(got.data(), want.data(), got.size());
        report("attention n_q " + std::to_string(c.n_q) + " n_k " + std::to_string(c.n_k) + " d " +
                   std::to_string(c.d),
               rg.has_value() && e <= 1e-5, "rel-L2 " + fmt(e));
    }
}

void test_quantize(CudaBackend& gpu) {
    const int64_t rows = 6, k = 512;
    auto src = gaussian(size_t(rows * k), 0.5f, 71);
    for (int qt : {2, 8, 12, 13, 14}) {
        const size_t rb = oracle_row_bytes(qt, k);
        std::vector<uint8_t> want(rb * rows);
        for (int64_t r = 0; r < rows; ++r) oracle_quantize_row(qt, &src[size_t(r * k)], &want[rb * r], k);
        auto t = gpu.quantize(f32(src, Shape{rows, k}), dtype_of(qt));
        if (qt == 8) {   // Q8_0 rows need 17/16 bytes per element, more than a Tensor holds
            report("quantize Q8_0 rejected", !t && t.error() == make_error_code(Error::INVALID_FORMAT));
            continue;
        }
        const bool ok = t.has_value() && t->dtype() == dtype_of(qt) && t->shape() == (Shape{rows, k}) &&
                        std::memcmp(t->data(), want.data(), want.size()) == 0;
        report(std::string("quantize ") + qname(qt), ok);
    }
    auto bad = gpu.quantize(f32(src, Shape{rows * 2, k / 2}), Dtype::Q4_K);   // k = 256 is fine; k = 100 is not
    report("quantize k=256", bad.has_value());
    std::vector<float> odd(100, 1.0f);
    auto r = gpu.quantize(f32(odd, Shape{1, 100}), Dtype::Q4_K);
    report("quantize ragged k rejected", !r && r.error() == make_error_code(Error::SHAPE_MISMATCH));
    auto r2 = gpu.quantize(f32(src, Shape{rows, k}), Dtype::Q4_1);
    report("quantize Q4_1 not available", !r2 && r2.error() == make_error_code(Error::BACKEND_NOT_AVAILABLE));
}

void test_cache_and_errors(CudaBackend& gpu) {
    const int64_t n_out = 64, k = 256;
    QWeights w = make_weights(12, n_out, k, 81);
    TensorView wq(w.packed.data(), Dtype::Q4_K, Shape{n_out, k});
    auto x = gaussian(size_t(k), 1.0f, 82);
    std::vector<float> y1(static_cast<size_t>(n_out)), y2(static_cast<size_t>(n_out));
    const size_t before = gpu.cached_weights();
    auto r1 = gpu.matmul(wq, f32(x, Shape{k, 1}), f32(y1, Shape{n_out, 1}));
    auto r2 = gpu.matmul(wq, f32(x, Shape{k, 1}), f32(y2, Shape{n_out, 1}));
    report("weight cache: one upload for repeated calls",
           r1 && r2 && gpu.cached_weights() == before + 1 && bit_equal(y1.data(), y2.data(), y1.size()));

    auto e1 = gpu.matmul(wq, f32(x, Shape{k / 2, 1}), f32(y1, Shape{n_out, 1}));
    report("matmul shape mismatch", !e1 && e1.error() == make_error_code(Error::SHAPE_MISMATCH));
    std::vector<uint8_t> raw(1024);
    auto e2 = gpu.matmul(TensorView(raw.data(), Dtype::Q4_1, Shape{4, 256}), f32(x, Shape{k, 1}),
                         f32(y1, Shape{4, 1}));
    report("matmul Q4_1 not available", !e2 && e2.error() == make_error_code(Error::BACKEND_NOT_AVAILABLE));
    std::vector<float> a(8), b(9), o(8);
    auto e3 = gpu.add(f32(a, Shape{8}), f32(b, Shape{9}), f32(o, Shape{8}));
    report("add shape mismatch", !e3 && e3.error() == make_error_code(Error::SHAPE_MISMATCH));
    report("supports", gpu.supports(Dtype::Q4_K) && gpu.supports(Dtype::Q6_K) && gpu.supports(Dtype::F32) &&
                           !gpu.supports(Dtype::Q4_1));
    report("type and name", gpu.type() == BackendType::CUDA && std::strlen(gpu.name()) > 0);
    report("synchronize", gpu.synchronize().has_value());
}

}  // namespace

int main() {
    DeviceConfig cfg;
    CudaBackend gpu(cfg);
    CPU_Backend cpu(cfg);
    if (!gpu.stream()) {
        std::printf("FAIL no CUDA device\n");
        return 2;
    }
    test_matmul_quantized(gpu, cpu);
    test_matmul_f32(gpu, cpu);
    test_elementwise(gpu, cpu);
    test_rope(gpu, cpu);
    test_attention(gpu, cpu);
    test_quantize(gpu);
    test_cache_and_errors(gpu);
    std::printf("%d failed\n", g_failed);
    return g_failed ? 1 : 0;
}
