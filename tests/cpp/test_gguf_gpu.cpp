// test_gguf_gpu.cpp -- test program: a GGUF file straight to the GPU.
//   1. hesa_gguf::File parses it, hesa_gguf::DeviceModel uploads every tensor
//      once (backend/device_model.cpp);
//   2. every 2-D tensor of a quantized type the kernels run goes through
//      hesa::CudaBackend::matmul as a device-resident weight view, against
//      device-resident activations (batch 1, and batch 3 with padded rows):
//      no host staging; the outputs are written to <outdir>/y_<name>.f32 and
//      y3_<name>.f32 for tests/test_gguf.py to compare with the oracle;
//   3. hesa_gguf::DecodeSession runs tokens through the decoder from position
//      0 and writes each step's logits to <outdir>/logits_<pos>.f32.
// Inputs written by the test: <outdir>/x_<k>.f32 (k floats) and
// <outdir>/x3_<k>.f32 (3 rows of k + 4 floats).
#include "backend/cuda_backend.hpp"
#include "backend/device_model.hpp"
#include "backend/gguf_file.hpp"
#include "hesa_cuda.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

namespace {

bool read_f32(const std::string& path, std::vector<float>& v) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) return false;
    std::fseek(f, 0, SEEK_END);
    const long n = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    v.resize(static_cast<size_t>(n) / 4);
    const size_t got = std::fread(v.data(), 4, v.size(), f);
    std::fclose(f);
    return got == v.size();
}

bool write_f32(const std::string& path, const std::vector<float>& v) {
    FILE* f = std::fopen(path.c_str(), "wb");
    if (!f) return false;
    const size_t put = std::fwrite(v.data(), 4, v.size(), f);
    std::fclose(f);
    return put == v.size();
}

int g_fail = 0;
void check(bool ok, const std::string& what) {
    std::printf("%s %s\n", ok ? "PASS" : "FAIL", what.c_str());
    if (!ok) ++g_fail;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 5) {
        std::fprintf(stderr, "usage: test_gguf_gpu <file.gguf> <outdir> <ctx> <token@pos> ...\n");
        return 2;
    }
    const std::string dir = argv[2];
    hesa_gguf::File file;
    int rc = file.open(argv[1]);
    check(rc == hesa_gguf::kOk, "parse " + file.error());
    if (rc) return 1;

    hesa::DeviceConfig cfg;
    hesa::CudaBackend be(cfg);
    hesa_gguf::DeviceModel dm;
    rc = dm.upload(file, be.device_id(), be.stream());
    check(rc == hesa_gguf::kOk && dm.bytes() > 0, "upload " + dm.error());
    if (rc) return 1;

    cudaStream_t s = static_cast<cudaStream_t>(be.stream());
    for (const auto& t : dm.tensors()) {
        hesa::Dtype dt;
        if (t.rows < 2 || !hesa::CudaBackend::dtype_of_gguf(t.type, dt) || !be.supports(dt) || dt == hesa::Dtype::F32)
            continue;
        const int64_t M = t.rows, K = t.cols;
        std::vector<float> x, x3;
        if (!read_f32(dir + "/x_" + std::to_string(K) + ".f32", x) || static_cast<int64_t>(x.size()) != K ||
            !read_f32(dir + "/x3_" + std::to_string(K) + ".f32", x3) ||
            static_cast<int64_t>(x3.size()) != 3 * (K + 4)) {
            check(false, "inputs for " + t.name);
            continue;
        }
        float *dx = nullptr, *dy = nullptr, *dx3 = nullptr, *dy3 = nullptr;
        const int64_t ldy = M + 4;
        cudaMalloc(&dx, K * 4);
        cudaMalloc(&dy, M * 4);
        cudaMalloc(&dx3, x3.size() * 4);
        cudaMalloc(&dy3, 3 * ldy * 4);
        cudaMemcpy(dx, x.data(), K * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(dx3, x3.data(), x3.size() * 4, cudaMemcpyHostToDevice);
        const hesa::TensorView w = hesa::CudaBackend::device_view(t.ptr, dt, M, K);
        auto r1 = be.matmul(w, hesa::CudaBackend::device_columns(dx, K, 1, K),
                            hesa::CudaBackend::device_columns(dy, M, 1, M), 1.0f);
        auto r3 = be.matmul(w, hesa::CudaBackend::device_columns(dx3, K, 3, K + 4),
                            hesa::CudaBackend::device_columns(dy3, M, 3, ldy), 1.0f);
        cudaStreamSynchronize(s);
        std::vector<float> y(M), y3(3 * ldy);
        cudaMemcpy(y.data(), dy, M * 4, cudaMemcpyDeviceToHost);
        cudaMemcpy(y3.data(), dy3, y3.size() * 4, cudaMemcpyDeviceToHost);
        check(r1.has_value() && r3.has_value() && write_f32(dir + "/y_" + t.name + ".f32", y) &&
                  write_f32(dir + "/y3_" + t.name + ".f32", y3),
              "device-resident matmul " + t.name);
        for (float* p : {dx, dy, dx3, dy3}) cudaFree(p);
    }
    check(be.cached_weights() == 0, "no host-pointer weight cache used");

    hesa_gguf::DecodeSession ses;
    rc = ses.init(file, dm, std::atoi(argv[3]), be.stream());
    check(rc == hesa_gguf::kOk, "decode session " + ses.error());
    if (rc) return 1;
    for (int a = 4; a < argc; ++a) {
        int tok = 0, pos = 0;
        if (std::sscanf(argv[a], "%d@%d", &tok, &pos) != 2) return 2;
        const float* lg = nullptr;
        rc = ses.step(tok, pos, &lg);
        std::vector<float> logits(static_cast<size_t>(ses.vocab()));
        cudaStreamSynchronize(s);
        if (rc == 0) cudaMemcpy(logits.data(), lg, logits.size() * 4, cudaMemcpyDeviceToHost);
        check(rc == 0 && write_f32(dir + "/logits_" + std::to_string(pos) + ".f32", logits),
              "decode step at " + std::to_string(pos) + " " + ses.error());
    }
    int status = -1;
    hesa_cuda_device_status(be.stream(), &status);
    check(status == 0, "device status");
    return g_fail ? 1 : 0;
}
