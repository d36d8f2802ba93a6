// quantize.cu -- deterministic round-to-nearest GGUF block quantizer on the GPU
// (the device half of the block codec): fp32 rows -> packed Q4_0 / Q8_0 /
// Q4_K / Q5_K / Q6_K rows in the layout the matvec kernels read.
//
// Q4_0 and Q8_0 follow the published ggml reference rounding (d from the
// signed value of largest magnitude / -8, q = min(15, trunc(x/d + 8.5)); d =
// amax/127, q = round(x/d)). The K-quants are a plain min/max RTN: per 32-weight
// sub-block scale = (max - min)/(levels - 1) with min clipped to <= 0, both
// 6-bit against the super-block maxima (Q4_K, Q5_K); Q6_K: sub-block scale =
// (signed value of largest magnitude)/-32 as int8 against d = (signed largest
// scale)/-128. Every operation is rounded separately (no contraction,
// correctly rounded division), so the bytes are identical to a sequential
// C implementation of the same steps compiled without FMA contraction.
//
// One thread per block: quantizing is set-up work (weight upload), not a hot
// path; the per-block loops stay in the order that makes the bytes exact.
#include "qtypes.cuh"
#include "quantize.h"

#include <cuda_fp16.h>

namespace hesa_cuda {
namespace {

// IEEE fp32 -> fp16 bit pattern, round to nearest even, in integer
// arithmetic: overflow to inf, subnormal halves, NaN kept quiet.
__device__ __forceinline__ uint16_t f2h_bits(float f) {
    const uint32_t x = __float_as_uint(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFFu) return static_cast<uint16_t>(sign | 0x7C00u | (man ? 0x200u : 0u));
    const int e = static_cast<int>(exp) - 127 + 15;
    if (e >= 31) return static_cast<uint16_t>(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return static_cast<uint16_t>(sign);
        man |= 0x800000u;
        const uint32_t shift = static_cast<uint32_t>(14 - e);
        uint32_t h = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return static_cast<uint16_t>(sign | h);
    }
    uint32_t h = sign | (static_cast<uint32_t>(e) << 10) | (man >> 13);
    const uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;   // a carry may reach the exponent: still RNE
    return static_cast<uint16_t>(h);
}
__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
__device__ __forceinline__ void wr16(uint8_t* p, uint16_t v) {
    p[0] = static_cast<uint8_t>(v & 0xFF);
    p[1] = static_cast<uint8_t>(v >> 8);
}

__device__ void quant_q4_0(const float* x, uint8_t* b) {
    float amax = 0.f, vmax = 0.f;
    for (int j = 0; j < 32; ++j) {
        const float a = fabsf(x[j]);
        if (a > amax) { amax = a; vmax = x[j]; }
    }
    const float d = __fdiv_rn(vmax, -8.f);
    const float id = d != 0.f ? __fdiv_rn(1.f, d) : 0.f;
    const uint16_t dh = f2h_bits(d);
    for (int j = 0; j < 16; ++j) {
        const float v0 = __fadd_rn(__fmul_rn(x[j], id), 8.5f);
        const float v1 = __fadd_rn(__fmul_rn(x[j + 16], id), 8.5f);
        const int q0 = clampi(__float2int_rz(v0), 0, 15);
        const int q1 = clampi(__float2int_rz(v1), 0, 15);
        b[2 + j] = static_cast<uint8_t>(q0 | (q1 << 4));
    }
    wr16(b, dh);
}

__device__ void quant_q8_0(const float* x, uint8_t* b) {
    float amax = 0.f;
    for (int j = 0; j < 32; ++j) amax = fabsf(x[j]) > amax ? fabsf(x[j]) : amax;
    const float d = __fdiv_rn(amax, 127.f);
    const float id = d != 0.f ? __fdiv_rn(1.f, d) : 0.f;
    const uint16_t dh = f2h_bits(d);
    for (int j = 0; j < 32; ++j) {
        const int q = clampi(__float2int_rz(roundf(__fmul_rn(x[j], id))), -128, 127);
        b[2 + j] = static_cast<uint8_t>(static_cast<int8_t>(q));
    }
    wr16(b, dh);
}

// Shared part of Q4_K / Q5_K: header (d, dmin, packed 6-bit scale/min pairs)
// and the sub-block levels q (0 .. nq-1) of the 256 weights, returned in q.
__device__ void quant_kq_asym(const float* x, uint8_t* b, int nq, uint8_t* q) {
    float scales[8], mins[8];
    float max_scale = 0.f, max_min = 0.f;
    for (int j = 0; j < 8; ++j) {
        float mn = x[32 * j], mx = x[32 * j];
        for (int l = 1; l < 32; ++l) {
            const float v = x[32 * j + l];
            if (v < mn) mn = v;
            if (v > mx) mx = v;
        }
        if (mn > 0.f) mn = 0.f;
        scales[j] = __fdiv_rn(__fsub_rn(mx, mn), static_cast<float>(nq - 1));
        mins[j] = -mn;
        if (scales[j] > max_scale) max_scale = scales[j];
        if (mins[j] > max_min) max_min = mins[j];
    }
    const uint16_t dh = f2h_bits(__fdiv_rn(max_scale, 63.f)), dminh = f2h_bits(__fdiv_rn(max_min, 63.f));
    const float dq = h2f_bits(dh), dminq = h2f_bits(dminh);
    int isc[8], imn[8];
    for (int j = 0; j < 8; ++j) {
        isc[j] = dq > 0.f ? clampi(__float2int_rz(roundf(__fdiv_rn(scales[j], dq))), 0, 63) : 0;
        imn[j] = dminq > 0.f ? clampi(__float2int_rz(roundf(__fdiv_rn(mins[j], dminq))), 0, 63) : 0;
    }
    wr16(b, dh);
    wr16(b + 2, dminh);
    for (int j = 0; j < 4; ++j) {
        b[4 + j] = static_cast<uint8_t>((isc[j] & 63) | ((isc[j + 4] >> 4) << 6));
        b[8 + j] = static_cast<uint8_t>((imn[j] & 63) | ((imn[j + 4] >> 4) << 6));
        b[12 + j] = static_cast<uint8_t>((isc[j + 4] & 15) | ((imn[j + 4] & 15) << 4));
    }
    for (int j = 0; j < 8; ++j) {
        const float ds = __fmul_rn(dq, static_cast<float>(isc[j]));
        const float dm = __fmul_rn(dminq, static_cast<float>(imn[j]));
        for (int l = 0; l < 32; ++l) {
            int v = 0;
            if (ds > 0.f) v = clampi(__float2int_rz(roundf(__fdiv_rn(__fadd_rn(x[32 * j + l], dm), ds))), 0, nq - 1);
            q[32 * j + l] = static_cast<uint8_t>(v);
        }
    }
}

__device__ void quant_q4_k(const float* x, uint8_t* b) {
    uint8_t q[256];
    quant_kq_asym(x, b, 16, q);
    uint8_t* qs = b + 16;
    for (int c = 0; c < 4; ++c)
        for (int l = 0; l < 32; ++l) qs[32 * c + l] = static_cast<uint8_t>(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
}

__device__ void quant_q5_k(const float* x, uint8_t* b) {
    uint8_t q[256];
    quant_kq_asym(x, b, 32, q);
    uint8_t* qh = b + 16;
    uint8_t* qs = b + 48;
    for (int l = 0; l < 32; ++l) qh[l] = 0;
    for (int c = 0; c < 4; ++c) {
        for (int l = 0; l < 32; ++l) {
            const int q0 = q[64 * c + l], q1 = q[64 * c + 32 + l];
            qs[32 * c + l] = static_cast<uint8_t>((q0 & 15) | ((q1 & 15) << 4));
            qh[l] |= static_cast<uint8_t>(((q0 >> 4) & 1) << (2 * c));
            qh[l] |= static_cast<uint8_t>(((q1 >> 4) & 1) << (2 * c + 1));
        }
    }
}

__device__ void quant_q6_k(const float* x, uint8_t* b) {
    float scales[16];
    float amax_s = 0.f, vmax_s = 0.f;
    for (int i = 0; i < 16; ++i) {
        float am = 0.f, vm = 0.f;
        for (int l = 0; l < 16; ++l) {
            const float v = x[16 * i + l];
            if (fabsf(v) > am) { am = fabsf(v); vm = v; }
        }
        scales[i] = __fdiv_rn(vm, -32.f);
        if (fabsf(scales[i]) > amax_s) { amax_s = fabsf(scales[i]); vmax_s = scales[i]; }
    }
    const uint16_t dh = f2h_bits(__fdiv_rn(vmax_s, -128.f));
    const float dq = h2f_bits(dh);
    int8_t isc[16];
    for (int i = 0; i < 16; ++i) {
        const int s = dq != 0.f ? __float2int_rz(roundf(__fdiv_rn(scales[i], dq))) : 0;
        isc[i] = static_cast<int8_t>(clampi(s, -128, 127));
    }
    uint8_t q[256];
    for (int i = 0; i < 16; ++i) {
        const float ds = __fmul_rn(dq, static_cast<float>(isc[i]));
        for (int l = 0; l < 16; ++l) {
            int v = 32;
            if (ds != 0.f) v = clampi(__float2int_rz(roundf(__fdiv_rn(x[16 * i + l], ds))) + 32, 0, 63);
            q[16 * i + l] = static_cast<uint8_t>(v);
        }
    }
    uint8_t* ql = b;
    uint8_t* qh = b + 128;
    for (int h = 0; h < 2; ++h) {
        for (int l = 0; l < 32; ++l) {
            const int q1 = q[128 * h + l], q2 = q[128 * h + l + 32];
            const int q3 = q[128 * h + l + 64], q4 = q[128 * h + l + 96];
            ql[64 * h + l] = static_cast<uint8_t>((q1 & 15) | ((q3 & 15) << 4));
            ql[64 * h + l + 32] = static_cast<uint8_t>((q2 & 15) | ((q4 & 15) << 4));
            qh[32 * h + l] = static_cast<uint8_t>((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
        }
    }
    for (int i = 0; i < 16; ++i) b[192 + i] = static_cast<uint8_t>(isc[i]);
    wr16(b + 208, dh);
}

template <int QT>
__global__ void __launch_bounds__(128) quantize_kernel(const float* __restrict__ src, int64_t n_rows, int64_t k,
                                                       int64_t ld, uint8_t* __restrict__ dst) {
    constexpr int BE = block_elems(QT), BB = block_bytes(QT);
    const int64_t nb = k / BE;
    const int64_t total = n_rows * nb;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / nb, blk = i - r * nb;
        const float* x = src + r * ld + blk * BE;
        uint8_t* b = dst + i * BB;
        if constexpr (QT == kQ4_0) quant_q4_0(x, b);
        else if constexpr (QT == kQ8_0) quant_q8_0(x, b);
        else if constexpr (QT == kQ4_K) quant_q4_k(x, b);
        else if constexpr (QT == kQ5_K) quant_q5_k(x, b);
        else quant_q6_k(x, b);
    }
}

template <int QT>
cudaError_t launch(const float* src, int64_t n_rows, int64_t k, int64_t ld, uint8_t* dst, cudaStream_t s) {
    const int64_t total = n_rows * (k / block_elems(QT));
    int64_t blocks = (total + 127) / 128;
    if (blocks > 148 * 64) blocks = 148 * 64;
    if (blocks < 1) blocks = 1;
    quantize_kernel<QT><<<static_cast<int>(blocks), 128, 0, s>>>(src, n_rows, k, ld, dst);
    return cudaGetLastError();
}

}  // namespace

cudaError_t quantize(int qtype, const float* src, int64_t n_rows, int64_t k, int64_t ld, void* dst,
                     cudaStream_t stream) {
    uint8_t* d = static_cast<uint8_t*>(dst);
    switch (qtype) {
        case kQ4_0: return launch<kQ4_0>(src, n_rows, k, ld, d, stream);
        case kQ8_0: return launch<kQ8_0>(src, n_rows, k, ld, d, stream);
        case kQ4_K: return launch<kQ4_K>(src, n_rows, k, ld, d, stream);
        case kQ5_K: return launch<kQ5_K>(src, n_rows, k, ld, d, stream);
        case kQ6_K: return launch<kQ6_K>(src, n_rows, k, ld, d, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace hesa_cuda
