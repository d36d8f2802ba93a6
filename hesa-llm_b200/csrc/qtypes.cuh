// qtypes.cuh -- GGUF block layouts and their exact scalar decoders on device.
//
// Byte sizes follow src/model/gguf_loader.cpp:26-35 of hesa-llm; the bit
// layout inside each block is the public GGUF format. Every expression that
// produces a weight value uses __fmul_rn/__fsub_rn so nvcc cannot contract it
// into an FMA: the result is bit-identical to the definition
// ((d*sc)*q - dmin*m with each operation rounded on its own).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace hesa_cuda {

enum QType : int { kQ4_0 = 2, kQ8_0 = 8, kQ4_K = 12, kQ5_K = 13, kQ6_K = 14 };

__host__ __device__ constexpr int block_elems(int qt) {
    return (qt == kQ4_0 || qt == kQ8_0) ? 32 : ((qt == kQ4_K || qt == kQ5_K || qt == kQ6_K) ? 256 : 0);
}

__host__ __device__ constexpr int block_bytes(int qt) {
    return qt == kQ4_0 ? 18 : qt == kQ8_0 ? 34 : qt == kQ4_K ? 144 : qt == kQ5_K ? 176 : qt == kQ6_K ? 210 : 0;
}

__host__ __device__ constexpr bool qtype_supported(int qt) { return block_elems(qt) != 0; }

__device__ __forceinline__ float h2f_bytes(const uint8_t* p) {
    const unsigned short h = static_cast<unsigned short>(p[0] | (p[1] << 8));
    return __half2float(__ushort_as_half(h));
}

// 6-bit (scale, min) pair j of the 12-byte K-quant scale field.
__device__ __forceinline__ void kq_scale_min(const uint8_t* s, int j, int& sc, int& m) {
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// K-quant scale/min pairs of sub-blocks 2c, 2c+1 (byte 0, byte 1 of each),
// from the first 16 bytes of a Q4_K/Q5_K block (h.x = d, dmin; h.y..h.w = the
// 12-byte scale field); the packing of kq_scale_min, two sub-blocks at once.
__device__ __forceinline__ void kq_pairs(const uint4& h, int c, uint32_t& sc2, uint32_t& m2) {
    const uint32_t s = 16u * (c & 1);
    if (c >> 1) {
        sc2 = ((h.w >> s) & 0x0F0Fu) | ((h.y >> (s + 2)) & 0x3030u);
        m2 = ((h.w >> (s + 4)) & 0x0F0Fu) | ((h.z >> (s + 2)) & 0x3030u);
    } else {
        sc2 = (h.y >> s) & 0x3F3Fu;
        m2 = (h.z >> s) & 0x3F3Fu;
    }
}

// Exact value of weight `i` (0 <= i < block_elems) of the block at `b`.
template <int QT>
__device__ __forceinline__ float deq_weight(const uint8_t* b, int i) {
    if constexpr (QT == kQ4_0) {
        const float d = h2f_bytes(b);
        const int j = i & 15;
        const int q = (i < 16) ? (b[2 + j] & 0x0F) : (b[2 + j] >> 4);
        return __fmul_rn(d, static_cast<float>(q - 8));
    } else if constexpr (QT == kQ8_0) {
        const float d = h2f_bytes(b);
        return __fmul_rn(d, static_cast<float>(static_cast<int8_t>(b[2 + i])));
    } else if constexpr (QT == kQ4_K || QT == kQ5_K) {
        const float d = h2f_bytes(b);
        const float dmin = h2f_bytes(b + 2);
        const int c = i >> 6;           // 64-weight chunk
        const int hi = (i >> 5) & 1;    // high nibble -> odd sub-block
        const int l = i & 31;
        const int j = 2 * c + hi;
        int sc, m;
        kq_scale_min(b + 4, j, sc, m);
        const uint8_t* qs = b + (QT == kQ4_K ? 16 : 48);
        int q = hi ? (qs[32 * c + l] >> 4) : (qs[32 * c + l] & 0x0F);
        if constexpr (QT == kQ5_K) q |= ((b[16 + l] >> j) & 1) << 4;
        return __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q)),
                         __fmul_rn(dmin, static_cast<float>(m)));
    } else {  // Q6_K
        const uint8_t* ql = b;
        const uint8_t* qh = b + 128;
        const int8_t* scales = reinterpret_cast<const int8_t*>(b + 192);
        const float d = h2f_bytes(b + 208);
        const int h = i >> 7;           // 128-weight half
        const int p = i & 127;
        const int g = p >> 5;           // 32-weight group inside the half
        const int l = p & 31;
        const uint8_t qlb = ql[64 * h + l + ((g & 1) ? 32 : 0)];
        const int nib = (g >= 2) ? (qlb >> 4) : (qlb & 0x0F);
        const int hb = (qh[32 * h + l] >> (2 * g)) & 3;
        const int q = (nib | (hb << 4)) - 32;
        const int is = 8 * h + (l >> 4) + 2 * g;
        return __fmul_rn(__fmul_rn(d, static_cast<float>(scales[is])), static_cast<float>(q));
    }
}

}  // namespace hesa_cuda
