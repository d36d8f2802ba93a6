// strip_core.cuh -- the decode core of the batch-1 row-strip kernel
// (qmatvec.cu, every input and output mode):
// the digit-plane form of x in shared memory, the per-type integer dot
// products of one quarter of a 256-weight unit, and the warp reductions.
//
//   * x is staged once per CTA as exact integers: per unit of 256
//     activations, X = rint(x / s) with s a power of two chosen so
//     |X| <= 2^22, split into three balanced int8 digits
//     X = 65536*D2 + 256*D1 + D0 (xdigits.cuh). The digit planes are
//     permuted per type so lane (unit j, quarter c) reads its 64 activations
//     with 12 conflict-free 128-bit loads and keeps them in registers.
//   * Quant values are unpacked to bytes and multiplied into the three digit
//     planes with DP4A (exact int32); sub-block scales are applied in int32,
//     the q offsets (-8, -32) and K-quant mins through per-group digit sums,
//     and the planes are combined in fp32 once per unit.
#pragma once

#include "hesa_common.cuh"
#include "qtypes.cuh"
#include "xdigits.cuh"
#include "peer_sync.cuh"

namespace hesa_cuda {
namespace strip {

constexpr int kWarps = 12;          // 384 threads: up to 168 registers each
constexpr int kThreads = kWarps * 32;

constexpr int kQPlaneStride = 208; // bytes per (unit, quarter): 3 digit planes x 64 B + 16 pad
constexpr int kQSumStride = 80;    // bytes per (unit, quarter): 4 groups x int4 digit sums + 16 pad

__host__ __device__ constexpr size_t x_region_bytes(int U) {
    return static_cast<size_t>(U) * 4 * (kQPlaneStride + kQSumStride) + ((static_cast<size_t>(U) * 4 + 15) & ~size_t(15));
}

__host__ __device__ constexpr int unit_bytes(int qt) {
    return qt == kQ4_K ? 144 : qt == kQ5_K ? 176 : qt == kQ6_K ? 210 : qt == kQ4_0 ? 144 : 272;
}


// Slot (quarter c, index i) of activation P (0..255 inside a unit), in the
// order the decoders consume it. Eight consecutive positions 8m..8m+7 always
// land in one quarter at eight consecutive indices.
template <int QT>
__device__ __forceinline__ void unit_pos_to_slot(int P, int& c, int& i) {
    if constexpr (QT == kQ6_K) {
        const int h = P >> 7, g = (P >> 5) & 3, s2 = (P >> 4) & 1, t = P & 15;
        c = 2 * h + s2;
        i = 16 * g + t;
    } else {
        c = P >> 6;
        i = P & 63;
    }
}

// Digit groups of a quarter: the weight blocks / sub-blocks whose integer
// corrections need sum_k X_k (32 activations; 16 for Q6_K).
template <int QT> __host__ __device__ constexpr int group_shift() { return QT == kQ6_K ? 4 : 5; }

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

// 16 bytes from a 2-byte aligned shared address: five aligned words, realigned
// with PRMT (selector 0x5432 takes bytes 2..5 of the pair).
__device__ __forceinline__ uint4 lds128_a2(const uint8_t* p) {
    const uint8_t* a = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(3));
    const uint32_t sel = (reinterpret_cast<uintptr_t>(p) & 2) ? 0x5432u : 0x3210u;
    const uint32_t w0 = lds32(a), w1 = lds32(a + 4), w2 = lds32(a + 8), w3 = lds32(a + 12),
                   w4 = lds32(a + 16);
    return make_uint4(prmt(w0, w1, sel), prmt(w1, w2, sel), prmt(w2, w3, sel), prmt(w3, w4, sel));
}

// The activations of one (unit, quarter) as the decoders see them: X = x/s as
// three balanced int8 digit planes, X = 65536*D2 + 256*D1 + D0, four digits
// per word (word w of a plane = quarter indices 4w..4w+3), the per-group digit
// sums, and the unit's scale s (a power of two).
struct XQuarter {
    uint32_t d[3][16];
    int ds[4][3];
    float s;
    float s16;     // s / 16, for products taken on 16 x (high nibble in place)
    float xs[2];   // sum_k x_k over groups 0 and 1 (K-quant min terms)
};

// Integer dot of 4 weight bytes (values that fit int8) with the 3 digit
// planes at word w: p[j] += sum_i q_i * D_j,i.
__device__ __forceinline__ void dot3(uint32_t q, const XQuarter& xq, int w, int (&p)[3]) {
    p[0] = __dp4a(static_cast<int>(q), static_cast<int>(xq.d[0][w]), p[0]);
    p[1] = __dp4a(static_cast<int>(q), static_cast<int>(xq.d[1][w]), p[1]);
    p[2] = __dp4a(static_cast<int>(q), static_cast<int>(xq.d[2][w]), p[2]);
}

// dp4a with unsigned bytes in a and signed bytes in b.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// As dot3 for unsigned weight bytes (0..255).
__device__ __forceinline__ void dot3u(uint32_t q, const XQuarter& xq, int w, int (&p)[3]) {
    p[0] = dp4a_us(q, xq.d[0][w], p[0]);
    p[1] = dp4a_us(q, xq.d[1][w], p[1]);
    p[2] = dp4a_us(q, xq.d[2][w], p[2]);
}

// sum_k x_k over group g of the quarter (fp32), from the digit sums.
__device__ __forceinline__ float xsum(const XQuarter& xq, int g) {
    return xq.s * combine3(xq.ds[g][0], xq.ds[g][1], xq.ds[g][2]);
}

// Contribution of quarter c of one unit of one row: sum over the quarter's
// 64 weights of deq(w) * x (without the row's output scale). `u` points at
// the unit in shared memory.
template <int QT>
__device__ __forceinline__ float unit_dot(const uint8_t* u, int c, const XQuarter& xq);

template <>
__device__ __forceinline__ float unit_dot<kQ4_K>(const uint8_t* u, int c, const XQuarter& xq) {
    const uint4 h = lds128(u);
    const uint4 qa = lds128(u + 16 + 32 * c);
    const uint4 qb = lds128(u + 32 + 32 * c);
    uint32_t sc2, m2;
    kq_pairs(h, c, sc2, m2);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    int lo[3] = {0, 0, 0}, hi[3] = {0, 0, 0};
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        dot3(q[t] & 0x0F0F0F0Fu, xq, t, lo);        // sub-block 2c: indices 4t..4t+3
        dot3u(q[t] & 0xF0F0F0F0u, xq, 8 + t, hi);   // sub-block 2c+1 (32+4t..), as 16 q
    }
    // 16 * (s0 * lo + s1 * q_hi . X): exact in int32 (|.| < 2^27)
    const int s0x16 = static_cast<int>(sc2 & 0xFF) << 4, s1 = static_cast<int>(sc2 >> 8);
    const float t = combine3(s0x16 * lo[0] + s1 * hi[0], s0x16 * lo[1] + s1 * hi[1], s0x16 * lo[2] + s1 * hi[2]);
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    const float mins = fmaf(static_cast<float>(m2 & 0xFF), xq.xs[0], static_cast<float>(m2 >> 8) * xq.xs[1]);
    return fmaf(d * xq.s16, t, -dmin * mins);
}

template <>
__device__ __forceinline__ float unit_dot<kQ5_K>(const uint8_t* u, int c, const XQuarter& xq) {
    const uint4 h = lds128(u);
    const uint4 ha = lds128(u + 16), hb = lds128(u + 32);   // qh, shared by the 4 quarters
    const uint4 qa = lds128(u + 48 + 32 * c);
    const uint4 qb = lds128(u + 64 + 32 * c);
    uint32_t sc2, m2;
    kq_pairs(h, c, sc2, m2);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const uint32_t qh[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
    const uint32_t sh = 2u * c;
    int lo[3] = {0, 0, 0}, hi[3] = {0, 0, 0};
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        const uint32_t hv = qh[t] >> sh;   // bit 0 of each byte: sub-block 2c, bit 1: 2c+1
        dot3((q[t] & 0x0F0F0F0Fu) | ((hv << 4) & 0x10101010u), xq, t, lo);
        dot3(((q[t] >> 4) & 0x0F0F0F0Fu) | ((hv << 3) & 0x10101010u), xq, 8 + t, hi);
    }
    const int s0 = static_cast<int>(sc2 & 0xFF), s1 = static_cast<int>(sc2 >> 8);
    const float t = combine3(s0 * lo[0] + s1 * hi[0], s0 * lo[1] + s1 * hi[1], s0 * lo[2] + s1 * hi[2]);
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    const float mins = fmaf(static_cast<float>(m2 & 0xFF), xq.xs[0], static_cast<float>(m2 >> 8) * xq.xs[1]);
    return fmaf(d * xq.s, t, -dmin * mins);
}

template <>
__device__ __forceinline__ float unit_dot<kQ6_K>(const uint8_t* u, int c, const XQuarter& xq) {
    // quarter c: half h = c>>1, positions l in [16*s2, 16*s2+16) of each of the
    // four 32-weight groups of that half; group g is sub-block 8h + s2 + 2g
    const int h = c >> 1, s2 = c & 1;
    const uint4 qa = lds128_a2(u + 64 * h + 16 * s2);
    const uint4 qb = lds128_a2(u + 64 * h + 32 + 16 * s2);
    const uint4 qv = lds128_a2(u + 128 + 32 * h + 16 * s2);
    const uint8_t* scp = u + 192 + 8 * h + s2;
    const int sc[4] = {static_cast<int8_t>(scp[0]), static_cast<int8_t>(scp[2]), static_cast<int8_t>(scp[4]),
                       static_cast<int8_t>(scp[6])};
    const uint32_t a[4] = {qa.x, qa.y, qa.z, qa.w};
    const uint32_t b[4] = {qb.x, qb.y, qb.z, qb.w};
    const uint32_t v[4] = {qv.x, qv.y, qv.z, qv.w};
    int g0[3] = {0, 0, 0}, g1[3] = {0, 0, 0}, g2[3] = {0, 0, 0}, g3[3] = {0, 0, 0};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        // q = nibble | (two high bits << 4), 0..63
        dot3((a[t] & 0x0F0F0F0Fu) | ((v[t] << 4) & 0x30303030u), xq, t, g0);
        dot3((b[t] & 0x0F0F0F0Fu) | ((v[t] << 2) & 0x30303030u), xq, 4 + t, g1);
        dot3(((a[t] >> 4) & 0x0F0F0F0Fu) | (v[t] & 0x30303030u), xq, 8 + t, g2);
        dot3(((b[t] >> 4) & 0x0F0F0F0Fu) | ((v[t] >> 2) & 0x30303030u), xq, 12 + t, g3);
    }
    // sum (q - 32) X per group, scaled by the signed sub-block scale
    int acc[3];
#pragma unroll
    for (int p = 0; p < 3; ++p)
        acc[p] = sc[0] * (g0[p] - 32 * xq.ds[0][p]) + sc[1] * (g1[p] - 32 * xq.ds[1][p]) +
                 sc[2] * (g2[p] - 32 * xq.ds[2][p]) + sc[3] * (g3[p] - 32 * xq.ds[3][p]);
    const float d = h2f_bytes(u + 208);
    return (d * xq.s) * combine3(acc[0], acc[1], acc[2]);
}

template <>
__device__ __forceinline__ float unit_dot<kQ4_0>(const uint8_t* u, int c, const XQuarter& xq) {
    // quarter c = blocks 2c and 2c+1: 36 bytes at 36c (4-byte aligned)
    const uint8_t* p = u + 36 * c;
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) w[i] = lds32(p + 4 * i);
    const float d0 = half_bits_to_float(w[0]);
    const float d1 = half_bits_to_float(w[4] >> 16);
    const uint32_t q0[4] = {prmt(w[0], w[1], 0x5432u), prmt(w[1], w[2], 0x5432u),
                            prmt(w[2], w[3], 0x5432u), prmt(w[3], w[4], 0x5432u)};
    const uint32_t q1[4] = {w[5], w[6], w[7], w[8]};
    int b0[3] = {0, 0, 0}, b1[3] = {0, 0, 0};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        // byte j low nibble -> weight j, high nibble -> weight j + 16
        dot3(q0[t] & 0x0F0F0F0Fu, xq, t, b0);
        dot3((q0[t] >> 4) & 0x0F0F0F0Fu, xq, 4 + t, b0);
        dot3(q1[t] & 0x0F0F0F0Fu, xq, 8 + t, b1);
        dot3((q1[t] >> 4) & 0x0F0F0F0Fu, xq, 12 + t, b1);
    }
    // sum (q - 8) X
    const float t0 = combine3(b0[0] - 8 * xq.ds[0][0], b0[1] - 8 * xq.ds[0][1], b0[2] - 8 * xq.ds[0][2]);
    const float t1 = combine3(b1[0] - 8 * xq.ds[1][0], b1[1] - 8 * xq.ds[1][1], b1[2] - 8 * xq.ds[1][2]);
    return xq.s * fmaf(d0, t0, d1 * t1);
}

template <>
__device__ __forceinline__ float unit_dot<kQ8_0>(const uint8_t* u, int c, const XQuarter& xq) {
    // quarter c = blocks 2c and 2c+1: 68 bytes at 68c (4-byte aligned)
    const uint8_t* p = u + 68 * c;
    uint32_t w[17];
#pragma unroll
    for (int i = 0; i < 17; ++i) w[i] = lds32(p + 4 * i);
    const float d0 = half_bits_to_float(w[0]);
    const float d1 = half_bits_to_float(w[8] >> 16);
    int b0[3] = {0, 0, 0}, b1[3] = {0, 0, 0};
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        dot3(prmt(w[t], w[t + 1], 0x5432u), xq, t, b0);
        dot3(w[9 + t], xq, 8 + t, b1);
    }
    return xq.s * fmaf(d0, combine3(b0[0], b0[1], b0[2]), d1 * combine3(b1[0], b1[1], b1[2]));
}


// Convert one unit (256 activations) to digit planes in shared memory; lane
// L holds positions 8L..8L+7 in v (digits as unit_digits makes them).
template <int QT>
__device__ __forceinline__ void stage_unit(int unit, int lane, const float (&v)[8], uint8_t* xplanes, uint8_t* xsums,
                                           float* xscale) {
    uint32_t dw[3][2];
    const float s = unit_digits(v, dw);
    int c, i0;
    unit_pos_to_slot<QT>(lane * 8, c, i0);
    uint8_t* qbase = xplanes + static_cast<size_t>(unit * 4 + c) * kQPlaneStride;
#pragma unroll
    for (int p = 0; p < 3; ++p) *reinterpret_cast<uint2*>(qbase + p * 64 + i0) = make_uint2(dw[p][0], dw[p][1]);
    // digit sums of the group (2 or 4 lanes): planes 0 and 1 travel packed in
    // one word (each sum of at most 32 digits fits 16 bits signed)
    int sums[3];
#pragma unroll
    for (int p = 0; p < 3; ++p)
        sums[p] = __dp4a(static_cast<int>(dw[p][0]), 0x01010101, __dp4a(static_cast<int>(dw[p][1]), 0x01010101, 0));
    int s01 = sums[0] + (sums[1] << 16), s2 = sums[2];
    s01 += __shfl_xor_sync(0xffffffffu, s01, 1);
    s2 += __shfl_xor_sync(0xffffffffu, s2, 1);
    if constexpr (QT != kQ6_K) {
        s01 += __shfl_xor_sync(0xffffffffu, s01, 2);
        s2 += __shfl_xor_sync(0xffffffffu, s2, 2);
    }
    const bool writer = (QT == kQ6_K) ? ((lane & 1) == 0) : ((lane & 3) == 0);
    if (writer) {
        const int s0 = static_cast<int>(static_cast<int16_t>(s01 & 0xFFFF));
        int* ds = reinterpret_cast<int*>(xsums + static_cast<size_t>(unit * 4 + c) * kQSumStride) +
                  4 * (i0 >> group_shift<QT>());
        *reinterpret_cast<int4*>(ds) = make_int4(s0, (s01 - s0) >> 16, s2, 0);
    }
    if (lane == 0) xscale[unit] = s;
}

// The activations of quarter qc of `unit`, from the staged planes into registers.
template <int QT>
__device__ __forceinline__ void load_xquarter(const uint8_t* xplanes, const uint8_t* xsums, const float* xscale,
                                              int unit, int qc, XQuarter& xq) {
    const uint8_t* qsrc = xplanes + static_cast<size_t>(unit * 4 + qc) * kQPlaneStride;
#pragma unroll
    for (int p = 0; p < 3; ++p) {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const uint4 w4 = lds128(qsrc + p * 64 + 16 * t);
            xq.d[p][4 * t] = w4.x; xq.d[p][4 * t + 1] = w4.y;
            xq.d[p][4 * t + 2] = w4.z; xq.d[p][4 * t + 3] = w4.w;
        }
    }
    const uint8_t* ssrc = xsums + static_cast<size_t>(unit * 4 + qc) * kQSumStride;
#pragma unroll
    for (int gg = 0; gg < (QT == kQ6_K ? 4 : 2); ++gg) {
        const int4 s4 = *reinterpret_cast<const int4*>(ssrc + 16 * gg);
        xq.ds[gg][0] = s4.x; xq.ds[gg][1] = s4.y; xq.ds[gg][2] = s4.z;
    }
    xq.s = xscale[unit];
    xq.s16 = xq.s * 0.0625f;
    if constexpr (QT == kQ4_K || QT == kQ5_K) {
        xq.xs[0] = xsum(xq, 0);
        xq.xs[1] = xsum(xq, 1);
    }
}


// Rows decoded together per group: four independent chains, three for the
// types whose quarter needs the most registers (Q5_K, Q6_K: four rows at once
// would exceed the 168 registers a thread has at 384 threads; measured 2,818
// vs 2,694 GB/s on Q6_K).
__host__ __device__ constexpr int strip_group_rows(int qt) { return (qt == kQ6_K || qt == kQ5_K) ? 3 : 4; }
constexpr int kStripBatch = 4;   // units of x one warp loads at a time

// Input transforms of the strip kernel's staging (decode-step fusions).
enum : int { kXPlain = 0, kXRmsNorm = 1, kXSiluMul = 2 };

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Positions 8*lane .. 8*lane+7 of unit u of a vector (zeros when u >= U).
__device__ __forceinline__ void load8(const float* __restrict__ src, int u, int lane, int U, float (&v)[8]) {
    if (u < U) {
        const float4* p = reinterpret_cast<const float4*>(src + static_cast<size_t>(u) * 256 + lane * 8);
        const float4 a = p[0], b = p[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 0.f;
    }
}

// silu(g) * u for the SwiGLU input. The value is rounded to 22 bits below its
// unit's maximum right after, so the fast exp and divide (a few ulp) change
// nothing that survives that rounding.
__device__ __forceinline__ float swiglu_x(float g, float u) { return __fdividef(g, 1.0f + __expf(-g)) * u; }

// load8 from a tagged vector (peer_sync.cuh), each value once its tag is
// `tag`, for the kStripBatch units u0 + jb * kWarps: the loads of two units
// are issued before the first of their tags is looked at (more would spill).
__device__ __forceinline__ void load8_ll_batch(const uint64_t* src, uint32_t tag, unsigned long long limit_ns, int u0,
                                               int lane, int U, float (&v)[kStripBatch][8], int* status,
                                               volatile int* failed) {
#pragma unroll
    for (int jh = 0; jh < kStripBatch; jh += 2) {
        uint64_t w[2][8];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int u = u0 + (jh + i) * kWarps;
            if (u < U) ld_ll8_issue(src + static_cast<size_t>(u) * 256, lane, w[i]);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int u = u0 + (jh + i) * kWarps;
            if (u < U) {
                ld_ll8_take(src + static_cast<size_t>(u) * 256, lane, w[i], tag, limit_ns, v[jh + i], status,
                            failed);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[jh + i][j] = 0.f;
            }
        }
    }
}

// SwiGLU input from a tagged vector (gate at src, up at src + k elements):
// v[jb] <- swiglu_x(gate, up) for the units u0 + jb * kWarps, the loads of
// both halves of two units issued before the first tag is looked at.
__device__ __forceinline__ void load8_ll_swiglu(const uint64_t* src, int64_t k, uint32_t tag,
                                                unsigned long long limit_ns, int u0, int lane, int U,
                                                float (&v)[kStripBatch][8], int* status, volatile int* failed) {
#pragma unroll
    for (int jh = 0; jh < kStripBatch; jh += 2) {
        uint64_t wg[2][8], wu[2][8];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int u = u0 + (jh + i) * kWarps;
            if (u < U) {
                ld_ll8_issue(src + static_cast<size_t>(u) * 256, lane, wg[i]);
                ld_ll8_issue(src + k + static_cast<size_t>(u) * 256, lane, wu[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int u = u0 + (jh + i) * kWarps;
            if (u < U) {
                float g[8], up[8];
                ld_ll8_take(src + static_cast<size_t>(u) * 256, lane, wg[i], tag, limit_ns, g, status, failed);
                ld_ll8_take(src + k + static_cast<size_t>(u) * 256, lane, wu[i], tag, limit_ns, up, status, failed);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[jh + i][j] = swiglu_x(g[j], up[j]);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[jh + i][j] = 0.f;
            }
        }
    }
}

// Sum of v[0..3] over the 32 lanes of a warp in 6 shuffles: afterwards the
// lanes with (lane & 7) == 0 hold the total of v[reduce4_row(lane)].
__device__ __forceinline__ int reduce4_row(int lane) { return ((lane >> 3) & 2) | ((lane >> 3) & 1); }

__device__ __forceinline__ float reduce4(const float (&v)[4], int lane) {
    const bool hi16 = lane & 16;
    float a0 = hi16 ? v[2] : v[0], a1 = hi16 ? v[3] : v[1];
    const float b0 = hi16 ? v[0] : v[2], b1 = hi16 ? v[1] : v[3];
    a0 += __shfl_xor_sync(0xffffffffu, b0, 16);
    a1 += __shfl_xor_sync(0xffffffffu, b1, 16);
    const bool hi8 = lane & 8;
    float c = hi8 ? a1 : a0;
    const float d = hi8 ? a0 : a1;
    c += __shfl_xor_sync(0xffffffffu, d, 8);
    c += __shfl_xor_sync(0xffffffffu, c, 4);
    c += __shfl_xor_sync(0xffffffffu, c, 2);
    c += __shfl_xor_sync(0xffffffffu, c, 1);
    return c;
}

// Quarter qc of rows rb, rb + rstep, ... (NR of them) against the lane's x.
template <int QT, int NR>
__device__ __forceinline__ void strip_rows(const uint8_t* rb, size_t rstep, int qc, const XQuarter& xq,
                                           float (&a)[4]) {
#pragma unroll
    for (int t = 0; t < NR; ++t) a[t] = unit_dot<QT>(rb + t * rstep, qc, xq);
}


}  // namespace strip
}  // namespace hesa_cuda
