// xdigits.cuh -- exact integer form of one unit of 256 activations, shared by
// the batch-1 kernels (qmatvec.cu) and the batched tensor-core kernel (qmm_tc.cu).
//
// Per unit, X = rint(x / s) with s = 2^(E-21), E the exponent of the unit's
// largest |x|, so |X| < 2^22; X is split into three balanced int8 digits,
// X = 65536*D2 + 256*D1 + D0. Products of the digits with integer weights are
// exact in int32; the planes are recombined in fp32 once per unit.
#pragma once
#include "hesa_common.cuh"

namespace hesa_cuda {

// Lane L of a warp holds positions 8L..8L+7 of the unit in v. Returns the
// unit's scale s (NaN if any activation of the unit is inf or NaN, so that
// every output it touches is NaN, as the fp32 sum would be) and the digit
// words of the lane's eight positions: dw[p][h] holds the plane-p digits of
// positions 8L+4h .. 8L+4h+3, one signed byte each, position order.
//
// The balanced digits of X (|X| < 2^22) are the bytes of X + 0x808080, each
// minus 128: adding 1.5 * 2^23 to x / s in one fused multiply-add rounds it to
// the integer X (nearest, ties to even, as rint) in the low mantissa bits, so
// X + 0x808080 is that float's bit pattern minus (0x4B400000 - 0x808080).
// PRMT gathers byte p of four such words into digit-plane word p, and XOR
// 0x80 per byte turns the biased bytes into signed digits.
__device__ __forceinline__ float unit_digits(const float (&v)[8], uint32_t (&dw)[3][2]) {
    // largest magnitude: max.NaN keeps a NaN, inf compares above every finite
    // value, and the bit patterns of non-negative floats order as integers
    float fm = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) fm = fmax_nan(fm, fabsf(v[j]));
    const uint32_t am = __reduce_max_sync(0xffffffffu, __float_as_uint(fm));
    const bool finite = am < 0x7F800000u;
    // exponent E of the largest magnitude: |x| < 2^(E+1); s = 2^(E-21)
    int E = static_cast<int>(am >> 23) - 127;
    if (E < -100) E = -100;  // activations below 2^-100 round to zero
    const float inv_s = __uint_as_float(static_cast<uint32_t>(21 - E + 127) << 23);
    uint32_t Y[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) Y[j] = __float_as_uint(fmaf(v[j], inv_s, 12582912.0f)) - 0x4ABF7F80u;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t* yy = Y + 4 * h;
        const uint32_t t01 = prmt(yy[0], yy[1], 0x5140u), t23 = prmt(yy[2], yy[3], 0x5140u);
        const uint32_t u01 = prmt(yy[0], yy[1], 0x0062u), u23 = prmt(yy[2], yy[3], 0x0062u);
        dw[0][h] = prmt(t01, t23, 0x5410u) ^ 0x80808080u;
        dw[1][h] = prmt(t01, t23, 0x7632u) ^ 0x80808080u;
        dw[2][h] = prmt(u01, u23, 0x5410u) ^ 0x80808080u;
    }
    // (digits of a non-finite unit are meaningless; its scale is NaN)
    return finite ? __uint_as_float(static_cast<uint32_t>(E - 21 + 127) << 23) : __int_as_float(0x7FC00000);
}

// 65536*a2 + 256*a1 + a0 in fp32.
__device__ __forceinline__ float combine3(int a0, int a1, int a2) {
    return fmaf(static_cast<float>(a2), 65536.f, fmaf(static_cast<float>(a1), 256.f, static_cast<float>(a0)));
}

}  // namespace hesa_cuda
