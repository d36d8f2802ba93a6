/*
 * hesa_oracle.c -- CPU restatement of the GGUF quantized matvec path.
 *
 * TEST INFRASTRUCTURE ONLY (the oracle the parity tests compare against). See hesa_oracle.h for what each
 * function restates and where its semantics come from. Compiled with
 * -O2 -ffp-contract=off (-fopenmp for the row-parallel loops).
 */
#include "hesa_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* fp16 <-> fp32                                                             */
/* ------------------------------------------------------------------------ */

float oracle_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do { man <<= 1; ++e; } while ((man & 0x400u) == 0);
            man &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + (127 - 15)) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t oracle_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFF) { /* inf / nan */
        return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0u));
    }
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u); /* overflow -> inf */
    if (e <= 0) {
        /* subnormal or zero in half precision */
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t half_man = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (half_man & 1u))) ++half_man;
        return (uint16_t)(sign | half_man);
    }
    uint32_t half = sign | ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) ++half; /* may carry into exp: correct */
    return (uint16_t)half;
}

/* ------------------------------------------------------------------------ */
/* Block geometry (src/model/gguf_loader.cpp:26-35)                          */
/* ------------------------------------------------------------------------ */

int oracle_block_elems(int qtype) {
    switch (qtype) {
        case ORACLE_Q4_0: case ORACLE_Q8_0: return 32;
        case ORACLE_Q4_K: case ORACLE_Q5_K: case ORACLE_Q6_K: return 256;
        default: return 0;
    }
}

int oracle_block_bytes(int qtype) {
    switch (qtype) {
        case ORACLE_Q4_0: return 18;
        case ORACLE_Q8_0: return 34;
        case ORACLE_Q4_K: return 144;
        case ORACLE_Q5_K: return 176;
        case ORACLE_Q6_K: return 210;
        default: return 0;
    }
}

size_t oracle_row_bytes(int qtype, int64_t k) {
    int be = oracle_block_elems(qtype);
    if (be == 0 || k % be != 0) return 0;
    return (size_t)(k / be) * (size_t)oracle_block_bytes(qtype);
}

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ------------------------------------------------------------------------ */
/* Dequantization: one block at a time                                       */
/* ------------------------------------------------------------------------ */

/* Q4_0: [d:f16][qs:16]; byte j -> weight j (low nibble), j+16 (high nibble);
 * value = d * (q - 8). */
static void deq_q4_0(const uint8_t* b, float* y) {
    const float d = oracle_fp16_to_fp32(rd16(b));
    const uint8_t* qs = b + 2;
    for (int j = 0; j < 16; ++j) {
        y[j]      = d * (float)((int)(qs[j] & 0x0F) - 8);
        y[j + 16] = d * (float)((int)(qs[j] >> 4) - 8);
    }
}

/* Q8_0: [d:f16][qs:int8 x32]; value = d * q. */
static void deq_q8_0(const uint8_t* b, float* y) {
    const float d = oracle_fp16_to_fp32(rd16(b));
    const int8_t* qs = (const int8_t*)(b + 2);
    for (int j = 0; j < 32; ++j) y[j] = d * (float)qs[j];
}

/* 6-bit (scale, min) pair j of the 12-byte K-quant scale field. */
static void kq_scale_min(const uint8_t* s, int j, int* sc, int* m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* Q4_K: [d:f16][dmin:f16][scales:12][qs:128]. 64-weight chunk c uses qs bytes
 * 32c..32c+31: low nibbles are sub-block 2c, high nibbles sub-block 2c+1.
 * value = (d*sc) * q - (dmin*m). */
static void deq_q4_k(const uint8_t* b, float* y) {
    const float d = oracle_fp16_to_fp32(rd16(b));
    const float dmin = oracle_fp16_to_fp32(rd16(b + 2));
    const uint8_t* sc = b + 4;
    const uint8_t* qs = b + 16;
    for (int c = 0; c < 4; ++c) {
        int s0, m0, s1, m1;
        kq_scale_min(sc, 2 * c, &s0, &m0);
        kq_scale_min(sc, 2 * c + 1, &s1, &m1);
        const float d0 = d * (float)s0, mm0 = dmin * (float)m0;
        const float d1 = d * (float)s1, mm1 = dmin * (float)m1;
        for (int l = 0; l < 32; ++l) {
            y[64 * c + l]      = d0 * (float)(qs[32 * c + l] & 0x0F) - mm0;
            y[64 * c + 32 + l] = d1 * (float)(qs[32 * c + l] >> 4) - mm1;
        }
    }
}

/* Q5_K: [d][dmin][scales:12][qh:32][qs:128]; as Q4_K plus a fifth bit: bit j
 * of qh[l] is the high bit of weight l of sub-block j. */
static void deq_q5_k(const uint8_t* b, float* y) {
    const float d = oracle_fp16_to_fp32(rd16(b));
    const float dmin = oracle_fp16_to_fp32(rd16(b + 2));
    const uint8_t* sc = b + 4;
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + 48;
    for (int c = 0; c < 4; ++c) {
        int s0, m0, s1, m1;
        kq_scale_min(sc, 2 * c, &s0, &m0);
        kq_scale_min(sc, 2 * c + 1, &s1, &m1);
        const float d0 = d * (float)s0, mm0 = dmin * (float)m0;
        const float d1 = d * (float)s1, mm1 = dmin * (float)m1;
        for (int l = 0; l < 32; ++l) {
            int q0 = (qs[32 * c + l] & 0x0F) | (((qh[l] >> (2 * c)) & 1) << 4);
            int q1 = (qs[32 * c + l] >> 4) | (((qh[l] >> (2 * c + 1)) & 1) << 4);
            y[64 * c + l]      = d0 * (float)q0 - mm0;
            y[64 * c + 32 + l] = d1 * (float)q1 - mm1;
        }
    }
}

/* Q6_K: [ql:128][qh:64][scales:int8 x16][d:f16]. Each 128-weight half h uses
 * ql[64h..64h+63] and qh[32h..32h+31]; 16-weight sub-block i has scale
 * scales[i]; q = (4 low bits | 2 high bits << 4) - 32; value = (d*sc) * q. */
static void deq_q6_k(const uint8_t* b, float* y) {
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* sc = (const int8_t*)(b + 192);
    const float d = oracle_fp16_to_fp32(rd16(b + 208));
    for (int h = 0; h < 2; ++h) {
        const uint8_t* l8 = ql + 64 * h;
        const uint8_t* h8 = qh + 32 * h;
        float* yy = y + 128 * h;
        const int8_t* s = sc + 8 * h;
        for (int l = 0; l < 32; ++l) {
            int is = l / 16;
            int q1 = (int)((l8[l] & 0x0F) | (((h8[l] >> 0) & 3) << 4)) - 32;
            int q2 = (int)((l8[l + 32] & 0x0F) | (((h8[l] >> 2) & 3) << 4)) - 32;
            int q3 = (int)((l8[l] >> 4) | (((h8[l] >> 4) & 3) << 4)) - 32;
            int q4 = (int)((l8[l + 32] >> 4) | (((h8[l] >> 6) & 3) << 4)) - 32;
            yy[l]      = (d * (float)s[is + 0]) * (float)q1;
            yy[l + 32] = (d * (float)s[is + 2]) * (float)q2;
            yy[l + 64] = (d * (float)s[is + 4]) * (float)q3;
            yy[l + 96] = (d * (float)s[is + 6]) * (float)q4;
        }
    }
}

int oracle_dequantize_row(int qtype, const void* src, float* dst, int64_t k) {
    const int be = oracle_block_elems(qtype);
    const int bb = oracle_block_bytes(qtype);
    if (be == 0 || k < 0 || k % be != 0) return 1;
    const uint8_t* p = (const uint8_t*)src;
    const int64_t nb = k / be;
    for (int64_t i = 0; i < nb; ++i) {
        const uint8_t* blk = p + i * bb;
        float* y = dst + i * be;
        switch (qtype) {
            case ORACLE_Q4_0: deq_q4_0(blk, y); break;
            case ORACLE_Q8_0: deq_q8_0(blk, y); break;
            case ORACLE_Q4_K: deq_q4_k(blk, y); break;
            case ORACLE_Q5_K: deq_q5_k(blk, y); break;
            case ORACLE_Q6_K: deq_q6_k(blk, y); break;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Quantization (seeded test-weight generator)                               */
/* ------------------------------------------------------------------------ */

static inline void wr16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)(v & 0xFF); p[1] = (uint8_t)(v >> 8); }

/* Round half away from zero, as ggml's reference Q8_0 quantizer rounds. */
static inline float round_away(float v) { return roundf(v); }

/* Q4_0, the published ggml reference rounding: d = (signed value of largest
 * magnitude) / -8, q = min(15, trunc(x/d + 8.5)). */
static void quant_q4_0(const float* x, uint8_t* b) {
    float amax = 0.0f, vmax = 0.0f;
    for (int j = 0; j < 32; ++j) {
        if (fabsf(x[j]) > amax) { amax = fabsf(x[j]); vmax = x[j]; }
    }
    const float d = vmax / -8.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    wr16(b, oracle_fp32_to_fp16(d));
    for (int j = 0; j < 16; ++j) {
        float v0 = x[j] * id + 8.5f;
        float v1 = x[j + 16] * id + 8.5f;
        int q0 = (int)v0; if (q0 > 15) q0 = 15; if (q0 < 0) q0 = 0;
        int q1 = (int)v1; if (q1 > 15) q1 = 15; if (q1 < 0) q1 = 0;
        b[2 + j] = (uint8_t)(q0 | (q1 << 4));
    }
}

/* Q8_0, the published ggml reference rounding: d = amax/127, q = round(x/d). */
static void quant_q8_0(const float* x, uint8_t* b) {
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) if (fabsf(x[j]) > amax) amax = fabsf(x[j]);
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    wr16(b, oracle_fp32_to_fp16(d));
    for (int j = 0; j < 32; ++j) {
        int q = (int)round_away(x[j] * id);
        if (q > 127) q = 127; if (q < -128) q = -128;
        b[2 + j] = (uint8_t)(int8_t)q;
    }
}

static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* Pack eight 6-bit (scale, min) pairs into the 12-byte K-quant field; the
 * inverse of kq_scale_min. */
static void kq_pack_scales(const int* sc, const int* m, uint8_t* s) {
    for (int j = 0; j < 4; ++j) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((m[j + 4] & 15) << 4));
    }
}

/* Asymmetric K-quant (Q4_K / Q5_K) with nq levels (16 or 32). Per 32-weight
 * sub-block: scale = (max - min)/(nq-1) with min clipped to <= 0, offset
 * = -min; both sets are quantized to 6 bits against the super-block maxima;
 * weights are then rounded against the quantized scale/offset. */
static void quant_kq_asym(const float* x, uint8_t* b, int nq, uint8_t* qout /* 256 */) {
    float scales[8], mins[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float mn = x[32 * j], mx = x[32 * j];
        for (int l = 1; l < 32; ++l) {
            float v = x[32 * j + l];
            if (v < mn) mn = v;
            if (v > mx) mx = v;
        }
        if (mn > 0.0f) mn = 0.0f;
        scales[j] = (mx - mn) / (float)(nq - 1);
        mins[j] = -mn;
        if (scales[j] > max_scale) max_scale = scales[j];
        if (mins[j] > max_min) max_min = mins[j];
    }
    const float d = max_scale / 63.0f;
    const float dmin = max_min / 63.0f;
    const uint16_t dh = oracle_fp32_to_fp16(d), dminh = oracle_fp32_to_fp16(dmin);
    const float dq = oracle_fp16_to_fp32(dh), dminq = oracle_fp16_to_fp32(dminh);
    int isc[8], imn[8];
    for (int j = 0; j < 8; ++j) {
        isc[j] = dq > 0.0f ? clampi((int)round_away(scales[j] / dq), 0, 63) : 0;
        imn[j] = dminq > 0.0f ? clampi((int)round_away(mins[j] / dminq), 0, 63) : 0;
    }
    wr16(b, dh);
    wr16(b + 2, dminh);
    kq_pack_scales(isc, imn, b + 4);
    for (int j = 0; j < 8; ++j) {
        const float ds = dq * (float)isc[j];
        const float dm = dminq * (float)imn[j];
        for (int l = 0; l < 32; ++l) {
            int q = 0;
            if (ds > 0.0f) q = clampi((int)round_away((x[32 * j + l] + dm) / ds), 0, nq - 1);
            qout[32 * j + l] = (uint8_t)q;
        }
    }
}

static void quant_q4_k(const float* x, uint8_t* b) {
    uint8_t q[256];
    quant_kq_asym(x, b, 16, q);
    uint8_t* qs = b + 16;
    for (int c = 0; c < 4; ++c)
        for (int l = 0; l < 32; ++l)
            qs[32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
}

static void quant_q5_k(const float* x, uint8_t* b) {
    uint8_t q[256];
    quant_kq_asym(x, b, 32, q);
    uint8_t* qh = b + 16;
    uint8_t* qs = b + 48;
    memset(qh, 0, 32);
    for (int c = 0; c < 4; ++c) {
        for (int l = 0; l < 32; ++l) {
            int q0 = q[64 * c + l], q1 = q[64 * c + 32 + l];
            qs[32 * c + l] = (uint8_t)((q0 & 15) | ((q1 & 15) << 4));
            qh[l] |= (uint8_t)(((q0 >> 4) & 1) << (2 * c));
            qh[l] |= (uint8_t)(((q1 >> 4) & 1) << (2 * c + 1));
        }
    }
}

/* Q6_K: symmetric, 16-weight sub-blocks. Sub-block scale = (signed value of
 * largest magnitude) / -32, quantized to int8 against d = max|scale|/127;
 * q = round(x / (d*sc)) + 32 clipped to 0..63. */
static void quant_q6_k(const float* x, uint8_t* b) {
    float scales[16];
    float amax_s = 0.0f, vmax_s = 0.0f;
    for (int i = 0; i < 16; ++i) {
        float am = 0.0f, vm = 0.0f;
        for (int l = 0; l < 16; ++l) {
            float v = x[16 * i + l];
            if (fabsf(v) > am) { am = fabsf(v); vm = v; }
        }
        scales[i] = vm / -32.0f;
        if (fabsf(scales[i]) > amax_s) { amax_s = fabsf(scales[i]); vmax_s = scales[i]; }
    }
    const float d = vmax_s / -128.0f;
    const uint16_t dh = oracle_fp32_to_fp16(d);
    const float dq = oracle_fp16_to_fp32(dh);
    int8_t isc[16];
    for (int i = 0; i < 16; ++i) {
        int s = dq != 0.0f ? (int)round_away(scales[i] / dq) : 0;
        isc[i] = (int8_t)clampi(s, -128, 127);
    }
    uint8_t q[256];
    for (int i = 0; i < 16; ++i) {
        const float ds = dq * (float)isc[i];
        for (int l = 0; l < 16; ++l) {
            int v = 32;
            if (ds != 0.0f) v = clampi((int)round_away(x[16 * i + l] / ds) + 32, 0, 63);
            q[16 * i + l] = (uint8_t)v;
        }
    }
    uint8_t* ql = b;
    uint8_t* qh = b + 128;
    memset(ql, 0, 128);
    memset(qh, 0, 64);
    for (int h = 0; h < 2; ++h) {
        for (int l = 0; l < 32; ++l) {
            int q1 = q[128 * h + l], q2 = q[128 * h + l + 32];
            int q3 = q[128 * h + l + 64], q4 = q[128 * h + l + 96];
            ql[64 * h + l] = (uint8_t)((q1 & 15) | ((q3 & 15) << 4));
            ql[64 * h + l + 32] = (uint8_t)((q2 & 15) | ((q4 & 15) << 4));
            qh[32 * h + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
        }
    }
    memcpy(b + 192, isc, 16);
    wr16(b + 208, dh);
}

int oracle_quantize_row(int qtype, const float* src, void* dst, int64_t k) {
    const int be = oracle_block_elems(qtype);
    const int bb = oracle_block_bytes(qtype);
    if (be == 0 || k < 0 || k % be != 0) return 1;
    uint8_t* p = (uint8_t*)dst;
    for (int64_t i = 0; i < k / be; ++i) {
        const float* x = src + i * be;
        uint8_t* b = p + i * bb;
        switch (qtype) {
            case ORACLE_Q4_0: quant_q4_0(x, b); break;
            case ORACLE_Q8_0: quant_q8_0(x, b); break;
            case ORACLE_Q4_K: quant_q4_k(x, b); break;
            case ORACLE_Q5_K: quant_q5_k(x, b); break;
            case ORACLE_Q6_K: quant_q6_k(x, b); break;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Contraction: cpu_matmul_f32 semantics on the dequantized row              */
/* ------------------------------------------------------------------------ */

int oracle_qmatvec(int qtype, const void* w, int64_t n_out, int64_t k,
                   const float* x, int64_t ldx, int64_t batch,
                   float* y, int64_t ldy, float scale, int n_threads) {
    const size_t rb = oracle_row_bytes(qtype, k);
    if (rb == 0 || n_out < 0 || batch < 1 || ldx < k || ldy < n_out) return 1;
    if (n_threads < 1) n_threads = 1;
    int err = 0;
#pragma omp parallel num_threads(n_threads)
    {
        float* row = (float*)malloc((size_t)k * sizeof(float));
        if (!row) {
#pragma omp atomic write
            err = 1;
        } else {
#pragma omp for schedule(static)
            for (int64_t n = 0; n < n_out; ++n) {
                oracle_dequantize_row(qtype, (const uint8_t*)w + (size_t)n * rb, row, k);
                for (int64_t b = 0; b < batch; ++b) {
                    const float* xb = x + b * ldx;
                    float sum = 0.0f;
                    for (int64_t i = 0; i < k; ++i) sum += row[i] * xb[i];
                    y[b * ldy + n] = sum * scale;
                }
            }
            free(row);
        }
    }
    return err;
}

/* ------------------------------------------------------------------------ */
/* Decode-step primitives                                                    */
/* ------------------------------------------------------------------------ */

/* cpu_rms_norm_f32 (cpu_backend.cpp:72-89) for one row. */
void oracle_rms_norm(const float* in, const float* weight, float* out,
                     int64_t n, float eps) {
    float sum_sq = 0.0f;
    for (int64_t j = 0; j < n; ++j) sum_sq += in[j] * in[j];
    const float inv_rms = 1.0f / sqrtf(sum_sq / (float)n + eps);
    for (int64_t j = 0; j < n; ++j) out[j] = in[j] * inv_rms * weight[j];
}

/* cpu_silu_f32 (cpu_backend.cpp:91-96) of gate, times up. */
void oracle_silu_mul(const float* gate, const float* up, float* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        const float g = gate[i];
        const float s = g / (1.0f + expf(-g));
        out[i] = s * up[i];
    }
}

/* The angle table of cpu_rope_f32 (cpu_backend.cpp:103-112) for one
 * position: freq_d = 1 / base^(2d/head_dim), theta = pos * freq_d. */
void oracle_rope_table(float* cos_out, float* sin_out, int32_t pos,
                       int64_t head_dim, float freq_base) {
    const int64_t half = head_dim / 2;
    for (int64_t d = 0; d < half; ++d) {
        const float freq = 1.0f / powf(freq_base, 2.0f * (float)d / (float)head_dim);
        const float theta = (float)pos * freq;
        cos_out[d] = cosf(theta);
        sin_out[d] = sinf(theta);
    }
}

/* cpu_rope_f32 (cpu_backend.cpp:98-120): rotate-half pairs (d, d+half). */
void oracle_rope(float* data, int32_t pos, int64_t n_heads, int64_t head_dim,
                 float freq_base) {
    const int64_t half = head_dim / 2;
    float* c = (float*)malloc((size_t)half * sizeof(float));
    float* s = (float*)malloc((size_t)half * sizeof(float));
    if (!c || !s) { free(c); free(s); return; }
    oracle_rope_table(c, s, pos, head_dim, freq_base);
    for (int64_t h = 0; h < n_heads; ++h) {
        float* row = data + h * head_dim;
        for (int64_t d = 0; d < half; ++d) {
            const float x0 = row[d], x1 = row[d + half];
            row[d] = x0 * c[d] - x1 * s[d];
            row[d + half] = x0 * s[d] + x1 * c[d];
        }
    }
    free(c);
    free(s);
}

/* Single-query attention with the semantics of the reference SDPA
 * (cpu_backend.cpp:225-294): score = (sum_d q*k) * (1/sqrt(head_dim)),
 * softmax as cpu_softmax_f32 (:48-70), out = sum_j p_j * v_j in j order.
 * Extended to GQA (kv head = h / (n_head/n_kv_head)) over fp16 K/V. The
 * output is zero-initialised (the reference accumulates into `out`). */
void oracle_attention_f16kv(const float* q, const uint16_t* k_cache,
                            const uint16_t* v_cache, float* out,
                            int64_t n_head, int64_t n_kv_head,
                            int64_t head_dim, int64_t n_ctx, int n_threads) {
    const int64_t group = n_head / n_kv_head;
    const float sc = 1.0f / sqrtf((float)head_dim);
    if (n_threads < 1) n_threads = 1;
#pragma omp parallel for num_threads(n_threads) schedule(static)
    for (int64_t h = 0; h < n_head; ++h) {
        const int64_t kvh = h / group;
        const float* qh = q + h * head_dim;
        float* p = (float*)malloc((size_t)n_ctx * sizeof(float));
        if (!p) continue;
        for (int64_t j = 0; j < n_ctx; ++j) {
            const uint16_t* kj = k_cache + (j * n_kv_head + kvh) * head_dim;
            float sum = 0.0f;
            for (int64_t d = 0; d < head_dim; ++d) sum += qh[d] * oracle_fp16_to_fp32(kj[d]);
            p[j] = sum * sc;
        }
        float mx = p[0];
        for (int64_t j = 1; j < n_ctx; ++j) if (p[j] > mx) mx = p[j];
        float s = 0.0f;
        for (int64_t j = 0; j < n_ctx; ++j) { p[j] = expf(p[j] - mx); s += p[j]; }
        const float inv = 1.0f / s;
        for (int64_t j = 0; j < n_ctx; ++j) p[j] *= inv;
        float* o = out + h * head_dim;
        for (int64_t d = 0; d < head_dim; ++d) o[d] = 0.0f;
        for (int64_t j = 0; j < n_ctx; ++j) {
            const uint16_t* vj = v_cache + (j * n_kv_head + kvh) * head_dim;
            for (int64_t d = 0; d < head_dim; ++d) o[d] += p[j] * oracle_fp16_to_fp32(vj[d]);
        }
        free(p);
    }
}

/* Llama-style decode step composed from the primitives above:
 *   for each layer:
 *     h = rms_norm(x, attn_norm)
 *     q = Wq h; k = Wk h; v = Wv h; rope(q), rope(k) at pos
 *     K/V slot pos % ctx <- fp16(k), fp16(v)
 *     a = attention(q, K, V over min(pos+1, ctx) slots)
 *     x = x + Wo a
 *     h = rms_norm(x, ffn_norm)
 *     x = x + W_down (silu(W_gate h) * (W_up h))
 *   logits = W_out rms_norm(x, out_norm)
 */
/* ------------------------------------------------------------------------ */
/* The same primitives with every sum accumulated in fp64 (each result       */
/* rounded to fp32 once). Not a restatement of the reference: a higher-      */
/* precision measuring instrument, used to tell how far the fp32 decode      */
/* step itself (the reference's arithmetic) is from the exact result.        */
/* ------------------------------------------------------------------------ */

static int qmatvec_f64(int qtype, const void* w, int64_t n_out, int64_t k, const float* x,
                       float* y, int n_threads) {
    const size_t rb = oracle_row_bytes(qtype, k);
    if (rb == 0 || n_out < 0) return 1;
    if (n_threads < 1) n_threads = 1;
    int err = 0;
#pragma omp parallel num_threads(n_threads)
    {
        float* row = (float*)malloc((size_t)k * sizeof(float));
        if (!row) {
#pragma omp atomic write
            err = 1;
        } else {
#pragma omp for schedule(static)
            for (int64_t n = 0; n < n_out; ++n) {
                oracle_dequantize_row(qtype, (const uint8_t*)w + (size_t)n * rb, row, k);
                double sum = 0.0;
                for (int64_t i = 0; i < k; ++i) sum += (double)row[i] * (double)x[i];
                y[n] = (float)sum;
            }
            free(row);
        }
    }
    return err;
}

static void rms_norm_f64(const float* in, const float* weight, float* out, int64_t n, float eps) {
    double ss = 0.0;
    for (int64_t j = 0; j < n; ++j) ss += (double)in[j] * (double)in[j];
    const double inv = 1.0 / sqrt(ss / (double)n + (double)eps);
    for (int64_t j = 0; j < n; ++j) out[j] = (float)((double)in[j] * inv * (double)weight[j]);
}

static void rope_f64(float* data, int32_t pos, int64_t n_heads, int64_t head_dim, float base) {
    const int64_t half = head_dim / 2;
    for (int64_t h = 0; h < n_heads; ++h) {
        float* row = data + h * head_dim;
        for (int64_t d = 0; d < half; ++d) {
            const double th = (double)pos * pow((double)base, -2.0 * (double)d / (double)head_dim);
            const double x0 = row[d], x1 = row[d + half];
            row[d] = (float)(x0 * cos(th) - x1 * sin(th));
            row[d + half] = (float)(x0 * sin(th) + x1 * cos(th));
        }
    }
}

static void attention_f64(const float* q, const uint16_t* k_cache, const uint16_t* v_cache, float* out,
                          int64_t n_head, int64_t n_kv_head, int64_t head_dim, int64_t n_ctx, int n_threads) {
    const int64_t group = n_head / n_kv_head;
    const double sc = 1.0 / sqrt((double)head_dim);
    if (n_threads < 1) n_threads = 1;
#pragma omp parallel for num_threads(n_threads) schedule(static)
    for (int64_t h = 0; h < n_head; ++h) {
        const int64_t kvh = h / group;
        const float* qh = q + h * head_dim;
        double* p = (double*)malloc((size_t)n_ctx * sizeof(double));
        double* o = (double*)calloc((size_t)head_dim, sizeof(double));
        if (p && o) {
            double mx = -1e300;
            for (int64_t j = 0; j < n_ctx; ++j) {
                const uint16_t* kj = k_cache + (j * n_kv_head + kvh) * head_dim;
                double sum = 0.0;
                for (int64_t d = 0; d < head_dim; ++d) sum += (double)qh[d] * (double)oracle_fp16_to_fp32(kj[d]);
                p[j] = sum * sc;
                if (p[j] > mx) mx = p[j];
            }
            double s = 0.0;
            for (int64_t j = 0; j < n_ctx; ++j) { p[j] = exp(p[j] - mx); s += p[j]; }
            for (int64_t j = 0; j < n_ctx; ++j) {
                const uint16_t* vj = v_cache + (j * n_kv_head + kvh) * head_dim;
                const double pj = p[j] / s;
                for (int64_t d = 0; d < head_dim; ++d) o[d] += pj * (double)oracle_fp16_to_fp32(vj[d]);
            }
            for (int64_t d = 0; d < head_dim; ++d) out[h * head_dim + d] = (float)o[d];
        }
        free(p);
        free(o);
    }
}

/* The decode step of oracle_decode_step with the fp64-accumulating
 * primitives above (the K/V rows written to the cache are the same fp16
 * roundings of the step's k and v). */
int oracle_decode_step_f64(const oracle_model_cfg* cfg, const oracle_layer* layers,
                           const float* out_norm, const void* w_out,
                           const float* x_in, int32_t pos, float* logits, int n_threads) {
    const int64_t D = cfg->d_model, HD = cfg->head_dim;
    const int64_t QD = cfg->n_head * HD, KD = cfg->n_kv_head * HD, F = cfg->d_ff;
    double* x = (double*)malloc((size_t)D * 8);
    float* xf = (float*)malloc((size_t)D * 4);
    float* h = (float*)malloc((size_t)D * 4);
    float* q = (float*)malloc((size_t)QD * 4);
    float* kk = (float*)malloc((size_t)KD * 4);
    float* vv = (float*)malloc((size_t)KD * 4);
    float* a = (float*)malloc((size_t)QD * 4);
    float* o = (float*)malloc((size_t)D * 4);
    float* g = (float*)malloc((size_t)F * 4);
    float* u = (float*)malloc((size_t)F * 4);
    int err = !(x && xf && h && q && kk && vv && a && o && g && u);
    if (!err) {
        for (int64_t i = 0; i < D; ++i) x[i] = x_in[i];
        const int64_t slot = pos % cfg->ctx;
        const int64_t n_ctx = (pos + 1 < cfg->ctx) ? pos + 1 : cfg->ctx;
        for (int64_t l = 0; l < cfg->n_layer && !err; ++l) {
            const oracle_layer* L = &layers[l];
            for (int64_t i = 0; i < D; ++i) xf[i] = (float)x[i];
            rms_norm_f64(xf, L->attn_norm, h, D, cfg->rms_eps);
            err |= qmatvec_f64(cfg->qtype, L->wq, QD, D, h, q, n_threads);
            err |= qmatvec_f64(cfg->qtype, L->wk, KD, D, h, kk, n_threads);
            err |= qmatvec_f64(cfg->qtype, L->wv, KD, D, h, vv, n_threads);
            rope_f64(q, pos, cfg->n_head, HD, cfg->rope_base);
            rope_f64(kk, pos, cfg->n_kv_head, HD, cfg->rope_base);
            for (int64_t i = 0; i < KD; ++i) {
                L->k_cache[slot * KD + i] = oracle_fp32_to_fp16(kk[i]);
                L->v_cache[slot * KD + i] = oracle_fp32_to_fp16(vv[i]);
            }
            attention_f64(q, L->k_cache, L->v_cache, a, cfg->n_head, cfg->n_kv_head, HD, n_ctx, n_threads);
            err |= qmatvec_f64(cfg->qtype, L->wo, D, QD, a, o, n_threads);
            for (int64_t i = 0; i < D; ++i) x[i] += o[i];
            for (int64_t i = 0; i < D; ++i) xf[i] = (float)x[i];
            rms_norm_f64(xf, L->ffn_norm, h, D, cfg->rms_eps);
            err |= qmatvec_f64(cfg->qtype, L->w_gate, F, D, h, g, n_threads);
            err |= qmatvec_f64(cfg->qtype, L->w_up, F, D, h, u, n_threads);
            for (int64_t i = 0; i < F; ++i) {
                const double gg = g[i];
                g[i] = (float)(gg / (1.0 + exp(-gg)) * (double)u[i]);
            }
            err |= qmatvec_f64(cfg->qtype, L->w_down, D, F, g, o, n_threads);
            for (int64_t i = 0; i < D; ++i) x[i] += o[i];
        }
        if (!err) {
            for (int64_t i = 0; i < D; ++i) xf[i] = (float)x[i];
            rms_norm_f64(xf, out_norm, h, D, cfg->rms_eps);
            err |= qmatvec_f64(cfg->qtype, w_out, cfg->vocab, D, h, logits, n_threads);
        }
    }
    free(x); free(xf); free(h); free(q); free(kk); free(vv); free(a); free(o); free(g); free(u);
    return err;
}

int oracle_decode_step(const oracle_model_cfg* cfg, const oracle_layer* layers,
                       const float* out_norm, const void* w_out,
                       const float* x_in, int32_t pos, float* logits,
                       int n_threads) {
    const int64_t D = cfg->d_model, HD = cfg->head_dim;
    const int64_t QD = cfg->n_head * HD, KD = cfg->n_kv_head * HD, F = cfg->d_ff;
    float* x = (float*)malloc((size_t)D * 4);
    float* h = (float*)malloc((size_t)D * 4);
    float* q = (float*)malloc((size_t)QD * 4);
    float* kk = (float*)malloc((size_t)KD * 4);
    float* vv = (float*)malloc((size_t)KD * 4);
    float* a = (float*)malloc((size_t)QD * 4);
    float* o = (float*)malloc((size_t)D * 4);
    float* g = (float*)malloc((size_t)F * 4);
    float* u = (float*)malloc((size_t)F * 4);
    int err = !(x && h && q && kk && vv && a && o && g && u);
    if (!err) {
        memcpy(x, x_in, (size_t)D * 4);
        const int64_t slot = pos % cfg->ctx;
        const int64_t n_ctx = (pos + 1 < cfg->ctx) ? pos + 1 : cfg->ctx;
        for (int64_t l = 0; l < cfg->n_layer && !err; ++l) {
            const oracle_layer* L = &layers[l];
            oracle_rms_norm(x, L->attn_norm, h, D, cfg->rms_eps);
            err |= oracle_qmatvec(cfg->qtype, L->wq, QD, D, h, D, 1, q, QD, 1.0f, n_threads);
            err |= oracle_qmatvec(cfg->qtype, L->wk, KD, D, h, D, 1, kk, KD, 1.0f, n_threads);
            err |= oracle_qmatvec(cfg->qtype, L->wv, KD, D, h, D, 1, vv, KD, 1.0f, n_threads);
            oracle_rope(q, pos, cfg->n_head, HD, cfg->rope_base);
            oracle_rope(kk, pos, cfg->n_kv_head, HD, cfg->rope_base);
            for (int64_t i = 0; i < KD; ++i) {
                L->k_cache[slot * KD + i] = oracle_fp32_to_fp16(kk[i]);
                L->v_cache[slot * KD + i] = oracle_fp32_to_fp16(vv[i]);
            }
            oracle_attention_f16kv(q, L->k_cache, L->v_cache, a, cfg->n_head,
                                   cfg->n_kv_head, HD, n_ctx, n_threads);
            err |= oracle_qmatvec(cfg->qtype, L->wo, D, QD, a, QD, 1, o, D, 1.0f, n_threads);
            for (int64_t i = 0; i < D; ++i) x[i] = x[i] + o[i];
            oracle_rms_norm(x, L->ffn_norm, h, D, cfg->rms_eps);
            err |= oracle_qmatvec(cfg->qtype, L->w_gate, F, D, h, D, 1, g, F, 1.0f, n_threads);
            err |= oracle_qmatvec(cfg->qtype, L->w_up, F, D, h, D, 1, u, F, 1.0f, n_threads);
            oracle_silu_mul(g, u, g, F);
            err |= oracle_qmatvec(cfg->qtype, L->w_down, D, F, g, F, 1, o, D, 1.0f, n_threads);
            for (int64_t i = 0; i < D; ++i) x[i] = x[i] + o[i];
        }
        if (!err) {
            oracle_rms_norm(x, out_norm, h, D, cfg->rms_eps);
            err |= oracle_qmatvec(cfg->qtype, w_out, cfg->vocab, D, h, D, 1, logits,
                                  cfg->vocab, 1.0f, n_threads);
        }
    }
    free(x); free(h); free(q); free(kk); free(vv); free(a); free(o); free(g); free(u);
    return err;
}
