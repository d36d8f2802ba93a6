/*
 * hesa_oracle.h -- CPU restatement of the GGUF block-quantized matvec path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the oracle: the parity tests,
 * smoke() and bench.py's CPU-baseline leg call it to produce expected values.
 * No product code path may link, load or call it.
 *
 * What it restates, and where the semantics come from:
 *   - block byte sizes and GGUF type ids: src/model/gguf_loader.cpp:19-38 and
 *     src/model/gguf_loader.hpp:15-45 of hesa-llm;
 *   - the bit layout inside each block: the public GGUF/ggml block format
 *     (Q4_0, Q8_0, Q4_K, Q5_K, Q6_K), cross-checked against the independent
 *     numpy decoder of the `gguf` 0.19.0 Python package (tests/golden);
 *   - the contraction: cpu_matmul_f32 (src/backend/cpu_backend.cpp:24-41),
 *     out = (sum_k a*b) * scale, fp32, k in increasing order, applied to the
 *     dequantized weight row;
 *   - the decode-step primitives: cpu_rms_norm_f32 (:72-89), cpu_silu_f32
 *     (:91-96), cpu_rope_f32 (:98-120), cpu_softmax_f32 (:48-70) and the SDPA
 *     scale 1/sqrt(head_dim) (:259).
 *
 * All arithmetic is compiled with -ffp-contract=off so every multiply and add
 * rounds separately, exactly as written.
 */
#ifndef HESA_ORACLE_H
#define HESA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF type ids (src/model/gguf_loader.hpp:15-45). */
enum {
    ORACLE_Q4_0 = 2,
    ORACLE_Q8_0 = 8,
    ORACLE_Q4_K = 12,
    ORACLE_Q5_K = 13,
    ORACLE_Q6_K = 14
};

float    oracle_fp16_to_fp32(uint16_t h);
uint16_t oracle_fp32_to_fp16(float f); /* round to nearest even */

int    oracle_block_elems(int qtype);  /* 32 or 256; 0 if unknown */
int    oracle_block_bytes(int qtype);  /* 18, 34, 144, 176, 210; 0 if unknown */
size_t oracle_row_bytes(int qtype, int64_t k);

/* Decode one row of k weights (k a multiple of the block size). 0 = ok. */
int oracle_dequantize_row(int qtype, const void* src, float* dst, int64_t k);

/* Deterministic round-to-nearest quantizer used to build seeded test weights.
 * Q4_0 and Q8_0 follow the published ggml reference rounding; the K-quants use
 * a min/max RTN of this library's own design (any valid block is acceptable
 * input to the matvec). 0 = ok. */
int oracle_quantize_row(int qtype, const float* src, void* dst, int64_t k);

/* y[b*ldy + n] = scale * sum_k deq(W[n,k]) * x[b*ldx + k], fp32, k ascending.
 * W is row-major [n_out, k] of packed blocks. Rows are split across
 * n_threads OpenMP threads; each row's sum is sequential, so the result does
 * not depend on the thread count. 0 = ok. */
int oracle_qmatvec(int qtype, const void* w, int64_t n_out, int64_t k,
                   const float* x, int64_t ldx, int64_t batch,
                   float* y, int64_t ldy, float scale, int n_threads);

/* Decode-step primitives (single token). */
void oracle_rms_norm(const float* in, const float* weight, float* out,
                     int64_t n, float eps);
void oracle_silu_mul(const float* gate, const float* up, float* out, int64_t n);
void oracle_rope(float* data, int32_t pos, int64_t n_heads, int64_t head_dim,
                 float freq_base);
void oracle_rope_table(float* cos_out, float* sin_out, int32_t pos,
                       int64_t head_dim, float freq_base);

/* Single-query GQA attention over an fp16 ring-buffer KV cache.
 * q: [n_head, head_dim] fp32; k_cache/v_cache: [ctx, n_kv_head, head_dim]
 * fp16 bits; attends to slots 0..n_ctx-1; out: [n_head, head_dim]. */
void oracle_attention_f16kv(const float* q, const uint16_t* k_cache,
                            const uint16_t* v_cache, float* out,
                            int64_t n_head, int64_t n_kv_head,
                            int64_t head_dim, int64_t n_ctx, int n_threads);

/* Llama-style decode step over Q-type weights (weights_* are packed rows).
 * See oracle_decode_step's definition for the exact op order. */
typedef struct {
    int64_t n_layer, d_model, n_head, n_kv_head, head_dim, d_ff, vocab;
    int64_t ctx;        /* KV ring capacity */
    float   rms_eps;
    float   rope_base;
    int     qtype;      /* type of every projection and the LM head */
} oracle_model_cfg;

typedef struct {
    const void*  wq;     /* [n_head*head_dim, d_model] */
    const void*  wk;     /* [n_kv_head*head_dim, d_model] */
    const void*  wv;
    const void*  wo;     /* [d_model, n_head*head_dim] */
    const void*  w_gate; /* [d_ff, d_model] */
    const void*  w_up;
    const void*  w_down; /* [d_model, d_ff] */
    const float* attn_norm; /* [d_model] */
    const float* ffn_norm;
    uint16_t*    k_cache;   /* [ctx, n_kv_head, head_dim] fp16 */
    uint16_t*    v_cache;
} oracle_layer;

/* x: [d_model] embedding of the current token (in), logits: [vocab] (out).
 * pos is the absolute position; the KV slot written is pos % ctx and the
 * attention spans min(pos+1, ctx) slots. */
int oracle_decode_step(const oracle_model_cfg* cfg, const oracle_layer* layers,
                       const float* out_norm, const void* w_out,
                       const float* x_in, int32_t pos, float* logits,
                       int n_threads);

/* oracle_decode_step with every sum accumulated in fp64 (the residual stream
 * kept in fp64, each primitive's result rounded to fp32 once): not the
 * reference's arithmetic, but a higher-precision measure of the exact result,
 * to separate the fp32 rounding of the reference's own step from a kernel's
 * deviation. Writes the same K/V slot. */
int oracle_decode_step_f64(const oracle_model_cfg* cfg, const oracle_layer* layers,
                           const float* out_norm, const void* w_out,
                           const float* x_in, int32_t pos, float* logits, int n_threads);

#ifdef __cplusplus
}
#endif
#endif
