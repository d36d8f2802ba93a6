/*
 * hesa_cuda.h -- C ABI of the B200 (sm_100a) CUDA backend for hesa-llm's
 * decode hot path: GGUF block-quantized weight x fp32 activation matvec with
 * fused dequantization.
 *
 * Conventions shared by every entry point:
 *   - Pointers are device pointers unless a parameter says "host". The
 *     library never allocates or frees device memory on these paths; the
 *     caller owns every buffer, including the workspace.
 *   - Weights W are row-major [n_out, k]: each row is k/block_elems packed
 *     GGUF blocks, rows back to back (the layout Model::load produces after
 *     reversing the GGUF dims, src/model/gguf_loader.cpp:291-316). W must be
 *     16-byte aligned.
 *   - qtype is the GGUF/ggml type id (src/model/gguf_loader.hpp:15-45):
 *     Q4_0 = 2, Q8_0 = 8, Q4_K = 12, Q5_K = 13, Q6_K = 14.
 *   - Return value: 0 on success, else a hesa::Error value
 *     (include/hesa/result.hpp:14-30): INVALID_ARGUMENT = 2,
 *     BACKEND_NOT_AVAILABLE = 3, SHAPE_MISMATCH = 6, INVALID_FORMAT = 8,
 *     CUDA_ERROR = 9, INTERNAL_ERROR = 14. Nothing throws across the ABI.
 *   - Calls are asynchronous on `stream` (a cudaStream_t; NULL is the legacy
 *     default stream).
 */
#ifndef HESA_CUDA_H
#define HESA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define HESA_CUDA_API __attribute__((visibility("default")))
#else
#define HESA_CUDA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum hesa_cuda_qtype {
    HESA_CUDA_Q4_0 = 2,
    HESA_CUDA_Q8_0 = 8,
    HESA_CUDA_Q4_K = 12,
    HESA_CUDA_Q5_K = 13,
    HESA_CUDA_Q6_K = 14
};

enum hesa_cuda_status {
    HESA_CUDA_OK = 0,
    HESA_CUDA_INVALID_ARGUMENT = 2,
    HESA_CUDA_BACKEND_NOT_AVAILABLE = 3,
    HESA_CUDA_SHAPE_MISMATCH = 6,
    HESA_CUDA_INVALID_FORMAT = 8,
    HESA_CUDA_ERROR = 9,
    HESA_CUDA_INTERNAL_ERROR = 14
};

/* Library version and the device architecture the kernels were built for
 * ("sm_100a"). */
HESA_CUDA_API const char* hesa_cuda_version(void);

/* Bytes of one packed row of k weights of qtype (0 if k is not a multiple of
 * the block size or qtype is unsupported). Mirrors gguf_type_size
 * (src/model/gguf_loader.cpp:19-38) for one row. */
HESA_CUDA_API size_t hesa_cuda_row_bytes(int qtype, int64_t k);

/* Device workspace the matvec needs for n_out x k at this batch, in bytes
 * (arrival counters, cross-CTA partial sums and, for batch >= 2, the staged
 * activations). The workspace must be zero-filled once before its first use;
 * every successful call leaves its counters at zero again, so it can be
 * reused by later calls on the same stream, at any batch up to the one it was
 * sized for. After a call that reports HESA_CUDA_ERROR, zero it again. */
HESA_CUDA_API size_t hesa_cuda_qmatvec_workspace_size(int qtype, int64_t n_out, int64_t k, int64_t batch);

/* y[b*ldy + n] = scale * sum_k deq(W[n,k]) * x[b*ldx + k]
 * for n < n_out, b < batch. fp32 activations and outputs.
 *
 * Replaces, for quantized `a`, hesa::Backend::matmul(TensorView a,
 * TensorView b, TensorView out, float scale) (include/hesa/backend.hpp:43-44)
 * whose CPU semantics are cpu_matmul_f32 (src/backend/cpu_backend.cpp:24-41):
 * a = W [n_out, k], b = x^T [k, batch], out = y^T [n_out, batch].
 * Batch 1 is one streaming pass over W on CUDA cores. Q4_K, Q5_K, Q8_0 and
 * Q4_0 with batch >= 3 (k a multiple of 256; batch 2 too when k > 24576) run
 * on the tensor cores, reading W once per 16 activation rows (Q4_K, Q5_K) or
 * once per 8 (Q8_0, Q4_0); Q6_K, and batch 2 with k <= 24576, make one pass
 * per batch column.
 * x and y must be 16-byte aligned with ldx, ldy multiples of 4.
 * The workspace is used by the batched kernel and the split-row kernel (rows
 * longer than 24576 weights, or matrices too tall for one strip of rows per
 * SM); a call that needs it and gets less than
 * hesa_cuda_qmatvec_workspace_size bytes fails with
 * HESA_CUDA_INVALID_ARGUMENT before launching anything.
 * Consecutive calls on one stream overlap (programmatic dependent launch):
 * a call starts fetching W while the previous kernel on the stream finishes,
 * and reads x only after that kernel has completed. W must therefore not be
 * written by the kernel launched immediately before the call. */
HESA_CUDA_API int hesa_cuda_qmatvec(int qtype, const void* w, int64_t n_out, int64_t k,
                                    const float* x, int64_t ldx, int64_t batch,
                                    float* y, int64_t ldy, float scale,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* hesa_cuda_qmatvec without a workspace argument, for callers that cannot
 * allocate device memory: code embedded in a host program that owns every
 * device allocation through its own pool or budget (a stray cudaMalloc would
 * break that accounting), or a serving loop that must not allocate after
 * start-up. Same arguments, semantics and results as hesa_cuda_qmatvec
 * (batch >= 2 takes one batch-1 pass per activation row instead of the
 * tensor-core path, which needs a workspace); it has no counterpart in the
 * reference.
 *   - Shapes the row-strip kernel takes (k <= 24576, the batch-1 path of
 *     hesa_cuda_qmatvec) need no scratch at all, at any n_out. Longer rows
 *     run the streaming kernel, whose scratch (arrival counters and
 *     cross-warp partial sums) is a fixed 512 KB array inside this library,
 *     held on every GPU that loads it until the process exits; there n_out is
 *     limited to 65536 rows, and larger n_out is rejected with
 *     HESA_CUDA_SHAPE_MISMATCH and a message before anything is launched.
 *   - Nothing is allocated: no cudaMalloc, cudaFree or allocating library
 *     call. The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture.
 *   - Every call shares the array and clears the part that must start at
 *     zero, so calls that overlap on the GPU (different streams, or several
 *     host threads) race and give wrong results: serialize them. */
HESA_CUDA_API int hesa_cuda_qmatvec_noalloc(int qtype, const void* w, int64_t n_out, int64_t k,
                                            const float* x, int64_t ldx, int64_t batch,
                                            float* y, int64_t ldy, float scale, void* stream);

/* out[r*ldo + i] = deq(W[r, i]) for r < n_rows, i < k: the exact fp32 value
 * of every weight, bit-identical to the GGUF definition ((d*sc)*q - dmin*m
 * with each operation rounded separately). Used for embedding-row lookups
 * and as the bit-exactness check of the decoders. Replaces nothing in the
 * reference (it has no dequantizer; CPU_Backend::quantize is a stub,
 * src/backend/cpu_backend.cpp:296-302). */
HESA_CUDA_API int hesa_cuda_dequantize(int qtype, const void* w, int64_t n_rows, int64_t k,
                                       float* out, int64_t ldo, void* stream);

/* dst <- src [n_rows, k] fp32 (row stride ld_src floats) quantized to
 * packed GGUF rows of qtype (n_rows * hesa_cuda_row_bytes(qtype, k) bytes),
 * deterministic round-to-nearest: Q4_0 / Q8_0 with the published ggml
 * reference rounding, the K-quants with a min/max RTN (6-bit sub-block
 * scale/min for Q4_K, Q5_K; int8 sub-block scales for Q6_K). The device
 * side of the block codec; the reference declares Backend::quantize
 * (include/hesa/backend.hpp:60) and leaves it unimplemented on the CPU
 * (src/backend/cpu_backend.cpp:296-302). src and dst are device pointers. */
HESA_CUDA_API int hesa_cuda_quantize(int qtype, const float* src, int64_t n_rows, int64_t k, int64_t ld_src,
                                     void* dst, void* stream);

/* ---------------------------------------------------------------------
 * Decode-step helpers (single token). Semantics of hesa-llm's CPU kernels,
 * src/backend/cpu_backend.cpp; `pos` arguments are a device int32 scalar
 * (pos_dev, so a captured CUDA graph replays for every token) or, when
 * pos_dev is NULL, the host value pos_host.
 * --------------------------------------------------------------------- */

/* y = scale * A @ x for row-major F32 A [n_out, k]: hesa::cpu_matmul_f32
 * (src/backend/cpu_backend.cpp:24-41) for F32 weights, as
 * Backend::matmul (include/hesa/backend.hpp:43-44) uses it. */
HESA_CUDA_API int hesa_cuda_matmul_f32(const float* a, int64_t n_out, int64_t k, const float* x, int64_t ldx,
                                       int64_t batch, float* y, int64_t ldy, float scale, void* stream);

/* out = in * (1/sqrt(mean(in^2) + eps)) * weight per row of n:
 * cpu_rms_norm_f32 (src/backend/cpu_backend.cpp:72-89), Backend::rms_norm
 * (include/hesa/backend.hpp:48-49). */
HESA_CUDA_API int hesa_cuda_rms_norm(const float* in, const float* weight, float* out, int64_t n_rows,
                                     int64_t n, float eps, void* stream);

/* out = silu(gate) * up, or silu(gate) when up is NULL: cpu_silu_f32
 * (src/backend/cpu_backend.cpp:91-96), Backend::silu (backend.hpp:52). */
HESA_CUDA_API int hesa_cuda_silu_mul(const float* gate, const float* up, float* out, int64_t n, void* stream);

/* out = a + b, out = a * b: cpu_add_f32 (cpu_backend.cpp:43-46) and
 * CPU_Backend::mul (cpu_backend.cpp:170-177); Backend::add/mul
 * (backend.hpp:45-46). */
HESA_CUDA_API int hesa_cuda_add(const float* a, const float* b, float* out, int64_t n, void* stream);
HESA_CUDA_API int hesa_cuda_mul(const float* a, const float* b, float* out, int64_t n, void* stream);

/* Row softmax over the last dimension: cpu_softmax_f32
 * (cpu_backend.cpp:48-70), Backend::softmax (backend.hpp:47). */
HESA_CUDA_API int hesa_cuda_softmax(const float* in, float* out, int64_t n_rows, int64_t n, void* stream);

/* HOST function: the rotate-half angle table of cpu_rope_f32
 * (cpu_backend.cpp:103-112), row p = [cos(theta_p,d) for d < head_dim/2,
 * sin(theta_p,d) for d < head_dim/2] with theta = p / base^(2d/head_dim),
 * for p in [0, n_pos). table_host holds n_pos * head_dim floats. */
HESA_CUDA_API int hesa_cuda_rope_table(float* table_host, int32_t n_pos, int64_t head_dim, float freq_base);

/* In-place rotate-half RoPE of data [n_heads, head_dim] at position pos,
 * from a device copy of hesa_cuda_rope_table with table_rows rows
 * (cpu_rope_f32, cpu_backend.cpp:98-120; Backend::rope, backend.hpp:50-51).
 * The position is *pos_dev when pos_dev is not NULL (read on the device, so a
 * captured graph serves every token), else pos_host. A device position
 * outside [0, table_rows) leaves data unchanged and sets device status 3. */
HESA_CUDA_API int hesa_cuda_rope(float* data, int64_t n_heads, int64_t head_dim, const float* table,
                                 int32_t table_rows, const int32_t* pos_dev, int32_t pos_host, void* stream);

/* Ring-buffer KV cache write: k_cache/v_cache [ctx, row_elems] fp16, slot
 * pos % ctx <- fp16(k), fp16(v) (round to nearest even). The KV cache of
 * the reference's design (docs/architecture.md:287-338). A negative device
 * position writes nothing and sets device status 3. */
HESA_CUDA_API int hesa_cuda_kv_store(const float* k, const float* v, void* k_cache, void* v_cache,
                                     int64_t row_elems, int64_t ctx, const int32_t* pos_dev, int32_t pos_host,
                                     void* stream);

/* Workspace bytes of hesa_cuda_attention (zero-filled once; left zeroed). */
HESA_CUDA_API size_t hesa_cuda_attention_workspace_size(int64_t n_head, int64_t head_dim, int64_t ctx);

/* Single-query attention over min(pos+1, ctx) slots of the fp16 ring:
 * out[h] = softmax(q[h] . K / sqrt(head_dim)) V with kv head
 * h / (n_head / n_kv_head). q, out: [n_head, head_dim] fp32; head_dim 64,
 * 128 or 256; caches 16-byte aligned, ctx <= 131072 slots. The SDPA of CPU_Backend (cpu_backend.cpp:225-294) extended to
 * GQA and the fp16 cache; Backend::scaled_dot_product_attention
 * (backend.hpp:55-57). */
HESA_CUDA_API int hesa_cuda_attention(const float* q, const void* k_cache, const void* v_cache, float* out,
                                      int64_t n_head, int64_t n_kv_head, int64_t head_dim, int64_t ctx,
                                      const int32_t* pos_dev, int32_t pos_host, void* workspace,
                                      size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------
 * Decode step of a Llama-style decoder (the reference's layer loop over
 * Backend ops: src/model, docs/architecture.md:287-338) on device tensors.
 * ------------------------------------------------------------------- */

typedef struct {
    int32_t n_layer, d_model, n_head, n_kv_head, head_dim, d_ff, vocab;
    int32_t ctx;        /* KV ring capacity (slots) */
    float   rms_eps;    /* RMSNorm epsilon (Backend::rms_norm default 1e-6) */
    float   rope_base;  /* unused by the step itself: the rope table carries it */
    int32_t qtype;      /* type of every projection and the LM head */
} hesa_cuda_model;

/* Device pointers of one layer. Weights are packed GGUF rows [n_out, k];
 * caches fp16 [ctx, n_kv_head * head_dim]. When wk starts right after the
 * rows of wq and wv right after wk (and w_up right after w_gate), the step
 * runs each group as one matvec. */
typedef struct {
    const void* wq;      /* [n_head * head_dim, d_model] */
    const void* wk;      /* [n_kv_head * head_dim, d_model] */
    const void* wv;
    const void* wo;      /* [d_model, n_head * head_dim] */
    const void* w_gate;  /* [d_ff, d_model] */
    const void* w_up;
    const void* w_down;  /* [d_model, d_ff] */
    const float* attn_norm;  /* [d_model] */
    const float* ffn_norm;
    void* k_cache;
    void* v_cache;
} hesa_cuda_layer;

/* Bytes of the decode step's workspace (intermediate vectors, attention and
 * matvec scratch); zero-fill it once, every step leaves it reusable. */
HESA_CUDA_API size_t hesa_cuda_decode_workspace_size(const hesa_cuda_model* model);

/* x <- row *token_dev of the quantized embedding table [vocab, d_model],
 * dequantized exactly. A token outside [0, vocab) leaves x unchanged and sets
 * device status 3. */
HESA_CUDA_API int hesa_cuda_embed(int qtype, const void* w_emb, int64_t vocab, int64_t d_model,
                                  const int32_t* token_dev, float* x, void* stream);

/* One token: logits [vocab] <- the decoder applied to the embedding x_embed
 * [d_model] at position *pos_dev, writing K and V of every layer into slot
 * pos % ctx of its caches and attending over min(pos + 1, ctx) slots.
 *   layers: HOST array of n_layer structs (device pointers inside);
 *   out_norm [d_model], w_out [vocab, d_model] packed rows;
 *   rope_table: device copy of hesa_cuda_rope_table with rope_rows rows.
 * Everything is enqueued on `stream` (capturable in a CUDA graph: the
 * position and token are read on the device). */
HESA_CUDA_API int hesa_cuda_decode_step(const hesa_cuda_model* model, const hesa_cuda_layer* layers,
                                        const float* out_norm, const void* w_out, const float* rope_table,
                                        int32_t rope_rows, const float* x_embed, const int32_t* pos_dev,
                                        float* logits, void* workspace, size_t workspace_bytes, void* stream);

/* ---- one sequence decoded on several GPUs (head-sharded decode step) ----
 * Rank r of `world` holds, per layer, the Q, K, V rows of its heads
 * [r*n_head/world, (r+1)*n_head/world) and kv heads likewise (joined: wk right
 * after wq's rows, wv after wk's), the KV caches of its kv heads
 * [ctx, n_kv_head/world * head_dim], its balanced row share of gate|up
 * (joined: its up rows right after its gate rows) and of the LM head (rows
 * [floor(r*n/world), floor((r+1)*n/world)) of each), and ALL of Wo and
 * W_down. Every rank keeps the residual vector itself. Per layer the
 * attention output and gate|up are gathered: the kernel that produces each
 * stores its part straight into every rank's buffer over NVLink, every value
 * as one 64-bit word with a tag naming the token and the place in the step,
 * and the kernel that consumes it reads each word once its tag is the
 * expected one (bounded wait: device status 4 when a peer does not deliver in
 * time) -- no fence, flag array or barrier launch per exchange. Wo and W_down
 * run whole on every rank: two exchanges per layer instead of four. The
 * buffers are peer allocations (hesa_cuda_peer_alloc / _open) of 8 bytes per
 * element, each vector rounded up to whole units of 256 elements and stored
 * in the interleaved word order of hesa_cuda_qmatvec_gather_tagged (16-byte
 * aligned); arrays are host arrays of `world` device pointers, entry p =
 * rank p's buffer as mapped in this process. The decomposition of the
 * reference's decode loop (docs/architecture.md:277-281) over the GPUs of one
 * node; no counterpart in the reference, which runs on one device. */
typedef struct {
    int32_t rank, world;
    uint64_t* const* a_peers;       /* [n_head * head_dim] attention outputs */
    uint64_t* const* gu_peers;      /* [2 * d_ff] gate | up (up at element d_ff) */
    uint64_t* const* logits_peers;  /* [vocab] */
    uint32_t* token_count;          /* this rank's token counter (device uint32, zero-initialised) */
} hesa_cuda_shard;

/* One token of the decoder on this rank: `layers` hold this rank's shards
 * (wo and w_down the whole matrices), w_out its LM-head rows; x_embed the
 * token's embedding (the same on every rank); logits [vocab] (this rank's
 * device memory) receives all the logits, bit-identical to
 * hesa_cuda_decode_step's.
 * Every rank must issue the same steps; the workspace is
 * hesa_cuda_decode_workspace_size(model) bytes (model = the full, unsharded
 * shape). n_head and n_kv_head must be multiples of world, n_layer < 512; the
 * shards must fit the row-strip kernel (k <= 24576; d_model <= 12288). Each
 * word a peer delivers is waited for at most the peer wait limit
 * (hesa_cuda_set_peer_wait_limit_us, read when the step is enqueued). */
HESA_CUDA_API int hesa_cuda_decode_step_sharded(const hesa_cuda_model* model, const hesa_cuda_shard* shard,
                                                const hesa_cuda_layer* layers, const float* out_norm,
                                                const void* w_out, const float* rope_table, int32_t rope_rows,
                                                const float* x_embed, const int32_t* pos_dev, float* logits,
                                                void* workspace, size_t workspace_bytes, void* stream);

/* Sticky device-side status of the kernels: 0 while nothing has gone wrong
 * in this process, else the first code recorded: 1 a bulk copy did not land
 * within the bounded wait, 2 a copy was still in flight when the kernel
 * gave up, 3 a device-side position outside the KV cache or the rope table,
 * 4 a peer rank did not reach hesa_cuda_peer_barrier, or did not deliver a
 * word of the sharded decode step, in time.
 * Reading synchronizes `stream`. hesa_cuda_clear_device_status resets it. */
HESA_CUDA_API int hesa_cuda_device_status(void* stream, int* status_out);

/* ---- row-sharded matvec with the output all-gather fused in ----
 * The rows of W are split over the GPUs of one node (rank r holds rows
 * [r0, r1)); every rank needs all of y. Replaces the NCCL all-gather that
 * follows a sharded CPU_Backend::matmul-equivalent call
 * (src/backend/cpu_backend.cpp:24-41 computes the unsharded product): each
 * rank's kernel stores its rows straight into the gathered buffer of every
 * rank over NVLink, and one barrier per step publishes completion. No
 * counterpart in the reference, which runs on one device.
 *
 * hesa_cuda_peer_alloc: the one entry point that allocates. cudaMalloc of
 * `bytes` (zero-filled) on the current device; *handle_out (host, 64 bytes)
 * receives its CUDA IPC handle for the other ranks. Free with
 * hesa_cuda_peer_free after every peer has closed it.
 * hesa_cuda_peer_open / hesa_cuda_peer_close: map / unmap another rank's
 * allocation from its 64-byte handle (not one from this process). */
HESA_CUDA_API int hesa_cuda_peer_alloc(size_t bytes, void** dev_ptr_out, void* handle_out);
HESA_CUDA_API int hesa_cuda_peer_free(void* dev_ptr);
HESA_CUDA_API int hesa_cuda_peer_open(const void* handle, void** dev_ptr_out);
HESA_CUDA_API int hesa_cuda_peer_close(void* dev_ptr);

/* y_shard = scale * W_shard . x for this rank's n_rows rows of W (batch 1;
 * k a multiple of 256, k <= 24576; W, x 16-byte aligned), stored into all
 * `world` ranks at once: row i goes to y_peers[b * world + p][i] for every p,
 * where y_peers (host array of 2 * world device pointers, as mapped in this
 * process) points at this shard's first row inside rank p's gathered buffer
 * for parity b, and b = *epoch & 1 (epoch: this rank's barrier count, device,
 * written by hesa_cuda_peer_barrier). Two parities let a rank store step s + 1
 * while a peer still reads step s; a gathered result stays valid until the
 * barrier of the step after next. */
HESA_CUDA_API int hesa_cuda_qmatvec_gather(int qtype, const void* w, int64_t n_rows, int64_t k, const float* x,
                                           float scale, float* const* y_peers, int world, const uint32_t* epoch,
                                           void* stream);

/* The same gathered matvec with every row sent as a tagged 64-bit word
 * (value bits | tag << 32, tag = sync[0] << 12 | 1): row i of the shard is
 * element row0 + i of the gathered vector, stored into y_peers[b * world + p]
 * (host array of 2 * world device pointers: word 0 of rank p's gathered
 * buffer for parity b, as mapped in this process, 16-byte aligned) for every
 * rank p, b = sync[0] & 1, where sync (device uint32[2], zero-initialised,
 * 8-byte aligned) is this rank's step count and collector ticket. Element g
 * is word ((g & ~255) | ((g >> 1) & 3) << 6 | ((g >> 3) & 31) << 1 | (g & 1))
 * of a buffer: inside each 256-element unit the words are interleaved so
 * that the strip kernel's lanes read them with coalesced loads; buffers hold
 * whole units. Ends with hesa_cuda_peer_collect instead of a barrier: no
 * fence, no flags, and the launch chain stays programmatic. Shapes the
 * row-strip kernel takes (k <= 24576) need no workspace (null, 0); longer
 * rows run the plain matvec into `workspace` (16-byte aligned, at least
 * hesa_cuda_gather_tagged_workspace_size bytes) and one more kernel sends
 * its rows. */
HESA_CUDA_API size_t hesa_cuda_gather_tagged_workspace_size(int qtype, int64_t n_rows, int64_t k);
HESA_CUDA_API int hesa_cuda_qmatvec_gather_tagged(int qtype, const void* w, int64_t n_rows, int64_t k,
                                                  const float* x, float scale, uint64_t* const* y_peers,
                                                  int64_t row0, int world, const uint32_t* sync, void* workspace,
                                                  size_t workspace_bytes, void* stream);

/* End of a step of tagged gathered matvecs on this rank: waits until each of
 * the n elements of this rank's buffer for the step's parity (word 0 at
 * `words` while sync[0] is even, at words + parity_stride while odd;
 * parity_stride a multiple of 256, at least n rounded up to 256) carries the
 * step's tag (each wait bounded by the peer wait limit, device status 4 on
 * expiry), writes their values to out[0..n), then advances sync[0]. A
 * gathered result in `out` stays valid until the next collect; the words of
 * a parity may be overwritten from the step after next on. */
HESA_CUDA_API int hesa_cuda_peer_collect(const uint64_t* words, int64_t n, int64_t parity_stride, float* out,
                                         uint32_t* sync, void* stream);

/* End of a step of gathered matvecs (enqueue it on the stream of those
 * matvecs: it starts after their grids have completed, which is what makes
 * their peer stores visible; it then fences at system scope): publishes
 * *epoch + 1 into slot `rank`
 * of every rank's flag array (flags: host array of `world` device pointers to
 * uint32[world], flags[p] = rank p's array as mapped here, flags[rank] this
 * rank's own), waits until every slot of this rank's array holds it, then
 * stores it into *epoch. Every rank must issue the same sequence of steps;
 * the wait is bounded (2 s, device status 4 on expiry), so the ranks must
 * reach it within that time of one another. */
HESA_CUDA_API int hesa_cuda_peer_barrier(uint32_t* const* flags, int rank, int world, uint32_t* epoch,
                                         void* stream);

/* How long each wait for a peer rank lasts (hesa_cuda_peer_barrier) before it
 * gives up, records device status 4 and returns, in microseconds; 0 restores
 * the default of 2 s, values above 60 s are refused. Applies to barriers and
 * sharded decode steps enqueued after the call (a CUDA graph keeps the limit it was captured
 * with). The host-side counterpart of a collective timeout: a rank that
 * dies between steps costs its peers at most this long per barrier, and the
 * status word tells them why. No counterpart in the reference (one device). */
HESA_CUDA_API int hesa_cuda_set_peer_wait_limit_us(uint32_t limit_us);
HESA_CUDA_API int hesa_cuda_clear_device_status(void* stream);

/* Last error message recorded on this host thread ("" if none). */
HESA_CUDA_API const char* hesa_cuda_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
