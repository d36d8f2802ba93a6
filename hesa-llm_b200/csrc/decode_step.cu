// decode_step.cu -- one token through a Llama-style decoder on device tensors:
// the layer loop of the reference's model (attention block, SwiGLU FFN,
// residual adds, final norm, LM head) issued as this library's kernels on one
// stream. Host code, plus the embedding-row lookup kernel.
//
// Per layer (the order the oracle's decode step restates):
//   h = rms_norm(x) ; [q|k|v] = Wqkv h ; rope(q), rope(k) ; KV[pos % ctx] = k, v
//   a = attention(q, KV[0 .. min(pos+1, ctx))) ; x += Wo a
//   h = rms_norm(x) ; [g|u] = Wgu h ; g = silu(g) * u ; x += Wdown g
// then logits = Wout rms_norm(x).
//
// Q, K and V (and gate and up) run as ONE matvec when their packed rows lie
// back to back in device memory (the upload can arrange that): the activation
// is staged once and the outputs come out as one vector. Where the row-strip
// kernel takes the shape, the norms and SwiGLU are applied while it stages its
// input and the residual adds happen in its epilogue, and rope and the KV
// write are one kernel: six launches per layer.
// The position (and the token of hesa_cuda_embed) is read from device memory
// by every kernel that needs it, so a CUDA graph captured once replays for
// every token.
#include "../../include/hesa_cuda.h"
#include "abi_errors.h"
#include "trace.h"
#include "decode_ops.h"
#include "hesa_common.cuh"
#include "qmatvec.h"
#include "qtypes.cuh"
#include "peer_sync.cuh"

#include <algorithm>
#include <cstdint>

namespace hesa_cuda {
namespace {

template <int QT>
__global__ void embed_kernel(const uint8_t* __restrict__ w, int vocab, int d_model, const int32_t* __restrict__ tok,
                             float* __restrict__ x, int* __restrict__ status) {
    constexpr int BE = block_elems(QT), BB = block_bytes(QT);
    const int t = *tok;
    if (t < 0 || t >= vocab) {   // no such row: leave x as is
        if (blockIdx.x == 0 && threadIdx.x == 0) record_status(status, kStatusBadPosition);
        return;
    }
    const uint8_t* row = w + static_cast<int64_t>(t) * (d_model / BE) * BB;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < d_model; i += gridDim.x * blockDim.x)
        x[i] = deq_weight<QT>(row + (i / BE) * BB, i % BE);
}

template <int QT>
cudaError_t launch_embed(const void* w, int vocab, int d, const int32_t* tok, float* x, int* status,
                         cudaStream_t s) {
    embed_kernel<QT><<<(d + 255) / 256, 256, 0, s>>>(static_cast<const uint8_t*>(w), vocab, d, tok, x, status);
    return cudaGetLastError();
}

size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

// Byte offsets of the step's buffers inside the caller's workspace.
struct Layout {
    size_t x, h, qkv, a, o, gu, att, att_bytes, qmv, qmv_bytes, total;
};

Layout layout(const hesa_cuda_model* m) {
    const size_t D = m->d_model, QD = static_cast<size_t>(m->n_head) * m->head_dim,
                 KD = static_cast<size_t>(m->n_kv_head) * m->head_dim, F = m->d_ff;
    Layout L{};
    size_t off = 0;
    L.x = off;   off += align256(D * 4);
    L.h = off;   off += align256(D * 4);
    L.qkv = off; off += align256((QD + 2 * KD) * 4);
    L.a = off;   off += align256(QD * 4);
    L.o = off;   off += align256(D * 4);
    L.gu = off;  off += align256(2 * F * 4);
    L.att_bytes = hesa_cuda_attention_workspace_size(m->n_head, m->head_dim, m->ctx);
    L.att = off; off += align256(L.att_bytes);
    const int64_t shapes[5][2] = {{static_cast<int64_t>(QD + 2 * KD), static_cast<int64_t>(D)},
                                  {static_cast<int64_t>(D), static_cast<int64_t>(QD)},
                                  {static_cast<int64_t>(2 * F), static_cast<int64_t>(D)},
                                  {static_cast<int64_t>(D), static_cast<int64_t>(F)},
                                  {static_cast<int64_t>(m->vocab), static_cast<int64_t>(D)}};
    L.qmv_bytes = 0;
    for (const auto& sh : shapes) {
        const size_t b = hesa_cuda_qmatvec_workspace_size(m->qtype, sh[0], sh[1], 1);
        if (b > L.qmv_bytes) L.qmv_bytes = b;
    }
    L.qmv = off; off += align256(L.qmv_bytes);
    L.total = off;
    return L;
}

bool model_ok(const hesa_cuda_model* m) {
    return m && m->n_layer > 0 && m->d_model > 0 && m->n_head > 0 && m->n_kv_head > 0 &&
           m->n_head % m->n_kv_head == 0 && m->head_dim > 0 && m->d_ff > 0 && m->vocab > 0 && m->ctx > 0 &&
           qtype_supported(m->qtype);
}

}  // namespace
}  // namespace hesa_cuda

using hesa_cuda::Layout;

extern "C" {

size_t hesa_cuda_decode_workspace_size(const hesa_cuda_model* m) {
    if (!hesa_cuda::model_ok(m)) return 0;
    return hesa_cuda::layout(m).total;
}

int hesa_cuda_embed(int qtype, const void* w_emb, int64_t vocab, int64_t d_model, const int32_t* token_dev,
                    float* x, void* stream) {
    HESA_TRACE("hesa_cuda_embed");
    using namespace hesa_cuda;
    if (!qtype_supported(qtype)) return record_error(HESA_CUDA_BACKEND_NOT_AVAILABLE, "unsupported qtype");
    if (!w_emb || !token_dev || !x) return record_error(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (vocab <= 0 || d_model <= 0 || d_model % block_elems(qtype) != 0 || vocab >= (int64_t(1) << 31) ||
        d_model >= (int64_t(1) << 31))
        return record_error(HESA_CUDA_SHAPE_MISMATCH, "bad shape");
    int* status = nullptr;
    cudaError_t e = status_word(&status);
    if (e == cudaSuccess) {
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        const int v = static_cast<int>(vocab), d = static_cast<int>(d_model);
        switch (qtype) {
            case kQ4_0: e = launch_embed<kQ4_0>(w_emb, v, d, token_dev, x, status, s); break;
            case kQ8_0: e = launch_embed<kQ8_0>(w_emb, v, d, token_dev, x, status, s); break;
            case kQ4_K: e = launch_embed<kQ4_K>(w_emb, v, d, token_dev, x, status, s); break;
            case kQ5_K: e = launch_embed<kQ5_K>(w_emb, v, d, token_dev, x, status, s); break;
            default:    e = launch_embed<kQ6_K>(w_emb, v, d, token_dev, x, status, s); break;
        }
    }
    return e == cudaSuccess ? HESA_CUDA_OK : record_cuda_error(e, "embed kernel");
}

int hesa_cuda_decode_step(const hesa_cuda_model* m, const hesa_cuda_layer* layers, const float* out_norm,
                          const void* w_out, const float* rope_table, int32_t rope_rows, const float* x_embed,
                          const int32_t* pos_dev, float* logits, void* workspace, size_t workspace_bytes,
                          void* stream) {
    HESA_TRACE("hesa_cuda_decode_step");
    using hesa_cuda::record_error;
    if (!hesa_cuda::model_ok(m)) return record_error(HESA_CUDA_SHAPE_MISMATCH, "bad model shape");
    if (!layers || !out_norm || !w_out || !rope_table || !x_embed || !pos_dev || !logits || !workspace)
        return record_error(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (rope_rows <= 0) return record_error(HESA_CUDA_SHAPE_MISMATCH, "empty rope table");
    const Layout L = hesa_cuda::layout(m);
    if (workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return record_error(HESA_CUDA_INVALID_ARGUMENT, "workspace too small or not 256-byte aligned");

    const int qt = m->qtype;
    const int64_t D = m->d_model, HD = m->head_dim, NH = m->n_head, NKV = m->n_kv_head;
    const int64_t QD = NH * HD, KD = NKV * HD, F = m->d_ff;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    float* x = reinterpret_cast<float*>(ws + L.x);
    float* h = reinterpret_cast<float*>(ws + L.h);
    float* q = reinterpret_cast<float*>(ws + L.qkv);
    float* k = q + QD;
    float* v = k + KD;
    float* a = reinterpret_cast<float*>(ws + L.a);
    float* o = reinterpret_cast<float*>(ws + L.o);
    float* g = reinterpret_cast<float*>(ws + L.gu);
    float* u = g + F;
    void* att_ws = ws + L.att;
    void* qmv_ws = ws + L.qmv;
    const size_t rb_d = hesa_cuda_row_bytes(qt, D), rb_qd = hesa_cuda_row_bytes(qt, QD),
                 rb_f = hesa_cuda_row_bytes(qt, F);
    if (!rb_d || !rb_qd || !rb_f)
        return record_error(HESA_CUDA_SHAPE_MISMATCH, "d_model, n_head*head_dim and d_ff must be block multiples");

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    auto mv = [&](const void* w, int64_t n_out, int64_t kk, const float* xin, float* yout) {
        return hesa_cuda_qmatvec(qt, w, n_out, kk, xin, kk, 1, yout, n_out, 1.0f, qmv_ws, L.qmv_bytes, stream);
    };
    using hesa_cuda::StripInput;
    auto fusable = [&](const void* w, int64_t n_out, int64_t kk, StripInput in) {
        return hesa_cuda::qmv_strip_fused_eligible(qt, w, n_out, kk, in);
    };
    auto fmv = [&](const void* w, int64_t n_out, int64_t kk, const float* xin, StripInput in, const float* nw,
                   float* yout, const float* resid) {
        const cudaError_t e = hesa_cuda::qmv_strip_fused(qt, w, n_out, kk, xin, in, nw, m->rms_eps, yout, resid,
                                                         1.0f, s);
        return e == cudaSuccess ? HESA_CUDA_OK : hesa_cuda::record_cuda_error(e, "fused matvec");
    };
    const cudaError_t ce = cudaMemcpyAsync(x, x_embed, D * 4, cudaMemcpyDeviceToDevice, s);
    int rc = ce == cudaSuccess ? HESA_CUDA_OK : hesa_cuda::record_cuda_error(ce, "copy of the embedding");
    for (int l = 0; l < m->n_layer && rc == HESA_CUDA_OK; ++l) {
        const hesa_cuda_layer& Ly = layers[l];
        if (!Ly.wq || !Ly.wk || !Ly.wv || !Ly.wo || !Ly.w_gate || !Ly.w_up || !Ly.w_down || !Ly.attn_norm ||
            !Ly.ffn_norm || !Ly.k_cache || !Ly.v_cache)
            return record_error(HESA_CUDA_INVALID_ARGUMENT, "null pointer in a layer");
        const uint8_t* wq = static_cast<const uint8_t*>(Ly.wq);
        const bool qkv_joined = Ly.wk == wq + QD * rb_d && Ly.wv == wq + (QD + KD) * rb_d;
        const bool gu_joined = Ly.w_up == static_cast<const uint8_t*>(Ly.w_gate) + F * rb_d;

        // attention block: q|k|v = W (norm x) ; rope + KV write ; x += Wo attention(q)
        if (qkv_joined && fusable(Ly.wq, QD + 2 * KD, D, StripInput::kRmsNorm)) {
            if (!rc) rc = fmv(Ly.wq, QD + 2 * KD, D, x, StripInput::kRmsNorm, Ly.attn_norm, q, nullptr);
        } else {
            if (!rc) rc = hesa_cuda_rms_norm(x, Ly.attn_norm, h, 1, D, m->rms_eps, stream);
            if (qkv_joined) {
                if (!rc) rc = mv(Ly.wq, QD + 2 * KD, D, h, q);
            } else {
                if (!rc) rc = mv(Ly.wq, QD, D, h, q);
                if (!rc) rc = mv(Ly.wk, KD, D, h, k);
                if (!rc) rc = mv(Ly.wv, KD, D, h, v);
            }
        }
        const bool att_fused = (reinterpret_cast<uintptr_t>(Ly.k_cache) & 15) == 0 &&
                               (reinterpret_cast<uintptr_t>(Ly.v_cache) & 15) == 0 &&
                               (HD == 64 || HD == 128 || HD == 256) && m->ctx <= 131072 &&
                               L.att_bytes >= hesa_cuda::attention_workspace_bytes(NH, HD, m->ctx);
        if (att_fused) {
            // rope, KV write and attention in one launch
            if (!rc) {
                const cudaError_t e = hesa_cuda::attention_rope(q, k, v, Ly.k_cache, Ly.v_cache, a, NH, NKV, HD,
                                                                rope_table, rope_rows, m->ctx, pos_dev, att_ws, s);
                if (e != cudaSuccess) rc = hesa_cuda::record_cuda_error(e, "attention with rope + KV write");
            }
        } else {
            if (!rc) {
                const cudaError_t e = hesa_cuda::rope_kv(q, k, v, Ly.k_cache, Ly.v_cache, NH, NKV, HD, rope_table,
                                                         rope_rows, m->ctx, pos_dev, s);
                if (e != cudaSuccess) rc = hesa_cuda::record_cuda_error(e, "rope + KV write");
            }
            if (!rc) rc = hesa_cuda_attention(q, Ly.k_cache, Ly.v_cache, a, NH, NKV, HD, m->ctx, pos_dev, 0, att_ws,
                                              L.att_bytes, stream);
        }
        if (fusable(Ly.wo, D, QD, StripInput::kPlain)) {
            if (!rc) rc = fmv(Ly.wo, D, QD, a, StripInput::kPlain, nullptr, x, x);
        } else {
            if (!rc) rc = mv(Ly.wo, D, QD, a, o);
            if (!rc) rc = hesa_cuda_add(x, o, x, D, stream);
        }
        // FFN block: g|u = W (norm x) ; x += Wdown (silu(g) * u)
        if (gu_joined && fusable(Ly.w_gate, 2 * F, D, StripInput::kRmsNorm)) {
            if (!rc) rc = fmv(Ly.w_gate, 2 * F, D, x, StripInput::kRmsNorm, Ly.ffn_norm, g, nullptr);
        } else {
            if (!rc) rc = hesa_cuda_rms_norm(x, Ly.ffn_norm, h, 1, D, m->rms_eps, stream);
            if (gu_joined) {
                if (!rc) rc = mv(Ly.w_gate, 2 * F, D, h, g);
            } else {
                if (!rc) rc = mv(Ly.w_gate, F, D, h, g);
                if (!rc) rc = mv(Ly.w_up, F, D, h, u);
            }
        }
        if (fusable(Ly.w_down, D, F, StripInput::kSiluMul)) {
            if (!rc) rc = fmv(Ly.w_down, D, F, g, StripInput::kSiluMul, nullptr, x, x);   // g|u contiguous
        } else {
            if (!rc) rc = hesa_cuda_silu_mul(g, u, g, F, stream);
            if (!rc) rc = mv(Ly.w_down, D, F, g, o);
            if (!rc) rc = hesa_cuda_add(x, o, x, D, stream);
        }
    }
    if (fusable(w_out, m->vocab, D, StripInput::kRmsNorm)) {
        if (!rc) rc = fmv(w_out, m->vocab, D, x, StripInput::kRmsNorm, out_norm, logits, nullptr);
    } else {
        if (!rc) rc = hesa_cuda_rms_norm(x, out_norm, h, 1, D, m->rms_eps, stream);
        if (!rc) rc = mv(w_out, m->vocab, D, h, logits);
    }
    return rc;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// head-sharded decode step
// ---------------------------------------------------------------------------
//
// Rank r of W holds the Q, K, V rows of its heads (and their KV caches), its
// row shares of gate|up and of the LM head, and all of Wo and W_down; the
// residual x stays local and plain on every rank. Per layer two vectors are
// exchanged, as tagged words (peer_sync.cuh): the attention output (each rank
// its heads) and gate|up (each rank its rows). Every rank then computes all
// rows of Wo and W_down itself -- 35 MB of the 113 MB of a 7B Q4_K layer --
// instead of exchanging the residual twice more: at batch 1 a launch's fixed
// cost (grid wait, staging of x, epilogue, the wait for the slowest rank)
// is worth more than those bytes (measured, 7B: the four-exchange form took
// 1.84 and 2.04 ms per token on 2 and 4 GPUs against 1.74 on one). Every
// output row is summed as in the unsharded step, so the logits are its
// logits bit for bit.

namespace hesa_cuda {
namespace {

// Tag low bits of the step's exchanges: (layer << 3) | phase (never 0).
enum : uint32_t { kPhAttn = 1, kPhGateUp = 3, kPhLogits = 5 };
constexpr uint32_t lo_of(int64_t layer, uint32_t phase) { return (static_cast<uint32_t>(layer) << 3) | phase; }

// The token's embedding into the plain residual; opens the token (one CTA:
// every thread reads the old count, then it is advanced).
__global__ void __launch_bounds__(1024) shard_begin_kernel(const float* __restrict__ x_embed, float* __restrict__ x,
                                                           int n, uint32_t* count) {
    const uint32_t c = *reinterpret_cast<volatile uint32_t*>(count) + 1u;
    for (int i = threadIdx.x; i < n; i += blockDim.x) x[i] = x_embed[i];
    __syncthreads();
    if (threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(count) = c;
}

// This rank's tagged logits into the caller's plain buffer.
__global__ void ll_unpack_kernel(const uint64_t* ll, float* __restrict__ out, int n, const uint32_t* count,
                                 uint32_t lo, unsigned long long limit_ns, int* status) {
    const uint32_t tag = ll_tag(count, lo);
    __shared__ int failed;
    if (threadIdx.x == 0) failed = 0;
    __syncthreads();
    // words in order (coalesced), each to its element (the tail of the last
    // unit holds none)
    const int n_words = (n + 255) & ~255;
    for (int w = blockIdx.x * blockDim.x + threadIdx.x; w < n_words; w += gridDim.x * blockDim.x) {
        const int e = static_cast<int>(ll_elem(w));
        if (e < n) out[e] = ld_ll_wait(ll + w, tag, limit_ns, status, &failed);
    }
}

}  // namespace
}  // namespace hesa_cuda

extern "C" int hesa_cuda_decode_step_sharded(const hesa_cuda_model* m, const hesa_cuda_shard* sh,
                                             const hesa_cuda_layer* layers, const float* out_norm, const void* w_out,
                                             const float* rope_table, int32_t rope_rows, const float* x_embed,
                                             const int32_t* pos_dev, float* logits, void* workspace,
                                             size_t workspace_bytes, void* stream) {
    HESA_TRACE("hesa_cuda_decode_step_sharded");
    using namespace hesa_cuda;
    if (!model_ok(m)) return record_error(HESA_CUDA_SHAPE_MISMATCH, "bad model shape");
    if (!sh || !layers || !out_norm || !w_out || !rope_table || !x_embed || !pos_dev || !logits || !workspace)
        return record_error(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    const int W = sh->world, r = sh->rank;
    if (W < 1 || W > kPeerSyncMax || r < 0 || r >= W) return record_error(HESA_CUDA_INVALID_ARGUMENT, "bad rank / world");
    if (!sh->a_peers || !sh->gu_peers || !sh->logits_peers || !sh->token_count)
        return record_error(HESA_CUDA_INVALID_ARGUMENT, "null shard buffer array");
    for (int p = 0; p < W; ++p) {
        if (!sh->a_peers[p] || !sh->gu_peers[p] || !sh->logits_peers[p])
            return record_error(HESA_CUDA_INVALID_ARGUMENT, "null peer buffer");
        if ((reinterpret_cast<uintptr_t>(sh->a_peers[p]) | reinterpret_cast<uintptr_t>(sh->gu_peers[p]) |
             reinterpret_cast<uintptr_t>(sh->logits_peers[p])) & 15)
            return record_error(HESA_CUDA_INVALID_ARGUMENT, "peer buffers must be 16-byte aligned");
    }
    if (m->n_head % W != 0 || m->n_kv_head % W != 0)
        return record_error(HESA_CUDA_SHAPE_MISMATCH, "n_head and n_kv_head must be multiples of world");
    if (m->n_layer >= 512) return record_error(HESA_CUDA_SHAPE_MISMATCH, "n_layer must be below 512");
    if (rope_rows <= 0) return record_error(HESA_CUDA_SHAPE_MISMATCH, "empty rope table");
    const Layout L = layout(m);
    if (workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return record_error(HESA_CUDA_INVALID_ARGUMENT, "workspace too small or not 256-byte aligned");

    const int qt = m->qtype;
    const int64_t D = m->d_model, HD = m->head_dim, F = m->d_ff, V = m->vocab;
    const int64_t QD = static_cast<int64_t>(m->n_head) * HD;
    const int64_t hl = m->n_head / W, kvl = m->n_kv_head / W;
    const int64_t qd_r = hl * HD, kd_r = kvl * HD;
    auto share = [&](int64_t n, int64_t& a, int64_t& b) {
        a = n * r / W;
        b = n * (r + 1) / W;
    };
    int64_t f0, f1, v0, v1;
    share(F, f0, f1);
    share(V, v0, v1);
    const size_t rb_d = hesa_cuda_row_bytes(qt, D), rb_qd = hesa_cuda_row_bytes(qt, QD),
                 rb_f = hesa_cuda_row_bytes(qt, F);
    if (!rb_d || !rb_qd || !rb_f)
        return record_error(HESA_CUDA_SHAPE_MISMATCH, "d_model, n_head*head_dim and d_ff must be block multiples");
    if (f1 <= f0 || v1 <= v0) return record_error(HESA_CUDA_SHAPE_MISMATCH, "an empty row share");
    using SI = StripInput;
    if (!qmv_strip_fused_eligible(qt, layers[0].wq, qd_r + 2 * kd_r, D, SI::kRmsNorm) ||
        !qmv_strip_fused_eligible(qt, layers[0].wo, D, QD, SI::kPlain) ||
        !qmv_strip_fused_eligible(qt, layers[0].w_gate, 2 * (f1 - f0), D, SI::kRmsNorm) ||
        !qmv_strip_fused_eligible(qt, layers[0].w_down, D, F, SI::kSiluMul) ||
        !qmv_strip_fused_eligible(qt, w_out, v1 - v0, D, SI::kRmsNorm))
        return record_error(HESA_CUDA_SHAPE_MISMATCH, "a shard does not fit the row-strip kernel");
    if ((HD != 64 && HD != 128 && HD != 256) || m->ctx > 131072)
        return record_error(HESA_CUDA_SHAPE_MISMATCH, "head_dim must be 64, 128 or 256, ctx <= 131072");
    int* status = nullptr;
    cudaError_t e = status_word(&status);
    if (e != cudaSuccess) return record_cuda_error(e, "status word");

    uint8_t* ws = static_cast<uint8_t*>(workspace);
    float* x = reinterpret_cast<float*>(ws + L.x);
    float* q = reinterpret_cast<float*>(ws + L.qkv);
    float* k = q + qd_r;
    float* v = k + kd_r;
    void* att_ws = ws + L.att;
    const uint32_t* cnt = sh->token_count;
    const unsigned long long limit_ns = peer_wait_limit();
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    // a tagged input vector (by its word 0)
    auto in = [&](const uint64_t* xt, uint32_t lo) {
        LLIn li = {};
        li.x = xt;
        li.count = cnt;
        li.x_lo = lo;
        li.limit_ns = limit_ns;
        return li;
    };
    // this rank's rows are elements off.. of every rank's vector (rows from
    // `split` on: elements off2..)
    auto out = [&](uint64_t* const* bufs, int64_t off, int64_t n_rows, int64_t off2, int64_t split, uint32_t lo) {
        LLOut o = {};
        for (int p = 0; p < W; ++p) o.y[p] = o.y2[p] = bufs[p];
        o.off = off;
        o.off2 = off2;
        o.split = static_cast<int>(split < n_rows ? split : n_rows);
        o.world = W;
        o.count = cnt;
        o.lo = lo;
        return o;
    };
    auto strip = [&](const void* w, int64_t n, int64_t kk, SI mode, const float* nw, const float* xp, float* y,
                     const float* resid, const LLIn& li, const LLOut& lo, const char* what) {
        const cudaError_t ce = qmv_strip_shard(qt, w, n, kk, mode, nw, m->rms_eps, 1.0f, xp, y, resid, li, lo, s);
        return ce == cudaSuccess ? HESA_CUDA_OK : record_cuda_error(ce, what);
    };

    shard_begin_kernel<<<1, 1024, 0, s>>>(x_embed, x, static_cast<int>(D), sh->token_count);
    e = cudaGetLastError();
    if (e != cudaSuccess) return record_cuda_error(e, "token start");
    uint64_t* a_out[kPeerSyncMax] = {};
    for (int p = 0; p < W; ++p) a_out[p] = sh->a_peers[p];
    int rc = HESA_CUDA_OK;
    for (int l = 0; l < m->n_layer && rc == HESA_CUDA_OK; ++l) {
        const hesa_cuda_layer& Ly = layers[l];
        if (!Ly.wq || !Ly.wk || !Ly.wv || !Ly.wo || !Ly.w_gate || !Ly.w_up || !Ly.w_down || !Ly.attn_norm ||
            !Ly.ffn_norm || !Ly.k_cache || !Ly.v_cache)
            return record_error(HESA_CUDA_INVALID_ARGUMENT, "null pointer in a layer");
        const uint8_t* wq = static_cast<const uint8_t*>(Ly.wq);
        if (Ly.wk != wq + qd_r * rb_d || Ly.wv != wq + (qd_r + kd_r) * rb_d ||
            Ly.w_up != static_cast<const uint8_t*>(Ly.w_gate) + (f1 - f0) * rb_d)
            return record_error(HESA_CUDA_INVALID_ARGUMENT, "Q|K|V and gate|up shards must be joined");
        if ((reinterpret_cast<uintptr_t>(Ly.k_cache) & 15) || (reinterpret_cast<uintptr_t>(Ly.v_cache) & 15))
            return record_error(HESA_CUDA_INVALID_ARGUMENT, "KV caches must be 16-byte aligned");
        // q|k|v of this rank's heads (local)
        rc = strip(Ly.wq, qd_r + 2 * kd_r, D, SI::kRmsNorm, Ly.attn_norm, x, q, nullptr, LLIn{}, LLOut{},
                   "sharded q|k|v");
        if (rc) break;
        // attention of this rank's heads -> every rank's a
        e = attention_rope_shard(q, k, v, Ly.k_cache, Ly.v_cache, nullptr, hl, kvl, HD, rope_table, rope_rows, m->ctx,
                                 pos_dev, att_ws, a_out, r * qd_r, W, cnt, lo_of(l, kPhAttn), s);
        if (e != cudaSuccess) return record_cuda_error(e, "sharded attention");
        // x += Wo a, all rows (local)
        rc = strip(Ly.wo, D, QD, SI::kPlain, nullptr, nullptr, x, x, in(sh->a_peers[r], lo_of(l, kPhAttn)), LLOut{},
                   "sharded Wo");
        // gate|up rows of this rank -> every rank's gate|up
        if (!rc)
            rc = strip(Ly.w_gate, 2 * (f1 - f0), D, SI::kRmsNorm, Ly.ffn_norm, x, nullptr, nullptr, LLIn{},
                       out(sh->gu_peers, f0, 2 * (f1 - f0), F + f0, f1 - f0, lo_of(l, kPhGateUp)), "sharded gate|up");
        // x += Wdown silu(g) u, all rows (local)
        if (!rc)
            rc = strip(Ly.w_down, D, F, SI::kSiluMul, nullptr, nullptr, x, x, in(sh->gu_peers[r], lo_of(l, kPhGateUp)),
                       LLOut{}, "sharded W_down");
    }
    const int64_t NL = m->n_layer;
    if (!rc)
        rc = strip(w_out, v1 - v0, D, SI::kRmsNorm, out_norm, x, nullptr, nullptr, LLIn{},
                   out(sh->logits_peers, v0, v1 - v0, 0, v1 - v0, lo_of(NL, kPhLogits)), "sharded LM head");
    if (!rc) {
        const int grid = static_cast<int>(std::min<int64_t>((V + 255) / 256, 148));
        ll_unpack_kernel<<<grid, 256, 0, s>>>(sh->logits_peers[r], logits, static_cast<int>(V), cnt,
                                              lo_of(NL, kPhLogits), limit_ns, status);
        e = cudaGetLastError();
        if (e != cudaSuccess) rc = record_cuda_error(e, "logits unpack");
    }
    return rc;
}
