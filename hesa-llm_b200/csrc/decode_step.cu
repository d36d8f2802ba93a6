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
#include "decode_ops.h"
#include "hesa_common.cuh"
#include "qmatvec.h"
#include "qtypes.cuh"

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
