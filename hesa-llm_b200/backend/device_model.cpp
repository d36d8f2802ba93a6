// device_model.cpp -- see device_model.hpp.
#include "device_model.hpp"

#include "hesa_cuda.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

namespace hesa_gguf {

namespace {

constexpr size_t kAlign = 256;
constexpr size_t kStage = size_t(32) << 20;   // bytes per pinned staging buffer (two of them)

size_t align_up(size_t n) { return (n + kAlign - 1) / kAlign * kAlign; }

bool kernel_qtype(uint32_t t) {
    return t == Q4_0 || t == Q8_0 || t == Q4_K || t == Q5_K || t == Q6_K;
}

// Upload order: the Q, K, V projections of each layer back to back, then its
// gate and up projections, then everything else in file order.
std::vector<size_t> upload_order(const File& f) {
    const auto& ts = f.tensors();
    std::vector<size_t> order;
    std::vector<bool> taken(ts.size(), false);
    auto take = [&](const std::string& name) {
        for (size_t i = 0; i < ts.size(); ++i)
            if (!taken[i] && ts[i].name == name && ts[i].bytes) {
                taken[i] = true;
                order.push_back(i);
                return;
            }
    };
    const int64_t n_layer = f.get_int(f.get_string("general.architecture") + ".block_count", 0);
    for (int64_t l = 0; l < n_layer && l < 100000; ++l) {
        const std::string b = "blk." + std::to_string(l) + ".";
        for (const char* n : {"attn_q", "attn_k", "attn_v", "ffn_gate", "ffn_up"}) take(b + n + ".weight");
    }
    for (size_t i = 0; i < ts.size(); ++i)
        if (!taken[i] && ts[i].bytes) order.push_back(i);
    return order;
}

}  // namespace

DeviceModel::~DeviceModel() { release(); }

void DeviceModel::release() {
    if (base_) {
        cudaSetDevice(device_);
        cudaFree(base_);
    }
    base_ = nullptr;
    bytes_ = 0;
    t_.clear();
    idx_.clear();
}

int DeviceModel::fail(int code, const std::string& what) {
    error_ = what;
    return code;
}

int DeviceModel::upload(const File& f, int device, void* stream) {
    release();
    device_ = device;
    if (cudaSetDevice(device) != cudaSuccess) return fail(9, "cudaSetDevice failed");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const auto order = upload_order(f);
    size_t total = 0;
    for (size_t i : order) total += align_up(f.tensors()[i].bytes);
    if (total == 0) return fail(kInvalidArgument, "no tensors to upload");
    if (cudaMalloc(&base_, total) != cudaSuccess) {
        base_ = nullptr;
        return fail(kOutOfMemory, "cudaMalloc of the model failed");
    }
    bytes_ = total;
    // copy through two pinned staging buffers: while one is on its way to the
    // GPU the host fills the other
    void* stage[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    int rc = kOk;
    for (int b = 0; b < 2 && rc == kOk; ++b) {
        if (cudaMallocHost(&stage[b], kStage) != cudaSuccess ||
            cudaEventCreateWithFlags(&done[b], cudaEventDisableTiming) != cudaSuccess)
            rc = fail(kOutOfMemory, "pinned staging buffers");
    }
    size_t off = 0;
    int cur = 0;
    bool pending[2] = {false, false};
    for (size_t n = 0; n < order.size() && rc == kOk; ++n) {
        const TensorInfo& ti = f.tensors()[order[n]];
        DeviceTensor dt;
        dt.name = ti.name;
        dt.ptr = static_cast<uint8_t*>(base_) + off;
        dt.bytes = ti.bytes;
        dt.type = ti.type;
        dt.rows = ti.rows();
        dt.cols = ti.cols();
        for (uint64_t done_b = 0; done_b < ti.bytes && rc == kOk;) {
            const size_t len = static_cast<size_t>(std::min<uint64_t>(kStage, ti.bytes - done_b));
            if (pending[cur] && cudaEventSynchronize(done[cur]) != cudaSuccess) {
                rc = fail(9, "staging copy failed");
                break;
            }
            std::memcpy(stage[cur], ti.data + done_b, len);
            if (cudaMemcpyAsync(static_cast<uint8_t*>(dt.ptr) + done_b, stage[cur], len, cudaMemcpyHostToDevice, s) !=
                    cudaSuccess ||
                cudaEventRecord(done[cur], s) != cudaSuccess) {
                rc = fail(9, "cudaMemcpyAsync of a tensor failed");
                break;
            }
            pending[cur] = true;
            cur ^= 1;
            done_b += len;
        }
        idx_[dt.name] = t_.size();
        t_.push_back(std::move(dt));
        off += align_up(ti.bytes);
    }
    if (rc == kOk && cudaStreamSynchronize(s) != cudaSuccess) rc = fail(9, "upload did not complete");
    for (int b = 0; b < 2; ++b) {
        if (done[b]) cudaEventDestroy(done[b]);
        if (stage[b]) cudaFreeHost(stage[b]);
    }
    if (rc != kOk) release();
    return rc;
}

const DeviceTensor* DeviceModel::find(const std::string& name) const {
    auto it = idx_.find(name);
    return it == idx_.end() ? nullptr : &t_[it->second];
}

// ---------------------------------------------------------------------------

DecodeSession::~DecodeSession() { release(); }

void DecodeSession::release() {
    for (void* p : {kv_, static_cast<void*>(rope_), static_cast<void*>(x_), static_cast<void*>(logits_), ws_,
                    static_cast<void*>(tok_pos_)})
        if (p) cudaFree(p);
    if (host_tp_) cudaFreeHost(host_tp_);
    kv_ = ws_ = nullptr;
    rope_ = x_ = logits_ = nullptr;
    tok_pos_ = host_tp_ = nullptr;
}

int DecodeSession::fail(int code, const std::string& what) {
    error_ = what;
    return code;
}

int DecodeSession::init(const File& f, const DeviceModel& m, int32_t ctx, void* stream) {
    release();
    stream_ = stream;
    if (f.llama_shape(shape_) != kOk) return fail(kInvalidFormat, "not a Llama-style decoder (metadata)");
    if (ctx <= 0) return fail(kInvalidArgument, "ctx must be positive");
    ctx_ = ctx;
    const LlamaShape& S = shape_;
    const int64_t hd = S.d_model / S.n_head;
    auto need = [&](const std::string& name, int64_t rows, int64_t cols, bool quant) -> const DeviceTensor* {
        const DeviceTensor* t = m.find(name);
        if (!t || t->rows != rows || t->cols != cols) return nullptr;
        if (quant ? !kernel_qtype(t->type) : t->type != F32) return nullptr;
        return t;
    };
    const DeviceTensor* emb = need("token_embd.weight", S.vocab, S.d_model, true);
    const DeviceTensor* out = m.find("output.weight") ? need("output.weight", S.vocab, S.d_model, true) : emb;
    const DeviceTensor* on = need("output_norm.weight", 1, S.d_model, false);
    if (!emb || !out || !on) return fail(kTensorNotFound, "token_embd / output / output_norm missing or of another shape");
    qtype_ = static_cast<int>(out->type);
    emb_qtype_ = static_cast<int>(emb->type);
    emb_ = emb->ptr;
    w_out_ = out->ptr;
    out_norm_ = static_cast<const float*>(on->ptr);

    hesa_cuda_model hm{};
    hm.n_layer = static_cast<int32_t>(S.n_layer);
    hm.d_model = static_cast<int32_t>(S.d_model);
    hm.n_head = static_cast<int32_t>(S.n_head);
    hm.n_kv_head = static_cast<int32_t>(S.n_kv_head);
    hm.head_dim = static_cast<int32_t>(hd);
    hm.d_ff = static_cast<int32_t>(S.d_ff);
    hm.vocab = static_cast<int32_t>(S.vocab);
    hm.ctx = ctx;
    hm.rms_eps = S.rms_eps;
    hm.rope_base = S.rope_base;
    hm.qtype = qtype_;

    if (cudaSetDevice(m.device()) != cudaSuccess) return fail(9, "cudaSetDevice failed");
    const size_t kd = static_cast<size_t>(S.n_kv_head * hd);
    const size_t cache = static_cast<size_t>(ctx) * kd * 2;   // fp16 bytes of one cache
    if (cudaMalloc(&kv_, cache * 2 * static_cast<size_t>(S.n_layer)) != cudaSuccess) {
        kv_ = nullptr;
        return fail(kOutOfMemory, "KV caches");
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(kv_, 0, cache * 2 * static_cast<size_t>(S.n_layer), s) != cudaSuccess)
        return fail(9, "KV clear");

    std::vector<hesa_cuda_layer> ls(static_cast<size_t>(S.n_layer));
    for (int64_t l = 0; l < S.n_layer; ++l) {
        const std::string b = "blk." + std::to_string(l) + ".";
        const DeviceTensor* wq = need(b + "attn_q.weight", S.n_head * hd, S.d_model, true);
        const DeviceTensor* wk = need(b + "attn_k.weight", S.n_kv_head * hd, S.d_model, true);
        const DeviceTensor* wv = need(b + "attn_v.weight", S.n_kv_head * hd, S.d_model, true);
        const DeviceTensor* wo = need(b + "attn_output.weight", S.d_model, S.n_head * hd, true);
        const DeviceTensor* wg = need(b + "ffn_gate.weight", S.d_ff, S.d_model, true);
        const DeviceTensor* wu = need(b + "ffn_up.weight", S.d_ff, S.d_model, true);
        const DeviceTensor* wd = need(b + "ffn_down.weight", S.d_model, S.d_ff, true);
        const DeviceTensor* an = need(b + "attn_norm.weight", 1, S.d_model, false);
        const DeviceTensor* fn = need(b + "ffn_norm.weight", 1, S.d_model, false);
        if (!wq || !wk || !wv || !wo || !wg || !wu || !wd || !an || !fn)
            return fail(kTensorNotFound, "layer " + std::to_string(l) + ": a tensor is missing or of another shape");
        for (const DeviceTensor* t : {wq, wk, wv, wo, wg, wu, wd})
            if (static_cast<int>(t->type) != qtype_)
                return fail(kInvalidFormat, "layer " + std::to_string(l) + ": projections of mixed quant types");
        hesa_cuda_layer& L = ls[static_cast<size_t>(l)];
        L.wq = wq->ptr; L.wk = wk->ptr; L.wv = wv->ptr; L.wo = wo->ptr;
        L.w_gate = wg->ptr; L.w_up = wu->ptr; L.w_down = wd->ptr;
        L.attn_norm = static_cast<const float*>(an->ptr);
        L.ffn_norm = static_cast<const float*>(fn->ptr);
        L.k_cache = static_cast<uint8_t*>(kv_) + (2 * static_cast<size_t>(l)) * cache;
        L.v_cache = static_cast<uint8_t*>(kv_) + (2 * static_cast<size_t>(l) + 1) * cache;
    }
    model_.assign(reinterpret_cast<const unsigned char*>(&hm), reinterpret_cast<const unsigned char*>(&hm) + sizeof(hm));
    layers_.assign(reinterpret_cast<const unsigned char*>(ls.data()),
                   reinterpret_cast<const unsigned char*>(ls.data()) + ls.size() * sizeof(hesa_cuda_layer));

    // rope angle table (the reference's float formulas, computed on the host)
    // for every position the model was trained for, and at least the ring
    rope_rows_ = static_cast<int32_t>(std::max<int64_t>(ctx, std::min<int64_t>(S.context, int64_t(1) << 20)));
    std::vector<float> table(static_cast<size_t>(rope_rows_) * hd);
    if (hesa_cuda_rope_table(table.data(), rope_rows_, hd, S.rope_base) != 0)
        return fail(kInvalidArgument, "rope table");
    ws_bytes_ = hesa_cuda_decode_workspace_size(&hm);
    if (!ws_bytes_) return fail(kInvalidFormat, "decode step does not take this shape");
    if (cudaMalloc(reinterpret_cast<void**>(&rope_), table.size() * 4) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&x_), static_cast<size_t>(S.d_model) * 4) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&logits_), static_cast<size_t>(S.vocab) * 4) != cudaSuccess ||
        cudaMalloc(&ws_, ws_bytes_) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&tok_pos_), 2 * sizeof(int32_t)) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void**>(&host_tp_), 2 * sizeof(int32_t)) != cudaSuccess)
        return fail(kOutOfMemory, "decode buffers");
    if (cudaMemcpyAsync(rope_, table.data(), table.size() * 4, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemsetAsync(ws_, 0, ws_bytes_, s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
        return fail(9, "decode set-up copies");
    return kOk;
}

int DecodeSession::enqueue_step() {
    if (!ws_) return fail(kInvalidArgument, "session not initialised");
    const auto* hm = reinterpret_cast<const hesa_cuda_model*>(model_.data());
    const auto* ls = reinterpret_cast<const hesa_cuda_layer*>(layers_.data());
    int rc = hesa_cuda_embed(emb_qtype_, emb_, shape_.vocab, shape_.d_model, tok_pos_, x_, stream_);
    if (rc != 0) return fail(rc, hesa_cuda_last_error());
    rc = hesa_cuda_decode_step(hm, ls, out_norm_, w_out_, rope_, rope_rows_, x_, tok_pos_ + 1, logits_, ws_, ws_bytes_,
                               stream_);
    if (rc != 0) return fail(rc, hesa_cuda_last_error());
    return kOk;
}

int DecodeSession::step(int32_t token, int32_t pos, const float** logits_dev) {
    if (!ws_) return fail(kInvalidArgument, "session not initialised");
    if (token < 0 || token >= shape_.vocab || pos < 0 || pos >= rope_rows_)
        return fail(kInvalidArgument, "token or position out of range");
    cudaStream_t s = static_cast<cudaStream_t>(stream_);
    // the pinned pair may still feed the previous step's copy
    if (cudaStreamSynchronize(s) != cudaSuccess) return fail(9, "stream");
    host_tp_[0] = token;
    host_tp_[1] = pos;
    if (cudaMemcpyAsync(tok_pos_, host_tp_, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, s) != cudaSuccess)
        return fail(9, "token copy");
    const int rc = enqueue_step();
    if (rc == kOk && logits_dev) *logits_dev = logits_;
    return rc;
}

}  // namespace hesa_gguf
