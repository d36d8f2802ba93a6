// abi.cu -- the extern "C" entry points declared in include/hesa_cuda.h.
//
// Validation happens here, on the host, before anything is launched: bad
// qtype, shape, stride, alignment or null pointer return an error code and
// launch nothing. CUDA errors map to HESA_CUDA_ERROR with the message kept
// per host thread.
#include "../../include/hesa_cuda.h"
#include "abi_errors.h"
#include "trace.h"
#include "qmatvec.h"
#include "qmm.h"
#include "quantize.h"
#include "qtypes.cuh"

#include <algorithm>
#include <cstring>
#include <string>

namespace {

thread_local std::string t_last_error;

int fail(int code, const char* what) {
    t_last_error = what;
    return code;
}

int cuda_fail(cudaError_t e, const char* where) {
    t_last_error = std::string(where) + ": " + cudaGetErrorString(e);
    return HESA_CUDA_ERROR;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

namespace hesa_cuda {
int record_error(int code, const char* what) { return fail(code, what); }
int record_cuda_error(cudaError_t e, const char* where) { return cuda_fail(e, where); }
}  // namespace hesa_cuda

extern "C" {

const char* hesa_cuda_version(void) { return "hesa-b200 0.1 sm_100a"; }

const char* hesa_cuda_last_error(void) { return t_last_error.c_str(); }

size_t hesa_cuda_row_bytes(int qtype, int64_t k) {
    const int be = hesa_cuda::block_elems(qtype);
    if (be == 0 || k <= 0 || k % be != 0) return 0;
    return static_cast<size_t>(k / be) * static_cast<size_t>(hesa_cuda::block_bytes(qtype));
}

size_t hesa_cuda_qmatvec_workspace_size(int qtype, int64_t n_out, int64_t k, int64_t batch) {
    if (!hesa_cuda::qtype_supported(qtype) || n_out <= 0 || k <= 0 || batch <= 0) return 0;
    size_t n = hesa_cuda::qmv_workspace_bytes(static_cast<int>(n_out));
    if (batch >= 2 && k % 256 == 0) {
        n = std::max(n, hesa_cuda::qmm_tc_workspace_bytes(qtype, n_out, k, batch));
        n = std::max(n, hesa_cuda::qmm_blk_workspace_bytes(qtype, n_out, k, batch));
    }
    return n;
}

int hesa_cuda_qmatvec(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, int64_t ldx,
                      int64_t batch, float* y, int64_t ldy, float scale, void* workspace,
                      size_t workspace_bytes, void* stream) {
    HESA_TRACE("hesa_cuda_qmatvec");
    if (!hesa_cuda::qtype_supported(qtype)) return fail(HESA_CUDA_BACKEND_NOT_AVAILABLE, "unsupported qtype");
    if (!w || !x || !y) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (n_out <= 0 || k <= 0 || batch <= 0) return fail(HESA_CUDA_SHAPE_MISMATCH, "non-positive dimension");
    if (n_out >= (int64_t(1) << 31) || k >= (int64_t(1) << 31))
        return fail(HESA_CUDA_SHAPE_MISMATCH, "dimension too large");
    if (k % hesa_cuda::block_elems(qtype) != 0)
        return fail(HESA_CUDA_SHAPE_MISMATCH, "k is not a multiple of the block size");
    if (ldx < k || (batch > 1 && ldy < n_out)) return fail(HESA_CUDA_SHAPE_MISMATCH, "leading dimension too small");
    if (!aligned16(w)) return fail(HESA_CUDA_INVALID_ARGUMENT, "weights must be 16-byte aligned");
    if (!aligned16(x) || !aligned16(y) || (ldx & 3) || (batch > 1 && (ldy & 3)))
        return fail(HESA_CUDA_INVALID_ARGUMENT, "x / y must be 16-byte aligned with ldx, ldy multiples of 4");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    // Two activation rows take two strip passes where the strip kernel applies
    // (4096 x 11008 Q4_K: 2 x 9.6 us against 23.3 us for one tcgen05 launch);
    // from three rows on, reading the weights once on the tensor cores wins
    // (23.5 against 28.8 us).
    const bool strip_ok = hesa_cuda::qmv_strip_eligible(qtype, w, n_out, k);
    if (hesa_cuda::qmm_tc_eligible(qtype, w, n_out, k, batch) && (batch >= 3 || !strip_ok)) {
        // several activation rows: tcgen05 matmul (A in TMEM), weights read once per 16 rows
        const size_t need = hesa_cuda::qmm_tc_workspace_bytes(qtype, n_out, k, batch);
        if (!workspace || workspace_bytes < need) return fail(HESA_CUDA_INVALID_ARGUMENT, "workspace too small");
        if (!aligned16(workspace)) return fail(HESA_CUDA_INVALID_ARGUMENT, "workspace must be 16-byte aligned");
        e = hesa_cuda::qmm_tc(qtype, w, n_out, k, x, ldx, batch, y, ldy, scale, workspace, s);
        if (e != cudaSuccess) return cuda_fail(e, "qmatvec tcgen05 kernel");
    } else if (hesa_cuda::qmm_blk_eligible(qtype, w, n_out, k, batch) && (batch >= 3 || !strip_ok)) {
        // Q8_0 / Q4_0 with several activation rows: tcgen05, one MMA per 32-weight block
        const size_t need = hesa_cuda::qmm_blk_workspace_bytes(qtype, n_out, k, batch);
        if (!workspace || workspace_bytes < need) return fail(HESA_CUDA_INVALID_ARGUMENT, "workspace too small");
        if (!aligned16(workspace)) return fail(HESA_CUDA_INVALID_ARGUMENT, "workspace must be 16-byte aligned");
        e = hesa_cuda::qmm_blk(qtype, w, n_out, k, x, ldx, batch, y, ldy, scale, workspace, s);
        if (e != cudaSuccess) return cuda_fail(e, "qmatvec tcgen05 block kernel");
    } else if (strip_ok) {
        // row strips: no workspace needed
        for (int64_t b = 0; b < batch; ++b) {
            e = hesa_cuda::qmv_strip(qtype, w, n_out, k, x + b * ldx, y + b * ldy, scale, s);
            if (e != cudaSuccess) return cuda_fail(e, "qmatvec strip kernel");
        }
    } else if (hesa_cuda::qmv_stream_eligible(qtype, w, n_out, k)) {
        const size_t need = hesa_cuda::qmv_workspace_bytes(static_cast<int>(n_out));
        if (!workspace || workspace_bytes < need) return fail(HESA_CUDA_INVALID_ARGUMENT, "workspace too small");
        if (!aligned16(workspace)) return fail(HESA_CUDA_INVALID_ARGUMENT, "workspace must be 16-byte aligned");
        for (int64_t b = 0; b < batch; ++b) {
            e = hesa_cuda::qmv_stream(qtype, w, n_out, k, x + b * ldx, y + b * ldy, scale, workspace, s, 0);
            if (e != cudaSuccess) return cuda_fail(e, "qmatvec stream kernel");
        }
    } else {
        e = hesa_cuda::qmv_rowwise(qtype, w, n_out, k, x, ldx, batch, y, ldy, scale, s);
        if (e != cudaSuccess) return cuda_fail(e, "qmatvec rowwise kernel");
    }
    return HESA_CUDA_OK;
}

int hesa_cuda_dequantize(int qtype, const void* w, int64_t n_rows, int64_t k, float* out, int64_t ldo,
                         void* stream) {
    HESA_TRACE("hesa_cuda_dequantize");
    if (!hesa_cuda::qtype_supported(qtype)) return fail(HESA_CUDA_BACKEND_NOT_AVAILABLE, "unsupported qtype");
    if (!w || !out) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (n_rows <= 0 || k <= 0 || k % hesa_cuda::block_elems(qtype) != 0 || ldo < k)
        return fail(HESA_CUDA_SHAPE_MISMATCH, "bad shape");
    cudaError_t e = hesa_cuda::dequantize(qtype, w, n_rows, k, out, ldo, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "dequantize kernel");
    return HESA_CUDA_OK;
}

int hesa_cuda_quantize(int qtype, const float* src, int64_t n_rows, int64_t k, int64_t ld_src, void* dst,
                       void* stream) {
    HESA_TRACE("hesa_cuda_quantize");
    if (!hesa_cuda::qtype_supported(qtype)) return fail(HESA_CUDA_BACKEND_NOT_AVAILABLE, "unsupported qtype");
    if (!src || !dst) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (n_rows <= 0 || k <= 0 || k % hesa_cuda::block_elems(qtype) != 0 || ld_src < k)
        return fail(HESA_CUDA_SHAPE_MISMATCH, "bad shape");
    cudaError_t e = hesa_cuda::quantize(qtype, src, n_rows, k, ld_src, dst, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "quantize kernel");
    return HESA_CUDA_OK;
}

int hesa_cuda_peer_alloc(size_t bytes, void** dev_ptr_out, void* handle_out) {
    if (!dev_ptr_out || !handle_out || bytes == 0) return fail(HESA_CUDA_INVALID_ARGUMENT, "bad peer_alloc arguments");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "peer_alloc cudaMalloc");
    e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(e, "peer_alloc");
    }
    static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
    std::memcpy(handle_out, &h, sizeof(h));
    *dev_ptr_out = p;
    return HESA_CUDA_OK;
}

int hesa_cuda_peer_free(void* dev_ptr) {
    if (!dev_ptr) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    const cudaError_t e = cudaFree(dev_ptr);
    return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "peer_free");
}

int hesa_cuda_peer_open(const void* handle, void** dev_ptr_out) {
    if (!handle || !dev_ptr_out) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "peer_open");
}

int hesa_cuda_peer_close(void* dev_ptr) {
    if (!dev_ptr) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
    return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "peer_close");
}

int hesa_cuda_qmatvec_gather(int qtype, const void* w, int64_t n_rows, int64_t k, const float* x, float scale,
                             float* const* y_peers, int world, const uint32_t* epoch, void* stream) {
    HESA_TRACE("hesa_cuda_qmatvec_gather");
    if (!hesa_cuda::qtype_supported(qtype)) return fail(HESA_CUDA_BACKEND_NOT_AVAILABLE, "unsupported qtype");
    if (!w || !x || !y_peers || !epoch) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (world < 1 || world > hesa_cuda::kMaxPeers) return fail(HESA_CUDA_INVALID_ARGUMENT, "world must be 1..8");
    if (n_rows <= 0 || k <= 0) return fail(HESA_CUDA_SHAPE_MISMATCH, "non-positive dimension");
    if (n_rows >= (int64_t(1) << 30) || k % 256 != 0)
        return fail(HESA_CUDA_SHAPE_MISMATCH, "gathered matvec needs k a multiple of 256");
    if (!aligned16(w) || !aligned16(x)) return fail(HESA_CUDA_INVALID_ARGUMENT, "W and x must be 16-byte aligned");
    if (!hesa_cuda::qmv_strip_eligible(qtype, w, n_rows, k))
        return fail(HESA_CUDA_SHAPE_MISMATCH, "gathered matvec needs k <= 24576");
    hesa_cuda::PeerOut out = {};
    for (int b = 0; b < 2; ++b)
        for (int p = 0; p < world; ++p) {
            if (!y_peers[b * world + p]) return fail(HESA_CUDA_INVALID_ARGUMENT, "null output pointer");
            out.y[b][p] = y_peers[b * world + p];
        }
    out.epoch = epoch;
    out.world = world;
    const cudaError_t e =
        hesa_cuda::qmv_strip_gather(qtype, w, n_rows, k, x, scale, out, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "gathered matvec kernel");
}

// Low bits of the tagged gather's tags: never 0, so the zero-filled words of a
// fresh allocation never pass for step 0's.
constexpr uint32_t kGatherTagLo = 1;

size_t hesa_cuda_gather_tagged_workspace_size(int qtype, int64_t n_rows, int64_t k) {
    if (!hesa_cuda::qtype_supported(qtype) || n_rows <= 0 || k <= 0 || k % 256 != 0) return 0;
    if (hesa_cuda::qmv_strip_shape_ok(qtype, n_rows, k)) return 0;
    // the plain matvec's workspace, then its output [n_rows] (256-byte aligned)
    const size_t mv = (hesa_cuda_qmatvec_workspace_size(qtype, n_rows, k, 1) + 255) & ~size_t(255);
    return mv + ((static_cast<size_t>(n_rows) * 4 + 255) & ~size_t(255));
}

int hesa_cuda_qmatvec_gather_tagged(int qtype, const void* w, int64_t n_rows, int64_t k, const float* x,
                                    float scale, uint64_t* const* y_peers, int64_t row0, int world,
                                    const uint32_t* sync, void* workspace, size_t workspace_bytes, void* stream) {
    HESA_TRACE("hesa_cuda_qmatvec_gather_tagged");
    if (!hesa_cuda::qtype_supported(qtype)) return fail(HESA_CUDA_BACKEND_NOT_AVAILABLE, "unsupported qtype");
    if (!w || !x || !y_peers || !sync) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (row0 < 0 || row0 >= (int64_t(1) << 40)) return fail(HESA_CUDA_INVALID_ARGUMENT, "bad row offset");
    if (world < 1 || world > hesa_cuda::kMaxPeers) return fail(HESA_CUDA_INVALID_ARGUMENT, "world must be 1..8");
    if (n_rows <= 0 || k <= 0) return fail(HESA_CUDA_SHAPE_MISMATCH, "non-positive dimension");
    if (n_rows >= (int64_t(1) << 30) || k % 256 != 0)
        return fail(HESA_CUDA_SHAPE_MISMATCH, "gathered matvec needs k a multiple of 256");
    if (!aligned16(w) || !aligned16(x)) return fail(HESA_CUDA_INVALID_ARGUMENT, "W and x must be 16-byte aligned");
    const bool strip = hesa_cuda::qmv_strip_eligible(qtype, w, n_rows, k);
    const size_t need = strip ? 0 : hesa_cuda_gather_tagged_workspace_size(qtype, n_rows, k);
    if (!strip && (!workspace || workspace_bytes < need || !aligned16(workspace)))
        return fail(HESA_CUDA_INVALID_ARGUMENT,
                    "this shape needs a workspace of hesa_cuda_gather_tagged_workspace_size bytes");
    hesa_cuda::LLOut out = {};
    for (int b = 0; b < 2; ++b)
        for (int p = 0; p < world; ++p) {
            uint64_t* q = y_peers[b * world + p];
            if (!q) return fail(HESA_CUDA_INVALID_ARGUMENT, "null output pointer");
            if (reinterpret_cast<uintptr_t>(q) & 15)
                return fail(HESA_CUDA_INVALID_ARGUMENT, "gathered buffers must be 16-byte aligned");
            (b == 0 ? out.y : out.y2)[p] = q;
        }
    out.off = row0;
    out.world = world;
    out.by_parity = 1;
    out.count = sync;
    out.lo = kGatherTagLo;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (strip) {
        const cudaError_t e = hesa_cuda::qmv_strip_gather_tagged(qtype, w, n_rows, k, x, scale, out, s);
        return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "tagged gathered matvec kernel");
    }
    // rows longer than the strip kernel takes: the plain matvec into the
    // workspace, then one kernel sends its rows to every rank
    const size_t mv = need - ((static_cast<size_t>(n_rows) * 4 + 255) & ~size_t(255));
    float* y_local = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + mv);
    const int rc = hesa_cuda_qmatvec(qtype, w, n_rows, k, x, k, 1, y_local, n_rows, scale, workspace, mv, stream);
    if (rc != HESA_CUDA_OK) return rc;
    const cudaError_t e = hesa_cuda::peer_scatter_tagged(y_local, n_rows, out, s);
    return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "tagged scatter kernel");
}

int hesa_cuda_peer_collect(const uint64_t* words, int64_t n, int64_t parity_stride, float* out, uint32_t* sync,
                           void* stream) {
    HESA_TRACE("hesa_cuda_peer_collect");
    if (!words || !out || !sync) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (n <= 0 || n >= (int64_t(1) << 30)) return fail(HESA_CUDA_SHAPE_MISMATCH, "word count must be 1 .. 2^30 - 1");
    if (parity_stride < ((n + 255) & ~int64_t(255)) || parity_stride % 256 != 0)
        return fail(HESA_CUDA_SHAPE_MISMATCH, "each parity holds whole units of 256 words");
    if ((reinterpret_cast<uintptr_t>(words) & 15) || (reinterpret_cast<uintptr_t>(sync) & 7))
        return fail(HESA_CUDA_INVALID_ARGUMENT, "words must be 16-byte and sync 8-byte aligned");
    const cudaError_t e = hesa_cuda::peer_collect(words, words + parity_stride, n, out, sync, kGatherTagLo,
                                                  static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "peer collect kernel");
}

int hesa_cuda_peer_barrier(uint32_t* const* flags, int rank, int world, uint32_t* epoch, void* stream) {
    HESA_TRACE("hesa_cuda_peer_barrier");
    if (!flags || !epoch) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (world < 1 || world > hesa_cuda::kMaxPeers || rank < 0 || rank >= world)
        return fail(HESA_CUDA_INVALID_ARGUMENT, "bad rank / world");
    for (int p = 0; p < world; ++p)
        if (!flags[p]) return fail(HESA_CUDA_INVALID_ARGUMENT, "null flag pointer");
    const cudaError_t e = hesa_cuda::peer_barrier(flags, rank, world, epoch, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "peer barrier kernel");
}

int hesa_cuda_set_peer_wait_limit_us(uint32_t limit_us) {
    if (limit_us > 60u * 1000u * 1000u) return fail(HESA_CUDA_INVALID_ARGUMENT, "peer wait limit above 60 s");
    hesa_cuda::set_peer_wait_limit(static_cast<unsigned long long>(limit_us) * 1000ull);
    return HESA_CUDA_OK;
}

int hesa_cuda_device_status(void* stream, int* status_out) {
    if (!status_out) return fail(HESA_CUDA_INVALID_ARGUMENT, "null status pointer");
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "synchronize");
    int v = 0;
    e = hesa_cuda::read_device_status(&v);
    if (e != cudaSuccess) return cuda_fail(e, "read device status");
    *status_out = v;
    return HESA_CUDA_OK;
}

int hesa_cuda_clear_device_status(void* stream) {
    cudaError_t e = hesa_cuda::clear_device_status(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "clear device status");
    return HESA_CUDA_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// decode-step helpers
// ---------------------------------------------------------------------------

#include "decode_ops.h"

#include <cmath>

extern "C" {

int hesa_cuda_matmul_f32(const float* a, int64_t n_out, int64_t k, const float* x, int64_t ldx, int64_t batch,
                         float* y, int64_t ldy, float scale, void* stream) {
    HESA_TRACE("hesa_cuda_matmul_f32");
    if (!a || !x || !y) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (n_out <= 0 || k <= 0 || batch <= 0 || ldx < k || (batch > 1 && ldy < n_out) ||
        n_out >= (int64_t(1) << 31) || k >= (int64_t(1) << 31))
        return fail(HESA_CUDA_SHAPE_MISMATCH, "bad shape");
    cudaError_t e = hesa_cuda::matmul_f32(a, n_out, k, x, ldx, batch, y, ldy, scale, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "matmul_f32");
}

int hesa_cuda_rms_norm(const float* in, const float* weight, float* out, int64_t n_rows, int64_t n, float eps,
                       void* stream) {
    if (!in || !weight || !out) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (n_rows <= 0 || n <= 0 || n_rows >= (int64_t(1) << 31) || n >= (int64_t(1) << 31))
        return fail(HESA_CUDA_SHAPE_MISMATCH, "bad shape");
    cudaError_t e = hesa_cuda::rms_norm(in, weight, out, n_rows, n, eps, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "rms_norm");
}

int hesa_cuda_silu_mul(const float* gate, const float* up, float* out, int64_t n, void* stream) {
    if (!gate || !out) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (n <= 0) return fail(HESA_CUDA_SHAPE_MISMATCH, "bad shape");
    cudaError_t e = hesa_cuda::silu_mul(gate, up, out, n, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "silu_mul");
}

int hesa_cuda_add(const float* a, const float* b, float* out, int64_t n, void* stream) {
    if (!a || !b || !out) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (n <= 0) return fail(HESA_CUDA_SHAPE_MISMATCH, "bad shape");
    cudaError_t e = hesa_cuda::binary(a, b, out, n, 0, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "add");
}

int hesa_cuda_mul(const float* a, const float* b, float* out, int64_t n, void* stream) {
    if (!a || !b || !out) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (n <= 0) return fail(HESA_CUDA_SHAPE_MISMATCH, "bad shape");
    cudaError_t e = hesa_cuda::binary(a, b, out, n, 1, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "mul");
}

int hesa_cuda_softmax(const float* in, float* out, int64_t n_rows, int64_t n, void* stream) {
    if (!in || !out) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (n_rows <= 0 || n <= 0 || n_rows >= (int64_t(1) << 31) || n >= (int64_t(1) << 31))
        return fail(HESA_CUDA_SHAPE_MISMATCH, "bad shape");
    cudaError_t e = hesa_cuda::softmax(in, out, n_rows, n, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "softmax");
}

int hesa_cuda_rope_table(float* table_host, int32_t n_pos, int64_t head_dim, float freq_base) {
    if (!table_host) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (n_pos <= 0 || head_dim <= 0 || (head_dim & 1)) return fail(HESA_CUDA_SHAPE_MISMATCH, "bad shape");
    const int64_t half = head_dim / 2;
    for (int32_t p = 0; p < n_pos; ++p) {
        float* row = table_host + static_cast<int64_t>(p) * head_dim;
        for (int64_t d = 0; d < half; ++d) {
            // the expressions of cpu_rope_f32, in float, with the host libm
            const float freq = 1.0f / std::pow(freq_base, 2.0f * static_cast<float>(d) / static_cast<float>(head_dim));
            const float theta = static_cast<float>(p) * freq;
            row[d] = std::cos(theta);
            row[half + d] = std::sin(theta);
        }
    }
    return HESA_CUDA_OK;
}

int hesa_cuda_rope(float* data, int64_t n_heads, int64_t head_dim, const float* table, int32_t table_rows,
                   const int32_t* pos_dev, int32_t pos_host, void* stream) {
    if (!data || !table) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (n_heads <= 0 || head_dim <= 0 || (head_dim & 1) || table_rows <= 0 ||
        (!pos_dev && (pos_host < 0 || pos_host >= table_rows)))
        return fail(HESA_CUDA_SHAPE_MISMATCH, "bad shape");
    cudaError_t e = hesa_cuda::rope(data, n_heads, head_dim, table, table_rows, pos_dev, pos_host,
                                    static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "rope");
}

int hesa_cuda_kv_store(const float* k, const float* v, void* k_cache, void* v_cache, int64_t row_elems, int64_t ctx,
                       const int32_t* pos_dev, int32_t pos_host, void* stream) {
    if (!k || !v || !k_cache || !v_cache) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (row_elems <= 0 || ctx <= 0 || (!pos_dev && pos_host < 0) || row_elems * ctx >= (int64_t(1) << 40))
        return fail(HESA_CUDA_SHAPE_MISMATCH, "bad shape");
    cudaError_t e = hesa_cuda::kv_store(k, v, k_cache, v_cache, row_elems, ctx, pos_dev, pos_host,
                                        static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "kv_store");
}

size_t hesa_cuda_attention_workspace_size(int64_t n_head, int64_t head_dim, int64_t ctx) {
    if (n_head <= 0 || head_dim <= 0 || ctx <= 0) return 0;
    return hesa_cuda::attention_workspace_bytes(n_head, head_dim, ctx);
}

int hesa_cuda_attention(const float* q, const void* k_cache, const void* v_cache, float* out, int64_t n_head,
                        int64_t n_kv_head, int64_t head_dim, int64_t ctx, const int32_t* pos_dev, int32_t pos_host,
                        void* workspace, size_t workspace_bytes, void* stream) {
    HESA_TRACE("hesa_cuda_attention");
    if (!q || !k_cache || !v_cache || !out || !workspace) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (!aligned16(k_cache) || !aligned16(v_cache))
        return fail(HESA_CUDA_INVALID_ARGUMENT, "KV caches must be 16-byte aligned");
    if (ctx > 131072) return fail(HESA_CUDA_SHAPE_MISMATCH, "ctx above 131072 slots");
    if (n_head <= 0 || n_kv_head <= 0 || n_head % n_kv_head != 0 || ctx <= 0 || (!pos_dev && pos_host < 0))
        return fail(HESA_CUDA_SHAPE_MISMATCH, "bad shape");
    if (head_dim != 64 && head_dim != 128 && head_dim != 256)
        return fail(HESA_CUDA_SHAPE_MISMATCH, "head_dim must be 64, 128 or 256");
    if (workspace_bytes < hesa_cuda::attention_workspace_bytes(n_head, head_dim, ctx))
        return fail(HESA_CUDA_INVALID_ARGUMENT, "workspace too small");
    cudaError_t e = hesa_cuda::attention(q, k_cache, v_cache, out, n_head, n_kv_head, head_dim, ctx, pos_dev,
                                         pos_host, workspace, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HESA_CUDA_OK : cuda_fail(e, "attention");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// allocation-free matvec
// ---------------------------------------------------------------------------

extern "C" int hesa_cuda_qmatvec_noalloc(int qtype, const void* w, int64_t n_out, int64_t k, const float* x,
                                         int64_t ldx, int64_t batch, float* y, int64_t ldy, float scale,
                                         void* stream) {
    HESA_TRACE("hesa_cuda_qmatvec_noalloc");
    if (!hesa_cuda::qtype_supported(qtype)) return fail(HESA_CUDA_BACKEND_NOT_AVAILABLE, "unsupported qtype");
    if (!w || !x || !y) return fail(HESA_CUDA_INVALID_ARGUMENT, "null pointer");
    if (n_out <= 0 || k <= 0 || batch <= 0) return fail(HESA_CUDA_SHAPE_MISMATCH, "non-positive dimension");
    if (n_out >= (int64_t(1) << 31) || k >= (int64_t(1) << 31))
        return fail(HESA_CUDA_SHAPE_MISMATCH, "dimension too large");
    if (k % hesa_cuda::block_elems(qtype) != 0)
        return fail(HESA_CUDA_SHAPE_MISMATCH, "k is not a multiple of the block size");
    if (ldx < k || (batch > 1 && ldy < n_out)) return fail(HESA_CUDA_SHAPE_MISMATCH, "leading dimension too small");
    if (!aligned16(w)) return fail(HESA_CUDA_INVALID_ARGUMENT, "weights must be 16-byte aligned");
    if (!aligned16(x) || !aligned16(y) || (ldx & 3) || (batch > 1 && (ldy & 3)))
        return fail(HESA_CUDA_INVALID_ARGUMENT, "x / y must be 16-byte aligned with ldx, ldy multiples of 4");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool strip = hesa_cuda::qmv_strip_eligible(qtype, w, n_out, k);
    const bool streaming = !strip && hesa_cuda::qmv_stream_eligible(qtype, w, n_out, k);
    if (streaming && n_out > hesa_cuda::qmv_noalloc_max_rows())
        return fail(HESA_CUDA_SHAPE_MISMATCH,
                    "n_out exceeds the 65536 rows the library's fixed scratch array covers at this k; "
                    "use hesa_cuda_qmatvec with a caller workspace");
    // the fixed array's device address, looked up on the first call on this
    // device whichever kernel the shape takes (so that call, made before any
    // stream capture, is the only one that queries the runtime for it)
    uint8_t* scratch = nullptr;
    cudaError_t e = hesa_cuda::qmv_noalloc_scratch(&scratch);
    if (e != cudaSuccess) return cuda_fail(e, "no-alloc scratch lookup");
    if (strip) {
        // the row-strip kernel reduces inside each CTA: no scratch, any n_out
        for (int64_t b = 0; b < batch; ++b) {
            e = hesa_cuda::qmv_strip(qtype, w, n_out, k, x + b * ldx, y + b * ldy, scale, s);
            if (e != cudaSuccess) return cuda_fail(e, "qmatvec strip kernel");
        }
    } else if (streaming) {
        // rows too long for the strip kernel: the streaming kernel, with its
        // scratch in the library's fixed array
        for (int64_t b = 0; b < batch; ++b) {
            e = hesa_cuda::qmv_stream_noalloc(qtype, w, n_out, k, x + b * ldx, y + b * ldy, scale, s);
            if (e != cudaSuccess) return cuda_fail(e, "qmatvec no-alloc stream kernel");
        }
    } else {
        // the row-wise kernel needs no scratch
        e = hesa_cuda::qmv_rowwise(qtype, w, n_out, k, x, ldx, batch, y, ldy, scale, s);
        if (e != cudaSuccess) return cuda_fail(e, "qmatvec rowwise kernel");
    }
    return HESA_CUDA_OK;
}
