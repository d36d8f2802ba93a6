// qmatvec.h -- host-side launchers of the matvec and dequant kernels
// (implemented in qmatvec.cu, called by abi.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace hesa_cuda {

// Upper bound on CTAs of the streaming kernel; sizes the workspace.
constexpr int kMaxGridCtas = 1024;

size_t qmv_workspace_bytes(int n_out);
bool qmv_stream_eligible(int qtype, const void* w, int64_t n_out, int64_t k);
int qmv_stream_grid(int qtype, int64_t n_out, int64_t k);

// Batch-1 streaming matvec on CUDA cores. workspace: qmv_workspace_bytes(n_out)
// bytes, zero-filled before first use (left zero-filled on success).
cudaError_t qmv_stream(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, float* y,
                       float scale, void* workspace, cudaStream_t stream, int grid_override);

// Same kernel with its scratch in a fixed device array owned by the library
// (no caller workspace, no allocation). Rows limited to qmv_noalloc_max_rows().
int64_t qmv_noalloc_max_rows();
// Device address of that array on the current device (cudaGetSymbolAddress,
// looked up once per device).
cudaError_t qmv_noalloc_scratch(uint8_t** out);
cudaError_t qmv_stream_noalloc(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, float* y,
                               float scale, cudaStream_t stream);

// Row-strip batch-1 matvec (k <= 24576): CTAs own contiguous rows, no workspace.
bool qmv_strip_eligible(int qtype, const void* w, int64_t n_out, int64_t k);
bool qmv_strip_shape_ok(int qtype, int64_t n_out, int64_t k);   // the same for a 16-byte aligned W
cudaError_t qmv_strip(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, float* y, float scale,
                      cudaStream_t stream);

// The strip kernel with a transformed input and an optional residual add, for
// the decode step: y = resid + scale * W . f(x) with f = identity, RMSNorm
// (x * inv_rms * norm_w, inv_rms = 1/sqrt(mean(x^2) + eps); k <= 12288) or
// SwiGLU (silu(x[i]) * x[k + i]; x holds 2k values). resid may equal y.
enum class StripInput { kPlain, kRmsNorm, kSiluMul };
bool qmv_strip_fused_eligible(int qtype, const void* w, int64_t n_out, int64_t k, StripInput in);
cudaError_t qmv_strip_fused(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, StripInput in,
                            const float* norm_w, float eps, float* y, const float* resid, float scale,
                            cudaStream_t stream);

// Row-sharded matvec with the all-gather fused into the epilogue: a rank's
// strip kernel stores its rows straight into the gathered output buffer of
// every rank (its own and its peers', mapped over NVLink with CUDA IPC).
// Buffers alternate by the parity of the rank's barrier count (peer_barrier
// increments it), so a rank may write step s + 1 into a peer while that peer
// still reads step s.
constexpr int kMaxPeers = 8;
struct PeerOut {
    float* y[2][kMaxPeers];   // [parity][rank]: where this shard's row 0 lands in that rank's buffer
    const uint32_t* epoch;    // this rank's barrier count (device); parity = *epoch & 1
    int world;                // number of ranks; 0 = plain output
};
cudaError_t qmv_strip_gather(int qtype, const void* w, int64_t n_rows, int64_t k, const float* x, float scale,
                             const PeerOut& out, cudaStream_t stream);

}  // namespace hesa_cuda
#include "peer_sync.cuh"
namespace hesa_cuda {

// The strip kernel of the sharded decode step: rows of y = scale * W . f(x)
// (+ a residual), f as qmv_strip_fused. Input: the tagged vector lin.x (and
// a tagged residual lin.resid, tagged outputs only) when lin.x is set, else
// the plain x. Output: every rank as tagged words (lout) when lout.world > 0,
// else the plain local y (+ the plain resid when set).
cudaError_t qmv_strip_shard(int qtype, const void* w, int64_t n_rows, int64_t k, StripInput in, const float* norm_w,
                            float eps, float scale, const float* x, float* y, const float* resid, const LLIn& lin,
                            const LLOut& lout, cudaStream_t stream);

// Row-sharded matvec whose rows reach every rank as tagged words: row i to
// element lout.off + i of lout.y[p] (of lout.y2[p] while the count is odd;
// lout.by_parity must be set; element order as peer_sync.cuh) with the tag
// (*lout.count << 12) | lout.lo. x is a plain local vector.
cudaError_t qmv_strip_gather_tagged(int qtype, const void* w, int64_t n_rows, int64_t k, const float* x, float scale,
                                    const LLOut& lout, cudaStream_t stream);

// y[0..n) (a plain local vector) to every rank as tagged words, as
// qmv_strip_gather_tagged stores its rows; for shapes the strip kernel does
// not take.
cudaError_t peer_scatter_tagged(const float* y, int64_t n, const LLOut& lout, cudaStream_t stream);

// End of a step of tagged gathers on this rank: waits (bounded by the peer
// wait limit; kStatusPeerTimeout on expiry) until each of the n elements of
// this rank's buffer of the step's parity (words0 while sync[0] is even,
// words1 while odd; whole units of 256 words) carries the tag
// (sync[0] << 12) | lo, writes their values to out, then advances sync[0]. sync[1] is the launch's CTA ticket (zero between
// launches). Launched with programmatic serialization; it waits for the grids
// before it.
cudaError_t peer_collect(const uint64_t* words0, const uint64_t* words1, int64_t n, float* out, uint32_t* sync,
                         uint32_t lo, cudaStream_t stream);

// Completion of the fused all-gathers of one step: every rank publishes
// *epoch + 1 into slot `rank` of every rank's flags (release, system scope),
// waits until all `world` slots of its own flags reach that value (acquire,
// bounded: on timeout the status word records kStatusPeerTimeout), then
// stores it into *epoch. flags[p] is rank p's flag array as mapped here.
cudaError_t peer_barrier(uint32_t* const* flags, int rank, int world, uint32_t* epoch, cudaStream_t stream);
// How long every peer wait enqueued from now on lasts before it records
// kStatusPeerTimeout (0 restores the default, 2 s).
void set_peer_wait_limit(unsigned long long ns);
unsigned long long peer_wait_limit();

// One warp per row, any k that is a multiple of the block size.
cudaError_t qmv_rowwise(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, int64_t ldx,
                        int64_t batch, float* y, int64_t ldy, float scale, cudaStream_t stream);

// Sticky status word of the bounded waits (0 = healthy).
cudaError_t read_device_status(int* out);
// Device address of the library's status word on the current device (kernels
// of other files record their failures there too).
cudaError_t status_word(int** out);
cudaError_t clear_device_status(cudaStream_t stream);

cudaError_t dequantize(int qtype, const void* w, int64_t n_rows, int64_t k, float* out, int64_t ldo,
                       cudaStream_t stream);

}  // namespace hesa_cuda
