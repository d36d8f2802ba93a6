// decode_ops.cu -- the non-matvec kernels of a Llama-style decode step
// (single token), with the semantics of hesa-llm's CPU kernels
// (src/backend/cpu_backend.cpp):
//   matmul_f32    cpu_matmul_f32 (:24-41) for F32 weights, one warp per row
//   rms_norm      cpu_rms_norm_f32 (:72-89): inv = 1/sqrt(mean(x^2) + eps)
//   silu_mul      cpu_silu_f32 (:91-96) of gate, times up
//   add / mul     cpu_add_f32 (:43-46) / CPU_Backend::mul (:170-177)
//   softmax       cpu_softmax_f32 (:48-70)
//   rope          cpu_rope_f32 (:98-120), rotate-half, angles from a table
//                 computed on the host with the reference's own formulas
//   kv_store      fp16 ring-buffer write of k and v at slot pos % ctx
//   attention     single-query SDPA (:225-294) over the fp16 ring, GQA,
//                 score scale 1/sqrt(head_dim), split over the context
//                 with a deterministic last-arrival combine per head
// The position is read from device memory so a captured CUDA graph can be
// replayed for every token.
#include "hesa_common.cuh"
#include "peer_sync.cuh"
#include "decode_ops.h"
#include "qmatvec.h"

#include <cuda/atomic>
#include <cuda_fp16.h>

namespace hesa_cuda {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__global__ void __launch_bounds__(256)
matmul_f32_kernel(const float* __restrict__ a, int n_out, int k, const float* __restrict__ x, int64_t ldx,
                  int batch, float* __restrict__ y, int64_t ldy, float scale) {
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
    if (row >= n_out) return;
    const float* ar = a + row * k;
    for (int b = 0; b < batch; ++b) {
        const float* xb = x + b * ldx;
        float acc = 0.f;
        for (int i = lane; i < k; i += 32) acc = fmaf(ar[i], xb[i], acc);
        acc = warp_sum(acc);
        if (lane == 0) y[b * ldy + row] = acc * scale;
    }
}

// One CTA of 1024 threads per row.
__global__ void __launch_bounds__(1024)
rms_norm_kernel(const float* __restrict__ in, const float* __restrict__ w, float* __restrict__ out, int n,
                float eps) {
    // up to kRmsCache values per thread stay in registers between the two
    // passes (every load of the row is issued before the reduction)
    constexpr int kRmsCache = 8;
    __shared__ float red[32];
    const float* row = in + static_cast<int64_t>(blockIdx.x) * n;
    float* o = out + static_cast<int64_t>(blockIdx.x) * n;
    float v[kRmsCache];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < kRmsCache; ++c) {
        const int i = threadIdx.x + c * blockDim.x;
        v[c] = i < n ? row[i] : 0.f;
        ss = fmaf(v[c], v[c], ss);
    }
    for (int i = threadIdx.x + kRmsCache * blockDim.x; i < n; i += blockDim.x) ss = fmaf(row[i], row[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) tot += red[i];
    const float inv = 1.0f / sqrtf(tot / static_cast<float>(n) + eps);
#pragma unroll
    for (int c = 0; c < kRmsCache; ++c) {
        const int i = threadIdx.x + c * blockDim.x;
        if (i < n) o[i] = v[c] * inv * w[i];
    }
    for (int i = threadIdx.x + kRmsCache * blockDim.x; i < n; i += blockDim.x) o[i] = row[i] * inv * w[i];
}

__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ o,
                                int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float v = g[i];
        o[i] = (v / (1.0f + expf(-v))) * (u ? u[i] : 1.0f);
    }
}

__global__ void binary_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ o,
                              int64_t n, int op) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        o[i] = op == 0 ? a[i] + b[i] : a[i] * b[i];
}

__global__ void __launch_bounds__(256)
softmax_kernel(const float* __restrict__ in, float* __restrict__ out, int n) {
    __shared__ float red[8];
    const float* row = in + static_cast<int64_t>(blockIdx.x) * n;
    float* o = out + static_cast<int64_t>(blockIdx.x) * n;
    const int nw = blockDim.x >> 5;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, row[i]);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = red[0];
    for (int i = 1; i < nw; ++i) m = fmaxf(m, red[i]);
    __syncthreads();
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf(row[i] - m);
        o[i] = e;
        s += e;
    }
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < nw; ++i) tot += red[i];
    const float inv = 1.0f / tot;
    for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] *= inv;
}

// data [n_heads, head_dim]; table row p holds cos[half] then sin[half]
__global__ void rope_kernel(float* __restrict__ data, int n_heads, int head_dim, const float* __restrict__ table,
                            int table_rows, const int32_t* __restrict__ pos_dev, int32_t pos_host,
                            int* __restrict__ status) {
    const int half = head_dim >> 1;
    const int32_t pos = pos_dev ? *pos_dev : pos_host;
    if (pos < 0 || pos >= table_rows) {   // no row of the table: leave data as is
        if (blockIdx.x == 0 && threadIdx.x == 0) record_status(status, kStatusBadPosition);
        return;
    }
    const float* cs = table + static_cast<int64_t>(pos) * head_dim;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_heads * half; i += gridDim.x * blockDim.x) {
        const int h = i / half, d = i - h * half;
        float* row = data + static_cast<int64_t>(h) * head_dim;
        const float c = cs[d], s = cs[half + d];
        const float x0 = row[d], x1 = row[d + half];
        // separately rounded products and sums, as cpu_rope_f32 computes them
        row[d] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        row[d + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
}

// rope of q (in place) and of k, and the fp16 KV write of the rotated k and
// of v into slot pos % ctx, in one kernel; same rounding as rope_kernel and
// kv_store_kernel.
__global__ void rope_kv_kernel(float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                               __half* __restrict__ kc, __half* __restrict__ vc, int n_head, int n_kv_head,
                               int head_dim, const float* __restrict__ table, int table_rows, int ctx,
                               const int32_t* __restrict__ pos_dev, int* __restrict__ status) {
    const int32_t pos = *pos_dev;
    if (pos < 0 || pos >= table_rows) {
        if (blockIdx.x == 0 && threadIdx.x == 0) record_status(status, kStatusBadPosition);
        return;
    }
    const int half = head_dim >> 1;
    const int64_t kd = static_cast<int64_t>(n_kv_head) * head_dim;
    const int64_t slot = pos % ctx;
    const float* cs = table + static_cast<int64_t>(pos) * head_dim;
    const int n_pairs = (n_head + n_kv_head) * half;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_pairs + static_cast<int>(kd);
         i += gridDim.x * blockDim.x) {
        if (i < n_pairs) {
            const int h = i / half, d = i - h * half;
            const float c = cs[d], sn = cs[half + d];
            if (h < n_head) {
                float* row = q + static_cast<int64_t>(h) * head_dim;
                const float x0 = row[d], x1 = row[d + half];
                row[d] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
                row[d + half] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
            } else {
                const int64_t off = static_cast<int64_t>(h - n_head) * head_dim;
                const float x0 = k[off + d], x1 = k[off + d + half];
                kc[slot * kd + off + d] = __float2half_rn(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
                kc[slot * kd + off + d + half] = __float2half_rn(__fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c)));
            }
        } else {
            const int64_t e = i - n_pairs;
            vc[slot * kd + e] = __float2half_rn(v[e]);
        }
    }
}

__global__ void kv_store_kernel(const float* __restrict__ k, const float* __restrict__ v, __half* __restrict__ kc,
                                __half* __restrict__ vc, int row_elems, int ctx, const int32_t* __restrict__ pos_dev,
                                int32_t pos_host, int* __restrict__ status) {
    const int32_t pos = pos_dev ? *pos_dev : pos_host;
    if (pos < 0) {   // no slot: write nothing
        if (blockIdx.x == 0 && threadIdx.x == 0) record_status(status, kStatusBadPosition);
        return;
    }
    const int64_t slot = pos % ctx;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < row_elems; i += gridDim.x * blockDim.x) {
        kc[slot * row_elems + i] = __float2half_rn(k[i]);
        vc[slot * row_elems + i] = __float2half_rn(v[i]);
    }
}

constexpr int kAttnWarps = 4;
constexpr int kAttnMaxDim = 256;
constexpr int kAttnPos = 8;   // positions per warp step
constexpr int kAttnMaxSplits = 1024;
constexpr int kAttnStage = 32;   // positions per pipeline stage: kAttnWarps warps x kAttnPos
constexpr int kAttnDepth = 3;    // stage buffers: three stages in flight (4 CTAs per SM at head_dim 128)
static_assert(kAttnStage == kAttnWarps * kAttnPos, "a stage is one step of every warp");

// DPL consecutive fp16 values (2, 4 or 8: one 4-, 8- or 16-byte load).
template <int DPL> struct HalfVec;
template <> struct HalfVec<2> {
    uint32_t w;
    __device__ float f(int i) const { return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> (16 * i)))); }
};
template <> struct HalfVec<4> {
    uint2 w;
    __device__ float f(int i) const {
        const uint32_t x = i < 2 ? w.x : w.y;
        return __half2float(__ushort_as_half(static_cast<unsigned short>(x >> (16 * (i & 1)))));
    }
};
template <> struct HalfVec<8> {
    uint4 w;
    __device__ float f(int i) const {
        const uint32_t x = i < 2 ? w.x : i < 4 ? w.y : i < 6 ? w.z : w.w;
        return __half2float(__ushort_as_half(static_cast<unsigned short>(x >> (16 * (i & 1)))));
    }
};
// 16-byte global -> shared copy that completes asynchronously (cp.async);
// cp_async_wait_all waits for this thread's copies.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                 ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// wait until at most kAttnDepth - 1 committed groups of this thread are still in flight
__device__ __forceinline__ void cp_async_wait_depth() {
    asm volatile("cp.async.wait_group %0;" ::"n"(kAttnDepth - 1) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

template <int DPL>
__device__ __forceinline__ HalfVec<DPL> load_halves(const __half* p) {
    HalfVec<DPL> v;
    if constexpr (DPL == 2) v.w = *reinterpret_cast<const uint32_t*>(p);
    else if constexpr (DPL == 4) v.w = *reinterpret_cast<const uint2*>(p);
    else v.w = *reinterpret_cast<const uint4*>(p);
    return v;
}

// grid (n_head, n_split); 4 warps; 128 positions per CTA. Each CTA reduces
// its context chunk to (max, sum, acc[head_dim]) and writes it to the
// workspace; the last CTA of the head (ticket) combines the splits in split
// order and writes out.
//
// A warp step takes 8 positions. Scores: lanes 4t .. 4t+3 score position t,
// lane (t, qq) taking the 16-byte pieces qq, qq+4, ... of the K row (a
// quarter-warp reads 64 contiguous bytes of two rows 16 bytes out of bank
// phase: K rows are padded by 16 bytes) against the matching pieces of q held
// in registers; two shuffles combine the four partial dots. The step's
// maximum and sum run over the lanes 4 apart (three shuffles each), one
// exponential per lane. P . V: lane owns head_dim/32 consecutive dims.
// With ROPE, the kernel also does the work of rope_kv_kernel for the decode
// step: q arrives unrotated and is rotated in registers (the pair (d, d +
// head_dim/2) sits in one lane), and the CTA whose chunk holds slot
// pos % ctx rotates this token's k, rounds k and v to fp16, puts them into
// that row of its shared-memory stage (over whatever the copy brought) and,
// for the first query head of each KV head, into the cache. Rounding as
// rope_kv_kernel, so the result equals rope_kv followed by the plain kernel.
struct AttnRope {
    const float* k_new;   // this token's k [n_kv_head * head_dim] (unrotated)
    const float* v_new;   // this token's v [n_kv_head * head_dim]
    __half* kc;           // the caches, written at slot pos % ctx
    __half* vc;
    const float* table;   // rope table [table_rows][head_dim]: cos, then sin
    int table_rows;
    int* status;
    // head-sharded decode: element h * head_dim + d of this rank's heads goes
    // to element peer_off + h * head_dim + d of the tagged vector at
    // peer_out[p] on every rank p (peer_sync.cuh); peer_world 0: to out
    uint64_t* peer_out[kPeerSyncMax];
    int64_t peer_off;
    int peer_world;
    const uint32_t* ll_count;
    uint32_t ll_lo;
};

template <int DPL, bool ROPE>  // dims per lane (head_dim / 32)
__global__ void __launch_bounds__(kAttnWarps * 32)
attention_kernel(const float* __restrict__ q, const __half* __restrict__ kc, const __half* __restrict__ vc,
                 float* __restrict__ out, int n_head, int n_kv_head, int ctx, const int32_t* __restrict__ pos_dev,
                 int32_t pos_host, int chunk, float* __restrict__ part, int* __restrict__ counters, AttnRope ri) {
    const int head_dim = DPL * 32;
    constexpr int HD = DPL * 32, KS = HD + 8;   // K rows in halves, padded by 16 bytes
    constexpr int QP = HD / 8 / 4;              // 16-byte pieces of q per lane
    const int h = blockIdx.x, split = blockIdx.y, n_split = gridDim.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int32_t pos = pos_dev ? *pos_dev : pos_host;
    if constexpr (ROPE) {
        if (pos < 0 || pos >= ri.table_rows) {   // uniform: every CTA leaves, no counter is touched
            if (h == 0 && split == 0 && threadIdx.x == 0) record_status(ri.status, kStatusBadPosition);
            return;
        }
    }
    const int n_ctx = pos + 1 < ctx ? pos + 1 : ctx;
    const int kvh = h / (n_head / n_kv_head);
    const int64_t row_stride = static_cast<int64_t>(n_kv_head) * head_dim;
    const float sc = 1.0f / sqrtf(static_cast<float>(head_dim));

    const int t8 = lane >> 2, qq = lane & 3;   // scoring: position t8 of the step, piece phase qq
    const int j0 = split * chunk;
    const int j1 = min(n_ctx, j0 + chunk);

    float m = -INFINITY, l = 0.f, acc[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] = 0.f;

    // The chunk streams through shared memory in stages of kAttnStage
    // positions, kAttnDepth buffers deep: the cp.async copies of stages s + 1
    // and s + 2 are in flight while stage s is computed (16-byte pieces, every thread issuing
    // its share). Each warp takes kAttnPos positions of every stage: the score
    // reductions interleave and the running softmax is rescaled once per step.
    extern __shared__ __align__(16) uint8_t attn_smem[];
    __half* sbuf = reinterpret_cast<__half*>(attn_smem);   // [kAttnDepth][K (padded rows) | V][kAttnStage]
    constexpr int kPieces = DPL * 32 * 2 / 16;               // 16-byte pieces per row
    const int rows = j1 > j0 ? j1 - j0 : 0;
    const int n_stage = (rows + kAttnStage - 1) / kAttnStage;
    const __half* kg = kc + static_cast<int64_t>(j0) * row_stride + static_cast<int64_t>(kvh) * head_dim;
    const __half* vg = vc + static_cast<int64_t>(j0) * row_stride + static_cast<int64_t>(kvh) * head_dim;
    auto issue = [&](int st) {
        if (st < n_stage) {
            __half* sk = sbuf + static_cast<int64_t>(st % kAttnDepth) * kAttnStage * (KS + HD);
            __half* sv = sk + kAttnStage * KS;
            const int r0 = st * kAttnStage, nr = min(kAttnStage, rows - r0);
            for (int c = threadIdx.x; c < nr * kPieces; c += blockDim.x) {
                const int r = c / kPieces, o = (c - r * kPieces) * 8;
                cp_async16(sk + r * KS + o, kg + static_cast<int64_t>(r0 + r) * row_stride + o);
                cp_async16(sv + r * head_dim + o, vg + static_cast<int64_t>(r0 + r) * row_stride + o);
            }
        }
        cp_async_commit();   // an empty group when there is no such stage
    };
    // With ROPE (the decode step, launched with programmatic stream
    // serialization) the first two stages are requested before waiting for the
    // previous kernel: the cache rows of earlier tokens are never written by it
    // (this token's row is patched in below); q, k and v are, so they are read
    // after the wait.
    if constexpr (ROPE) {
        issue(0);
        issue(1);
        issue(2);
        grid_dep_wait();
    }
    float qv[QP][8];
#pragma unroll
    for (int c = 0; c < QP; ++c)
#pragma unroll
        for (int i = 0; i < 8; ++i) qv[c][i] = q[static_cast<int64_t>(h) * HD + 8 * (4 * c + qq) + i];

    // ROPE: this token's row (slot pos % ctx), when it falls in this chunk
    constexpr int kNewPer = (HD + kAttnWarps * 32 - 1) / (kAttnWarps * 32);   // elements per thread
    int new_stage = -1, new_row = 0;
    __half new_k[kNewPer], new_v[kNewPer];
    if constexpr (ROPE) {
        const float* cs = ri.table + static_cast<int64_t>(pos) * HD;
        // q pieces c and c + QP/2 hold dims d and d + HD/2
#pragma unroll
        for (int c = 0; c < QP / 2; ++c)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int d = 8 * (4 * c + qq) + i;
                const float cd = cs[d], sd = cs[HD / 2 + d];
                const float x0 = qv[c][i], x1 = qv[c + QP / 2][i];
                qv[c][i] = __fsub_rn(__fmul_rn(x0, cd), __fmul_rn(x1, sd));
                qv[c + QP / 2][i] = __fadd_rn(__fmul_rn(x0, sd), __fmul_rn(x1, cd));
            }
        const int slot = pos % ctx;
        if (slot >= j0 && slot < j1) {
            new_stage = (slot - j0) / kAttnStage;
            new_row = (slot - j0) % kAttnStage;
            const float* kn = ri.k_new + static_cast<int64_t>(kvh) * HD;
            const float* vn = ri.v_new + static_cast<int64_t>(kvh) * HD;
#pragma unroll
            for (int t = 0; t < kNewPer; ++t) {
                const int e = threadIdx.x + t * kAttnWarps * 32;   // element e of the row
                if (e < HD) {
                    const int d = e < HD / 2 ? e : e - HD / 2;
                    const float cd = cs[d], sd = cs[HD / 2 + d];
                    const float x0 = kn[d], x1 = kn[d + HD / 2];
                    const float r = e < HD / 2 ? __fsub_rn(__fmul_rn(x0, cd), __fmul_rn(x1, sd))
                                               : __fadd_rn(__fmul_rn(x0, sd), __fmul_rn(x1, cd));
                    new_k[t] = __float2half_rn(r);
                    new_v[t] = __float2half_rn(vn[e]);
                    if (h % (n_head / n_kv_head) == 0) {
                        const int64_t o = static_cast<int64_t>(slot) * row_stride + static_cast<int64_t>(kvh) * HD + e;
                        ri.kc[o] = new_k[t];
                        ri.vc[o] = new_v[t];
                    }
                }
            }
        }
    }
    if constexpr (!ROPE) {
        issue(0);
        issue(1);
        issue(2);
    }
    for (int st = 0; st < n_stage; ++st) {
        cp_async_wait_depth();   // stage st has landed (stages st + 1, st + 2 may still be in flight)
        __syncthreads();
        if constexpr (ROPE) {
            if (st == new_stage) {   // CTA-uniform
                __half* pk = sbuf + static_cast<int64_t>(st % kAttnDepth) * kAttnStage * (KS + HD);
                __half* pv = pk + kAttnStage * KS;
#pragma unroll
                for (int t = 0; t < kNewPer; ++t) {
                    const int e = threadIdx.x + t * kAttnWarps * 32;
                    if (e < HD) {
                        pk[new_row * KS + e] = new_k[t];
                        pv[new_row * HD + e] = new_v[t];
                    }
                }
                __syncthreads();
            }
        }
        const __half* sk = sbuf + static_cast<int64_t>(st % kAttnDepth) * kAttnStage * (KS + HD);
        const __half* sv = sk + kAttnStage * KS;
        const int jb = j0 + st * kAttnStage + warp * kAttnPos;   // this warp's first position
        if (jb < j1) {
            const int sb = j0 + st * kAttnStage;   // first position of the stage
            // scores of the step's 8 positions, four lanes each
            float a = 0.f;
            {
                const int r = min(jb + t8, j1 - 1) - sb;   // past the chunk: repeat, masked
                const __half* kr = sk + r * KS;
#pragma unroll
                for (int c = 0; c < QP; ++c) {
                    const uint4 kk = *reinterpret_cast<const uint4*>(kr + 8 * (4 * c + qq));
                    const float2 k0 = __half22float2(*reinterpret_cast<const __half2*>(&kk.x));
                    const float2 k1 = __half22float2(*reinterpret_cast<const __half2*>(&kk.y));
                    const float2 k2 = __half22float2(*reinterpret_cast<const __half2*>(&kk.z));
                    const float2 k3 = __half22float2(*reinterpret_cast<const __half2*>(&kk.w));
                    a = fmaf(qv[c][0], k0.x, a);
                    a = fmaf(qv[c][1], k0.y, a);
                    a = fmaf(qv[c][2], k1.x, a);
                    a = fmaf(qv[c][3], k1.y, a);
                    a = fmaf(qv[c][4], k2.x, a);
                    a = fmaf(qv[c][5], k2.y, a);
                    a = fmaf(qv[c][6], k3.x, a);
                    a = fmaf(qv[c][7], k3.y, a);
                }
                a += __shfl_xor_sync(0xffffffffu, a, 1);
                a += __shfl_xor_sync(0xffffffffu, a, 2);
            }
            const float sco = jb + t8 < j1 ? a * sc : -INFINITY;
            float mx = fmaxf(m, sco);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float corr = expf(m - mx);   // 0 on the first step (m = -inf)
            const float p = expf(sco - mx);    // 0 for a masked position
            float ps = p;
            ps += __shfl_xor_sync(0xffffffffu, ps, 4);
            ps += __shfl_xor_sync(0xffffffffu, ps, 8);
            ps += __shfl_xor_sync(0xffffffffu, ps, 16);
            l = fmaf(l, corr, ps);
#pragma unroll
            for (int i = 0; i < DPL; ++i) acc[i] *= corr;
#pragma unroll
            for (int t = 0; t < kAttnPos; ++t) {
                const float pt = __shfl_sync(0xffffffffu, p, 4 * t);
                const int r = min(jb + t, j1 - 1) - sb;
                const HalfVec<DPL> vv = load_halves<DPL>(sv + r * HD + lane * DPL);
#pragma unroll
                for (int i = 0; i < DPL; ++i) acc[i] = fmaf(pt, vv.f(i), acc[i]);
            }
            m = mx;
        }
        __syncthreads();   // every warp is done with this buffer before it is refilled
        issue(st + kAttnDepth);
    }
    cp_async_wait_all();   // nothing left in flight (the trailing groups are empty)
    if constexpr (ROPE) grid_dep_launch();   // the next launch may take the SMs this grid leaves

    // combine the 4 warps of the CTA
    __shared__ float s_m[kAttnWarps], s_l[kAttnWarps];
    __shared__ float s_acc[kAttnWarps][kAttnMaxDim];
    __shared__ int s_last;
    if (lane == 0) {
        s_m[warp] = m;
        s_l[warp] = l;
    }
#pragma unroll
    for (int i = 0; i < DPL; ++i) s_acc[warp][lane * DPL + i] = acc[i];
    __syncthreads();
    float* mine = part + (static_cast<int64_t>(h) * n_split + split) * (head_dim + 2);
    if (warp == 0) {
        float M = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, s_m[w]);
        float L = 0.f;
        float a[DPL];
#pragma unroll
        for (int i = 0; i < DPL; ++i) a[i] = 0.f;
        for (int w = 0; w < kAttnWarps; ++w) {
            const float f = s_m[w] == -INFINITY ? 0.f : expf(s_m[w] - M);
            L = fmaf(s_l[w], f, L);
#pragma unroll
            for (int i = 0; i < DPL; ++i) a[i] = fmaf(s_acc[w][lane * DPL + i], f, a[i]);
        }
#pragma unroll
        for (int i = 0; i < DPL; ++i) mine[2 + lane * DPL + i] = a[i];
        if (lane == 0) {
            mine[0] = M;
            mine[1] = L;
        }
        __syncwarp();
        if (lane == 0) {
            cuda::atomic_ref<int, cuda::thread_scope_device> cnt(counters[h]);
            s_last = cnt.fetch_add(1, cuda::memory_order_acq_rel) == n_split - 1;
        }
    }
    __syncthreads();
    if (s_last) {
        // the last CTA of the head combines the splits in one pass over them:
        // warp w folds splits w, w + 4, ... into a running (max, sum, acc),
        // rescaling as the maximum grows; the four warp results are then
        // merged in warp order (deterministic)
        cuda::atomic_thread_fence(cuda::memory_order_acquire, cuda::thread_scope_device);
        const float* base = part + static_cast<int64_t>(h) * n_split * (head_dim + 2);
        float Mw = -INFINITY, LL = 0.f, o[DPL];
#pragma unroll
        for (int i = 0; i < DPL; ++i) o[i] = 0.f;
#pragma unroll 4
        for (int s2 = warp; s2 < n_split; s2 += kAttnWarps) {
            const float* p = base + s2 * (head_dim + 2);
            const float ms = p[0];
            const float mn = fmaxf(Mw, ms);
            const float fo = Mw == -INFINITY ? 0.f : expf(Mw - mn);
            const float fs = ms == -INFINITY ? 0.f : expf(ms - mn);
            LL = fmaf(p[1], fs, LL * fo);
#pragma unroll
            for (int i = 0; i < DPL; ++i) o[i] = fmaf(p[2 + lane * DPL + i], fs, o[i] * fo);
            Mw = mn;
        }
        if (lane == 0) {
            s_m[warp] = Mw;
            s_l[warp] = LL;
        }
#pragma unroll
        for (int i = 0; i < DPL; ++i) s_acc[warp][lane * DPL + i] = o[i];
        __syncthreads();
        if (warp == 0) {
            float M = s_m[0];
#pragma unroll
            for (int w = 1; w < kAttnWarps; ++w) M = fmaxf(M, s_m[w]);
            float f[kAttnWarps];
#pragma unroll
            for (int w = 0; w < kAttnWarps; ++w) f[w] = s_m[w] == -INFINITY ? 0.f : expf(s_m[w] - M);
            float L = 0.f;
#pragma unroll
            for (int w = 0; w < kAttnWarps; ++w) L = fmaf(s_l[w], f[w], L);
            const float inv = 1.0f / L;
#pragma unroll
            for (int i = 0; i < DPL; ++i) {
                float a = 0.f;
#pragma unroll
                for (int w = 0; w < kAttnWarps; ++w) a = fmaf(s_acc[w][lane * DPL + i], f[w], a);
                const int64_t o = static_cast<int64_t>(h) * head_dim + lane * DPL + i;
                if (ri.peer_world == 0) {
                    out[o] = a * inv;
                } else {
                    const uint32_t tag = ll_tag(ri.ll_count, ri.ll_lo);
                    const int64_t at = ll_pos(ri.peer_off + o);
                    for (int p = 0; p < ri.peer_world; ++p) st_ll(ri.peer_out[p] + at, a * inv, tag);
                }
            }
            if (lane == 0) {
                cuda::atomic_ref<int, cuda::thread_scope_device> cnt(counters[h]);
                cnt.store(0, cuda::memory_order_relaxed);
            }
        }
    }
}

int grid_for(int64_t n, int threads, int cap = 148 * 8) {
    int64_t g = (n + threads - 1) / threads;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return static_cast<int>(g);
}

}  // namespace

cudaError_t matmul_f32(const float* a, int64_t n_out, int64_t k, const float* x, int64_t ldx, int64_t batch,
                       float* y, int64_t ldy, float scale, cudaStream_t s) {
    matmul_f32_kernel<<<static_cast<int>((n_out + 7) / 8), 256, 0, s>>>(a, static_cast<int>(n_out),
                                                                        static_cast<int>(k), x, ldx,
                                                                        static_cast<int>(batch), y, ldy, scale);
    return cudaGetLastError();
}

cudaError_t rms_norm(const float* in, const float* w, float* out, int64_t n_rows, int64_t n, float eps,
                     cudaStream_t s) {
    rms_norm_kernel<<<static_cast<int>(n_rows), 1024, 0, s>>>(in, w, out, static_cast<int>(n), eps);
    return cudaGetLastError();
}

cudaError_t silu_mul(const float* g, const float* u, float* o, int64_t n, cudaStream_t s) {
    silu_mul_kernel<<<grid_for(n, 256), 256, 0, s>>>(g, u, o, n);
    return cudaGetLastError();
}

cudaError_t binary(const float* a, const float* b, float* o, int64_t n, int op, cudaStream_t s) {
    binary_kernel<<<grid_for(n, 256), 256, 0, s>>>(a, b, o, n, op);
    return cudaGetLastError();
}

cudaError_t softmax(const float* in, float* out, int64_t n_rows, int64_t n, cudaStream_t s) {
    softmax_kernel<<<static_cast<int>(n_rows), 256, 0, s>>>(in, out, static_cast<int>(n));
    return cudaGetLastError();
}

cudaError_t rope(float* data, int64_t n_heads, int64_t head_dim, const float* table, int32_t table_rows,
                 const int32_t* pos_dev, int32_t pos_host, cudaStream_t s) {
    int* status = nullptr;
    cudaError_t e = status_word(&status);
    if (e != cudaSuccess) return e;
    rope_kernel<<<grid_for(n_heads * head_dim / 2, 256, 64), 256, 0, s>>>(
        data, static_cast<int>(n_heads), static_cast<int>(head_dim), table, table_rows, pos_dev, pos_host, status);
    return cudaGetLastError();
}

cudaError_t kv_store(const float* k, const float* v, void* kc, void* vc, int64_t row_elems, int64_t ctx,
                     const int32_t* pos_dev, int32_t pos_host, cudaStream_t s) {
    int* status = nullptr;
    cudaError_t e = status_word(&status);
    if (e != cudaSuccess) return e;
    kv_store_kernel<<<grid_for(row_elems, 256, 64), 256, 0, s>>>(k, v, static_cast<__half*>(kc),
                                                                  static_cast<__half*>(vc),
                                                                  static_cast<int>(row_elems),
                                                                  static_cast<int>(ctx), pos_dev, pos_host, status);
    return cudaGetLastError();
}

cudaError_t rope_kv(float* q, const float* k, const float* v, void* kc, void* vc, int64_t n_head, int64_t n_kv_head,
                    int64_t head_dim, const float* table, int32_t table_rows, int64_t ctx, const int32_t* pos_dev,
                    cudaStream_t s) {
    int* status = nullptr;
    cudaError_t e = status_word(&status);
    if (e != cudaSuccess) return e;
    const int64_t n = (n_head + n_kv_head) * (head_dim / 2) + n_kv_head * head_dim;
    rope_kv_kernel<<<grid_for(n, 256, 148 * 4), 256, 0, s>>>(
        q, k, v, static_cast<__half*>(kc), static_cast<__half*>(vc), static_cast<int>(n_head),
        static_cast<int>(n_kv_head), static_cast<int>(head_dim), table, table_rows, static_cast<int>(ctx), pos_dev,
        status);
    return cudaGetLastError();
}

size_t attention_workspace_bytes(int64_t n_head, int64_t head_dim, int64_t ctx) {
    const int64_t n_split = attention_splits(ctx);
    const size_t counters = ((static_cast<size_t>(n_head) * 4) + 255) & ~size_t(255);
    return counters + static_cast<size_t>(n_head) * n_split * (head_dim + 2) * 4;
}

int attention_splits(int64_t ctx) {
    // 128 positions per CTA: four 32-position stages
    int64_t n = (ctx + 127) / 128;
    if (n < 1) n = 1;
    if (n > kAttnMaxSplits) n = kAttnMaxSplits;
    return static_cast<int>(n);
}

template <int DPL, bool ROPE>
cudaError_t launch_attention(dim3 grid, size_t smem, cudaStream_t s, const float* q, const __half* k, const __half* v,
                             float* out, int nh, int nkv, int c, const int32_t* pos_dev, int32_t pos_host, int chunk,
                             float* part, int* counters, const AttnRope& ri) {
    if (smem > 48 * 1024) {
        static int set[64] = {0};
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
        if (set[dev] < static_cast<int>(smem)) {
            e = cudaFuncSetAttribute(attention_kernel<DPL, ROPE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem));
            if (e != cudaSuccess) return e;
            set[dev] = static_cast<int>(smem);
        }
    }
    if constexpr (!ROPE) {
        attention_kernel<DPL, ROPE><<<grid, kAttnWarps * 32, smem, s>>>(q, k, v, out, nh, nkv, c, pos_dev,
                                                                         pos_host, chunk, part, counters, ri);
        return cudaGetLastError();
    } else {
        // programmatic stream serialization: the CTAs may start while the
        // previous kernel finishes; the kernel waits for it before reading q, k, v
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = grid;
        cfg.blockDim = dim3(kAttnWarps * 32);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, attention_kernel<DPL, ROPE>, q, k, v, out, nh, nkv, c, pos_dev, pos_host,
                                  chunk, part, counters, ri);
    }
}

template <bool ROPE>
cudaError_t attention_any(const float* q, const void* kc, const void* vc, float* out, int64_t n_head,
                          int64_t n_kv_head, int64_t head_dim, int64_t ctx, const int32_t* pos_dev, int32_t pos_host,
                          void* workspace, const AttnRope& ri, cudaStream_t s) {
    const int n_split = attention_splits(ctx);
    const int chunk = static_cast<int>((ctx + n_split - 1) / n_split);
    int* counters = static_cast<int*>(workspace);
    float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                           (((static_cast<size_t>(n_head) * 4) + 255) & ~size_t(255)));
    dim3 grid(static_cast<unsigned>(n_head), static_cast<unsigned>(n_split));
    const __half* k = static_cast<const __half*>(kc);
    const __half* v = static_cast<const __half*>(vc);
    const int nh = static_cast<int>(n_head), nkv = static_cast<int>(n_kv_head), c = static_cast<int>(ctx);
    // kAttnDepth stage buffers of K (rows padded by 16 bytes) and V
    const size_t smem = static_cast<size_t>(kAttnDepth * kAttnStage) * static_cast<size_t>(2 * head_dim + 8) * 2;
    switch (head_dim) {
        case 64:
            return launch_attention<2, ROPE>(grid, smem, s, q, k, v, out, nh, nkv, c, pos_dev, pos_host, chunk, part,
                                             counters, ri);
        case 128:
            return launch_attention<4, ROPE>(grid, smem, s, q, k, v, out, nh, nkv, c, pos_dev, pos_host, chunk, part,
                                             counters, ri);
        case 256:
            return launch_attention<8, ROPE>(grid, smem, s, q, k, v, out, nh, nkv, c, pos_dev, pos_host, chunk, part,
                                             counters, ri);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t attention(const float* q, const void* kc, const void* vc, float* out, int64_t n_head,
                      int64_t n_kv_head, int64_t head_dim, int64_t ctx, const int32_t* pos_dev, int32_t pos_host,
                      void* workspace, cudaStream_t s) {
    return attention_any<false>(q, kc, vc, out, n_head, n_kv_head, head_dim, ctx, pos_dev, pos_host, workspace,
                                AttnRope{}, s);
}

cudaError_t attention_rope(const float* q, const float* k_new, const float* v_new, void* kc, void* vc, float* out,
                           int64_t n_head, int64_t n_kv_head, int64_t head_dim, const float* table,
                           int32_t table_rows, int64_t ctx, const int32_t* pos_dev, void* workspace,
                           cudaStream_t s) {
    return attention_rope_shard(q, k_new, v_new, kc, vc, out, n_head, n_kv_head, head_dim, table, table_rows, ctx,
                                pos_dev, workspace, nullptr, 0, 0, nullptr, 0u, s);
}

cudaError_t attention_rope_shard(const float* q, const float* k_new, const float* v_new, void* kc, void* vc,
                                 float* out, int64_t n_head, int64_t n_kv_head, int64_t head_dim, const float* table,
                                 int32_t table_rows, int64_t ctx, const int32_t* pos_dev, void* workspace,
                                 uint64_t* const* peer_out, int64_t peer_off, int peer_world, const uint32_t* ll_count,
                                 uint32_t ll_lo, cudaStream_t s) {
    int* status = nullptr;
    cudaError_t e = status_word(&status);
    if (e != cudaSuccess) return e;
    if (peer_world < 0 || peer_world > kPeerSyncMax || (peer_world > 0 && (!peer_out || !ll_count)))
        return cudaErrorInvalidValue;
    AttnRope ri = {};
    ri.k_new = k_new;
    ri.v_new = v_new;
    ri.kc = static_cast<__half*>(kc);
    ri.vc = static_cast<__half*>(vc);
    ri.table = table;
    ri.table_rows = table_rows;
    ri.status = status;
    ri.peer_world = peer_world;
    ri.peer_off = peer_off;
    for (int p = 0; p < peer_world; ++p) {
        if (!peer_out[p]) return cudaErrorInvalidValue;
        ri.peer_out[p] = peer_out[p];
    }
    ri.ll_count = ll_count;
    ri.ll_lo = ll_lo;
    return attention_any<true>(q, kc, vc, out, n_head, n_kv_head, head_dim, ctx, pos_dev, 0, workspace, ri, s);
}

}  // namespace hesa_cuda
