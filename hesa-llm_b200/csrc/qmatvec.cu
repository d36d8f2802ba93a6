// qmatvec.cu -- streaming GGUF-block matvec on CUDA cores (batch 1) for sm_100a,
// plus the exact dequantizer and a generic per-row kernel for odd shapes.
//
// Streaming kernel (qmv_stream_kernel):
//   * Work is a grid of cells: (row group of 4 rows; 2 for Q8_0) x (unit of 256 weights
//     = one K-quant super-block or eight 32-weight blocks). Every warp of the
//     persistent grid owns a contiguous, equal-sized range of cells in
//     row-group-major order, so HBM traffic is balanced to +-1 cell per warp
//     whatever n_out and k are.
//   * A warp step covers up to 8 consecutive units of one row group. Lane 0
//     copies the step's row segments (contiguous bytes of W) into a
//     private ring of shared-memory stages with cp.async.bulk; the ring runs
//     up to kMaxStages steps ahead of the decode, so the copy engine keeps
//     ~100 KB per SM in flight.
//   * x is staged once per CTA in shared memory as exact integers: per unit
//     of 256 activations, X = rint(x / s) with s a power of two chosen so
//     |X| <= 2^22 (22 bits below the unit's largest magnitude), split into
//     three balanced int8 digits X = 65536*D2 + 256*D1 + D0. The digit planes
//     are permuted per type so lane (unit j, quarter c) reads its 64
//     activations with 12 conflict-free 128-bit loads and keeps them in
//     registers for all rows of the group.
//   * Four lanes share a unit; lane c decodes a quarter (64 weights): quant
//     values are unpacked to bytes with one or two LOP3/shifts per 4 weights
//     and multiplied into the three digit planes with DP4A, an exact int32
//     dot product. Sub-block scales are applied in int32 (sc * sum q*D), the
//     q offsets (-8, -32) through per-group digit sums, and the three planes
//     are combined in fp32 once per unit. The only rounding besides the final
//     fp32 sums is the representation of x: relative L2 error of y below
//     ~1e-6 for any activation distribution (each unit's error is bounded by
//     2^-22 of its own largest |x|).
//   * Row sums are reduced with warp shuffles. A row group split between
//     warps is combined deterministically: every warp writes its partial to
//     the workspace, and the last to arrive (acq_rel counter) adds the
//     partials in warp order and writes y.
#include "hesa_common.cuh"
#include "qtypes.cuh"
#include "qmatvec.h"
#include "xdigits.cuh"
#include "strip_core.cuh"
#include "peer_sync.cuh"

#include <cuda/atomic>

namespace hesa_cuda {

// The library's sticky status word (0 = healthy); kernels get its address.
__device__ int g_hesa_status = 0;

namespace {

using namespace strip;

constexpr int kMaxRows = 4;        // rows per row group (x register reuse factor), Q8_0: 2
constexpr int kUnitsPerStep = 8;   // units per warp step (4 lanes per unit)
constexpr int kMaxStages = 4;
constexpr int kMaxSmem = 227 * 1024;

__host__ __device__ constexpr int slot_bytes(int qt) {
    // one row segment of up to kUnitsPerStep units, plus room for the <16 B
    // alignment offset of its first byte and the 4-byte over-read of the
    // unaligned loads
    return ((kUnitsPerStep * unit_bytes(qt) + 15) / 16) * 16 + 32;
}

__host__ __device__ constexpr int rows_of(int qt) { return qt == kQ8_0 ? 2 : kMaxRows; }

__host__ __device__ constexpr int stage_bytes(int qt) { return rows_of(qt) * slot_bytes(qt); }

// Division-free walk over a warp's cells in row-group-major order: a step
// covers up to kUnitsPerStep units of one row group.
struct Cursor {
    int64_t c;  // next cell
    int g;      // its row group
    int u;      // its unit within the row group
};

__device__ __forceinline__ int step_units(const Cursor& cur, int64_t c_end, int U) {
    int n = U - cur.u;
    if (n > kUnitsPerStep) n = kUnitsPerStep;
    const int64_t left = c_end - cur.c;
    if (left < n) n = static_cast<int>(left);
    return n;
}

__device__ __forceinline__ void advance(Cursor& cur, int n, int U) {
    cur.c += n;
    cur.u += n;
    if (cur.u == U) {
        cur.u = 0;
        ++cur.g;
    }
}

// Warp that owns cell c when C cells are split over W warps as [wC/W, (w+1)C/W).
// With W <= C every warp owns at least one cell.
__device__ __forceinline__ int64_t owner_warp(int64_t c, int64_t C, int64_t W) {
    return ((c + 1) * W - 1) / C;
}

template <int QT>
__global__ void __launch_bounds__(kThreads, 1)
qmv_stream_kernel(const uint8_t* __restrict__ w, int n_out, int k, const float* __restrict__ x,
                  float* __restrict__ y, float scale, int* __restrict__ counters,
                  float* __restrict__ partials, int n_stages, int* __restrict__ status) {
    constexpr int R = rows_of(QT);
    constexpr int UB = unit_bytes(QT);
    constexpr int SLOT = slot_bytes(QT);
    constexpr int STAGE = stage_bytes(QT);
    extern __shared__ __align__(128) uint8_t smem[];

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int U = k >> 8;                                     // units per row
    const int G = (n_out + R - 1) / R;                        // row groups
    const int64_t C = static_cast<int64_t>(G) * U;           // cells
    const int64_t W = static_cast<int64_t>(gridDim.x) * kWarps;
    const int64_t gw = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
    const int64_t c_begin = gw * C / W, c_end = (gw + 1) * C / W;
    const size_t pitch = static_cast<size_t>(U) * UB;
    const size_t total_bytes = pitch * static_cast<size_t>(n_out);
    const size_t total_floor16 = total_bytes & ~size_t(15);

    // shared memory: [x digit planes: U*4*kQPlaneStride][digit sums: U*4*kQSumStride]
    //                [unit scales: U f32][stages][mbarriers]
    uint8_t* xplanes = smem;
    uint8_t* xsums = xplanes + static_cast<size_t>(U) * 4 * kQPlaneStride;
    float* xscale = reinterpret_cast<float*>(xsums + static_cast<size_t>(U) * 4 * kQSumStride);
    uint8_t* stage_base = smem + x_region_bytes(U);
    uint8_t* my_stages = stage_base + static_cast<size_t>(warp) * n_stages * STAGE;
    uint64_t* bars = reinterpret_cast<uint64_t*>(stage_base + static_cast<size_t>(kWarps) * n_stages * STAGE) +
                     warp * kMaxStages;

    if (lane == 0) {
        for (int s = 0; s < n_stages; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncwarp();

    Cursor first;
    first.c = c_begin;
    first.g = static_cast<int>(c_begin / U);
    first.u = static_cast<int>(c_begin - static_cast<int64_t>(first.g) * U);

    // ---- producer (lane 0): copy the R row segments of one step ----
    auto issue = [&](const Cursor& cur, int n, int stage) {
        uint8_t* dst = my_stages + stage * STAGE;
        uint32_t tx = 0;
        const uint8_t* srcs[R];
        uint32_t lens[R];
        const size_t base = static_cast<size_t>(cur.g) * R * pitch + static_cast<size_t>(cur.u) * UB;
#pragma unroll
        for (int r = 0; r < R; ++r) {
            lens[r] = 0;
            srcs[r] = nullptr;
            if (cur.g * R + r >= n_out) continue;
            const size_t start = base + r * pitch;
            const size_t end = start + static_cast<size_t>(n) * UB;
            const size_t a0 = start & ~size_t(15);
            size_t a1 = (end + 15) & ~size_t(15);
            if (a1 > total_floor16) {
                // the last < 16 bytes of W: plain loads, never past the buffer
                a1 = total_floor16 > a0 ? total_floor16 : a0;
                for (size_t b = a1; b < end; ++b) dst[r * SLOT + (b - a0)] = w[b];
            }
            srcs[r] = w + a0;
            lens[r] = static_cast<uint32_t>(a1 - a0);
            tx += lens[r];
        }
        mbar_arrive_expect_tx(&bars[stage], tx);
#pragma unroll
        for (int r = 0; r < R; ++r)
            if (lens[r]) bulk_g2s(dst + r * SLOT, srcs[r], lens[r], &bars[stage]);
    };

    // Prime the ring before staging x so the copies overlap the staging.
    Cursor prod = first;
    int prod_step = 0;
    if (lane == 0) {
        while (prod_step < n_stages && prod.c < c_end) {
            const int n = step_units(prod, c_end, U);
            issue(prod, n, prod_step);
            advance(prod, n, U);
            ++prod_step;
        }
    }

    // ---- stage x: per unit of 256 activations, X = rint(x / s) with s a power
    // of two chosen so |X| <= 2^22, split into three balanced int8 digits
    // (X = 65536*D2 + 256*D1 + D0) stored as permuted digit planes, plus the
    // per-group digit sums the bias corrections use. One warp per unit; the
    // loads of a batch of units are issued together.
    constexpr int kBatch = 4;
    for (int ub = warp; ub < U; ub += kWarps * kBatch) {
        float v[kBatch][8];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int unit = ub + j * kWarps;
            if (unit < U) {
                const float4* xp = reinterpret_cast<const float4*>(x + static_cast<size_t>(unit) * 256 + lane * 8);
                const float4 va = xp[0], vb = xp[1];
                v[j][0] = va.x; v[j][1] = va.y; v[j][2] = va.z; v[j][3] = va.w;
                v[j][4] = vb.x; v[j][5] = vb.y; v[j][6] = vb.z; v[j][7] = vb.w;
            }
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int unit = ub + j * kWarps;
            if (unit < U) stage_unit<QT>(unit, lane, v[j], xplanes, xsums, xscale);
        }
    }
    __syncthreads();

    // ---- consumer: all lanes ----
    const int ju = lane >> 2;   // unit within the step
    const int qc = lane & 3;    // quarter within the unit
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;

    bool failed = false;
    Cursor cons = first;
    int cons_step = 0;
    while (cons.c < c_end) {
        const int n = step_units(cons, c_end, U);
        const int g = cons.g, u0 = cons.u;
        const int stage = cons_step % n_stages;
        const uint32_t parity = static_cast<uint32_t>(cons_step / n_stages) & 1u;
        // every lane waits; the warp leaves together if any lane gave up
        const bool landed = mbar_wait_bounded(&bars[stage], parity, status, kStatusWaitTimeout);
        if (!__all_sync(0xffffffffu, landed)) {
            failed = true;
            break;
        }
        const uint8_t* st = my_stages + stage * STAGE;
        if (ju < n) {
            const int unit = u0 + ju;
            // this lane's activations, kept in registers for the R rows
            XQuarter xq;
            load_xquarter<QT>(xplanes, xsums, xscale, unit, qc, xq);
            const size_t base = static_cast<size_t>(g) * R * pitch + static_cast<size_t>(u0) * UB;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (g * R + r < n_out) {
                    const size_t start = base + r * pitch;
                    const uint8_t* up = st + r * SLOT + (start & 15) + ju * UB;
                    acc[r] += unit_dot<QT>(up, qc, xq);
                }
            }
        }
        __syncwarp();
        advance(cons, n, U);
        ++cons_step;

        // refill this stage with the step n_stages ahead
        if (lane == 0 && prod.c < c_end) {
            fence_proxy_async_smem();
            const int n2 = step_units(prod, c_end, U);
            issue(prod, n2, stage);
            advance(prod, n2, U);
            ++prod_step;
        }

        // flush the row group when the walk leaves it (or the range ends)
        if (cons.c >= c_end || cons.u == 0) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
            }
            const int64_t g_first = static_cast<int64_t>(g) * U;
            const int64_t g_last = g_first + U;   // exclusive
            if (lane == 0) {
                if (g_first >= c_begin && g_last <= c_end) {
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const int row = g * R + r;
                        if (row < n_out) y[row] = acc[r] * scale;
                    }
                } else {
                    // split group: partial -> workspace, last arrival sums in warp order
                    const int slot = (g_first <= c_begin) ? 0 : 1;   // head group : tail group
                    float* mine = partials + (gw * 2 + slot) * kMaxRows;
#pragma unroll
                    for (int r = 0; r < R; ++r) mine[r] = acc[r];
                    const int64_t w_first = owner_warp(g_first, C, W);
                    const int64_t w_last = owner_warp(g_last - 1, C, W);
                    const int n_parts = static_cast<int>(w_last - w_first + 1);
                    cuda::atomic_ref<int, cuda::thread_scope_device> cnt(counters[g]);
                    const int prev = cnt.fetch_add(1, cuda::memory_order_acq_rel);
                    if (prev == n_parts - 1) {
                        float tot[R];
#pragma unroll
                        for (int r = 0; r < R; ++r) tot[r] = 0.f;
                        for (int64_t ow = w_first; ow <= w_last; ++ow) {
                            const int64_t oc0 = ow * C / W;
                            const int oslot = (ow == w_first && oc0 / U != g) ? 1 : 0;
                            const float* pp = partials + (ow * 2 + oslot) * kMaxRows;
#pragma unroll
                            for (int r = 0; r < R; ++r) tot[r] += pp[r];
                        }
#pragma unroll
                        for (int r = 0; r < R; ++r) {
                            const int row = g * R + r;
                            if (row < n_out) y[row] = tot[r] * scale;
                        }
                        cnt.store(0, cuda::memory_order_relaxed);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r] = 0.f;
        }
    }

    if (failed && lane == 0) {
        // drain: wait (bounded) for every copy this warp still has in flight
        for (int s = cons_step; s < prod_step; ++s) {
            if (!mbar_wait_bounded(&bars[s % n_stages], static_cast<uint32_t>(s / n_stages) & 1u, status,
                                   kStatusDrainTimeout))
                break;
        }
    }
}

// ---------------------------------------------------------------------------
// Row-strip kernel (qmv_strip_kernel): the batch-1 path for k <= 24576.
//
//   * CTA b owns the contiguous rows [b*n_out/G, (b+1)*n_out/G) (balanced to
//     one row). Its bytes are one contiguous range of W, streamed as chunks of
//     chunk_rows whole rows, one cp.async.bulk per chunk, into a ring of up to
//     kStripMaxSlots shared-memory slots; most of the range is in flight
//     from the first microsecond.
//   * x is converted to digit planes once per CTA (one warp per unit of 256)
//     while the first copies are in flight.
//   * Lane (slice s, quarter-column q) owns 64 weights of every row r with
//     r = s (mod slices): unit q/4, quarter q%4. It loads that quarter of x
//     once and keeps it in registers for all its rows. Whole warps belong to
//     one slice; its quarter-columns are spread evenly over them.
//   * Per row, a warp's lanes are reduced with shuffles and lane 0 stores
//     the warp's partial in shared memory; at the end the CTA adds the warps'
//     partials of each row in a fixed order. No workspace, deterministic.
//   * A chunk's slot is refilled by the last warp to finish it (shared
//     counter), so no thread waits on the producer side.
// ---------------------------------------------------------------------------

constexpr int kStripMaxSlots = 16;

constexpr int kStripSmemMax = 226 * 1024;

// Where a strip kernel's rows go: the plain local y, every rank's gathered
// buffer (PeerOut), or every rank as tagged words (LLOut). Each destination,
// and a tagged input (LLX), is its own instantiation, so the plain matvec
// carries none of the others' code or registers.
enum : int { kOutPlain = 0, kOutPeer = 1, kOutTagged = 2 };

template <int QT, bool LLX, int OUT>
__global__ void __launch_bounds__(kThreads, 1)
qmv_strip_kernel(const uint8_t* __restrict__ w, int n_out, int k, const float* __restrict__ x,
                 float* __restrict__ y, float scale, int chunk_rows, int n_slots, int slot_stride, int rows_cap,
                 int xmode, const float* __restrict__ norm_w, float eps, const float* __restrict__ resid,
                 PeerOut peer, LLIn lin, LLOut lout, int* __restrict__ status) {
    constexpr int UB = unit_bytes(QT);
    extern __shared__ __align__(128) uint8_t smem[];

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int U = k >> 8;
    const int QC = 4 * U;                      // quarter-columns
    const int wps = (QC + 31) >> 5;            // warps per row slice
    const int RS = kWarps / wps;               // row slices (host: wps <= kWarps)
    const int active_warps = RS * wps;
    const int slice = warp / wps;
    const int wq = warp - slice * wps;         // warp index inside its slice
    // quarter-columns spread evenly over the slice's warps (e.g. 172 as 5 x 29
    // + 27, not 5 x 32 + 12), so no scheduler partition gets more than its
    // share of the decode
    const int lpw = (QC + wps - 1) / wps;
    const int q = wq * lpw + lane;
    const bool wactive = slice < RS;
    const bool qactive = wactive && lane < lpw && q < QC;
    const int unit = q >> 2, qc = q & 3;
    const int r0 = static_cast<int>(static_cast<int64_t>(blockIdx.x) * n_out / gridDim.x);
    const int r1 = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * n_out / gridDim.x);
    const int nrows = r1 - r0;
    const size_t pitch = static_cast<size_t>(U) * UB;
    const size_t total_floor16 = (pitch * static_cast<size_t>(n_out)) & ~size_t(15);
    const int CR = chunk_rows;                 // multiple of RS
    const int n_chunks = (nrows + CR - 1) / CR;

    // shared memory: [x digit planes, sums, scales (x_region_bytes)][slots]
    //                [partials: rows_cap x wps f32][full mbarriers][done counters][issued]
    uint8_t* xplanes = smem;
    uint8_t* xsums = xplanes + static_cast<size_t>(U) * 4 * kQPlaneStride;
    float* xscale = reinterpret_cast<float*>(xsums + static_cast<size_t>(U) * 4 * kQSumStride);
    uint8_t* slots = smem + x_region_bytes(U);
    float* part = reinterpret_cast<float*>(slots + static_cast<size_t>(n_slots) * slot_stride);
    uint64_t* full = reinterpret_cast<uint64_t*>(
        reinterpret_cast<uint8_t*>(part) + ((static_cast<size_t>(rows_cap) * wps * 4 + 15) & ~size_t(15)));
    int* done = reinterpret_cast<int*>(full + kStripMaxSlots);
    int* issued = done + kStripMaxSlots;
    float* red = reinterpret_cast<float*>(issued + kStripMaxSlots);   // kWarps floats

    // set once a wait for a tagged input of this CTA ran out (later waits
    // then take what they read)
    __shared__ int s_ll_failed;
    if (threadIdx.x == 0) {
        for (int s = 0; s < n_slots; ++s) {
            mbar_init(&full[s], 1);
            done[s] = 0;
            issued[s] = -1;
        }
        s_ll_failed = 0;
        fence_mbar_init();
    }
    __syncthreads();

    // copy chunk j (rows [j*CR, j*CR + CR) of this CTA) into its slot
    auto issue = [&](int j) {
        const int slot = j % n_slots;
        const int lr0 = j * CR;
        const int lr1 = min(nrows, lr0 + CR);
        const size_t start = static_cast<size_t>(r0 + lr0) * pitch;
        const size_t end = static_cast<size_t>(r0 + lr1) * pitch;
        const size_t a0 = start & ~size_t(15);
        size_t a1 = (end + 15) & ~size_t(15);
        uint8_t* dst = slots + static_cast<size_t>(slot) * slot_stride;
        if (a1 > total_floor16) {
            // the last < 16 bytes of W: plain loads, never past the buffer
            a1 = total_floor16 > a0 ? total_floor16 : a0;
            for (size_t b = a1; b < end; ++b) dst[b - a0] = w[b];
        }
        issued[slot] = j;
        mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(a1 - a0));
        // each weight byte is read once: evict-first in L2 (sweep 3,010 -> 3,080 GB/s)
        if (a1 > a0)
            bulk_g2s_policy(dst, w + a0, static_cast<uint32_t>(a1 - a0), &full[slot], l2_policy_evict_first());
    };

    // The weights never come from the previous kernel on the stream, so the
    // first chunk is fetched before waiting for it; x may, so it is read
    // after. The other slots are filled once x is staged: a flood of incoming
    // copies during the staging slows the staging more than it gains
    // (measured: 9.25 vs 10.45 us for a 4096x11008 Q4_K launch).
    if (threadIdx.x == 0) issue(0);
    // Tagged inputs too: a kernel that started spinning on them before the
    // previous grid completed held the sharded 7B step 2.06 against 1.80 ms
    // per token on two GPUs (its polling competes with the producer)
    grid_dep_wait();
    // tagged inputs (sharded decode step): the tags of this token
    // (the counts are read here, not where the tags are needed, so that the
    // epilogue does not start with a round trip to L2)
    uint32_t x_tag = 0, rtag = 0, out_tag = 0;
    if constexpr (LLX) {
        x_tag = ll_tag(lin.count, lin.x_lo);
        rtag = (x_tag & ~0xFFFu) | lin.resid_lo;
    }
    if constexpr (OUT == kOutTagged) out_tag = ll_tag(lout.count, lout.lo);
    // The tagged epilogue walks the words of this CTA's rows in word order
    // (consecutive threads, consecutive words: whole lines over NVLink) --
    // rows [ra, rb) of the shard are elements voff + ra .. of the output.
    // The residual word of this thread's first row is read now (it arrived
    // with the input of an earlier kernel) and checked in the epilogue.
    uint64_t resid_w = 0;
    if constexpr (LLX && OUT == kOutTagged) {
        if (lin.resid) {
            const int64_t A = lout.off + r0, B = lout.off + r1;
            const int64_t e = ll_elem((A & ~int64_t(255)) + threadIdx.x);
            if (e >= A && e < B) resid_w = ld_ll(lin.resid + ll_pos(lin.resid_off + (e - lout.off)));
        }
    }

    // x as digit planes, converted once per CTA (one warp per unit of 256;
    // the loads of a batch of units are issued together). The input may be
    // transformed on the way (decode-step fusions): RMSNorm, x * inv_rms * w
    // with inv_rms = 1 / sqrt(mean(x^2) + eps) (every unit in one batch: the
    // host keeps U <= kWarps * kStripBatch), or SwiGLU, silu(x[i]) * x[k + i].
    if (xmode == kXRmsNorm) {
        float v[kStripBatch][8];
        float ss = 0.f;
        if constexpr (LLX) {
            load8_ll_batch(lin.x, x_tag, lin.limit_ns, warp, lane, U, v, status, &s_ll_failed);
#pragma unroll
            for (int jb = 0; jb < kStripBatch; ++jb)
#pragma unroll
                for (int j = 0; j < 8; ++j) ss = fmaf(v[jb][j], v[jb][j], ss);
        } else {
#pragma unroll
            for (int jb = 0; jb < kStripBatch; ++jb) {
                load8(x, warp + jb * kWarps, lane, U, v[jb]);
#pragma unroll
                for (int j = 0; j < 8; ++j) ss = fmaf(v[jb][j], v[jb][j], ss);
            }
        }
        ss = warp_sum_f(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w8 = 0; w8 < kWarps; ++w8) tot += red[w8];
        const float inv = 1.0f / sqrtf(tot / static_cast<float>(k) + eps);
#pragma unroll
        for (int jb = 0; jb < kStripBatch; ++jb) {
            const int u = warp + jb * kWarps;
            if (u < U) {
                float wn[8];
                load8(norm_w, u, lane, U, wn);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[jb][j] = __fmul_rn(__fmul_rn(v[jb][j], inv), wn[j]);
                stage_unit<QT>(u, lane, v[jb], xplanes, xsums, xscale);
            }
        }
    } else {
        for (int ub = warp; ub < U; ub += kWarps * kStripBatch) {
            float v[kStripBatch][8];
            if constexpr (LLX) {
                if (xmode == kXSiluMul)
                    load8_ll_swiglu(lin.x, k, x_tag, lin.limit_ns, ub, lane, U, v, status, &s_ll_failed);
                else
                    load8_ll_batch(lin.x, x_tag, lin.limit_ns, ub, lane, U, v, status, &s_ll_failed);
            } else {
#pragma unroll
                for (int jb = 0; jb < kStripBatch; ++jb) {
                    const int u = ub + jb * kWarps;
                    load8(x, u, lane, U, v[jb]);
                    if (xmode == kXSiluMul && u < U) {
                        float up[8];
                        load8(x + k, u, lane, U, up);
#pragma unroll
                        for (int j = 0; j < 8; ++j) v[jb][j] = swiglu_x(v[jb][j], up[j]);
                    }
                }
            }
#pragma unroll
            for (int jb = 0; jb < kStripBatch; ++jb) {
                const int u = ub + jb * kWarps;
                if (u < U) stage_unit<QT>(u, lane, v[jb], xplanes, xsums, xscale);
            }
        }
    }
    if (threadIdx.x == 0)
        for (int j = 1; j < n_slots && j < n_chunks; ++j) issue(j);
    __syncthreads();

    // this lane's quarter of x, in registers for every row it processes
    XQuarter xq;
    if (qactive) load_xquarter<QT>(xplanes, xsums, xscale, unit, qc, xq);

    // The next kernel on the stream may start its CTAs once every CTA here has
    // issued its last copy (measured: 94.5 vs 97.1 us per sweep step of eight
    // matvecs against a trigger at the start).
    bool triggered = false;
    const int trigger_chunk = n_chunks > n_slots ? n_chunks - n_slots : 0;
    bool failed = false;
    if (wactive) {
        for (int j = 0; j < n_chunks; ++j) {
            if (j == trigger_chunk) {
                grid_dep_launch();
                triggered = true;
            }
            const int slot = j % n_slots;
            const uint32_t parity = static_cast<uint32_t>(j / n_slots) & 1u;
            const bool landed = mbar_wait_bounded(&full[slot], parity, status, kStatusWaitTimeout);
            if (!__all_sync(0xffffffffu, landed)) {
                failed = true;
                break;
            }
            const int lr0 = j * CR;
            const int lr1 = min(nrows, lr0 + CR);
            const uint8_t* base = slots + static_cast<size_t>(slot) * slot_stride +
                                  ((static_cast<size_t>(r0 + lr0) * pitch) & 15) + static_cast<size_t>(unit) * UB;
            // this slice's rows of the chunk, GR at a time: independent
            // decode chains, then one transposing reduction for the group.
            // The row count of a group is warp-uniform; each count has its
            // own code so no decode is issued for a missing row.
            constexpr int GR = strip_group_rows(QT);
            for (int i0 = lr0 + slice; i0 < lr1; i0 += GR * RS) {
                float a[4] = {0.f, 0.f, 0.f, 0.f};
                const uint8_t* rb = base + static_cast<size_t>(i0 - lr0) * pitch;
                const size_t rstep = static_cast<size_t>(RS) * pitch;
                const int nv = (lr1 - i0 + RS - 1) / RS;
                if (qactive) {
                    if (nv >= GR) strip_rows<QT, GR>(rb, rstep, qc, xq, a);
                    else if (nv == 3) strip_rows<QT, 3>(rb, rstep, qc, xq, a);
                    else if (nv == 2) strip_rows<QT, 2>(rb, rstep, qc, xq, a);
                    else strip_rows<QT, 1>(rb, rstep, qc, xq, a);
                }
                const int rr = reduce4_row(lane);
                const int row = i0 + RS * rr;
                const float tot = reduce4(a, lane);
                if ((lane & 7) == 0 && rr < GR && row < lr1) part[row * wps + wq] = tot;
            }
            __syncwarp();
            if (lane == 0) {
                // the last warp out of the chunk refills its slot
                if (atomicAdd(&done[slot], 1) == active_warps - 1) {
                    done[slot] = 0;
                    if (j + n_slots < n_chunks) {
                        fence_proxy_async_smem();
                        issue(j + n_slots);
                    }
                }
            }
        }
    }
    if (!triggered) grid_dep_launch();
    failed = __syncthreads_or(failed);
    if (failed) {
        // drain: wait (bounded) for the copy last issued into every slot
        if (threadIdx.x == 0) {
            for (int s = 0; s < n_slots; ++s) {
                const int j = issued[s];
                if (j >= 0 && !mbar_wait_bounded(&full[s], static_cast<uint32_t>(j / n_slots) & 1u, status,
                                                 kStatusDrainTimeout))
                    break;
            }
        }
        return;
    }
    if constexpr (OUT == kOutTagged) {
        // every row to every rank, tagged with this step's place (sharded
        // decode step, tagged gather)
        const uint32_t tag = out_tag;
        const bool odd = lout.by_parity && ((tag >> 12) & 1u);
        auto emit = [&](int ra, int rb, int64_t voff, uint64_t* const* bufs) {
            if (ra >= rb) return;
            const int64_t A = voff + ra, B = voff + rb;
            const int64_t w1 = (B + 255) & ~int64_t(255);
            bool first = true;
            for (int64_t w = (A & ~int64_t(255)) + threadIdx.x; w < w1; w += blockDim.x, first = false) {
                const int64_t e = ll_elem(w);
                if (e < A || e >= B) continue;
                const int row = static_cast<int>(e - voff), i = row - r0;
                float s = 0.f;
                for (int t = 0; t < wps; ++t) s += part[i * wps + t];
                float val = s * scale;
                if constexpr (LLX) {
                    if (lin.resid) {
                        const uint64_t* rp = lin.resid + ll_pos(lin.resid_off + row);
                        const float rv = first ? ll_value(rp, resid_w, rtag, lin.limit_ns, status, &s_ll_failed)
                                               : ld_ll_wait(rp, rtag, lin.limit_ns, status, &s_ll_failed);
                        val = __fadd_rn(rv, val);
                    }
                }
                for (int p = 0; p < lout.world; ++p) st_ll(bufs[p] + w, val, tag);
            }
        };
        if (lout.by_parity) {
            emit(r0, r1, lout.off, odd ? lout.y2 : lout.y);
        } else {
            emit(r0, min(r1, lout.split), lout.off, lout.y);
            emit(max(r0, lout.split), r1, lout.off2 - lout.split, lout.y2);
        }
    } else if constexpr (OUT == kOutPlain) {
        for (int i = threadIdx.x; i < nrows; i += blockDim.x) {
            float s = 0.f;
            for (int t = 0; t < wps; ++t) s += part[i * wps + t];
            const float val = s * scale;
            y[r0 + i] = resid ? __fadd_rn(resid[r0 + i], val) : val;   // residual add, rounded as a separate add
        }
    } else {
        // fused all-gather: every rank's buffer of this step's parity gets the
        // rows (peer stores over NVLink). No fence here: the stores are
        // performed when this grid completes, and the barrier kernel that
        // publishes the step is launched without programmatic serialization,
        // so it starts only after that (a system-scope fence in every thread
        // held each launch about 7 us longer)
        const int par = static_cast<int>(*peer.epoch & 1u);
        for (int i = threadIdx.x; i < nrows; i += blockDim.x) {
            float s = 0.f;
            for (int t = 0; t < wps; ++t) s += part[i * wps + t];
            const float val = s * scale;
            for (int p = 0; p < peer.world; ++p) peer.y[par][p][r0 + i] = val;
        }
    }
}

// Generic kernel for shapes the streaming kernel does not take (k not a
// multiple of 256, W not 16-byte aligned, tiny matrices): one warp per row,
// exact per-weight decode from global memory, fp32 FMA, shuffle reduction.
template <int QT>
__global__ void __launch_bounds__(256)
qmv_rowwise_kernel(const uint8_t* __restrict__ w, int n_out, int k, const float* __restrict__ x,
                   int64_t ldx, int batch, float* __restrict__ y, int64_t ldy, float scale) {
    constexpr int BE = block_elems(QT), BB = block_bytes(QT);
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
    if (row >= n_out) return;
    const uint8_t* wr = w + row * static_cast<int64_t>(k / BE) * BB;
    for (int b = 0; b < batch; ++b) {
        const float* xb = x + b * ldx;
        float acc = 0.f;
        for (int i = lane; i < k; i += 32) acc = fmaf(deq_weight<QT>(wr + (i / BE) * BB, i % BE), xb[i], acc);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) y[b * ldy + row] = acc * scale;
    }
}

template <int QT>
__global__ void __launch_bounds__(256)
dequant_kernel(const uint8_t* __restrict__ w, int64_t n_rows, int64_t k, float* __restrict__ out, int64_t ldo) {
    constexpr int BE = block_elems(QT), BB = block_bytes(QT);
    const int64_t total = n_rows * k;
    const int64_t nb = k / BE;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = e / k, i = e - r * k;
        const uint8_t* blk = w + (r * nb + i / BE) * BB;
        out[r * ldo + i] = deq_weight<QT>(blk, static_cast<int>(i % BE));
    }
}

int g_num_sms[64] = {0};
int* g_status_ptr[64] = {nullptr};

int device_sms() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (dev < 0 || dev >= 64) return 148;
    if (g_num_sms[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        g_num_sms[dev] = n;
    }
    return g_num_sms[dev];
}

// Device address of g_hesa_status for the current device (looked up once).
cudaError_t status_ptr(int** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!g_status_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_hesa_status);
        if (e != cudaSuccess) return e;
        g_status_ptr[dev] = static_cast<int*>(p);
    }
    *out = g_status_ptr[dev];
    return cudaSuccess;
}

template <int QT>
cudaError_t launch_stream(const uint8_t* w, int n_out, int k, const float* x, float* y, float scale,
                          int* counters, float* partials, int grid, cudaStream_t stream) {
    const int U = k >> 8;
    const size_t x_bytes = x_region_bytes(U);
    const size_t per_stage = static_cast<size_t>(kWarps) * stage_bytes(QT);
    const size_t bar_bytes = static_cast<size_t>(kWarps) * kMaxStages * 8;
    if (x_bytes + per_stage + bar_bytes > static_cast<size_t>(kMaxSmem)) return cudaErrorInvalidValue;
    int n_stages = static_cast<int>((kMaxSmem - x_bytes - bar_bytes) / per_stage);
    if (n_stages > kMaxStages) n_stages = kMaxStages;
    const size_t smem = x_bytes + n_stages * per_stage + bar_bytes;
    // raise the kernel's dynamic shared-memory limit once per device
    static int smem_set[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (smem_set[dev] < kMaxSmem) {
        e = cudaFuncSetAttribute(qmv_stream_kernel<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
        if (e != cudaSuccess) return e;
        smem_set[dev] = kMaxSmem;
    }
    int* status = nullptr;
    e = status_ptr(&status);
    if (e != cudaSuccess) return e;
    qmv_stream_kernel<QT><<<grid, kThreads, smem, stream>>>(w, n_out, k, x, y, scale, counters, partials,
                                                            n_stages, status);
    return cudaGetLastError();
}

struct StripPlan {
    int grid = 0, chunk_rows = 0, n_slots = 0, slot_stride = 0, rows_cap = 0;
    size_t smem = 0;
};

// Launch geometry of the row-strip kernel: one CTA per SM (at most one per
// row), chunks of up to four rows per row slice (at most 56 KB), and as many
// ring slots as shared memory holds (no more than the CTA has chunks).
bool plan_strip(int qt, int64_t n_out, int64_t k, StripPlan& p) {
    if (!qtype_supported(qt) || k % 256 != 0 || n_out < 1) return false;
    const int U = static_cast<int>(k >> 8);
    const int wps = (4 * U + 31) / 32;
    if (wps > kWarps) return false;
    const int RS = kWarps / wps;
    const size_t pitch = static_cast<size_t>(U) * unit_bytes(qt);
    int64_t grid = device_sms();
    if (grid > n_out) grid = n_out;
    p.grid = static_cast<int>(grid);
    p.rows_cap = static_cast<int>((n_out + grid - 1) / grid);
    const size_t part_bytes = (static_cast<size_t>(p.rows_cap) * wps * 4 + 15) & ~size_t(15);
    const size_t ctrl = kStripMaxSlots * (8 + 4 + 4) + 64;   // + the RMSNorm reduction scratch
    const size_t fixed = x_region_bytes(U) + part_bytes + ctrl;
    if (fixed >= static_cast<size_t>(kStripSmemMax)) return false;
    const size_t budget = kStripSmemMax - fixed;
    // rows per slice per chunk: 4 (one 4-row group) when a chunk stays within
    // 56 KB, else fewer
    int m = static_cast<int>(57344 / (static_cast<size_t>(RS) * pitch));
    if (m > 4) m = 4;
    if (m < 1) m = 1;
    const int max_m = (p.rows_cap + RS - 1) / RS;
    if (m > max_m) m = max_m;
    for (; m >= 1; --m) {
        const int CR = RS * m;
        const size_t stride = ((static_cast<size_t>(CR) * pitch + 15) & ~size_t(15)) + 32;
        const int n_chunks = (p.rows_cap + CR - 1) / CR;
        int slots = static_cast<int>(budget / stride);
        if (slots > kStripMaxSlots) slots = kStripMaxSlots;
        if (slots > n_chunks) slots = n_chunks;
        if (slots >= 2 || (slots == 1 && n_chunks == 1)) {
            p.chunk_rows = CR;
            p.n_slots = slots;
            p.slot_stride = static_cast<int>(stride);
            p.smem = x_region_bytes(U) + slots * stride + part_bytes + ctrl;
            return true;
        }
    }
    return false;
}

template <int QT, bool LLX, int OUT>
cudaError_t launch_strip(const uint8_t* w, int n_out, int k, const float* x, float* y, float scale,
                         const StripPlan& p, int xmode, const float* norm_w, float eps, const float* resid,
                         const PeerOut& peer, const LLIn& lin, const LLOut& lout, cudaStream_t stream) {
    static int smem_set[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (smem_set[dev] < kStripSmemMax) {
        // the plan's budget (the kernel's few bytes of static shared memory
        // come on top, within the 227 KB a CTA may have)
        e = cudaFuncSetAttribute(qmv_strip_kernel<QT, LLX, OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kStripSmemMax);
        if (e != cudaSuccess) return e;
        smem_set[dev] = kStripSmemMax;
    }
    int* status = nullptr;
    e = status_ptr(&status);
    if (e != cudaSuccess) return e;
    // programmatic stream serialization: the CTAs may start while the previous
    // kernel on the stream finishes; the kernel waits for it before reading x
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, qmv_strip_kernel<QT, LLX, OUT>, w, n_out, k, x, y, scale, p.chunk_rows, p.n_slots,
                              p.slot_stride, p.rows_cap, xmode, norm_w, eps, resid, peer, lin, lout, status);
}

// launch_strip for a runtime quant type
template <bool LLX, int OUT>
cudaError_t launch_strip_qt(int qtype, const uint8_t* w, int n_out, int k, const float* x, float* y, float scale,
                            const StripPlan& p, int xmode, const float* norm_w, float eps, const float* resid,
                            const PeerOut& peer, const LLIn& lin, const LLOut& lout, cudaStream_t stream) {
    switch (qtype) {
        case kQ4_0: return launch_strip<kQ4_0, LLX, OUT>(w, n_out, k, x, y, scale, p, xmode, norm_w, eps, resid, peer, lin, lout, stream);
        case kQ8_0: return launch_strip<kQ8_0, LLX, OUT>(w, n_out, k, x, y, scale, p, xmode, norm_w, eps, resid, peer, lin, lout, stream);
        case kQ4_K: return launch_strip<kQ4_K, LLX, OUT>(w, n_out, k, x, y, scale, p, xmode, norm_w, eps, resid, peer, lin, lout, stream);
        case kQ5_K: return launch_strip<kQ5_K, LLX, OUT>(w, n_out, k, x, y, scale, p, xmode, norm_w, eps, resid, peer, lin, lout, stream);
        case kQ6_K: return launch_strip<kQ6_K, LLX, OUT>(w, n_out, k, x, y, scale, p, xmode, norm_w, eps, resid, peer, lin, lout, stream);
        default: return cudaErrorInvalidValue;
    }
}

template <int QT>
cudaError_t launch_rowwise(const uint8_t* w, int n_out, int k, const float* x, int64_t ldx, int batch, float* y,
                           int64_t ldy, float scale, cudaStream_t stream) {
    const int grid = (n_out + 7) / 8;
    qmv_rowwise_kernel<QT><<<grid, 256, 0, stream>>>(w, n_out, k, x, ldx, batch, y, ldy, scale);
    return cudaGetLastError();
}

template <int QT>
cudaError_t launch_dequant(const uint8_t* w, int64_t n_rows, int64_t k, float* out, int64_t ldo,
                           cudaStream_t stream) {
    const int64_t total = n_rows * k;
    int64_t blocks = (total + 255) / 256;
    const int64_t cap = static_cast<int64_t>(device_sms()) * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    dequant_kernel<QT><<<static_cast<int>(blocks), 256, 0, stream>>>(w, n_rows, k, out, ldo);
    return cudaGetLastError();
}

}  // namespace

// ---------------------------------------------------------------------------
// host entry points (called by the C ABI)
// ---------------------------------------------------------------------------

size_t qmv_workspace_bytes(int n_out) {
    // counters for the largest number of row groups (2-row groups of Q8_0)
    const size_t groups = (static_cast<size_t>(n_out) + 1) / 2;
    const size_t counters = ((groups * sizeof(int)) + 255) & ~size_t(255);
    const size_t partials = static_cast<size_t>(kMaxGridCtas) * kWarps * 2 * kMaxRows * sizeof(float);
    return counters + partials;
}

static int64_t stream_cells(int qtype, int64_t n_out, int64_t k) {
    const int R = rows_of(qtype);
    return ((n_out + R - 1) / R) * (k / 256);
}

bool qmv_stream_eligible(int qtype, const void* w, int64_t n_out, int64_t k) {
    // every warp of the grid must own at least one cell (the split-group
    // combine counts every warp between the first and the last owner)
    return (k % 256 == 0) && (reinterpret_cast<uintptr_t>(w) % 16 == 0) &&
           stream_cells(qtype, n_out, k) >= kWarps && k <= 32768 && n_out < (int64_t(1) << 30);
}

int qmv_stream_grid(int qtype, int64_t n_out, int64_t k) {
    const int64_t cells = stream_cells(qtype, n_out, k);
    // at least ~4 cells per warp so the per-step overhead amortises, and never
    // more warps than cells
    int64_t grid = device_sms();
    const int64_t want = (cells + 4 * kWarps - 1) / (4 * kWarps);
    if (want < grid) grid = want;
    if (grid * kWarps > cells) grid = cells / kWarps;
    if (grid < 1) grid = 1;
    if (grid > kMaxGridCtas) grid = kMaxGridCtas;
    return static_cast<int>(grid);
}

cudaError_t qmv_stream(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, float* y,
                       float scale, void* workspace, cudaStream_t stream, int grid_override) {
    if (!qtype_supported(qtype)) return cudaErrorInvalidValue;
    const int R = rows_of(qtype);
    const size_t groups = (static_cast<size_t>(n_out) + R - 1) / R;
    int* counters = static_cast<int*>(workspace);
    float* partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                               (((groups * sizeof(int)) + 255) & ~size_t(255)));
    int grid = grid_override > 0 ? grid_override : qmv_stream_grid(qtype, n_out, k);
    const int64_t cells = stream_cells(qtype, n_out, k);
    if (static_cast<int64_t>(grid) * kWarps > cells) grid = static_cast<int>(cells / kWarps);
    if (grid < 1 || grid > kMaxGridCtas) return cudaErrorInvalidValue;
    const uint8_t* wb = static_cast<const uint8_t*>(w);
    const int n = static_cast<int>(n_out), kk = static_cast<int>(k);
    switch (qtype) {
        case kQ4_0: return launch_stream<kQ4_0>(wb, n, kk, x, y, scale, counters, partials, grid, stream);
        case kQ8_0: return launch_stream<kQ8_0>(wb, n, kk, x, y, scale, counters, partials, grid, stream);
        case kQ4_K: return launch_stream<kQ4_K>(wb, n, kk, x, y, scale, counters, partials, grid, stream);
        case kQ5_K: return launch_stream<kQ5_K>(wb, n, kk, x, y, scale, counters, partials, grid, stream);
        case kQ6_K: return launch_stream<kQ6_K>(wb, n, kk, x, y, scale, counters, partials, grid, stream);
        default: return cudaErrorInvalidValue;
    }
}

bool qmv_strip_shape_ok(int qtype, int64_t n_out, int64_t k) {
    StripPlan p;
    return n_out < (int64_t(1) << 30) && plan_strip(qtype, n_out, k, p);
}

bool qmv_strip_eligible(int qtype, const void* w, int64_t n_out, int64_t k) {
    return (reinterpret_cast<uintptr_t>(w) % 16 == 0) && qmv_strip_shape_ok(qtype, n_out, k);
}

cudaError_t qmv_strip(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, float* y, float scale,
                      cudaStream_t stream) {
    return qmv_strip_fused(qtype, w, n_out, k, x, StripInput::kPlain, nullptr, 0.f, y, nullptr, scale, stream);
}

bool qmv_strip_fused_eligible(int qtype, const void* w, int64_t n_out, int64_t k, StripInput in) {
    if (!qmv_strip_eligible(qtype, w, n_out, k)) return false;
    return in != StripInput::kRmsNorm || k <= static_cast<int64_t>(kWarps) * kStripBatch * 256;
}

cudaError_t qmv_strip_fused(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, StripInput in,
                            const float* norm_w, float eps, float* y, const float* resid, float scale,
                            cudaStream_t stream) {
    StripPlan p;
    if (!plan_strip(qtype, n_out, k, p)) return cudaErrorInvalidValue;
    if (in == StripInput::kRmsNorm && (!norm_w || k > static_cast<int64_t>(kWarps) * kStripBatch * 256))
        return cudaErrorInvalidValue;
    const int xm = in == StripInput::kRmsNorm ? kXRmsNorm : in == StripInput::kSiluMul ? kXSiluMul : kXPlain;
    const uint8_t* wb = static_cast<const uint8_t*>(w);
    const int n = static_cast<int>(n_out), kk = static_cast<int>(k);
    return launch_strip_qt<false, kOutPlain>(qtype, wb, n, kk, x, y, scale, p, xm, norm_w, eps, resid, PeerOut{},
                                             LLIn{}, LLOut{}, stream);
}

cudaError_t qmv_strip_gather(int qtype, const void* w, int64_t n_rows, int64_t k, const float* x, float scale,
                             const PeerOut& out_in, cudaStream_t stream) {
    StripPlan p;
    if (!plan_strip(qtype, n_rows, k, p) || out_in.world < 1 || out_in.world > kMaxPeers || !out_in.epoch)
        return cudaErrorInvalidValue;
    const uint8_t* wb = static_cast<const uint8_t*>(w);
    const int n = static_cast<int>(n_rows), kk = static_cast<int>(k);
    return launch_strip_qt<false, kOutPeer>(qtype, wb, n, kk, x, nullptr, scale, p, kXPlain, nullptr, 0.f, nullptr,
                                            out_in, LLIn{}, LLOut{}, stream);
}

cudaError_t qmv_strip_shard(int qtype, const void* w, int64_t n_rows, int64_t k, StripInput in, const float* norm_w,
                            float eps, float scale, const float* x, float* y, const float* resid, const LLIn& lin,
                            const LLOut& lout, cudaStream_t stream) {
    StripPlan p;
    const bool llx = lin.x != nullptr, tagged = lout.world > 0;
    if (!plan_strip(qtype, n_rows, k, p) || (llx ? (!lin.count || x) : (!x || lin.resid)) || lout.world < 0 ||
        lout.world > kPeerSyncMax || (tagged && (!lout.count || y || resid)) ||
        (!tagged && (!y || lin.resid)) || (llx && tagged && resid))
        return cudaErrorInvalidValue;
    if (in == StripInput::kRmsNorm && (!norm_w || k > static_cast<int64_t>(kWarps) * kStripBatch * 256))
        return cudaErrorInvalidValue;
    const int xm = in == StripInput::kRmsNorm ? kXRmsNorm : in == StripInput::kSiluMul ? kXSiluMul : kXPlain;
    const uint8_t* wb = static_cast<const uint8_t*>(w);
    const int n = static_cast<int>(n_rows), kk = static_cast<int>(k);
    if (llx && tagged)
        return launch_strip_qt<true, kOutTagged>(qtype, wb, n, kk, nullptr, nullptr, scale, p, xm, norm_w, eps, nullptr,
                                                 PeerOut{}, lin, lout, stream);
    if (llx)
        return launch_strip_qt<true, kOutPlain>(qtype, wb, n, kk, nullptr, y, scale, p, xm, norm_w, eps, resid,
                                                PeerOut{}, lin, lout, stream);
    if (tagged)
        return launch_strip_qt<false, kOutTagged>(qtype, wb, n, kk, x, nullptr, scale, p, xm, norm_w, eps, nullptr,
                                                  PeerOut{}, lin, lout, stream);
    return launch_strip_qt<false, kOutPlain>(qtype, wb, n, kk, x, y, scale, p, xm, norm_w, eps, resid, PeerOut{}, lin,
                                             lout, stream);
}

cudaError_t qmv_strip_gather_tagged(int qtype, const void* w, int64_t n_rows, int64_t k, const float* x, float scale,
                                    const LLOut& lout, cudaStream_t stream) {
    StripPlan p;
    if (!plan_strip(qtype, n_rows, k, p) || !x || lout.world < 1 || lout.world > kPeerSyncMax || !lout.count ||
        !lout.by_parity)
        return cudaErrorInvalidValue;
    const uint8_t* wb = static_cast<const uint8_t*>(w);
    const int n = static_cast<int>(n_rows), kk = static_cast<int>(k);
    return launch_strip_qt<false, kOutTagged>(qtype, wb, n, kk, x, nullptr, scale, p, kXPlain, nullptr, 0.f, nullptr,
                                              PeerOut{}, LLIn{}, lout, stream);
}

cudaError_t qmv_rowwise(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, int64_t ldx,
                        int64_t batch, float* y, int64_t ldy, float scale, cudaStream_t stream) {
    const uint8_t* wb = static_cast<const uint8_t*>(w);
    const int n = static_cast<int>(n_out), kk = static_cast<int>(k), b = static_cast<int>(batch);
    switch (qtype) {
        case kQ4_0: return launch_rowwise<kQ4_0>(wb, n, kk, x, ldx, b, y, ldy, scale, stream);
        case kQ8_0: return launch_rowwise<kQ8_0>(wb, n, kk, x, ldx, b, y, ldy, scale, stream);
        case kQ4_K: return launch_rowwise<kQ4_K>(wb, n, kk, x, ldx, b, y, ldy, scale, stream);
        case kQ5_K: return launch_rowwise<kQ5_K>(wb, n, kk, x, ldx, b, y, ldy, scale, stream);
        case kQ6_K: return launch_rowwise<kQ6_K>(wb, n, kk, x, ldx, b, y, ldy, scale, stream);
        default: return cudaErrorInvalidValue;
    }
}

// ---------------------------------------------------------------------------
// Allocation-free variant of the batch-1 streaming matvec.
//
// The streaming kernel needs scratch for the row groups that straddle two
// warps (arrival counters and partial sums). hesa_cuda_qmatvec takes it from
// the caller; this variant keeps it in the fixed array below instead, for
// callers that may not allocate device memory at all. The array lives in
// every GPU that loads the library until the process exits.
//   counters: kNoAllocGroups ints   (row groups of 2 rows -> n_out <= 65536)
//   partials: kMaxGridCtas * kWarps * 2 * kMaxRows floats
// In host code `g_noalloc_scratch` only names the symbol; its device address
// comes from cudaGetSymbolAddress, looked up once per device with that device
// current, on the first call there.
// ---------------------------------------------------------------------------

constexpr size_t kNoAllocGroups = 32768;
constexpr size_t kNoAllocCounterBytes = kNoAllocGroups * sizeof(int);
constexpr size_t kNoAllocPartialBytes = static_cast<size_t>(kMaxGridCtas) * kWarps * 2 * kMaxRows * sizeof(float);
constexpr size_t kNoAllocScratchBytes = kNoAllocCounterBytes + kNoAllocPartialBytes;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

static uint8_t* g_noalloc_ptr[64] = {nullptr};

int64_t qmv_noalloc_max_rows() { return static_cast<int64_t>(kNoAllocGroups) * 2; }

cudaError_t qmv_noalloc_scratch(uint8_t** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_noalloc_ptr[dev] = static_cast<uint8_t*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return cudaSuccess;
}

cudaError_t qmv_stream_noalloc(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, float* y,
                               float scale, cudaStream_t stream) {
    if (!qtype_supported(qtype) || n_out > qmv_noalloc_max_rows()) return cudaErrorInvalidValue;
    uint8_t* scratch = nullptr;
    cudaError_t e = qmv_noalloc_scratch(&scratch);
    if (e != cudaSuccess) return e;
    // the counters must start at zero; the array keeps whatever the last call
    // (possibly a failed one) left there
    const int R = rows_of(qtype);
    const size_t groups = (static_cast<size_t>(n_out) + R - 1) / R;
    e = cudaMemsetAsync(scratch, 0, groups * sizeof(int), stream);
    if (e != cudaSuccess) return e;
    int* counters = reinterpret_cast<int*>(scratch);
    float* partials = reinterpret_cast<float*>(scratch + kNoAllocCounterBytes);
    int grid = qmv_stream_grid(qtype, n_out, k);
    const int64_t cells = stream_cells(qtype, n_out, k);
    if (static_cast<int64_t>(grid) * kWarps > cells) grid = static_cast<int>(cells / kWarps);
    if (grid < 1 || grid > kMaxGridCtas) return cudaErrorInvalidValue;
    const uint8_t* wb = static_cast<const uint8_t*>(w);
    const int n = static_cast<int>(n_out), kk = static_cast<int>(k);
    switch (qtype) {
        case kQ4_0: return launch_stream<kQ4_0>(wb, n, kk, x, y, scale, counters, partials, grid, stream);
        case kQ8_0: return launch_stream<kQ8_0>(wb, n, kk, x, y, scale, counters, partials, grid, stream);
        case kQ4_K: return launch_stream<kQ4_K>(wb, n, kk, x, y, scale, counters, partials, grid, stream);
        case kQ5_K: return launch_stream<kQ5_K>(wb, n, kk, x, y, scale, counters, partials, grid, stream);
        case kQ6_K: return launch_stream<kQ6_K>(wb, n, kk, x, y, scale, counters, partials, grid, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t status_word(int** out) { return status_ptr(out); }

cudaError_t read_device_status(int* out) {
    return cudaMemcpyFromSymbol(out, g_hesa_status, sizeof(int));
}

cudaError_t clear_device_status(cudaStream_t stream) {
    static const int zero = 0;
    cudaError_t e = cudaMemcpyToSymbolAsync(g_hesa_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return e;
    return cudaStreamSynchronize(stream);
}

cudaError_t dequantize(int qtype, const void* w, int64_t n_rows, int64_t k, float* out, int64_t ldo,
                       cudaStream_t stream) {
    const uint8_t* wb = static_cast<const uint8_t*>(w);
    switch (qtype) {
        case kQ4_0: return launch_dequant<kQ4_0>(wb, n_rows, k, out, ldo, stream);
        case kQ8_0: return launch_dequant<kQ8_0>(wb, n_rows, k, out, ldo, stream);
        case kQ4_K: return launch_dequant<kQ4_K>(wb, n_rows, k, out, ldo, stream);
        case kQ5_K: return launch_dequant<kQ5_K>(wb, n_rows, k, out, ldo, stream);
        case kQ6_K: return launch_dequant<kQ6_K>(wb, n_rows, k, out, ldo, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace hesa_cuda
