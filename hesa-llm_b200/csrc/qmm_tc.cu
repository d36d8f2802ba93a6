// qmm_tc.cu -- batched Q4_K / Q5_K matmul on the 5th-generation tensor cores
// (tcgen05, TMEM, TMA; sm_100a): Y[b, :] = scale * W . X[b, :] for 2..16
// activation rows per launch.
//
// Numerics are the batch-1 kernels' (qmatvec.cu): per unit of 256
// activations and per activation row, X = rint(x / s) as three balanced int8
// digit planes (xdigits.cuh), so every weight-level x digit product and every
// sum over a unit is exact in int32; the planes are combined in fp32 once per
// unit with the row's super-block scale, and the min terms
// dmin * m_j * sum(x over sub-block j) come from per-sub-block sums of x.
//
// The sub-block scale is folded into the weight operand: sc = lo + 2^S hi
// (S = 4 for Q4_K, 3 for Q5_K) so that q*lo and q*hi fit a byte; one 32-bit
// multiply scales four packed levels without carries. Per unit of a 128-row
// tile:
//   * each of the 128 rows is one TMEM lane: its thread unpacks the row's
//     levels and writes the folded operand for the unit (two halves of 64
//     columns, k packed four per column) into TMEM with tcgen05.st;
//   * the activations' digit planes (3 x rows, padded to N = 32 or 48 "column
//     planes") sit in shared memory in the canonical K-major core-matrix
//     layout (8 rows x 16 bytes per core matrix);
//   * one thread of its own warp issues 16 tcgen05.mma kind::i8 (u8 x s8 ->
//     s32, M = 128, K = 32: eight k-steps for each half) with A from TMEM, B
//     from shared memory, the two accumulators in TMEM, and commits them to
//     an mbarrier;
//   * the row threads read the accumulators back (tcgen05.ld) and apply the
//     unit's scales.
// A and the accumulators are double-buffered in TMEM, so a unit's unpacking,
// the previous unit's MMAs and the one before's epilogue overlap.
//
// Work: S K-slices of the units x the 128-row tiles, as items (slice, tile)
// split into equal contiguous ranges, one per CTA (one CTA per SM). A CTA
// stages its slice's activations once (again only if its range crosses into
// the next slice). A producer warp streams the weights with 2-D TMA tensor
// copies: 128 rows x 2 units per copy, into a ring of shared-memory slots.
// Slices of a tile are added by the last of their CTAs to finish (ticket), in
// slice order, so results do not depend on scheduling.
#include "hesa_common.cuh"
#include "qtypes.cuh"
#include "xdigits.cuh"
#include "qmm.h"
#include "qmatvec.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda/atomic>

#include <algorithm>
#include <cmath>

namespace hesa_cuda {

namespace {

constexpr int kRows = 128;                          // weight rows per tile = TMEM lanes
constexpr int kRowWarps = 8;                        // two per TMEM lane quarter
constexpr int kThreads = (kRowWarps + 2) * 32;      // + the producer warp and the MMA warp
constexpr int kSU = 2;                              // units per weight copy
constexpr int kWSlots = 3;
constexpr int kPlanSms = 148;
constexpr int kMaxCols = 16;                        // activation rows per launch
constexpr uint32_t kTmemCols = 512;
constexpr int kMaxItems = 64;                       // items per CTA (tickets kept for the end)
constexpr size_t kSmemMax = 227 * 1024 - 1024;

__host__ __device__ constexpr int tc_ub(int qt) { return qt == kQ4_K ? 144 : 176; }
__host__ __device__ constexpr int tc_qs(int qt) { return qt == kQ4_K ? 16 : 48; }
// MMA N: 3 digit planes x BP activation rows, padded to a multiple of 16
template <int NBT> __host__ __device__ constexpr int tc_n() { return NBT == 1 ? 32 : 48; }
// units per slice at most
template <int NBT> __host__ __device__ constexpr int tc_ku() { return NBT == 1 ? 8 : 6; }
// per unit of the slice in shared memory: B operand [k-step 8][k half 2][N/8][8 rows][16 B], then
// per activation row 12 floats: s, sum_k x_k over sub-blocks 0..7, pad
template <int NBT> __host__ __device__ constexpr uint32_t tc_xb() { return static_cast<uint32_t>(tc_n<NBT>()) * 256; }
template <int NBT> __host__ __device__ constexpr uint32_t tc_xub() { return tc_xb<NBT>() + 8 * NBT * 48; }
template <int QT> __host__ __device__ constexpr uint32_t tc_slot() { return kRows * kSU * tc_ub(QT); }

// ---- tcgen05 --------------------------------------------------------------
// Shared-memory matrix descriptor, K-major without swizzle: start address,
// LBO = byte distance between the two 16-byte k halves of a k-step, SBO =
// byte distance between 8-row core matrices, descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// D (+)= A . B, A from TMEM, B from shared memory, kind::i8, one CTA.
__device__ __forceinline__ void tc_mma_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(d),
        "r"(a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// NC consecutive columns of this warp's 32 lanes (one per thread)
template <int NC>
__device__ __forceinline__ void tc_ld(uint32_t taddr, uint32_t (&v)[NC]) {
    static_assert(NC == 4 || NC == 8, "tc_ld width");
    if constexpr (NC == 4) {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                     : "r"(taddr));
    } else {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                     : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                       "=r"(v[7])
                     : "r"(taddr));
    }
}
// wait for this thread's tcgen05.ld; the registers are redefined after it so
// no use can be scheduled before the wait
template <int NC>
__device__ __forceinline__ void tc_wait_ld(uint32_t (&v)[NC]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < NC; ++i) asm volatile("" : "+r"(v[i]));
}

__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// Byte j (compile-time) of w, zero-extended.
template <int J>
__device__ __forceinline__ uint32_t byte_at(uint32_t w) {
    return prmt(w, 0u, 0x4440u + J);
}

// One warp: unit u of activation row b (zeros for b >= batch) into the unit's
// block: digit plane p of row b is B row (column plane) p*BP + b.
template <int NBT>
__device__ __forceinline__ void tc_stage_pair(const float* __restrict__ x, int64_t ldx, int batch, int u, int b,
                                              int lane, uint8_t* blk) {
    constexpr int BP = 8 * NBT, N = tc_n<NBT>();
    float v[8];
    if (b < batch) {
        const float4* src = reinterpret_cast<const float4*>(x + b * ldx + static_cast<int64_t>(u) * 256 + lane * 8);
        const float4 p = src[0], q = src[1];
        v[0] = p.x; v[1] = p.y; v[2] = p.z; v[3] = p.w;
        v[4] = q.x; v[5] = q.y; v[6] = q.z; v[7] = q.w;
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 0.f;
    }
    uint32_t dw[3][2];
    const float s = unit_digits(v, dw);
    // positions 8L..8L+7: k-step L/4, k half (L/2)&1, bytes 8(L&1)..+7 of the core row
    const int st = lane >> 2, h = (lane >> 1) & 1, off = 8 * (lane & 1);
#pragma unroll
    for (int p = 0; p < 3; ++p) {
        const int cp = p * BP + b;
        *reinterpret_cast<uint2*>(blk + st * 2 * (N / 8) * 128 + h * (N / 8) * 128 + (cp >> 3) * 128 + (cp & 7) * 16 +
                                  off) = make_uint2(dw[p][0], dw[p][1]);
    }
    int sums[3];
#pragma unroll
    for (int p = 0; p < 3; ++p) {
        sums[p] = __dp4a(static_cast<int>(dw[p][0]), 0x01010101, __dp4a(static_cast<int>(dw[p][1]), 0x01010101, 0));
        sums[p] += __shfl_xor_sync(0xffffffffu, sums[p], 1);
        sums[p] += __shfl_xor_sync(0xffffffffu, sums[p], 2);
    }
    float* info = reinterpret_cast<float*>(blk + tc_xb<NBT>()) + b * 12;
    if ((lane & 3) == 0) info[1 + (lane >> 2)] = s * combine3(sums[0], sums[1], sums[2]);
    if (lane == 0) info[0] = s;
}

template <int QT, int NBT>
__global__ void __launch_bounds__(kThreads, 1)
qmm_tc_kernel(const __grid_constant__ CUtensorMap wmap2, const __grid_constant__ CUtensorMap wmap1, int n_out, int U,
              int S, const float* __restrict__ x, int64_t ldx, float* __restrict__ y, int64_t ldy, int batch,
              float scale, float* __restrict__ partials, int* __restrict__ tickets, int* __restrict__ status) {
    constexpr int BP = 8 * NBT, HB = BP / 2, N = tc_n<NBT>(), UB = tc_ub(QT), QO = tc_qs(QT), KU = tc_ku<NBT>();
    constexpr uint32_t XB = tc_xb<NBT>(), XUB = tc_xub<NBT>(), SLOT = tc_slot<QT>();
    constexpr int SBITS = QT == kQ4_K ? 4 : 3;
    constexpr uint32_t LOM = QT == kQ4_K ? 0x0F0F0F0Fu : 0x07070707u;
    constexpr uint32_t IDESC = (2u << 4) | (0u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
                               (static_cast<uint32_t>(kRows >> 4) << 24);
    constexpr uint32_t KSTEP = 2 * (N / 8) * 128;   // B bytes per k-step
    // TMEM columns: A buffers at 0 and 128 (low half +0, high half +64), accumulators at 256 + 2N*buf (+N high)
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t wfull[kWSlots], wfree[kWSlots], aready[2], dready[2], dfree[2];
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;
    __shared__ int item_old[kMaxItems];

    const int RT = (n_out + kRows - 1) / kRows;
    const int64_t I = static_cast<int64_t>(S) * RT, G = gridDim.x, cta = blockIdx.x;
    const int i0 = static_cast<int>(cta * I / G), i1 = static_cast<int>((cta + 1) * I / G);
    uint8_t* sx = smem;
    uint8_t* sw = smem + static_cast<size_t>(KU) * XUB;
    volatile int* abort_v = &abort_flag;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kWSlots; ++i) {
            mbar_init(&wfull[i], 1);
            mbar_init(&wfree[i], kRowWarps);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&aready[i], kRowWarps);
            mbar_init(&dready[i], 1);
            mbar_init(&dfree[i], kRowWarps);
        }
        abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    if (warp == kRowWarps) {
        // ---- producer: the weight copies, 128 rows x (up to) 2 units each ----
        if (lane == 0) {
            int cq = 0;
            for (int it = i0; it < i1 && !*abort_v; ++it) {
                const int s = it / RT, rt = it - s * RT;
                const int u0 = s * U / S, nu = (s + 1) * U / S - u0;
                for (int g = 0; 2 * g < nu; ++g, ++cq) {
                    const int slot = cq % kWSlots;
                    if (cq >= kWSlots &&
                        !mbar_wait_bounded(&wfree[slot], static_cast<uint32_t>(cq / kWSlots - 1) & 1u, status,
                                           kStatusWaitTimeout)) {
                        *abort_v = 1;
                        break;
                    }
                    const int wd = 2 * g + 1 < nu ? 2 : 1;
                    mbar_arrive_expect_tx(&wfull[slot], static_cast<uint32_t>(kRows * wd * UB));
                    tma_load_2d(sw + static_cast<size_t>(slot) * SLOT, wd == 2 ? &wmap2 : &wmap1,
                                (u0 + 2 * g) * UB / 2, rt * kRows, &wfull[slot]);
                }
            }
            // every copy of this CTA is issued: the next kernel on the stream may
            // start its CTAs on the SMs this grid leaves (its weight copies overlap
            // this grid's tail; it reads x and writes y only after this grid ends).
            // Measured: B = 8 on 4096 x 11008, 24.2 -> 21.9 us per matvec
            grid_dep_launch();
            // the last copies into each slot have landed before the CTA may exit
            for (int c = cq > kWSlots ? cq - kWSlots : 0; c < cq; ++c)
                if (!mbar_wait_bounded(&wfull[c % kWSlots], static_cast<uint32_t>(c / kWSlots) & 1u, status,
                                       kStatusDrainTimeout))
                    break;
        }
        return;
    }
    if (warp == kRowWarps + 1) {
        // ---- MMA warp: one thread issues every unit's MMAs once its operand is in TMEM ----
        if (lane == 0) {
            int q = 0;
            for (int it = i0; it < i1 && !*abort_v; ++it) {
                const int s = it / RT;
                const int nu = (s + 1) * U / S - s * U / S;
                for (int ui = 0; ui < nu; ++ui, ++q) {
                    bool go = mbar_wait_bounded(&aready[q & 1], static_cast<uint32_t>(q >> 1) & 1u, status,
                                                kStatusWaitTimeout);
                    if (go && q >= 2)
                        go = mbar_wait_bounded(&dfree[q & 1], static_cast<uint32_t>((q >> 1) - 1) & 1u, status,
                                               kStatusWaitTimeout);
                    if (!go || *abort_v) {
                        *abort_v = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a = tmem + static_cast<uint32_t>(128 * (q & 1));
                    const uint32_t d = tmem + 256u + static_cast<uint32_t>(2 * N * (q & 1));
                    const uint32_t xb = smem_addr(sx + static_cast<size_t>(ui) * XUB);
#pragma unroll
                    for (int st = 0; st < 8; ++st) {
                        const uint64_t bd = umma_desc(xb + st * KSTEP, (N / 8) * 128, 128);
                        tc_mma_ts(d, a + 8 * st, bd, IDESC, st > 0);
                        tc_mma_ts(d + N, a + 64 + 8 * st, bd, IDESC, st > 0);
                    }
                    tc_commit(&dready[q & 1]);
                }
            }
        }
        return;
    }

    // ---- row warps ----
    const int wq = warp & 3, hf = warp >> 2;
    const int row_t = 32 * wq + lane;                        // row within the tile = TMEM lane
    const uint32_t tlane = static_cast<uint32_t>(32 * wq) << 16;
    grid_dep_wait();   // x may be written by the previous grid

    auto stage_slice = [&](int s) {
        const int u0 = s * U / S, nu = (s + 1) * U / S - u0;
        // zero the slice's blocks (padding column planes stay zero), then convert
        uint4* z = reinterpret_cast<uint4*>(sx);
        for (int i = threadIdx.x; i < static_cast<int>(nu * XUB / 16); i += kRowWarps * 32) z[i] = make_uint4(0, 0, 0, 0);
        named_barrier(1, kRowWarps * 32);
        for (int pr = warp; pr < nu * BP; pr += kRowWarps)
            tc_stage_pair<NBT>(x, ldx, batch, u0 + pr / BP, pr % BP, lane, sx + static_cast<size_t>(pr / BP) * XUB);
        fence_proxy_async_smem();   // the tensor cores read the planes through the async proxy
        named_barrier(1, kRowWarps * 32);
    };

    int q = 0, cq_base = 0, cur_s = -1, n_items = 0;
    for (int it = i0; it < i1; ++it) {
        const int s = it / RT, rt = it - s * RT;
        const int nu = (s + 1) * U / S - s * U / S;
        if (s != cur_s) {
            if (cur_s >= 0) named_barrier(1, kRowWarps * 32);   // every MMA and read of the old slice is done
            stage_slice(s);
            cur_s = s;
        }
        float acc[HB];
#pragma unroll
        for (int i = 0; i < HB; ++i) acc[i] = 0.f;
        uint4 hdr = make_uint4(0, 0, 0, 0), hdr_prev = make_uint4(0, 0, 0, 0);
        for (int ui = 0; ui <= nu; ++ui) {
            if (ui < nu) {
                // ---- unit ui: folded levels of this thread's row into A buffer q%2 ----
                const int cqu = cq_base + ui / 2, slot = cqu % kWSlots;
                const int wd = 2 * (ui / 2) + 1 < nu ? 2 : 1;
                bool ok = !*abort_v;
                if (ok && (ui & 1) == 0) {
                    ok = mbar_wait_bounded(&wfull[slot], static_cast<uint32_t>(cqu / kWSlots) & 1u, status,
                                           kStatusWaitTimeout);
                    if (!ok) *abort_v = 1;
                }
                ok = __all_sync(0xffffffffu, ok);
                const uint8_t* rowp = sw + static_cast<size_t>(slot) * SLOT + row_t * (wd * UB) + (ui & 1) * UB;
                if (ok) {
                    hdr = lds128(rowp);
                    const uint32_t sc03 = hdr.y & 0x3F3F3F3Fu;
                    const uint32_t sc47 = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
                    // sub-blocks 4hf .. 4hf+3 (this warp's k-steps)
                    const uint32_t scw = hf ? sc47 : sc03;
                    const uint32_t slo = scw & LOM, shi = (scw >> SBITS) & LOM;
                    const uint4 r0 = lds128(rowp + QO + 64 * hf), r1 = lds128(rowp + QO + 64 * hf + 16);
                    const uint4 r2 = lds128(rowp + QO + 64 * hf + 32), r3 = lds128(rowp + QO + 64 * hf + 48);
                    // k-steps 4hf + jj: sub-block pair jj/2 uses qs bytes 64hf + 32(jj/2) .. +31
                    const uint32_t raw[2][8] = {{r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w},
                                                {r2.x, r2.y, r2.z, r2.w, r3.x, r3.y, r3.z, r3.w}};
                    uint32_t qh[8];
                    if constexpr (QT == kQ5_K) {
                        const uint4 h0 = lds128(rowp + 16), h1 = lds128(rowp + 32);
                        qh[0] = h0.x; qh[1] = h0.y; qh[2] = h0.z; qh[3] = h0.w;
                        qh[4] = h1.x; qh[5] = h1.y; qh[6] = h1.z; qh[7] = h1.w;
                    }
                    const uint32_t abuf = tmem + tlane + static_cast<uint32_t>(128 * (q & 1));
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        const int j = 4 * hf + jj;   // sub-block = k-step
                        uint32_t lo_s, hi_s;
                        if (jj == 0) { lo_s = byte_at<0>(slo); hi_s = byte_at<0>(shi); }
                        else if (jj == 1) { lo_s = byte_at<1>(slo); hi_s = byte_at<1>(shi); }
                        else if (jj == 2) { lo_s = byte_at<2>(slo); hi_s = byte_at<2>(shi); }
                        else { lo_s = byte_at<3>(slo); hi_s = byte_at<3>(shi); }
                        uint32_t wlo[8], whi[8];
#pragma unroll
                        for (int c = 0; c < 8; ++c) {
                            uint32_t qv = (raw[jj >> 1][c] >> (4 * (jj & 1))) & 0x0F0F0F0Fu;
                            if constexpr (QT == kQ5_K) qv |= ((qh[c] >> j) & 0x01010101u) << 4;
                            wlo[c] = qv * lo_s;
                            whi[c] = qv * hi_s;
                        }
                        tc_st8(abuf + 8 * j, wlo);
                        tc_st8(abuf + 64 + 8 * j, whi);
                    }
                    tc_wait_st();
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&aready[q & 1]);
                    if ((ui & 1) == 1 || ui == nu - 1) mbar_arrive(&wfree[slot]);   // the copy is consumed
                }
                __syncwarp();
            }
            if (ui >= 1) {
                // ---- epilogue of unit ui-1 (its accumulators and header) ----
                const int qp = q - 1;   // unit index of ui-1 (q counts the units transformed so far)
                bool ok = !*abort_v;
                if (ok) {
                    ok = mbar_wait_bounded(&dready[qp & 1], static_cast<uint32_t>(qp >> 1) & 1u, status,
                                           kStatusWaitTimeout);
                    if (!ok) *abort_v = 1;
                }
                ok = __all_sync(0xffffffffu, ok);
                tc_fence_after();
                if (ok) {
                    const uint32_t d = tmem + tlane + 256u + static_cast<uint32_t>(2 * N * (qp & 1));
                    uint32_t lo[3][HB], hi[3][HB];
#pragma unroll
                    for (int p = 0; p < 3; ++p) {
                        tc_ld<HB>(d + p * BP + hf * HB, lo[p]);
                        tc_ld<HB>(d + N + p * BP + hf * HB, hi[p]);
                    }
#pragma unroll
                    for (int p = 0; p < 3; ++p) {
                        tc_wait_ld<HB>(lo[p]);
                        tc_wait_ld<HB>(hi[p]);
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&dfree[qp & 1]);
                    const uint4 hp = hdr_prev;
                    const float dd = half_bits_to_float(hp.x), dmin = half_bits_to_float(hp.x >> 16);
                    const uint32_t m03 = hp.z & 0x3F3F3F3Fu;
                    const uint32_t m47 = ((hp.w >> 4) & 0x0F0F0F0Fu) | ((hp.z >> 2) & 0x30303030u);
                    const float m[8] = {static_cast<float>(byte_at<0>(m03)), static_cast<float>(byte_at<1>(m03)),
                                        static_cast<float>(byte_at<2>(m03)), static_cast<float>(byte_at<3>(m03)),
                                        static_cast<float>(byte_at<0>(m47)), static_cast<float>(byte_at<1>(m47)),
                                        static_cast<float>(byte_at<2>(m47)), static_cast<float>(byte_at<3>(m47))};
                    const float* info = reinterpret_cast<const float*>(sx + static_cast<size_t>(ui - 1) * XUB + XB);
#pragma unroll
                    for (int jb = 0; jb < HB; ++jb) {
                        const float* inf = info + (hf * HB + jb) * 12;
                        const float4 i0 = *reinterpret_cast<const float4*>(inf);
                        const float4 i1 = *reinterpret_cast<const float4*>(inf + 4);
                        const float xs8 = inf[8];
                        int pl[3];
#pragma unroll
                        for (int p = 0; p < 3; ++p)
                            pl[p] = static_cast<int>(lo[p][jb]) + (static_cast<int>(hi[p][jb]) << SBITS);
                        const float tv = combine3(pl[0], pl[1], pl[2]);
                        float mins = m[0] * i0.y;
                        mins = fmaf(m[1], i0.z, mins);
                        mins = fmaf(m[2], i0.w, mins);
                        mins = fmaf(m[3], i1.x, mins);
                        mins = fmaf(m[4], i1.y, mins);
                        mins = fmaf(m[5], i1.z, mins);
                        mins = fmaf(m[6], i1.w, mins);
                        mins = fmaf(m[7], xs8, mins);
                        acc[jb] += fmaf(dd * i0.x, tv, -dmin * mins);
                    }
                } else {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&dfree[qp & 1]);
                }
            }
            hdr_prev = hdr;
            if (ui < nu) ++q;
        }
        cq_base += (nu + 1) / 2;

        // ---- item output: this thread's row, columns hf*HB .. +HB ----
        const int row = rt * kRows + row_t;
        if (S == 1) {
            if (row < n_out) {
#pragma unroll
                for (int jb = 0; jb < HB; ++jb) {
                    const int b = hf * HB + jb;
                    if (b < batch) y[b * ldy + row] = acc[jb] * scale;
                }
            }
        } else {
            float* pr = partials + (static_cast<size_t>(s) * RT * kRows + rt * kRows + row_t) * BP + hf * HB;
#pragma unroll
            for (int jb = 0; jb < HB; ++jb) pr[jb] = acc[jb];   // the whole tile, rows past n_out included
            named_barrier(1, kRowWarps * 32);
            if (threadIdx.x == 0) {
                // the ticket's result is only needed at the end: its latency hides behind the next items
                cuda::atomic_ref<int, cuda::thread_scope_device> tk(tickets[rt]);
                item_old[n_items < kMaxItems ? n_items : kMaxItems - 1] = tk.fetch_add(1, cuda::memory_order_acq_rel);
            }
        }
        ++n_items;
    }

    // ---- the slice sums of the tiles this CTA finished last, in slice order ----
    named_barrier(1, kRowWarps * 32);
    if (S > 1 && !*abort_v) {
        int k = 0;
        for (int it = i0; it < i1; ++it, ++k) {
            const int rt = it % RT;
            if (item_old[k] != S - 1) continue;
            const int row = rt * kRows + row_t;
            float sum[HB];
#pragma unroll
            for (int jb = 0; jb < HB; ++jb) sum[jb] = 0.f;
            for (int ss = 0; ss < S; ++ss) {
                const float* pr = partials + (static_cast<size_t>(ss) * RT * kRows + rt * kRows + row_t) * BP + hf * HB;
#pragma unroll
                for (int jb = 0; jb < HB; ++jb) sum[jb] += __ldcg(pr + jb);
            }
            if (row < n_out) {
#pragma unroll
                for (int jb = 0; jb < HB; ++jb) {
                    const int b = hf * HB + jb;
                    if (b < batch) y[b * ldy + row] = sum[jb] * scale;
                }
            }
            if (threadIdx.x == 0) tickets[rt] = 0;   // leave the workspace zeroed
        }
    }
    tc_fence_before();
    named_barrier(1, kRowWarps * 32);
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

struct TcPlan {
    int nbt, S, grid;
    size_t smem, part_bytes, ticket_bytes;
};

constexpr size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

TcPlan make_tc_plan(int qt, int64_t n_out, int64_t k, int cols) {
    TcPlan p{};
    p.nbt = cols <= 8 ? 1 : 2;
    const int KU = p.nbt == 1 ? tc_ku<1>() : tc_ku<2>(), BP = 8 * p.nbt;
    const int U = static_cast<int>(k / 256);
    const int RT = static_cast<int>((n_out + kRows - 1) / kRows);
    // slices: the fewest that fit KU units and keep the items of the CTAs balanced
    const int s_min = (U + KU - 1) / KU;
    double best = -1.0;
    for (int S = s_min; S <= U && S <= s_min + 8; ++S) {
        const int64_t items = static_cast<int64_t>(S) * RT;
        const int64_t g = items < kPlanSms ? items : kPlanSms;
        const double per = static_cast<double>(items) / static_cast<double>(g);
        const double eff = per / std::ceil(per) * (static_cast<double>(g) / kPlanSms);
        if (eff > best + 0.03) {
            best = eff;
            p.S = S;
            p.grid = static_cast<int>(g);
        }
    }
    const size_t xs = static_cast<size_t>(KU) * (p.nbt == 1 ? tc_xub<1>() : tc_xub<2>());
    const size_t slots = static_cast<size_t>(kWSlots) * (qt == kQ4_K ? tc_slot<kQ4_K>() : tc_slot<kQ5_K>());
    p.smem = xs + slots;
    p.part_bytes = p.S > 1 ? align256(static_cast<size_t>(p.S) * RT * kRows * BP * 4) : 0;
    // tickets at the start of the workspace, inside the region the batch-1
    // split-row kernel keeps zeroed (one int per 2 rows; RT <= that)
    p.ticket_bytes = align256(((static_cast<size_t>(n_out) + 1) / 2) * 4);
    return p;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    return fn;
}

// W as a 2-D tensor of 16-bit elements [n_out][row_bytes / 2]; box = `units` units x 128 rows.
bool encode_wmap(CUtensorMap* map, const void* w, int64_t n_out, int64_t row_bytes, int units, int ub) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes / 2), static_cast<cuuint64_t>(n_out)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(units * ub / 2), static_cast<cuuint32_t>(kRows)};
    const cuuint32_t elem[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(w), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int QT, int NBT>
cudaError_t launch_tc(const void* w, int n_out, int k, const float* x, int64_t ldx, int cols, float* y, int64_t ldy,
                      float scale, uint8_t* ws, const TcPlan& p, cudaStream_t stream) {
    constexpr int UB = tc_ub(QT);
    const int U = k / 256;
    CUtensorMap m2, m1;
    if (!encode_wmap(&m2, w, n_out, static_cast<int64_t>(U) * UB, 2, UB) ||
        !encode_wmap(&m1, w, n_out, static_cast<int64_t>(U) * UB, 1, UB))
        return cudaErrorInvalidValue;
    int* tickets = reinterpret_cast<int*>(ws);
    float* partials = reinterpret_cast<float*>(ws + p.ticket_bytes);
    int* status = nullptr;
    cudaError_t e = status_word(&status);
    if (e != cudaSuccess) return e;
    static bool attr_set[64] = {};   // per template instance and device
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(qmm_tc_kernel<QT, NBT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kSmemMax));
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(p.grid), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, qmm_tc_kernel<QT, NBT>, m2, m1, n_out, U, p.S, x, ldx, y, ldy, cols, scale,
                              partials, tickets, status);
}

}  // namespace

bool qmm_tc_eligible(int qtype, const void* w, int64_t n_out, int64_t k, int64_t batch) {
    if (qtype != kQ4_K && qtype != kQ5_K) return false;
    if (batch < 2 || n_out <= 0 || k <= 0 || k % 256 != 0) return false;
    if ((reinterpret_cast<uintptr_t>(w) & 15) != 0) return false;
    // items per CTA are bounded by the ticket list; the tensor map takes
    // rows of up to 2^32 elements and 2^31 - 1 rows
    const TcPlan p = make_tc_plan(qtype, n_out, k, kMaxCols);
    const int64_t RT = (n_out + kRows - 1) / kRows;
    return (static_cast<int64_t>(p.S) * RT + p.grid - 1) / p.grid <= kMaxItems && n_out < (int64_t(1) << 31) &&
           p.smem <= kSmemMax;
}

size_t qmm_tc_workspace_bytes(int qtype, int64_t n_out, int64_t k, int64_t batch) {
    if ((qtype != kQ4_K && qtype != kQ5_K) || batch < 2) return 0;
    // launches of kMaxCols rows, then the remainder
    size_t n = 0;
    for (int64_t cols : {batch >= kMaxCols ? int64_t(kMaxCols) : int64_t(0), batch % kMaxCols}) {
        if (cols <= 0) continue;
        const TcPlan p = make_tc_plan(qtype, n_out, k, static_cast<int>(cols));
        n = std::max(n, p.ticket_bytes + p.part_bytes);
    }
    return n;
}

cudaError_t qmm_tc(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, int64_t ldx, int64_t batch,
                   float* y, int64_t ldy, float scale, void* workspace, cudaStream_t stream) {
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    for (int64_t b0 = 0; b0 < batch; b0 += kMaxCols) {
        const int cols = static_cast<int>(batch - b0 < kMaxCols ? batch - b0 : kMaxCols);
        const TcPlan p = make_tc_plan(qtype, n_out, k, cols);
        const float* xb = x + b0 * ldx;
        float* yb = y + b0 * ldy;
        const int n = static_cast<int>(n_out), kk = static_cast<int>(k);
        cudaError_t e;
        if (qtype == kQ4_K)
            e = p.nbt == 1 ? launch_tc<kQ4_K, 1>(w, n, kk, xb, ldx, cols, yb, ldy, scale, ws, p, stream)
                           : launch_tc<kQ4_K, 2>(w, n, kk, xb, ldx, cols, yb, ldy, scale, ws, p, stream);
        else if (qtype == kQ5_K)
            e = p.nbt == 1 ? launch_tc<kQ5_K, 1>(w, n, kk, xb, ldx, cols, yb, ldy, scale, ws, p, stream)
                           : launch_tc<kQ5_K, 2>(w, n, kk, xb, ldx, cols, yb, ldy, scale, ws, p, stream);
        else
            e = cudaErrorInvalidValue;
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace hesa_cuda
