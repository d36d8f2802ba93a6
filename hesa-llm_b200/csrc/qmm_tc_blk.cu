// qmm_tc_blk.cu -- batched Q8_0 / Q4_0 matmul on the 5th-generation tensor
// cores (tcgen05, TMEM, TMA; sm_100a): Y[b, :] = scale * W . X[b, :] for 2..8
// activation rows per launch (more rows: one launch per 8).
//
// The 32-weight blocks of Q8_0 and Q4_0 carry their own fp16 scale d, and a
// tcgen05.mma of kind::i8 has K = 32: one MMA per block, each into its own
// TMEM accumulator, D_j = q_j . X (M = 128 weight rows, N = 32 column planes:
// 3 digit planes x 8 activation rows, the batch-1 kernels' exact int8 form of
// x, xdigits.cuh). The block scales are applied afterwards in fp32, per block:
//   Q8_0: y_b += d_j * s_b * (65536*D2 + 256*D1 + D0)      (q signed, A = s8)
//   Q4_0: y_b += d_j * (s_b * (...) - 8 * sum_{k in j} x_bk) (q = 0..15, A = u8)
// Per unit of 256 weights (8 blocks) of a 128-row tile:
//   * transform warps (16 rows of the tile each, lanes over (row, block)
//     pieces so that their shared-memory reads meet no bank conflict) copy the
//     levels out of the TMA-staged GGUF blocks into the A operand in shared
//     memory (canonical K-major core matrices, one byte per level) and the
//     eight block scales of every row into a small header ring;
//   * one thread of the MMA warp issues the eight MMAs and commits them to an
//     mbarrier;
//   * epilogue warps (two per lane quarter, one per half of the activation
//     rows) read the accumulators back (tcgen05.ld) and scale them.
// The A operand (two 32 KB buffers in shared memory) and the accumulators (two
// sets of 8 x 32 TMEM columns: all 512) are double-buffered, so the transform
// of unit q+1, the MMAs of unit q and the epilogue of unit q-1 overlap. Work
// split, weight streaming (2-D TMA tensor copies of 128 rows, no multicast),
// the ticketed, ordered sum of K slices and the dependent-launch trigger after
// a CTA's last weight copy are those of qmm_tc.cu.
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
constexpr int kXWarps = 8;                          // transform warps, two per TMEM lane quarter
constexpr int kEWarps = 8;                          // epilogue warps, two per TMEM lane quarter
constexpr int kCompute = kXWarps + kEWarps;
constexpr int kThreads = (kCompute + 2) * 32;       // + the producer warp and the MMA warp
constexpr int kHdrRing = 4;                         // units' block scales in flight from transform to epilogue
constexpr int kWSlots = 3;
constexpr int kPlanSms = 148;
constexpr int kMaxCols = 8;                         // activation rows per launch
constexpr int kN = 32;                              // MMA N: 3 digit planes x 8 rows, padded
constexpr uint32_t kTmemCols = 512;                 // two accumulator buffers of 8 blocks x kN
constexpr int kMaxItems = 64;                       // items per CTA (tickets kept for the end)
constexpr size_t kSmemMax = 227 * 1024 - 10 * 1024;  // dynamic; the static header ring and barriers take the rest

// bytes of one unit (8 blocks) of a row, units per weight copy, units per slice
__host__ __device__ constexpr int blk_ub(int qt) { return qt == kQ8_0 ? 272 : 144; }
__host__ __device__ constexpr int blk_su(int qt) { return qt == kQ8_0 ? 1 : 2; }
__host__ __device__ constexpr int blk_ku(int qt) { return qt == kQ8_0 ? 6 : 5; }
template <int QT> __host__ __device__ constexpr uint32_t blk_slot() { return kRows * blk_su(QT) * blk_ub(QT); }
// per unit of the slice in shared memory: B operand [k-step 8][k half 2][kN/8][8 rows][16 B], then
// per activation row 12 floats: s, sum_k x_k over blocks 0..7, pad
constexpr uint32_t kXB = kN * 256;
constexpr uint32_t kXUB = kXB + 8 * 48;
// A operand of one unit-tile: [k-step 8][k half 2][row group 16][8 rows][16 B]; two buffers
constexpr uint32_t kAB = kRows * 256;
// column plane (B row, D column) of digit plane p of activation row b: each
// epilogue warp's 12 columns (rows 4h .. 4h+3, all planes) are contiguous
__host__ __device__ constexpr int tc_cp(int p, int b) { return (b >> 2) * 16 + p * 4 + (b & 3); }

// Wait for phase `parity` of `bar` by polling, without suspending the thread:
// for the MMA thread, which hands every unit on and whose wake-up from a
// suspending wait (measured ~0.3 us) would be on the critical path. Bounded like
// mbar_wait_bounded.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, int* status, int code) {
    if (mbar_test_wait(bar, parity)) return true;
    const unsigned long long t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_test_wait(bar, parity)) return true;
        if ((i & 255u) == 0 && global_timer_ns() - t0 > HESA_WAIT_LIMIT_NS) {
            record_status(status, code);
            return false;
        }
    }
}

// ---- tcgen05 --------------------------------------------------------------
// Shared-memory matrix descriptor, K-major without swizzle: start address,
// LBO = byte distance between the two 16-byte k halves of a k-step, SBO =
// byte distance between 8-row core matrices, descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// D = A . B (no accumulation), A and B from shared memory, kind::i8, one CTA.
__device__ __forceinline__ void tc_mma_ss(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(0), "r"(0)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// 16 consecutive columns of this warp's 32 lanes (one lane per thread)
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
// wait for this thread's tcgen05.ld; the registers are redefined after it so
// no use can be scheduled before the wait
template <int NC>
__device__ __forceinline__ void tc_wait_ld(uint32_t (&v)[NC]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < NC; ++i) asm volatile("" : "+r"(v[i]));
}


// Byte j (compile-time) of w, zero-extended.
template <int J>
__device__ __forceinline__ uint32_t byte_at(uint32_t w) {
    return prmt(w, 0u, 0x4440u + J);
}

// One warp: the eight activations of lane L (positions 8L..8L+7) of unit u of
// activation row b (zeros for b >= batch).
__device__ __forceinline__ void tc_load_pair(const float* __restrict__ x, int64_t ldx, int batch, int u, int b,
                                             int lane, float (&v)[8]) {
    if (b < batch) {
        const float4* src = reinterpret_cast<const float4*>(x + b * ldx + static_cast<int64_t>(u) * 256 + lane * 8);
        const float4 p = src[0], q = src[1];
        v[0] = p.x; v[1] = p.y; v[2] = p.z; v[3] = p.w;
        v[4] = q.x; v[5] = q.y; v[6] = q.z; v[7] = q.w;
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 0.f;
    }
}

// One warp: the digit planes of one unit of activation row b (loaded by
// tc_load_pair) into the unit's block at column planes tc_cp(p, b).
__device__ __forceinline__ void tc_store_pair(const float (&v)[8], int b, int lane, uint8_t* blk) {
    uint32_t dw[3][2];
    const float s = unit_digits(v, dw);
    // positions 8L..8L+7: k-step L/4, k half (L/2)&1, bytes 8(L&1)..+7 of the core row
    const int st = lane >> 2, h = (lane >> 1) & 1, off = 8 * (lane & 1);
#pragma unroll
    for (int p = 0; p < 3; ++p) {
        const int cp = tc_cp(p, b);
        *reinterpret_cast<uint2*>(blk + st * 2 * (kN / 8) * 128 + h * (kN / 8) * 128 + (cp >> 3) * 128 + (cp & 7) * 16 +
                                  off) = make_uint2(dw[p][0], dw[p][1]);
    }
    int sums[3];
#pragma unroll
    for (int p = 0; p < 3; ++p) {
        sums[p] = __dp4a(static_cast<int>(dw[p][0]), 0x01010101, __dp4a(static_cast<int>(dw[p][1]), 0x01010101, 0));
        sums[p] += __shfl_xor_sync(0xffffffffu, sums[p], 1);
        sums[p] += __shfl_xor_sync(0xffffffffu, sums[p], 2);
    }
    float* info = reinterpret_cast<float*>(blk + kXB) + b * 12;
    if ((lane & 3) == 0) info[1 + (lane >> 2)] = s * combine3(sums[0], sums[1], sums[2]);
    if (lane == 0) info[0] = s;
}

// One transform warp's share of a unit: rows 16w .. 16w+15 of the tile, all 8
// blocks, from the staged GGUF copy (row r's unit at `copy + r * row_stride +
// unit_off`) into the A operand `abuf` (block j of row r: 32 levels at
// k-step j, two 16-byte k halves) and the rows' fp16 block scales into
// `hdr` (row r: 8 scales in block order).
//
// Lanes take (row, block) pieces, not whole rows: the rows of a copy are 272
// (Q8_0) or 288 (Q4_0) bytes apart, so 32 lanes on 32 rows read four banks
// between them. Q8_0: a step is 8 rows x 4 blocks of one parity (blocks
// 0,2,4,6 start 0/17/2/19 words mod 32 into a row, rows 4 banks apart: all 32
// lanes on distinct banks), and each quarter-warp writes 8 rows of one block,
// 128 contiguous bytes of A. Q4_0: a step is 4 rows x 8 blocks (rows 8 banks
// apart, blocks 0,4,9,13,18,22,27,31 words in: distinct banks).
template <int QT>
__device__ __forceinline__ void blk_transform(const uint8_t* copy, int row_stride, int unit_off, uint8_t* abuf,
                                              uint4* hdr, int warp, int lane) {
    constexpr uint32_t AHALF = (kRows / 8) * 128, ASTEP = 2 * AHALF;
    auto put = [&](int r, int j, uint32_t d, const uint32_t (&lo)[4], const uint32_t (&hi)[4]) {
        uint8_t* dst = abuf + j * ASTEP + (r >> 3) * 128 + (r & 7) * 16;
        *reinterpret_cast<uint4*>(dst) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<uint4*>(dst + AHALF) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        reinterpret_cast<unsigned short*>(hdr + r)[j] = static_cast<unsigned short>(d);
    };
    if constexpr (QT == kQ8_0) {
#pragma unroll
        for (int g = 0; g < 2; ++g) {
#pragma unroll
            for (int par = 0; par < 2; ++par) {
                const int r = 16 * warp + 8 * g + (lane & 7);
                const int j = 2 * (lane >> 3) + par;
                // block j (34 bytes: d, then 32 levels) starts 34j bytes into the
                // unit: on a word boundary for even j, two bytes past one for odd j
                const uint8_t* b = copy + static_cast<size_t>(r) * row_stride + unit_off + 34 * j - 2 * par;
                uint32_t w[9];
#pragma unroll
                for (int c = 0; c < 9; ++c) w[c] = *reinterpret_cast<const uint32_t*>(b + 4 * c);
                uint32_t q[8];
#pragma unroll
                for (int c = 0; c < 8; ++c) q[c] = par ? w[c + 1] : prmt(w[c], w[c + 1], 0x5432u);
                const uint32_t lo[4] = {q[0], q[1], q[2], q[3]}, hi[4] = {q[4], q[5], q[6], q[7]};
                put(r, j, par ? (w[0] >> 16) : (w[0] & 0xFFFFu), lo, hi);
            }
        }
    } else {
#pragma unroll
        for (int st = 0; st < 4; ++st) {
            const int r = 16 * warp + 4 * st + (lane & 3);
            const int j = lane >> 2;
            // block j (18 bytes: d, then 16 bytes of nibbles) starts 18j bytes in:
            // on a word boundary for even j, two bytes past one for odd j
            const int sh = (18 * j) & 2;
            const uint8_t* b = copy + static_cast<size_t>(r) * row_stride + unit_off + 18 * j - sh;
            uint32_t w[5];
#pragma unroll
            for (int c = 0; c < 5; ++c) w[c] = *reinterpret_cast<const uint32_t*>(b + 4 * c);
            const uint32_t sel = sh ? 0x7654u : 0x5432u;
            uint32_t lo[4], hi[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                // byte i: level of weight i in the low nibble, of weight i + 16 in the high one
                const uint32_t qv = prmt(w[c], w[c + 1], sel);
                lo[c] = qv & 0x0F0F0F0Fu;
                hi[c] = (qv >> 4) & 0x0F0F0F0Fu;
            }
            put(r, j, (w[0] >> (8 * sh)) & 0xFFFFu, lo, hi);
        }
    }
}

template <int QT>
__global__ void __launch_bounds__(kThreads, 1)
qmm_blk_kernel(const __grid_constant__ CUtensorMap wmapN, const __grid_constant__ CUtensorMap wmap1, int n_out, int U,
               int S, const float* __restrict__ x, int64_t ldx, float* __restrict__ y, int64_t ldy, int batch,
               float scale, float* __restrict__ partials, int* __restrict__ tickets, int* __restrict__ status) {
    constexpr int UB = blk_ub(QT), SU = blk_su(QT), KU = blk_ku(QT), HB = kMaxCols / 2;
    constexpr uint32_t SLOT = blk_slot<QT>();
    // s32 accumulators, A = s8 (Q8_0) or u8 (Q4_0) levels, B = s8 digits, N = kN, M = 128
    constexpr uint32_t IDESC = (2u << 4) | ((QT == kQ8_0 ? 1u : 0u) << 7) | (1u << 10) |
                               (static_cast<uint32_t>(kN >> 3) << 17) | (static_cast<uint32_t>(kRows >> 4) << 24);
    constexpr uint32_t KSTEP = 2 * (kN / 8) * 128;     // B bytes per k-step
    constexpr uint32_t AHALF = (kRows / 8) * 128;     // A: byte distance of the two k halves of a k-step
    constexpr uint32_t ASTEP = 2 * AHALF;             // A bytes per k-step
    // shared memory: the slice's activation blocks, two A operands, the weight slots
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t wfull[kWSlots], wfree[kWSlots], aready[2], dready[2], dfree[2],
        hready[kHdrRing];
    __shared__ __align__(16) uint4 hdrs[kHdrRing][kRows];   // the 8 block scales (fp16) of the units in flight
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;
    __shared__ int item_old[kMaxItems];

    const int RT = (n_out + kRows - 1) / kRows;
    const int64_t I = static_cast<int64_t>(S) * RT, G = gridDim.x, cta = blockIdx.x;
    const int i0 = static_cast<int>(cta * I / G), i1 = static_cast<int>((cta + 1) * I / G);
    uint8_t* sx = smem;
    uint8_t* sa = smem + static_cast<size_t>(KU) * kXUB;
    uint8_t* sw = sa + 2 * kAB;
    volatile int* abort_v = &abort_flag;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    // the producer thread sets up its own barriers and issues the first weight
    // copies before the CTA-wide set-up (weights never depend on the previous
    // grid); the other roles touch these barriers only after it
    int cq = 0, it_p = i0, g_p = 0;   // producer position: next copy, item, copy within the item
    auto produce = [&](bool first_round) {
        while (it_p < i1 && !*abort_v) {
            const int s = it_p / RT, rt = it_p - s * RT;
            const int u0 = s * U / S, nu = (s + 1) * U / S - u0;
            if (SU * g_p >= nu) {
                ++it_p;
                g_p = 0;
                continue;
            }
            const int slot = cq % kWSlots;
            if (cq >= kWSlots) {
                if (first_round) return;   // the first round fills the free slots only
                if (!mbar_wait_bounded(&wfree[slot], static_cast<uint32_t>(cq / kWSlots - 1) & 1u, status,
                                       kStatusWaitTimeout)) {
                    *abort_v = 1;
                    return;
                }
            }
            const int wd = SU * g_p + SU <= nu ? SU : 1;
            mbar_arrive_expect_tx(&wfull[slot], static_cast<uint32_t>(kRows * wd * UB));
            tma_load_2d(sw + static_cast<size_t>(slot) * SLOT, wd == SU ? &wmapN : &wmap1, (u0 + SU * g_p) * UB / 2,
                        rt * kRows, &wfull[slot]);
            ++cq;
            ++g_p;
        }
    };
    if (threadIdx.x == kCompute * 32) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&wmapN) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&wmap1) : "memory");
        abort_flag = 0;
        for (int i = 0; i < kWSlots; ++i) {
            mbar_init(&wfull[i], 1);
            mbar_init(&wfree[i], kXWarps);
        }
        fence_mbar_init();
        produce(true);
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&aready[i], kXWarps);
            mbar_init(&dready[i], 1);
            mbar_init(&dfree[i], kEWarps);
        }
        for (int i = 0; i < kHdrRing; ++i) mbar_init(&hready[i], kXWarps);
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

    if (warp == kCompute) {
        // ---- producer: the remaining weight copies ----
        if (lane == 0) {
            produce(false);
            // every copy of this CTA is issued: the next kernel on the stream may
            // start its CTAs on the SMs this grid leaves (measured: Q8_0, B = 8 on
            // 4096 x 11008, 27.4 -> 24.8 us per matvec)
            grid_dep_launch();
            // the last copies into each slot have landed before the CTA may exit
            for (int c = cq > kWSlots ? cq - kWSlots : 0; c < cq; ++c)
                if (!mbar_wait_bounded(&wfull[c % kWSlots], static_cast<uint32_t>(c / kWSlots) & 1u, status,
                                       kStatusDrainTimeout))
                    break;
        }
        return;
    }
    if (warp == kCompute + 1) {
        // ---- MMA warp: one thread issues the eight block MMAs of every unit ----
        if (lane == 0) {
            int q = 0;
            const uint32_t a0 = smem_addr(sa);
            for (int it = i0; it < i1 && !*abort_v; ++it) {
                const int s = it / RT;
                const int nu = (s + 1) * U / S - s * U / S;
                for (int ui = 0; ui < nu; ++ui, ++q) {
                    bool go = mbar_wait_spin(&aready[q & 1], static_cast<uint32_t>(q >> 1) & 1u, status,
                                             kStatusWaitTimeout);
                    if (go && q >= 2)
                        go = mbar_wait_spin(&dfree[q & 1], static_cast<uint32_t>((q >> 1) - 1) & 1u, status,
                                            kStatusWaitTimeout);
                    if (!go || *abort_v) {
                        *abort_v = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem + static_cast<uint32_t>(256 * (q & 1));
                    const uint32_t ab = a0 + static_cast<uint32_t>(kAB * (q & 1));
                    const uint32_t xb = smem_addr(sx + static_cast<size_t>(ui) * kXUB);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        tc_mma_ss(d + static_cast<uint32_t>(kN * j), umma_desc(ab + j * ASTEP, AHALF, 128),
                                  umma_desc(xb + j * KSTEP, (kN / 8) * 128, 128), IDESC);
                    // completion frees A buffer q%2 for the transform warps and hands
                    // accumulator buffer q%2 to the epilogue warps
                    tc_commit(&dready[q & 1]);
                }
            }
        }
        return;
    }

    // ---- compute warps: transform warps 0..kXWarps-1, epilogue warps
    // kXWarps..kCompute-1. Warp w reaches TMEM lanes 32*(w%4) .. +31: its rows
    // of the tile. ----
    const bool is_x = warp < kXWarps;
    const int wq = warp & 3, hf = (is_x ? warp : warp - kXWarps) >> 2;
    const int row_t = 32 * wq + lane;                        // row within the tile = TMEM lane
    const uint32_t tlane = static_cast<uint32_t>(32 * wq) << 16;

    // the padding column planes of the activation blocks stay zero: clear them once
    {
        uint4* z = reinterpret_cast<uint4*>(sx);
        for (int i = threadIdx.x; i < static_cast<int>(KU * kXUB / 16); i += kCompute * 32) z[i] = make_uint4(0, 0, 0, 0);
    }
    grid_dep_wait();   // x may be written by the previous grid

    // every compute warp stages the slice's activations: all of a warp's loads
    // are in flight before it converts the first unit
    auto stage_slice = [&](int s) {
        constexpr int PW = (KU * kMaxCols + kCompute - 1) / kCompute;
        const int u0 = s * U / S, nu = (s + 1) * U / S - u0;
        const int P = nu * kMaxCols;   // (unit, activation row) pairs; rows >= batch are zeros
        float v[PW][8];
#pragma unroll
        for (int i = 0; i < PW; ++i) {
            const int pr = warp + i * kCompute;
            if (pr < P) tc_load_pair(x, ldx, batch, u0 + pr / kMaxCols, pr % kMaxCols, lane, v[i]);
        }
#pragma unroll
        for (int i = 0; i < PW; ++i) {
            const int pr = warp + i * kCompute;
            if (pr < P) tc_store_pair(v[i], pr % kMaxCols, lane, sx + static_cast<size_t>(pr / kMaxCols) * kXUB);
        }
        fence_proxy_async_smem();   // the tensor cores read the planes through the async proxy
        named_barrier(1, kCompute * 32);
    };

    int q = 0, cq_base = 0, cur_s = -1, n_items = 0;
    for (int it = i0; it < i1; ++it) {
        const int s = it / RT, rt = it - s * RT;
        const int nu = (s + 1) * U / S - s * U / S;
        if (s != cur_s) {
            // every MMA of the old slice is complete (the epilogue warps waited for the
            // last one) and no epilogue reads its activation sums any more
            if (cur_s >= 0) named_barrier(1, kCompute * 32);
            stage_slice(s);
            cur_s = s;
        }
        if (is_x) {
            // ---- transform: unit ui of this warp's 16 rows into A buffer q%2 ----
            for (int ui = 0; ui < nu; ++ui, ++q) {
                const int cqu = cq_base + ui / SU, slot = cqu % kWSlots;
                const int wd = SU * (ui / SU) + SU <= nu ? SU : 1;
                bool ok = !*abort_v;
                if (ok && ui % SU == 0) {
                    ok = mbar_wait_bounded(&wfull[slot], static_cast<uint32_t>(cqu / kWSlots) & 1u, status,
                                           kStatusWaitTimeout);
                    if (!ok) *abort_v = 1;
                }
                if (ok && q >= 2) {
                    // the MMAs of unit q-2 (the last reader of this A buffer) are complete
                    ok = mbar_wait_bounded(&dready[q & 1], static_cast<uint32_t>((q >> 1) - 1) & 1u, status,
                                           kStatusWaitTimeout);
                    if (!ok) *abort_v = 1;
                }
                ok = __all_sync(0xffffffffu, ok);
                if (ok) {
                    // a copy of wd units is [row][wd units]
                    blk_transform<QT>(sw + static_cast<size_t>(slot) * SLOT, wd * UB, (ui % SU) * UB,
                                      sa + static_cast<size_t>(kAB) * (q & 1), hdrs[q % kHdrRing], warp, lane);
                }
                fence_proxy_async_smem();   // the tensor cores read the operand through the async proxy
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&aready[q & 1]);
                    mbar_arrive(&hready[q % kHdrRing]);
                    if (ui % SU == SU - 1 || ui == nu - 1) mbar_arrive(&wfree[slot]);   // the copy is consumed
                }
                __syncwarp();
            }
            cq_base += (nu + SU - 1) / SU;
            continue;
        }

        // ---- epilogue: unit ui, this thread's row, activation rows 4hf .. 4hf+3 ----
        float acc[HB];
#pragma unroll
        for (int i = 0; i < HB; ++i) acc[i] = 0.f;
        for (int ui = 0; ui < nu; ++ui, ++q) {
            bool ok = !*abort_v;
            if (ok) {
                ok = mbar_wait_bounded(&dready[q & 1], static_cast<uint32_t>(q >> 1) & 1u, status, kStatusWaitTimeout);
                if (ok)
                    ok = mbar_wait_bounded(&hready[q % kHdrRing], static_cast<uint32_t>(q / kHdrRing) & 1u, status,
                                           kStatusWaitTimeout);
                if (!ok) *abort_v = 1;
            }
            ok = __all_sync(0xffffffffu, ok);
            tc_fence_after();
            if (ok) {
                // the scales are read before dfree lets the ring entry be rewritten
                const uint4 hp = hdrs[q % kHdrRing][row_t];
                const uint32_t dw[4] = {hp.x, hp.y, hp.z, hp.w};
                const float* info = reinterpret_cast<const float*>(sx + static_cast<size_t>(ui) * kXUB + kXB);
                float sb[HB];
#pragma unroll
                for (int jb = 0; jb < HB; ++jb) sb[jb] = info[(hf * HB + jb) * 12];
                const uint32_t d = tmem + tlane + static_cast<uint32_t>(256 * (q & 1) + 16 * hf);
#pragma unroll
                for (int j = 0; j < 8; j += 2) {
                    uint32_t va[16], vb[16];
                    tc_ld16(d + static_cast<uint32_t>(kN * j), va);
                    tc_ld16(d + static_cast<uint32_t>(kN * (j + 1)), vb);
                    tc_wait_ld<16>(va);
                    tc_wait_ld<16>(vb);
                    const float da = half_bits_to_float(dw[j >> 1]), db = half_bits_to_float(dw[j >> 1] >> 16);
#pragma unroll
                    for (int jb = 0; jb < HB; ++jb) {
                        const float ta = combine3(static_cast<int>(va[jb]), static_cast<int>(va[HB + jb]),
                                                  static_cast<int>(va[2 * HB + jb]));
                        const float tb = combine3(static_cast<int>(vb[jb]), static_cast<int>(vb[HB + jb]),
                                                  static_cast<int>(vb[2 * HB + jb]));
                        if constexpr (QT == kQ8_0) {
                            acc[jb] = fmaf(da * sb[jb], ta, acc[jb]);
                            acc[jb] = fmaf(db * sb[jb], tb, acc[jb]);
                        } else {
                            // the -8 offset of every level: 8 * sum of x over the block
                            const float* inf = info + (hf * HB + jb) * 12 + 1;
                            acc[jb] = fmaf(da, fmaf(sb[jb], ta, -8.f * inf[j]), acc[jb]);
                            acc[jb] = fmaf(db, fmaf(sb[jb], tb, -8.f * inf[j + 1]), acc[jb]);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&dfree[q & 1]);
        }

        // ---- item output: this thread's row, activation rows hf*HB .. +HB ----
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
            float* pr = partials + (static_cast<size_t>(s) * RT * kRows + rt * kRows + row_t) * kMaxCols + hf * HB;
#pragma unroll
            for (int jb = 0; jb < HB; ++jb) pr[jb] = acc[jb];   // the whole tile, rows past n_out included
            named_barrier(2, kEWarps * 32);
            if (threadIdx.x == kXWarps * 32) {
                // the ticket's result is only needed at the end: its latency hides behind the next items
                cuda::atomic_ref<int, cuda::thread_scope_device> tk(tickets[rt]);
                item_old[n_items < kMaxItems ? n_items : kMaxItems - 1] = tk.fetch_add(1, cuda::memory_order_acq_rel);
            }
        }
        ++n_items;
    }

    // ---- the slice sums of the tiles this CTA finished last, in slice order ----
    if (!is_x) {
        named_barrier(2, kEWarps * 32);
        if (S > 1 && !*abort_v) {
            int k = 0;
            for (int it = i0; it < i1; ++it, ++k) {
                const int rt = it % RT;
                if (item_old[k] != S - 1) continue;
                const int row = rt * kRows + row_t;
                float sum[HB];
#pragma unroll
                for (int jb = 0; jb < HB; ++jb) sum[jb] = 0.f;
                // four slices' loads in flight at a time; the sum order stays the slice order
#pragma unroll 4
                for (int ss = 0; ss < S; ++ss) {
                    const float4 v = __ldcg(reinterpret_cast<const float4*>(
                        partials + (static_cast<size_t>(ss) * RT * kRows + rt * kRows + row_t) * kMaxCols + hf * HB));
                    sum[0] += v.x;
                    sum[1] += v.y;
                    sum[2] += v.z;
                    sum[3] += v.w;
                }
                if (row < n_out) {
#pragma unroll
                    for (int jb = 0; jb < HB; ++jb) {
                        const int b = hf * HB + jb;
                        if (b < batch) y[b * ldy + row] = sum[jb] * scale;
                    }
                }
                if (threadIdx.x == kXWarps * 32) tickets[rt] = 0;   // leave the workspace zeroed
            }
        }
    }
    tc_fence_before();
    named_barrier(1, kCompute * 32);
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

static_assert(kMaxCols == 8 && kN == 32, "the epilogue's column layout assumes 8 activation rows per launch");

struct BlkPlan {
    int S, grid;
    size_t smem, part_bytes, ticket_bytes;
};

constexpr size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

BlkPlan make_blk_plan(int qt, int64_t n_out, int64_t k) {
    BlkPlan p{};
    const int KU = blk_ku(qt);
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
    const size_t slots = static_cast<size_t>(kWSlots) * (qt == kQ8_0 ? blk_slot<kQ8_0>() : blk_slot<kQ4_0>());
    p.smem = static_cast<size_t>(KU) * kXUB + 2 * kAB + slots;
    p.part_bytes = p.S > 1 ? align256(static_cast<size_t>(p.S) * RT * kRows * kMaxCols * 4) : 0;
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

template <int QT>
cudaError_t launch_blk(const void* w, int n_out, int k, const float* x, int64_t ldx, int cols, float* y, int64_t ldy,
                       float scale, uint8_t* ws, const BlkPlan& p, cudaStream_t stream) {
    constexpr int UB = blk_ub(QT), SU = blk_su(QT);
    const int U = k / 256;
    CUtensorMap mN, m1;
    if (!encode_wmap(&mN, w, n_out, static_cast<int64_t>(U) * UB, SU, UB) ||
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
        e = cudaFuncSetAttribute(qmm_blk_kernel<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
    return cudaLaunchKernelEx(&cfg, qmm_blk_kernel<QT>, mN, m1, n_out, U, p.S, x, ldx, y, ldy, cols, scale, partials,
                              tickets, status);
}

}  // namespace

bool qmm_blk_eligible(int qtype, const void* w, int64_t n_out, int64_t k, int64_t batch) {
    if (qtype != kQ8_0 && qtype != kQ4_0) return false;
    if (batch < 2 || n_out <= 0 || k <= 0 || k % 256 != 0) return false;
    if ((reinterpret_cast<uintptr_t>(w) & 15) != 0) return false;
    // items per CTA are bounded by the ticket list; the tensor map takes rows
    // of up to 2^32 elements and 2^31 - 1 rows
    const BlkPlan p = make_blk_plan(qtype, n_out, k);
    const int64_t RT = (n_out + kRows - 1) / kRows;
    return (static_cast<int64_t>(p.S) * RT + p.grid - 1) / p.grid <= kMaxItems && n_out < (int64_t(1) << 31) &&
           p.smem <= kSmemMax;
}

size_t qmm_blk_workspace_bytes(int qtype, int64_t n_out, int64_t k, int64_t batch) {
    if ((qtype != kQ8_0 && qtype != kQ4_0) || batch < 2 || k % 256 != 0) return 0;
    // every launch (8 activation rows, or the remainder) has the same plan
    const BlkPlan p = make_blk_plan(qtype, n_out, k);
    return p.ticket_bytes + p.part_bytes;
}

cudaError_t qmm_blk(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, int64_t ldx, int64_t batch,
                    float* y, int64_t ldy, float scale, void* workspace, cudaStream_t stream) {
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const BlkPlan p = make_blk_plan(qtype, n_out, k);
    for (int64_t b0 = 0; b0 < batch; b0 += kMaxCols) {
        const int cols = static_cast<int>(batch - b0 < kMaxCols ? batch - b0 : kMaxCols);
        const float* xb = x + b0 * ldx;
        float* yb = y + b0 * ldy;
        const int n = static_cast<int>(n_out), kk = static_cast<int>(k);
        cudaError_t e;
        if (qtype == kQ8_0)
            e = launch_blk<kQ8_0>(w, n, kk, xb, ldx, cols, yb, ldy, scale, ws, p, stream);
        else if (qtype == kQ4_0)
            e = launch_blk<kQ4_0>(w, n, kk, xb, ldx, cols, yb, ldy, scale, ws, p, stream);
        else
            e = cudaErrorInvalidValue;
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace hesa_cuda
