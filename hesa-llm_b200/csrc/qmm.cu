// qmm.cu -- batched quantized matmul on the tensor cores (sm_100a):
// Y[b, :] = scale * W . X[b, :] for 2..16 activation rows per launch,
// W packed Q4_K / Q5_K rows.
//
// Numerics are the batch-1 kernels' (qmatvec.cu): per unit of 256
// activations and per activation row, X = rint(x / s) as three balanced int8
// digit planes (xdigits.cuh). Every product of a weight level with a digit is
// exact in int32: mma.sync m16n8k32 u8 x s8 -> s32 takes the (scale-folded)
// levels as A (16 weight rows x 32 k) and the digit planes as B (32 k x 8
// "column planes", one (activation row, plane) pair each); the three planes
// are combined in fp32 once per unit, with the min terms
// dmin * m_j * sum(x over sub-block j) taken from per-sub-block sums of the
// staged activations.
//
// One launch (qmm_kernel): every CTA owns a K-slice of the units and a range
// of rows. It converts its slice's activations into shared memory in the
// exact order of the MMA B fragments (one conflict-free 128-bit shared load
// per lane and fragment pair), streams its rows through a ring of slots with
// bulk copies, and adds the slices of a row range through a ticket (the last
// slice to finish adds them in slice order), so results do not depend on
// scheduling.
//
// The k order inside one MMA is permuted (a thread's 8 contiguous weight
// bytes feed its k slots 4t..4t+3 and 16+4t..16+4t+3); the staged digits use
// the same permutation, so the dot products are unchanged.
#include "hesa_common.cuh"
#include "qtypes.cuh"
#include "xdigits.cuh"
#include "qmm.h"
#include "qmatvec.h"

#include <cuda/atomic>

namespace hesa_cuda {

namespace {

constexpr int kFragBytes = 512;         // B fragments of one (unit, 64-k chunk, n-tile)
constexpr int kInfoFloats = 12;         // per (unit, activation row): s, xs[8], pad
constexpr int kPlanSms = 148;           // grid of at most one CTA on each of 148 SMs
constexpr int kMaxColsPerLaunch = 16;

__host__ __device__ constexpr int qmm_unit_bytes(int qt) { return qt == kQ4_K ? 144 : 176; }
__host__ __device__ constexpr int qmm_qs_offset(int qt) { return qt == kQ4_K ? 16 : 48; }

__device__ __forceinline__ uint2 lds64(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint4 lds128q(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// ---------------------------------------------------------------------------
// Activation staging: one warp per (unit, activation row). Lane L holds positions
// 8L..8L+7 of the unit; they belong to 64-k chunk c = L/8 and feed the B
// fragment of MMA thread (g = row % 8, t = L % 4), half (L/4) % 2: bytes
// 0..7 are its sub-block 2c digits, bytes 8..15 its sub-block 2c+1 digits.
// Rows >= batch (padding up to 8 or 16) stage zeros.
// A unit block (xunit_bytes<NBT>() bytes, one per unit of the slice):
//   [chunk 4][n-tile NT][lane 32][16 B] B fragments, n-tile = plane * NBT + row / 8
//   [row BP][12 floats]: s, then sum_k x_k over sub-blocks 0..7
// ---------------------------------------------------------------------------
template <int NBT>
__host__ __device__ constexpr uint32_t xunit_bytes() {
    return 4 * 3 * NBT * kFragBytes + 8 * NBT * kInfoFloats * 4;
}

// One warp: unit u of activation row b (zeros for b >= batch) into the unit's
// block `blk` (fragments, then s and the sub-block sums), as described above.
template <int NBT>
__device__ __forceinline__ void stage_pair(const float* __restrict__ x, int64_t ldx, int batch, int u, int b, int lane,
                                           uint8_t* blk) {
    constexpr int NT = 3 * NBT;
    float v[8];
    if (b < batch) {
        const float4* src = reinterpret_cast<const float4*>(x + b * ldx + static_cast<int64_t>(u) * 256 + lane * 8);
        const float4 p = src[0], q = src[1];
        v[0] = p.x; v[1] = p.y; v[2] = p.z; v[3] = p.w;
        v[4] = q.x; v[5] = q.y; v[6] = q.z; v[7] = q.w;
    } else {
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) v[jj] = 0.f;
    }
    uint32_t dw[3][2];
    const float s = unit_digits(v, dw);
    const int c = lane >> 3, half = (lane >> 2) & 1, t = lane & 3;
    uint8_t* dst = blk + c * NT * kFragBytes + ((b & 7) * 4 + t) * 16 + half * 8;
#pragma unroll
    for (int p = 0; p < 3; ++p)
        *reinterpret_cast<uint2*>(dst + (p * NBT + (b >> 3)) * kFragBytes) = make_uint2(dw[p][0], dw[p][1]);
    // digit sums of sub-block lane/4 (four lanes, 32 positions)
    int sums[3];
#pragma unroll
    for (int p = 0; p < 3; ++p) {
        sums[p] = __dp4a(static_cast<int>(dw[p][0]), 0x01010101, __dp4a(static_cast<int>(dw[p][1]), 0x01010101, 0));
        sums[p] += __shfl_xor_sync(0xffffffffu, sums[p], 1);
        sums[p] += __shfl_xor_sync(0xffffffffu, sums[p], 2);
    }
    float* info = reinterpret_cast<float*>(blk + 4 * NT * kFragBytes) + b * kInfoFloats;
    if ((lane & 3) == 0) info[1 + (lane >> 2)] = s * combine3(sums[0], sums[1], sums[2]);
    if (lane == 0) info[0] = s;
}

// ---------------------------------------------------------------------------
// Matmul (qmm_kernel). Grid: S K-slices x P row ranges (S * P <= 148), one CTA
// per SM. CTA (s, p):
//   * units [u0, u1) of slice s (U split into S near-equal runs of at most KU
//     units): their staged activations are copied into shared memory once;
//   * rows [r0, r1) of range p (the m16 tiles split into P near-equal runs),
//     streamed 32 rows at a time through a ring of slots: one bulk copy per
//     row (its (u1 - u0) units, a contiguous run of about 1 KB), issued by
//     the 32 lanes of one warp at once; rows are padded in shared memory to a
//     stride of 32 mod 128 bytes so fragment loads do not conflict;
//   * 2*KU warps, (m16 tile of the slot) x (unit of the slice); after each
//     slot the units are added in unit order in shared memory and the slot's
//     rows written to y (S = 1) or as this slice's partial;
//   * S > 1: the last CTA of a row range to finish (ticket) adds the S
//     partials in slice order, so results do not depend on scheduling.
// ---------------------------------------------------------------------------
constexpr int kSlotRows = 32;
constexpr int kMaxSlots = 8;
constexpr size_t kSmemMax = 227 * 1024 - 1024;   // dynamic part: the 227 KB per block less room for static

// Units per slice at most: 8 for up to 8 activation rows, 6 for up to 16.
template <int NBT> __host__ __device__ constexpr int qmm_ku() { return NBT == 1 ? 8 : 6; }
template <int NBT> __host__ __device__ constexpr int qmm_threads() { return 2 * qmm_ku<NBT>() * 32; }

// D += A . B (u8 x s8 -> s32) for one m16n8k32 tile.
__device__ __forceinline__ void mma_u8s8_acc(const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int (&d)[4]) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// The 6-bit scales and mins of the eight sub-blocks of a K-quant block, one
// byte each: sc[0..3], sc[4..7], m[0..3], m[4..7] (the packing of
// kq_scale_min, all eight at once; h.y..h.w = the 12-byte scale field).
__device__ __forceinline__ void kq_unpack8(const uint4& h, uint32_t& sc03, uint32_t& sc47, uint32_t& m03,
                                           uint32_t& m47) {
    sc03 = h.y & 0x3F3F3F3Fu;
    m03 = h.z & 0x3F3F3F3Fu;
    sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    m47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
}

// Byte j (compile-time) of w, zero-extended.
template <int J>
__device__ __forceinline__ uint32_t byte_of(uint32_t w) {
    return prmt(w, 0u, 0x4440u + J);
}

// One unit (256 k) of MT m16 tiles of weight rows (rows row0 .. +16*MT,
// `wst` bytes apart, starting at the unit's block) against every activation
// row, added to acc[m-tile][row half][n-tile][col].
//
// The sub-block scale is folded into the weight operand: sc = lo + 2^S hi
// with S = 4 (Q4_K: q <= 15, lo <= 15, hi <= 3) or 3 (Q5_K: q <= 31,
// lo, hi <= 7), so q*lo and q*hi fit a byte and one 32-bit multiply scales
// four packed levels without carries. The two halves accumulate inside the
// MMA over the whole unit (no per-sub-block integer multiply-add), and the
// unit's integer dot per digit plane is acc_lo + 2^S acc_hi (|.| < 2^26).
template <int QT, int NBT, int MT>
__device__ __forceinline__ void qmm_unit(const uint8_t* sw, int wst, const uint8_t* sxf, const float* sinf, int row0,
                                         int lane, float (&acc)[MT][2][NBT][2]) {
    constexpr int NT = 3 * NBT, QO = qmm_qs_offset(QT);
    constexpr int SB = QT == kQ4_K ? 4 : 3;
    constexpr uint32_t LOM = QT == kQ4_K ? 0x0F0F0F0Fu : 0x07070707u;
    const int g = lane >> 2, t = lane & 3;
    const uint8_t* ub[MT][2];
    uint4 hd[MT][2];
    uint32_t slo[MT][2][2], shi[MT][2][2];   // [m-tile][row half][sc 0..3 / 4..7], packed bytes
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            ub[mt][h] = sw + (row0 + 16 * mt + 8 * h + g) * wst;
            hd[mt][h] = lds128q(ub[mt][h]);
            uint32_t sc03, sc47, m03, m47;
            kq_unpack8(hd[mt][h], sc03, sc47, m03, m47);
            slo[mt][h][0] = sc03 & LOM;
            slo[mt][h][1] = sc47 & LOM;
            shi[mt][h][0] = (sc03 >> SB) & LOM;
            shi[mt][h][1] = (sc47 >> SB) & LOM;
        }
    int alo_acc[MT][NT][4], ahi_acc[MT][NT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int r = 0; r < 4; ++r) alo_acc[mt][n][r] = ahi_acc[mt][n][r] = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint4 xf[NT];
#pragma unroll
        for (int n = 0; n < NT; ++n) xf[n] = lds128q(sxf + (c * NT + n) * kFragBytes + lane * 16);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const uint2 q0 = lds64(ub[mt][0] + QO + 32 * c + 8 * t);
            const uint2 q1 = lds64(ub[mt][1] + QO + 32 * c + 8 * t);
            // levels of sub-blocks 2c (low nibbles) and 2c+1 (high nibbles); A
            // register order: (row g, k 0-3), (row g+8, k 0-3), (row g, k 16-19), (row g+8, k 16-19)
            uint32_t qa[4] = {q0.x & 0x0F0F0F0Fu, q1.x & 0x0F0F0F0Fu, q0.y & 0x0F0F0F0Fu, q1.y & 0x0F0F0F0Fu};
            uint32_t qb[4] = {(q0.x >> 4) & 0x0F0F0F0Fu, (q1.x >> 4) & 0x0F0F0F0Fu, (q0.y >> 4) & 0x0F0F0F0Fu,
                              (q1.y >> 4) & 0x0F0F0F0Fu};
            if constexpr (QT == kQ5_K) {
                // fifth bit of weight l of sub-block j: bit j of qh[l]
                const uint2 h0 = lds64(ub[mt][0] + 16 + 8 * t);
                const uint2 h1 = lds64(ub[mt][1] + 16 + 8 * t);
                const uint32_t hv[4] = {h0.x >> (2 * c), h1.x >> (2 * c), h0.y >> (2 * c), h1.y >> (2 * c)};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    qa[i] |= (hv[i] << 4) & 0x10101010u;
                    qb[i] |= (hv[i] << 3) & 0x10101010u;
                }
            }
            // scale halves of sub-blocks 2c, 2c+1 for rows g (h 0) and g+8 (h 1)
            const int wsel = c >> 1;
            const uint32_t la0 = (2 * c) % 4 == 0 ? byte_of<0>(slo[mt][0][wsel]) : byte_of<2>(slo[mt][0][wsel]);
            const uint32_t la1 = (2 * c) % 4 == 0 ? byte_of<0>(slo[mt][1][wsel]) : byte_of<2>(slo[mt][1][wsel]);
            const uint32_t lb0 = (2 * c) % 4 == 0 ? byte_of<1>(slo[mt][0][wsel]) : byte_of<3>(slo[mt][0][wsel]);
            const uint32_t lb1 = (2 * c) % 4 == 0 ? byte_of<1>(slo[mt][1][wsel]) : byte_of<3>(slo[mt][1][wsel]);
            const uint32_t ha0 = (2 * c) % 4 == 0 ? byte_of<0>(shi[mt][0][wsel]) : byte_of<2>(shi[mt][0][wsel]);
            const uint32_t ha1 = (2 * c) % 4 == 0 ? byte_of<0>(shi[mt][1][wsel]) : byte_of<2>(shi[mt][1][wsel]);
            const uint32_t hb0 = (2 * c) % 4 == 0 ? byte_of<1>(shi[mt][0][wsel]) : byte_of<3>(shi[mt][0][wsel]);
            const uint32_t hb1 = (2 * c) % 4 == 0 ? byte_of<1>(shi[mt][1][wsel]) : byte_of<3>(shi[mt][1][wsel]);
            const uint32_t a_lo_a[4] = {qa[0] * la0, qa[1] * la1, qa[2] * la0, qa[3] * la1};
            const uint32_t a_hi_a[4] = {qa[0] * ha0, qa[1] * ha1, qa[2] * ha0, qa[3] * ha1};
            const uint32_t a_lo_b[4] = {qb[0] * lb0, qb[1] * lb1, qb[2] * lb0, qb[3] * lb1};
            const uint32_t a_hi_b[4] = {qb[0] * hb0, qb[1] * hb1, qb[2] * hb0, qb[3] * hb1};
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                mma_u8s8_acc(a_lo_a, xf[n].x, xf[n].y, alo_acc[mt][n]);
                mma_u8s8_acc(a_hi_a, xf[n].x, xf[n].y, ahi_acc[mt][n]);
                mma_u8s8_acc(a_lo_b, xf[n].z, xf[n].w, alo_acc[mt][n]);
                mma_u8s8_acc(a_hi_b, xf[n].z, xf[n].w, ahi_acc[mt][n]);
            }
        }
    }
    // planes -> fp32, row scales, min terms
    float rd[MT][2], rdmin[MT][2], rm[MT][2][8];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            rd[mt][h] = half_bits_to_float(hd[mt][h].x);
            rdmin[mt][h] = half_bits_to_float(hd[mt][h].x >> 16);
            uint32_t sc03, sc47, m03, m47;
            kq_unpack8(hd[mt][h], sc03, sc47, m03, m47);
            rm[mt][h][0] = static_cast<float>(byte_of<0>(m03));
            rm[mt][h][1] = static_cast<float>(byte_of<1>(m03));
            rm[mt][h][2] = static_cast<float>(byte_of<2>(m03));
            rm[mt][h][3] = static_cast<float>(byte_of<3>(m03));
            rm[mt][h][4] = static_cast<float>(byte_of<0>(m47));
            rm[mt][h][5] = static_cast<float>(byte_of<1>(m47));
            rm[mt][h][6] = static_cast<float>(byte_of<2>(m47));
            rm[mt][h][7] = static_cast<float>(byte_of<3>(m47));
        }
#pragma unroll
    for (int tb = 0; tb < NBT; ++tb)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            // column 8*tb + 2*t + e: its scale s and sub-block sums
            const float* inf = sinf + (8 * tb + 2 * t + e) * kInfoFloats;
            const float4 i0 = *reinterpret_cast<const float4*>(inf);
            const float4 i1 = *reinterpret_cast<const float4*>(inf + 4);
            const float cx[8] = {i0.y, i0.z, i0.w, i1.x, i1.y, i1.z, i1.w, inf[8]};
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int ci = 2 * h + e;
                    int pl[3];
#pragma unroll
                    for (int p = 0; p < 3; ++p)
                        pl[p] = alo_acc[mt][p * NBT + tb][ci] + (ahi_acc[mt][p * NBT + tb][ci] << SB);
                    const float tv = combine3(pl[0], pl[1], pl[2]);
                    float mins = rm[mt][h][0] * cx[0];
#pragma unroll
                    for (int q = 1; q < 8; ++q) mins = fmaf(rm[mt][h][q], cx[q], mins);
                    acc[mt][h][tb][e] += fmaf(rd[mt][h] * i0.x, tv, -rdmin[mt][h] * mins);
                }
        }
}

template <int QT, int NBT>
__global__ void __launch_bounds__(qmm_threads<NBT>(), 1)
qmm_kernel(const uint8_t* __restrict__ w, int n_out, int U, int S, int P, const float* __restrict__ x, int64_t ldx,
           float* __restrict__ y, int64_t ldy, int batch, float scale, int n_slots, int wst,
           float* __restrict__ partials, int* __restrict__ tickets, int* __restrict__ status) {
    constexpr int BP = 8 * NBT, NT = 3 * NBT, UB = qmm_unit_bytes(QT), KU = qmm_ku<NBT>(), kAcc = 4 * NBT;
    constexpr int kWarps = 2 * KU, kThreads = kWarps * 32;
    constexpr uint32_t XB = 4 * NT * kFragBytes, XUB = xunit_bytes<NBT>();
    constexpr int kRed = 2 * KU * 32 * kAcc;   // floats per buffer: (m16 tile, unit, lane)
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int abort_flag, last_flag, issued_hi;

    const int s = blockIdx.x % S, p = blockIdx.x / S;
    const int u0 = s * U / S, u1 = (s + 1) * U / S, nu = u1 - u0;
    const int m16 = (n_out + 15) / 16;
    const int r0 = 16 * static_cast<int>(static_cast<int64_t>(p) * m16 / P);
    const int r1 = min(n_out, 16 * static_cast<int>(static_cast<int64_t>(p + 1) * m16 / P));
    const int n_chunks = (r1 - r0 + kSlotRows - 1) / kSlotRows;
    const size_t pitch = static_cast<size_t>(U) * UB;
    const uint32_t seg = static_cast<uint32_t>(nu) * UB;
    const size_t slot_bytes = static_cast<size_t>(kSlotRows) * wst;

    uint8_t* sx = smem;
    uint8_t* slots = sx + static_cast<size_t>(KU) * XUB;
    float* red = reinterpret_cast<float*>(slots + static_cast<size_t>(n_slots) * slot_bytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * kRed);
    volatile int* abort_v = &abort_flag;

    // chunk j (rows r0 + 32j ..) into slot j % n_slots: one row per lane of the calling warp
    auto issue_rows = [&](int j, int lane) {
        const int slot = j % n_slots;
        const int rb = r0 + j * kSlotRows;
        const int nr = min(kSlotRows, r1 - rb);
        if (lane == 0) mbar_arrive_expect_tx(&full[slot], seg * static_cast<uint32_t>(nr));
        __syncwarp();
        if (lane < nr) {
            fence_proxy_async_smem();
            bulk_g2s(slots + slot * slot_bytes + lane * wst, w + static_cast<size_t>(rb + lane) * pitch +
                     static_cast<size_t>(u0) * UB, seg, &full[slot]);
        }
    };

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        for (int q = 0; q < n_slots; ++q) mbar_init(&full[q], 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == 0) {
        const int first = n_chunks < n_slots ? n_chunks : n_slots;
        for (int j = 0; j < first; ++j) issue_rows(j, lane);   // the weights do not depend on earlier grids
        if (lane == 0) issued_hi = first;
    }
    // the activations of the slice, converted in place (x may come from the previous grid)
    grid_dep_wait();
    for (int pr = warp; pr < nu * BP; pr += kWarps)
        stage_pair<NBT>(x, ldx, batch, u0 + pr / BP, pr % BP, lane, sx + static_cast<size_t>(pr / BP) * XUB);
    __syncthreads();

    const int mt = warp & 1, ph = warp >> 1;
    for (int j = 0; j < n_chunks; ++j) {
        const int slot = j % n_slots;
        float acc[1][2][NBT][2];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int tb = 0; tb < NBT; ++tb) acc[0][h][tb][0] = acc[0][h][tb][1] = 0.f;
        bool landed = false;
        if (!*abort_v) {
            landed = mbar_wait_bounded(&full[slot], static_cast<uint32_t>(j / n_slots) & 1u, status,
                                       kStatusWaitTimeout);
            if (!landed) *abort_v = 1;
        }
        if (__all_sync(0xffffffffu, landed)) {
            for (int uu = ph; uu < nu; uu += KU)
                qmm_unit<QT, NBT, 1>(slots + slot * slot_bytes + uu * UB, wst, sx + static_cast<size_t>(uu) * XUB,
                                     reinterpret_cast<const float*>(sx + static_cast<size_t>(uu) * XUB + XB), 16 * mt,
                                     lane, acc);
        }
        // slot end: the units meet in shared memory (double-buffered by slot parity)
        float* rbuf = red + (j & 1) * kRed;
        {
            float* r = rbuf + ((mt * KU + ph) * 32 + lane) * kAcc;
            int i = 0;
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int tb = 0; tb < NBT; ++tb)
#pragma unroll
                    for (int e = 0; e < 2; ++e) r[i++] = acc[0][h][tb][e];
        }
        named_barrier(1, kThreads);   // every warp is also done with the slot's rows
        if (warp == kWarps - 1 && j + n_slots < n_chunks && !*abort_v) {
            issue_rows(j + n_slots, lane);
            if (lane == 0) issued_hi = j + n_slots + 1;
        }
        // units added in unit order, every thread a share of the chunk's (row, column) pairs
        for (int idx = threadIdx.x; idx < kSlotRows * BP; idx += kThreads) {
            const int rr = idx / BP, b = idx - rr * BP;
            const int m = rr >> 4, h = (rr >> 3) & 1, ln = (rr & 7) * 4 + ((b >> 1) & 3);
            const int i = (h * NBT + (b >> 3)) * 2 + (b & 1);
            float v = 0.f;
#pragma unroll
            for (int q = 0; q < KU; ++q) v += rbuf[((m * KU + q) * 32 + ln) * kAcc + i];
            const int row = r0 + j * kSlotRows + rr;
            if (row < r1 && b < batch) {
                if (S == 1)
                    y[b * ldy + row] = v * scale;
                else
                    partials[(static_cast<size_t>(s) * n_out + row) * BP + b] = v;
            }
        }
    }

    __syncthreads();
    if (*abort_v) {
        // error exit: wait (bounded) for the copies still in flight
        if (threadIdx.x == 0) {
            for (int j = issued_hi > n_slots ? issued_hi - n_slots : 0; j < issued_hi; ++j)
                if (!mbar_wait_bounded(&full[j % n_slots], static_cast<uint32_t>(j / n_slots) & 1u, status,
                                       kStatusDrainTimeout))
                    break;
        }
        return;
    }
    if (S == 1) return;
    // the last slice to finish adds the S partials of the row range in slice order
    if (threadIdx.x == 0) {
        cuda::atomic_ref<int, cuda::thread_scope_device> tk(tickets[p]);
        const int old = tk.fetch_add(1, cuda::memory_order_acq_rel);
        last_flag = old == S - 1;
        if (old == S - 1) tk.store(0, cuda::memory_order_relaxed);   // leave it zeroed
    }
    __syncthreads();
    if (!last_flag) return;
    const int nr = r1 - r0;
    for (int idx = threadIdx.x; idx < nr * BP; idx += kThreads) {
        const int row = r0 + idx / BP, b = idx - (idx / BP) * BP;
        const float* pp = partials + static_cast<size_t>(row) * BP + b;
        float sum = 0.f;
#pragma unroll 4
        for (int ss = 0; ss < S; ++ss) sum += __ldcg(pp + static_cast<size_t>(ss) * n_out * BP);
        if (b < batch) y[b * ldy + row] = sum * scale;
    }
}

struct QmmPlan {
    int nbt, S, P, n_slots, wst;
    size_t smem, part_bytes, ticket_bytes;
};

constexpr size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

QmmPlan make_plan(int qt, int64_t n_out, int64_t k, int cols) {
    QmmPlan p{};
    p.nbt = cols <= 8 ? 1 : 2;
    const int KU = p.nbt == 1 ? qmm_ku<1>() : qmm_ku<2>(), BP = 8 * p.nbt, UB = qmm_unit_bytes(qt);
    const size_t XUB = p.nbt == 1 ? xunit_bytes<1>() : xunit_bytes<2>();
    const int U = static_cast<int>(k / 256);
    const int m16 = static_cast<int>((n_out + 15) / 16);
    p.S = (U + KU - 1) / KU;
    p.P = kPlanSms / p.S;
    if (p.P < 1) p.P = 1;
    if (p.P > m16) p.P = m16;
    int st = ((KU * UB + 15) / 16) * 16;
    st += ((32 - st % 128) + 128) % 128;   // rows 32 bytes apart modulo 128: conflict-free fragment loads
    p.wst = st;
    const size_t xs = static_cast<size_t>(KU) * XUB;
    const size_t red = static_cast<size_t>(2) * 2 * KU * 32 * (4 * p.nbt) * 4;
    const size_t bars = kMaxSlots * 8;
    const size_t slot = static_cast<size_t>(kSlotRows) * st;
    size_t ns = (kSmemMax - xs - red - bars) / slot;
    if (ns > static_cast<size_t>(kMaxSlots)) ns = kMaxSlots;
    p.n_slots = static_cast<int>(ns);
    p.smem = xs + ns * slot + red + bars;
    p.part_bytes = p.S > 1 ? align256(static_cast<size_t>(p.S) * n_out * BP * 4) : 0;
    // the tickets sit at the start of the workspace inside a region as large
    // as the batch-1 split-row kernel's arrival counters (one int per 2 rows):
    // the parts of a shared workspace that must stay zero coincide, and each
    // kernel's scratch only overlaps the other's scratch
    p.ticket_bytes = align256(((static_cast<size_t>(n_out) + 1) / 2) * 4);
    return p;
}

size_t plan_workspace(const QmmPlan& p) { return p.ticket_bytes + p.part_bytes; }

template <int QT, int NBT>
cudaError_t launch_qmm(const uint8_t* w, int n_out, int k, const float* x, int64_t ldx, int cols, float* y,
                       int64_t ldy, float scale, uint8_t* ws, const QmmPlan& p, cudaStream_t stream) {
    const int U = k / 256;
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
        e = cudaFuncSetAttribute(qmm_kernel<QT, NBT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kSmemMax));
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(p.S * p.P), 1, 1);
    cfg.blockDim = dim3(qmm_threads<NBT>(), 1, 1);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, qmm_kernel<QT, NBT>, w, n_out, U, p.S, p.P, x, ldx, y, ldy, cols, scale,
                              p.n_slots, p.wst, partials, tickets, status);
}

}  // namespace

bool qmm_eligible(int qtype, const void* w, int64_t n_out, int64_t k, int64_t batch) {
    if (qtype != kQ4_K && qtype != kQ5_K) return false;
    if (batch < 2 || n_out <= 0 || k <= 0 || k % 256 != 0) return false;
    if ((reinterpret_cast<uintptr_t>(w) & 15) != 0) return false;
    // a row segment of a slice is one bulk copy (< 2^32 bytes); rows index in int
    return n_out < (int64_t(1) << 31) && k < (int64_t(1) << 31);
}

size_t qmm_workspace_bytes(int qtype, int64_t n_out, int64_t k, int64_t batch) {
    if (qtype != kQ4_K && qtype != kQ5_K) return 0;
    const int cols = batch < kMaxColsPerLaunch ? static_cast<int>(batch) : kMaxColsPerLaunch;
    return plan_workspace(make_plan(qtype, n_out, k, cols));
}

cudaError_t qmm(int qtype, const void* w, int64_t n_out, int64_t k, const float* x, int64_t ldx, int64_t batch,
                float* y, int64_t ldy, float scale, void* workspace, cudaStream_t stream) {
    const uint8_t* wb = static_cast<const uint8_t*>(w);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    for (int64_t b0 = 0; b0 < batch; b0 += kMaxColsPerLaunch) {
        const int cols = static_cast<int>(batch - b0 < kMaxColsPerLaunch ? batch - b0 : kMaxColsPerLaunch);
        const QmmPlan p = make_plan(qtype, n_out, k, cols);
        const float* xb = x + b0 * ldx;
        float* yb = y + b0 * ldy;
        const int n = static_cast<int>(n_out), kk = static_cast<int>(k);
        cudaError_t e;
        if (qtype == kQ4_K)
            e = p.nbt == 1 ? launch_qmm<kQ4_K, 1>(wb, n, kk, xb, ldx, cols, yb, ldy, scale, ws, p, stream)
                           : launch_qmm<kQ4_K, 2>(wb, n, kk, xb, ldx, cols, yb, ldy, scale, ws, p, stream);
        else if (qtype == kQ5_K)
            e = p.nbt == 1 ? launch_qmm<kQ5_K, 1>(wb, n, kk, xb, ldx, cols, yb, ldy, scale, ws, p, stream)
                           : launch_qmm<kQ5_K, 2>(wb, n, kk, xb, ldx, cols, yb, ldy, scale, ws, p, stream);
        else
            e = cudaErrorInvalidValue;
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace hesa_cuda
