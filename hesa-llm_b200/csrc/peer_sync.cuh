// peer_sync.cuh -- the low-latency exchange of the head-sharded decode step:
// every value a rank sends travels with a tag in the same 64-bit word.
//
// A producer stores (value bits | tag << 32) into every rank's buffer with
// one 64-bit store per element (st.volatile.global.u64: a naturally aligned
// 64-bit access is single-copy atomic, over NVLink too); a consumer loads the
// word (ld.volatile.global, no L1) and uses the value once the tag is the one
// it expects, re-reading until then (bounded by %globaltimer -- the limit the
// host set with set_peer_wait_limit, carried in LLIn -- on expiry it records
// kStatusPeerTimeout and goes on with what it read). The tag names
// the token and the place in the step -- (count << 12) | (layer << 3 | phase)
// with `count` this rank's token counter in device memory -- so a word left
// from an earlier step can never pass for a new one, and no fence, flag array
// or barrier is needed: the data is its own flag. Plain peer loads and stores
// only: no multimem, no multicast object.
//
// Word order: element g of a tagged vector lives at word ll_pos(g). Inside
// each unit of 256 elements, element 8L + i (the eight a lane of the strip
// kernel's staging holds, L = 0..31) is at word (i / 2) * 64 + 2L + (i % 2),
// so each of the four 16-byte loads a lane makes for its eight elements is
// one fully coalesced 512-byte access of the warp (in natural order the
// lanes were 64 bytes apart: four times the L2 requests, and the staging of
// every kernel of the sharded step took 2-3x as long). A tagged vector's
// buffer holds whole units.
#pragma once

#include "hesa_common.cuh"

namespace hesa_cuda {

constexpr int kPeerSyncMax = 8;

__device__ __forceinline__ uint32_t ll_tag(const uint32_t* count, uint32_t lo) {
    return (*reinterpret_cast<const volatile uint32_t*>(count) << 12) | lo;
}

__device__ __forceinline__ void st_ll(uint64_t* p, float v, uint32_t tag) {
    const uint64_t word = static_cast<uint64_t>(__float_as_uint(v)) | (static_cast<uint64_t>(tag) << 32);
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(word) : "memory");
}

__device__ __forceinline__ uint64_t ld_ll(const uint64_t* p) {
    uint64_t w;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// The value at p once its tag is `tag`: the wait, out of line (a word that is
// not there yet is the rare case, and an inlined loop per load point made the
// staging code large enough to stall on instruction fetch). `*failed` (a
// per-CTA shared flag) is set, and the status word records
// kStatusPeerTimeout, when the wait runs out; later waits of the CTA then
// return whatever they read without waiting.
static __device__ __noinline__ float ld_ll_slow(const uint64_t* p, uint32_t tag, unsigned long long limit_ns,
                                                int* status, volatile int* failed) {
    uint64_t w = ld_ll(p);
    if (static_cast<uint32_t>(w >> 32) == tag || *failed) return __uint_as_float(static_cast<uint32_t>(w));
    const unsigned long long t0 = global_timer_ns();
    for (;;) {
        w = ld_ll(p);
        if (static_cast<uint32_t>(w >> 32) == tag) break;
        if (global_timer_ns() - t0 > limit_ns) {
            record_status(status, kStatusPeerTimeout);
            *failed = 1;
            break;
        }
    }
    return __uint_as_float(static_cast<uint32_t>(w));
}

// The value of word w (read from p) if its tag is `tag`, else ld_ll_slow.
__device__ __forceinline__ float ll_value(const uint64_t* p, uint64_t w, uint32_t tag, unsigned long long limit_ns,
                                          int* status, volatile int* failed) {
    return static_cast<uint32_t>(w >> 32) == tag ? __uint_as_float(static_cast<uint32_t>(w))
                                                 : ld_ll_slow(p, tag, limit_ns, status, failed);
}

__device__ __forceinline__ float ld_ll_wait(const uint64_t* p, uint32_t tag, unsigned long long limit_ns, int* status,
                                            volatile int* failed) {
    return ll_value(p, ld_ll(p), tag, limit_ns, status, failed);
}

// Word of element g, and element of word w (inverse), in the order above.
__host__ __device__ __forceinline__ int64_t ll_pos(int64_t g) {
    return (g & ~int64_t(255)) | (((g >> 1) & 3) << 6) | (((g >> 3) & 31) << 1) | (g & 1);
}
__host__ __device__ __forceinline__ int64_t ll_elem(int64_t w) {
    return (w & ~int64_t(255)) | (((w >> 1) & 31) << 3) | (((w >> 6) & 3) << 1) | (w & 1);
}

// Two consecutive words in one 16-byte load (each 64-bit element of the
// vector is still a single-copy atomic access).
__device__ __forceinline__ void ld_ll2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Elements 8 * lane .. 8 * lane + 7 of the unit at `unit` (its word 0):
// word j of w is element 8 * lane + j, read at unit + ll_word8(lane, j).
__device__ __forceinline__ int ll_word8(int lane, int j) { return (j >> 1) * 64 + 2 * lane + (j & 1); }

// The eight words in four coalesced 16-byte loads, issued without looking at
// them, so that the loads of several units overlap.
__device__ __forceinline__ void ld_ll8_issue(const uint64_t* unit, int lane, uint64_t (&w)[8]) {
#pragma unroll
    for (int j = 0; j < 8; j += 2) ld_ll2(unit + ll_word8(lane, j), w[j], w[j + 1]);
}

// v[j] <- the value of w[j] if its tag is `tag`, else the value once a
// re-read of its word shows that tag.
__device__ __forceinline__ void ld_ll8_take(const uint64_t* unit, int lane, const uint64_t (&w)[8], uint32_t tag,
                                            unsigned long long limit_ns, float (&v)[8], int* status,
                                            volatile int* failed) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = ll_value(unit + ll_word8(lane, j), w[j], tag, limit_ns, status, failed);
}

// Tagged inputs of a kernel of the sharded step (null pointers: plain inputs).
// Vectors are given by their word 0 (element g at ll_pos(g)).
struct LLIn {
    const uint64_t* x;       // the input vector (2k elements for a SwiGLU input, up at element k)
    const uint64_t* resid;   // the residual vector; row i of this shard is its element resid_off + i
    int64_t resid_off;
    const uint32_t* count;   // this rank's token counter
    uint32_t x_lo, resid_lo; // the tags' low bits
    unsigned long long limit_ns;  // how long one word is waited for
};

// Tagged outputs: row i of this shard is element off + i of the vector at
// y[p] on every rank p (rows from `split` on: element off2 + (i - split) of
// y2[p]); with by_parity set, every row goes to element off + i of y[p] while
// the count is even and of y2[p] while it is odd (two buffers a step apart,
// so a rank may store step s + 1 while a peer still collects step s).
struct LLOut {
    uint64_t* y[kPeerSyncMax];
    uint64_t* y2[kPeerSyncMax];
    int64_t off, off2;
    int split, world, by_parity;
    const uint32_t* count;
    uint32_t lo;
};

}  // namespace hesa_cuda
