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

// The value at p once its tag is `tag`. `ok` turns false (and the status word
// records kStatusPeerTimeout) when the wait runs out; later calls then return
// whatever they read without waiting.
__device__ __forceinline__ float ld_ll_wait(const uint64_t* p, uint32_t tag, unsigned long long limit_ns, int* status,
                                            bool& ok) {
    uint64_t w = ld_ll(p);
    if (static_cast<uint32_t>(w >> 32) == tag || !ok) return __uint_as_float(static_cast<uint32_t>(w));
    const unsigned long long t0 = global_timer_ns();
    for (;;) {
        w = ld_ll(p);
        if (static_cast<uint32_t>(w >> 32) == tag) break;
        if (global_timer_ns() - t0 > limit_ns) {
            record_status(status, kStatusPeerTimeout);
            ok = false;
            break;
        }
    }
    return __uint_as_float(static_cast<uint32_t>(w));
}

// Two consecutive words in one 16-byte load (each 64-bit element of the
// vector is still a single-copy atomic access).
__device__ __forceinline__ void ld_ll2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// The eight words at p (16-byte aligned) in four 16-byte loads, issued
// without looking at them, so that the loads of several groups overlap.
__device__ __forceinline__ void ld_ll8_issue(const uint64_t* p, uint64_t (&w)[8]) {
#pragma unroll
    for (int j = 0; j < 8; j += 2) ld_ll2(p + j, w[j], w[j + 1]);
}

// v[j] <- the value of w[j] (read from p + j) if its tag is `tag`, else the
// value once a re-read of p + j shows that tag.
__device__ __forceinline__ void ld_ll8_take(const uint64_t* p, const uint64_t (&w)[8], uint32_t tag,
                                            unsigned long long limit_ns, float (&v)[8], int* status, bool& ok) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        v[j] = static_cast<uint32_t>(w[j] >> 32) == tag ? __uint_as_float(static_cast<uint32_t>(w[j]))
                                                          : ld_ll_wait(p + j, tag, limit_ns, status, ok);
    }
}

// Tagged inputs of a kernel of the sharded step (null pointers: plain inputs).
struct LLIn {
    const uint64_t* x;       // the input vector (2k words for a SwiGLU input)
    const uint64_t* resid;   // this shard's row 0 of the residual
    const uint32_t* count;   // this rank's token counter
    uint32_t x_lo, resid_lo; // the tags' low bits
    unsigned long long limit_ns;  // how long one word is waited for
};

// Tagged outputs: row i of this shard goes to y[p] + i of every rank p (rows
// from `split` on to y2[p] + (i - split)); with by_parity set, every row goes
// to y[p] + i while the count is even and to y2[p] + i while it is odd (two
// buffers a step apart, so a rank may store step s + 1 while a peer still
// collects step s).
struct LLOut {
    uint64_t* y[kPeerSyncMax];
    uint64_t* y2[kPeerSyncMax];
    int split, world, by_parity;
    const uint32_t* count;
    uint32_t lo;
};

}  // namespace hesa_cuda
