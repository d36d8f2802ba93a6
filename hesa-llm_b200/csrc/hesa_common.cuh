// hesa_common.cuh -- shared device helpers for the sm_100a kernels.
//
// * 1-D bulk copies global -> shared (cp.async.bulk) completing on an
//   mbarrier transaction count; the copy engine streams the GGUF blocks into
//   shared memory while the warps decode the previous stage.
// * Every wait is bounded by %globaltimer: after HESA_WAIT_LIMIT_NS the
//   waiting thread records a code in the library's status word (a device
//   address every kernel receives as an argument) and gives up, so a lost
//   copy can never hang the GPU.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace hesa_cuda {

enum : int {
    kStatusWaitTimeout = 1,     // a stage's bulk copy did not land in time
    kStatusDrainTimeout = 2,    // a copy still in flight during the error exit
    kStatusBadPosition = 3,     // a device-side position outside the cache / rope table
    kStatusPeerTimeout = 4,     // a peer rank did not reach the all-gather barrier in time
};

constexpr unsigned long long HESA_WAIT_LIMIT_NS = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long global_timer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// The status word is sticky: the first failure wins, the host reads and
// clears it through the C ABI.
__device__ __forceinline__ void record_status(int* status, int code) {
    atomicCAS(status, 0, code);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

// Global -> shared bulk copy of `bytes` (multiple of 16; both addresses
// 16-byte aligned), completing on `bar`'s transaction count.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_addr(dst_smem)), "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// L2 policy for data read once (streamed weights): its lines are the first
// to be evicted, so the stream does not push activations, KV rows or the
// next kernel's inputs out of L2.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// bulk_g2s with an L2 cache policy for the source lines.
__device__ __forceinline__ void bulk_g2s_policy(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                                uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_addr(dst_smem)), "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// 2-D tiled tensor copy (TMA) of the box at element coordinates (x, y) of the
// tensor map into shared memory, completing on `bar`. No cluster multicast.
__device__ __forceinline__ void tma_load_2d(void* dst_smem, const void* tensor_map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_addr(dst_smem)), "l"(tensor_map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// Named barrier `id` (1..15) over `count` threads (a multiple of 32).
__device__ __forceinline__ void named_barrier(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// As mbar_try_wait, but the thread may be suspended for up to `hint_ns`
// while the phase is incomplete: it is woken when the phase completes, so a
// waiting warp takes no issue slots from the warps that are decoding.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        "selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns) : "memory");
    return ok != 0;
}

// Non-blocking: has phase `parity` of `bar` completed?
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Plain arrive (count 1) on `bar`; the arrival state is not needed.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Wait for phase `parity` of `bar` to complete. Returns false (and records
// `code` in *status) if it has not completed within HESA_WAIT_LIMIT_NS.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* status, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_timer_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;  // sleep up to 20 us per try
        if (global_timer_ns() - t0 > HESA_WAIT_LIMIT_NS) {
            record_status(status, code);
            return false;
        }
    }
}

__device__ __forceinline__ float half_bits_to_float(uint32_t h16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h16 & 0xFFFFu)));
}

// Packed fp32x2 FMA (sm_100): d = a * b + c on two lanes of a 64-bit pair.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(*reinterpret_cast<unsigned long long*>(&d))
        : "l"(*reinterpret_cast<const unsigned long long*>(&a)),
          "l"(*reinterpret_cast<const unsigned long long*>(&b)),
          "l"(*reinterpret_cast<const unsigned long long*>(&c)));
    return d;
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("add.rn.f32x2 %0, %1, %2;"
        : "=l"(*reinterpret_cast<unsigned long long*>(&d))
        : "l"(*reinterpret_cast<const unsigned long long*>(&a)),
          "l"(*reinterpret_cast<const unsigned long long*>(&b)));
    return d;
}

// Programmatic dependent launch. grid_dep_wait blocks until the grids this one
// depends on (the previous kernel on the stream, when launched with
// programmatic stream serialization) have completed and their writes are
// visible; grid_dep_launch lets the next such kernel start its CTAs as SMs
// free up. Both are no-ops for a normal launch.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// max with NaN propagation (max.NaN.f32): a NaN in either input gives NaN.
__device__ __forceinline__ float fmax_nan(float a, float b) {
    float d;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

}  // namespace hesa_cuda
