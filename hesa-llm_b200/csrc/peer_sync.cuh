// peer_sync.cuh -- the cross-rank barrier at the end of a kernel whose CTAs
// store their results into the buffers of every rank (peer stores over
// NVLink, CUDA IPC mappings).
//
// grid_end_peer_barrier, called by every thread of every CTA as the kernel's
// last action: each CTA makes its stores visible at system scope
// (fence.sc.sys after a CTA barrier, by one thread) and counts itself on this
// rank's ticket; the last CTA of the grid then publishes the step -- lane p
// stores epoch + 1 into slot `rank` of rank p's flag array (st.release.sys)
// -- and waits, bounded, until slot p of its own array carries it
// (ld.acquire.sys), i.e. until every rank's grid has stored its part here.
// On expiry it records kStatusPeerTimeout and returns. It then stores the
// new epoch and clears the ticket. The next kernel on the stream, launched
// with programmatic stream serialization, reads the gathered data only after
// griddepcontrol.wait, that is after this whole grid -- the waiting CTA
// included -- has completed: no separate barrier launch breaks the chain.
// Plain peer loads and stores only: no multimem, no multicast object.
#pragma once

#include "hesa_common.cuh"

namespace hesa_cuda {

constexpr int kPeerSyncMax = 8;

struct PeerSync {
    uint32_t* flags[kPeerSyncMax];   // flags[p]: rank p's flag array as mapped here
    uint32_t* epoch;                 // this rank's barrier count (device)
    int* ticket;                     // this rank's arrival counter (device, zero between steps)
    unsigned long long limit_ns;     // how long to wait for the peers
    int rank, world;                 // world 0: no barrier
};

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Has the counter at p reached e? (modular: counts wrap after 2^32 steps)
__device__ __forceinline__ bool peer_reached(const uint32_t* p, uint32_t e) {
    return static_cast<int32_t>(ld_acquire_sys_u32(p) - e) >= 0;
}

__device__ __forceinline__ void grid_end_peer_barrier(const PeerSync& ps, int* status) {
    if (ps.world <= 0) return;
    __shared__ int s_last_cta;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();   // this CTA's peer stores, visible to every rank
        const int n_cta = static_cast<int>(gridDim.x * gridDim.y * gridDim.z);
        s_last_cta = atomicAdd(ps.ticket, 1) == n_cta - 1;
    }
    __syncthreads();
    if (!s_last_cta || threadIdx.x >= 32) return;
    const int t = threadIdx.x;
    const uint32_t e = *ps.epoch + 1u;
    if (t < ps.world) {
        __threadfence_system();   // every CTA's stores (observed through the ticket) before the flag
        st_release_sys_u32(ps.flags[t] + ps.rank, e);
        const uint32_t* mine = ps.flags[ps.rank] + t;
        if (!peer_reached(mine, e)) {
            const unsigned long long t0 = global_timer_ns();
            for (;;) {
                __nanosleep(64);
                if (peer_reached(mine, e)) break;
                if (global_timer_ns() - t0 > ps.limit_ns) {
                    record_status(status, kStatusPeerTimeout);
                    break;
                }
            }
        }
    }
    __syncwarp();
    if (t == 0) {
        *ps.epoch = e;
        *ps.ticket = 0;
    }
}

}  // namespace hesa_cuda
