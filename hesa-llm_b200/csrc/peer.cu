// peer.cu -- completion barrier of the all-gathers fused into row-sharded
// matvecs (see PeerOut in qmatvec.h).
//
// The strip kernels of a step store their rows into every rank's gathered
// buffer over NVLink; the barrier kernel is launched after them without
// programmatic serialization, so it starts once their grids (and stores)
// have completed. On each rank's stream, lane p then publishes the step
// number into slot `rank` of rank p's flag array (st.release.sys) and waits
// until slot p of this rank's own array carries it (ld.acquire.sys). When every lane has seen its peer, all
// ranks have finished storing this step's rows here. Plain peer loads and
// stores only: no multimem, no multicast object.
#include "hesa_common.cuh"
#include "qmatvec.h"

namespace hesa_cuda {
namespace {

struct PeerFlags {
    uint32_t* flags[kMaxPeers];   // flags[p]: rank p's flag array, mapped here
    uint32_t* epoch;              // this rank's barrier count
    unsigned long long limit_ns;  // how long to wait for the peers
    int rank, world;
};

// How long a barrier waits for its peers (set_peer_wait_limit); read when a
// barrier is enqueued, so a captured graph keeps the value of its capture.
unsigned long long g_peer_limit_ns = HESA_WAIT_LIMIT_NS;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Has the counter at p reached e? (modular: counts wrap after 2^32 steps)
__device__ __forceinline__ bool reached(const uint32_t* p, uint32_t e) {
    return static_cast<int32_t>(ld_acquire_sys(p) - e) >= 0;
}

__global__ void __launch_bounds__(32) peer_barrier_kernel(PeerFlags f, int* __restrict__ status) {
    const int t = threadIdx.x;
    const uint32_t e = *f.epoch + 1u;
    __syncwarp();
    if (t < f.world) {
        __threadfence_system();
        st_release_sys(f.flags[t] + f.rank, e);
        const uint32_t* mine = f.flags[f.rank] + t;
        if (!reached(mine, e)) {
            const unsigned long long t0 = global_timer_ns();
            for (;;) {
                __nanosleep(100);
                if (reached(mine, e)) break;
                if (global_timer_ns() - t0 > f.limit_ns) {
                    record_status(status, kStatusPeerTimeout);
                    break;
                }
            }
        }
    }
    __syncwarp();
    if (t == 0) *f.epoch = e;
}

}  // namespace

cudaError_t peer_barrier(uint32_t* const* flags, int rank, int world, uint32_t* epoch, cudaStream_t stream) {
    if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world || !epoch || !flags)
        return cudaErrorInvalidValue;
    PeerFlags f = {};
    for (int p = 0; p < world; ++p) {
        if (!flags[p]) return cudaErrorInvalidValue;
        f.flags[p] = flags[p];
    }
    f.epoch = epoch;
    f.limit_ns = g_peer_limit_ns;
    f.rank = rank;
    f.world = world;
    int* status = nullptr;
    cudaError_t e = status_word(&status);
    if (e != cudaSuccess) return e;
    peer_barrier_kernel<<<1, 32, 0, stream>>>(f, status);
    return cudaGetLastError();
}

void set_peer_wait_limit(unsigned long long ns) { g_peer_limit_ns = ns ? ns : HESA_WAIT_LIMIT_NS; }

unsigned long long peer_wait_limit() { return g_peer_limit_ns; }

}  // namespace hesa_cuda
