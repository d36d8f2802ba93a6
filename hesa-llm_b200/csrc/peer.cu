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
//
// The tagged form (peer_collect) needs neither the fence nor the flags: the
// strip kernels store every row into every rank as a 64-bit word carrying the
// step's tag (peer_sync.cuh), and each rank's collector reads its own buffer
// until every word carries the tag. It is launched with programmatic
// serialization like the matvecs, so the chain of launches stays unbroken.
#include "hesa_common.cuh"
#include "qmatvec.h"

#include <algorithm>

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

constexpr int kCollectThreads = 256;

__global__ void __launch_bounds__(kCollectThreads) peer_collect_kernel(const uint64_t* words0, const uint64_t* words1,
                                                                      int n, float* __restrict__ out, uint32_t* sync,
                                                                      uint32_t lo, unsigned long long limit_ns,
                                                                      int* __restrict__ status) {
    grid_dep_wait();
    // the next step's matvecs may start their CTAs on the SMs this grid
    // leaves free; they wait for its completion before reading the count
    grid_dep_launch();
    const uint32_t c = *reinterpret_cast<volatile uint32_t*>(sync);
    const uint32_t tag = (c << 12) | lo;
    const uint64_t* src = (c & 1u) ? words1 : words0;
    __shared__ int failed;
    if (threadIdx.x == 0) failed = 0;
    __syncthreads();
    // words in order (coalesced), each to its element; the words of the last
    // unit past n hold no element
    const int n_words = (n + 255) & ~255;
    for (int w = blockIdx.x * kCollectThreads + threadIdx.x; w < n_words; w += gridDim.x * kCollectThreads) {
        const int e = static_cast<int>(ll_elem(w));
        if (e < n) out[e] = ld_ll_wait(src + w, tag, limit_ns, status, &failed);
    }
    // the last CTA to finish advances the count (every CTA has read it by then)
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(sync + 1, 1u) == gridDim.x - 1) {
            sync[1] = 0;
            *reinterpret_cast<volatile uint32_t*>(sync) = c + 1u;
        }
    }
}

// y[i] to every rank as tagged words (LLOut with by_parity): the gathered
// form of a matvec computed by a kernel without the tagged epilogue.
__global__ void __launch_bounds__(kCollectThreads) peer_scatter_kernel(const float* __restrict__ y, int n, LLOut o) {
    grid_dep_wait();
    grid_dep_launch();
    const uint32_t tag = ll_tag(o.count, o.lo);
    const bool odd = (tag >> 12) & 1u;
    for (int i = blockIdx.x * kCollectThreads + threadIdx.x; i < n; i += gridDim.x * kCollectThreads) {
        const float v = y[i];
        const int64_t at = ll_pos(o.off + i);
        for (int p = 0; p < o.world; ++p) st_ll((odd ? o.y2[p] : o.y[p]) + at, v, tag);
    }
}

cudaError_t launch_pdl(const void* fn, int grid, void** args, cudaStream_t stream) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kCollectThreads);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t collect_grid(int64_t n, int& grid) {
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    // one CTA per SM at most: every word is touched once
    grid = static_cast<int>(std::min<int64_t>((n + kCollectThreads - 1) / kCollectThreads, sms));
    return cudaSuccess;
}

}  // namespace

cudaError_t peer_scatter_tagged(const float* y, int64_t n, const LLOut& lout, cudaStream_t stream) {
    if (!y || n < 1 || n >= (int64_t(1) << 30) || lout.world < 1 || lout.world > kPeerSyncMax || !lout.count ||
        !lout.by_parity)
        return cudaErrorInvalidValue;
    int grid = 0;
    cudaError_t e = collect_grid(n, grid);
    if (e != cudaSuccess) return e;
    int nn = static_cast<int>(n);
    LLOut o = lout;
    void* args[] = {&y, &nn, &o};
    return launch_pdl(reinterpret_cast<const void*>(peer_scatter_kernel), grid, args, stream);
}

cudaError_t peer_collect(const uint64_t* words0, const uint64_t* words1, int64_t n, float* out, uint32_t* sync,
                         uint32_t lo, cudaStream_t stream) {
    if (!words0 || !words1 || !out || !sync || n < 1 || n >= (int64_t(1) << 30) || lo >= (1u << 12))
        return cudaErrorInvalidValue;
    int* status = nullptr;
    cudaError_t e = status_word(&status);
    if (e != cudaSuccess) return e;
    int grid = 0;
    e = collect_grid(n, grid);
    if (e != cudaSuccess) return e;
    int nn = static_cast<int>(n);
    unsigned long long limit = g_peer_limit_ns;
    void* args[] = {&words0, &words1, &nn, &out, &sync, &lo, &limit, &status};
    return launch_pdl(reinterpret_cast<const void*>(peer_collect_kernel), grid, args, stream);
}

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
