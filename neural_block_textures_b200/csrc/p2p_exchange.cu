// Peer-memory all-gather kernel (layout and protocol in p2p_exchange.h).
#include "kernels.h"
#include "p2p_exchange.h"

namespace ntcb {

namespace {

constexpr int kP2PThreads = 256;
constexpr int kP2PBlocks = 32;                 // co-resident on any GPU, so the spinning CTAs never starve the last one
constexpr uint32_t kP2PPollLimit = 1u << 22;   // polls of >= 256 ns each: a bound of a few seconds per exchange

__device__ __forceinline__ uint32_t* flags_of(char* base) { return reinterpret_cast<uint32_t*>(base); }
__device__ __forceinline__ uint32_t* counters_of(char* base) { return reinterpret_cast<uint32_t*>(base) + kP2PMaxRanks; }
__device__ __forceinline__ char* stage_of(char* base, const P2PArgs& a, int par, int q) {
    return base + kP2PHeader + ((size_t)par * a.world + q) * a.cap;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid-stride copy of n bytes; 16-byte vectors when both ends and n allow it, else 4-byte words (every exchanged
// block is a whole number of floats). Loads bypass L1 (.cg): the source may have been written by another GPU.
__device__ __forceinline__ void copy_bytes(char* __restrict__ d, const char* __restrict__ s, size_t n) {
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
    if ((((uintptr_t)d | (uintptr_t)s | n) & 15u) == 0) {
        const uint4* s4 = reinterpret_cast<const uint4*>(s);
        uint4* d4 = reinterpret_cast<uint4*>(d);
        for (size_t i = tid; i < n / 16; i += stride) d4[i] = __ldcg(s4 + i);
    } else {
        const uint32_t* s1 = reinterpret_cast<const uint32_t*>(s);
        uint32_t* d1 = reinterpret_cast<uint32_t*>(d);
        for (size_t i = tid; i < n / 4; i += stride) d1[i] = __ldcg(s1 + i);
    }
}

__global__ void __launch_bounds__(kP2PThreads) k_p2p_allgather(P2PArgs a, char* dst, size_t bytes, uint32_t epoch, int* err) {
    const int r = a.rank, G = a.world, par = (int)(epoch & 1u);
    // 1. this rank's block into every peer's staging
    for (int q = 0; q < G; q++)
        if (q != r) copy_bytes(stage_of(a.base[q], a, par, r), dst + (size_t)r * bytes, bytes);
    __threadfence_system();
    __syncthreads();
    // 2. the last CTA to finish its stores signals every peer
    __shared__ int last, ok;
    if (threadIdx.x == 0) {
        const uint32_t prev = atomicAdd(&counters_of(a.base[r])[par], 1u);
        last = prev == gridDim.x - 1;
    }
    __syncthreads();
    if (last) {
        __threadfence_system();
        if (threadIdx.x == 0) counters_of(a.base[r])[par] = 0u;   // reused two exchanges later, after this kernel
        if (threadIdx.x < G && threadIdx.x != r) st_release_sys(&flags_of(a.base[threadIdx.x])[r], epoch);
    }
    // 3. wait until every peer has delivered this exchange here (bounded)
    if (threadIdx.x == 0) {
        ok = 1;
        const uint32_t* mine = flags_of(a.base[r]);
        for (int q = 0; q < G && ok; q++) {
            if (q == r) continue;
            uint32_t polls = 0;
            while ((int32_t)(ld_acquire_sys(mine + q) - epoch) < 0) {
                if (++polls > kP2PPollLimit) { ok = 0; atomicExch(err, 2); break; }
                __nanosleep(256);
            }
        }
    }
    __syncthreads();
    if (!ok) return;
    // 4. the peers' staged blocks into place
    for (int q = 0; q < G; q++)
        if (q != r) copy_bytes(dst + (size_t)q * bytes, stage_of(a.base[r], a, par, q), bytes);
}

}  // namespace

void launch_p2p_allgather(cudaStream_t s, const P2PArgs& a, void* dst, size_t bytes, uint32_t epoch, int* err) {
    k_p2p_allgather<<<kP2PBlocks, kP2PThreads, 0, s>>>(a, static_cast<char*>(dst), bytes, epoch, err);
    NTCB_CHECK(cudaGetLastError());
}

}  // namespace ntcb
