// Peer-memory all-gather kernel (layout and protocol in p2p_exchange.h).
#include "kernels.h"
#include "p2p_exchange.h"

#include <algorithm>

namespace ntcb {

namespace {

constexpr int kP2PThreads = 512;
constexpr uint32_t kP2PSpinPolls = 256;        // polls of a line before backing off with __nanosleep

__device__ __forceinline__ char* stage_of(char* base, const P2PArgs& a, int par, int q) {
    return base + kP2PHeader + ((size_t)par * a.world + q) * a.cap;
}

// One 16-byte line = two 64-bit elements {epoch << 32 | word}. A 64-bit element is written and read as one
// access, so a reader that sees an element's epoch also sees its word; no fence or separate flag is needed.
__device__ __forceinline__ void st_line(void* p, uint64_t lo, uint64_t hi) {
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(lo), "l"(hi) : "memory");
}
__device__ __forceinline__ void ld_line(const void* p, uint64_t& lo, uint64_t& hi) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(lo), "=l"(hi) : "l"(p) : "memory");
}

__global__ void __launch_bounds__(kP2PThreads) k_p2p_allgather(P2PArgs a, char* dst, size_t bytes, uint32_t epoch, uint32_t poll_limit,
                                                                int* err) {
    const int r = a.rank, G = a.world, par = (int)(epoch & 1u);
    const size_t nwords = bytes / 4, nlines = (nwords + 1) / 2;
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
    const uint64_t tag = (uint64_t)epoch << 32;
    // 1. this rank's block, two words per line, into every peer's staging
    const uint32_t* src = reinterpret_cast<const uint32_t*>(dst + (size_t)r * bytes);
    for (size_t i = tid; i < nlines; i += stride) {
        const uint32_t w0 = src[2 * i], w1 = 2 * i + 1 < nwords ? src[2 * i + 1] : 0u;
        for (int q = 0; q < G; q++)
            if (q != r) st_line(stage_of(a.base[q], a, par, r) + 16 * i, tag | w0, tag | w1);
    }
    // 2. every peer's lines of this exchange, as they arrive (bounded), into place
    for (int q = 0; q < G; q++) {
        if (q == r) continue;
        const char* s = stage_of(a.base[r], a, par, q);
        uint32_t* out = reinterpret_cast<uint32_t*>(dst + (size_t)q * bytes);
        for (size_t i = tid; i < nlines; i += stride) {
            uint64_t lo, hi;
            uint32_t polls = 0;
            for (;;) {
                ld_line(s + 16 * i, lo, hi);
                if ((uint32_t)(lo >> 32) == epoch && (uint32_t)(hi >> 32) == epoch) break;
                if (++polls > poll_limit) { atomicExch(err, 2); return; }
                if (polls > kP2PSpinPolls) __nanosleep(128);
            }
            out[2 * i] = (uint32_t)lo;
            if (2 * i + 1 < nwords) out[2 * i + 1] = (uint32_t)hi;
        }
    }
}

}  // namespace

size_t p2p_stage_bytes(size_t bytes) { return ((bytes / 4 + 1) / 2) * 16; }

void launch_p2p_allgather(cudaStream_t s, const P2PArgs& a, void* dst, size_t bytes, uint32_t epoch, uint32_t poll_limit, int* err) {
    const int nsm = device_sm_count();
    const size_t lines = (bytes / 4 + 1) / 2;
    const int grid = (int)std::max<size_t>(1, std::min<size_t>((size_t)nsm, (lines + kP2PThreads - 1) / kP2PThreads));
    k_p2p_allgather<<<grid, kP2PThreads, 0, s>>>(a, static_cast<char*>(dst), bytes, epoch, std::max(1u, poll_limit), err);
    NTCB_CHECK(cudaGetLastError());
}

}  // namespace ntcb
