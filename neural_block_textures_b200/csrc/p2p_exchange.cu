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

// Work is spread over (peer, line) tasks, task t = line i of peer slot j (t = j * nlines + i, consecutive threads on
// consecutive lines of one peer): phase 1 stores this rank's line i into peer j's staging, phase 2 polls peer j's
// line i in this rank's staging. Each thread finishes all its stores before its first poll, so no poll waits on a
// store of its own GPU that has not been issued.
__global__ void __launch_bounds__(kP2PThreads) k_p2p_allgather(P2PArgs a, char* dst, size_t bytes, uint32_t epoch, uint32_t poll_limit,
                                                                int* err) {
    const int r = a.rank, G = a.world, par = (int)(epoch & 1u);
    const uint32_t nwords = (uint32_t)(bytes / 4), nlines = (nwords + 1) / 2;
    const uint32_t ntasks = nlines * (uint32_t)(G - 1);
    const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x, stride = gridDim.x * blockDim.x;
    const uint64_t tag = (uint64_t)epoch << 32;
    // 1. this rank's block, two words per line, into every peer's staging
    const uint32_t* src = reinterpret_cast<const uint32_t*>(dst + (size_t)r * bytes);
    for (uint32_t t = tid; t < ntasks; t += stride) {
        const uint32_t j = t / nlines, i = t - j * nlines;
        const int q = (int)j + ((int)j >= r ? 1 : 0);
        const uint32_t w0 = src[2 * i], w1 = 2 * i + 1 < nwords ? src[2 * i + 1] : 0u;
        st_line(stage_of(a.base[q], a, par, r) + 16 * (size_t)i, tag | w0, tag | w1);
    }
    // 2. every peer's lines of this exchange, as they arrive (bounded), into place
    for (uint32_t t = tid; t < ntasks; t += stride) {
        const uint32_t j = t / nlines, i = t - j * nlines;
        const int q = (int)j + ((int)j >= r ? 1 : 0);
        const char* s = stage_of(a.base[r], a, par, q) + 16 * (size_t)i;
        uint64_t lo, hi;
        uint32_t polls = 0;
        for (;;) {
            ld_line(s, lo, hi);
            if ((uint32_t)(lo >> 32) == epoch && (uint32_t)(hi >> 32) == epoch) break;
            if (++polls > poll_limit) { atomicExch(err, 2); return; }
            if (polls > kP2PSpinPolls) __nanosleep(128);
        }
        uint32_t* out = reinterpret_cast<uint32_t*>(dst + (size_t)q * bytes);
        out[2 * i] = (uint32_t)lo;
        if (2 * i + 1 < nwords) out[2 * i + 1] = (uint32_t)hi;
    }
}

}  // namespace

size_t p2p_stage_bytes(size_t bytes) { return ((bytes / 4 + 1) / 2) * 16; }

void launch_p2p_allgather(cudaStream_t s, const P2PArgs& a, void* dst, size_t bytes, uint32_t epoch, uint32_t poll_limit, int* err) {
    const int nsm = device_sm_count();
    const size_t tasks = (bytes / 4 + 1) / 2 * (size_t)std::max(1, a.world - 1);
    // 32-bit task indices: ntcb_p2p_export refuses staging for blocks of 2^31 / (world - 1) lines or more, and the
    // sharded iteration checks every block against that staging
    if (tasks >= (1ull << 31)) NTCB_CHECK(cudaErrorInvalidValue);
    // at most one CTA per SM: every CTA is resident at once, so a polling CTA never holds back a CTA whose stores a
    // peer is waiting for
    const int grid = (int)std::max<size_t>(1, std::min<size_t>((size_t)nsm, (tasks + kP2PThreads - 1) / kP2PThreads));
    k_p2p_allgather<<<grid, kP2PThreads, 0, s>>>(a, static_cast<char*>(dst), bytes, epoch, std::max(1u, poll_limit), err);
    NTCB_CHECK(cudaGetLastError());
}

}  // namespace ntcb
