// Peer-memory all-gather for the sharded iteration (one process and one GPU per rank, NVLink / NVSwitch peers).
//
// Every rank owns one exchange buffer, mapped into every other rank's address space with CUDA IPC:
//   [flags: kMaxRanks u32, slot q = the last exchange epoch rank q delivered here] [arrival counters: 2 u32]
//   [staging: 2 parities x world x cap bytes, block q of a parity = rank q's contribution]
// One kernel per exchange pushes the rank's own block into every peer's staging (parity = epoch & 1), signals each
// peer with a system-scope release store of the epoch into its flag slot, waits (bounded) until every peer's flag
// on this rank has reached the epoch, and copies the peers' staged blocks into place. The staging keeps a fast
// rank from overwriting a slower peer's live buffer while that peer still reads it; two parities let a rank
// start exchange e + 1 while a peer still copies out exchange e (no rank can run two exchanges ahead, since each
// exchange waits for every peer).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace ntcb {

constexpr int kP2PMaxRanks = 8;
constexpr size_t kP2PHeader = 256;   // flags + counters, padded

struct P2PArgs {
    int world = 1, rank = 0;
    size_t cap = 0;                            // bytes of one rank's staging block
    char* base[kP2PMaxRanks] = {};             // every rank's exchange buffer (this rank's own at [rank])
};

// In-place all-gather of `bytes` per rank over the exchange buffers: rank r's block is at dst + r * bytes on entry,
// every rank's block is there on exit. bytes <= cap. A wait that runs out sets *err = 2 and the kernel returns
// without copying (the host reports it at the next synchronising call).
void launch_p2p_allgather(cudaStream_t s, const P2PArgs& a, void* dst, size_t bytes, uint32_t epoch, int* err);

}  // namespace ntcb
