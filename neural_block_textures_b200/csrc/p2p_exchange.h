// Peer-memory all-gather for the sharded iteration (one process and one GPU per rank, NVLink / NVSwitch peers).
//
// Every rank owns one exchange buffer, mapped into every other rank's address space with CUDA IPC:
//   [kP2PHeader bytes: the rank's token slots of ntcb_p2p_barrier] [staging: 2 parities x world x cap bytes, block q of a parity = rank q's lines]
// A block travels as 16-byte lines of two 64-bit elements {epoch << 32 | one 4-byte word}: the data carries its own
// arrival flag (the low-latency line format NCCL's LL protocol uses), so one kernel per exchange stores the rank's
// own block as lines into every peer's staging (parity = epoch & 1) and then polls its own staging, line by line
// (bounded), until every peer's lines carry this exchange's epoch, copying the words into place. No fence, counter
// or separate flag is involved, and no CTA waits for another CTA of its own GPU. The staging keeps a fast rank from
// overwriting a slower peer's live buffer while that peer still reads it; two parities let a rank start exchange
// e + 1 while a peer still reads exchange e (no rank can run two exchanges ahead, since each exchange waits for
// every peer's lines), and an older exchange's lines in the same parity carry epoch e - 2, never e.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace ntcb {

constexpr int kP2PMaxRanks = 8;
constexpr size_t kP2PHeader = 256;   // bytes before the staging (barrier tokens; keeps the staging 256-byte aligned)

struct P2PArgs {
    int world = 1, rank = 0;
    size_t cap = 0;                            // bytes of one rank's staging block (p2p_stage_bytes of the largest block)
    char* base[kP2PMaxRanks] = {};             // every rank's exchange buffer (this rank's own at [rank])
};

// Staging bytes of a block of `bytes` (a multiple of 4): 16 per two words.
size_t p2p_stage_bytes(size_t bytes);
// Polls of one staged line before a wait is declared failed (>= 128 ns each after the first 256): a few seconds.
constexpr uint32_t kP2PPollLimit = 1u << 22;
// In-place all-gather of `bytes` per rank over the exchange buffers: rank r's block is at dst + r * bytes on entry,
// every rank's block is there on exit. p2p_stage_bytes(bytes) <= cap, bytes a multiple of 4. A line that has not
// arrived after poll_limit polls sets *err = 2 and its thread returns (the host reads the word at its next
// synchronising call).
void launch_p2p_allgather(cudaStream_t s, const P2PArgs& a, void* dst, size_t bytes, uint32_t epoch, uint32_t poll_limit, int* err);

}  // namespace ntcb
