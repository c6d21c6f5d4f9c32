// Runtime binding of NCCL for the library's own multi-GPU iteration (ntcb_comm_* / ntcb_shard_*_iteration).
//
// NCCL is opened with dlopen("libnccl.so.2") the first time a communicator is needed, so single-GPU users
// (and the reference trainer linked against this library) never load it. In a process that already has NCCL
// loaded (torch's copy), dlopen returns that library.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <string>

namespace ntcb::nccl {

constexpr int kUniqueIdBytes = 128;

// Fills id (kUniqueIdBytes bytes) with a new NCCL unique id; false + reason when NCCL cannot be loaded.
bool unique_id(unsigned char* id, std::string& why);
// A communicator of `world` ranks on the current device; nullptr + reason on failure.
void* comm_init(const unsigned char* id, int world, int rank, std::string& why);
void comm_destroy(void* comm);
// In-place all-gather of `bytes` per rank: rank r's block is at buf + r * bytes on entry, every rank's block is
// there on exit (NCCL's in-place form). Exits the process on an NCCL error (the trainer's callers have no
// error path).
void all_gather_inplace(void* comm, void* buf, size_t bytes, int rank, cudaStream_t s);
// NCCL's version code (e.g. 22809), 0 when not loaded.
int version();

}  // namespace ntcb::nccl
