// One-shot all-reduce of FP32 buffers over peer memory (internal to the library).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace lsso {

constexpr int kPeerMaxRanks = 8;

// Layout of one rank's exchange region (cudaMalloc'ed by the library, shared
// with the other ranks through a CUDA IPC handle).  Flags are written by the
// peers with system-scope release stores; word j of an array belongs to rank j.
constexpr size_t kPeerArriveOffset = 0;    // u32[8]: rank j's data of exchange e is complete
constexpr size_t kPeerDepartOffset = 128;  // u32[8]: rank j has finished reading every region for exchange e
constexpr size_t kPeerCounterOffset = 256; // u32: CTAs of the running exchange that are done (reset by the last)
constexpr size_t kPeerEpochOffset = 384;   // u32: exchanges completed by this rank
constexpr size_t kPeerDataOffset = 512;    // FP32 values

struct PeerArgs {
  char* region[kPeerMaxRanks];  // every rank's region as mapped in this process (own one at [rank])
  int world;
  int rank;
  int64_t first;                // index of the first value exchanged (a multiple of 4)
  int64_t count;                // FP32 values exchanged per region
  float scale;                  // applied to the sum (1/world for an average)
  float* out;                   // [count], 16-byte aligned, local
  int* status;                  // device status word
  unsigned long long limit_ns;  // bound of each wait on the peers
};

cudaError_t launch_peer_allreduce(const PeerArgs& a, int sm_count, cudaStream_t stream);

}  // namespace lsso
