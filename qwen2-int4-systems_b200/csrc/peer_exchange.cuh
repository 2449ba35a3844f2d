// Peer-memory exchange for the column-split MLP (see peer_exchange.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace qi4 {

constexpr int kMaxPeers = 8;  // ranks of one NVLink / NVSwitch node

// Where the SwiGLU pass of one rank stores its shard, and whom it tells.
struct PeerTargets {
  float* out[kMaxPeers];        // every rank's gathered [M, ld] FP32 buffer (this rank's own included)
  uint32_t* flags[kMaxPeers];   // every rank's flag array (world words); slot `rank` is written
  uint32_t* counter;            // this rank's CTA counter (zero between calls)
  int64_t ld, col0;             // row pitch of the gathered buffers, first column of the shard
  int world, rank;
  uint32_t epoch;
};

cudaError_t launch_swiglu_scatter(const void* g, const void* u, int dtype, const PeerTargets& t, int64_t M, int64_t n,
                                  cudaStream_t stream, int num_sms);
cudaError_t launch_flag_wait(const uint32_t* flags, int world, uint32_t epoch, uint64_t limit_ns,
                             cudaStream_t stream);
int read_peer_error(cudaStream_t stream);

}  // namespace qi4
