// Symmetric peer memory over CUDA IPC (see csrc/core/peer.cpp).
#pragma once

#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "kernels.h"

namespace turbol {

class PeerMemory {
 public:
  PeerMemory(size_t payload_bytes, int device);
  ~PeerMemory();
  PeerMemory(const PeerMemory&) = delete;
  PeerMemory& operator=(const PeerMemory&) = delete;

  std::string Handle() const;                                    // this rank's IPC handle (64 bytes)
  void Open(const std::vector<std::string>& handles, int rank);  // map every other rank's buffer
  TbPeerTable Table() const;
  unsigned* DoneCounter() const;
  int* ErrorWord() const;
  // Epoch of the replicated-Adam step (its own sequence, separate from the
  // other collectives on this buffer).
  unsigned* RepEpoch() const;
  void* Payload() const;  // local payload base (device pointer)
  size_t PayloadBytes() const { return total_bytes_ - header_bytes_; }
  int rank() const { return rank_; }
  int world() const { return world_; }
  int device() const { return device_; }

 private:
  int device_ = 0, rank_ = 0, world_ = 0;
  size_t header_bytes_ = 0, total_bytes_ = 0;
  void* local_ = nullptr;
  void* counters_ = nullptr;
  std::vector<void*> bases_;
};

}  // namespace turbol
