// PeerMemory: one symmetric device buffer per rank, shared with every other
// rank of the node through CUDA IPC, so kernels can load from and store to
// peer HBM over NVLink directly (see csrc/kernels/comm.cu).
//
// Layout of every rank's buffer: [flag header, 256-byte aligned][payload].
// The handle exchange itself is left to the caller (a torch.distributed
// all_gather_object or the TcpStore); this class only allocates, exports and
// opens.  Local counters (call epoch, finished-block count, error word) live in
// a separate, non-shared allocation.
#include "turbol/peer.hpp"

#include <cstring>
#include <stdexcept>

#include "kernels.h"

namespace turbol {

namespace {
void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
}  // namespace

PeerMemory::PeerMemory(size_t payload_bytes, int device) : device_(device) {
  ck(cudaSetDevice(device), "cudaSetDevice");
  header_bytes_ = align256(tb_peer_header_bytes());
  total_bytes_ = header_bytes_ + align256(payload_bytes);
  ck(cudaMalloc(&local_, total_bytes_), "cudaMalloc(peer buffer)");
  ck(cudaMemset(local_, 0, total_bytes_), "cudaMemset(peer buffer)");
  ck(cudaMalloc(&counters_, 256), "cudaMalloc(peer counters)");
  ck(cudaMemset(counters_, 0, 256), "cudaMemset(peer counters)");
  ck(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
}

PeerMemory::~PeerMemory() {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device_);
  for (size_t r = 0; r < bases_.size(); ++r)
    if (static_cast<int>(r) != rank_ && bases_[r] != nullptr) cudaIpcCloseMemHandle(bases_[r]);
  if (local_) cudaFree(local_);
  if (counters_) cudaFree(counters_);
  cudaSetDevice(prev);
}

std::string PeerMemory::Handle() const {
  cudaIpcMemHandle_t h;
  ck(cudaIpcGetMemHandle(&h, local_), "cudaIpcGetMemHandle");
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

void PeerMemory::Open(const std::vector<std::string>& handles, int rank) {
  if (handles.empty() || handles.size() > TB_MAX_PEERS) throw std::invalid_argument("PeerMemory: 1..8 ranks");
  if (rank < 0 || rank >= static_cast<int>(handles.size())) throw std::invalid_argument("PeerMemory: bad rank");
  ck(cudaSetDevice(device_), "cudaSetDevice");
  rank_ = rank;
  world_ = static_cast<int>(handles.size());
  bases_.assign(world_, nullptr);
  for (int r = 0; r < world_; ++r) {
    if (r == rank) {
      bases_[r] = local_;
      continue;
    }
    if (handles[r].size() != sizeof(cudaIpcMemHandle_t)) throw std::invalid_argument("PeerMemory: bad handle");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles[r].data(), sizeof(h));
    void* p = nullptr;
    ck(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    bases_[r] = p;
  }
}

TbPeerTable PeerMemory::Table() const {
  if (world_ == 0) throw std::runtime_error("PeerMemory: Open() first");
  TbPeerTable t{};
  for (int r = 0; r < world_; ++r) {
    t.base[r] = static_cast<char*>(bases_[r]) + header_bytes_;
    t.hdr[r] = bases_[r];
  }
  t.epoch_ctr = reinterpret_cast<unsigned*>(counters_);
  t.rank = rank_;
  t.world = world_;
  return t;
}

unsigned* PeerMemory::DoneCounter() const { return reinterpret_cast<unsigned*>(static_cast<char*>(counters_) + 64); }
int* PeerMemory::ErrorWord() const { return reinterpret_cast<int*>(static_cast<char*>(counters_) + 128); }
unsigned* PeerMemory::RepEpoch() const { return reinterpret_cast<unsigned*>(static_cast<char*>(counters_) + 192); }
void* PeerMemory::Payload() const { return static_cast<char*>(local_) + header_bytes_; }

}  // namespace turbol
