// GAE with a compiled-in workspace: see gae_static_scratch.h for who needs it
// and the contract.  The kernels are tb_gae's (advantage.cu): this file only
// supplies the workspace from a file-scope device array instead of the
// caller, and never allocates.
#include "gae_static_scratch.h"

#include <cuda_runtime.h>

#include <mutex>

#include "kernels.h"

namespace {

// The workspace: one per device that loads this library, alive until exit.
static __device__ __align__(256) float g_gae_scratch[TB_GAE_STATIC_SCRATCH_FLOATS];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_ptr[kMaxDevices] = {nullptr};

// Device address of g_gae_scratch on the current device.  In host code the
// symbol itself is only a host-side stand-in, so the address must come from
// cudaGetSymbolAddress, once per device, with that device current.
int resolve(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) return static_cast<int>(cudaErrorInvalidDevice);
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_gae_scratch);
    if (e != cudaSuccess) return static_cast<int>(e);
    g_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_ptr[dev];
  return 0;
}

}  // namespace

extern "C" {

int tb_gae_static_scratch_init(void) {
  float* p = nullptr;
  return resolve(&p);
}

int tb_gae_static_scratch_fits(int T, int N) {
  if (T <= 0 || N <= 0) return 1;
  return tb_gae_scratch_bytes(T, N) <= sizeof(float) * static_cast<size_t>(TB_GAE_STATIC_SCRATCH_FLOATS) ? 1 : 0;
}

int tb_gae_static_scratch(const float* rewards, const float* values, const uint8_t* dones, float* advantages,
                          float* returns, double* stats, int T, int N, float gamma, float lam, cudaStream_t stream) {
  if (T <= 0 || N <= 0) return 0;
  if (!tb_gae_static_scratch_fits(T, N)) return static_cast<int>(cudaErrorInvalidValue);
  float* scratch = nullptr;
  const int e = resolve(&scratch);
  if (e != 0) return e;
  return tb_gae(rewards, values, dones, advantages, returns, stats, scratch, T, N, gamma, lam, stream);
}

}  // extern "C"
