// Device-side helpers shared by every turbol_b200 kernel: counter-based RNG,
// the device error word, bounded waits and warp/block reductions.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <utility>
#include <vector>

namespace tb {

// Raises a kernel's dynamic shared memory limit above the 48 KB default.  The
// attribute belongs to the function in the current device's context, so it is
// set once per (function, device) pair.
inline cudaError_t ensure_dyn_smem(const void* fn, int bytes) {
  static std::mutex mu;
  static std::vector<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& d : done)
    if (d.first == fn && d.second == dev) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.emplace_back(fn, dev);
  return e;
}

// ---------------------------------------------------------------------------
// Philox4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw, "Parallel
// Random Numbers: As Easy as 1, 2, 3", SC'11).  Stateless: the same (key,
// counter) gives the same four words on every thread, launch and device, so a
// kernel inside a CUDA graph stays reproducible when its counter comes from
// device memory.
// ---------------------------------------------------------------------------
struct Philox {
  static constexpr uint32_t kMul0 = 0xD2511F53u, kMul1 = 0xCD9E8D57u;
  static constexpr uint32_t kWeyl0 = 0x9E3779B9u, kWeyl1 = 0xBB67AE85u;

  __device__ __forceinline__ static uint4 round(uint4 c, uint2 k) {
    const uint32_t lo0 = kMul0 * c.x, hi0 = __umulhi(kMul0, c.x);
    const uint32_t lo1 = kMul1 * c.z, hi1 = __umulhi(kMul1, c.z);
    return make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
  }
  // 4 random words for (seed, c0, c1, c2).
  __device__ __forceinline__ static uint4 gen(uint64_t seed, uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3 = 0) {
    uint4 c = make_uint4(c0, c1, c2, c3);
    uint2 k = make_uint2(static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
#pragma unroll
    for (int r = 0; r < 10; ++r) {
      c = round(c, k);
      k.x += kWeyl0;
      k.y += kWeyl1;
    }
    return c;
  }
};

// Uniform float in [0, 1) from the top 24 bits of a word.
__device__ __forceinline__ float u01(uint32_t x) { return static_cast<float>(x >> 8) * (1.0f / 16777216.0f); }
// Uniform float in (0, 1): never 0, never 1 (safe under log).
__device__ __forceinline__ float u01_open(uint32_t x) {
  return (static_cast<float>(x >> 8) + 0.5f) * (1.0f / 16777216.0f);
}
// Uniform integer in [0, n) by the multiply-shift reduction (bias < n / 2^32).
__device__ __forceinline__ uint32_t uniform_int(uint32_t x, uint32_t n) {
  return static_cast<uint32_t>((static_cast<uint64_t>(x) * n) >> 32);
}

// ---------------------------------------------------------------------------
// Device error word.  A kernel that detects an out-of-range index or a wait
// that ran out records the first failure here and returns; it never traps, so
// the context stays usable and the host turns the word into a Status.
// ---------------------------------------------------------------------------
struct ErrorWord {
  unsigned int code;       // 0 = ok
  unsigned int kernel_id;  // which kernel reported it
  unsigned long long info; // failing index / wait site
};

enum ErrorCode : unsigned int {
  kErrNone = 0,
  kErrIndex = 1,
  kErrTimeout = 2,
  kErrShape = 3,
};

__device__ __forceinline__ void report_error(ErrorWord* ew, unsigned code, unsigned kernel_id, unsigned long long info) {
  if (ew == nullptr) return;
  if (atomicCAS(&ew->code, 0u, code) == 0u) {
    ew->kernel_id = kernel_id;
    ew->info = info;
    __threadfence_system();
  }
}

// ---------------------------------------------------------------------------
// Reductions.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
template <typename T>
__device__ __forceinline__ T warp_max(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Sums `v` over the block; the result is valid in every thread.  `smem` needs
// blockDim.x / 32 entries.
template <typename T>
__device__ __forceinline__ T block_sum(T v, T* smem) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) smem[wid] = v;
  __syncthreads();
  T r = (lane < nw) ? smem[lane] : T(0);
  r = warp_sum(r);
  return r;
}

// Bounded spin on a 32-bit flag in (possibly peer) memory: returns true once
// *flag >= expect, false after `max_iters` polls.  Acquire semantics at system
// scope so data written before the peer's release store is visible.
__device__ __forceinline__ bool wait_flag_geq(const volatile unsigned int* flag, unsigned int expect, long long max_iters) {
  for (long long it = 0; it < max_iters; ++it) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v >= expect) return true;
    __nanosleep(64);
  }
  return false;
}

__device__ __forceinline__ void store_release_sys(unsigned int* flag, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(v) : "memory");
}

}  // namespace tb
