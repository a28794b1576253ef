// The CUDA runtime as the host core sees it.
//
// Normal build (TURBOL_CUDA=1): <cuda_runtime.h> and torch's current-stream
// accessor.  CPU-only build (TURBOL_CUDA=0: no CUDA toolkit, a CPU build of
// torch is enough): the handful of runtime types and calls the host code
// names, each answering "no CUDA device".  The device branches of the engines
// are unreachable there (no CUDA tensor can exist), and the kernel launchers
// they would call are stubs that return cudaErrorNoDevice
// (csrc/cpu_only/kernel_stubs.cpp).  The reference's minimal tree is likewise
// a CPU-only build of its core (turbol/CMakeLists.txt:1-34).
#pragma once

#ifndef TURBOL_CUDA
#define TURBOL_CUDA 1
#endif

#if TURBOL_CUDA
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime.h>

namespace turbol {
inline cudaStream_t CurrentStream(int device) { return c10::cuda::getCurrentCUDAStream(device).stream(); }
}  // namespace turbol
#else
#include <stddef.h>

typedef struct CUstream_st* cudaStream_t;
typedef struct CUevent_st* cudaEvent_t;
typedef enum cudaError_enum_compat {
  cudaSuccess = 0,
  cudaErrorInvalidValue = 1,
  cudaErrorNoDevice = 100,
} cudaError_t;
enum { cudaStreamNonBlocking = 1 };

inline cudaError_t cudaGetDeviceCount(int* n) {
  if (n) *n = 0;
  return cudaErrorNoDevice;
}
inline cudaError_t cudaSetDevice(int) { return cudaErrorNoDevice; }
inline cudaError_t cudaGetDevice(int* d) {
  if (d) *d = 0;
  return cudaErrorNoDevice;
}
inline cudaError_t cudaMemGetInfo(size_t* f, size_t* t) {
  if (f) *f = 0;
  if (t) *t = 0;
  return cudaErrorNoDevice;
}
inline cudaError_t cudaGetLastError() { return cudaSuccess; }
inline cudaError_t cudaDeviceSynchronize() { return cudaErrorNoDevice; }
inline const char* cudaGetErrorString(cudaError_t e) {
  return e == cudaSuccess ? "no error" : (e == cudaErrorNoDevice ? "no CUDA device (CPU-only build)" : "invalid value");
}
inline cudaError_t cudaEventCreate(cudaEvent_t* e) {
  if (e) *e = nullptr;
  return cudaErrorNoDevice;
}
inline cudaError_t cudaEventDestroy(cudaEvent_t) { return cudaSuccess; }
inline cudaError_t cudaEventRecord(cudaEvent_t, cudaStream_t = nullptr) { return cudaErrorNoDevice; }
inline cudaError_t cudaEventSynchronize(cudaEvent_t) { return cudaErrorNoDevice; }
inline cudaError_t cudaEventElapsedTime(float* ms, cudaEvent_t, cudaEvent_t) {
  if (ms) *ms = 0.f;
  return cudaErrorNoDevice;
}
inline cudaError_t cudaDeviceGetStreamPriorityRange(int* lo, int* hi) {
  if (lo) *lo = 0;
  if (hi) *hi = 0;
  return cudaErrorNoDevice;
}
inline cudaError_t cudaStreamCreateWithPriority(cudaStream_t* s, unsigned, int) {
  if (s) *s = nullptr;
  return cudaErrorNoDevice;
}
inline cudaError_t cudaStreamDestroy(cudaStream_t) { return cudaSuccess; }

namespace turbol {
inline cudaStream_t CurrentStream(int) { return nullptr; }
}  // namespace turbol
#endif
