// GAE entry point that allocates nothing (no counterpart in the reference,
// which has no such entry point: its gae_compute needs no workspace because it
// runs one serial thread per environment).
//
// Who needs it: callers that cannot call cudaMalloc — code running inside a
// memory-pool-managed or sandboxed host process that forbids device
// allocations, a caller holding a stream that is being captured into a CUDA
// graph that must not grow the pool, or a plugin that only receives raw
// device pointers from its host application.  They pass inputs and outputs;
// the chunk-scan workspace is a fixed array compiled into this library.
//
// Contract:
//   * Same math and shapes as tb_gae (kernels.h): rewards / dones [T, N],
//     values [T+1, N], advantages / returns [T, N], optional fp64 stats [2]
//     that the call adds the sum and sum of squares of the advantages into
//     (zero them first if you want this call's moments alone).
//   * The workspace holds TB_GAE_STATIC_SCRATCH_FLOATS floats (1 MiB).  A call
//     whose chunked scan needs more returns cudaErrorInvalidValue and does
//     nothing; tb_gae_static_scratch_fits(T, N) says in advance.  Under the
//     current chunk rule no shape needs more: N >= 32768 needs no workspace,
//     and smaller N uses at most min(64, T, ceil(65536 / N)) chunks of
//     2 * N floats, i.e. below 2 * (65536 + N) < 196,608 floats; the check
//     guards a future change of that rule.
//   * Set-up: the first call on a device resolves the array's device address
//     with cudaGetSymbolAddress for the current device and caches it; make
//     that first call (or tb_gae_static_scratch_init) before any stream
//     capture, with the target device current.  The cached address belongs
//     to the device's current context: after cudaDeviceReset on that device
//     it is stale and the entry point must not be called again in the same
//     process.
//   * Every call on a device shares the one array and leaves its contents
//     behind; every element a call reads it first writes, so nothing needs
//     clearing between calls.  Calls that overlap on the GPU (different
//     streams, no ordering) race on the array: serialize them.
//   * Every GPU that loads this library holds the array until the process
//     exits.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define TB_GAE_STATIC_SCRATCH_FLOATS (256 * 1024)

#ifdef __cplusplus
extern "C" {
#endif

// Resolves the workspace address on the current device (optional: the first
// tb_gae_static_scratch call does it too).  Returns a cudaError_t.
int tb_gae_static_scratch_init(void);
// 1 if the chunked scan for [T, N] fits the fixed workspace, else 0.
int tb_gae_static_scratch_fits(int T, int N);
int tb_gae_static_scratch(const float* rewards, const float* values, const uint8_t* dones, float* advantages,
                          float* returns, double* stats, int T, int N, float gamma, float lam, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
