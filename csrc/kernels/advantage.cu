// Advantage kernels: GAE over [T, N] rollouts and GRPO group-normalized
// advantages.
//
// GAE recurrence (same as the reference turbol_vllm/src/cuda/gae.cu:31-44):
//   delta_t = r_t + gamma * (1 - done_t) * V_{t+1} - V_t
//   A_t     = delta_t + gamma * lambda * (1 - done_t) * A_{t+1},   A_T = 0
//   R_t     = A_t + V_t
// values has T+1 rows (row T is the bootstrap value).
//
// Each step is an affine map A_t = a_t + c_t * A_{t+1}, so chunks of T compose:
// when N alone does not fill the GPU (N < 32K), T is cut into C chunks, pass 1
// reduces every (chunk, env) to one map (alpha, beta) in a [2, C, N] scratch,
// and pass 2 folds the later chunks' maps into the carry and writes A and R.
// At N >= 32K one pass with C = 1 already has 1K+ warps in flight and reads the
// inputs once.  The sum and sum of squares of A are accumulated (fp64) for
// global advantage normalization.
#include <cuda_runtime.h>
#include <stdint.h>

#include "device_common.cuh"
#include "kernels.h"

namespace {

constexpr int kBlock = 256;

__global__ void gae_chunk_maps_kernel(const float* __restrict__ rew, const float* __restrict__ val,
                                      const uint8_t* __restrict__ done, float* __restrict__ scratch, int T, int N,
                                      int C, int chunk, float gamma, float gl) {
  const int env = blockIdx.x * blockDim.x + threadIdx.x;
  const int c = blockIdx.y;
  if (env >= N) return;
  const int t0 = c * chunk, t1 = min(T, t0 + chunk);
  float alpha = 0.f, beta = 1.f;
#pragma unroll 4
  for (int t = t1 - 1; t >= t0; --t) {
    const size_t o = static_cast<size_t>(t) * N + env;
    const float nd = done[o] ? 0.f : 1.f;
    const float delta = rew[o] + gamma * nd * val[o + N] - val[o];
    const float ct = gl * nd;
    alpha = delta + ct * alpha;
    beta = ct * beta;
  }
  scratch[static_cast<size_t>(c) * N + env] = alpha;
  scratch[static_cast<size_t>(C + c) * N + env] = beta;
}

__global__ void gae_final_kernel(const float* __restrict__ rew, const float* __restrict__ val,
                                 const uint8_t* __restrict__ done, const float* __restrict__ scratch,
                                 float* __restrict__ adv, float* __restrict__ ret, double* __restrict__ stats, int T,
                                 int N, int C, int chunk, float gamma, float gl) {
  __shared__ double red[kBlock / 32];
  const int env = blockIdx.x * blockDim.x + threadIdx.x;
  const int c = blockIdx.y;
  double s1 = 0.0, s2 = 0.0;
  if (env < N) {
    float carry = 0.f;
    for (int k = C - 1; k > c; --k)
      carry = scratch[static_cast<size_t>(k) * N + env] + scratch[static_cast<size_t>(C + k) * N + env] * carry;
    const int t0 = c * chunk, t1 = min(T, t0 + chunk);
    float a = carry;
    float ls1 = 0.f, ls2 = 0.f;
#pragma unroll 4
    for (int t = t1 - 1; t >= t0; --t) {
      const size_t o = static_cast<size_t>(t) * N + env;
      const float nd = done[o] ? 0.f : 1.f;
      const float v = val[o];
      const float delta = rew[o] + gamma * nd * val[o + N] - v;
      a = delta + gl * nd * a;
      adv[o] = a;
      if (ret) ret[o] = a + v;
      ls1 += a;
      ls2 += a * a;
    }
    s1 = ls1;
    s2 = ls2;
  }
  if (stats != nullptr) {
    s1 = tb::block_sum(s1, red);
    s2 = tb::block_sum(s2, red);
    if (threadIdx.x == 0) {
      atomicAdd(&stats[0], s1);
      atomicAdd(&stats[1], s2);
    }
  }
}

// GRPO: adv_i = (r_i - mean_g) / (std_g + eps) over each group of G
// consecutive rewards (sample std, G - 1 in the denominator).
__global__ void grpo_adv_kernel(const float* __restrict__ r, float* __restrict__ adv, int groups, int G, float eps,
                                int scale_by_std) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= groups) return;
  const float* x = r + static_cast<size_t>(g) * G;
  float m = 0.f;
  for (int k = 0; k < G; ++k) m += x[k];
  m /= static_cast<float>(G);
  float v = 0.f;
  for (int k = 0; k < G; ++k) v += (x[k] - m) * (x[k] - m);
  const float sd = G > 1 ? sqrtf(v / static_cast<float>(G - 1)) : 0.f;
  const float inv = scale_by_std ? 1.f / (sd + eps) : 1.f;
  for (int k = 0; k < G; ++k) adv[static_cast<size_t>(g) * G + k] = (x[k] - m) * inv;
}

}  // namespace

extern "C" {

int tb_gae_chunks_for(int T, int N) {
  if (N >= 32768 || T <= 1) return 1;
  int c = (65536 + N - 1) / N;
  if (c > T) c = T;
  if (c > 64) c = 64;
  return c < 1 ? 1 : c;
}

size_t tb_gae_scratch_bytes(int T, int N) {
  const int C = tb_gae_chunks_for(T, N);
  return C > 1 ? sizeof(float) * 2 * static_cast<size_t>(C) * N : 0;
}

int tb_gae(const float* rew, const float* val, const uint8_t* done, float* adv, float* ret, double* stats,
           float* scratch, int T, int N, float gamma, float lam, cudaStream_t s) {
  if (T <= 0 || N <= 0) return 0;
  const int C = tb_gae_chunks_for(T, N);
  if (C > 1 && scratch == nullptr) return static_cast<int>(cudaErrorInvalidValue);
  const int chunk = (T + C - 1) / C;
  const int Ceff = (T + chunk - 1) / chunk;
  dim3 grid((N + kBlock - 1) / kBlock, Ceff);
  if (Ceff > 1)
    gae_chunk_maps_kernel<<<grid, kBlock, 0, s>>>(rew, val, done, scratch, T, N, Ceff, chunk, gamma, gamma * lam);
  gae_final_kernel<<<grid, kBlock, 0, s>>>(rew, val, done, scratch, adv, ret, stats, T, N, Ceff, chunk, gamma,
                                           gamma * lam);
  return static_cast<int>(cudaGetLastError());
}

int tb_grpo_advantage(const float* rewards, float* adv, int groups, int G, float eps, int scale_by_std,
                      cudaStream_t s) {
  if (groups <= 0) return 0;
  grpo_adv_kernel<<<(groups + kBlock - 1) / kBlock, kBlock, 0, s>>>(rewards, adv, groups, G, eps, scale_by_std);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
