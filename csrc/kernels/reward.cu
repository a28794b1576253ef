// Reward kernels on token ids (the GPU-native scoring path of RewardEngine).
//
//   * hash reward: reward_i = (FNV-1a-64 over the little-endian bytes of the
//     response's int32 token ids  mod 1000) / 1000 — a deterministic stand-in
//     for a learned reward model, computed where the tokens already live.
//   * rule reward on token sequences: the reference's rule score
//     (turbol_vllm/src/reward/reward_engine.cpp:110-125: +format_bonus when the
//     response ends with the "." token, + length_penalty * (len - target)^2,
//     clipped to +-reward_clip).
//   * masked sequence KL: coef * mean over valid tokens of the k1 (lp - ref)
//     or k3 (exp(ref - lp) - (ref - lp) - 1) estimator
//     (reference reward_engine.cpp:127-152 is the k1 form on the host).
//   * centring / whitening of a reward batch (reference reward_engine.cpp:154-165
//     centres only; whitening is selectable).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "device_common.cuh"
#include "kernels.h"

namespace {

constexpr int kBlock = 256;

__global__ void hash_reward_kernel(const int* __restrict__ ids, const int* __restrict__ lens, int B, int T,
                                   float* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B) return;
  const int L = lens ? min(lens[i], T) : T;
  uint64_t h = 0xcbf29ce484222325ull;  // FNV-1a 64 offset basis
  const int* x = ids + static_cast<size_t>(i) * T;
  for (int t = 0; t < L; ++t) {
    uint32_t w = static_cast<uint32_t>(x[t]);
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      h ^= (w & 0xffu);
      h *= 0x100000001b3ull;  // FNV-1a 64 prime
      w >>= 8;
    }
  }
  out[i] = static_cast<float>(h % 1000ull) / 1000.0f;
}

__global__ void rule_reward_kernel(const int* __restrict__ ids, const int* __restrict__ lens, int B, int T,
                                   int period_id, float format_bonus, float length_penalty, int target_len,
                                   float clip, float* __restrict__ rule, float* __restrict__ total) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B) return;
  const int L = lens ? min(lens[i], T) : T;
  float s = 0.f;
  if (L > 0 && ids[static_cast<size_t>(i) * T + L - 1] == period_id) s += format_bonus;
  const float d = static_cast<float>(L - target_len);
  s += length_penalty * d * d;
  if (rule) rule[i] = s;
  if (total) total[i] = fmaxf(-clip, fminf(clip, s));
}

// One warp per sequence.
__global__ void masked_kl_kernel(const float* __restrict__ lp, const float* __restrict__ ref,
                                 const float* __restrict__ mask, int B, int T, float coef, int k3,
                                 float* __restrict__ out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= B) return;
  float s = 0.f, c = 0.f;
  for (int t = lane; t < T; t += 32) {
    const size_t o = static_cast<size_t>(warp) * T + t;
    if (mask[o] > 0.5f) {
      const float d = lp[o] - ref[o];
      s += k3 ? (__expf(-d) + d - 1.f) : d;
      c += 1.f;
    }
  }
  s = tb::warp_sum(s);
  c = tb::warp_sum(c);
  if (lane == 0) out[warp] = c > 0.f ? coef * s / c : 0.f;
}

// Single-block batch normalization (B up to a few 100K).
__global__ void normalize_kernel(float* __restrict__ r, int B, int whiten, float eps) {
  __shared__ float red[kBlock / 32];
  float s = 0.f;
  for (int i = threadIdx.x; i < B; i += blockDim.x) s += r[i];
  const float mean = tb::block_sum(s, red) / static_cast<float>(B);
  float inv = 1.f;
  if (whiten) {
    float v = 0.f;
    for (int i = threadIdx.x; i < B; i += blockDim.x) v += (r[i] - mean) * (r[i] - mean);
    v = tb::block_sum(v, red) / static_cast<float>(B);
    inv = 1.f / (sqrtf(v) + eps);
  }
  for (int i = threadIdx.x; i < B; i += blockDim.x) r[i] = (r[i] - mean) * inv;
}

}  // namespace

extern "C" {

int tb_hash_reward(const int* ids, const int* lens, int B, int T, float* out, cudaStream_t s) {
  if (B <= 0) return 0;
  hash_reward_kernel<<<(B + kBlock - 1) / kBlock, kBlock, 0, s>>>(ids, lens, B, T, out);
  return static_cast<int>(cudaGetLastError());
}

int tb_rule_reward(const int* ids, const int* lens, int B, int T, int period_id, float format_bonus,
                   float length_penalty, int target_len, float clip, float* rule, float* total, cudaStream_t s) {
  if (B <= 0) return 0;
  rule_reward_kernel<<<(B + kBlock - 1) / kBlock, kBlock, 0, s>>>(ids, lens, B, T, period_id, format_bonus,
                                                                  length_penalty, target_len, clip, rule, total);
  return static_cast<int>(cudaGetLastError());
}

int tb_masked_kl(const float* lp, const float* ref, const float* mask, int B, int T, float coef, int k3, float* out,
                 cudaStream_t s) {
  if (B <= 0) return 0;
  const long long threads = static_cast<long long>(B) * 32;
  masked_kl_kernel<<<static_cast<unsigned>((threads + kBlock - 1) / kBlock), kBlock, 0, s>>>(lp, ref, mask, B, T,
                                                                                            coef, k3, out);
  return static_cast<int>(cudaGetLastError());
}

int tb_normalize_rewards(float* r, int B, int whiten, float eps, cudaStream_t s) {
  if (B <= 0) return 0;
  normalize_kernel<<<1, kBlock, 0, s>>>(r, B, whiten, eps);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
