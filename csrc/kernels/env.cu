// Vectorized environment kernels: the reference's linear system and CartPole
// with in-kernel auto-reset, plus the fused PPO rollout step (sample action
// from the policy's logits, step CartPole, store the transition) that removes
// the separate sample / step / push launches of a rollout step.
//
// Parity:
//   * linear env  — reference turbol_vllm/src/cuda/env_dynamics.cu:11-52 and the
//     CPU path in turbol_vllm/src/env/gpu_environment.cpp:10-18,113-135.  The
//     reset hash is the reference's (kept so CPU/CUDA resets stay comparable to
//     the reference bit for bit); the step uses round-to-nearest mul/add without
//     FMA contraction so it equals the CPU loop bit for bit.
//   * CartPole    — classic cart-pole equations (Barto, Sutton & Anderson 1983,
//     Euler integration, dt 0.02, |x|>2.4 or |theta|>12 deg terminates, 500-step
//     truncation, U[-0.05,0.05] reset); the reference only names it
//     (docs/SPECIFICATION.md:640-672).
//
// One thread per environment; CartPole state is one float4 (16-byte aligned,
// one vector load/store per env).  A step over 65,536 envs moves ~3 MB, so
// these launches are latency bound; the rollout driver captures them in a
// CUDA graph.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "device_common.cuh"
#include "kernels.h"

namespace {

constexpr int kBlock = 256;

__device__ __forceinline__ float ref_reset_unit(unsigned i, unsigned d, unsigned seed) {
  unsigned h = seed ^ (i * 73856093u) ^ (d * 19349663u);
  h ^= h >> 13;
  h *= 2654435761u;
  h ^= h >> 16;
  return static_cast<float>(h & 0xFFFFu) / 65535.0f;
}

__global__ void linear_reset_kernel(float* __restrict__ state, int n, int d, unsigned seed) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  for (int k = 0; k < d; ++k) {
    const float u = ref_reset_unit(static_cast<unsigned>(i), static_cast<unsigned>(k), seed);
    state[static_cast<size_t>(i) * d + k] = __fmul_rn(__fsub_rn(__fmul_rn(u, 2.0f), 1.0f), 0.1f);
  }
}

__global__ void linear_step_kernel(const float* __restrict__ state, const float* __restrict__ action,
                                   float* __restrict__ next_state, float* __restrict__ reward,
                                   uint8_t* __restrict__ done, int n, int d, int a, float decay, float force,
                                   float thr) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float cost = 0.0f, first = 0.0f;
  for (int k = 0; k < d; ++k) {
    const int ak = k < a ? k : a - 1;
    const float v = __fadd_rn(__fmul_rn(decay, state[static_cast<size_t>(i) * d + k]),
                              __fmul_rn(force, action[static_cast<size_t>(i) * a + ak]));
    next_state[static_cast<size_t>(i) * d + k] = v;
    cost = __fadd_rn(cost, __fmul_rn(v, v));
    if (k == 0) first = v;
  }
  reward[i] = -cost;
  done[i] = fabsf(first) > thr ? 1 : 0;
}

// ----------------------------------------------------------------------------
// CartPole
// ----------------------------------------------------------------------------
__device__ __forceinline__ float4 cartpole_initial(uint64_t seed, unsigned env, unsigned episode, float range) {
  const uint4 r = tb::Philox::gen(seed, env, episode, 0x43504F4Cu /* "CPOL" */);
  return make_float4((tb::u01(r.x) * 2.f - 1.f) * range, (tb::u01(r.y) * 2.f - 1.f) * range,
                     (tb::u01(r.z) * 2.f - 1.f) * range, (tb::u01(r.w) * 2.f - 1.f) * range);
}

// Advances one cart-pole by dt; returns true when the episode terminated.
__device__ __forceinline__ bool cartpole_physics(float4& s, int action, const TbCartPoleParams& p) {
  const float total_mass = p.masscart + p.masspole;
  const float polemass_length = p.masspole * p.length;
  const float force = action == 1 ? p.force_mag : -p.force_mag;
  float sin_t, cos_t;
  sincosf(s.z, &sin_t, &cos_t);
  const float temp = (force + polemass_length * s.w * s.w * sin_t) / total_mass;
  const float theta_acc =
      (p.gravity * sin_t - cos_t * temp) / (p.length * (4.0f / 3.0f - p.masspole * cos_t * cos_t / total_mass));
  const float x_acc = temp - polemass_length * theta_acc * cos_t / total_mass;
  s.x = s.x + p.tau * s.y;
  s.y = s.y + p.tau * x_acc;
  s.z = s.z + p.tau * s.w;
  s.w = s.w + p.tau * theta_acc;
  return s.x < -p.x_threshold || s.x > p.x_threshold || s.z < -p.theta_threshold || s.z > p.theta_threshold;
}

// Completed-episode statistics: warp-aggregated so a burst of resets costs one
// atomic per warp.  stats[0] += sum of returns, stats[1] += episodes,
// stats[2] += sum of lengths.
__device__ __forceinline__ void record_episode(float* stats, bool finished, float ret, int len) {
  if (stats == nullptr) return;
  const unsigned m = __ballot_sync(0xffffffffu, finished);
  if (m == 0) return;
  float r = finished ? ret : 0.f, l = finished ? static_cast<float>(len) : 0.f;
  r = tb::warp_sum(r);
  l = tb::warp_sum(l);
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(&stats[0], r);
    atomicAdd(&stats[1], static_cast<float>(__popc(m)));
    atomicAdd(&stats[2], l);
  }
}

__global__ void cartpole_reset_kernel(float4* __restrict__ state, int* __restrict__ ep_len, float* __restrict__ ep_ret,
                                      unsigned* __restrict__ ep_count, int n, uint64_t seed, float range) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  state[i] = cartpole_initial(seed, i, 0, range);
  ep_len[i] = 0;
  ep_ret[i] = 0.f;
  ep_count[i] = 0;
}

__global__ void cartpole_step_kernel(float4* __restrict__ state, const int* __restrict__ action,
                                     float4* __restrict__ obs_out, float* __restrict__ reward,
                                     uint8_t* __restrict__ done, int* __restrict__ ep_len,
                                     float* __restrict__ ep_ret, unsigned* __restrict__ ep_count,
                                     float* __restrict__ stats, int n, uint64_t seed, TbCartPoleParams p) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const bool active = i < n;
  bool finished = false;
  float fin_ret = 0.f;
  int fin_len = 0;
  if (active) {
    float4 s = state[i];
    const bool term = cartpole_physics(s, action[i], p);
    const int len = ep_len[i] + 1;
    const float ret = ep_ret[i] + 1.0f;
    finished = term || len >= p.max_steps;
    if (finished) {
      const unsigned e = ep_count[i] + 1;
      ep_count[i] = e;
      s = cartpole_initial(seed, i, e, p.init_range);
      ep_len[i] = 0;
      ep_ret[i] = 0.f;
      fin_ret = ret;
      fin_len = len;
    } else {
      ep_len[i] = len;
      ep_ret[i] = ret;
    }
    state[i] = s;
    if (obs_out != nullptr) obs_out[i] = s;
    reward[i] = 1.0f;
    done[i] = finished ? 1 : 0;
  }
  record_episode(stats, finished, fin_ret, fin_len);
}

// Next-step policy input: the observation as bf16, padded to 8 features
// (one 16-byte store; the tensor-core MLP's first layer reads K = 8).
__device__ __forceinline__ void write_obs_bf16(uint16_t* out, int i, float4 s) {
  __nv_bfloat162 a = __floats2bfloat162_rn(s.x, s.y), b = __floats2bfloat162_rn(s.z, s.w);
  uint4 v;
  v.x = *reinterpret_cast<uint32_t*>(&a);
  v.y = *reinterpret_cast<uint32_t*>(&b);
  v.z = 0u;
  v.w = 0u;
  reinterpret_cast<uint4*>(out)[i] = v;
}

// Fused PPO rollout step for CartPole with a categorical policy over A actions:
//   action ~ Categorical(softmax(logits)) by the Gumbel-max trick,
//   logp = logits[a] - logsumexp(logits),
//   the pre-step observation, action, logp, value, reward and done are written
//   to row t of the rollout storage, and `state` advances in place (it is the
//   next step's policy input).
__global__ void ppo_cartpole_act_step_kernel(const float* __restrict__ logits, int A, int ldl,
                                             const float* __restrict__ values, int ldv, float4* __restrict__ state,
                                             uint16_t* __restrict__ obs_bf16,
                                             int* __restrict__ ep_len, float* __restrict__ ep_ret,
                                             unsigned* __restrict__ ep_count, float* __restrict__ stats,
                                             float4* __restrict__ obs_buf, int* __restrict__ act_buf,
                                             float* __restrict__ logp_buf, float* __restrict__ val_buf,
                                             float* __restrict__ rew_buf, uint8_t* __restrict__ done_buf,
                                             const long long* __restrict__ iter_ptr, int t, int n,
                                             uint64_t policy_seed, uint64_t env_seed, TbCartPoleParams p) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const bool active = i < n;
  bool finished = false;
  float fin_ret = 0.f;
  int fin_len = 0;
  if (active) {
    const long long it = iter_ptr ? *iter_ptr : 0;
    const float* l = logits + static_cast<size_t>(i) * ldl;
    float mx = -INFINITY;
    for (int k = 0; k < A; ++k) mx = fmaxf(mx, l[k]);
    float se = 0.f;
    for (int k = 0; k < A; ++k) se += __expf(l[k] - mx);
    const float lse = mx + __logf(se);
    int best = 0;
    float best_v = -INFINITY;
    for (int k = 0; k < A; k += 4) {
      const uint4 r = tb::Philox::gen(policy_seed, static_cast<uint32_t>(i), static_cast<uint32_t>(t + k),
                                      static_cast<uint32_t>(it), static_cast<uint32_t>(it >> 32));
      const uint32_t w[4] = {r.x, r.y, r.z, r.w};
      for (int j = 0; j < 4 && k + j < A; ++j) {
        const float g = -__logf(-__logf(tb::u01_open(w[j])));
        const float v = l[k + j] + g;
        if (v > best_v) {
          best_v = v;
          best = k + j;
        }
      }
    }
    float4 s = state[i];
    obs_buf[static_cast<size_t>(t) * n + i] = s;
    act_buf[static_cast<size_t>(t) * n + i] = best;
    logp_buf[static_cast<size_t>(t) * n + i] = l[best] - lse;
    val_buf[static_cast<size_t>(t) * n + i] = values[static_cast<size_t>(i) * ldv];

    const bool term = cartpole_physics(s, best, p);
    const int len = ep_len[i] + 1;
    const float ret = ep_ret[i] + 1.0f;
    finished = term || len >= p.max_steps;
    if (finished) {
      const unsigned e = ep_count[i] + 1;
      ep_count[i] = e;
      s = cartpole_initial(env_seed, i, e, p.init_range);
      ep_len[i] = 0;
      ep_ret[i] = 0.f;
      fin_ret = ret;
      fin_len = len;
    } else {
      ep_len[i] = len;
      ep_ret[i] = ret;
    }
    state[i] = s;
    if (obs_bf16 != nullptr) write_obs_bf16(obs_bf16, i, s);
    rew_buf[static_cast<size_t>(t) * n + i] = 1.0f;
    done_buf[static_cast<size_t>(t) * n + i] = finished ? 1 : 0;
  }
  record_episode(stats, finished, fin_ret, fin_len);
}

__global__ void pad_obs_bf16_kernel(const float4* __restrict__ s, uint16_t* __restrict__ out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) write_obs_bf16(out, i, s[i]);
}

inline int grid_for(int n) { return (n + kBlock - 1) / kBlock; }

}  // namespace

extern "C" {

int tb_env_linear_reset(float* state, int n, int d, unsigned seed, cudaStream_t s) {
  if (n <= 0) return 0;
  linear_reset_kernel<<<grid_for(n), kBlock, 0, s>>>(state, n, d, seed);
  return static_cast<int>(cudaGetLastError());
}

int tb_env_linear_step(const float* state, const float* action, float* next_state, float* reward, uint8_t* done,
                       int n, int d, int a, float decay, float force, float thr, cudaStream_t s) {
  if (n <= 0) return 0;
  linear_step_kernel<<<grid_for(n), kBlock, 0, s>>>(state, action, next_state, reward, done, n, d, a, decay, force,
                                                    thr);
  return static_cast<int>(cudaGetLastError());
}

int tb_cartpole_reset(float* state, int* ep_len, float* ep_ret, unsigned* ep_count, int n, unsigned long long seed,
                      float init_range, cudaStream_t s) {
  if (n <= 0) return 0;
  cartpole_reset_kernel<<<grid_for(n), kBlock, 0, s>>>(reinterpret_cast<float4*>(state), ep_len, ep_ret, ep_count, n,
                                                       seed, init_range);
  return static_cast<int>(cudaGetLastError());
}

int tb_cartpole_step(float* state, const int* action, float* obs_out, float* reward, uint8_t* done, int* ep_len,
                     float* ep_ret, unsigned* ep_count, float* stats, int n, unsigned long long seed,
                     TbCartPoleParams p, cudaStream_t s) {
  if (n <= 0) return 0;
  cartpole_step_kernel<<<grid_for(n), kBlock, 0, s>>>(reinterpret_cast<float4*>(state), action,
                                                      reinterpret_cast<float4*>(obs_out), reward, done, ep_len,
                                                      ep_ret, ep_count, stats, n, seed, p);
  return static_cast<int>(cudaGetLastError());
}

int tb_pad_obs_bf16(const float* state, void* out, int n, cudaStream_t s) {
  if (n <= 0) return 0;
  pad_obs_bf16_kernel<<<grid_for(n), kBlock, 0, s>>>(reinterpret_cast<const float4*>(state),
                                                     static_cast<uint16_t*>(out), n);
  return static_cast<int>(cudaGetLastError());
}

int tb_ppo_cartpole_act_step(const float* logits, int A, int ldl, const float* values, int ldv, float* state,
                             void* obs_bf16, int* ep_len,
                             float* ep_ret, unsigned* ep_count, float* stats, float* obs_buf, int* act_buf,
                             float* logp_buf, float* val_buf, float* rew_buf, uint8_t* done_buf,
                             const long long* iter_ptr, int t, int n, unsigned long long policy_seed,
                             unsigned long long env_seed, TbCartPoleParams p, cudaStream_t s) {
  if (n <= 0) return 0;
  ppo_cartpole_act_step_kernel<<<grid_for(n), kBlock, 0, s>>>(
      logits, A, ldl, values, ldv, reinterpret_cast<float4*>(state), static_cast<uint16_t*>(obs_bf16), ep_len, ep_ret,
      ep_count, stats,
      reinterpret_cast<float4*>(obs_buf), act_buf, logp_buf, val_buf, rew_buf, done_buf, iter_ptr, t, n, policy_seed,
      env_seed, p);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
