// Fused kernels for the linear Gaussian actor-critic (the reference
// PolicyEngine's model, turbol_vllm/src/policy/policy_engine.cpp:23-138):
//
//   mean = tanh(W_a x + b_a)   [act_dim],   value = W_c x + b_c
//
// * act:  one thread per row: mean, Gaussian noise (Philox + Box-Muller),
//         a = clamp(mean + std * noise, -1, 1) and its log-density.
// * grad: the gradient of the clipped-PPO policy loss plus the value loss for
//         rows [obs | act | adv | ret (| old_logp)], summed over the batch by
//         warp reductions and one atomic per parameter and block into the flat
//         fp32 gradient (zeroed by the caller); layout W_a, b_a, W_c, b_c.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "device_common.cuh"
#include "kernels.h"

namespace {

constexpr int kMaxObs = 64, kMaxAct = 16, kThreads = 256;

__global__ void __launch_bounds__(kThreads) lin_gauss_act_kernel(const float* __restrict__ x, const float* __restrict__ p,
                                                                 float* __restrict__ act, float* __restrict__ logp,
                                                                 int N, int O, int A, float stdv, uint64_t seed,
                                                                 uint32_t counter) {
  __shared__ float sp[kMaxAct * kMaxObs + kMaxAct];
  for (int i = threadIdx.x; i < A * O + A; i += blockDim.x) sp[i] = p[i];
  __syncthreads();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= N) return;
  float xr[kMaxObs];
  for (int k = 0; k < O; ++k) xr[k] = x[static_cast<long long>(row) * O + k];
  const float var = stdv * stdv, c = -0.5f * logf(2.f * 3.14159265358979f * var);
  float lp = 0.f;
  for (int j0 = 0; j0 < A; j0 += 2) {
    const uint4 r = tb::Philox::gen(seed, static_cast<uint32_t>(row), static_cast<uint32_t>(j0), counter);
    // Box-Muller: two standard normals from two uniforms
    const float rad = sqrtf(-2.f * logf(tb::u01_open(r.x)));
    float s, co;
    sincospif(2.f * tb::u01(r.y), &s, &co);
    const float nz[2] = {rad * co, rad * s};
    for (int t = 0; t < 2 && j0 + t < A; ++t) {
      const int j = j0 + t;
      float z = sp[A * O + j];
      for (int k = 0; k < O; ++k) z += sp[j * O + k] * xr[k];
      const float m = tanhf(z);
      const float a = fminf(1.f, fmaxf(-1.f, m + stdv * nz[t]));
      act[static_cast<long long>(row) * A + j] = a;
      lp += -0.5f * (a - m) * (a - m) / var + c;
    }
  }
  logp[row] = lp;
}

__global__ void __launch_bounds__(kThreads) lin_gauss_grad_kernel(const float* __restrict__ batch, int row_w,
                                                                  const float* __restrict__ p, float* __restrict__ g,
                                                                  int N, int O, int A, float stdv, float clip,
                                                                  float vf_coef, int has_old) {
  __shared__ float sp[kMaxAct * kMaxObs + kMaxAct + kMaxObs + 1];
  __shared__ float sg[kMaxAct * kMaxObs + kMaxAct + kMaxObs + 1];
  const int P = A * O + A + O + 1;
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    sp[i] = p[i];
    sg[i] = 0.f;
  }
  __syncthreads();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  const bool valid = row < N;
  const float* b = batch + static_cast<long long>(valid ? row : 0) * row_w;
  float xr[kMaxObs];
  for (int k = 0; k < O; ++k) xr[k] = valid ? b[k] : 0.f;
  const float var = stdv * stdv, c = -0.5f * logf(2.f * 3.14159265358979f * var);
  const float adv = valid ? b[O + A] : 0.f, ret = valid ? b[O + A + 1] : 0.f;
  float m[kMaxAct], lp = 0.f;
  for (int j = 0; j < A; ++j) {
    float z = sp[A * O + j];
    for (int k = 0; k < O; ++k) z += sp[j * O + k] * xr[k];
    m[j] = tanhf(z);
    const float a = valid ? b[O + j] : 0.f;
    lp += -0.5f * (a - m[j]) * (a - m[j]) / var + c;
  }
  const float old = (valid && has_old) ? b[O + A + 2] : lp;
  const float ratio = __expf(lp - old);
  const float unc = ratio * adv, clp = fminf(fmaxf(ratio, 1.f - clip), 1.f + clip) * adv;
  const float inv_n = 1.f / static_cast<float>(N);
  // d(-min(unclipped, clipped)) / d logp
  float g_lp = 0.f;
  if (unc <= clp) g_lp = -unc;
  else if (ratio > 1.f - clip && ratio < 1.f + clip) g_lp = -unc;
  g_lp = valid ? g_lp * inv_n : 0.f;
  const int lane = threadIdx.x & 31;
  for (int j = 0; j < A; ++j) {
    const float a = valid ? b[O + j] : 0.f;
    const float gz = g_lp * (a - m[j]) / var * (1.f - m[j] * m[j]);
    for (int k = 0; k < O; ++k) {
      const float s = tb::warp_sum(gz * xr[k]);
      if (lane == 0) atomicAdd(&sg[j * O + k], s);
    }
    const float s = tb::warp_sum(gz);
    if (lane == 0) atomicAdd(&sg[A * O + j], s);
  }
  // value head: vf * mean((v - ret)^2)
  float v = sp[A * O + A + O];
  for (int k = 0; k < O; ++k) v += sp[A * O + A + k] * xr[k];
  const float gv = valid ? vf_coef * 2.f * (v - ret) * inv_n : 0.f;
  for (int k = 0; k < O; ++k) {
    const float s = tb::warp_sum(gv * xr[k]);
    if (lane == 0) atomicAdd(&sg[A * O + A + k], s);
  }
  const float s = tb::warp_sum(gv);
  if (lane == 0) atomicAdd(&sg[A * O + A + O], s);
  __syncthreads();
  for (int i = threadIdx.x; i < P; i += blockDim.x) atomicAdd(&g[i], sg[i]);
}

}  // namespace

extern "C" {

int tb_lin_gauss_act(const float* x, const float* params, float* act, float* logp, int N, int O, int A, float stdv,
                     uint64_t seed, uint32_t counter, cudaStream_t s) {
  if (N <= 0) return 0;
  if (O <= 0 || O > kMaxObs || A <= 0 || A > kMaxAct) return static_cast<int>(cudaErrorInvalidValue);
  lin_gauss_act_kernel<<<(N + kThreads - 1) / kThreads, kThreads, 0, s>>>(x, params, act, logp, N, O, A, stdv, seed,
                                                                          counter);
  return static_cast<int>(cudaGetLastError());
}

int tb_lin_gauss_grad(const float* batch, int row_w, const float* params, float* grad, int N, int O, int A,
                      float stdv, float clip, float vf_coef, int has_old, cudaStream_t s) {
  if (N <= 0) return 0;
  if (O <= 0 || O > kMaxObs || A <= 0 || A > kMaxAct) return static_cast<int>(cudaErrorInvalidValue);
  if (row_w < O + A + 2 + (has_old ? 1 : 0)) return static_cast<int>(cudaErrorInvalidValue);
  lin_gauss_grad_kernel<<<(N + kThreads - 1) / kThreads, kThreads, 0, s>>>(batch, row_w, params, grad, N, O, A, stdv,
                                                                           clip, vf_coef, has_old);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
