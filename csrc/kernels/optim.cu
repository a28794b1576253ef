// Fused optimizer and elementwise kernels.
//
//   * Adam/AdamW over one flat fp32 parameter buffer (Kingma & Ba 2015;
//     decoupled weight decay per Loshchilov & Hutter 2019), with an optional
//     bf16 shadow copy written in the same pass (the low-precision weights the
//     forward reads), an optional gradient pre-scale (1/world for a data-parallel
//     sum) and optional global-norm clipping.  The step count lives in device
//     memory so the update can sit inside a CUDA graph.
//   * Elementwise fill / add-scalar / scale / add / sub / copy for the
//     TensorUtils API (reference turbol_vllm/src/cuda/math_utils.cu:10-70),
//     vectorised as float4 with a grid-stride loop.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "device_common.cuh"
#include "kernels.h"

namespace {

constexpr int kBlock = 256;

inline unsigned grid_1d(long long n, int per_thread) {
  long long g = (n / per_thread + kBlock - 1) / kBlock;
  if (g > 148 * 8) g = 148 * 8;
  return static_cast<unsigned>(g < 1 ? 1 : g);
}

__device__ __forceinline__ float adam_one(float& p, float g, float& m, float& v, float lr, float b1, float b2,
                                          float eps, float wd, float bc1, float bc2) {
  m = b1 * m + (1.f - b1) * g;
  v = b2 * v + (1.f - b2) * g * g;
  const float mh = m / bc1, vh = v / bc2;
  p = p - lr * (mh / (sqrtf(vh) + eps) + wd * p);
  return p;
}

__global__ void adam_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                            float* __restrict__ v, __nv_bfloat16* __restrict__ pb, long long n, TbAdamParams hp,
                            const long long* __restrict__ step_ptr, const float* __restrict__ gnorm_sq) {
  const long long step = (step_ptr ? *step_ptr : hp.step) + 1;
  const float bc1 = 1.f - powf(hp.beta1, static_cast<float>(step));
  const float bc2 = 1.f - powf(hp.beta2, static_cast<float>(step));
  float gs = hp.grad_scale;
  if (gnorm_sq != nullptr && hp.max_grad_norm > 0.f) {
    const float norm = sqrtf(*gnorm_sq) * hp.grad_scale;
    if (norm > hp.max_grad_norm) gs *= hp.max_grad_norm / (norm + 1e-6f);
  }
  const long long n4 = n / 4;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4; i += stride) {
    float4 P = reinterpret_cast<float4*>(p)[i];
    const float4 G = reinterpret_cast<const float4*>(g)[i];
    float4 M = reinterpret_cast<float4*>(m)[i];
    float4 V = reinterpret_cast<float4*>(v)[i];
    adam_one(P.x, G.x * gs, M.x, V.x, hp.lr, hp.beta1, hp.beta2, hp.eps, hp.weight_decay, bc1, bc2);
    adam_one(P.y, G.y * gs, M.y, V.y, hp.lr, hp.beta1, hp.beta2, hp.eps, hp.weight_decay, bc1, bc2);
    adam_one(P.z, G.z * gs, M.z, V.z, hp.lr, hp.beta1, hp.beta2, hp.eps, hp.weight_decay, bc1, bc2);
    adam_one(P.w, G.w * gs, M.w, V.w, hp.lr, hp.beta1, hp.beta2, hp.eps, hp.weight_decay, bc1, bc2);
    reinterpret_cast<float4*>(p)[i] = P;
    reinterpret_cast<float4*>(m)[i] = M;
    reinterpret_cast<float4*>(v)[i] = V;
    if (pb) {
      __nv_bfloat162 lo = __floats2bfloat162_rn(P.x, P.y), hi = __floats2bfloat162_rn(P.z, P.w);
      reinterpret_cast<__nv_bfloat162*>(pb)[2 * i] = lo;
      reinterpret_cast<__nv_bfloat162*>(pb)[2 * i + 1] = hi;
    }
  }
  for (long long i = n4 * 4 + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    float P = p[i], M = m[i], V = v[i];
    adam_one(P, g[i] * gs, M, V, hp.lr, hp.beta1, hp.beta2, hp.eps, hp.weight_decay, bc1, bc2);
    p[i] = P;
    m[i] = M;
    v[i] = V;
    if (pb) pb[i] = __float2bfloat16_rn(P);
  }
}

__global__ void sumsq_kernel(const float* __restrict__ x, long long n, float* __restrict__ out) {
  __shared__ float red[kBlock / 32];
  float s = 0.f;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    s += x[i] * x[i];
  s = tb::block_sum(s, red);
  if (threadIdx.x == 0) atomicAdd(out, s);
}

// op: 0 fill(a), 1 add_scalar(x + a), 2 scale(x * a), 3 add(x + y), 4 sub(x - y), 5 copy(x)
__global__ void ew_kernel(float* __restrict__ out, const float* __restrict__ x, const float* __restrict__ y,
                          long long n, float a, int op) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const bool vec = ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(x) |
                     reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  const long long n4 = vec ? n / 4 : 0;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4; i += stride) {
    float4 r;
    const float4 X = (op >= 1) ? reinterpret_cast<const float4*>(x)[i] : make_float4(0, 0, 0, 0);
    const float4 Y = (op == 3 || op == 4) ? reinterpret_cast<const float4*>(y)[i] : make_float4(0, 0, 0, 0);
    switch (op) {
      case 0: r = make_float4(a, a, a, a); break;
      case 1: r = make_float4(X.x + a, X.y + a, X.z + a, X.w + a); break;
      case 2: r = make_float4(X.x * a, X.y * a, X.z * a, X.w * a); break;
      case 3: r = make_float4(X.x + Y.x, X.y + Y.y, X.z + Y.z, X.w + Y.w); break;
      case 4: r = make_float4(X.x - Y.x, X.y - Y.y, X.z - Y.z, X.w - Y.w); break;
      default: r = X; break;
    }
    reinterpret_cast<float4*>(out)[i] = r;
  }
  for (long long i = n4 * 4 + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    float r;
    switch (op) {
      case 0: r = a; break;
      case 1: r = x[i] + a; break;
      case 2: r = x[i] * a; break;
      case 3: r = x[i] + y[i]; break;
      case 4: r = x[i] - y[i]; break;
      default: r = x[i]; break;
    }
    out[i] = r;
  }
}

}  // namespace

extern "C" {

int tb_adam(float* p, const float* g, float* m, float* v, void* p_bf16, long long n, TbAdamParams hp,
            const long long* step_ptr, const float* gnorm_sq, cudaStream_t s) {
  if (n <= 0) return 0;
  adam_kernel<<<grid_1d(n, 4), kBlock, 0, s>>>(p, g, m, v, static_cast<__nv_bfloat16*>(p_bf16), n, hp, step_ptr,
                                              gnorm_sq);
  return static_cast<int>(cudaGetLastError());
}

int tb_sumsq(const float* x, long long n, float* out, cudaStream_t s) {
  if (n <= 0) return 0;
  sumsq_kernel<<<grid_1d(n, 1), kBlock, 0, s>>>(x, n, out);
  return static_cast<int>(cudaGetLastError());
}

int tb_elementwise(float* out, const float* x, const float* y, long long n, float a, int op, cudaStream_t s) {
  if (n <= 0) return 0;
  ew_kernel<<<grid_1d(n, 4), kBlock, 0, s>>>(out, x, y, n, a, op);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
