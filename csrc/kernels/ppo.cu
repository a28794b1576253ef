// PPO training-side kernels for vectorized-env policies:
//   * minibatch gather through an on-device random permutation (a Feistel
//     bijection with cycle walking), fused with global advantage normalization;
//   * the categorical clipped-surrogate loss with value loss and entropy bonus,
//     forward and backward in one pass (one thread per sample);
//   * device counters that CUDA-graph-captured loops read instead of host
//     immediates.
//
// The loss follows Schulman et al., "Proximal Policy Optimization Algorithms"
// (2017), eq. 7 and 9.  The reference's PolicyEngine::Update
// (turbol_vllm/src/policy/policy_engine.cpp:103-138) is REINFORCE with no clip;
// its Gaussian mode is kept in the Python engine, this kernel is the PPO path.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "device_common.cuh"
#include "kernels.h"

namespace {

constexpr int kBlock = 256;

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
  // integer finaliser (Murmur3 fmix32)
  x ^= x >> 16;
  x *= 0x85ebca6bu;
  x ^= x >> 13;
  x *= 0xc2b2ae35u;
  x ^= x >> 16;
  return x;
}

// Bijection on [0, 2^bits) (balanced/unbalanced Feistel, 4 rounds), walked
// until it lands in [0, M).  M <= 2^bits < 2M, so the expected number of
// walks is below 2.
__device__ __forceinline__ uint32_t feistel_perm(uint32_t x, uint32_t M, int bits, uint32_t key) {
  const int lb = bits / 2, rb = bits - lb;
  const uint32_t lmask = (1u << lb) - 1u, rmask = (1u << rb) - 1u;
  do {
    uint32_t l = x >> rb, r = x & rmask;
    // 4 rounds; the halves alternate widths, so use an even round count
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if ((k & 1) == 0) {
        const uint32_t nl = (l ^ mix32(r ^ (key + k * 0x9E3779B9u))) & lmask;
        l = nl;
      } else {
        const uint32_t nr = (r ^ mix32(l ^ (key + k * 0x9E3779B9u))) & rmask;
        r = nr;
      }
    }
    x = (l << rb) | r;
  } while (x >= M);
  return x;
}

// Gathers minibatch `mb` of epoch `epoch` (read from a device counter when
// step_ptr != null: step = epoch * n_mb + mb).
__global__ void ppo_gather_kernel(const float* __restrict__ obs, int obs_dim, const int* __restrict__ act,
                                  const float* __restrict__ logp, const float* __restrict__ adv,
                                  const float* __restrict__ ret, const float* __restrict__ val,
                                  const double* __restrict__ adv_stats, float* __restrict__ o_obs,
                                  int* __restrict__ o_act, float* __restrict__ o_logp, float* __restrict__ o_adv,
                                  float* __restrict__ o_ret, float* __restrict__ o_val, __nv_bfloat16* __restrict__ o_obs_bf16,
                                  int total, int bits,
                                  int mb_size, int n_mb, const long long* __restrict__ step_ptr,
                                  const long long* __restrict__ iter_ptr, long long step_imm,
                                  unsigned long long seed, int normalize) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= mb_size) return;
  const long long step = step_ptr ? *step_ptr : step_imm;
  const long long it = iter_ptr ? *iter_ptr : 0;
  const int epoch = static_cast<int>(step / n_mb), mb = static_cast<int>(step % n_mb);
  const uint32_t key = mix32(static_cast<uint32_t>(seed) ^ mix32(static_cast<uint32_t>(it) * 0x27d4eb2fu) ^
                             mix32(static_cast<uint32_t>(epoch) + 0x165667b1u));
  const uint32_t pos = static_cast<uint32_t>(mb) * mb_size + i;
  const uint32_t j = feistel_perm(pos, static_cast<uint32_t>(total), bits, key);
  for (int k = 0; k < obs_dim; ++k) {
    const float x = obs[static_cast<size_t>(j) * obs_dim + k];
    if (o_obs) o_obs[static_cast<size_t>(i) * obs_dim + k] = x;
    if (o_obs_bf16) o_obs_bf16[static_cast<size_t>(i) * 8 + k] = __float2bfloat16_rn(x);
  }
  if (o_obs_bf16)
    for (int k = obs_dim; k < 8; ++k) o_obs_bf16[static_cast<size_t>(i) * 8 + k] = __float2bfloat16_rn(0.f);
  o_act[i] = act[j];
  o_logp[i] = logp[j];
  float a = adv[j];
  if (normalize && adv_stats != nullptr) {
    const double n = static_cast<double>(total);
    const double mean = adv_stats[0] / n;
    double var = (adv_stats[1] - n * mean * mean) / fmax(n - 1.0, 1.0);
    var = var > 0.0 ? var : 0.0;
    a = static_cast<float>((static_cast<double>(a) - mean) / (sqrt(var) + 1e-8));
  }
  o_adv[i] = a;
  o_ret[i] = ret[j];
  if (o_val) o_val[i] = val[j];
}

// Categorical PPO loss.  Per sample:
//   logp = l[a] - lse(l), ratio = exp(logp - old), pg = -min(ratio*A, clip(ratio)*A)
//   v    = 0.5 * (V - R)^2  (or the clipped-value max form when vclip > 0)
//   H    = -sum p log p
//   loss = mean(pg) + vf_coef * mean(v) - ent_coef * mean(H)
// Writes d loss / d logits and d loss / d V (already divided by B) and adds
// [pg, v, H, approx_kl, clipfrac] sums into stats[0..4].
template <int A>
__global__ void ppo_loss_kernel(const float* __restrict__ logits, const float* __restrict__ value,
                                const int* __restrict__ act, const float* __restrict__ old_logp,
                                const float* __restrict__ adv, const float* __restrict__ ret,
                                const float* __restrict__ old_val, float* __restrict__ dlogits,
                                float* __restrict__ dvalue, float* __restrict__ stats, int B, float clip,
                                float vclip, float vf_coef, float ent_coef) {
  __shared__ float red[kBlock / 32];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  float s_pg = 0.f, s_v = 0.f, s_h = 0.f, s_kl = 0.f, s_cf = 0.f;
  if (i < B) {
    float l[A], p[A];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < A; ++k) {
      l[k] = logits[static_cast<size_t>(i) * A + k];
      mx = fmaxf(mx, l[k]);
    }
    float se = 0.f;
#pragma unroll
    for (int k = 0; k < A; ++k) {
      p[k] = __expf(l[k] - mx);
      se += p[k];
    }
    const float inv = 1.f / se, lse = mx + __logf(se);
    float H = 0.f;
#pragma unroll
    for (int k = 0; k < A; ++k) {
      p[k] *= inv;
      H -= p[k] * (l[k] - lse);
    }
    const int a = act[i];
    const float lp = l[a] - lse;
    const float lr = lp - old_logp[i];
    const float ratio = __expf(lr);
    const float Ad = adv[i];
    const float un = ratio * Ad;
    const float rc = fminf(fmaxf(ratio, 1.f - clip), 1.f + clip);
    const float cl = rc * Ad;
    const bool use_unclipped = un <= cl || (ratio > 1.f - clip && ratio < 1.f + clip);
    const float pg = -fminf(un, cl);
    const float dlp = use_unclipped ? -Ad * ratio : 0.f;  // d pg / d logp

    const float V = value[i], R = ret[i];
    float vl, dv;
    if (vclip > 0.f && old_val != nullptr) {
      const float ov = old_val[i];
      const float vc = ov + fminf(fmaxf(V - ov, -vclip), vclip);
      const float e1 = (V - R) * (V - R), e2 = (vc - R) * (vc - R);
      if (e1 >= e2) {
        vl = 0.5f * e1;
        dv = V - R;
      } else {
        vl = 0.5f * e2;
        dv = (fabsf(V - ov) < vclip) ? (vc - R) : 0.f;
      }
    } else {
      vl = 0.5f * (V - R) * (V - R);
      dv = V - R;
    }
    const float scale = 1.f / static_cast<float>(B);
#pragma unroll
    for (int k = 0; k < A; ++k) {
      const float logpk = l[k] - lse;
      // d(logp_a)/d l_k = [k==a] - p_k ;  dH/dl_k = -p_k (log p_k + H)
      const float g = dlp * ((k == a ? 1.f : 0.f) - p[k]) + ent_coef * p[k] * (logpk + H);
      dlogits[static_cast<size_t>(i) * A + k] = g * scale;
    }
    dvalue[i] = vf_coef * dv * scale;
    s_pg = pg;
    s_v = vl;
    s_h = H;
    s_kl = (ratio - 1.f) - lr;  // k3 estimator of KL(old || new)
    s_cf = fabsf(ratio - 1.f) > clip ? 1.f : 0.f;
  }
  if (stats) {
    s_pg = tb::block_sum(s_pg, red);
    s_v = tb::block_sum(s_v, red);
    s_h = tb::block_sum(s_h, red);
    s_kl = tb::block_sum(s_kl, red);
    s_cf = tb::block_sum(s_cf, red);
    if (threadIdx.x == 0) {
      atomicAdd(&stats[0], s_pg);
      atomicAdd(&stats[1], s_v);
      atomicAdd(&stats[2], s_h);
      atomicAdd(&stats[3], s_kl);
      atomicAdd(&stats[4], s_cf);
      atomicAdd(&stats[5], static_cast<float>(min(B - static_cast<int>(blockIdx.x) * kBlock, kBlock)));
    }
  }
}

// Same loss, on the tensor-core MLP's padded layout: logits [B, ldl] and values
// [B, ldv] (column 0) in fp32; writes bf16 gradients d logits and d value, 8
// columns each with row stride ldd (padding columns zero), already divided by B.
template <int A>
__global__ void ppo_loss_padded_kernel(const float* __restrict__ logits, int ldl, const float* __restrict__ value,
                                       int ldv, const int* __restrict__ act, const float* __restrict__ old_logp,
                                       const float* __restrict__ adv, const float* __restrict__ ret,
                                       __nv_bfloat16* __restrict__ dlog, __nv_bfloat16* __restrict__ dval, int ldd,
                                       float* __restrict__ stats, int B, float clip, float vf_coef, float ent_coef,
                                       float* __restrict__ db_log, float* __restrict__ db_val) {
  __shared__ float red[kBlock / 32];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  float s_pg = 0.f, s_v = 0.f, s_h = 0.f, s_kl = 0.f, s_cf = 0.f;
  float gsum[A + 1];  // column sums of the bf16 gradients (output-bias gradients)
#pragma unroll
  for (int k = 0; k <= A; ++k) gsum[k] = 0.f;
  if (i < B) {
    float l[A], p[A];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < A; ++k) {
      l[k] = logits[static_cast<size_t>(i) * ldl + k];
      mx = fmaxf(mx, l[k]);
    }
    float se = 0.f;
#pragma unroll
    for (int k = 0; k < A; ++k) {
      p[k] = __expf(l[k] - mx);
      se += p[k];
    }
    const float inv = 1.f / se, lse = mx + __logf(se);
    float H = 0.f;
#pragma unroll
    for (int k = 0; k < A; ++k) {
      p[k] *= inv;
      H -= p[k] * (l[k] - lse);
    }
    const int a = act[i];
    const float lp = l[a] - lse;
    const float lr = lp - old_logp[i];
    const float ratio = __expf(lr);
    const float Ad = adv[i];
    const float un = ratio * Ad;
    const float cl = fminf(fmaxf(ratio, 1.f - clip), 1.f + clip) * Ad;
    const bool use_unclipped = un <= cl || (ratio > 1.f - clip && ratio < 1.f + clip);
    const float dlp = use_unclipped ? -Ad * ratio : 0.f;
    const float V = value[static_cast<size_t>(i) * ldv], R = ret[i];
    const float scale = 1.f / static_cast<float>(B);
    __nv_bfloat16 g8[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float g = 0.f;
      if (k < A) g = (dlp * ((k == a ? 1.f : 0.f) - p[k]) + ent_coef * p[k] * ((l[k] - lse) + H)) * scale;
      g8[k] = __float2bfloat16_rn(g);
      if (k < A) gsum[k] = __bfloat162float(g8[k]);
    }
    *reinterpret_cast<uint4*>(dlog + static_cast<size_t>(i) * ldd) = *reinterpret_cast<uint4*>(g8);
    __nv_bfloat16 v8[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v8[k] = __float2bfloat16_rn(k == 0 ? vf_coef * (V - R) * scale : 0.f);
    gsum[A] = __bfloat162float(v8[0]);
    *reinterpret_cast<uint4*>(dval + static_cast<size_t>(i) * ldd) = *reinterpret_cast<uint4*>(v8);
    s_pg = -fminf(un, cl);
    s_v = 0.5f * (V - R) * (V - R);
    s_h = H;
    s_kl = (ratio - 1.f) - lr;
    s_cf = fabsf(ratio - 1.f) > clip ? 1.f : 0.f;
  }
  if (stats) {
    s_pg = tb::block_sum(s_pg, red);
    s_v = tb::block_sum(s_v, red);
    s_h = tb::block_sum(s_h, red);
    s_kl = tb::block_sum(s_kl, red);
    s_cf = tb::block_sum(s_cf, red);
    if (threadIdx.x == 0) {
      atomicAdd(&stats[0], s_pg);
      atomicAdd(&stats[1], s_v);
      atomicAdd(&stats[2], s_h);
      atomicAdd(&stats[3], s_kl);
      atomicAdd(&stats[4], s_cf);
      atomicAdd(&stats[5], static_cast<float>(min(B - static_cast<int>(blockIdx.x) * kBlock, kBlock)));
    }
  }
  if (db_log != nullptr) {
#pragma unroll
    for (int k = 0; k <= A; ++k) {
      const float t = tb::block_sum(gsum[k], red);
      if (threadIdx.x == 0) atomicAdd(k < A ? &db_log[k] : db_val, t);
    }
  }
}

// out[c] = sum over rows of x[r, c] (bf16 in, fp32 out).  Each block sums a
// chunk of rows for a span of columns and adds its partial atomically; `out`
// is zeroed by the launcher.
__global__ void colsum_bf16_kernel(const __nv_bfloat16* __restrict__ x, long long ld, int rows, int cols,
                                   int rows_per_block, float* __restrict__ out) {
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  const int r0 = blockIdx.x * rows_per_block, r1 = min(rows, r0 + rows_per_block);
  float s = 0.f;
  for (int r = r0; r < r1; ++r) s += __bfloat162float(x[static_cast<long long>(r) * ld + c]);
  atomicAdd(&out[c], s);
}

__global__ void counter_add_kernel(long long* c, long long v) { *c += v; }

// ---------------------------------------------------------------- small-K dense layer
// y[M, N] = act(x[M, 8] . W[N, 8]^T + b) for the first layer of an MLP whose
// input has at most 8 features (bf16 in, fp32 accumulation, bf16 out).  A
// tensor-core tile would be 87% zero padding in K and bound by its epilogue.
// Here a thread owns 4 output columns: their 32 weights and 4 biases live in
// registers (few registers: many resident warps to hide the load latency), and
// it walks a chunk of rows, 4 rows in flight; the lanes of a warp share each
// row's 16-byte input (one broadcast load) and write 32 neighbouring 8-byte
// column groups (256 contiguous bytes).
constexpr int kDenseCols = 4;  // output columns per thread (W slice in 32 registers)
__global__ void __launch_bounds__(256) dense_k8_fwd_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                           const __nv_bfloat16* __restrict__ W,
                                                           const float* __restrict__ bias,
                                                           __nv_bfloat16* __restrict__ y, long long ldy, int M, int N,
                                                           int act, int rows_per_block) {
  constexpr int C = kDenseCols;
  const int groups = N / C;
  const int g = threadIdx.x % groups;           // column group of this thread
  const int rsub = threadIdx.x / groups;        // row offset within a block step
  const int rstep = blockDim.x / groups;
  if (rsub >= rstep) return;
  float w[C][8], b[C];
#pragma unroll
  for (int j = 0; j < C; ++j) {
    const uint4 u = *reinterpret_cast<const uint4*>(W + (g * C + j) * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __bfloat1622float2(h[k]);
      w[j][2 * k] = f.x;
      w[j][2 * k + 1] = f.y;
    }
    b[j] = bias ? bias[g * C + j] : 0.f;
  }
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(M, r0 + rows_per_block);
  constexpr int kR = 4;  // rows in flight per thread
  for (int rb = r0 + rsub; rb < r1; rb += kR * rstep) {
    uint4 xu[kR];
#pragma unroll
    for (int q = 0; q < kR; ++q) {
      const int r = rb + q * rstep;
      xu[q] = r < r1 ? *reinterpret_cast<const uint4*>(x + r * ldx) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int q = 0; q < kR; ++q) {
      const int r = rb + q * rstep;
      const __nv_bfloat162* xh = reinterpret_cast<const __nv_bfloat162*>(&xu[q]);
      float xv[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(xh[k]);
        xv[2 * k] = f.x;
        xv[2 * k + 1] = f.y;
      }
      float o[C];
#pragma unroll
      for (int j = 0; j < C; ++j) {
        float acc = b[j];
#pragma unroll
        for (int k = 0; k < 8; ++k) acc = fmaf(xv[k], w[j][k], acc);
        if (act == 1) {
          float t;
          asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(acc));
          acc = t;
        }
        o[j] = acc;
      }
      uint2 ou;
      __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&ou);
      oh[0] = __floats2bfloat162_rn(o[0], o[1]);
      oh[1] = __floats2bfloat162_rn(o[2], o[3]);
      if (r < r1) *reinterpret_cast<uint2*>(y + r * ldy + g * C) = ou;
    }
  }
}

// dW[N, 8] += dz[M, N]^T . x[M, 8]: thread = one output column j over a chunk
// of rows (coalesced dz reads, x rows broadcast), 8 partial sums reduced with
// one atomic each per thread.
constexpr int kWgRows = 256;
__global__ void __launch_bounds__(256) dense_k8_wgrad_kernel(const __nv_bfloat16* __restrict__ dz, long long ldz,
                                                             const __nv_bfloat16* __restrict__ x, long long ldx,
                                                             float* __restrict__ dW, int M, int N) {
  __shared__ float sx[kWgRows][8];
  const int r0 = blockIdx.y * kWgRows;
  const int nr = min(kWgRows, M - r0);
  for (int i = threadIdx.x; i < nr * 8; i += blockDim.x) {
    const int r = i / 8, k = i % 8;
    sx[r][k] = __bfloat162float(x[(r0 + r) * ldx + k]);
  }
  __syncthreads();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= N) return;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const __nv_bfloat16* col = dz + static_cast<long long>(r0) * ldz + j;
  for (int r = 0; r < nr; ++r) {
    const float d = __bfloat162float(col[static_cast<long long>(r) * ldz]);
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = fmaf(d, sx[r][k], acc[k]);
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) atomicAdd(dW + j * 8 + k, acc[k]);
}

// Weight gradient of a layer with 8 features on one side, out = A^T X summed
// over M rows, with A bf16 [M, N] (N <= 512, N % 32 == 0) and X bf16 [M, 8]
// per column block: columns [b*xblock, (b+1)*xblock) of A pair with X's
// columns [8b, 8b+8) (block-diagonal heads).  Two passes, no atomics: in
// skinny8_partial_kernel a warp covers 32 columns (4 threads of 8 columns) x 8
// row-lanes, streams a slice of the rows with 16-byte loads (4 rows in flight
// per thread, 64 products per thread), folds its row-lanes with shuffles and
// writes one partial [N * 8] per CTA to `part`; skinny8_reduce_kernel adds
// the CTAs' partials and writes out[(j, k)] at j*os_j + k*os_k + b*os_blk.
constexpr int kSkUnroll = 4;
constexpr int kSkThreads = 512;  // mlp_head_dz_kernel
__global__ void __launch_bounds__(512) skinny8_partial_kernel(
    const __nv_bfloat16* __restrict__ A, long long lda, const __nv_bfloat16* __restrict__ X, long long ldx,
    int xblock, float* __restrict__ part, int M, int N, int rows_per_block) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tc = lane & 3, rl = lane >> 2;  // column thread within the warp's 32 columns, row-lane 0..7
  const int j0 = warp * 32 + tc * 8, blk = j0 / xblock;
  const int r0 = blockIdx.x * rows_per_block, r1 = min(M, r0 + rows_per_block);
  float acc[8][8];
#pragma unroll
  for (int c = 0; c < 8; ++c)
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[c][k] = 0.f;
  for (int rb = r0 + rl; rb < r1; rb += 8 * kSkUnroll) {
    uint4 a[kSkUnroll], x[kSkUnroll];
#pragma unroll
    for (int u = 0; u < kSkUnroll; ++u) {
      const int r = rb + 8 * u;
      const bool ok = r < r1;
      a[u] = ok ? *reinterpret_cast<const uint4*>(A + static_cast<long long>(r) * lda + j0) : make_uint4(0u, 0u, 0u, 0u);
      x[u] = ok ? *reinterpret_cast<const uint4*>(X + static_cast<long long>(r) * ldx + 8 * blk)
                : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < kSkUnroll; ++u) {
      const __nv_bfloat162* ah = reinterpret_cast<const __nv_bfloat162*>(&a[u]);
      const __nv_bfloat162* xh = reinterpret_cast<const __nv_bfloat162*>(&x[u]);
      float av[8], xv[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 fa = __bfloat1622float2(ah[q]), fx = __bfloat1622float2(xh[q]);
        av[2 * q] = fa.x;
        av[2 * q + 1] = fa.y;
        xv[2 * q] = fx.x;
        xv[2 * q + 1] = fx.y;
      }
#pragma unroll
      for (int c = 0; c < 8; ++c)
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[c][k] = fmaf(av[c], xv[k], acc[c][k]);
    }
  }
  // fold the 8 row-lanes (lane bits 2..4); every lane of a column thread ends with the sums
#pragma unroll
  for (int c = 0; c < 8; ++c)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float v = acc[c][k];
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      acc[c][k] = v;
    }
  // row-lane rl stores column j0 + rl's 8 values
  float* dst = part + static_cast<long long>(blockIdx.x) * N * 8 + (j0 + rl) * 8;
  float outv[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float v = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) v = (c == rl) ? acc[c][k] : v;
    outv[k] = v;
  }
  reinterpret_cast<float4*>(dst)[0] = make_float4(outv[0], outv[1], outv[2], outv[3]);
  reinterpret_cast<float4*>(dst)[1] = make_float4(outv[4], outv[5], outv[6], outv[7]);
}

// Sum of `parts` partials part[b * n + i] for n outputs: 32 outputs per CTA,
// 32 thread groups each summing every 32nd partial, then a shared-memory fold.
// Element i goes to out[map(i)] (store, or add with accumulate).
template <typename Map>
__device__ __forceinline__ void reduce_parts(const float* __restrict__ part, int parts, int n, int accumulate,
                                             Map map) {
  __shared__ float sm[32][33];
  const int oi = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int i = blockIdx.x * 32 + oi;
  float s = 0.f;
  if (i < n)
    for (int b = g; b < parts; b += 32) s += part[static_cast<long long>(b) * n + i];
  sm[g][oi] = s;
  __syncthreads();
  if (g == 0 && i < n) {
    float t = 0.f;
    for (int q = 0; q < 32; ++q) t += sm[q][oi];
    float* o = map(i);
    *o = accumulate ? *o + t : t;
  }
}

__global__ void __launch_bounds__(1024) skinny8_reduce_kernel(const float* __restrict__ part, int parts, int N,
                                                              int xblock, float* __restrict__ out, long long os_j,
                                                              long long os_k, long long os_blk, int accumulate) {
  reduce_parts(part, parts, N * 8, accumulate, [&](int i) {
    const int j = i / 8, k = i % 8;
    return out + (j / xblock) * os_blk + j * os_j + k * os_k;
  });
}

// Backward through an output layer with 8 outputs per head into a tanh hidden
// layer: dZ[r, j] = (sum_k dOut[r, 8b + k] W[8b + k, j]) * (1 - H[r, j]^2) for
// the head b = j / xblock owning column j, and db[j] += sum_r dZ[r, j].
// dOut bf16 [M, 8 * heads], H bf16 [M, N], W bf16 [8 * heads, N] (row
// stride ldw), dZ bf16 [M, N]; db fp32 [N] (accumulated atomically: zeroed by
// the caller).  Each thread keeps its 8 columns' 8 x 8 weights in registers and
// streams rows with 16-byte loads, 4 rows in flight: a bandwidth-bound pass
// instead of a K = 16 tensor-core GEMM whose time goes to its epilogue.
__global__ void __launch_bounds__(kSkThreads) mlp_head_dz_kernel(
    const __nv_bfloat16* __restrict__ dout, long long ldd, const __nv_bfloat16* __restrict__ H, long long ldh,
    const __nv_bfloat16* __restrict__ W, long long ldw, int xblock, __nv_bfloat16* __restrict__ dz, long long ldz,
    float* __restrict__ part, int M, int N, int rows_per_block) {
  __shared__ float red[512];
  const int tpr = N / 8;
  const int lanes = kSkThreads / tpr;
  const int t = threadIdx.x % tpr, rl = threadIdx.x / tpr;
  for (int i = threadIdx.x; i < N; i += blockDim.x) red[i] = 0.f;
  __syncthreads();
  const int j0 = 8 * t, blk = j0 / xblock;
  if (rl < lanes) {
  float w[8][8];  // w[k][c] = W[8 blk + k, j0 + c]
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint4 u = *reinterpret_cast<const uint4*>(W + static_cast<long long>(8 * blk + k) * ldw + j0);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __bfloat1622float2(h[q]);
      w[k][2 * q] = f.x;
      w[k][2 * q + 1] = f.y;
    }
  }
  float dbs[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) dbs[c] = 0.f;
  const int r0 = blockIdx.x * rows_per_block, r1 = min(M, r0 + rows_per_block);
  for (int rb = r0 + rl; rb < r1; rb += lanes * kSkUnroll) {
    uint4 hu[kSkUnroll], du[kSkUnroll];
#pragma unroll
    for (int u = 0; u < kSkUnroll; ++u) {
      const int r = rb + u * lanes;
      const bool ok = r < r1;
      hu[u] = ok ? *reinterpret_cast<const uint4*>(H + static_cast<long long>(r) * ldh + j0) : make_uint4(0u, 0u, 0u, 0u);
      du[u] = ok ? *reinterpret_cast<const uint4*>(dout + static_cast<long long>(r) * ldd + 8 * blk)
                 : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < kSkUnroll; ++u) {
      const int r = rb + u * lanes;
      const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&hu[u]);
      const __nv_bfloat162* dh = reinterpret_cast<const __nv_bfloat162*>(&du[u]);
      float hv[8], dv[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 fh = __bfloat1622float2(hh[q]), fd = __bfloat1622float2(dh[q]);
        hv[2 * q] = fh.x;
        hv[2 * q + 1] = fh.y;
        dv[2 * q] = fd.x;
        dv[2 * q + 1] = fd.y;
      }
      float o[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) acc = fmaf(dv[k], w[k][c], acc);
        o[c] = acc * (1.f - hv[c] * hv[c]);
      }
      if (r < r1) {
        uint4 pk;
        __nv_bfloat162* ph = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
        for (int q = 0; q < 4; ++q) ph[q] = __floats2bfloat162_rn(o[2 * q], o[2 * q + 1]);
        *reinterpret_cast<uint4*>(dz + static_cast<long long>(r) * ldz + j0) = pk;
#pragma unroll
        for (int c = 0; c < 8; ++c) dbs[c] += o[c];
      }
    }
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) atomicAdd(&red[j0 + c], dbs[c]);  // shared memory
  }
  __syncthreads();
  for (int i = threadIdx.x; i < N; i += blockDim.x) part[static_cast<long long>(blockIdx.x) * N + i] = red[i];
}

// db[j] (+)= sum over the CTAs' partials [parts, N].
__global__ void __launch_bounds__(1024) colsum_parts_kernel(const float* __restrict__ part, int parts, int N,
                                                            float* __restrict__ db, int accumulate) {
  reduce_parts(part, parts, N, accumulate, [&](int j) { return db + j; });
}

// Output layer with 8 outputs per head: out[r, 8b + k] = b[8b + k] + sum over
// the head's columns j of H[r, j] W[8b + k, j] (fp32 out).  A sub-warp of
// xblock / 8 lanes covers one row of one head (8 columns per lane, the head's
// 8 x 8 weights per lane in registers), sums across its lanes with shuffles,
// and every warp keeps one head; rows stream with 16-byte loads, 4 in flight.
__global__ void __launch_bounds__(256) mlp_head_fwd_kernel(const __nv_bfloat16* __restrict__ H, long long ldh,
                                                           const __nv_bfloat16* __restrict__ W, long long ldw,
                                                           const float* __restrict__ bias, float* __restrict__ out,
                                                           long long ldo, int xblock, int heads, int M) {
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (gridDim.x * blockDim.x) >> 5;
  const int L = xblock / 8, G = 32 / L;  // lanes per row, rows per warp step
  const int head = gw % heads;
  const int c0 = head * xblock + (lane % L) * 8;
  float w[8][8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint4 u = *reinterpret_cast<const uint4*>(W + static_cast<long long>(8 * head + k) * ldw + c0);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __bfloat1622float2(h[q]);
      w[k][2 * q] = f.x;
      w[k][2 * q + 1] = f.y;
    }
  }
  const int kk = lane % L;  // the output this lane writes (lanes 0..7 of a row group)
  const float bk = (kk < 8 && bias) ? bias[8 * head + kk] : 0.f;
  const int step = (nw / heads) * G;
  // the loop bound is uniform across the warp (the shuffles below need every lane)
  for (int wb = (gw / heads) * G; wb < M; wb += 4 * step) {
    const int rb = wb + lane / L;
    uint4 hu[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int r = rb + u * step;
      hu[u] = r < M ? *reinterpret_cast<const uint4*>(H + static_cast<long long>(r) * ldh + c0)
                    : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int r = rb + u * step;
      const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&hu[u]);
      float hv[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(hh[q]);
        hv[2 * q] = f.x;
        hv[2 * q + 1] = f.y;
      }
      float acc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float a = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) a = fmaf(hv[c], w[k][c], a);
        acc[k] = a;
      }
      for (int off = L / 2; off >= 1; off >>= 1)
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], off);
      float v = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) v = (k == kk) ? acc[k] : v;
      if (r < M && kk < 8) out[static_cast<long long>(r) * ldo + 8 * head + kk] = v + bk;
    }
  }
}

}  // namespace

extern "C" {

int tb_ppo_gather(const float* obs, int obs_dim, const int* act, const float* logp, const float* adv, const float* ret,
                  const float* val, const double* adv_stats, float* o_obs, int* o_act, float* o_logp, float* o_adv,
                  float* o_ret, float* o_val, void* o_obs_bf16, int total, int mb_size, int n_mb,
                  const long long* step_ptr, const long long* iter_ptr, long long step_imm, unsigned long long seed,
                  int normalize, cudaStream_t s) {
  if (mb_size <= 0) return 0;
  if (o_obs_bf16 != nullptr && obs_dim > 8) return static_cast<int>(cudaErrorInvalidValue);
  if (static_cast<long long>(mb_size) * n_mb > total) return static_cast<int>(cudaErrorInvalidValue);
  int bits = 1;
  while ((1LL << bits) < total) ++bits;
  ppo_gather_kernel<<<(mb_size + kBlock - 1) / kBlock, kBlock, 0, s>>>(
      obs, obs_dim, act, logp, adv, ret, val, adv_stats, o_obs, o_act, o_logp, o_adv, o_ret, o_val,
      static_cast<__nv_bfloat16*>(o_obs_bf16), total, bits,
      mb_size, n_mb, step_ptr, iter_ptr, step_imm, seed, normalize);
  return static_cast<int>(cudaGetLastError());
}

int tb_ppo_loss(const float* logits, int A, const float* value, const int* act, const float* old_logp,
                const float* adv, const float* ret, const float* old_val, float* dlogits, float* dvalue, float* stats,
                int B, float clip, float vclip, float vf_coef, float ent_coef, cudaStream_t s) {
  if (B <= 0) return 0;
  const int g = (B + kBlock - 1) / kBlock;
#define TB_PPO_CASE(K)                                                                                          \
  case K:                                                                                                       \
    ppo_loss_kernel<K><<<g, kBlock, 0, s>>>(logits, value, act, old_logp, adv, ret, old_val, dlogits, dvalue,   \
                                            stats, B, clip, vclip, vf_coef, ent_coef);                          \
    break;
  switch (A) {
    TB_PPO_CASE(2)
    TB_PPO_CASE(3)
    TB_PPO_CASE(4)
    TB_PPO_CASE(6)
    TB_PPO_CASE(8)
    TB_PPO_CASE(16)
    default:
      return static_cast<int>(cudaErrorInvalidValue);
  }
#undef TB_PPO_CASE
  return static_cast<int>(cudaGetLastError());
}

int tb_ppo_loss_padded(const float* logits, int ldl, int A, const float* value, int ldv, const int* act,
                       const float* old_logp, const float* adv, const float* ret, void* dlog_bf16, void* dval_bf16,
                       int ldd, float* stats, int B, float clip, float vf_coef, float ent_coef, float* db_log,
                       float* db_val, cudaStream_t s) {
  if (B <= 0) return 0;
  if (ldd % 8 || (reinterpret_cast<uintptr_t>(dlog_bf16) & 15) || (reinterpret_cast<uintptr_t>(dval_bf16) & 15))
    return static_cast<int>(cudaErrorInvalidValue);
  if ((db_log == nullptr) != (db_val == nullptr)) return static_cast<int>(cudaErrorInvalidValue);
  if (db_log) {
    cudaMemsetAsync(db_log, 0, sizeof(float) * A, s);
    cudaMemsetAsync(db_val, 0, sizeof(float), s);
  }
  const int g = (B + kBlock - 1) / kBlock;
  auto* dl = static_cast<__nv_bfloat16*>(dlog_bf16);
  auto* dv = static_cast<__nv_bfloat16*>(dval_bf16);
#define TB_PPO_CASE(K)                                                                                           \
  case K:                                                                                                        \
    ppo_loss_padded_kernel<K><<<g, kBlock, 0, s>>>(logits, ldl, value, ldv, act, old_logp, adv, ret, dl, dv, ldd, \
                                                   stats, B, clip, vf_coef, ent_coef, db_log, db_val);          \
    break;
  switch (A) {
    TB_PPO_CASE(2)
    TB_PPO_CASE(3)
    TB_PPO_CASE(4)
    TB_PPO_CASE(6)
    TB_PPO_CASE(8)
    default:
      return static_cast<int>(cudaErrorInvalidValue);
  }
#undef TB_PPO_CASE
  return static_cast<int>(cudaGetLastError());
}

int tb_colsum_bf16(const void* x, long long ld, int rows, int cols, float* out, int accumulate, cudaStream_t s) {
  if (rows <= 0 || cols <= 0) return 0;
  if (!accumulate) cudaMemsetAsync(out, 0, sizeof(float) * cols, s);
  const int rpb = 256;
  dim3 grid((rows + rpb - 1) / rpb, (cols + kBlock - 1) / kBlock);
  colsum_bf16_kernel<<<grid, kBlock, 0, s>>>(static_cast<const __nv_bfloat16*>(x), ld, rows, cols, rpb, out);
  return static_cast<int>(cudaGetLastError());
}

int tb_counter_add(long long* counter, long long v, cudaStream_t s) {
  counter_add_kernel<<<1, 1, 0, s>>>(counter, v);
  return static_cast<int>(cudaGetLastError());
}

int tb_dense_k8_fwd(const void* x, long long ldx, const void* W, const float* bias, void* y, long long ldy, int M,
                    int N, int act, cudaStream_t s) {
  return tb_dense_k8_fwd_rows(x, ldx, W, bias, y, ldy, M, N, act, 0, s);
}

int tb_dense_k8_fwd_rows(const void* x, long long ldx, const void* W, const float* bias, void* y, long long ldy,
                         int M, int N, int act, int rows_hint, cudaStream_t s) {
  if (M <= 0) return 0;
  if (N % 8 || N > 1024 || ldx % 8 || ldy % 8 || (reinterpret_cast<uintptr_t>(W) & 15) || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(y) & 15))
    return static_cast<int>(cudaErrorInvalidValue);
  // one thread per column group (N / 4 <= 256 threads), as many row lanes as fit in 256 threads
  const int groups = N / kDenseCols;
  if (groups > 256) return static_cast<int>(cudaErrorInvalidValue);
  const int rstep = 256 / groups;
  int rows = 32;
  if (rows_hint > 0) {
    rows = rows_hint < rstep ? rstep : rows_hint;  // rows per CTA (each CTA loads its weight slice once)
  } else {
    while (rows > rstep && (static_cast<long long>(M) + rows - 1) / rows < 4 * 148) rows /= 2;
  }
  const unsigned grid = static_cast<unsigned>((M + rows - 1) / rows);
  dense_k8_fwd_kernel<<<grid, rstep * groups, 0, s>>>(static_cast<const __nv_bfloat16*>(x), ldx,
                                                      static_cast<const __nv_bfloat16*>(W), bias,
                                                      static_cast<__nv_bfloat16*>(y), ldy, M, N, act, rows);
  return static_cast<int>(cudaGetLastError());
}

static int sk_grid(int M, int* per) {  // one CTA per SM, each a contiguous slice of rows
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  *per = (M + sms - 1) / sms;
  return (M + *per - 1) / *per;
}

size_t tb_skinny8_scratch_floats(int N) {
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return static_cast<size_t>(sms) * 8 * static_cast<size_t>(N > 0 ? N : 0);
}

int tb_skinny8_wgrad(const void* A, long long lda, const void* X, long long ldx, int xblock, float* out,
                     long long os_j, long long os_k, long long os_blk, int M, int N, int accumulate, float* scratch,
                     size_t scratch_floats, cudaStream_t s) {
  if (N <= 0 || N > 512 || N % 32 || xblock <= 0 || xblock % 8 || N % xblock || lda % 8 || ldx % 8 ||
      (reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(X) & 15) || M < 0)
    return static_cast<int>(cudaErrorInvalidValue);
  int per = 1;
  const int grid = M > 0 ? sk_grid(M, &per) : 0;
  if (static_cast<size_t>(grid) * N * 8 > scratch_floats) return static_cast<int>(cudaErrorInvalidValue);
  if (grid > 0)
    skinny8_partial_kernel<<<grid, N, 0, s>>>(static_cast<const __nv_bfloat16*>(A), lda,
                                               static_cast<const __nv_bfloat16*>(X), ldx, xblock, scratch, M, N, per);
  skinny8_reduce_kernel<<<(N * 8 + 31) / 32, 1024, 0, s>>>(scratch, grid, N, xblock, out, os_j, os_k, os_blk,
                                                            accumulate);
  return static_cast<int>(cudaGetLastError());
}

int tb_mlp_head_dz(const void* dout, long long ldd, const void* H, long long ldh, const void* W, long long ldw,
                   int xblock, void* dz, long long ldz, float* db, int M, int N, int accumulate, float* scratch,
                   size_t scratch_floats, cudaStream_t s) {
  if (N <= 0 || N > 512 || N % 8 || xblock <= 0 || xblock % 8 || N % xblock || ldd % 8 || ldh % 8 || ldw % 8 ||
      ldz % 8 || (reinterpret_cast<uintptr_t>(dout) & 15) || (reinterpret_cast<uintptr_t>(H) & 15) ||
      (reinterpret_cast<uintptr_t>(W) & 15) || (reinterpret_cast<uintptr_t>(dz) & 15) || M < 0)
    return static_cast<int>(cudaErrorInvalidValue);
  int per = 1;
  const int grid = M > 0 ? sk_grid(M, &per) : 0;
  if (static_cast<size_t>(grid) * N > scratch_floats) return static_cast<int>(cudaErrorInvalidValue);
  if (grid > 0)
    mlp_head_dz_kernel<<<grid, kSkThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(dout), ldd,
                                                    static_cast<const __nv_bfloat16*>(H), ldh,
                                                    static_cast<const __nv_bfloat16*>(W), ldw, xblock,
                                                    static_cast<__nv_bfloat16*>(dz), ldz, scratch, M, N, per);
  colsum_parts_kernel<<<(N + 31) / 32, 1024, 0, s>>>(scratch, grid, N, db, accumulate);
  return static_cast<int>(cudaGetLastError());
}

int tb_mlp_head_fwd(const void* H, long long ldh, const void* W, long long ldw, const float* bias, float* out,
                    long long ldo, int xblock, int heads, int M, cudaStream_t s) {
  if (M <= 0) return 0;
  if (xblock < 64 || xblock > 256 || (xblock & (xblock - 1)) || heads < 1 || ldh % 8 || ldw % 8 ||
      (reinterpret_cast<uintptr_t>(H) & 15) || (reinterpret_cast<uintptr_t>(W) & 15) || ldo < 8 * heads)
    return static_cast<int>(cudaErrorInvalidValue);
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // 8 warps per CTA, an even number of warps per head
  const int grid = sms * 4;
  mlp_head_fwd_kernel<<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(H), ldh,
                                            static_cast<const __nv_bfloat16*>(W), ldw, bias, out, ldo, xblock, heads,
                                            M);
  return static_cast<int>(cudaGetLastError());
}

int tb_dense_k8_wgrad(const void* dz, long long ldz, const void* x, long long ldx, float* dW, int M, int N,
                      int accumulate, cudaStream_t s) {
  if (!accumulate) cudaMemsetAsync(dW, 0, sizeof(float) * 8 * static_cast<size_t>(N), s);
  if (M <= 0) return 0;
  dim3 grid((N + 255) / 256, (M + kWgRows - 1) / kWgRows);
  dense_k8_wgrad_kernel<<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(dz), ldz,
                                             static_cast<const __nv_bfloat16*>(x), ldx, dW, M, N);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
