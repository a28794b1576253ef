// PPO output layer, loss and output-layer backward in one pass over H2.
//
// The actor-critic's last layer has A logits (actor head) and one value
// (critic head) per row, so its forward, the clipped-surrogate loss and its
// backward are per-row work on the hidden activations H2 = [H2a | H2c]
// (bf16 [M, 2H]).  Run as separate launches they stream H2 three times (the
// output GEMM, the dW3 pass, the dZ2 pass) and round-trip the logits and the
// logit gradients through memory.  Here one warp owns a row at a time: lanes
// 0-15 hold H/16 columns of the actor half, lanes 16-31 the same of the critic
// half, with the matching output-layer weights in registers.
//   forward   logits[k] = b3a[k] + H2a . W3a[k],  value = b3c + H2c . W3c
//             (16-lane shuffle sums, then every lane has all A + 1 outputs)
//   loss      Schulman et al. 2017 eq. 7 + 9 per row (as ppo_loss_padded in
//             ppo.cu): dlog[k], dval already divided by the minibatch size M
//   backward  dZ2a[j] = (sum_k dlog[k] W3a[k, j]) (1 - H2a[j]^2),
//             dZ2c[j] = dval W3c[j] (1 - H2c[j]^2)   (bf16 out, [M, 2H])
//   sums      db2 = sum_r dZ2, dW3a[k] = sum_r dlog[k] H2a, dW3c = sum_r dval H2c,
//             db3, and the loss statistics, kept per lane in registers
// Each CTA folds its warps' sums in a fixed order into one partial row;
// ppo_head_reduce sums the CTAs' partials in a fixed order (no atomics, the
// result does not depend on scheduling) and writes the gradients into the flat
// gradient buffer and adds the statistics.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "device_common.cuh"
#include "kernels.h"

namespace {

using bf16 = __nv_bfloat16;
constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int kStats = 6;  // pg, value loss, entropy, approx kl, clip fraction, rows

// Partial row layout (floats): db2 [2H] | dW3a [A][H] | dW3c [H] | db3a [A] | db3c | stats [6]
__host__ __device__ __forceinline__ int part_len(int H, int A) { return 2 * H + A * H + H + A + 1 + kStats; }

template <int CPL>
__device__ __forceinline__ void load_row(const bf16* p, float* h) {
#pragma unroll
  for (int q = 0; q < CPL / 8; ++q) {
    const uint4 u = *reinterpret_cast<const uint4*>(p + 8 * q);
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(b[e]);
      h[8 * q + 2 * e] = f.x;
      h[8 * q + 2 * e + 1] = f.y;
    }
  }
}

// Rows in flight per warp: a ring of shared-memory slots filled by cp.async,
// so a warp keeps kRing row loads outstanding (the pass is bound by how many
// bytes are in flight per SM, not by arithmetic).
constexpr int kRing = 4;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Shared memory of one CTA (bytes): per warp a ring of kRing slots of (one
// H2 row, 4 row scalars); the final fold reuses the same area.
template <int A, int CPL>
struct HeadSmem {
  static constexpr int H = 16 * CPL;
  static constexpr int kSlot = 2 * H * 2 + 16;  // bf16 row + act, old logp, adv, ret
  static constexpr int kRingBytes = kWarps * kRing * kSlot;
  static constexpr int kFold = kWarps * (2 * H + A * H + H + A + 1 + kStats) * 4;
  static constexpr int kTotal = kRingBytes > kFold ? kRingBytes : kFold;
};

// CPL = H / 16 columns per lane; A actions (categorical).
template <int A, int CPL>
__global__ void __launch_bounds__(kThreads, 2) ppo_head_kernel(
    const bf16* __restrict__ H2, long long ldh, const bf16* __restrict__ W3, long long ldw,
    const float* __restrict__ b3, int crow, const int* __restrict__ act, const float* __restrict__ old_logp,
    const float* __restrict__ adv, const float* __restrict__ ret, bf16* __restrict__ dz, long long ldz,
    float* __restrict__ part, int M, float clip, float vf_coef, float ent_coef) {
  using S = HeadSmem<A, CPL>;
  constexpr int H = S::H;
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* ring_base = smem;
  float* red = reinterpret_cast<float*>(smem);  // the fold, after the loop
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const bool critic = lane >= 16;
  const int col = (critic ? H : 0) + (lane & 15) * CPL;  // first column of this lane in H2 / dZ2
  // output-layer weights of this lane's columns, in registers for the whole
  // pass: actor rows 0..A-1, or the critic row
  float wt[A][CPL];
#pragma unroll
  for (int k = 0; k < A; ++k) {
    if (critic && k > 0) {
#pragma unroll
      for (int c = 0; c < CPL; ++c) wt[k][c] = 0.f;
    } else {
      load_row<CPL>(W3 + static_cast<long long>(critic ? crow : k) * ldw + col, wt[k]);
    }
  }
  float bl[A];
#pragma unroll
  for (int k = 0; k < A; ++k) bl[k] = b3[k];
  const float bv = b3[crow];
  const float inv_m = 1.f / static_cast<float>(M);

  float db2[CPL], gw[A][CPL];
#pragma unroll
  for (int c = 0; c < CPL; ++c) {
    db2[c] = 0.f;
#pragma unroll
    for (int k = 0; k < A; ++k) gw[k][c] = 0.f;
  }
  float gb[A + 1];
#pragma unroll
  for (int k = 0; k <= A; ++k) gb[k] = 0.f;
  float st_pg = 0.f, st_v = 0.f, st_h = 0.f, st_kl = 0.f, st_cf = 0.f, st_n = 0.f;

  const int gw_id = blockIdx.x * kWarps + w, n_warps = gridDim.x * kWarps;
  uint8_t* ring = ring_base + w * kRing * S::kSlot;
  // Lane l stages bytes [l * 2 CPL, (l + 1) * 2 CPL) of a row: exactly the
  // columns it reads back, so its own cp.async wait covers them; lanes 0-3
  // stage the row's action, old log-prob, advantage and return.
  auto issue = [&](int slot, int r) {
    if (r < M) {
      uint8_t* dst = ring + slot * S::kSlot;
      const bf16* src = H2 + static_cast<long long>(r) * ldh + col;
#pragma unroll
      for (int q = 0; q < CPL / 8; ++q) cp_async16(dst + (col + 8 * q) * 2, src + 8 * q);
      if (lane < 4) {
        const void* sp = lane == 0 ? static_cast<const void*>(act + r)
                         : lane == 1 ? static_cast<const void*>(old_logp + r)
                         : lane == 2 ? static_cast<const void*>(adv + r)
                                     : static_cast<const void*>(ret + r);
        cp_async4(dst + 2 * H * 2 + 4 * lane, sp);
      }
    }
    cp_async_commit();  // one group per slot, empty past the end
  };
#pragma unroll
  for (int q = 0; q < kRing; ++q) issue(q, gw_id + q * n_warps);
  int slot = 0;
  for (int r = gw_id; r < M; r += n_warps) {
    cp_async_wait<kRing - 1>();  // this lane's copies of the oldest slot are done
    const uint8_t* cur = ring + slot * S::kSlot;
    float h[CPL];
    load_row<CPL>(reinterpret_cast<const bf16*>(cur) + col, h);
    float scal = lane < 4 ? *reinterpret_cast<const float*>(cur + 2 * H * 2 + 4 * lane) : 0.f;
    const int a = __float_as_int(__shfl_sync(0xffffffffu, scal, 0));
    const float old = __shfl_sync(0xffffffffu, scal, 1), Ad = __shfl_sync(0xffffffffu, scal, 2),
                R = __shfl_sync(0xffffffffu, scal, 3);
    __syncwarp();
    issue(slot, r + kRing * n_warps);  // refill the slot just read
    slot = slot + 1 == kRing ? 0 : slot + 1;
    // ---- forward: partial dot products, then sums over the 16 lanes of a half
    float s[A];
#pragma unroll
    for (int k = 0; k < A; ++k) {
      float acc = 0.f;
#pragma unroll
      for (int c = 0; c < CPL; ++c) acc = fmaf(h[c], wt[k][c], acc);
      s[k] = acc;
    }
#pragma unroll
    for (int k = 0; k < A; ++k) {
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) s[k] += __shfl_xor_sync(0xffffffffu, s[k], o);
    }
    // actor lanes hold the logit sums in s[k], critic lanes the value sum in s[0]
    float l[A];
#pragma unroll
    for (int k = 0; k < A; ++k) {
      const float other = __shfl_xor_sync(0xffffffffu, s[k], 16);
      l[k] = (critic ? other : s[k]) + bl[k];
    }
    const float vs = __shfl_xor_sync(0xffffffffu, s[0], 16);  // every lane takes part in the exchange
    const float V = (critic ? s[0] : vs) + bv;
    // ---- loss (every lane, same values)
    float mx = l[0];
#pragma unroll
    for (int k = 1; k < A; ++k) mx = fmaxf(mx, l[k]);
    float p[A], se = 0.f;
#pragma unroll
    for (int k = 0; k < A; ++k) {
      p[k] = __expf(l[k] - mx);
      se += p[k];
    }
    const float inv = 1.f / se, lse = mx + __logf(se);
    float ent = 0.f;
#pragma unroll
    for (int k = 0; k < A; ++k) {
      p[k] *= inv;
      ent -= p[k] * (l[k] - lse);
    }
    float la = l[0];
#pragma unroll
    for (int k = 1; k < A; ++k) la = (k == a) ? l[k] : la;
    const float lr = (la - lse) - old;
    const float ratio = __expf(lr);
    const float un = ratio * Ad;
    const float cl = fminf(fmaxf(ratio, 1.f - clip), 1.f + clip) * Ad;
    const bool use_unclipped = un <= cl || (ratio > 1.f - clip && ratio < 1.f + clip);
    const float dlp = use_unclipped ? -Ad * ratio : 0.f;
    float dl[A];
#pragma unroll
    for (int k = 0; k < A; ++k)
      dl[k] = (dlp * ((k == a ? 1.f : 0.f) - p[k]) + ent_coef * p[k] * ((l[k] - lse) + ent)) * inv_m;
    const float dv = vf_coef * (V - R) * inv_m;
    // ---- backward through the output layer and the tanh
    float dzv[CPL];
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      float g = 0.f;
      if (critic) {
        g = dv * wt[0][c];
      } else {
#pragma unroll
        for (int k = 0; k < A; ++k) g = fmaf(dl[k], wt[k][c], g);
      }
      dzv[c] = g * (1.f - h[c] * h[c]);
      db2[c] += dzv[c];
      if (critic) {
        gw[0][c] = fmaf(dv, h[c], gw[0][c]);
      } else {
#pragma unroll
        for (int k = 0; k < A; ++k) gw[k][c] = fmaf(dl[k], h[c], gw[k][c]);
      }
    }
    bf16* dst = dz + static_cast<long long>(r) * ldz + col;
#pragma unroll
    for (int q = 0; q < CPL / 8; ++q) {
      uint4 pk;
      __nv_bfloat162* ph = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
      for (int e = 0; e < 4; ++e) ph[e] = __floats2bfloat162_rn(dzv[8 * q + 2 * e], dzv[8 * q + 2 * e + 1]);
      *reinterpret_cast<uint4*>(dst + 8 * q) = pk;
    }
    if (lane == 0) {
#pragma unroll
      for (int k = 0; k < A; ++k) gb[k] += dl[k];
      gb[A] += dv;
      st_pg += -fminf(un, cl);
      st_v += 0.5f * (V - R) * (V - R);
      st_h += ent;
      st_kl += (ratio - 1.f) - lr;
      st_cf += fabsf(ratio - 1.f) > clip ? 1.f : 0.f;
      st_n += 1.f;
    }
  }
  // ---- this warp's sums into its shared-memory row, then a fixed-order fold
  cp_async_wait<0>();
  __syncthreads();  // every warp is done with its ring (the fold reuses it)
  const int L = part_len(H, A);
  float* row = red + w * L;
#pragma unroll
  for (int c = 0; c < CPL; ++c) {
    row[col + c] = db2[c];  // db2 [2H]
    if (critic) {
      row[2 * H + A * H + (col - H) + c] = gw[0][c];  // dW3c [H]
    } else {
#pragma unroll
      for (int k = 0; k < A; ++k) row[2 * H + k * H + col + c] = gw[k][c];  // dW3a [A][H]
    }
  }
  if (lane == 0) {
    float* tail = row + 2 * H + A * H + H;
#pragma unroll
    for (int k = 0; k <= A; ++k) tail[k] = gb[k];
    tail[A + 1] = st_pg;
    tail[A + 2] = st_v;
    tail[A + 3] = st_h;
    tail[A + 4] = st_kl;
    tail[A + 5] = st_cf;
    tail[A + 6] = st_n;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < L; i += kThreads) {
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < kWarps; ++q) t += red[q * L + i];
    part[static_cast<long long>(blockIdx.x) * L + i] = t;
  }
}

// Sums the CTAs' partial rows (fixed order) and scatters: db2 -> g_b2[j],
// dW3a[k][j] -> g_w3[k, j], dW3c[j] -> g_w3[crow, H + j], db3 -> g_b3[k] and
// g_b3[crow] (gradients are written, not accumulated), statistics -> stats[0..5]
// (added).
__global__ void __launch_bounds__(1024) ppo_head_reduce_kernel(const float* __restrict__ part, int parts, int H,
                                                               int A, int crow, float* __restrict__ g_w3,
                                                               long long ldw, float* __restrict__ g_b3,
                                                               float* __restrict__ g_b2, float* __restrict__ stats) {
  __shared__ float sm[32][33];
  const int n = part_len(H, A);
  const int oi = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int i = blockIdx.x * 32 + oi;
  float s = 0.f;
  if (i < n)
    for (int b = g; b < parts; b += 32) s += part[static_cast<long long>(b) * n + i];
  sm[g][oi] = s;
  __syncthreads();
  if (g != 0 || i >= n) return;
  float t = 0.f;
  for (int q = 0; q < 32; ++q) t += sm[q][oi];
  int j = i;
  if (j < 2 * H) { g_b2[j] = t; return; }
  j -= 2 * H;
  if (j < A * H) { g_w3[static_cast<long long>(j / H) * ldw + (j % H)] = t; return; }
  j -= A * H;
  if (j < H) { g_w3[static_cast<long long>(crow) * ldw + H + j] = t; return; }
  j -= H;
  if (j < A) { g_b3[j] = t; return; }
  if (j == A) { g_b3[crow] = t; return; }
  j -= A + 1;
  if (stats && j < kStats) stats[j] += t;
}

template <int A, int CPL>
int launch_head(const TbPpoHeadArgs* a, cudaStream_t s) {
  const int L = part_len(16 * CPL, A);
  const size_t smem = HeadSmem<A, CPL>::kTotal;
  auto k = ppo_head_kernel<A, CPL>;
  tb::ensure_dyn_smem(reinterpret_cast<const void*>(k), static_cast<int>(smem));
  k<<<a->parts, kThreads, smem, s>>>(static_cast<const bf16*>(a->H2), a->ldh, static_cast<const bf16*>(a->W3),
                                     a->ldw, a->b3, a->crow, a->act, a->old_logp, a->adv, a->ret,
                                     static_cast<bf16*>(a->dz), a->ldz, a->part, a->M, a->clip, a->vf_coef,
                                     a->ent_coef);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return static_cast<int>(e);
  const int blocks = (L + 31) / 32;
  ppo_head_reduce_kernel<<<blocks, 1024, 0, s>>>(a->part, a->parts, 16 * CPL, A, a->crow, a->g_w3, a->ldgw, a->g_b3,
                                                 a->g_b2, a->stats);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace

extern "C" {

long long tb_ppo_head_part_numel(int H, int A, int parts) {
  return static_cast<long long>(part_len(H, A)) * parts;
}

int tb_ppo_head_default_parts(int H, int A) {
  // one partial row per resident CTA: SMs x CTAs that fit on an SM
  int dev = 0, sms = 148, per_sm = 1;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  size_t smem = 0;
  const void* fn = nullptr;
  if (A == 2 && H == 256) {
    fn = reinterpret_cast<const void*>(ppo_head_kernel<2, 16>);
    smem = HeadSmem<2, 16>::kTotal;
  }
  if (A == 2 && H == 128) {
    fn = reinterpret_cast<const void*>(ppo_head_kernel<2, 8>);
    smem = HeadSmem<2, 8>::kTotal;
  }
  if (fn != nullptr) {
    tb::ensure_dyn_smem(fn, static_cast<int>(smem));
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, smem) != cudaSuccess || per_sm < 1)
      per_sm = 1;
  }
  cudaGetLastError();
  return sms * per_sm;
}

int tb_ppo_head(const TbPpoHeadArgs* a, cudaStream_t s) {
  if (a->M <= 0) return 0;
  if (a->parts <= 0 || (a->ldh % 8) || (a->ldz % 8) || (a->ldw % 8) || a->crow < a->A ||
      (reinterpret_cast<uintptr_t>(a->H2) & 15) || (reinterpret_cast<uintptr_t>(a->dz) & 15) ||
      (reinterpret_cast<uintptr_t>(a->W3) & 15))
    return static_cast<int>(cudaErrorInvalidValue);
  if (a->A == 2) {
    switch (a->H) {
      case 256: return launch_head<2, 16>(a, s);
      case 128: return launch_head<2, 8>(a, s);
      default: break;
    }
  }
  return static_cast<int>(cudaErrorInvalidValue);
}

}  // extern "C"
