// Filtered token sampling: temperature, top-k, top-p (nucleus) and an end-of-
// sequence stop, for the decode loop of the rollout engine.
//
// The reference passes top_p and top_k to its sampler
// (turbol_vllm/include/turbol/rollout/rollout_engine.hpp:8-17,
// turbol_vllm/python/turbol/vllm_inference.py:182-186); here they are one
// kernel, one CTA (1024 threads) per row of bf16 logits [B, V].
//
// Thresholds are exact without sorting the vocabulary.  A bf16 logit maps to
// a 16-bit key whose unsigned order is the float order; two histogram passes
// (high byte, then the low byte inside the selected high-byte bin) find
//   * top-k: the key of the k-th largest logit (every token whose logit ties
//     with it is kept as well);
//   * top-p: among the tokens kept by top-k, the largest key tau such that the
//     tokens with key >= tau hold at least p of the kept probability mass.
//     Masses are summed in 2^-40 fixed point with integer atomics, so the
//     threshold does not depend on the order in which threads add.
// The token is then drawn by inverse-CDF sampling over the kept tokens (one
// Philox uniform per (seed, row, step), a block scan of per-thread masses, the
// owning thread re-walks its own elements), the same scheme as the unfiltered
// sampler in llm.cu.  The returned log-probability is that of the token under
// the full temperature-scaled softmax (the distribution a trainer recomputes),
// not under the truncated one.
//
// End of sequence: with eos_id >= 0, a row whose done flag is set emits
// pad_id with log-prob 0 and skips all work; a row that samples eos_id sets its
// done flag, records its length (step + 1) and increments the done counter,
// which the host reads every few decode steps to stop early.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "device_common.cuh"
#include "kernels.h"

namespace {

using bf16 = __nv_bfloat16;
constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr float kMassScale = 1099511627776.f;  // 2^40

__device__ __forceinline__ uint32_t key_of(uint16_t b) {
  return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
}

// Walks this thread's elements of the row in a fixed order (16-byte chunks of
// 8 logits strided across the block, then the scalar tail) and calls
// f(index, raw bf16 bits).
template <typename F>
__device__ __forceinline__ void walk(const bf16* __restrict__ x, int V, int nv, F&& f) {
  const int tid = threadIdx.x;
  for (int c = tid; c < nv; c += kThreads) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + static_cast<long long>(c) * 8);
    const uint16_t* h = reinterpret_cast<const uint16_t*>(&u);
#pragma unroll
    for (int k = 0; k < 8; ++k) f(c * 8 + k, h[k]);
  }
  const uint16_t* xs = reinterpret_cast<const uint16_t*>(x);
  for (int i = nv * 8 + tid; i < V; i += kThreads) f(i, xs[i]);
}

__device__ __forceinline__ float bits_to_float(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// The bin b of hist[256] with  sum_{j>b} hist[j] < target <= sum_{j>=b} hist[j]
// (target >= 1); writes sum_{j>b} hist[j] to *above.  Run by warp 0: lane l
// owns bins [8l, 8l+8).  Returns -1 (on lane 0) if the total is below target.
template <typename T>
__device__ int find_crossing(const T* hist, T target, T* above) {
  const int lane = threadIdx.x & 31;
  T own = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) own += hist[lane * 8 + j];
  // inclusive suffix sum over lanes (from lane 31 down)
  T suf = own;
  for (int o = 1; o < 32; o <<= 1) {
    const T y = __shfl_down_sync(0xffffffffu, suf, o);
    if (lane + o < 32) suf += y;
  }
  const T above_lane = suf - own;  // mass of the lanes above this one
  int found = -1;
  T found_above = 0;
  if (above_lane < target && target <= suf) {
    T acc = above_lane;
    for (int j = 7; j >= 0; --j) {
      const T h = hist[lane * 8 + j];
      if (acc < target && target <= acc + h) {
        found = lane * 8 + j;
        found_above = acc;
        break;
      }
      acc += h;
    }
  }
  // exactly one lane found the crossing (or none if the total is short)
  const unsigned who = __ballot_sync(0xffffffffu, found >= 0);
  if (who == 0) return -1;
  const int src = __ffs(who) - 1;
  found = __shfl_sync(0xffffffffu, found, src);
  found_above = __shfl_sync(0xffffffffu, found_above, src);
  if (lane == 0) *above = found_above;
  return found;
}

__global__ void __launch_bounds__(kThreads) sample_filtered_kernel(
    const bf16* __restrict__ logits, long long ld, int V, float temperature, int top_k, float top_p,
    unsigned long long seed, const long long* __restrict__ step_ptr, long long step_imm, int* __restrict__ out_tok,
    float* __restrict__ out_logp, int* __restrict__ tok_mat, float* __restrict__ lp_mat, int ld_mat,
    const unsigned long long* __restrict__ seed_ptr, const float* __restrict__ temp_ptr, int eos_id, int pad_id,
    uint8_t* __restrict__ done, int* __restrict__ lengths, int* __restrict__ n_done) {
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const long long step = step_ptr ? *step_ptr : step_imm;
  if (eos_id >= 0 && done != nullptr && done[row]) {
    if (tid == 0) {
      out_tok[row] = pad_id;
      if (out_logp) out_logp[row] = 0.f;
      if (tok_mat && step >= 0 && step < ld_mat) tok_mat[static_cast<long long>(row) * ld_mat + step] = pad_id;
      if (lp_mat && step >= 0 && step < ld_mat) lp_mat[static_cast<long long>(row) * ld_mat + step] = 0.f;
    }
    return;
  }
  const bf16* x = logits + static_cast<long long>(row) * ld;
  if (seed_ptr) seed = *seed_ptr;
  if (temp_ptr) temperature = *temp_ptr;
  const bool greedy = temperature <= 0.f;
  const float inv_t = greedy ? 1.f : 1.f / temperature;
  const bool vec = (V % 8 == 0) && (ld % 8 == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
  const int nv = vec ? V / 8 : 0;

  __shared__ unsigned long long s_hist[256];
  __shared__ float s_a[kWarps], s_b[kWarps];
  __shared__ int s_i[kWarps];
  __shared__ float s_M, s_S, s_target;
  __shared__ int s_tok, s_owner, s_bin;
  __shared__ unsigned long long s_above, s_total;
  __shared__ uint32_t s_tau;

  // ---- pass 1: max of the scaled logits, sum of exp below it, argmax
  float m = -INFINITY, sm = 0.f, best = -INFINITY;
  int best_i = 0;
  walk(x, V, nv, [&](int i, uint16_t b) {
    const float z = bits_to_float(b) * inv_t;
    if (z != z) return;  // NaN logits are never sampled
    if (z > best) { best = z; best_i = i; }
    if (z > m) {
      sm = sm * __expf(m - z) + 1.f;
      m = z;
    } else if (z != -INFINITY) {
      sm += __expf(z - m);
    }
  });
  {
    float bm = m, bb = best;
    int bi = best_i;
    for (int o = 16; o > 0; o >>= 1) {
      bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
      const float ob = __shfl_xor_sync(0xffffffffu, bb, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > bb || (ob == bb && oi < bi)) { bb = ob; bi = oi; }
    }
    if (lane == 0) { s_a[w] = bm; s_b[w] = bb; s_i[w] = bi; }
    __syncthreads();
    if (w == 0) {
      bm = s_a[lane];
      bb = s_b[lane];
      bi = s_i[lane];
      for (int o = 16; o > 0; o >>= 1) {
        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
        const float ob = __shfl_xor_sync(0xffffffffu, bb, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > bb || (ob == bb && oi < bi)) { bb = ob; bi = oi; }
      }
      if (lane == 0) { s_M = bm; s_tok = bi; }
    }
    __syncthreads();
  }
  const float M = s_M;
  {  // full normalizer S (for the returned log-prob)
    float wt = (m == -INFINITY) ? 0.f : sm * __expf(m - M);
    for (int o = 16; o > 0; o >>= 1) wt += __shfl_xor_sync(0xffffffffu, wt, o);
    if (lane == 0) s_a[w] = wt;
    __syncthreads();
    if (w == 0) {
      float t = s_a[lane];
      for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      if (lane == 0) s_S = t;
    }
    __syncthreads();
  }

  if (!greedy) {
    // ---- thresholds (keys >= tau are kept)
    if (tid == 0) s_tau = 0u;
    __syncthreads();
    if (top_k > 0 && top_k < V) {
      // pass 2: counts by the key's high byte
      for (int j = tid; j < 256; j += kThreads) s_hist[j] = 0ull;
      __syncthreads();
      walk(x, V, nv, [&](int, uint16_t b) {
        if (bits_to_float(b) != bits_to_float(b)) return;
        atomicAdd(&s_hist[key_of(b) >> 8], 1ull);
      });
      __syncthreads();
      if (w == 0) {
        unsigned long long above;
        const int bin = find_crossing<unsigned long long>(s_hist, static_cast<unsigned long long>(top_k), &above);
        if (lane == 0) { s_bin = bin; s_above = above; }
      }
      __syncthreads();
      const int hi = s_bin;
      if (hi >= 0) {
        const unsigned long long need = static_cast<unsigned long long>(top_k) - s_above;
        __syncthreads();
        // pass 3: counts by the low byte inside the selected high-byte bin
        for (int j = tid; j < 256; j += kThreads) s_hist[j] = 0ull;
        __syncthreads();
        walk(x, V, nv, [&](int, uint16_t b) {
          const uint32_t k = key_of(b);
          if ((k >> 8) == static_cast<uint32_t>(hi) && bits_to_float(b) == bits_to_float(b))
            atomicAdd(&s_hist[k & 255u], 1ull);
        });
        __syncthreads();
        if (w == 0) {
          unsigned long long above;
          const int lo = find_crossing<unsigned long long>(s_hist, need, &above);
          if (lane == 0 && lo >= 0) s_tau = (static_cast<uint32_t>(hi) << 8) | static_cast<uint32_t>(lo);
        }
        __syncthreads();
      }
    }
    if (top_p > 0.f && top_p < 1.f) {
      const uint32_t tau_k = s_tau;
      // pass 4: kept probability mass by high byte (fixed point)
      for (int j = tid; j < 256; j += kThreads) s_hist[j] = 0ull;
      __syncthreads();
      walk(x, V, nv, [&](int, uint16_t b) {
        const float z = bits_to_float(b) * inv_t;
        const uint32_t k = key_of(b);
        if (z != z || k < tau_k || z == -INFINITY) return;
        const unsigned long long q = __float2ull_rz(__expf(z - M) * kMassScale);
        if (q) atomicAdd(&s_hist[k >> 8], q);
      });
      __syncthreads();
      if (w == 0) {
        unsigned long long tot = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) tot += s_hist[lane * 8 + j];
        for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
        unsigned long long target = static_cast<unsigned long long>(ceil(static_cast<double>(top_p) * static_cast<double>(tot)));
        if (target < 1ull) target = 1ull;
        if (target > tot) target = tot;
        unsigned long long above = 0;
        const int bin = tot ? find_crossing<unsigned long long>(s_hist, target, &above) : -1;
        if (lane == 0) { s_bin = bin; s_above = above; s_total = target; }
      }
      __syncthreads();
      const int hi = s_bin;
      if (hi >= 0) {
        const unsigned long long need = s_total - s_above;
        __syncthreads();
        // pass 5: mass by low byte inside that bin
        for (int j = tid; j < 256; j += kThreads) s_hist[j] = 0ull;
        __syncthreads();
        walk(x, V, nv, [&](int, uint16_t b) {
          const float z = bits_to_float(b) * inv_t;
          const uint32_t k = key_of(b);
          if (z != z || k < tau_k || (k >> 8) != static_cast<uint32_t>(hi) || z == -INFINITY) return;
          const unsigned long long q = __float2ull_rz(__expf(z - M) * kMassScale);
          if (q) atomicAdd(&s_hist[k & 255u], q);
        });
        __syncthreads();
        if (w == 0) {
          unsigned long long above;
          const int lo = find_crossing<unsigned long long>(s_hist, need, &above);
          if (lane == 0 && lo >= 0) {
            const uint32_t tau_p = (static_cast<uint32_t>(hi) << 8) | static_cast<uint32_t>(lo);
            if (tau_p > s_tau) s_tau = tau_p;
          }
        }
        __syncthreads();
      }
    }
    const uint32_t tau = s_tau;
    // ---- pass 6: this thread's kept mass, block scan, inverse-CDF pick
    float wt = 0.f;
    walk(x, V, nv, [&](int, uint16_t b) {
      const float z = bits_to_float(b) * inv_t;
      if (z == z && z != -INFINITY && key_of(b) >= tau) wt += __expf(z - M);
    });
    float inc = wt;
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += y;
    }
    __syncthreads();
    if (lane == 31) s_a[w] = inc;
    __syncthreads();
    if (w == 0) {
      float t = s_a[lane];
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += y;
      }
      s_b[lane] = t;
      if (lane == 31) {
        const uint4 r = tb::Philox::gen(seed, 0x53414D50u, static_cast<uint32_t>(row), static_cast<uint32_t>(step),
                                        static_cast<uint32_t>(step >> 32));
        s_target = tb::u01_open(r.x) * t;
        s_owner = -1;
      }
    }
    __syncthreads();
    const float excl = inc - wt + (w > 0 ? s_b[w - 1] : 0.f);
    const float target = s_target;
    if (wt > 0.f && excl <= target && target < excl + wt) atomicMax(&s_owner, tid);
    __syncthreads();
    if (s_owner < 0) {  // rounding past the end: the last thread with mass
      if (wt > 0.f) atomicMax(&s_owner, tid);
      __syncthreads();
    }
    if (tid == s_owner) {
      float acc = excl;
      int tok = -1, last_i = -1;
      walk(x, V, nv, [&](int i, uint16_t b) {
        const float z = bits_to_float(b) * inv_t;
        if (z != z || z == -INFINITY || key_of(b) < tau) return;
        acc += __expf(z - M);
        last_i = i;
        if (tok < 0 && acc > target) tok = i;
      });
      s_tok = tok >= 0 ? tok : last_i;
    }
    __syncthreads();
  }
  if (tid == 0) {
    const int tok = s_tok;
    const float lp = bits_to_float(reinterpret_cast<const uint16_t*>(x)[tok]) * inv_t - (M + __logf(s_S));
    out_tok[row] = tok;
    if (out_logp) out_logp[row] = lp;
    if (tok_mat && step >= 0 && step < ld_mat) tok_mat[static_cast<long long>(row) * ld_mat + step] = tok;
    if (lp_mat && step >= 0 && step < ld_mat) lp_mat[static_cast<long long>(row) * ld_mat + step] = lp;
    if (eos_id >= 0 && tok == eos_id && done != nullptr) {
      done[row] = 1;
      if (lengths) lengths[row] = static_cast<int>(step + 1);
      if (n_done) atomicAdd(n_done, 1);
    }
  }
}

}  // namespace

extern "C" int tb_sample_filtered(const void* logits, long long ld, int B, int V, float temperature, int top_k,
                                  float top_p, unsigned long long seed, const long long* step_ptr, long long step_imm,
                                  int* out_tok, float* out_logp, int* tok_mat, float* lp_mat, int ld_mat,
                                  const unsigned long long* seed_ptr, const float* temp_ptr, int eos_id, int pad_id,
                                  unsigned char* done, int* lengths, int* n_done, cudaStream_t s) {
  if (B <= 0) return 0;
  if (V <= 0 || (eos_id >= 0 && done == nullptr)) return static_cast<int>(cudaErrorInvalidValue);
  sample_filtered_kernel<<<B, kThreads, 0, s>>>(static_cast<const bf16*>(logits), ld, V, temperature, top_k, top_p,
                                                seed, step_ptr, step_imm, out_tok, out_logp, tok_mat, lp_mat, ld_mat,
                                                seed_ptr, temp_ptr, eos_id, pad_id, done, lengths, n_done);
  return static_cast<int>(cudaGetLastError());
}
