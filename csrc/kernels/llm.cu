// Transformer kernels for the RLHF policy (everything but the GEMMs and the
// prefill/training attention): RMSNorm forward/backward, RoPE, embedding
// forward/backward, SwiGLU backward, paged KV-cache writes, paged GQA decode
// attention, temperature sampling, chunked LM-head log-probabilities with the
// in-place logits gradient, and the GRPO per-token loss.
//
// Layout conventions: activations are row-major [tokens, features] bf16; a
// fused QKV row is [q heads | k heads | v heads] x head_dim; the paged KV cache
// is [num_blocks, kv_heads, block_size, head_dim] bf16 (one contiguous
// block_size x head_dim tile per kv head), addressed through a per-sequence
// block table.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "device_common.cuh"
#include "kernels.h"

namespace {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float bf(bf16 x) { return __bfloat162float(x); }

// 8 bf16 <-> 8 floats through one 16-byte access
__device__ __forceinline__ void ld8(const bf16* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void st8(bf16* p, const float* f) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

// ------------------------------------------------------------------ RMSNorm
// One warp per row; D % 256 == 0 (8 bf16 per lane per step).
__global__ void rmsnorm_fwd_kernel(const bf16* __restrict__ x, const float* __restrict__ w, bf16* __restrict__ y,
                                   float* __restrict__ rstd_out, int T, int D, float eps) {
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= T) return;
  const bf16* xr = x + static_cast<long long>(row) * D;
  float ss = 0.f;
  for (int c = lane * 8; c < D; c += 256) {
    float f[8];
    ld8(xr + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
  }
  ss = tb::warp_sum(ss);
  const float r = rsqrtf(ss / static_cast<float>(D) + eps);
  if (rstd_out && lane == 0) rstd_out[row] = r;
  bf16* yr = y + static_cast<long long>(row) * D;
  for (int c = lane * 8; c < D; c += 256) {
    float f[8];
    ld8(xr + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] *= r * w[c + i];
    st8(yr + c, f);
  }
}

// dx = r * (w*dy - xhat * mean(xhat * w * dy)),  dw += sum_rows dy * xhat.
// A block of 8 warps walks `rows_per_block` rows; each lane keeps its dw
// partial for D/32 columns in registers (D <= 8192) and adds it atomically once.
template <int MAXV>
__global__ void rmsnorm_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                                   const float* __restrict__ w, const float* __restrict__ rstd,
                                   bf16* __restrict__ dx, const bf16* __restrict__ dx_add, float* __restrict__ dw,
                                   int T, int D, int rows_per_block) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  float dwp[MAXV];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) dwp[i] = 0.f;
  const int r0 = blockIdx.x * rows_per_block, r1 = min(T, r0 + rows_per_block);
  for (int row = r0 + warp; row < r1; row += nw) {
    const long long o = static_cast<long long>(row) * D;
    const float r = rstd[row];
    float dot = 0.f;
#pragma unroll
    for (int s = 0; s < MAXV / 8; ++s) {
      const int c = s * 256 + lane * 8;
      if (c < D) {
        float g[8], xv[8];
        ld8(dy + o + c, g);
        ld8(x + o + c, xv);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float xh = xv[i] * r;
          dot += xh * w[c + i] * g[i];
          dwp[s * 8 + i] += g[i] * xh;
        }
      }
    }
    dot = tb::warp_sum(dot) / static_cast<float>(D);
#pragma unroll
    for (int s = 0; s < MAXV / 8; ++s) {
      const int c = s * 256 + lane * 8;
      if (c < D) {
        float g[8], xv[8], out[8];
        ld8(dy + o + c, g);
        ld8(x + o + c, xv);
        float add[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (dx_add) ld8(dx_add + o + c, add);
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] = r * (w[c + i] * g[i] - xv[i] * r * dot) + add[i];
        st8(dx + o + c, out);
      }
    }
  }
#pragma unroll
  for (int s = 0; s < MAXV / 8; ++s) {
    const int c = s * 256 + lane * 8;
    if (c < D) {
#pragma unroll
      for (int i = 0; i < 8; ++i) atomicAdd(dw + c + i, dwp[s * 8 + i]);
    }
  }
}

// ------------------------------------------------------------------ RoPE
// Rotate-half RoPE in place on the q and k heads of fused QKV rows.
// table: [max_pos, D/2] float2 (cos, sin).  sign = -1 applies the inverse
// rotation (the backward pass).
__global__ void rope_kernel(bf16* __restrict__ qkv, long long ld, const int* __restrict__ pos,
                            const float2* __restrict__ table, int T, int n_rot_heads, int D, float sign) {
  const int half = D / 2;
  const long long total = static_cast<long long>(T) * n_rot_heads * (half / 4);
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int j4 = static_cast<int>(e % (half / 4));
    const long long th = e / (half / 4);
    const int h = static_cast<int>(th % n_rot_heads);
    const int t = static_cast<int>(th / n_rot_heads);
    bf16* base = qkv + static_cast<long long>(t) * ld + static_cast<long long>(h) * D;
    const float2* tab = table + static_cast<long long>(pos[t]) * half;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = j4 * 4 + k;
      const float2 cs = tab[j];
      const float s = sign * cs.y;
      const float x1 = bf(base[j]), x2 = bf(base[j + half]);
      base[j] = __float2bfloat16_rn(x1 * cs.x - x2 * s);
      base[j + half] = __float2bfloat16_rn(x2 * cs.x + x1 * s);
    }
  }
}

// ------------------------------------------------------------------ embedding
__global__ void embed_fwd_kernel(const int* __restrict__ ids, const bf16* __restrict__ W, bf16* __restrict__ out,
                                 int T, int D, int V, int* __restrict__ err) {
  const long long total = static_cast<long long>(T) * (D / 8);
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(e / (D / 8)), c = static_cast<int>(e % (D / 8)) * 8;
    int id = ids[t];
    if (id < 0 || id >= V) {
      if (err) atomicCAS(err, 0, 1);
      id = 0;
    }
    *reinterpret_cast<uint4*>(out + static_cast<long long>(t) * D + c) =
        *reinterpret_cast<const uint4*>(W + static_cast<long long>(id) * D + c);
  }
}

__global__ void embed_bwd_kernel(const int* __restrict__ ids, const bf16* __restrict__ dout, float* __restrict__ dW,
                                 int T, int D, int V) {
  const long long total = static_cast<long long>(T) * (D / 8);
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(e / (D / 8)), c = static_cast<int>(e % (D / 8)) * 8;
    const int id = ids[t];
    if (id < 0 || id >= V) continue;
    float g[8];
    ld8(dout + static_cast<long long>(t) * D + c, g);
    float* dst = dW + static_cast<long long>(id) * D + c;
#pragma unroll
    for (int i = 0; i < 8; ++i) atomicAdd(dst + i, g[i]);
  }
}

// ------------------------------------------------------------------ SwiGLU backward
// gu: interleaved [T, 2F] (gate 2j, up 2j+1), dh: [T, F] -> dgu [T, 2F]
__global__ void swiglu_bwd_kernel(const bf16* __restrict__ gu, const bf16* __restrict__ dh, bf16* __restrict__ dgu,
                                  long long T, int F) {
  const long long total = T * (F / 4);
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long t = e / (F / 4);
    const int j = static_cast<int>(e % (F / 4)) * 4;
    float x[8], g4[4];
    ld8(gu + t * 2 * F + 2 * j, x);
    const uint2 u = *reinterpret_cast<const uint2*>(dh + t * F + j);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    g4[0] = a.x;
    g4[1] = a.y;
    g4[2] = b.x;
    g4[3] = b.y;
    float o[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float g = x[2 * k], up = x[2 * k + 1];
      const float sg = 1.f / (1.f + __expf(-g));
      const float silu = g * sg;
      o[2 * k] = g4[k] * up * (sg * (1.f + g * (1.f - sg)));
      o[2 * k + 1] = g4[k] * silu;
    }
    st8(dgu + t * 2 * F + 2 * j, o);
  }
}

// gu: interleaved [T, 2F] -> act [T, F] = silu(gate) * up
__global__ void swiglu_fwd_kernel(const bf16* __restrict__ gu, bf16* __restrict__ act, long long T, int F) {
  const long long total = T * (F / 4);
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long t = e / (F / 4);
    const int j = static_cast<int>(e % (F / 4)) * 4;
    float x[8];
    ld8(gu + t * 2 * F + 2 * j, x);
    __nv_bfloat162 o[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float g0 = x[4 * k], u0 = x[4 * k + 1], g1 = x[4 * k + 2], u1 = x[4 * k + 3];
      o[k] = __floats2bfloat162_rn(g0 / (1.f + __expf(-g0)) * u0, g1 / (1.f + __expf(-g1)) * u1);
    }
    *reinterpret_cast<uint2*>(act + t * F + j) = *reinterpret_cast<uint2*>(o);
  }
}

// ------------------------------------------------------------------ KV cache
// k, v rows of the fused QKV output -> paged cache at each token's slot.
__global__ void kv_write_kernel(const bf16* __restrict__ qkv, long long ld, int k_off, int v_off,
                                const int* __restrict__ seq_of_token, const int* __restrict__ pos,
                                const int* __restrict__ block_table, int max_blocks, bf16* __restrict__ kc,
                                bf16* __restrict__ vc, int T, int Hk, int D, int bs) {
  const long long total = static_cast<long long>(T) * Hk * (D / 8);
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(e % (D / 8)) * 8;
    const long long th = e / (D / 8);
    const int h = static_cast<int>(th % Hk), t = static_cast<int>(th / Hk);
    const int s = seq_of_token[t], p = pos[t];
    const int blk = block_table[static_cast<long long>(s) * max_blocks + p / bs];
    const long long dst = ((static_cast<long long>(blk) * Hk + h) * bs + (p % bs)) * D + c;
    const bf16* row = qkv + static_cast<long long>(t) * ld;
    *reinterpret_cast<uint4*>(kc + dst) = *reinterpret_cast<const uint4*>(row + k_off + h * D + c);
    *reinterpret_cast<uint4*>(vc + dst) = *reinterpret_cast<const uint4*>(row + v_off + h * D + c);
  }
}

// ------------------------------------------------------------------ decode attention
// One CTA per (sequence, kv head): the G = Hq / Hk query heads of the group
// share each K/V block load.  Warps take cache positions round-robin, keep an
// online softmax per query head, and merge through shared memory.
// D = 128: each lane owns 4 dims.
template <int G>
__global__ void __launch_bounds__(128) decode_attn_kernel(const bf16* __restrict__ q, long long ldq,
                                                         const bf16* __restrict__ kc, const bf16* __restrict__ vc,
                                                         const int* __restrict__ block_table, int max_blocks,
                                                         const int* __restrict__ ctx_len, bf16* __restrict__ out,
                                                         long long ldo, int Hk, int bs, float scale) {
  constexpr int D = 128, NW = 4;
  const int s = blockIdx.x / Hk, hk = blockIdx.x % Hk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = ctx_len[s];
  float qv[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const bf16* qp = q + static_cast<long long>(s) * ldq + static_cast<long long>(hk * G + g) * D + lane * 4;
    const uint2 u = *reinterpret_cast<const uint2*>(qp);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    qv[g][0] = a.x * scale;
    qv[g][1] = a.y * scale;
    qv[g][2] = b.x * scale;
    qv[g][3] = b.y * scale;
  }
  float m[G], l[G], acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[g][i] = 0.f;
  }
  const int* bt = block_table + static_cast<long long>(s) * max_blocks;
  for (int p = warp; p < L; p += NW) {
    const int blk = bt[p / bs];
    const long long off = ((static_cast<long long>(blk) * Hk + hk) * bs + (p % bs)) * D + lane * 4;
    const uint2 ku = *reinterpret_cast<const uint2*>(kc + off);
    const uint2 vu = *reinterpret_cast<const uint2*>(vc + off);
    const __nv_bfloat162* kh = reinterpret_cast<const __nv_bfloat162*>(&ku);
    const __nv_bfloat162* vh = reinterpret_cast<const __nv_bfloat162*>(&vu);
    const float2 k0 = __bfloat1622float2(kh[0]), k1 = __bfloat1622float2(kh[1]);
    const float2 v0 = __bfloat1622float2(vh[0]), v1 = __bfloat1622float2(vh[1]);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float sc = qv[g][0] * k0.x + qv[g][1] * k0.y + qv[g][2] * k1.x + qv[g][3] * k1.y;
      sc = tb::warp_sum(sc);
      const float mn = fmaxf(m[g], sc);
      const float corr = __expf(m[g] - mn), pw = __expf(sc - mn);
      l[g] = l[g] * corr + pw;
      acc[g][0] = acc[g][0] * corr + pw * v0.x;
      acc[g][1] = acc[g][1] * corr + pw * v0.y;
      acc[g][2] = acc[g][2] * corr + pw * v1.x;
      acc[g][3] = acc[g][3] * corr + pw * v1.y;
      m[g] = mn;
    }
  }
  __shared__ float sm[NW][G], sl[NW][G], sacc[NW][G][D];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      sm[warp][g] = m[g];
      sl[warp][g] = l[g];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) sacc[warp][g][lane * 4 + i] = acc[g][i];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int g = e / D, d = e % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, sm[w][g]);
    float Lsum = 0.f, o = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      if (sm[w][g] == -INFINITY) continue;
      const float c = __expf(sm[w][g] - M);
      Lsum += sl[w][g] * c;
      o += sacc[w][g][d] * c;
    }
    out[static_cast<long long>(s) * ldo + static_cast<long long>(hk * G + g) * D + d] =
        __float2bfloat16_rn(Lsum > 0.f ? o / Lsum : 0.f);
  }
}

// ------------------------------------------------------------------ sampling
// One CTA per row of logits [B, V] (bf16): token = argmax(logit/T + Gumbel)
// with Philox noise keyed by (seed, row, step); also returns the token's
// log-probability under softmax(logit / T).  temperature <= 0: greedy.
__global__ void __launch_bounds__(1024) sample_kernel(const bf16* __restrict__ logits, long long ld, int V,
                                                     float temperature, unsigned long long seed,
                                                     const long long* __restrict__ step_ptr, long long step_imm,
                                                     int* __restrict__ out_tok, float* __restrict__ out_logp,
                                                     int* __restrict__ tok_mat, float* __restrict__ lp_mat,
                                                     int ld_mat) {
  const int row = blockIdx.x;
  const bf16* x = logits + static_cast<long long>(row) * ld;
  const float inv_t = temperature > 0.f ? 1.f / temperature : 1.f;
  const bool greedy = temperature <= 0.f;
  const long long step = step_ptr ? *step_ptr : step_imm;
  float mx = -INFINITY, best = -INFINITY;
  int best_i = 0;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float z = bf(x[i]) * inv_t;
    mx = fmaxf(mx, z);
    float key = z;
    if (!greedy) {
      const uint4 r = tb::Philox::gen(seed, static_cast<uint32_t>(i), static_cast<uint32_t>(row),
                                      static_cast<uint32_t>(step), static_cast<uint32_t>(step >> 32));
      key = z - __logf(-__logf(tb::u01_open(r.x)));
    }
    if (key > best) {
      best = key;
      best_i = i;
    }
  }
  __shared__ float s_m[32], s_b[32];
  __shared__ int s_i[32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (ob > best || (ob == best && oi < best_i)) {
      best = ob;
      best_i = oi;
    }
  }
  if (lane == 0) {
    s_m[w] = mx;
    s_b[w] = best;
    s_i[w] = best_i;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    mx = lane < nw ? s_m[lane] : -INFINITY;
    best = lane < nw ? s_b[lane] : -INFINITY;
    best_i = lane < nw ? s_i[lane] : 0;
    for (int o = 16; o > 0; o >>= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (ob > best || (ob == best && oi < best_i)) {
        best = ob;
        best_i = oi;
      }
    }
    if (lane == 0) {
      s_m[0] = mx;
      s_i[0] = best_i;
    }
  }
  __syncthreads();
  mx = s_m[0];
  float se = 0.f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) se += __expf(bf(x[i]) * inv_t - mx);
  __shared__ float s_red[32];
  se = tb::block_sum(se, s_red);
  if (threadIdx.x == 0) {
    const int tok = s_i[0];
    const float lp = bf(x[tok]) * inv_t - (mx + __logf(se));
    out_tok[row] = tok;
    if (out_logp) out_logp[row] = lp;
    // generation matrices [B, ld_mat]: column = the decode step (device counter)
    if (tok_mat && step >= 0 && step < ld_mat) tok_mat[static_cast<long long>(row) * ld_mat + step] = tok;
    if (lp_mat && step >= 0 && step < ld_mat) lp_mat[static_cast<long long>(row) * ld_mat + step] = lp;
  }
}

// ------------------------------------------------------------------ LM-head log-probs
// One CTA per token row of logits [T, V]: logp[t] = z[target] - lse(z).
// With dlogp (the loss gradient w.r.t. logp[t]) the row is overwritten in place
// by d loss / d logits = dlogp[t] * (onehot(target) - softmax(z)).
__global__ void __launch_bounds__(1024) logprob_kernel(bf16* __restrict__ logits, long long ld, int V,
                                                      const int* __restrict__ target, float* __restrict__ logp,
                                                      const float* __restrict__ dlogp, float inv_temp) {
  const int row = blockIdx.x;
  bf16* x = logits + static_cast<long long>(row) * ld;
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float z = bf(x[i]) * inv_temp;
    if (z > m) {
      s = s * __expf(m - z) + 1.f;
      m = z;
    } else {
      s += __expf(z - m);
    }
  }
  // merge (m, s) pairs across the block
  __shared__ float sm[32], ss[32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
    m = nm;
  }
  if (lane == 0) {
    sm[w] = m;
    ss[w] = s;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? sm[lane] : -INFINITY;
    s = lane < nw ? ss[lane] : 0.f;
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
      const float nm = fmaxf(m, om);
      s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
      m = nm;
    }
    if (lane == 0) {
      sm[0] = m;
      ss[0] = s;
    }
  }
  __syncthreads();
  const float lse = sm[0] + __logf(ss[0]);
  const int tgt = target[row];
  const float zt = (tgt >= 0 && tgt < V) ? bf(x[tgt]) * inv_temp : 0.f;
  __syncthreads();
  if (threadIdx.x == 0 && logp) logp[row] = zt - lse;
  if (dlogp != nullptr) {
    const float g = dlogp[row];
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float p = __expf(bf(x[i]) * inv_temp - lse);
      x[i] = __float2bfloat16_rn(g * inv_temp * ((i == tgt ? 1.f : 0.f) - p));
    }
  }
}

// ------------------------------------------------------------------ GRPO loss
// Per token t of sequence b (mask > 0 marks response tokens):
//   r = exp(lp - old), pg = -min(r A_b, clip(r) A_b), kl = exp(ref - lp) - (ref - lp) - 1
//   loss = (1/B) sum_b (1/n_b) sum_t (pg + beta kl)
// dlp = d loss / d lp; stats += [pg sum, kl sum, clipped tokens, tokens].
__global__ void grpo_loss_kernel(const float* __restrict__ lp, const float* __restrict__ old_lp,
                                 const float* __restrict__ ref_lp, const float* __restrict__ adv,
                                 const float* __restrict__ mask, float* __restrict__ dlp, float* __restrict__ stats,
                                 int B, int T, float clip, float beta, float inv_total_seqs) {
  const int b = blockIdx.x;
  __shared__ float red[32];
  float cnt = 0.f;
  for (int t = threadIdx.x; t < T; t += blockDim.x) cnt += mask[static_cast<long long>(b) * T + t] > 0.f ? 1.f : 0.f;
  cnt = tb::block_sum(cnt, red);
  const float inv_n = cnt > 0.f ? 1.f / cnt : 0.f;
  const float A = adv[b];
  float s_pg = 0.f, s_kl = 0.f, s_cf = 0.f;
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    const long long o = static_cast<long long>(b) * T + t;
    if (!(mask[o] > 0.f)) {
      dlp[o] = 0.f;
      continue;
    }
    const float l = lp[o];
    const float lr = l - old_lp[o];
    const float r = __expf(lr);
    const float un = r * A, cl = fminf(fmaxf(r, 1.f - clip), 1.f + clip) * A;
    const bool use_un = un <= cl || (r > 1.f - clip && r < 1.f + clip);
    const float d = ref_lp ? ref_lp[o] - l : 0.f;
    const float ed = __expf(d);
    const float g_pg = use_un ? -A * r : 0.f;
    const float g_kl = ref_lp ? beta * (1.f - ed) : 0.f;
    dlp[o] = (g_pg + g_kl) * inv_n * inv_total_seqs;
    s_pg += -fminf(un, cl);
    s_kl += ref_lp ? (ed - d - 1.f) : 0.f;
    s_cf += fabsf(r - 1.f) > clip ? 1.f : 0.f;
  }
  if (stats) {
    s_pg = tb::block_sum(s_pg, red);
    s_kl = tb::block_sum(s_kl, red);
    s_cf = tb::block_sum(s_cf, red);
    if (threadIdx.x == 0) {
      atomicAdd(&stats[0], s_pg * inv_n * inv_total_seqs);
      atomicAdd(&stats[1], s_kl * inv_n * inv_total_seqs);
      atomicAdd(&stats[2], s_cf);
      atomicAdd(&stats[3], cnt);
    }
  }
}

inline unsigned grid_for(long long work, int block = 256) {
  long long g = (work + block - 1) / block;
  if (g > 148 * 16) g = 148 * 16;
  return static_cast<unsigned>(g < 1 ? 1 : g);
}

}  // namespace

extern "C" {

int tb_rmsnorm_fwd(const void* x, const float* w, void* y, float* rstd, int T, int D, float eps, cudaStream_t s) {
  if (T <= 0) return 0;
  if (D % 256) return static_cast<int>(cudaErrorInvalidValue);
  rmsnorm_fwd_kernel<<<(T + 7) / 8, 256, 0, s>>>(static_cast<const bf16*>(x), w, static_cast<bf16*>(y), rstd, T, D,
                                                  eps);
  return static_cast<int>(cudaGetLastError());
}

int tb_rmsnorm_bwd(const void* dy, const void* x, const float* w, const float* rstd, void* dx, const void* dx_add,
                   float* dw, int T, int D, cudaStream_t s) {
  if (T <= 0) return 0;
  if (D % 256 || D > 8192) return static_cast<int>(cudaErrorInvalidValue);
  const int rpb = 64;
  const unsigned g = (T + rpb - 1) / rpb;
  auto* a = static_cast<const bf16*>(dy);
  auto* b = static_cast<const bf16*>(x);
  auto* o = static_cast<bf16*>(dx);
  auto* ad = static_cast<const bf16*>(dx_add);
  if (D <= 2048)
    rmsnorm_bwd_kernel<64><<<g, 256, 0, s>>>(a, b, w, rstd, o, ad, dw, T, D, rpb);
  else if (D <= 4096)
    rmsnorm_bwd_kernel<128><<<g, 256, 0, s>>>(a, b, w, rstd, o, ad, dw, T, D, rpb);
  else
    rmsnorm_bwd_kernel<256><<<g, 256, 0, s>>>(a, b, w, rstd, o, ad, dw, T, D, rpb);
  return static_cast<int>(cudaGetLastError());
}

int tb_rope(void* qkv, long long ld, const int* pos, const void* table, int T, int n_rot_heads, int D, int inverse,
            cudaStream_t s) {
  if (T <= 0) return 0;
  if (D % 8) return static_cast<int>(cudaErrorInvalidValue);
  const long long work = static_cast<long long>(T) * n_rot_heads * (D / 8);
  rope_kernel<<<grid_for(work), 256, 0, s>>>(static_cast<bf16*>(qkv), ld, pos, static_cast<const float2*>(table), T,
                                             n_rot_heads, D, inverse ? -1.f : 1.f);
  return static_cast<int>(cudaGetLastError());
}

int tb_embed_fwd(const int* ids, const void* W, void* out, int T, int D, int V, int* err, cudaStream_t s) {
  if (T <= 0) return 0;
  if (D % 8) return static_cast<int>(cudaErrorInvalidValue);
  embed_fwd_kernel<<<grid_for(static_cast<long long>(T) * D / 8), 256, 0, s>>>(
      ids, static_cast<const bf16*>(W), static_cast<bf16*>(out), T, D, V, err);
  return static_cast<int>(cudaGetLastError());
}

int tb_embed_bwd(const int* ids, const void* dout, float* dW, int T, int D, int V, cudaStream_t s) {
  if (T <= 0) return 0;
  embed_bwd_kernel<<<grid_for(static_cast<long long>(T) * D / 8), 256, 0, s>>>(ids, static_cast<const bf16*>(dout), dW,
                                                                               T, D, V);
  return static_cast<int>(cudaGetLastError());
}

int tb_swiglu_bwd(const void* gu, const void* dh, void* dgu, long long T, int F, cudaStream_t s) {
  if (T <= 0) return 0;
  if (F % 4) return static_cast<int>(cudaErrorInvalidValue);
  swiglu_bwd_kernel<<<grid_for(T * F / 4), 256, 0, s>>>(static_cast<const bf16*>(gu), static_cast<const bf16*>(dh),
                                                        static_cast<bf16*>(dgu), T, F);
  return static_cast<int>(cudaGetLastError());
}

int tb_swiglu_fwd(const void* gu, void* act, long long T, int F, cudaStream_t s) {
  if (T <= 0) return 0;
  if (F % 4) return static_cast<int>(cudaErrorInvalidValue);
  swiglu_fwd_kernel<<<grid_for(T * F / 4), 256, 0, s>>>(static_cast<const bf16*>(gu), static_cast<bf16*>(act), T, F);
  return static_cast<int>(cudaGetLastError());
}

int tb_kv_write(const void* qkv, long long ld, int k_off, int v_off, const int* seq_of_token, const int* pos,
                const int* block_table, int max_blocks, void* kc, void* vc, int T, int Hk, int D, int bs,
                cudaStream_t s) {
  if (T <= 0) return 0;
  kv_write_kernel<<<grid_for(static_cast<long long>(T) * Hk * D / 8), 256, 0, s>>>(
      static_cast<const bf16*>(qkv), ld, k_off, v_off, seq_of_token, pos, block_table, max_blocks,
      static_cast<bf16*>(kc), static_cast<bf16*>(vc), T, Hk, D, bs);
  return static_cast<int>(cudaGetLastError());
}

int tb_decode_attention(const void* q, long long ldq, const void* kc, const void* vc, const int* block_table,
                        int max_blocks, const int* ctx_len, void* out, long long ldo, int B, int Hq, int Hk, int D,
                        int bs, float scale, cudaStream_t s) {
  if (B <= 0) return 0;
  if (D != 128 || Hq % Hk) return static_cast<int>(cudaErrorInvalidValue);
  const int G = Hq / Hk;
  const dim3 grid(B * Hk);
  auto* qq = static_cast<const bf16*>(q);
  auto* k = static_cast<const bf16*>(kc);
  auto* v = static_cast<const bf16*>(vc);
  auto* o = static_cast<bf16*>(out);
  switch (G) {
    case 1: decode_attn_kernel<1><<<grid, 128, 0, s>>>(qq, ldq, k, v, block_table, max_blocks, ctx_len, o, ldo, Hk, bs, scale); break;
    case 2: decode_attn_kernel<2><<<grid, 128, 0, s>>>(qq, ldq, k, v, block_table, max_blocks, ctx_len, o, ldo, Hk, bs, scale); break;
    case 4: decode_attn_kernel<4><<<grid, 128, 0, s>>>(qq, ldq, k, v, block_table, max_blocks, ctx_len, o, ldo, Hk, bs, scale); break;
    case 6: decode_attn_kernel<6><<<grid, 128, 0, s>>>(qq, ldq, k, v, block_table, max_blocks, ctx_len, o, ldo, Hk, bs, scale); break;
    case 8: decode_attn_kernel<8><<<grid, 128, 0, s>>>(qq, ldq, k, v, block_table, max_blocks, ctx_len, o, ldo, Hk, bs, scale); break;
    default: return static_cast<int>(cudaErrorInvalidValue);
  }
  return static_cast<int>(cudaGetLastError());
}

int tb_sample(const void* logits, long long ld, int B, int V, float temperature, unsigned long long seed,
              const long long* step_ptr, long long step_imm, int* out_tok, float* out_logp, int* tok_mat,
              float* lp_mat, int ld_mat, cudaStream_t s) {
  if (B <= 0) return 0;
  sample_kernel<<<B, 1024, 0, s>>>(static_cast<const bf16*>(logits), ld, V, temperature, seed, step_ptr, step_imm,
                                    out_tok, out_logp, tok_mat, lp_mat, ld_mat);
  return static_cast<int>(cudaGetLastError());
}

int tb_logprob(void* logits, long long ld, int T, int V, const int* target, float* logp, const float* dlogp,
               float inv_temp, cudaStream_t s) {
  if (T <= 0) return 0;
  logprob_kernel<<<T, 1024, 0, s>>>(static_cast<bf16*>(logits), ld, V, target, logp, dlogp, inv_temp);
  return static_cast<int>(cudaGetLastError());
}

int tb_grpo_loss(const float* lp, const float* old_lp, const float* ref_lp, const float* adv, const float* mask,
                 float* dlp, float* stats, int B, int T, float clip, float beta, float inv_total_seqs,
                 cudaStream_t s) {
  if (B <= 0) return 0;
  grpo_loss_kernel<<<B, 256, 0, s>>>(lp, old_lp, ref_lp, adv, mask, dlp, stats, B, T, clip, beta, inv_total_seqs);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
