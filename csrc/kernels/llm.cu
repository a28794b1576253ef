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
#include "pdl.cuh"

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
  tb::pdl_wait();
  tb::pdl_trigger();
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
                                   float* __restrict__ part, int T, int D, int rows_per_block) {
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
  // weight gradient: the block's warps combine in shared memory, then one
  // global atomic per column per block (not per warp)
  __shared__ float sdw[MAXV * 32];
  for (int c = threadIdx.x; c < D; c += blockDim.x) sdw[c] = 0.f;
  __syncthreads();
#pragma unroll
  for (int s = 0; s < MAXV / 8; ++s) {
    const int c = s * 256 + lane * 8;
    if (c < D) {
#pragma unroll
      for (int i = 0; i < 8; ++i) atomicAdd(sdw + c + i, dwp[s * 8 + i]);
    }
  }
  __syncthreads();
  if (part) {  // one partial row per block, summed by rms_parts_add_kernel (no contended atomics)
    for (int c = threadIdx.x; c < D; c += blockDim.x) part[static_cast<long long>(blockIdx.x) * D + c] = sdw[c];
  } else {
    for (int c = threadIdx.x; c < D; c += blockDim.x) atomicAdd(dw + c, sdw[c]);
  }
}

// dw[c] += sum over `parts` block partials [parts, D]: 32 columns per CTA, 32
// thread groups each summing every 32nd partial, then a shared-memory fold.
__global__ void __launch_bounds__(1024) rms_parts_add_kernel(const float* __restrict__ part, int parts, int D,
                                                             float* __restrict__ dw) {
  __shared__ float sm[32][33];
  const int ci = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + ci;
  float s = 0.f;
  if (c < D)
    for (int b = g; b < parts; b += 32) s += part[static_cast<long long>(b) * D + c];
  sm[g][ci] = s;
  __syncthreads();
  if (g == 0 && c < D) {
    float t = 0.f;
    for (int q = 0; q < 32; ++q) t += sm[q][ci];
    dw[c] += t;
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
  tb::pdl_wait();
  tb::pdl_trigger();
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

// RoPE on the q and k heads of fused QKV rows (in place) and the paged-cache
// write of the rotated k and of v, in one pass (the decode step's pair of
// rope_kernel + kv_write_kernel).  Per token: (Hq + Hk) x D/8 rotation items
// (4 rotated pairs each; k items also store their 8 values into the cache)
// and Hk x D/8 v-copy items.
__global__ void rope_kv_write_kernel(bf16* __restrict__ qkv, long long ld, const int* __restrict__ pos,
                                     const float2* __restrict__ table, int Hq, int Hk, int D,
                                     const int* __restrict__ seq_of_token, const int* __restrict__ block_table,
                                     int max_blocks, bf16* __restrict__ kc, bf16* __restrict__ vc, int T, int bs) {
  tb::pdl_wait();
  tb::pdl_trigger();
  const int half = D / 2, q4 = half / 4;
  const long long rot = static_cast<long long>(Hq + Hk) * q4, per_tok = rot + static_cast<long long>(Hk) * (D / 8);
  const long long total = static_cast<long long>(T) * per_tok;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(e / per_tok);
    const long long r = e - static_cast<long long>(t) * per_tok;
    const int p = pos[t];
    bf16* row = qkv + static_cast<long long>(t) * ld;
    auto slot = [&](int kh) {
      const int blk = block_table[static_cast<long long>(seq_of_token[t]) * max_blocks + p / bs];
      return ((static_cast<long long>(blk) * Hk + kh) * bs + (p % bs)) * D;
    };
    if (r < rot) {
      const int h = static_cast<int>(r / q4), j = static_cast<int>(r % q4) * 4;
      bf16* base = row + static_cast<long long>(h) * D;
      const float2* tab = table + static_cast<long long>(p) * half;
      __align__(8) bf16 lo[4], hi[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 cs = tab[j + k];
        const float x1 = bf(base[j + k]), x2 = bf(base[j + k + half]);
        lo[k] = __float2bfloat16_rn(x1 * cs.x - x2 * cs.y);
        hi[k] = __float2bfloat16_rn(x2 * cs.x + x1 * cs.y);
        base[j + k] = lo[k];
        base[j + k + half] = hi[k];
      }
      if (h >= Hq) {
        bf16* dst = kc + slot(h - Hq);
        *reinterpret_cast<uint2*>(dst + j) = *reinterpret_cast<const uint2*>(lo);
        *reinterpret_cast<uint2*>(dst + j + half) = *reinterpret_cast<const uint2*>(hi);
      }
    } else {
      const long long v = r - rot;
      const int kh = static_cast<int>(v / (D / 8)), c = static_cast<int>(v % (D / 8)) * 8;
      *reinterpret_cast<uint4*>(vc + slot(kh) + c) =
          *reinterpret_cast<const uint4*>(row + static_cast<long long>(Hq + Hk) * D + kh * D + c);
    }
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

// Tensor-core decode attention (block_size 16, head_dim 128).  CTA = (sequence,
// kv head); the G query heads of the group are the rows of a 16-row MMA tile
// (rows >= G are zero).  Warp w walks KV blocks w, w+4, ...: each 16-token K
// and V block is staged into the warp's shared memory with cp.async (double
// buffered), S = Q K^T and O += P V run as bf16 mma.sync m16n8k16, the online
// softmax runs on the accumulator fragments, and the four warps merge their
// (max, sum, O) partials at the end.
namespace dtc {
__device__ __forceinline__ uint32_t saddr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ int swz(int row, int chunk) { return row * 256 + ((chunk ^ (row & 7)) << 4); }
__device__ __forceinline__ void mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack(float x, float y) {
  __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&h);
}
// 16 token rows x 128 dims of one KV block -> swizzled smem tile (8 x 16 B per lane)
__device__ __forceinline__ void stage(uint8_t* tile, const bf16* src, int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane + 32 * i, r = e >> 4, c = e & 15;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr(tile + swz(r, c))), "l"(src + r * 128 + c * 8)
                 : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}
}  // namespace dtc

constexpr int kDecTcSmem = 4 * 2 * 2 * 16 * 256;  // warps x stages x {K, V} x 16 tokens x 256 B

__global__ void __launch_bounds__(128) decode_attn_tc_kernel(const bf16* __restrict__ q, long long ldq,
                                                            const bf16* __restrict__ kc, const bf16* __restrict__ vc,
                                                            const int* __restrict__ block_table, int max_blocks,
                                                            const int* __restrict__ ctx_len, bf16* __restrict__ out,
                                                            long long ldo, int Hk, int G, float scale, int n_split,
                                                            float* __restrict__ part, int* __restrict__ counters) {
  tb::pdl_wait();
  tb::pdl_trigger();
  constexpr int D = 128, BS = 16, NW = 4;
  extern __shared__ __align__(128) uint8_t dyn_smem[];
  auto sKV = reinterpret_cast<uint8_t(*)[2][2][BS * 256]>(dyn_smem);  // [warp][stage][K/V]
  // after the main loop the staging area is reused for the partial outputs
  auto sm_o = reinterpret_cast<float(*)[16][D + 4]>(dyn_smem);
  __shared__ float sm_m[NW][16], sm_l[NW][16];
  // context split: CTA (sequence, kv head, chunk c) takes blocks [c nblk / n_split, (c + 1) nblk / n_split)
  const int c_split = blockIdx.x % n_split, sh = blockIdx.x / n_split;
  const int s = sh / Hk, hk = sh % Hk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const int L = ctx_len[s];
  const int nblk = (L + BS - 1) / BS;
  // Q fragments for the G query heads (rows g < G), pre-scaled into log2 units
  const float qs = scale * 1.4426950408889634f;
  uint32_t qa[8][4];
  const bf16* qrow = q + static_cast<long long>(s) * ldq + static_cast<long long>(hk * G + g) * D;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    uint32_t lo = 0u, hi = 0u;
    if (g < G) {
      const __nv_bfloat162 x0 = *reinterpret_cast<const __nv_bfloat162*>(qrow + kk * 16 + 2 * t4);
      const __nv_bfloat162 x1 = *reinterpret_cast<const __nv_bfloat162*>(qrow + kk * 16 + 8 + 2 * t4);
      const float2 f0 = __bfloat1622float2(x0), f1 = __bfloat1622float2(x1);
      lo = dtc::pack(f0.x * qs, f0.y * qs);
      hi = dtc::pack(f1.x * qs, f1.y * qs);
    }
    qa[kk][0] = lo;
    qa[kk][1] = 0u;  // rows g + 8 >= 8 >= G: padding
    qa[kk][2] = hi;
    qa[kk][3] = 0u;
  }
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m = -INFINITY, l = 0.f;
  const int* bt = block_table + static_cast<long long>(s) * max_blocks;
  auto src_k = [&](int j) { return kc + (static_cast<long long>(bt[j]) * Hk + hk) * BS * D; };
  auto src_v = [&](int j) { return vc + (static_cast<long long>(bt[j]) * Hk + hk) * BS * D; };
  const int jb0 = static_cast<int>(static_cast<long long>(c_split) * nblk / n_split);
  const int jb1 = static_cast<int>(static_cast<long long>(c_split + 1) * nblk / n_split);
  int st = 0;
  if (jb0 + warp < jb1) {
    dtc::stage(sKV[warp][0][0], src_k(jb0 + warp), lane);
    dtc::stage(sKV[warp][0][1], src_v(jb0 + warp), lane);
  }
  for (int j = jb0 + warp; j < jb1; j += NW) {
    const int jn = j + NW;
    if (jn < jb1) {
      dtc::stage(sKV[warp][st ^ 1][0], src_k(jn), lane);
      dtc::stage(sKV[warp][st ^ 1][1], src_v(jn), lane);
      asm volatile("cp.async.wait_group 2;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncwarp();
    const uint8_t* tk = sKV[warp][st][0];
    const uint8_t* tv = sKV[warp][st][1];
    if ((j + 1) * BS > L) {
      // slots past the context hold stale (possibly non-finite) values: zero
      // their V rows so that p = 0 contributes exactly 0 (K rows are masked below)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int e = lane + 32 * i, r = e >> 4, c = e & 15;
        if (j * BS + r >= L) *reinterpret_cast<uint4*>(sKV[warp][st][1] + dtc::swz(r, c)) = make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
    }
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t b[4];
      const int row = (lane & 7) + 8 * (lane >> 4);
      const int chunk = kk * 2 + ((lane >> 3) & 1);
      asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                   : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3])
                   : "r"(dtc::saddr(tk + dtc::swz(row, chunk))));
      dtc::mma(sc[0], qa[kk], b[0], b[1]);
      dtc::mma(sc[1], qa[kk], b[2], b[3]);
    }
    // row g of the tile: tokens n*8 + 2*t4 + {0,1}
    const int base = j * BS;
    float mx = m;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        if (base + n * 8 + 2 * t4 + e >= L) sc[n][e] = -INFINITY;
        mx = fmaxf(mx, sc[n][e]);
      }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float corr = (m == -INFINITY) ? 0.f : exp2f(m - mx);
    float p[2][2], rs = 0.f;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        p[n][e] = sc[n][e] == -INFINITY ? 0.f : exp2f(sc[n][e] - mx);
        rs += p[n][e];
      }
    l = l * corr + rs;
    m = mx;
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      o[d][0] *= corr;
      o[d][1] *= corr;
    }
    const uint32_t pa[4] = {dtc::pack(p[0][0], p[0][1]), 0u, dtc::pack(p[1][0], p[1][1]), 0u};
#pragma unroll
    for (int d = 0; d < 16; d += 2) {
      uint32_t b[4];
      const int row = (lane & 7) + 8 * ((lane >> 3) & 1);
      const int chunk = d + (lane >> 4);
      asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                   : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3])
                   : "r"(dtc::saddr(tv + dtc::swz(row, chunk))));
      dtc::mma(o[d], pa, b[0], b[1]);
      dtc::mma(o[d + 1], pa, b[2], b[3]);
    }
    __syncwarp();
    st ^= 1;
  }
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  __syncthreads();  // every warp is done reading its staging tiles
  if (t4 == 0) {
    sm_m[warp][g] = m;
    sm_l[warp][g] = l;
  }
#pragma unroll
  for (int d = 0; d < 16; ++d) {
    sm_o[warp][g][d * 8 + 2 * t4] = o[d][0];
    sm_o[warp][g][d * 8 + 2 * t4 + 1] = o[d][1];
  }
  __syncthreads();
  // this CTA's chunk: partial [G][D + 2] = (unnormalized o, m in log2 units, l)
  float* mine = part ? part + (static_cast<long long>(sh) * n_split + c_split) * G * (D + 2) : nullptr;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int r = e / D, d = e % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, sm_m[w][r]);
    float Ls = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      if (sm_m[w][r] == -INFINITY) continue;
      const float c = exp2f(sm_m[w][r] - M);
      Ls += sm_l[w][r] * c;
      acc += sm_o[w][r][d] * c;
    }
    if (n_split == 1) {
      out[static_cast<long long>(s) * ldo + static_cast<long long>(hk * G + r) * D + d] =
          __float2bfloat16_rn(Ls > 0.f ? acc / Ls : 0.f);
    } else {
      mine[r * (D + 2) + d] = acc;
      if (d == 0) {
        mine[r * (D + 2) + D] = M;
        mine[r * (D + 2) + D + 1] = Ls;
      }
    }
  }
  if (n_split == 1) return;
  // the last chunk of (sequence, kv head) to finish merges the chunks (flash-decoding)
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(counters + sh, 1) == n_split - 1 ? 1 : 0;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float* all = part + static_cast<long long>(sh) * n_split * G * (D + 2);
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int r = e / D, d = e % D;
    float M = -INFINITY;
    for (int c = 0; c < n_split; ++c) M = fmaxf(M, __ldcg(all + (c * G + r) * (D + 2) + D));
    float Ls = 0.f, acc = 0.f;
    for (int c = 0; c < n_split; ++c) {
      const float* pc = all + (c * G + r) * (D + 2);
      const float mc = __ldcg(pc + D);
      if (mc == -INFINITY) continue;
      const float w = exp2f(mc - M);
      Ls += __ldcg(pc + D + 1) * w;
      acc += __ldcg(pc + d) * w;
    }
    out[static_cast<long long>(s) * ldo + static_cast<long long>(hk * G + r) * D + d] =
        __float2bfloat16_rn(Ls > 0.f ? acc / Ls : 0.f);
  }
  if (threadIdx.x == 0) counters[sh] = 0;  // ready for the next call (CUDA-graph replays)
}

// ------------------------------------------------------------------ sampling
// One CTA per row of logits [B, V] (bf16), temperature T (<= 0: greedy).
// Sampling is exact inverse-CDF sampling from softmax(logit / T), done with
// one exp per element:
//   pass 1  each thread keeps an online (max, sum of exp) over its elements
//           (16-byte loads of 8 logits, interleaved across threads) and the
//           argmax; the block combines them into the row max M and S.
//   pick    one Philox uniform u per (seed, row, step); the threads' scaled
//           sums, scanned in thread order, locate the thread whose elements
//           hold the quantile u * S; that thread re-walks its own elements
//           (the same order) to find the token.  Any fixed order of the
//           categories gives the same distribution.
// Also returns the token's log-probability z_tok / T - (M + log S), and with
// tok_mat / lp_mat writes both into column `step` (a device counter).
__device__ __forceinline__ void online_add(float& m, float& s, float z) {
  if (z > m) {
    s = s * __expf(m - z) + 1.f;
    m = z;
  } else if (z != -INFINITY) {
    s += __expf(z - m);
  }
}

__global__ void __launch_bounds__(1024) sample_kernel(const bf16* __restrict__ logits, long long ld, int V,
                                                     float temperature, unsigned long long seed,
                                                     const long long* __restrict__ step_ptr, long long step_imm,
                                                     int* __restrict__ out_tok, float* __restrict__ out_logp,
                                                     int* __restrict__ tok_mat, float* __restrict__ lp_mat,
                                                     int ld_mat, const unsigned long long* __restrict__ seed_ptr,
                                                     const float* __restrict__ temp_ptr) {
  const int row = blockIdx.x;
  const bf16* x = logits + static_cast<long long>(row) * ld;
  if (seed_ptr) seed = *seed_ptr;
  if (temp_ptr) temperature = *temp_ptr;
  const float inv_t = temperature > 0.f ? 1.f / temperature : 1.f;
  const bool greedy = temperature <= 0.f;
  const long long step = step_ptr ? *step_ptr : step_imm;
  const int tid = threadIdx.x, nt = blockDim.x;
  const bool vec = (V % 8 == 0) && (ld % 8 == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
  const int nv = vec ? V / 8 : 0;
  float m = -INFINITY, sm = 0.f, best = -INFINITY;
  int best_i = 0;
  for (int c = tid; c < nv; c += nt) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + c * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __bfloat1622float2(h[k]);
      const float z0 = f.x * inv_t, z1 = f.y * inv_t;
      if (z0 > best) { best = z0; best_i = c * 8 + 2 * k; }
      if (z1 > best) { best = z1; best_i = c * 8 + 2 * k + 1; }
      online_add(m, sm, z0);
      online_add(m, sm, z1);
    }
  }
  for (int i = nv * 8 + tid; i < V; i += nt) {
    const float z = bf(x[i]) * inv_t;
    if (z > best) { best = z; best_i = i; }
    online_add(m, sm, z);
  }
  // ---- block max / argmax, then the sum rescaled to the block max
  __shared__ float s_a[32], s_b[32];
  __shared__ int s_i[32];
  __shared__ float s_M, s_S, s_target;
  __shared__ int s_tok, s_owner;
  const int lane = tid & 31, w = tid >> 5, nw = nt >> 5;
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
    bm = lane < nw ? s_a[lane] : -INFINITY;
    bb = lane < nw ? s_b[lane] : -INFINITY;
    bi = lane < nw ? s_i[lane] : 0;
    for (int o = 16; o > 0; o >>= 1) {
      bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
      const float ob = __shfl_xor_sync(0xffffffffu, bb, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > bb || (ob == bb && oi < bi)) { bb = ob; bi = oi; }
    }
    if (lane == 0) { s_M = bm; s_tok = bi; }
  }
  __syncthreads();
  const float M = s_M;
  const float wt = (m == -INFINITY) ? 0.f : sm * __expf(m - M);  // this thread's share of S
  // inclusive scan of wt in thread order (warp scans + a scan of warp totals)
  float inc = wt;
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  __syncthreads();
  if (lane == 31) s_a[w] = inc;
  __syncthreads();
  if (w == 0) {
    float t = lane < nw ? s_a[lane] : 0.f;
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < nw) s_b[lane] = t;  // inclusive warp-total prefix
    if (lane == 31) {
      s_S = t;
      const uint4 r = tb::Philox::gen(seed, 0x53414D50u, static_cast<uint32_t>(row), static_cast<uint32_t>(step),
                                      static_cast<uint32_t>(step >> 32));
      s_target = tb::u01_open(r.x) * t;
      s_owner = -1;
    }
  }
  __syncthreads();
  const float S = s_S;
  if (!greedy) {
    const float excl = inc - wt + (w > 0 ? s_b[w - 1] : 0.f);
    const float target = s_target;
    // the owner: excl <= target < excl + wt; rounding past the end falls to the last thread with mass
    if (wt > 0.f && excl <= target && (target < excl + wt)) atomicMax(&s_owner, tid);
    __syncthreads();
    if (s_owner < 0) {
      if (wt > 0.f) atomicMax(&s_owner, tid);
      __syncthreads();
    }
    if (tid == s_owner) {
      float acc = excl;
      int tok = -1, last_i = -1;
      for (int c = tid; c < nv; c += nt) {
        const uint4 u = *reinterpret_cast<const uint4*>(x + c * 8);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __bfloat1622float2(h[k]);
          const float z0 = f.x * inv_t, z1 = f.y * inv_t;
          if (z0 != -INFINITY) { acc += __expf(z0 - M); last_i = c * 8 + 2 * k; if (tok < 0 && acc > target) tok = last_i; }
          if (z1 != -INFINITY) { acc += __expf(z1 - M); last_i = c * 8 + 2 * k + 1; if (tok < 0 && acc > target) tok = last_i; }
        }
      }
      for (int i = nv * 8 + tid; i < V; i += nt) {
        const float z = bf(x[i]) * inv_t;
        if (z != -INFINITY) { acc += __expf(z - M); last_i = i; if (tok < 0 && acc > target) tok = i; }
      }
      s_tok = tok >= 0 ? tok : last_i;
    }
    __syncthreads();
  }
  if (tid == 0) {
    const int tok = s_tok;
    const float lp = bf(x[tok]) * inv_t - (M + __logf(S));
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
  // 16-byte loads of 8 logits where the row allows it
  const bool vec = (V % 8 == 0) && (ld % 8 == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
  const int nv = vec ? V / 8 : 0;
  for (int c = threadIdx.x; c < nv; c += blockDim.x) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + c * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __bfloat1622float2(h[k]);
      online_add(m, s, f.x * inv_temp);
      online_add(m, s, f.y * inv_temp);
    }
  }
  for (int i = nv * 8 + threadIdx.x; i < V; i += blockDim.x) online_add(m, s, bf(x[i]) * inv_temp);
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
    for (int c = threadIdx.x; c < nv; c += blockDim.x) {
      uint4 u = *reinterpret_cast<const uint4*>(x + c * 8);
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]);
        const int i0 = c * 8 + 2 * k;
        const float p0 = __expf(f.x * inv_temp - lse), p1 = __expf(f.y * inv_temp - lse);
        h[k] = __floats2bfloat162_rn(g * inv_temp * ((i0 == tgt ? 1.f : 0.f) - p0),
                                     g * inv_temp * ((i0 + 1 == tgt ? 1.f : 0.f) - p1));
      }
      *reinterpret_cast<uint4*>(x + c * 8) = u;
    }
    for (int i = nv * 8 + threadIdx.x; i < V; i += blockDim.x) {
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

// Per-token clipped PPO loss of an RLHF policy with a value head, forward and
// backward in one pass over R tokens:
//   ratio = exp(lp - old_lp);  pg = -min(ratio A, clip(ratio, 1 -+ c) A)
//   v_c = old_v + clip(v - old_v, -+ vc);  vf = 0.5 max((v - ret)^2, (v_c - ret)^2)
//   loss = norm (sum pg + vf_coef sum vf)
// dlp / dv are d loss / d lp and d loss / d v (ties of min / max split the
// gradient evenly, clip passes it inside its range); stats += {sum pg * norm,
// sum vf * norm, tokens with |ratio - 1| > c, tokens}.
__global__ void ppo_token_loss_kernel(const float* __restrict__ lp, const float* __restrict__ old_lp,
                                      const float* __restrict__ adv, const float* __restrict__ v,
                                      const float* __restrict__ old_v, const float* __restrict__ ret,
                                      float* __restrict__ dlp, float* __restrict__ dv, float* __restrict__ stats,
                                      long long R, float clip, float vclip, float vf_coef, float norm) {
  __shared__ float red[32];
  float s_pg = 0.f, s_vf = 0.f, s_cf = 0.f, s_n = 0.f;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < R;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float A = adv[i];
    const float r = __expf(lp[i] - old_lp[i]);
    const float rc = fminf(fmaxf(r, 1.f - clip), 1.f + clip);
    const float un = r * A, cl = rc * A;
    const bool inside = r >= 1.f - clip && r <= 1.f + clip;
    // d(-min(un, cl))/d lp: the unclipped branch carries -A r, the clipped one -A r only inside the range
    const float g_un = -A * r, g_cl = inside ? -A * r : 0.f;
    const float g_pg = un < cl ? g_un : (un > cl ? g_cl : 0.5f * (g_un + g_cl));
    dlp[i] = g_pg * norm;
    const float vv = v[i], ov = old_v[i], rt = ret[i];
    const float dd = vv - ov;
    const float vc = ov + fminf(fmaxf(dd, -vclip), vclip);
    const float a = vv - rt, b = vc - rt;
    const float a2 = a * a, b2 = b * b;
    const float db = (dd >= -vclip && dd <= vclip) ? b : 0.f;  // d(0.5 b^2)/dv through the clip
    const float g_vf = a2 > b2 ? a : (b2 > a2 ? db : 0.5f * (a + db));
    dv[i] = vf_coef * g_vf * norm;
    s_pg += -fminf(un, cl);
    s_vf += 0.5f * fmaxf(a2, b2);
    s_cf += fabsf(r - 1.f) > clip ? 1.f : 0.f;
    s_n += 1.f;
  }
  if (stats) {
    s_pg = tb::block_sum(s_pg, red);
    s_vf = tb::block_sum(s_vf, red);
    s_cf = tb::block_sum(s_cf, red);
    s_n = tb::block_sum(s_n, red);
    if (threadIdx.x == 0) {
      atomicAdd(&stats[0], s_pg * norm);
      atomicAdd(&stats[1], s_vf * norm);
      atomicAdd(&stats[2], s_cf);
      atomicAdd(&stats[3], s_n);
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
  return static_cast<int>(tb::launch_pdl(rmsnorm_fwd_kernel, dim3((T + 7) / 8), dim3(256), 0, s,
                                         static_cast<const bf16*>(x), w, static_cast<bf16*>(y), rstd, T, D, eps));
}

size_t tb_rmsnorm_bwd_ws_floats(int D) { return static_cast<size_t>(2 * 148) * (D > 0 ? D : 0); }

int tb_rmsnorm_bwd(const void* dy, const void* x, const float* w, const float* rstd, void* dx, const void* dx_add,
                   float* dw, int T, int D, cudaStream_t s) {
  return tb_rmsnorm_bwd_ws(dy, x, w, rstd, dx, dx_add, dw, T, D, nullptr, 0, s);
}

int tb_rmsnorm_bwd_ws(const void* dy, const void* x, const float* w, const float* rstd, void* dx, const void* dx_add,
                      float* dw, int T, int D, float* ws, size_t ws_floats, cudaStream_t s) {
  if (T <= 0) return 0;
  if (D % 256 || D > 8192) return static_cast<int>(cudaErrorInvalidValue);
  // ~2 blocks per SM
  int rpb = (T + 2 * 148 - 1) / (2 * 148);
  if (rpb < 8) rpb = 8;
  const unsigned g = (T + rpb - 1) / rpb;
  float* part = (ws && static_cast<size_t>(g) * D <= ws_floats) ? ws : nullptr;
  auto* a = static_cast<const bf16*>(dy);
  auto* b = static_cast<const bf16*>(x);
  auto* o = static_cast<bf16*>(dx);
  auto* ad = static_cast<const bf16*>(dx_add);
  if (D <= 2048)
    rmsnorm_bwd_kernel<64><<<g, 256, 0, s>>>(a, b, w, rstd, o, ad, dw, part, T, D, rpb);
  else if (D <= 4096)
    rmsnorm_bwd_kernel<128><<<g, 256, 0, s>>>(a, b, w, rstd, o, ad, dw, part, T, D, rpb);
  else
    rmsnorm_bwd_kernel<256><<<g, 256, 0, s>>>(a, b, w, rstd, o, ad, dw, part, T, D, rpb);
  if (part) rms_parts_add_kernel<<<(D + 31) / 32, 1024, 0, s>>>(part, static_cast<int>(g), D, dw);
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
  return static_cast<int>(tb::launch_pdl(embed_fwd_kernel, dim3(grid_for(static_cast<long long>(T) * D / 8)), dim3(256),
                                         0, s, ids, static_cast<const bf16*>(W), static_cast<bf16*>(out), T, D, V, err));
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

int tb_rope_kv_write(void* qkv, long long ld, const int* pos, const void* table, int Hq, int Hk, int D,
                     const int* seq_of_token, const int* block_table, int max_blocks, void* kc, void* vc, int T, int bs,
                     cudaStream_t s) {
  if (T <= 0) return 0;
  if (D % 8 || ld % 8) return static_cast<int>(cudaErrorInvalidValue);
  const long long work = static_cast<long long>(T) * ((Hq + Hk) * (D / 8) + Hk * (D / 8));
  return static_cast<int>(tb::launch_pdl(rope_kv_write_kernel, dim3(grid_for(work)), dim3(256), 0, s,
                                         static_cast<bf16*>(qkv), ld, pos, static_cast<const float2*>(table), Hq, Hk,
                                         D, seq_of_token, block_table, max_blocks, static_cast<bf16*>(kc),
                                         static_cast<bf16*>(vc), T, bs));
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
  if (bs == 16 && G <= 8) {
    const cudaError_t e = tb::ensure_dyn_smem(reinterpret_cast<const void*>(decode_attn_tc_kernel), kDecTcSmem);
    if (e != cudaSuccess) return static_cast<int>(e);
    return static_cast<int>(tb::launch_pdl(decode_attn_tc_kernel, grid, dim3(128), kDecTcSmem, s, qq, ldq, k, v,
                                           block_table, max_blocks, ctx_len, o, ldo, Hk, G, scale, 1,
                                           static_cast<float*>(nullptr), static_cast<int*>(nullptr)));
  }
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

int tb_decode_attention_splits(int B, int Hk) {
  int dev = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (tb::ensure_dyn_smem(reinterpret_cast<const void*>(decode_attn_tc_kernel), kDecTcSmem) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_attn_tc_kernel, 128, kDecTcSmem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 3;
  if (sms <= 0) sms = 148;
  const long long slots = static_cast<long long>(sms) * per_sm, units = static_cast<long long>(B) * Hk;
  // waves x (1 / split) for a long context: the smallest wins, ties to fewer chunks
  int best = 1;
  double best_t = static_cast<double>((units + slots - 1) / slots);
  for (int sp = 2; sp <= 8; ++sp) {
    const double t = static_cast<double>((units * sp + slots - 1) / slots) / sp;
    if (t < best_t * 0.97) {
      best_t = t;
      best = sp;
    }
  }
  return best;
}

size_t tb_decode_attention_part_floats(int B, int Hq, int Hk, int n_split) {
  return static_cast<size_t>(B) * Hk * n_split * (Hq / Hk) * (128 + 2);
}

int tb_decode_attention_split(const void* q, long long ldq, const void* kc, const void* vc, const int* block_table,
                              int max_blocks, const int* ctx_len, void* out, long long ldo, int B, int Hq, int Hk,
                              int D, int bs, float scale, int n_split, float* part, int* counters, cudaStream_t s) {
  if (n_split <= 1)
    return tb_decode_attention(q, ldq, kc, vc, block_table, max_blocks, ctx_len, out, ldo, B, Hq, Hk, D, bs, scale, s);
  const int G = Hq / Hk;
  if (B <= 0) return 0;
  if (D != 128 || bs != 16 || G > 8 || Hq % Hk || part == nullptr || counters == nullptr)
    return static_cast<int>(cudaErrorInvalidValue);
  const cudaError_t e = tb::ensure_dyn_smem(reinterpret_cast<const void*>(decode_attn_tc_kernel), kDecTcSmem);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(tb::launch_pdl(decode_attn_tc_kernel, dim3(B * Hk * n_split), dim3(128), kDecTcSmem, s,
                                         static_cast<const bf16*>(q), ldq, static_cast<const bf16*>(kc),
                                         static_cast<const bf16*>(vc), block_table, max_blocks, ctx_len,
                                         static_cast<bf16*>(out), ldo, Hk, G, scale, n_split, part, counters));
}

int tb_sample(const void* logits, long long ld, int B, int V, float temperature, unsigned long long seed,
              const long long* step_ptr, long long step_imm, int* out_tok, float* out_logp, int* tok_mat,
              float* lp_mat, int ld_mat, const unsigned long long* seed_ptr, const float* temp_ptr,
              cudaStream_t s) {
  if (B <= 0) return 0;
  sample_kernel<<<B, 1024, 0, s>>>(static_cast<const bf16*>(logits), ld, V, temperature, seed, step_ptr, step_imm,
                                    out_tok, out_logp, tok_mat, lp_mat, ld_mat, seed_ptr, temp_ptr);
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

int tb_ppo_token_loss(const float* lp, const float* old_lp, const float* adv, const float* v, const float* old_v,
                      const float* ret, float* dlp, float* dv, float* stats, long long R, float clip, float vclip,
                      float vf_coef, float norm, cudaStream_t s) {
  if (R <= 0) return 0;
  ppo_token_loss_kernel<<<grid_for(R), 256, 0, s>>>(lp, old_lp, adv, v, old_v, ret, dlp, dv, stats, R, clip, vclip,
                                                     vf_coef, norm);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
