// Causal GQA flash-attention forward on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), sm_100a, bf16 in / bf16 out, head_dim 128.
//
// One CTA computes 128 query rows of one (sequence, query head) and walks the
// key/value tiles of 64 keys up to the diagonal:
//
//   S_j = Q K_j^T          tcgen05.mma M=128 N=64  K=128 -> TMEM (64 columns)
//   P_j = exp2(S_j - m)    softmax warpgroup, bf16 into a swizzled smem tile
//   O  += P_j V_j          tcgen05.mma M=128 N=128 K=64  -> TMEM (128 columns)
//
// Roles (256 threads):
//   warp 0      one thread issues the TMA loads: Q once (two 64-column boxes),
//               then K_0, V_0, K_1, V_1, ... through a ring of three 16 KB slots;
//   warp 1      one thread issues the MMAs and commits barriers;
//   warp 2      allocates / frees 256 TMEM columns (S at 0, O at 128);
//   warps 4-7   softmax and epilogue: thread r owns query row r = TMEM lane r.
//
// Online softmax with a lazily updated reference maximum: a row's reference
// max m only moves when a tile's max exceeds it by more than 8 (log2 units),
// so P stays <= 256 and the O accumulator in TMEM is rescaled (tcgen05.ld,
// multiply, tcgen05.st) only on those rare updates.  The final O / l and the
// log-sum-exp use the same m, so the result is exact either way.
//
// Two CTAs fit on an SM (96 KB of shared memory and 256 TMEM columns each), so
// one CTA's softmax overlaps the other's MMAs.  Every wait is bounded; on a
// timeout the CTA records error site 21, drains its own copies and MMAs, frees
// TMEM and returns.
//
// Operand layouts (128-byte swizzle, as TMA writes them):
//   Q  A operand, K-major: two atoms [128 rows x 64 d] of 16 KB.
//   K  B operand, K-major (N = keys): two atoms [64 keys x 64 d] of 8 KB.
//   V  B operand, MN-major (N = d contiguous): two 64-wide d blocks of
//      [64 keys x 128 B], 8 KB apart (the descriptor's leading offset).
//   P  A operand, K-major (K = keys): one atom [128 rows x 64 keys]; the
//      softmax threads write it with the same XOR swizzle TMA uses
//      (16-byte chunk c of row r at chunk c ^ (r & 7)).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <mutex>

#include "device_common.cuh"
#include "kernels.h"
#include "sm100_primitives.cuh"

namespace {

using namespace tb::sm100;
using bf16 = __nv_bfloat16;

constexpr int D = 128, BQ = 128, BKV = 64, kSlots = 3, kThreads = 256;
constexpr int kQBytes = BQ * D * 2;      // 32768
constexpr int kTileBytes = BKV * D * 2;  // 16384 (one K or V tile)
constexpr int kPBytes = BQ * BKV * 2;    // 16384
constexpr int kOffRing = kQBytes;
constexpr int kOffP = kOffRing + kSlots * kTileBytes;
constexpr int kOffBar = kOffP + kPBytes;
constexpr int kSmemBytes = kOffBar + 128 + 1024;  // + barriers, + alignment slack
constexpr uint32_t kTmemCols = 256, kTmemO = 128;
constexpr float kRescaleThreshold = 8.f;  // log2 units: P <= 2^8

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Ties registers written by tcgen05.ld to the preceding tcgen05.wait::ld, so
// that no use of them is scheduled before the wait.
template <int N>
__device__ __forceinline__ void after_wait(uint32_t* r) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Order in which the forward streams K/V tiles through the ring: K_0, then
// (K_{j+1}, V_j) for every j, so the scores of the next tile can be computed
// while the softmax of the current one runs.
__device__ __forceinline__ void fwd_tile_order(int i, int n, bool& is_v, int& j) {
  if (i == 0) {
    is_v = false;
    j = 0;
    return;
  }
  const int t = i - 1;
  j = t >> 1;
  is_v = (t & 1) || j + 1 >= n;
  if (!is_v) j += 1;
}

__global__ void __launch_bounds__(kThreads, 2)
    fa_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, bf16* __restrict__ ob, long long ldo,
                     float* __restrict__ lse, int T, int Hq, int Hk, float scale_log2, int n_qt, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;
  uint64_t* ring_full = bars + 1;   // [kSlots]
  uint64_t* ring_empty = bars + 4;  // [kSlots]
  uint64_t* s_full = bars + 7;  // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* p_empty = bars + 10;
  uint64_t* o_full = bars + 11;
  uint64_t* drain = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.x);  // the longest (last) query tiles first
  const int bh = blockIdx.y, b = bh / Hq, h = bh % Hq, hk = h / (Hq / Hk);
  const int q0 = qt * BQ;
  const int row_base = b * T;
  const int n_kv = (min(q0 + BQ, T) + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&ring_full[i], 1);
      mbar_init(&ring_empty[i], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_full, 4);
    mbar_init(p_empty, 1);
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch(&tmQ);
    tma_prefetch(&tmK);
    tma_prefetch(&tmV);
  }
  if (warp == 2) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------ TMA producer
    mbar_arrive_expect_tx(q_full, kQBytes);
    tma_load_2d(smem, &tmQ, q_full, h * D, row_base + q0);
    tma_load_2d(smem + kQBytes / 2, &tmQ, q_full, h * D + 64, row_base + q0);
    int issued = 0;
    for (int i = 0; i < 2 * n_kv && !*abort_flag; ++i) {
      const int slot = i % kSlots;
      const uint32_t ph = static_cast<uint32_t>(i / kSlots) & 1u;
      if (!mbar_wait(&ring_empty[slot], ph ^ 1u, abort_flag)) break;
      uint8_t* dst = smem + kOffRing + slot * kTileBytes;
      bool is_v;
      int jt;
      fwd_tile_order(i, n_kv, is_v, jt);
      const CUtensorMap* m = is_v ? &tmV : &tmK;
      const int y = row_base + jt * BKV;
      mbar_arrive_expect_tx(&ring_full[slot], kTileBytes);
      tma_load_2d(dst, m, &ring_full[slot], hk * D, y);
      tma_load_2d(dst + kTileBytes / 2, m, &ring_full[slot], hk * D + 64, y);
      ++issued;
    }
    if (*abort_flag) {
      // wait (bounded) for this CTA's copies still in flight before it exits
      const unsigned long long t0 = global_ns();
      while (!mbar_try_wait(q_full, 0) && global_ns() - t0 < 100000000ull) {
      }
      for (int i = issued - (issued < kSlots ? issued : kSlots); i < issued; ++i) {
        const unsigned long long t1 = global_ns();
        while (!mbar_try_wait(&ring_full[i % kSlots], static_cast<uint32_t>(i / kSlots) & 1u) &&
               global_ns() - t1 < 100000000ull) {
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------ MMA issuer
    constexpr uint32_t id_s = idesc_bf16(BQ, BKV, 0, 0);
    constexpr uint32_t id_o = idesc_bf16(BQ, D, 0, 1);
    const uint32_t t_s = tmem_base, t_o = tmem_base + kTmemO;
    const uint32_t sq = smem_u32(smem), sp = smem_u32(smem + kOffP);
    bool ok = mbar_wait(q_full, 0, abort_flag), any = false;
    if (ok) tc_fence_after();
    int ci = 0;  // ring tiles consumed, in the producer's order
    auto take = [&](uint32_t& saddr, int& slot) -> bool {
      slot = ci % kSlots;
      if (!mbar_wait(&ring_full[slot], static_cast<uint32_t>(ci / kSlots) & 1u, abort_flag)) return false;
      tc_fence_after();
      saddr = smem_u32(smem + kOffRing + slot * kTileBytes);
      ++ci;
      return true;
    };
    auto issue_s = [&](int j) -> bool {  // S_j = Q K_j^T into score buffer j & 1
      uint32_t sk;
      int slot;
      if (!take(sk, slot)) return false;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint64_t ad = smem_desc_sw128(sq + (kk >> 2) * (kQBytes / 2) + (kk & 3) * 32, 16, 1024);
        const uint64_t bd = smem_desc_sw128(sk + (kk >> 2) * (kTileBytes / 2) + (kk & 3) * 32, 16, 1024);
        mma_f16(t_s + 64 * (j & 1), ad, bd, id_s, kk > 0 ? 1u : 0u);
      }
      any = true;
      mma_commit(&ring_empty[slot]);
      mma_commit(&s_full[j & 1]);
      return true;
    };
    if (ok) ok = issue_s(0);
    for (int j = 0; ok && j < n_kv; ++j) {
      // the next tile's scores overlap this tile's softmax (its buffer was read by softmax j-1)
      if (j + 1 < n_kv && !issue_s(j + 1)) {
        ok = false;
        break;
      }
      // P_j written (and S_j read, O rescaled) by the softmax warpgroup
      if (!mbar_wait(p_full, static_cast<uint32_t>(j) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv;
      int slot;
      if (!take(sv, slot)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int kk = 0; kk < BKV / 16; ++kk) {
        const uint64_t ad = smem_desc_sw128(sp + kk * 32, 16, 1024);
        const uint64_t bd = smem_desc_sw128(sv + kk * 2048, kTileBytes / 2, 1024);
        mma_f16(t_o, ad, bd, id_o, (j > 0 || kk > 0) ? 1u : 0u);
      }
      mma_commit(&ring_empty[slot]);
      mma_commit(p_empty);
    }
    if (ok) mma_commit(o_full);
    if (any) {
      // every MMA this thread issued completes before TMEM is freed
      mma_commit(drain);
      const unsigned long long t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 1000000000ull) {
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ softmax + epilogue
    const int r = threadIdx.x - 128;  // TMEM lane == query row within the tile
    const int row = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem_base + lane_off, t_o = tmem_base + lane_off + kTmemO;
    uint8_t* prow = smem + kOffP + r * 128;
    const int sw = r & 7;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const uint32_t t_sj = t_s + 64 * (j & 1);
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[j & 1], static_cast<uint32_t>(j >> 1) & 1u, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const int k0 = j * BKV;
      const bool diag = k0 + BKV - 1 > q0;  // a key of this tile may lie past some row of the query tile
      // pass 1: the tile's row max (S is read twice from TMEM rather than held in registers)
      // (four independent max chains: one warp per SM sub-partition leaves little latency hiding)
      float mx[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) mx[e] = -INFINITY;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t sv[32];
        tmem_ld_x32(t_sj + half * 32, sv);
        tmem_wait_ld();
        after_wait<32>(sv);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          float x = __uint_as_float(sv[c]);
          if (diag && k0 + half * 32 + c > row) x = -INFINITY;
          mx[c & 3] = fmaxf(mx[c & 3], x);
        }
      }
      const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * scale_log2;
      const bool need = mt > m_ref + kRescaleThreshold;  // always true on the first tile (col 0 <= row)
      float alpha = 1.f;
      if (need) {
        alpha = ex2(m_ref - mt);  // 0 when m_ref is -inf
        m_ref = mt;
        l *= alpha;
      }
      if (j > 0) {
        // P_{j-1} V_{j-1} has finished reading the P tile and accumulating into O
        ok = __all_sync(0xffffffffu, mbar_wait(p_empty, static_cast<uint32_t>(j - 1) & 1u, abort_flag));
        if (!ok) break;
        tc_fence_after();
      }
      if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int cc = 0; cc < D / 32; ++cc) {
          uint32_t ov[32];
          tmem_ld_x32(t_o + cc * 32, ov);
          tmem_wait_ld();
          after_wait<32>(ov);
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
          tmem_st_x32(t_o + cc * 32, ov);
        }
        tmem_wait_st();
      }
      // pass 2: P = exp2(S - m) as bf16 into the swizzled P tile
      float sm[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t sv[32];
        tmem_ld_x32(t_sj + half * 32, sv);
        tmem_wait_ld();
        after_wait<32>(sv);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int col = half * 32 + 8 * c + 2 * e;
            float x0 = __uint_as_float(sv[8 * c + 2 * e]) * scale_log2 - m_ref;
            float x1 = __uint_as_float(sv[8 * c + 2 * e + 1]) * scale_log2 - m_ref;
            if (diag && k0 + col > row) x0 = -INFINITY;
            if (diag && k0 + col + 1 > row) x1 = -INFINITY;
            const float p0 = ex2(x0), p1 = ex2(x1);
            sm[e] += p0 + p1;
            w[e] = pack_bf16(p0, p1);
          }
          *reinterpret_cast<uint4*>(prow + (((half * 4 + c) ^ sw) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      l += (sm[0] + sm[1]) + (sm[2] + sm[3]);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(o_full, 0, abort_flag));
    if (ok) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      bf16* O = ob + static_cast<long long>(row_base + row) * ldo + h * D;
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t ov[32];
        tmem_ld_x32(t_o + cc * 32, ov);
        tmem_wait_ld();
        after_wait<32>(ov);
        if (row < T) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 u;
            u.x = pack_bf16(__uint_as_float(ov[8 * g + 0]) * inv, __uint_as_float(ov[8 * g + 1]) * inv);
            u.y = pack_bf16(__uint_as_float(ov[8 * g + 2]) * inv, __uint_as_float(ov[8 * g + 3]) * inv);
            u.z = pack_bf16(__uint_as_float(ov[8 * g + 4]) * inv, __uint_as_float(ov[8 * g + 5]) * inv);
            u.w = pack_bf16(__uint_as_float(ov[8 * g + 6]) * inv, __uint_as_float(ov[8 * g + 7]) * inv);
            *reinterpret_cast<uint4*>(O + cc * 32 + g * 8) = u;
          }
        }
      }
      if (lse != nullptr && row < T)
        lse[(static_cast<long long>(b) * Hq + h) * T + row] = (m_ref + __log2f(l)) * 0.6931471805599453f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag && err != nullptr) atomicCAS(err, 0, 21);
}

// ============================================================ backward
// Both passes run on the tensor cores with the same pattern: one MMA thread,
// one TMA thread, 8 elementwise warps (two per TMEM lane quarter, each owning
// 32 of the 64 columns of a score tile), score tiles double-buffered in TMEM
// so the MMAs of step s+1 overlap the elementwise work of step s, and the
// gradient products of step s issued after the scores of step s+1.
//
//   dK/dV pass  CTA = 128 keys of one KV head, for the query heads of its
//               share of the group and every 64-query tile at or after the
//               diagonal:
//                 S^T = K Q^T,  dP^T = V dO^T            (M=128 keys, N=64)
//                 P^T = exp(S^T - lse),  dS^T = P^T (dP^T - delta)
//                 dV += P^T dO,  dK += dS^T Q            (M=128 keys, N=128)
//   dQ pass     CTA = 128 queries of one query head, every 64-key tile up to
//               the diagonal:
//                 S = Q K^T,  dP = dO V^T                (M=128 queries, N=64)
//                 dS = P (dP - delta),  dQ += dS K       (N=128)
//
// The same shared-memory tile serves as a K-major B operand (rows = keys or
// queries, d contiguous) for the score MMAs and as an MN-major B operand
// (N = d contiguous) for the gradient MMAs.
//
// When the query heads of a group are split over several CTAs (to fill the
// SMs at short sequences), dK/dV are summed in an fp32 workspace with
// red.global.add.v4.f32 and converted to bf16 by a small kernel.
constexpr int kBwdThreads = 384;  // warps 0 TMA, 1 MMA, 2 TMEM, 3 idle, 4-11 elementwise

__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// smem layout of the dK/dV pass (offsets from the 1024-aligned base): the
// (Q, dO) ring is three steps deep so the loads of step s+2 are in flight
// while step s runs; P^T and dS^T are single tiles (the elementwise warps of
// step s+1 write them once the gradient MMAs of step s have read them).
constexpr int kKvSlots = 3;
constexpr int kKvOffK = 0, kKvOffV = 32768, kKvOffRing = 65536;  // ring: 3 x (Q 16 KB + dO 16 KB)
constexpr int kKvOffP = kKvOffRing + kKvSlots * 32768;            // 16 KB
constexpr int kKvOffDS = kKvOffP + 16384;                         // 16 KB
constexpr int kKvOffLsd = kKvOffDS + 16384;                       // 8 warps x (32 lse2 + 32 delta) floats
constexpr int kKvOffBar = kKvOffLsd + 8 * 64 * 4;
constexpr int kKvSmem = kKvOffBar + 128 + 1024;

__global__ void __launch_bounds__(kBwdThreads, 1)
    fa_bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                          const float* __restrict__ lse, const float* __restrict__ delta, bf16* __restrict__ dk,
                          bf16* __restrict__ dv, long long lddqkv, float* __restrict__ ws_k,
                          float* __restrict__ ws_v, long long ldws, int T, int Hq, int Hk, int heads_per_cta,
                          float scale, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kKvOffBar);
  uint64_t* kv_full = bars;
  uint64_t* ring_full = bars + 1;   // [3]
  uint64_t* ring_empty = bars + 4;  // [3]
  uint64_t* st_full = bars + 7;     // [2]
  uint64_t* pd_full = bars + 9;
  uint64_t* pd_empty = bars + 10;
  uint64_t* acc_full = bars + 11;
  uint64_t* drain = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = blockIdx.x, bhk = blockIdx.y, b = bhk / Hk, hk = bhk % Hk;
  const int G = Hq / Hk, h_first = hk * G + blockIdx.z * heads_per_cta;
  const int k0 = kt * 128;
  const int i_lo = k0 / 64, n_q = (T + 63) / 64 - i_lo;
  const int n_steps = heads_per_cta * n_q;
  const float l2e = 1.4426950408889634f, sl2 = scale * l2e;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < kKvSlots; ++i) {
      mbar_init(&ring_full[i], 1);
      mbar_init(&ring_empty[i], 1);
    }
    mbar_init(&st_full[0], 1);
    mbar_init(&st_full[1], 1);
    mbar_init(pd_full, 8);
    mbar_init(pd_empty, 1);
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch(&tmQ);
    tma_prefetch(&tmK);
    tma_prefetch(&tmV);
    tma_prefetch(&tmDO);
  }
  if (warp == 2) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------ TMA producer
    mbar_arrive_expect_tx(kv_full, 65536);
    for (int a = 0; a < 2; ++a) {
      tma_load_2d(smem + kKvOffK + a * 16384, &tmK, kv_full, hk * D + 64 * a, b * T + k0);
      tma_load_2d(smem + kKvOffV + a * 16384, &tmV, kv_full, hk * D + 64 * a, b * T + k0);
    }
    int issued = 0;
    for (int s = 0; s < n_steps && !*abort_flag; ++s) {
      const int slot = s % kKvSlots;
      if (!mbar_wait(&ring_empty[slot], (static_cast<uint32_t>(s / kKvSlots) & 1u) ^ 1u, abort_flag)) break;
      const int h = h_first + s / n_q, q0 = (i_lo + s % n_q) * 64;
      uint8_t* dst = smem + kKvOffRing + slot * 32768;
      mbar_arrive_expect_tx(&ring_full[slot], 32768);
      for (int a = 0; a < 2; ++a) {
        tma_load_2d(dst + a * 8192, &tmQ, &ring_full[slot], h * D + 64 * a, b * T + q0);
        tma_load_2d(dst + 16384 + a * 8192, &tmDO, &ring_full[slot], h * D + 64 * a, b * T + q0);
      }
      ++issued;
    }
    if (*abort_flag) {
      const unsigned long long t0 = global_ns();
      while (!mbar_try_wait(kv_full, 0) && global_ns() - t0 < 100000000ull) {
      }
      for (int s = issued - (issued < kKvSlots ? issued : kKvSlots); s < issued; ++s) {
        const unsigned long long t1 = global_ns();
        while (!mbar_try_wait(&ring_full[s % kKvSlots], static_cast<uint32_t>(s / kKvSlots) & 1u) &&
               global_ns() - t1 < 100000000ull) {
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------ MMA issuer
    constexpr uint32_t id_s = idesc_bf16(128, 64, 0, 0);
    constexpr uint32_t id_g = idesc_bf16(128, 128, 0, 1);
    const uint32_t sk = smem_u32(smem + kKvOffK), sv = smem_u32(smem + kKvOffV);
    bool ok = mbar_wait(kv_full, 0, abort_flag), any = false;
    auto grads = [&](int t) -> bool {
      const int slot = t % kKvSlots;
      if (!mbar_wait(pd_full, static_cast<uint32_t>(t) & 1u, abort_flag)) return false;
      tc_fence_after();
      const uint32_t sq = smem_u32(smem + kKvOffRing + slot * 32768), sdo = sq + 16384;
      const uint32_t sp = smem_u32(smem + kKvOffP), sds = smem_u32(smem + kKvOffDS);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t acc = (t > 0 || kk > 0) ? 1u : 0u;
        mma_f16(tmem_base + 256, smem_desc_sw128(sp + kk * 32, 16, 1024),
                smem_desc_sw128(sdo + kk * 2048, 8192, 1024), id_g, acc);
        mma_f16(tmem_base + 384, smem_desc_sw128(sds + kk * 32, 16, 1024),
                smem_desc_sw128(sq + kk * 2048, 8192, 1024), id_g, acc);
      }
      mma_commit(&ring_empty[slot]);
      mma_commit(pd_empty);
      return true;
    };
    if (ok) tc_fence_after();
    for (int s = 0; ok && s < n_steps; ++s) {
      const int bs = s & 1, slot = s % kKvSlots;
      if (!mbar_wait(&ring_full[slot], static_cast<uint32_t>(s / kKvSlots) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sq = smem_u32(smem + kKvOffRing + slot * 32768), sdo = sq + 16384;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t ao = (kk >> 2) * 16384 + (kk & 3) * 32, bo = (kk >> 2) * 8192 + (kk & 3) * 32;
        mma_f16(tmem_base + 64 * bs, smem_desc_sw128(sk + ao, 16, 1024), smem_desc_sw128(sq + bo, 16, 1024), id_s,
                kk > 0 ? 1u : 0u);
        mma_f16(tmem_base + 128 + 64 * bs, smem_desc_sw128(sv + ao, 16, 1024), smem_desc_sw128(sdo + bo, 16, 1024),
                id_s, kk > 0 ? 1u : 0u);
      }
      any = true;
      mma_commit(&st_full[bs]);
      if (s > 0 && !grads(s - 1)) ok = false;
    }
    if (ok && n_steps > 0) ok = grads(n_steps - 1);
    if (ok) mma_commit(acc_full);
    if (any) {
      mma_commit(drain);
      const unsigned long long t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 1000000000ull) {
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ elementwise: P^T, dS^T
    const int quarter = warp & 3, half = (warp - 4) >> 2;
    const int r = quarter * 32 + lane, key = k0 + r, sw = r & 7;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    float* L = reinterpret_cast<float*>(smem + kKvOffLsd) + (warp - 4) * 64;
    bool ok = true;
    // lse / delta of this warp's 32 query columns, loaded one step ahead
    auto fetch = [&](int s, float& fl, float& fd) {
      const int h = h_first + s / n_q, q = (i_lo + s % n_q) * 64 + half * 32 + lane;
      const long long idx = (static_cast<long long>(b) * Hq + h) * T + q;
      fl = q < T ? lse[idx] * l2e : __int_as_float(0x7f800000);
      fd = q < T ? delta[idx] : 0.f;
    };
    float nl = 0.f, nd = 0.f;
    if (n_steps > 0) fetch(0, nl, nd);
    for (int s = 0; s < n_steps; ++s) {
      const int bs = s & 1;
      const int q0 = (i_lo + s % n_q) * 64;
      // L[0, 32): lse in log2 units, L[32, 64): delta
      __syncwarp();
      L[lane] = nl;
      L[32 + lane] = nd;
      __syncwarp();
      if (s + 1 < n_steps) fetch(s + 1, nl, nd);
      ok = __all_sync(0xffffffffu, mbar_wait(&st_full[bs], static_cast<uint32_t>(s >> 1) & 1u, abort_flag));
      if (!ok) break;
      tc_fence_after();
      uint32_t sv[32], dv_[32];
      tmem_ld_x32(tmem_base + lane_off + 64 * bs + half * 32, sv);
      tmem_ld_x32(tmem_base + lane_off + 128 + 64 * bs + half * 32, dv_);
      tmem_wait_ld();
      after_wait<32>(sv);
      after_wait<32>(dv_);
      const bool diag = q0 < k0 + 128;
      uint32_t pw[16], dw[16];
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        const int cc = half * 32 + c;
        float p0 = ex2(__uint_as_float(sv[c]) * sl2 - L[c]);
        float p1 = ex2(__uint_as_float(sv[c + 1]) * sl2 - L[c + 1]);
        if (diag && key > q0 + cc) p0 = 0.f;
        if (diag && key > q0 + cc + 1) p1 = 0.f;
        const float d0 = p0 * (__uint_as_float(dv_[c]) - L[32 + c]);
        const float d1 = p1 * (__uint_as_float(dv_[c + 1]) - L[32 + c + 1]);
        pw[c >> 1] = pack_bf16(p0, p1);
        dw[c >> 1] = pack_bf16(d0, d1);
      }
      // the gradient MMAs of step s-1 have read the P^T / dS^T tiles
      ok = __all_sync(0xffffffffu, mbar_wait(pd_empty, (static_cast<uint32_t>(s) & 1u) ^ 1u, abort_flag));
      if (!ok) break;
      uint8_t* prow = smem + kKvOffP + r * 128;
      uint8_t* drow = smem + kKvOffDS + r * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int chunk = ((half * 4 + c) ^ sw) << 4;
        *reinterpret_cast<uint4*>(prow + chunk) = make_uint4(pw[4 * c], pw[4 * c + 1], pw[4 * c + 2], pw[4 * c + 3]);
        *reinterpret_cast<uint4*>(drow + chunk) = make_uint4(dw[4 * c], dw[4 * c + 1], dw[4 * c + 2], dw[4 * c + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pd_full);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, abort_flag));
    if (ok) {
      tc_fence_after();
      // dV at TMEM columns [256, 384), dK at [384, 512); this warp: 64 of the 128 d columns
#pragma unroll 1
      for (int m = 0; m < 2; ++m) {
#pragma unroll 1
        for (int cc = 0; cc < 2; ++cc) {
          const int col = half * 64 + cc * 32;
          uint32_t ov[32];
          tmem_ld_x32(tmem_base + lane_off + 256 + 128 * m + col, ov);
          tmem_wait_ld();
          after_wait<32>(ov);
          if (key < T) {
            const float f = m == 1 ? scale : 1.f;
            const long long row = static_cast<long long>(b) * T + key;
            if (ws_k != nullptr) {
              float* dst = (m == 1 ? ws_k : ws_v) + row * ldws + hk * D + col;
#pragma unroll
              for (int g = 0; g < 8; ++g)
                red_add_v4(dst + 4 * g, __uint_as_float(ov[4 * g]) * f, __uint_as_float(ov[4 * g + 1]) * f,
                           __uint_as_float(ov[4 * g + 2]) * f, __uint_as_float(ov[4 * g + 3]) * f);
            } else {
              bf16* dst = (m == 1 ? dk : dv) + row * lddqkv + hk * D + col;
#pragma unroll
              for (int g = 0; g < 4; ++g) {
                uint4 u;
                u.x = pack_bf16(__uint_as_float(ov[8 * g + 0]) * f, __uint_as_float(ov[8 * g + 1]) * f);
                u.y = pack_bf16(__uint_as_float(ov[8 * g + 2]) * f, __uint_as_float(ov[8 * g + 3]) * f);
                u.z = pack_bf16(__uint_as_float(ov[8 * g + 4]) * f, __uint_as_float(ov[8 * g + 5]) * f);
                u.w = pack_bf16(__uint_as_float(ov[8 * g + 6]) * f, __uint_as_float(ov[8 * g + 7]) * f);
                *reinterpret_cast<uint4*>(dst + g * 8) = u;
              }
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
  if (threadIdx.x == 0 && *abort_flag && err != nullptr) atomicCAS(err, 0, 22);
}

// smem layout of the dQ pass
constexpr int kDqOffQ = 0, kDqOffDO = 32768, kDqOffRing = 65536;  // ring: 3 x (K 16 KB + V 16 KB)
constexpr int kDqSlots = 3;
constexpr int kDqOffDS = kDqOffRing + kDqSlots * 32768;           // 2 x 16 KB
constexpr int kDqOffBar = kDqOffDS + 2 * 16384;
constexpr int kDqSmem = kDqOffBar + 128 + 1024;

__global__ void __launch_bounds__(kBwdThreads, 1)
    fa_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                        const float* __restrict__ lse, const float* __restrict__ delta, bf16* __restrict__ dq,
                        long long lddqkv, int T, int Hq, int Hk, float scale, int n_qt, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kDqOffBar);
  uint64_t* q_full = bars;
  uint64_t* ring_full = bars + 1;   // [3]
  uint64_t* ring_empty = bars + 4;  // [3]
  uint64_t* st_full = bars + 7;     // [2]
  uint64_t* pd_full = bars + 9;     // [2]
  uint64_t* pd_empty = bars + 11;   // [2]
  uint64_t* acc_full = bars + 13;
  uint64_t* drain = bars + 14;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.x);
  const int bh = blockIdx.y, b = bh / Hq, h = bh % Hq, hk = h / (Hq / Hk);
  const int q0 = qt * 128;
  const int n_kv = (min(q0 + 128, T) + 63) / 64;
  const float l2e = 1.4426950408889634f, sl2 = scale * l2e;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kDqSlots; ++i) {
      mbar_init(&ring_full[i], 1);
      mbar_init(&ring_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&st_full[i], 1);
      mbar_init(&pd_full[i], 8);
      mbar_init(&pd_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch(&tmQ);
    tma_prefetch(&tmK);
    tma_prefetch(&tmV);
    tma_prefetch(&tmDO);
  }
  if (warp == 2) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    mbar_arrive_expect_tx(q_full, 65536);
    for (int a = 0; a < 2; ++a) {
      tma_load_2d(smem + kDqOffQ + a * 16384, &tmQ, q_full, h * D + 64 * a, b * T + q0);
      tma_load_2d(smem + kDqOffDO + a * 16384, &tmDO, q_full, h * D + 64 * a, b * T + q0);
    }
    int issued = 0;
    for (int j = 0; j < n_kv && !*abort_flag; ++j) {
      const int slot = j % kDqSlots;
      if (!mbar_wait(&ring_empty[slot], (static_cast<uint32_t>(j / kDqSlots) & 1u) ^ 1u, abort_flag)) break;
      uint8_t* dst = smem + kDqOffRing + slot * 32768;
      mbar_arrive_expect_tx(&ring_full[slot], 32768);
      for (int a = 0; a < 2; ++a) {
        tma_load_2d(dst + a * 8192, &tmK, &ring_full[slot], hk * D + 64 * a, b * T + j * 64);
        tma_load_2d(dst + 16384 + a * 8192, &tmV, &ring_full[slot], hk * D + 64 * a, b * T + j * 64);
      }
      ++issued;
    }
    if (*abort_flag) {
      const unsigned long long t0 = global_ns();
      while (!mbar_try_wait(q_full, 0) && global_ns() - t0 < 100000000ull) {
      }
      for (int j = issued - (issued < kDqSlots ? issued : kDqSlots); j < issued; ++j) {
        const unsigned long long t1 = global_ns();
        while (!mbar_try_wait(&ring_full[j % kDqSlots], static_cast<uint32_t>(j / kDqSlots) & 1u) &&
               global_ns() - t1 < 100000000ull) {
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t id_s = idesc_bf16(128, 64, 0, 0);
    constexpr uint32_t id_g = idesc_bf16(128, 128, 0, 1);
    const uint32_t sq = smem_u32(smem + kDqOffQ), sdo = smem_u32(smem + kDqOffDO);
    bool ok = mbar_wait(q_full, 0, abort_flag), any = false;
    auto grads = [&](int t) -> bool {
      const int bt = t & 1, slot = t % kDqSlots;
      if (!mbar_wait(&pd_full[bt], static_cast<uint32_t>(t >> 1) & 1u, abort_flag)) return false;
      tc_fence_after();
      const uint32_t sk = smem_u32(smem + kDqOffRing + slot * 32768);
      const uint32_t sds = smem_u32(smem + kDqOffDS + bt * 16384);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_f16(tmem_base + 256, smem_desc_sw128(sds + kk * 32, 16, 1024),
                smem_desc_sw128(sk + kk * 2048, 8192, 1024), id_g, (t > 0 || kk > 0) ? 1u : 0u);
      mma_commit(&ring_empty[slot]);
      mma_commit(&pd_empty[bt]);
      return true;
    };
    if (ok) tc_fence_after();
    for (int j = 0; ok && j < n_kv; ++j) {
      const int bs = j & 1, slot = j % kDqSlots;
      if (!mbar_wait(&ring_full[slot], static_cast<uint32_t>(j / kDqSlots) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sk = smem_u32(smem + kDqOffRing + slot * 32768), sv = sk + 16384;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t ao = (kk >> 2) * 16384 + (kk & 3) * 32, bo = (kk >> 2) * 8192 + (kk & 3) * 32;
        mma_f16(tmem_base + 64 * bs, smem_desc_sw128(sq + ao, 16, 1024), smem_desc_sw128(sk + bo, 16, 1024), id_s,
                kk > 0 ? 1u : 0u);
        mma_f16(tmem_base + 128 + 64 * bs, smem_desc_sw128(sdo + ao, 16, 1024), smem_desc_sw128(sv + bo, 16, 1024),
                id_s, kk > 0 ? 1u : 0u);
      }
      any = true;
      mma_commit(&st_full[bs]);
      if (j > 0 && !grads(j - 1)) ok = false;
    }
    if (ok) ok = grads(n_kv - 1);
    if (ok) mma_commit(acc_full);
    if (any) {
      mma_commit(drain);
      const unsigned long long t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 1000000000ull) {
      }
    }
  } else if (warp >= 4) {
    const int quarter = warp & 3, half = (warp - 4) >> 2;
    const int r = quarter * 32 + lane, row = q0 + r, sw = r & 7;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const long long li = (static_cast<long long>(b) * Hq + h) * T + row;
    const float lse2 = row < T ? lse[li] * l2e : 0.f, dl = row < T ? delta[li] : 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int bs = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&st_full[bs], static_cast<uint32_t>(j >> 1) & 1u, abort_flag));
      if (!ok) break;
      tc_fence_after();
      uint32_t sv[32], dv_[32];
      tmem_ld_x32(tmem_base + lane_off + 64 * bs + half * 32, sv);
      tmem_ld_x32(tmem_base + lane_off + 128 + 64 * bs + half * 32, dv_);
      tmem_wait_ld();
      after_wait<32>(sv);
      after_wait<32>(dv_);
      const int kb = j * 64 + half * 32;
      const bool diag = kb + 31 > q0;
      uint32_t dw[16];
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        float p0 = ex2(__uint_as_float(sv[c]) * sl2 - lse2);
        float p1 = ex2(__uint_as_float(sv[c + 1]) * sl2 - lse2);
        if (diag && kb + c > row) p0 = 0.f;
        if (diag && kb + c + 1 > row) p1 = 0.f;
        dw[c >> 1] = pack_bf16(p0 * (__uint_as_float(dv_[c]) - dl), p1 * (__uint_as_float(dv_[c + 1]) - dl));
      }
      ok = __all_sync(0xffffffffu,
                      mbar_wait(&pd_empty[bs], (static_cast<uint32_t>(j >> 1) & 1u) ^ 1u, abort_flag));
      if (!ok) break;
      uint8_t* drow = smem + kDqOffDS + bs * 16384 + r * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(drow + (((half * 4 + c) ^ sw) << 4)) =
            make_uint4(dw[4 * c], dw[4 * c + 1], dw[4 * c + 2], dw[4 * c + 3]);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pd_full[bs]);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, abort_flag));
    if (ok) {
      tc_fence_after();
#pragma unroll 1
      for (int cc = 0; cc < 2; ++cc) {
        const int col = half * 64 + cc * 32;
        uint32_t ov[32];
        tmem_ld_x32(tmem_base + lane_off + 256 + col, ov);
        tmem_wait_ld();
        after_wait<32>(ov);
        if (row < T) {
          bf16* dst = dq + (static_cast<long long>(b) * T + row) * lddqkv + h * D + col;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 u;
            u.x = pack_bf16(__uint_as_float(ov[8 * g + 0]) * scale, __uint_as_float(ov[8 * g + 1]) * scale);
            u.y = pack_bf16(__uint_as_float(ov[8 * g + 2]) * scale, __uint_as_float(ov[8 * g + 3]) * scale);
            u.z = pack_bf16(__uint_as_float(ov[8 * g + 4]) * scale, __uint_as_float(ov[8 * g + 5]) * scale);
            u.w = pack_bf16(__uint_as_float(ov[8 * g + 6]) * scale, __uint_as_float(ov[8 * g + 7]) * scale);
            *reinterpret_cast<uint4*>(dst + g * 8) = u;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
  if (threadIdx.x == 0 && *abort_flag && err != nullptr) atomicCAS(err, 0, 23);
}

// dK/dV fp32 workspace [B*T, Hk*128] x 2 -> bf16 slices of the gradient buffer
__global__ void dkdv_ws_to_bf16_kernel(const float* __restrict__ wk, const float* __restrict__ wv, long long ldws,
                                       bf16* __restrict__ dk, bf16* __restrict__ dv, long long lddqkv, long long rows,
                                       int cols) {
  const long long n8 = rows * (cols / 8);
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < 2 * n8;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const bool isv = i >= n8;
    const long long e = isv ? i - n8 : i;
    const long long row = e / (cols / 8);
    const int c = static_cast<int>(e % (cols / 8)) * 8;
    const float4* src = reinterpret_cast<const float4*>((isv ? wv : wk) + row * ldws + c);
    const float4 a = src[0], bq = src[1];
    uint4 u;
    u.x = pack_bf16(a.x, a.y);
    u.y = pack_bf16(a.z, a.w);
    u.z = pack_bf16(bq.x, bq.y);
    u.w = pack_bf16(bq.z, bq.w);
    *reinterpret_cast<uint4*>((isv ? dv : dk) + row * lddqkv + c) = u;
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// [rows, cols] bf16 with row stride ld (elements); box {64 cols, box_rows}, 128-byte swizzle.
bool head_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long ld, int box_rows) {
  EncodeTiledFn f = encode_fn();
  if (!f) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t es[2] = {1, 1};
  return f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

extern "C" int tb_flash_attn_fwd_tc(const void* q, const void* k, const void* v, long long ld, void* o, long long ldo,
                                    float* lse, int B, int T, int Hq, int Hk, float scale, int* err,
                                    cudaStream_t s) {
  if (B <= 0 || T <= 0) return 0;
  if (Hq <= 0 || Hk <= 0 || Hq % Hk || (ld % 8) || (ldo % 8)) return static_cast<int>(cudaErrorInvalidValue);
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(o)) & 15u)
    return static_cast<int>(cudaErrorMisalignedAddress);
  const long long rows = static_cast<long long>(B) * T;
  CUtensorMap mq, mk, mv;
  if (!head_map(&mq, q, rows, static_cast<long long>(Hq) * D, ld, BQ) ||
      !head_map(&mk, k, rows, static_cast<long long>(Hk) * D, ld, BKV) ||
      !head_map(&mv, v, rows, static_cast<long long>(Hk) * D, ld, BKV))
    return static_cast<int>(cudaErrorInvalidValue);
  tb::ensure_dyn_smem(reinterpret_cast<const void*>(fa_fwd_tc_kernel), kSmemBytes);
  const int n_qt = (T + BQ - 1) / BQ;
  dim3 grid(n_qt, B * Hq);
  fa_fwd_tc_kernel<<<grid, kThreads, kSmemBytes, s>>>(mq, mk, mv, static_cast<bf16*>(o), ldo, lse, T, Hq, Hk,
                                                       scale * 1.4426950408889634f, n_qt, err);
  return static_cast<int>(cudaGetLastError());
}

extern "C" size_t tb_flash_attn_bwd_ws_bytes(int B, int T, int Hk) {
  return 2ull * static_cast<size_t>(B) * T * Hk * D * sizeof(float);
}

extern "C" int tb_flash_attn_bwd_tc(const void* q, const void* k, const void* v, long long ld, const void* o,
                                    long long ldo, const void* dout, long long lddo, const float* lse, float* delta,
                                    void* dq, void* dk, void* dv, long long lddqkv, int B, int T, int Hq, int Hk,
                                    float scale, float* ws, size_t ws_bytes, int* err, cudaStream_t s) {
  if (B <= 0 || T <= 0) return 0;
  if (Hq <= 0 || Hk <= 0 || Hq % Hk || (ld % 8) || (ldo % 8) || (lddo % 8) || (lddqkv % 8))
    return static_cast<int>(cudaErrorInvalidValue);
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(dout) | reinterpret_cast<uintptr_t>(dq) | reinterpret_cast<uintptr_t>(dk) |
       reinterpret_cast<uintptr_t>(dv)) & 15u)
    return static_cast<int>(cudaErrorMisalignedAddress);
  int e = tb_flash_attn_delta(o, ldo, dout, lddo, delta, B, T, Hq, s);
  if (e != 0) return e;
  const long long rows = static_cast<long long>(B) * T;
  const long long qc = static_cast<long long>(Hq) * D, kc = static_cast<long long>(Hk) * D;
  CUtensorMap mq64, mq128, mk64, mk128, mv64, mv128, mdo64, mdo128;
  if (!head_map(&mq64, q, rows, qc, ld, 64) || !head_map(&mq128, q, rows, qc, ld, 128) ||
      !head_map(&mk64, k, rows, kc, ld, 64) || !head_map(&mk128, k, rows, kc, ld, 128) ||
      !head_map(&mv64, v, rows, kc, ld, 64) || !head_map(&mv128, v, rows, kc, ld, 128) ||
      !head_map(&mdo64, dout, rows, qc, lddo, 64) || !head_map(&mdo128, dout, rows, qc, lddo, 128))
    return static_cast<int>(cudaErrorInvalidValue);
  // split the query heads of a group over CTAs until the dK/dV grid covers the SMs twice
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int G = Hq / Hk, n_kt = (T + 127) / 128;
  const long long base_ctas = static_cast<long long>(n_kt) * B * Hk;
  int split = 1;
  const bool have_ws = ws != nullptr && ws_bytes >= tb_flash_attn_bwd_ws_bytes(B, T, Hk);
  if (have_ws)
    while (split < G && base_ctas * split < 2LL * sms) {
      int nxt = split + 1;
      while (G % nxt) ++nxt;
      split = nxt;
    }
  float* wk = split > 1 ? ws : nullptr;
  float* wv = split > 1 ? ws + rows * kc : nullptr;
  if (split > 1) {
    e = static_cast<int>(cudaMemsetAsync(ws, 0, tb_flash_attn_bwd_ws_bytes(B, T, Hk), s));
    if (e != 0) return e;
  }
  tb::ensure_dyn_smem(reinterpret_cast<const void*>(fa_bwd_dkdv_tc_kernel), kKvSmem);
  dim3 g1(n_kt, B * Hk, split);
  fa_bwd_dkdv_tc_kernel<<<g1, kBwdThreads, kKvSmem, s>>>(
      mq64, mk128, mv128, mdo64, lse, delta, static_cast<bf16*>(dk), static_cast<bf16*>(dv), lddqkv, wk, wv, kc, T,
      Hq, Hk, G / split, scale, err);
  if (split > 1)
    dkdv_ws_to_bf16_kernel<<<4 * sms, 256, 0, s>>>(wk, wv, kc, static_cast<bf16*>(dk), static_cast<bf16*>(dv),
                                                    lddqkv, rows, static_cast<int>(kc));
  tb::ensure_dyn_smem(reinterpret_cast<const void*>(fa_bwd_dq_tc_kernel), kDqSmem);
  const int n_qt = (T + 127) / 128;
  dim3 g2(n_qt, B * Hq);
  fa_bwd_dq_tc_kernel<<<g2, kBwdThreads, kDqSmem, s>>>(mq128, mk64, mv64, mdo128, lse, delta, static_cast<bf16*>(dq),
                                                       lddqkv, T, Hq, Hk, scale, n_qt, err);
  return static_cast<int>(cudaGetLastError());
}
