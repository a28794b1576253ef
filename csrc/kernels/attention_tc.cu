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
  uint64_t* s_full = bars + 7;
  uint64_t* p_full = bars + 8;
  uint64_t* o_full = bars + 9;
  uint64_t* drain = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);
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
    mbar_init(s_full, 1);
    mbar_init(p_full, 4);
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
      const CUtensorMap* m = (i & 1) ? &tmV : &tmK;
      const int y = row_base + (i >> 1) * BKV;
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
    for (int j = 0; ok && j < n_kv; ++j) {
      int i = 2 * j, slot = i % kSlots;
      if (!mbar_wait(&ring_full[slot], static_cast<uint32_t>(i / kSlots) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sk = smem_u32(smem + kOffRing + slot * kTileBytes);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint64_t ad = smem_desc_sw128(sq + (kk >> 2) * (kQBytes / 2) + (kk & 3) * 32, 16, 1024);
        const uint64_t bd = smem_desc_sw128(sk + (kk >> 2) * (kTileBytes / 2) + (kk & 3) * 32, 16, 1024);
        mma_f16(t_s, ad, bd, id_s, kk > 0 ? 1u : 0u);
      }
      any = true;
      mma_commit(&ring_empty[slot]);
      mma_commit(s_full);
      // P_j written (and S_j read, O rescaled) by the softmax warpgroup
      if (!mbar_wait(p_full, static_cast<uint32_t>(j) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      i = 2 * j + 1;
      slot = i % kSlots;
      if (!mbar_wait(&ring_full[slot], static_cast<uint32_t>(i / kSlots) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sv = smem_u32(smem + kOffRing + slot * kTileBytes);
#pragma unroll
      for (int kk = 0; kk < BKV / 16; ++kk) {
        const uint64_t ad = smem_desc_sw128(sp + kk * 32, 16, 1024);
        const uint64_t bd = smem_desc_sw128(sv + kk * 2048, kTileBytes / 2, 1024);
        mma_f16(t_o, ad, bd, id_o, (j > 0 || kk > 0) ? 1u : 0u);
      }
      mma_commit(&ring_empty[slot]);
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
      ok = __all_sync(0xffffffffu, mbar_wait(s_full, static_cast<uint32_t>(j) & 1u, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const int k0 = j * BKV;
      const bool diag = k0 + BKV - 1 > q0;  // a key of this tile may lie past some row of the query tile
      // pass 1: the tile's row max (S is read twice from TMEM rather than held in registers)
      float mt = -INFINITY;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t sv[32];
        tmem_ld_x32(t_s + half * 32, sv);
        tmem_wait_ld();
        after_wait<32>(sv);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          float x = __uint_as_float(sv[c]) * scale_log2;
          if (diag && k0 + half * 32 + c > row) x = -INFINITY;
          mt = fmaxf(mt, x);
        }
      }
      const bool need = mt > m_ref + kRescaleThreshold;  // always true on the first tile (col 0 <= row)
      float alpha = 1.f;
      if (need) {
        alpha = ex2(m_ref - mt);  // 0 when m_ref is -inf
        m_ref = mt;
        l *= alpha;
      }
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O_{j-1} is complete (the commit behind s_full covers the previous P.V)
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
      float sum = 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t sv[32];
        tmem_ld_x32(t_s + half * 32, sv);
        tmem_wait_ld();
        after_wait<32>(sv);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int col = half * 32 + 8 * c + 2 * e;
            float x0 = __uint_as_float(sv[8 * c + 2 * e]) * scale_log2;
            float x1 = __uint_as_float(sv[8 * c + 2 * e + 1]) * scale_log2;
            if (diag && k0 + col > row) x0 = -INFINITY;
            if (diag && k0 + col + 1 > row) x1 = -INFINITY;
            const float p0 = ex2(x0 - m_ref), p1 = ex2(x1 - m_ref);
            sum += p0 + p1;
            w[e] = pack_bf16(p0, p1);
          }
          *reinterpret_cast<uint4*>(prow + (((half * 4 + c) ^ sw) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      l += sum;
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
