// bf16 GEMM on the 5th-generation tensor cores (tcgen05) for sm_100a.
//
//   C[M, N] = epilogue( A[M, K] . B[N, K]^T )      fp32 accumulation in TMEM
//
// Operands may be K-major (row-major with K contiguous: an activation X[M, K]
// or an nn.Linear weight W[N, K]) or MN-major (row-major with M or N
// contiguous: the transposed operands of the weight and input gradients), so
// forward (Y = X W^T), input gradient (dX = dY W) and weight gradient
// (dW = dY^T X) all run without materialized transposes.
//
// Structure: persistent CTAs (at most one per SM), 128 x BN x 64 tiles,
// warp-specialized:
//   warp 0      one thread issues TMA tile loads (128-byte swizzle, no
//               multicast) into a ring of shared-memory stages;
//   warp 1      one thread issues tcgen05.mma (M=128, N=BN, K=16) into a TMEM
//               accumulator and commits each stage back to the producer;
//   warp 2      allocates / frees TMEM (two accumulators of BN columns, so the
//               epilogue of one tile overlaps the MMAs of the next);
//   warps 4-7   epilogue: tcgen05.ld 32 columns at a time, fused bias /
//               activation / tanh-backward / residual / SwiGLU, vectorized
//               global stores, or fp32 atomic accumulation for split-K and
//               gradient accumulation.
// All waits are bounded (sm100_primitives.cuh): on timeout the kernel records
// an error, drains its own in-flight copies and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <mutex>

#include "kernels.h"
#include "device_common.cuh"
#include "pdl.cuh"
#include "sm100_primitives.cuh"

namespace {

using namespace tb::sm100;

constexpr int BM = 128, BK = 64;
constexpr int kEpiWarps = 8;                    // two per TMEM lane quarter
constexpr int kThreads = 128 + 32 * kEpiWarps;  // warps 0-3: TMA, MMA, TMEM, spare

// Tensor-parallel collectives fused into the GEMM (see the TP section below).
constexpr int kTpMaxRanks = TB_MAX_PEERS;
constexpr int kTpSubRows = 8;    // rows per all-gather push unit (one ready flag each)
constexpr int kTpMaxSub = 2048;  // push units per source rank (rows per rank <= 16384)
struct TpHdr {                    // one per rank, at the start of its symmetric buffer
  unsigned ready[2][kTpMaxRanks][kTpMaxSub];  // AG: [parity][src][unit] arrivals of the src's push warps
                                              // (zeroed again by this rank once consumed)
  unsigned consumed[kTpMaxRanks];             // AG: rank p has finished reading its staging (epoch)
  unsigned rs_arrivals[2];                    // RS: [parity] CTA arrivals from every source (monotonic)
  unsigned rs_consumed[kTpMaxRanks];          // RS: rank p has finished reading its receive slots (epoch)
};
struct TpArgs {
  int rank, world, rows_per_rank;  // rows_per_rank (Mloc): a multiple of 128
  unsigned* epoch_ctr;             // epoch of this op's previous call (local device memory)
  unsigned* done_ctr;              // local CTA counter
  TpHdr* hdr[kTpMaxRanks];         // every rank's header
  char* data[kTpMaxRanks];         // every rank's data region (AG staging or RS receive slots)
  long long parity_bytes;          // bytes per parity half of a data region
  const __nv_bfloat16* shard;      // AG: this rank's rows [Mloc, K]
  long long ld_shard;
  __nv_bfloat16* gather_out;       // AG, optional: the gathered A [M, K] is also written here
  long long ld_gather;
  int* err;
  unsigned long long* trace;  // optional [grid][8] timestamps (diagnostics)
};

struct DevArgs {
  int M, N, K;
  int m_tiles, n_tiles, splits, kb_per_split, k_blocks;
  void* C;
  long long ldc;
  int c_fp32, c_atomic, c_add;  // atomic: split-K partials into C; add: C += result (owned elements)
  const float* bias;
  const __nv_bfloat16* aux;
  long long ld_aux;
  int epi;
  float alpha;
  float* ws;      // split-K partials [splits, M, N] (null: atomics into C)
  int* slot_cnt;  // in-kernel split-K fix-up: one arrival counter per (tile, epilogue warp); null: reduce pass
  float* colsum;  // optional: column sums of the epilogue output, accumulated atomically
  int* error;
  __nv_bfloat16* c2;  // EPI_SWIGLU, optional: the raw gate/up accumulator [M, N] (bf16), row stride ldc2
  long long ldc2;
  int kg_ntiles;      // block-diagonal B: n-tiles per diagonal block (0 = off); k_blocks is then per block
  int kg_packed;      // block-diagonal B stored packed: only the diagonal blocks, side by side along its inner dim
  TpArgs tp;
};

// Workspace layout for split-K: [kCntBytes of fix-up counters][partials].
constexpr int kCntSlots = 8192;
constexpr size_t kCntBytes = kCntSlots * sizeof(int);
// With at most this many splits the last warp to finish a slice sums the
// partials itself; more splits go through the bandwidth-parallel reduce pass.
constexpr int kMaxFixupSplits = 4;

template <int BN>
struct Smem {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int kBarOffset = kStages * kStageBytes;
  static constexpr int kStgOffset = kBarOffset + 256;     // per-warp store staging (bf16 outputs)
  static constexpr int kStgWords = 20;                     // 16 words of a 32-column row + 4 pad
  static constexpr int kStgBytes = kEpiWarps * 32 * kStgWords * 4;
  static constexpr int kTotal = kStgOffset + kStgBytes + 1024;  // + slack for 1024-B alignment
};

// Hardware tanh approximation (relative error ~2^-11, below bf16 resolution).
__device__ __forceinline__ float fast_tanh(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float fast_silu(float x) { return x / (1.f + __expf(-x)); }

// 16 bf16 loaded as two 16-byte vectors when aligned.
__device__ __forceinline__ void load_bf16x16(const __nv_bfloat16* p, float* out, int valid) {
  if (valid >= 16 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    const uint4 a = reinterpret_cast<const uint4*>(p)[0], b = reinterpret_cast<const uint4*>(p)[1];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* g = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 x = __bfloat1622float2(h[j]), y = __bfloat1622float2(g[j]);
      out[2 * j] = x.x;
      out[2 * j + 1] = x.y;
      out[8 + 2 * j] = y.x;
      out[8 + 2 * j + 1] = y.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) out[j] = j < valid ? __bfloat162float(p[j]) : 0.f;
  }
}

// Sums 32 columns over the warp's 32 rows by a butterfly transpose-reduce
// (31 shuffles); afterwards lane L holds the sum of column L.
__device__ __forceinline__ float warp_colsum32(float* v, int lane) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int j = 0; j < off; ++j) {
      const float send = upper ? v[j] : v[j + off];
      const float recv = __shfl_xor_sync(0xffffffffu, send, off);
      v[j] = (upper ? v[j + off] : v[j]) + recv;
    }
  }
  return v[0];
}

// Applies the epilogue to 32 accumulator columns [c0, c0+32) of row `row`
// (row >= M rows still join the warp-wide column sum with zeros).
// mode kEpiFull: scale by alpha and run the epilogue; kEpiPartial: scale and
// store the split-K partial; kEpiFinal: epilogue of already-scaled summed partials.
enum { kEpiFull = 0, kEpiPartial = 1, kEpiFinal = 2 };
__device__ __forceinline__ void unpack_bf16x32(uint4 q0, uint4 q1, uint4 q2, uint4 q3, float* out) {
  const uint4 q[4] = {q0, q1, q2, q3};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      out[8 * i + 2 * j] = f.x;
      out[8 * i + 2 * j + 1] = f.y;
    }
  }
}

// Stores 32 bf16 columns [c0, c0 + valid) of this lane's row into base (row
// stride ld): when whole and aligned, transposed through the warp's shared
// staging so each store instruction writes 8 whole 64-byte row segments.
// Every lane of the warp calls it (rows >= M are masked).
__device__ __forceinline__ void store_bf16_row32(__nv_bfloat16* base, long long ld, int M, int row0, int row, int c0,
                                                 const float* v, int valid, int lane, uint32_t* stg) {
  if (valid == 32 && (ld % 8) == 0 && (c0 % 8) == 0 && (reinterpret_cast<uintptr_t>(base) & 15) == 0) {
    uint4* mine = reinterpret_cast<uint4*>(stg + lane * 20);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 pk;
      __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
      for (int j = 0; j < 4; ++j) hh[j] = __floats2bfloat162_rn(v[8 * q + 2 * j], v[8 * q + 2 * j + 1]);
      mine[q] = pk;
    }
    __syncwarp();
    const int seg = lane & 3;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int r = it * 8 + (lane >> 2);
      const uint4 w = *reinterpret_cast<const uint4*>(stg + r * 20 + seg * 4);
      if (row0 + r < M) *reinterpret_cast<uint4*>(base + static_cast<long long>(row0 + r) * ld + c0 + seg * 8) = w;
    }
    __syncwarp();
  } else if (row < M) {
    __nv_bfloat16* C = base + static_cast<long long>(row) * ld + c0;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid) C[j] = __float2bfloat16_rn(v[j]);
  }
}

// pre: a0..a3 hold the row's 32 aux values, already loaded (16 bytes each).
// kSwBwd: the instantiation that runs the SwiGLU-backward epilogue (kept out
// of the others, whose register budget it would otherwise take).
template <bool kSwBwd = false>
__device__ __forceinline__ void epilogue32(const DevArgs& p, int row, int c0, float* v, int ks, int lane,
                                           uint32_t* stg, int row0, int mode, void* cbase, bool pre = false,
                                           uint4 a0 = uint4{}, uint4 a1 = uint4{}, uint4 a2 = uint4{},
                                           uint4 a3 = uint4{}) {
  const int N = p.N, epi = p.epi;
  const bool row_ok = row < p.M;
  const int valid = min(32, N - c0);
  const bool partial = mode == kEpiPartial;
  if (p.alpha != 1.f && mode != kEpiFinal) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] *= p.alpha;
  }
  if (partial) {  // split-K partial: raw accumulator, no epilogue yet
    if (row_ok) {
      float* W = p.ws + (static_cast<long long>(ks) * p.M + row) * N + c0;
      if (valid == 32 && (reinterpret_cast<uintptr_t>(W) & 15) == 0) {
#pragma unroll
        for (int j = 0; j < 8; ++j) reinterpret_cast<float4*>(W)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < valid) W[j] = v[j];
      }
    }
    return;
  }
  if ((epi == TB_EPI_BIAS || epi == TB_EPI_BIAS_TANH || epi == TB_EPI_BIAS_SILU) && p.bias && ks == 0) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] += (j < valid) ? __ldg(p.bias + c0 + j) : 0.f;
  }
  if (epi == TB_EPI_BIAS_TANH) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = fast_tanh(v[j]);
  } else if (epi == TB_EPI_BIAS_SILU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = fast_silu(v[j]);
  } else if ((epi == TB_EPI_TANH_BWD || epi == TB_EPI_RESIDUAL) && row_ok) {
    float h[32];
    if (pre) {
      unpack_bf16x32(a0, a1, a2, a3, h);
    } else {
      const __nv_bfloat16* a = p.aux + static_cast<long long>(row) * p.ld_aux + c0;
      load_bf16x16(a, h, valid);
      load_bf16x16(a + 16, h + 16, valid - 16);
    }
    if (epi == TB_EPI_TANH_BWD) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= 1.f - h[j] * h[j];
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += h[j];
    }
  }
  if constexpr (kSwBwd) {
    // acc = d out[:, c0..c0+32) of out = silu(gate) * up; aux holds the
    // interleaved (gate, up) columns [M, 2N]; C receives d(gate, up) [M, 2N].
    // Two halves of 16 output columns, each giving 32 interleaved columns.
    __nv_bfloat16* C = static_cast<__nv_bfloat16*>(cbase);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int vh = valid - 16 * h;  // valid output columns in this half (may be <= 0)
      if (vh <= 0) break;             // uniform across the warp
      float d[32];
      if (row_ok) {
        const __nv_bfloat16* g = p.aux + static_cast<long long>(row) * p.ld_aux + 2 * (c0 + 16 * h);
        load_bf16x16(g, d, 2 * vh);
        load_bf16x16(g + 16, d + 16, 2 * vh - 16);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float x = d[2 * j], u = d[2 * j + 1], dy = v[16 * h + j];
          const float sg = 1.f / (1.f + __expf(-x));
          d[2 * j] = dy * u * (sg * (1.f + x * (1.f - sg)));
          d[2 * j + 1] = dy * x * sg;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) d[j] = 0.f;
      }
      store_bf16_row32(C, p.ldc, p.M, row0, row, 2 * (c0 + 16 * h), d, vh >= 16 ? 32 : 2 * vh, lane, stg);
    }
    return;
  }
  if (epi == TB_EPI_SWIGLU) {
    // interleaved gate/up columns: out[c/2] = silu(gate) * up
    if (p.c2 != nullptr) store_bf16_row32(p.c2, p.ldc2, p.M, row0, row, c0, v, valid, lane, stg);
    if (!row_ok) return;
    const int oc0 = c0 / 2;
    const int Nout = N / 2;
    float o[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j] = fast_silu(v[2 * j]) * v[2 * j + 1];
    if (p.c_fp32) {
      float* C = static_cast<float*>(cbase) + static_cast<long long>(row) * p.ldc + oc0;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (oc0 + j < Nout) C[j] = o[j];
    } else {
      __nv_bfloat16* C = static_cast<__nv_bfloat16*>(cbase) + static_cast<long long>(row) * p.ldc + oc0;
      if (oc0 + 16 <= Nout && (reinterpret_cast<uintptr_t>(C) & 15) == 0) {
        uint4 pk[2];
        __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(pk);
#pragma unroll
        for (int j = 0; j < 8; ++j) hh[j] = __floats2bfloat162_rn(o[2 * j], o[2 * j + 1]);
        reinterpret_cast<uint4*>(C)[0] = pk[0];
        reinterpret_cast<uint4*>(C)[1] = pk[1];
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (oc0 + j < Nout) C[j] = __float2bfloat16_rn(o[j]);
      }
    }
    return;
  }
  if (p.colsum != nullptr) {
    float t[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) t[j] = row_ok ? v[j] : 0.f;
    const float cs = warp_colsum32(t, lane);
    if (lane < valid) atomicAdd(p.colsum + c0 + lane, cs);
  }
  if (!row_ok && (p.c_atomic || p.c_fp32)) return;
  if (p.c_atomic) {
    float* C = static_cast<float*>(cbase) + static_cast<long long>(row) * p.ldc + c0;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid) atomicAdd(C + j, v[j]);
    return;
  }
  if (p.c_add) {  // C += result; this thread owns these elements (no split-K)
    float* C = static_cast<float*>(cbase) + static_cast<long long>(row) * p.ldc + c0;
    if (valid == 32 && (reinterpret_cast<uintptr_t>(C) & 15) == 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float4 o = reinterpret_cast<float4*>(C)[j];
        o.x += v[4 * j];
        o.y += v[4 * j + 1];
        o.z += v[4 * j + 2];
        o.w += v[4 * j + 3];
        reinterpret_cast<float4*>(C)[j] = o;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < valid) C[j] += v[j];
    }
    return;
  }
  if (p.c_fp32) {
    float* C = static_cast<float*>(cbase) + static_cast<long long>(row) * p.ldc + c0;
    if (valid == 32 && (reinterpret_cast<uintptr_t>(C) & 15) == 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) reinterpret_cast<float4*>(C)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < valid) C[j] = v[j];
    }
  } else {
    __nv_bfloat16* C = static_cast<__nv_bfloat16*>(cbase) + static_cast<long long>(row) * p.ldc + c0;
    if (valid == 32 && (p.ldc % 8) == 0 && (reinterpret_cast<uintptr_t>(cbase) & 15) == 0) {
      // transpose through shared memory so each store instruction writes
      // 8 whole 64-byte row segments instead of 32 scattered 16-byte pieces
      // four 16-byte stores per lane: with the 80-byte row pitch the 8 lanes
      // of each store phase hit disjoint banks
      uint4* mine = reinterpret_cast<uint4*>(stg + lane * 20);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 pk;
        __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
        for (int j = 0; j < 4; ++j) hh[j] = __floats2bfloat162_rn(v[8 * q + 2 * j], v[8 * q + 2 * j + 1]);
        mine[q] = pk;
      }
      __syncwarp();
      const int seg = lane & 3;
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int r = it * 8 + (lane >> 2);
        const uint4 w = *reinterpret_cast<const uint4*>(stg + r * 20 + seg * 4);
        if (row0 + r < p.M)
          *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(cbase) + static_cast<long long>(row0 + r) * p.ldc + c0 +
                                    seg * 8) = w;
      }
      __syncwarp();
    } else if (row_ok) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < valid) C[j] = __float2bfloat16_rn(v[j]);
    }
  }
}

// Split-K fix-up of one warp slice: rows [row0, row0+32) x columns
// [col0, col0+COLS), summed over the splits' partials (in split order) with
// the epilogue applied.  Lanes run along columns (float4 each), so every load
// and store instruction covers whole 256- or 512-byte row segments, and the
// partial loads of a block of rows are all issued before they are used.
template <int COLS>
__device__ __forceinline__ void fixup_slice(const DevArgs& p, int row0, int col0, int lane) {
  constexpr int LPR = COLS / 4;   // lanes per row
  constexpr int RPI = 32 / LPR;   // rows per instruction
  constexpr int RB = 4;           // rows per load batch (per lane)
  const int c = col0 + (lane % LPR) * 4;
  const int nvalid = min(4, p.N - c);  // <= 0: a lane past the last column (still joins the shuffles)
  const bool vec = nvalid == 4 && (p.N % 4) == 0;
  const int epi = p.epi;
  float b[4] = {0.f, 0.f, 0.f, 0.f};
  if ((epi == TB_EPI_BIAS || epi == TB_EPI_BIAS_TANH || epi == TB_EPI_BIAS_SILU) && p.bias) {
#pragma unroll
    for (int j = 0; j < 4; ++j) b[j] = j < nvalid ? __ldg(p.bias + c + j) : 0.f;
  }
  float cs[4] = {0.f, 0.f, 0.f, 0.f};
  const long long plane = static_cast<long long>(p.M) * p.N;
#pragma unroll 1
  for (int r0 = lane / LPR; nvalid > 0 && r0 < 32; r0 += RPI * RB) {
    float v[RB][4];
#pragma unroll
    for (int u = 0; u < RB; ++u) v[u][0] = v[u][1] = v[u][2] = v[u][3] = 0.f;
#pragma unroll
    for (int sp = 0; sp < kMaxFixupSplits; ++sp) {
      if (sp >= p.splits) break;
#pragma unroll
      for (int u = 0; u < RB; ++u) {
        const int row = row0 + r0 + u * RPI;
        if (row >= p.M) continue;
        const float* W = p.ws + sp * plane + static_cast<long long>(row) * p.N + c;
        if (vec) {
          const float4 x = __ldcg(reinterpret_cast<const float4*>(W));
          v[u][0] += x.x;
          v[u][1] += x.y;
          v[u][2] += x.z;
          v[u][3] += x.w;
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (j < nvalid) v[u][j] += __ldcg(W + j);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < RB; ++u) {
      const int row = row0 + r0 + u * RPI;
      if (row >= p.M) continue;
      float* x = v[u];
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] += b[j];
      if (epi == TB_EPI_BIAS_TANH) {
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = fast_tanh(x[j]);
      } else if (epi == TB_EPI_BIAS_SILU) {
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = fast_silu(x[j]);
      } else if (epi == TB_EPI_RESIDUAL || epi == TB_EPI_TANH_BWD) {
        const __nv_bfloat16* a = p.aux + static_cast<long long>(row) * p.ld_aux + c;
        float h[4];
        if (nvalid == 4 && (reinterpret_cast<uintptr_t>(a) & 7) == 0) {
          const uint2 u2 = *reinterpret_cast<const uint2*>(a);
          const float2 h0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u2.x));
          const float2 h1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u2.y));
          h[0] = h0.x;
          h[1] = h0.y;
          h[2] = h1.x;
          h[3] = h1.y;
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) h[j] = j < nvalid ? __bfloat162float(a[j]) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = epi == TB_EPI_RESIDUAL ? x[j] + h[j] : x[j] * (1.f - h[j] * h[j]);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) cs[j] += x[j];
      if (p.c_fp32) {
        float* C = static_cast<float*>(p.C) + static_cast<long long>(row) * p.ldc + c;
        if (nvalid == 4 && (reinterpret_cast<uintptr_t>(C) & 15) == 0) {
          float4 o = make_float4(x[0], x[1], x[2], x[3]);
          if (p.c_add) {
            const float4 q = *reinterpret_cast<const float4*>(C);
            o.x += q.x;
            o.y += q.y;
            o.z += q.z;
            o.w += q.w;
          }
          *reinterpret_cast<float4*>(C) = o;
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (j < nvalid) C[j] = p.c_add ? C[j] + x[j] : x[j];
        }
      } else {
        __nv_bfloat16* C = static_cast<__nv_bfloat16*>(p.C) + static_cast<long long>(row) * p.ldc + c;
        if (nvalid == 4 && (reinterpret_cast<uintptr_t>(C) & 7) == 0) {
          __nv_bfloat162 lo = __floats2bfloat162_rn(x[0], x[1]), hi = __floats2bfloat162_rn(x[2], x[3]);
          uint2 o;
          o.x = *reinterpret_cast<uint32_t*>(&lo);
          o.y = *reinterpret_cast<uint32_t*>(&hi);
          *reinterpret_cast<uint2*>(C) = o;
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (j < nvalid) C[j] = __float2bfloat16_rn(x[j]);
        }
      }
    }
  }
  if (p.colsum != nullptr) {
    // lanes with the same columns hold different rows: fold them, then one atomic per column
#pragma unroll
    for (int off = LPR; off < 32; off <<= 1)
#pragma unroll
      for (int j = 0; j < 4; ++j) cs[j] += __shfl_xor_sync(0xffffffffu, cs[j], off);
    if (lane < LPR)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (j < nvalid) atomicAdd(p.colsum + c + j, cs[j]);
  }
}

// Work unit w -> (tile, K split).  Tiles run in panels of kPanel m-tiles:
// within a panel the m-tile index moves fastest, so a wave of ~148 tiles
// covers ~16 row blocks x ~9 column blocks and re-reads far less of A and B
// from DRAM than sweeping all row blocks per column block.
constexpr int kPanel = 16;
__device__ __forceinline__ void work_coords(const DevArgs& p, int w, int& m0, int& nt, int& ks, int& kb0, int& kb1) {
  const int tiles = p.m_tiles * p.n_tiles;
  const int t = w % tiles;
  ks = w / tiles;
  const int panel = t / (kPanel * p.n_tiles);
  const int within = t - panel * kPanel * p.n_tiles;
  const int gm = min(kPanel, p.m_tiles - panel * kPanel);
  const int mt = panel * kPanel + within % gm;
  nt = within / gm;
  m0 = mt * BM;
  kb0 = ks * p.kb_per_split;
  kb1 = min(p.k_blocks, kb0 + p.kb_per_split);
  if (p.kg_ntiles > 0) {  // block-diagonal B: only the K range of this tile's diagonal block
    const int g = nt / p.kg_ntiles;
    kb0 += g * p.k_blocks;
    kb1 += g * p.k_blocks;
  }
}

// 32 columns without the wait (callers batch loads, then wait once).
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// ---------------------------------------------------------------- TP helpers
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* q) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(q) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* q, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(q), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_sys_add(unsigned* q, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(q), "r"(v) : "memory");
}
// Bounded wait until *q >= target (epochs compared wrap-safe).  On timeout
// records `site` in the error word, raises the CTA's abort flag and returns false.
__device__ __forceinline__ bool tp_wait_geq(const unsigned* q, unsigned target, int* err, int site,
                                            volatile int* abort_flag) {
  const unsigned long long t0 = global_ns();
  while (static_cast<int>(ld_acquire_sys(q) - target) < 0) {
    if (*abort_flag) return false;
    if (global_ns() - t0 > kWaitBudgetNs) {
      if (err) atomicCAS(err, 0, site);
      *abort_flag = 1;
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// All-gather push split: the (peer, row, 16-byte vector) space of one rank's
// pushes, T_all = (world - 1) * rows * vpr vectors, is cut into `nw` equal
// contiguous ranges, one per push warp.  A unit of kTpSubRows rows is complete
// when every warp whose range overlaps it has arrived.
__device__ __forceinline__ long long push_begin(long long w, long long nw, long long T_all) { return w * T_all / nw; }
__device__ __forceinline__ long long push_worker_of(long long i, long long nw, long long T_all) {
  return ((i + 1) * nw - 1) / T_all;
}

// TP = 0: plain GEMM.  TP = 1: all-gather -> GEMM (rows of A are sharded over
// the ranks; remote shards arrive by peer stores into local staging).  TP = 2:
// GEMM -> reduce-scatter (each output tile is stored into the receive slot of
// the rank that owns its rows; tp_rs_finish_kernel sums the slots).  TP = 3:
// split-K with the in-kernel fix-up (a separate instantiation keeps that code
// out of the other variants' epilogue).  TP = 4: plain GEMM with the
// SwiGLU-backward epilogue (also a separate instantiation, for the same reason).
template <int BN, bool A_MN, bool B_MN, int TP>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmA3,
                        DevArgs p) {
  using S = Smem<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
  uint64_t* empty = full + S::kStages;
  uint64_t* tfull = empty + S::kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = p.m_tiles * p.n_tiles * p.splits;
  constexpr bool kTp = TP == 1 || TP == 2;  // a tensor-parallel collective variant
  if (kTp && p.tp.trace && threadIdx.x == 0) p.tp.trace[blockIdx.x * 8 + 0] = global_ns();
  const unsigned epoch = kTp ? *p.tp.epoch_ctr + 1u : 0u;
  const unsigned parity = epoch & 1u;
  const int mloc = kTp ? p.tp.rows_per_rank : 0;
  // all-gather: start with this rank's own row tiles while the remote shards arrive
  // all-gather: own rows first (they need no transfer); reduce-scatter: the
  // next rank's rows first, own rows last, so the peer stores of the first
  // wave of tiles overlap the MMAs of the later ones
  const int first_mt = TP == 1 ? (p.tp.rank * mloc) / BM
                       : TP == 2 ? (((p.tp.rank + 1) % p.tp.world) * mloc) / BM : 0;
  auto tile_m0 = [&](int m0) { return kTp ? ((m0 / BM + first_mt) % p.m_tiles) * BM : m0; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 32 * kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch(&tmA);
    tma_prefetch(&tmB);
    if (TP == 1) {
      tma_prefetch(&tmA2);
      tma_prefetch(&tmA3);
    }
  }
  if (warp == 2) tmem_alloc(tmem_slot, 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if constexpr (!kTp) {
    // launched with programmatic dependent launch: global memory only after the preceding kernel
    tb::pdl_wait();
    tb::pdl_trigger();
  }

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------ TMA producer
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    for (int w = blockIdx.x; w < total && !*abort_flag; w += gridDim.x) {
      int m0, nt, ks, kb0, kb1;
      work_coords(p, w, m0, nt, ks, kb0, kb1);
      m0 = tile_m0(m0);
      const int n0 = nt * BN;
      int a_src = 0;  // TP == 1: rank that owns these rows
      if constexpr (TP == 1) {
        a_src = m0 / mloc;
        if (a_src != p.tp.rank) {
          // the push units of this tile: complete once every push warp of
          // rank a_src whose range overlaps a unit has arrived
          const int sub0 = (m0 - a_src * mloc) / kTpSubRows;
          const unsigned* rdy = p.tp.hdr[p.tp.rank]->ready[parity][a_src];
          if (p.tp.trace && p.tp.trace[blockIdx.x * 8 + 3] == 0) p.tp.trace[blockIdx.x * 8 + 3] = global_ns();
          const long long vpr = p.K / 8, T = static_cast<long long>(mloc) * vpr;
          const long long T_all = (p.tp.world - 1) * T, nw = 2ll * gridDim.x;  // every rank runs the same grid
          const int pi = p.tp.rank < a_src ? p.tp.rank : p.tp.rank - 1;     // this rank's index among a_src's peers
          bool ok = true;
          for (int j = 0; j < BM / kTpSubRows && ok; ++j) {
            const long long lo = pi * T + static_cast<long long>(sub0 + j) * kTpSubRows * vpr;
            const long long hi = lo + kTpSubRows * vpr - 1;
            const unsigned need = static_cast<unsigned>(push_worker_of(hi, nw, T_all) - push_worker_of(lo, nw, T_all) + 1);
            ok = tp_wait_geq(rdy + sub0 + j, need, p.tp.err, 11, abort_flag);
          }
          if (!ok) break;
          asm volatile("fence.proxy.async.global;" ::: "memory");  // peer stores -> TMA reads
          if (p.tp.trace && p.tp.trace[blockIdx.x * 8 + 4] == 0) p.tp.trace[blockIdx.x * 8 + 4] = global_ns();
        }
      }
      // packed block-diagonal B: its inner coordinate is local to the block
      const int goff = p.kg_packed ? (nt / p.kg_ntiles) * p.k_blocks * BK : 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) break;
        uint8_t* sa = smem + stage * S::kStageBytes;
        uint8_t* sb = sa + S::kABytes;
        mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
        const int k0 = kb * BK;
        if (A_MN) {
#pragma unroll
          for (int j = 0; j < BM / 64; ++j) tma_load_2d(sa + j * 64 * BK * 2, &tmA, &full[stage], m0 + 64 * j, k0);
        } else if (TP == 1) {
          if (a_src == p.tp.rank) tma_load_2d(sa, &tmA, &full[stage], k0, m0 - a_src * mloc);
          else tma_load_2d(sa, parity ? &tmA3 : &tmA2, &full[stage], k0, m0);
        } else {
          tma_load_2d(sa, &tmA, &full[stage], k0, m0);
        }
        if (B_MN) {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            tma_load_2d(sb + j * 64 * BK * 2, &tmB, &full[stage], n0 - goff + 64 * j, k0);
        } else {
          tma_load_2d(sb, &tmB, &full[stage], k0 - goff, n0);
        }
        ++issued;
        if (++stage == S::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    if (*abort_flag) {
      // drain: wait (bounded) for the loads of the last min(issued, stages) stages
      const int n = issued < S::kStages ? issued : S::kStages;
      int st = stage;
      uint32_t ph = phase;
      for (int i = 0; i < n; ++i) {
        if (--st < 0) {
          st = S::kStages - 1;
          ph ^= 1;
        }
        const unsigned long long t0 = global_ns();
        while (!mbar_try_wait(&full[st], ph) && global_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_bf16(BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool any = false;
    for (int w = blockIdx.x; w < total && !*abort_flag; w += gridDim.x) {
      int m0, nt, ks, kb0, kb1;
      work_coords(p, w, m0, nt, ks, kb0, kb1);
      if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) break;
      tc_fence_after();
      const uint32_t d = tmem_base + acc * BN;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + stage * S::kStageBytes);
        const uint32_t sb = sa + S::kABytes;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // K-major: +32 bytes per K=16 step inside the 128-byte swizzle atom.
          // MN-major: +2048 bytes (two 8-row K groups) per step; 64-wide MN
          // blocks are 64*BK*2 bytes apart (LBO).
          const uint64_t ad = A_MN ? smem_desc_sw128(sa + kk * 2048, 64 * BK * 2, 1024)
                                   : smem_desc_sw128(sa + kk * 32, 16, 1024);
          const uint64_t bd = B_MN ? smem_desc_sw128(sb + kk * 2048, 64 * BK * 2, 1024)
                                   : smem_desc_sw128(sb + kk * 32, 16, 1024);
          mma_f16(d, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&empty[stage]);
        any = true;
        if (++stage == S::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      mma_commit(&tfull[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    // make sure every MMA this thread issued has finished before TMEM is freed
    if (any) {
      mma_commit(drain);
      const unsigned long long t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < 1000000000ull) {
      }
    }
  } else if (TP == 1 && (warp == 2 || warp == 3)) {
    // ------------------------------------------------ all-gather push (warps 2, 3)
    // Unit u (8 rows of this rank's shard, for one peer) goes into that peer's
    // staging by peer stores over NVLink (16 16-byte loads in flight per lane),
    // then one release flag per unit.
    if constexpr (TP == 1) {
      const int W = p.tp.world, r = p.tp.rank, K = p.K;
      const long long vpr = K / 8, T = static_cast<long long>(mloc) * vpr, T_all = (W - 1) * T;
      const long long nw = 2ll * gridDim.x, wk = 2ll * blockIdx.x + (warp - 2);
      const long long b0 = push_begin(wk, nw, T_all), b1 = push_begin(wk + 1, nw, T_all);
      if (b1 > b0) {
        // the peers have finished reading this parity's staging from two calls ago
        int ok = 1;
        if (lane == 0 && epoch > 2u)
          for (int o = 0; o < W && ok; ++o)
            if (o != r) ok = tp_wait_geq(&p.tp.hdr[r]->consumed[o], epoch - 2u, p.tp.err, 12, abort_flag) ? 1 : 0;
        if (__shfl_sync(0xffffffffu, ok, 0)) {
          const char* src_base = reinterpret_cast<const char*>(p.tp.shard);
          constexpr int kDepth = 16;
          for (long long e0 = b0 + lane; e0 < b1; e0 += 32 * kDepth) {
            uint4 v[kDepth];
            uint32_t pk[kDepth], rw[kDepth], cc[kDepth];  // peer index, row, vector column (32-bit: T_all < 2^31)
#pragma unroll
            for (int q = 0; q < kDepth; ++q) {
              const uint32_t e = static_cast<uint32_t>(e0 + q * 32);
              pk[q] = e / static_cast<uint32_t>(T);
              const uint32_t within = e - pk[q] * static_cast<uint32_t>(T);
              rw[q] = within / static_cast<uint32_t>(vpr);
              cc[q] = within - rw[q] * static_cast<uint32_t>(vpr);
              if (e0 + q * 32 < b1)
                v[q] = *reinterpret_cast<const uint4*>(src_base + (rw[q] * p.tp.ld_shard + cc[q] * 8ll) * 2);
            }
#pragma unroll
            for (int q = 0; q < kDepth; ++q) {
              if (e0 + q * 32 < b1) {
                const int peer = static_cast<int>(pk[q]) >= r ? static_cast<int>(pk[q]) + 1 : static_cast<int>(pk[q]);
                __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.tp.data[peer] + parity * p.tp.parity_bytes);
                *reinterpret_cast<uint4*>(dst + (static_cast<long long>(r) * mloc + rw[q]) * K + cc[q] * 8) = v[q];
              }
            }
          }
          asm volatile("fence.acq_rel.sys;" ::: "memory");
          __syncwarp();
          // one arrival per unit this range touched
          const long long u_first = b0 / (kTpSubRows * vpr), u_last = (b1 - 1) / (kTpSubRows * vpr);
          for (long long u = u_first + lane; u <= u_last; u += 32) {  // u indexes (peer, unit) pairs
            const int nsub = mloc / kTpSubRows;
            const int pi = static_cast<int>(u / nsub), sub = static_cast<int>(u % nsub);
            const int peer = pi >= r ? pi + 1 : pi;
            red_release_sys_add(&p.tp.hdr[peer]->ready[parity][r][sub], 1u);
          }
        }
      }
      if (p.tp.trace && lane == 0) p.tp.trace[blockIdx.x * 8 + 1 + (warp - 2)] = global_ns();
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ epilogue: 8 warps; warp (4 + q + 4h)
    // reads TMEM lane quarter q (rows 32q..32q+31) and column half h.
    const int sub = warp & 3;
    const int half = (warp - 4) >> 2;
    const int r_in_tile = sub * 32 + lane;
    uint32_t* stg = reinterpret_cast<uint32_t*>(smem + S::kStgOffset) + (warp - 4) * 32 * S::kStgWords;
    int acc = 0;
    uint32_t acc_phase = 0;
    const int mode = p.ws != nullptr ? kEpiPartial : kEpiFull;
    unsigned rs_ready = epoch <= 2u ? 0xffffffffu : 0u;  // bit o: rank o's slots may be written
    for (int w = blockIdx.x; w < total; w += gridDim.x) {
      int m0, nt, ks, kb0, kb1;
      work_coords(p, w, m0, nt, ks, kb0, kb1);
      m0 = tile_m0(m0);
      const int n0 = nt * BN;
      void* cbase = p.C;
      if constexpr (TP == 2) {
        // this tile's rows belong to rank `o`: store into o's receive slot for
        // this source rank, addressed so that the global row index applies
        const int o = m0 / mloc;
        if (!((rs_ready >> o) & 1u)) {  // o has finished reading this parity's slots from two calls ago
          int ok = 1;
          if (lane == 0) ok = tp_wait_geq(&p.tp.hdr[p.tp.rank]->rs_consumed[o], epoch - 2u, p.tp.err, 13, abort_flag);
          if (!__shfl_sync(0xffffffffu, ok, 0)) break;
          rs_ready |= 1u << o;
        }
        cbase = p.tp.data[o] + parity * p.tp.parity_bytes +
                (static_cast<long long>(p.tp.rank) - o) * mloc * p.N * 2;
      }
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag)) break;
      tc_fence_after();
      const int row = m0 + r_in_tile;
      const uint32_t base = tmem_base + acc * BN + (static_cast<uint32_t>(sub * 32) << 16);
      constexpr int kStep = BN / 2 >= 64 ? 64 : 32;  // columns per TMEM load batch
      // epilogues that read an aux matrix: issue this row's aux loads before
      // the TMEM loads so the two latencies overlap
      const bool aux_rows = (p.epi == TB_EPI_TANH_BWD || p.epi == TB_EPI_RESIDUAL) && mode != kEpiPartial &&
                            row < p.M;
#pragma unroll 1
      for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += kStep) {
        uint4 ax[kStep / 8];
        bool pre = false;
        if (aux_rows && n0 + c + kStep <= p.N) {
          const __nv_bfloat16* a = p.aux + static_cast<long long>(row) * p.ld_aux + n0 + c;
          if ((reinterpret_cast<uintptr_t>(a) & 15) == 0) {
            pre = true;
#pragma unroll
            for (int q = 0; q < kStep / 8; ++q) ax[q] = reinterpret_cast<const uint4*>(a)[q];
          }
        }
        uint32_t r[64];
        tmem_ld32_nowait(base + c, r);
        if constexpr (kStep == 64) tmem_ld32_nowait(base + c + 32, r + 32);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (n0 + c < p.N)
          epilogue32<TP == 4>(p, row, n0 + c, v, ks, lane, stg, m0 + sub * 32, mode, cbase, pre, ax[0], ax[1], ax[2],
                              ax[3]);
        if constexpr (kStep == 64) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[32 + j]);
          if (n0 + c + 32 < p.N)
            epilogue32<TP == 4>(p, row, n0 + c + 32, v, ks, lane, stg, m0 + sub * 32, mode, cbase, pre, ax[kStep / 8 - 4],
                       ax[kStep / 8 - 3], ax[kStep / 8 - 2], ax[kStep / 8 - 1]);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
      if constexpr (TP == 3) {
        // In-kernel split-K fix-up, per warp slice (32 rows x BN/2 columns):
        // publish this split's partial, count arrivals, and let the last of
        // the `splits` warps that own the slice sum every partial (in split
        // order, so the result does not depend on arrival order) and run the
        // full epilogue.  Warp-local: no barrier across warps, no waiting.
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          const int slot = (w % (p.m_tiles * p.n_tiles)) * kEpiWarps + (warp - 4);
          last = atomicAdd(p.slot_cnt + slot, 1) == p.splits - 1;
          if (last) atomicExch(p.slot_cnt + slot, 0);  // leave the counter zero for the next launch
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence();
          fixup_slice<BN / 2>(p, m0 + sub * 32, n0 + half * (BN / 2), lane);
        }
      }
    }
  }
  if (TP == 2 && warp >= 4) __threadfence_system();  // this thread's peer stores, before the arrival below
  if (kTp && p.tp.trace && threadIdx.x == 128) p.tp.trace[blockIdx.x * 8 + 5] = global_ns();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem_base, 2 * BN);
  if (threadIdx.x == 0 && *abort_flag && p.error) atomicCAS(p.error, 0, TB_GEMM_ERR_TIMEOUT);  // keeps a site code
  if constexpr (TP == 1) {
    if (p.tp.gather_out != nullptr) {
      // Copy-out of the gathered A (a training backward needs it for the weight
      // gradient): each warp copies whole push units, own rows from the shard,
      // remote rows from this rank's staging once the unit's arrivals are
      // complete.  It runs before this CTA counts itself done, so no peer can
      // refill this parity's staging underneath it.
      const int W = p.tp.world, r = p.tp.rank, K = p.K;
      const long long vpr = K / 8, T = static_cast<long long>(mloc) * vpr;
      const long long T_all = (W - 1) * T, nw = 2ll * gridDim.x;
      constexpr int kWarps = kThreads / 32;
      const int units = p.M / kTpSubRows;
      const __nv_bfloat16* staged =
          reinterpret_cast<const __nv_bfloat16*>(p.tp.data[r] + parity * p.tp.parity_bytes);
      for (int u = blockIdx.x * kWarps + warp; u < units; u += gridDim.x * kWarps) {
        int go = lane == 0 ? (*abort_flag ? 0 : 1) : 0;
        const int row0 = u * kTpSubRows, src = row0 / mloc;
        const __nv_bfloat16* from = staged + static_cast<long long>(row0) * K;
        long long ld = K;
        if (src == r) {
          from = p.tp.shard + static_cast<long long>(row0 - r * mloc) * p.tp.ld_shard;
          ld = p.tp.ld_shard;
        } else if (lane == 0 && go) {
          const int sub = (row0 - src * mloc) / kTpSubRows;
          const int pi = r < src ? r : r - 1;  // this rank's index among src's peers
          const long long lo = pi * T + static_cast<long long>(sub) * kTpSubRows * vpr;
          const long long hi = lo + kTpSubRows * vpr - 1;
          const unsigned need = static_cast<unsigned>(push_worker_of(hi, nw, T_all) - push_worker_of(lo, nw, T_all) + 1);
          go = tp_wait_geq(&p.tp.hdr[r]->ready[parity][src][sub], need, p.tp.err, 15, abort_flag) ? 1 : 0;
        }
        if (!__shfl_sync(0xffffffffu, go, 0)) break;
        for (long long e = lane; e < kTpSubRows * vpr; e += 32) {
          const long long i = e / vpr, c = e - i * vpr;
          const uint4 v = __ldcg(reinterpret_cast<const uint4*>(from + i * ld + c * 8));
          *reinterpret_cast<uint4*>(p.tp.gather_out + (row0 + i) * p.tp.ld_gather + c * 8) = v;
        }
      }
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      // the last CTA: every CTA has finished reading staging -> tell the peers
      __threadfence();
      if (atomicAdd(p.tp.done_ctr, 1u) == gridDim.x - 1) {
        *p.tp.done_ctr = 0;
        // reset this parity's arrival counters (every CTA has consumed them)
        const int nsub = mloc / kTpSubRows;
        for (int o = 0; o < p.tp.world; ++o)
          if (o != p.tp.rank)
            for (int u = 0; u < nsub; ++u) p.tp.hdr[p.tp.rank]->ready[parity][o][u] = 0u;
        __threadfence();
        for (int o = 0; o < p.tp.world; ++o)
          if (o != p.tp.rank) st_release_sys(&p.tp.hdr[o]->consumed[p.tp.rank], epoch);
        *p.tp.epoch_ctr = epoch;
      }
    }
  } else if constexpr (TP == 2) {
    if (threadIdx.x == 0) {
      __threadfence_system();
      for (int o = 0; o < p.tp.world; ++o) red_release_sys_add(&p.tp.hdr[o]->rs_arrivals[parity], 1u);
    }
  }
}

// C = sum over splits of the partials, then the epilogue (bias, activation,
// residual add or tanh backward).  A block owns 64
// float4 column groups of the output; its 4 warps-groups each sum every 4th
// partial with 4 loads in flight, then combine through shared memory, so the
// pass streams the workspace at bandwidth instead of walking the splits
// serially.
constexpr int kRedItems = 64, kRedGroups = 4;
__global__ void __launch_bounds__(kRedItems* kRedGroups) splitk_reduce_kernel(DevArgs p) {
  __shared__ float4 part[kRedGroups][kRedItems];
  const int n4 = (p.N + 3) / 4;
  const long long items = static_cast<long long>(p.M) * n4;
  const int li = threadIdx.x % kRedItems, g = threadIdx.x / kRedItems;
  const long long item = static_cast<long long>(blockIdx.x) * kRedItems + li;
  const bool vec = (p.N % 4) == 0;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  int row = 0, c = 0, valid = 0;
  if (item < items) {
    row = static_cast<int>(item / n4);
    c = static_cast<int>(item - static_cast<long long>(row) * n4) * 4;
    valid = min(4, p.N - c);
    const long long stride = static_cast<long long>(p.M) * p.N;
    const float* W = p.ws + static_cast<long long>(row) * p.N + c;
    int k = g;
    for (; k + 3 * kRedGroups < p.splits; k += 4 * kRedGroups) {
      float4 x[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float* q = W + (k + u * kRedGroups) * stride;
        x[u] = vec ? *reinterpret_cast<const float4*>(q)
                   : make_float4(q[0], valid > 1 ? q[1] : 0.f, valid > 2 ? q[2] : 0.f, valid > 3 ? q[3] : 0.f);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        acc.x += x[u].x;
        acc.y += x[u].y;
        acc.z += x[u].z;
        acc.w += x[u].w;
      }
    }
    for (; k < p.splits; k += kRedGroups) {
      const float* q = W + k * stride;
      const float4 x = vec ? *reinterpret_cast<const float4*>(q)
                           : make_float4(q[0], valid > 1 ? q[1] : 0.f, valid > 2 ? q[2] : 0.f, valid > 3 ? q[3] : 0.f);
      acc.x += x.x;
      acc.y += x.y;
      acc.z += x.z;
      acc.w += x.w;
    }
  }
  part[g][li] = acc;
  __syncthreads();
  if (g != 0 || item >= items) return;
#pragma unroll
  for (int q = 1; q < kRedGroups; ++q) {
    acc.x += part[q][li].x;
    acc.y += part[q][li].y;
    acc.z += part[q][li].z;
    acc.w += part[q][li].w;
  }
  const float s[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (j >= valid) continue;
    float v = s[j];
    if ((p.epi == TB_EPI_BIAS || p.epi == TB_EPI_BIAS_TANH || p.epi == TB_EPI_BIAS_SILU) && p.bias) v += p.bias[c + j];
    if (p.epi == TB_EPI_BIAS_TANH) v = fast_tanh(v);
    if (p.epi == TB_EPI_BIAS_SILU) v = fast_silu(v);
    if (p.epi == TB_EPI_RESIDUAL || p.epi == TB_EPI_TANH_BWD) {
      const float h = __bfloat162float(p.aux[static_cast<long long>(row) * p.ld_aux + c + j]);
      v = p.epi == TB_EPI_RESIDUAL ? v + h : v * (1.f - h * h);
    }
    if (p.colsum) atomicAdd(p.colsum + c + j, v);
    if (p.c_fp32) {
      float* C = static_cast<float*>(p.C) + static_cast<long long>(row) * p.ldc + c + j;
      if (p.c_add) *C += v;
      else *C = v;
    } else {
      static_cast<__nv_bfloat16*>(p.C)[static_cast<long long>(row) * p.ldc + c + j] = __float2bfloat16_rn(v);
    }
  }
}

// --------------------------------------------------------------------------
// host side: tensor maps through the driver entry point (no libcuda link)
// --------------------------------------------------------------------------
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

// 2D bf16 row-major matrix [rows, cols] with leading dimension ld (elements);
// box = {64 cols, box_rows}, 128-byte swizzle, zero fill out of bounds.
bool make_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long ld, int box_rows) {
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

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// Tile width and split count.  When K may be split (a workspace or atomics
// are available), BN = 256 and K is split if the tiles cover less than half
// the SMs, into as many splits as fit in one wave, each keeping at least 4
// k-blocks.  Otherwise BN = 256 unless the 256-wide tiles would not cover the
// SMs once; then 128, or 64 if 128-wide tiles would not cover half of them
// (narrow tiles multiply the CTAs that stream operands, which is what bounds
// GEMMs with few rows such as decode-time projections).
struct Plan {
  int BN, m_tiles, n_tiles, k_blocks, splits;
};
Plan make_plan(int M, int N, int K, int bn_hint, int split_k, bool can_split, size_t ws_bytes) {
  Plan pl{};
  const int sms = num_sms();
  pl.m_tiles = (M + BM - 1) / BM;
  pl.k_blocks = (K + BK - 1) / BK;
  if (bn_hint == 64 || bn_hint == 128 || bn_hint == 256) {
    pl.BN = bn_hint;
  } else {
    pl.BN = N > 128 ? 256 : 128;
    // narrow tiles only where K will not be split (splitting keeps the wide,
    // more efficient tiles busy instead)
    const bool may_split = split_k > 1 || (split_k <= 0 && can_split);
    if (!may_split) {
      if (pl.BN == 256 && pl.m_tiles * ((N + 255) / 256) < sms) pl.BN = 128;
      if (pl.BN == 128 && N > 64 && pl.m_tiles * ((N + 127) / 128) < sms / 2) pl.BN = 64;
    }
  }
  pl.n_tiles = (N + pl.BN - 1) / pl.BN;
  const int tiles = pl.m_tiles * pl.n_tiles;
  int splits = split_k;
  if (splits <= 0) {
    splits = 1;
    if (can_split && tiles < sms / 2) {
      splits = sms / tiles;
      const int max_s = (pl.k_blocks + 3) / 4;
      if (splits > max_s) splits = max_s;
      const size_t per_split = sizeof(float) * static_cast<size_t>(M) * N;
      if (ws_bytes != 0 && ws_bytes != static_cast<size_t>(-1)) {
        const size_t fit = ws_bytes > kCntBytes ? (ws_bytes - kCntBytes) / per_split : 0;
        if (static_cast<size_t>(splits) > fit && fit >= 2) splits = static_cast<int>(fit);  // prefer partials over atomics
      }
      if (splits < 1) splits = 1;
    }
  }
  pl.splits = splits;
  return pl;
}

template <int BN, bool A_MN, bool B_MN, int TP = 0>
int launch(const CUtensorMap& ta, const CUtensorMap& tbm, const DevArgs& p, int grid, cudaStream_t s,
           const CUtensorMap* ta2 = nullptr, const CUtensorMap* ta3 = nullptr) {
  using S = Smem<BN>;
  auto k = gemm_tcgen05_kernel<BN, A_MN, B_MN, TP>;
  tb::ensure_dyn_smem(reinterpret_cast<const void*>(k), S::kTotal);
  if constexpr (TP != 1 && TP != 2) {
    // single-GPU variants: programmatic dependent launch (the prologue overlaps the previous kernel)
    return static_cast<int>(tb::launch_pdl(k, dim3(grid), dim3(kThreads), S::kTotal, s, ta, tbm,
                                           ta2 ? *ta2 : ta, ta3 ? *ta3 : ta, p));
  }
  k<<<grid, kThreads, S::kTotal, s>>>(ta, tbm, ta2 ? *ta2 : ta, ta3 ? *ta3 : ta, p);
  return static_cast<int>(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Reduce-scatter finish: out[Mloc, N] = sum over source ranks of this rank's
// receive slots (+ bias, + residual), once every CTA of every rank's GEMM has
// arrived.  Then tells the peers that the slots of this parity may be reused.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) tp_rs_finish_kernel(TpArgs t, int N, const float* __restrict__ bias,
                                                           const __nv_bfloat16* __restrict__ res, long long ld_res,
                                                           __nv_bfloat16* __restrict__ out, long long ldo,
                                                           unsigned* tgt, unsigned add) {
  const unsigned epoch = *t.epoch_ctr + 1u, parity = epoch & 1u;
  const unsigned target = tgt[parity] + add;
  __shared__ int s_ok;
  __shared__ int s_abort;
  if (threadIdx.x == 0) {
    s_abort = 0;
    s_ok = tp_wait_geq(&t.hdr[t.rank]->rs_arrivals[parity], target, t.err, 14,
                       reinterpret_cast<volatile int*>(&s_abort)) ? 1 : 0;
  }
  __syncthreads();
  const int W = t.world, mloc = t.rows_per_rank;
  if (s_ok) {
    const char* base = t.data[t.rank] + parity * t.parity_bytes;
    const long long slot = static_cast<long long>(mloc) * N;  // elements per source slot
    const long long nvec = slot / 8;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < nvec;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
      const long long e = i * 8;
      const int row = static_cast<int>(e / N), col = static_cast<int>(e - static_cast<long long>(row) * N);
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int src = 0; src < W; ++src) {
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(base) + src * (slot / 8) + i);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __bfloat1622float2(h[k]);
          acc[2 * k] += f.x;
          acc[2 * k + 1] += f.y;
        }
      }
      if (bias) {
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] += bias[col + k];
      }
      if (res) {
        const uint4 u = *reinterpret_cast<const uint4*>(res + row * ld_res + col);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __bfloat1622float2(h[k]);
          acc[2 * k] += f.x;
          acc[2 * k + 1] += f.y;
        }
      }
      uint4 o;
      __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int k = 0; k < 4; ++k) oh[k] = __floats2bfloat162_rn(acc[2 * k], acc[2 * k + 1]);
      *reinterpret_cast<uint4*>(out + row * ldo + col) = o;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(t.done_ctr, 1u) == gridDim.x - 1) {
      *t.done_ctr = 0;
      for (int o = 0; o < W; ++o) st_release_sys(&t.hdr[o]->rs_consumed[t.rank], epoch);  // self included
      tgt[parity] = target;
      *t.epoch_ctr = epoch;
    }
  }
}

unsigned long long* g_tp_trace = nullptr;

bool fill_tp(TpArgs* tp, const TbTpComm* c) {
  if (c->world < 1 || c->world > kTpMaxRanks || c->rank < 0 || c->rank >= c->world) return false;
  tp->rank = c->rank;
  tp->world = c->world;
  tp->rows_per_rank = c->rows_per_rank;
  tp->epoch_ctr = c->epoch_ctr;
  tp->done_ctr = c->done_ctr;
  for (int i = 0; i < kTpMaxRanks; ++i) {
    tp->hdr[i] = static_cast<TpHdr*>(c->hdr[i]);
    tp->data[i] = static_cast<char*>(c->data[i]);
  }
  tp->parity_bytes = c->parity_bytes;
  tp->err = c->err;
  tp->trace = g_tp_trace;
  tp->gather_out = static_cast<__nv_bfloat16*>(c->gather_out);
  tp->ld_gather = c->ld_gather;
  return true;
}

}  // namespace

extern "C" {

int tb_gemm_bf16(const TbGemmArgs* a, cudaStream_t stream) {
  if (a->M <= 0 || a->N <= 0) return 0;
  if (a->K <= 0) return static_cast<int>(cudaErrorInvalidValue);
  // TMA: row strides must be multiples of 16 bytes, base 16-byte aligned.
  if ((a->lda % 8) || (a->ldb % 8) || (reinterpret_cast<uintptr_t>(a->A) & 15) ||
      (reinterpret_cast<uintptr_t>(a->B) & 15))
    return static_cast<int>(cudaErrorInvalidValue);
  const bool swiglu = a->epi == TB_EPI_SWIGLU;
  const bool swiglu_bwd = a->epi == TB_EPI_SWIGLU_BWD;
  if (swiglu && ((a->N % 2) || a->colsum)) return static_cast<int>(cudaErrorInvalidValue);
  if (swiglu_bwd && (a->a_mn || a->c_fp32 || a->aux == nullptr || a->colsum || a->c_accumulate || (a->ld_aux % 8) ||
                     (reinterpret_cast<uintptr_t>(a->aux) & 15)))
    return static_cast<int>(cudaErrorInvalidValue);
  if (a->C2 && (!swiglu || (a->ldc2 % 8) || (reinterpret_cast<uintptr_t>(a->C2) & 15)))
    return static_cast<int>(cudaErrorInvalidValue);
  const bool ws_epi_ok = !swiglu && !swiglu_bwd;
  const bool atomic_ok = a->c_fp32 && (a->epi == TB_EPI_NONE || a->epi == TB_EPI_BIAS) && !a->colsum;
  const bool have_ws = a->workspace != nullptr && ws_epi_ok &&
                       a->workspace_bytes >= kCntBytes + 2 * sizeof(float) * static_cast<size_t>(a->M) * a->N;
  const int kg = a->kgroup;
  if (kg != 0 && (kg < 0 || kg % 64 || a->N % kg || a->K != a->N || swiglu || swiglu_bwd))
    return static_cast<int>(cudaErrorInvalidValue);
  // block-diagonal B: the tile width must divide the block, K is one block
  int bn_hint = a->bn_hint;
  if (kg && (bn_hint == 0 || kg % bn_hint)) bn_hint = kg % 256 == 0 ? 256 : (kg % 128 == 0 ? 128 : 64);
  const Plan pl = make_plan(a->M, a->N, kg ? kg : a->K, bn_hint, a->split_k, have_ws || atomic_ok,
                            have_ws ? a->workspace_bytes : 0);
  const int BN = pl.BN;
  CUtensorMap ta, tbm;
  // A: K-major -> matrix [M, K]; MN-major -> matrix [K, M]
  const bool okA = a->a_mn ? make_map(&ta, a->A, a->K, a->M, a->lda, BK) : make_map(&ta, a->A, a->M, a->K, a->lda, BM);
  // packed block-diagonal B: its inner dimension is one block (kg) wide
  const int b_inner_n = kg && a->kgroup_packed ? kg : a->N, b_inner_k = kg && a->kgroup_packed ? kg : a->K;
  const bool okB = a->b_mn ? make_map(&tbm, a->B, a->K, b_inner_n, a->ldb, BK)
                           : make_map(&tbm, a->B, a->N, b_inner_k, a->ldb, BN);
  if (!okA || !okB) return static_cast<int>(cudaErrorInvalidValue);

  DevArgs p{};
  p.M = a->M;
  p.N = a->N;
  p.K = a->K;
  p.m_tiles = pl.m_tiles;
  p.n_tiles = pl.n_tiles;
  p.k_blocks = pl.k_blocks;
  const int tiles = p.m_tiles * p.n_tiles;
  const size_t per_split = sizeof(float) * static_cast<size_t>(a->M) * a->N;
  p.kb_per_split = (p.k_blocks + pl.splits - 1) / pl.splits;
  p.splits = (p.k_blocks + p.kb_per_split - 1) / p.kb_per_split;
  // split-K: partials go to the caller's workspace (summed in-kernel by the
  // last warp to finish a slice, or by one reduce pass for many splits), or,
  // without a workspace, atomically into an fp32 C
  const bool use_ws = p.splits > 1 && have_ws && kCntBytes + static_cast<size_t>(p.splits) * per_split <= a->workspace_bytes;
  const bool fixup = use_ws && p.splits <= kMaxFixupSplits && tiles * kEpiWarps <= kCntSlots;
  if (p.splits > 1 && !use_ws && !atomic_ok) return static_cast<int>(cudaErrorInvalidValue);
  p.C = a->C;
  p.ldc = a->ldc;
  p.c_fp32 = a->c_fp32;
  p.c_atomic = (p.splits > 1 && !use_ws) ? 1 : 0;
  p.c_add = (a->c_accumulate && !p.c_atomic && (!use_ws || fixup)) ? 1 : 0;
  if ((p.c_atomic || a->c_accumulate) && !a->c_fp32) return static_cast<int>(cudaErrorInvalidValue);
  if (p.splits > 1 && !use_ws && !a->c_accumulate) {
    // atomic split-K adds partial sums into a zeroed C
    if (a->ldc == a->N) {
      cudaMemsetAsync(a->C, 0, per_split, stream);
    } else {
      cudaMemset2DAsync(a->C, sizeof(float) * a->ldc, 0, sizeof(float) * a->N, a->M, stream);
    }
  }
  if (a->colsum) cudaMemsetAsync(a->colsum, 0, sizeof(float) * a->N, stream);
  p.bias = a->bias;
  p.aux = static_cast<const __nv_bfloat16*>(a->aux);
  p.ld_aux = a->ld_aux;
  p.epi = a->epi;
  p.alpha = a->alpha == 0.f ? 1.f : a->alpha;
  p.ws = use_ws ? reinterpret_cast<float*>(static_cast<char*>(a->workspace) + kCntBytes) : nullptr;
  p.slot_cnt = fixup ? static_cast<int*>(a->workspace) : nullptr;
  p.colsum = (use_ws && !fixup) ? nullptr : a->colsum;
  p.error = a->error;
  p.c2 = static_cast<__nv_bfloat16*>(a->C2);
  p.ldc2 = a->ldc2;
  p.kg_ntiles = kg ? kg / BN : 0;
  p.kg_packed = kg && a->kgroup_packed ? 1 : 0;
  const int total = tiles * p.splits;
  const int grid = total < num_sms() ? total : num_sms();
  const int am = a->a_mn ? 1 : 0, bm = a->b_mn ? 1 : 0;
  int err = 0;
#define TB_GEMM_DISPATCH2(BNV, MODE)                                                   \
  if (!am && !bm) err = launch<BNV, false, false, MODE>(ta, tbm, p, grid, stream);     \
  else if (!am && bm) err = launch<BNV, false, true, MODE>(ta, tbm, p, grid, stream);  \
  else if (am && !bm) err = launch<BNV, true, false, MODE>(ta, tbm, p, grid, stream);  \
  else err = launch<BNV, true, true, MODE>(ta, tbm, p, grid, stream);
#define TB_GEMM_DISPATCH(BNV)                                                      \
  if (swiglu_bwd) {                                                                \
    if (am) return static_cast<int>(cudaErrorInvalidValue);                        \
    err = bm ? launch<BNV, false, true, 4>(ta, tbm, p, grid, stream)               \
             : launch<BNV, false, false, 4>(ta, tbm, p, grid, stream);             \
  } else if (fixup) {                                                              \
    TB_GEMM_DISPATCH2(BNV, 3)                                                      \
  } else {                                                                         \
    TB_GEMM_DISPATCH2(BNV, 0)                                                      \
  }
  if (BN == 256) {
    TB_GEMM_DISPATCH(256)
  } else if (BN == 128) {
    TB_GEMM_DISPATCH(128)
  } else {
    TB_GEMM_DISPATCH(64)
  }
#undef TB_GEMM_DISPATCH
#undef TB_GEMM_DISPATCH2
  if (err != 0 || !use_ws || fixup) return err;
  DevArgs r = p;
  r.colsum = a->colsum;
  r.c_atomic = 0;
  r.c_add = a->c_accumulate ? 1 : 0;
  const long long work = static_cast<long long>(a->M) * ((a->N + 3) / 4);
  const long long g = (work + kRedItems - 1) / kRedItems;
  splitk_reduce_kernel<<<static_cast<unsigned>(g), kRedItems * kRedGroups, 0, stream>>>(r);
  return static_cast<int>(cudaGetLastError());
}

size_t tb_gemm_workspace_bytes(int M, int N, int K) {
  // enough for the automatic tile width and split count of this shape
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const Plan pl = make_plan(M, N, K, 0, 0, true, static_cast<size_t>(-1));
  if (pl.splits < 2) return 0;
  return kCntBytes + sizeof(float) * static_cast<size_t>(M) * N * pl.splits;
}

size_t tb_tp_header_bytes(void) { return (sizeof(TpHdr) + 4095) / 4096 * 4096; }

#define TB_TP_DISPATCH(TPV, BNV, BMN)                                                                \
  (BMN ? launch<BNV, false, true, TPV>(ta, tbm, p, grid, stream, &ta2, &ta3)                       \
       : launch<BNV, false, false, TPV>(ta, tbm, p, grid, stream, &ta2, &ta3))

int tb_tp_ag_gemm(const TbTpComm* c, const TbGemmArgs* a, cudaStream_t stream) {
  const int W = c->world, mloc = c->rows_per_rank;
  if (a->M <= 0 || a->N <= 0) return 0;
  if (a->epi == TB_EPI_SWIGLU_BWD || (a->C2 && a->epi != TB_EPI_SWIGLU))
    return static_cast<int>(cudaErrorInvalidValue);
  if (a->a_mn || a->K <= 0 || a->K % 8 || a->lda % 8 || a->ldb % 8 || mloc % BM || a->M != W * mloc ||
      mloc / kTpSubRows > kTpMaxSub || a->workspace || a->colsum || a->c_accumulate ||
      c->parity_bytes < 2ll * a->M * a->K || c->parity_bytes % 16 || (reinterpret_cast<uintptr_t>(a->A) & 15) ||
      (reinterpret_cast<uintptr_t>(a->B) & 15) ||
      (c->gather_out && ((reinterpret_cast<uintptr_t>(c->gather_out) & 15) || c->ld_gather % 8 || c->ld_gather < a->K)))
    return static_cast<int>(cudaErrorInvalidValue);
  const Plan pl = make_plan(a->M, a->N, a->K, a->bn_hint, 1, false, 0);
  const int BN = pl.BN;
  if (g_tp_trace) cudaMemsetAsync(g_tp_trace, 0, 148 * 8 * 8, stream);
  CUtensorMap ta, ta2, ta3, tbm;
  const bool ok = make_map(&ta, a->A, mloc, a->K, a->lda, BM) &&
                  make_map(&ta2, c->data[c->rank], a->M, a->K, a->K, BM) &&
                  make_map(&ta3, static_cast<char*>(c->data[c->rank]) + c->parity_bytes, a->M, a->K, a->K, BM) &&
                  (a->b_mn ? make_map(&tbm, a->B, a->K, a->N, a->ldb, BK) : make_map(&tbm, a->B, a->N, a->K, a->ldb, BN));
  if (!ok) return static_cast<int>(cudaErrorInvalidValue);
  DevArgs p{};
  p.M = a->M;
  p.N = a->N;
  p.K = a->K;
  p.m_tiles = pl.m_tiles;
  p.n_tiles = pl.n_tiles;
  p.k_blocks = pl.k_blocks;
  p.splits = 1;
  p.kb_per_split = pl.k_blocks;
  p.C = a->C;
  p.ldc = a->ldc;
  p.c_fp32 = a->c_fp32;
  p.bias = a->bias;
  p.aux = static_cast<const __nv_bfloat16*>(a->aux);
  p.ld_aux = a->ld_aux;
  p.epi = a->epi;
  p.alpha = a->alpha == 0.f ? 1.f : a->alpha;
  p.error = a->error;
  p.c2 = static_cast<__nv_bfloat16*>(a->C2);
  p.ldc2 = a->ldc2;
  if (!fill_tp(&p.tp, c)) return static_cast<int>(cudaErrorInvalidValue);
  p.tp.shard = static_cast<const __nv_bfloat16*>(a->A);
  p.tp.ld_shard = a->lda;
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  const bool bmn = a->b_mn != 0;
  if (BN == 256) return TB_TP_DISPATCH(1, 256, bmn);
  if (BN == 128) return TB_TP_DISPATCH(1, 128, bmn);
  return TB_TP_DISPATCH(1, 64, bmn);
}

int tb_tp_gemm_rs(const TbTpComm* c, const TbGemmArgs* a, void* out, long long ldo, const float* bias,
                  const void* residual, long long ld_res, cudaStream_t stream) {
  const int W = c->world, mloc = c->rows_per_rank;
  if (a->M <= 0 || a->N <= 0) return 0;
  if (a->a_mn || a->K <= 0 || a->lda % 8 || a->ldb % 8 || a->N % 8 || ldo % 8 || (residual && ld_res % 8) ||
      mloc % BM || a->M != W * mloc || a->epi != TB_EPI_NONE || a->workspace || a->colsum || a->c_accumulate ||
      c->parity_bytes < 2ll * W * mloc * a->N || (reinterpret_cast<uintptr_t>(a->A) & 15) ||
      (reinterpret_cast<uintptr_t>(a->B) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (reinterpret_cast<uintptr_t>(residual) & 15) || c->rs_target == nullptr)
    return static_cast<int>(cudaErrorInvalidValue);
  const Plan pl = make_plan(a->M, a->N, a->K, a->bn_hint, 1, false, 0);
  const int BN = pl.BN;
  CUtensorMap ta, tbm;
  const bool ok = make_map(&ta, a->A, a->M, a->K, a->lda, BM) &&
                  (a->b_mn ? make_map(&tbm, a->B, a->K, a->N, a->ldb, BK) : make_map(&tbm, a->B, a->N, a->K, a->ldb, BN));
  if (!ok) return static_cast<int>(cudaErrorInvalidValue);
  const CUtensorMap& ta2 = ta;
  const CUtensorMap& ta3 = ta;
  DevArgs p{};
  p.M = a->M;
  p.N = a->N;
  p.K = a->K;
  p.m_tiles = pl.m_tiles;
  p.n_tiles = pl.n_tiles;
  p.k_blocks = pl.k_blocks;
  p.splits = 1;
  p.kb_per_split = pl.k_blocks;
  p.C = nullptr;
  p.ldc = a->N;
  p.c_fp32 = 0;
  p.epi = TB_EPI_NONE;
  p.alpha = a->alpha == 0.f ? 1.f : a->alpha;
  p.error = a->error;
  if (!fill_tp(&p.tp, c)) return static_cast<int>(cudaErrorInvalidValue);
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  const bool bmn = a->b_mn != 0;
  int err;
  if (BN == 256) err = TB_TP_DISPATCH(2, 256, bmn);
  else if (BN == 128) err = TB_TP_DISPATCH(2, 128, bmn);
  else err = TB_TP_DISPATCH(2, 64, bmn);
  if (err) return err;
  TpArgs t = p.tp;
  t.epoch_ctr = c->epoch_ctr;
  const long long nvec = static_cast<long long>(mloc) * a->N / 8;
  long long g = (nvec + 255) / 256;
  if (g > 4ll * num_sms()) g = 4ll * num_sms();
  if (g < 1) g = 1;
  tp_rs_finish_kernel<<<static_cast<unsigned>(g), 256, 0, stream>>>(
      t, a->N, bias, static_cast<const __nv_bfloat16*>(residual), ld_res, static_cast<__nv_bfloat16*>(out), ldo,
      c->rs_target, static_cast<unsigned>(W * grid));
  return static_cast<int>(cudaGetLastError());
}
#undef TB_TP_DISPATCH

// Diagnostics: with a device buffer of at least 148 * 8 uint64, later
// all-gather GEMMs record per-CTA globaltimer stamps (start, push end of warps
// 2 and 3, first remote wait begin / end, main loop end).  nullptr turns it off.
void tb_tp_set_trace(void* p) { g_tp_trace = static_cast<unsigned long long*>(p); }

}  // extern "C"
