// Small-M ("decode") bf16 GEMM on tcgen05, weight-stationary, with the K
// split over a thread-block cluster and reduced through distributed shared
// memory.
//
//   C[T, N] = epilogue( X[T, K] . W[N, K]^T ),   T tokens (any count; 256 per pass)
//
// At decode time T is the number of sequences in the batch (a few hundred)
// and the projection weight is almost all of the traffic.  The general GEMM
// (gemm_tcgen05.cu) tiles the output 128 tokens x BN columns, so every tile
// re-reads its 128 token rows for only BN weight columns, and with few token
// tiles most SMs idle or stream the same rows again.  Here the operands swap
// roles:
//   * the MMA's M side is a 128-row tile of W and its N side is all T tokens
//     of the pass (N = T rounded up to 16, at most 256), so the weight crosses
//     from DRAM exactly once and one MMA covers every token;
//   * K is split over a cluster of S CTAs (grid.x = S; grid.y = weight tiles,
//     one cluster each): each CTA accumulates its K range in TMEM, copies the
//     [128 x T] fp32 partial into its own shared memory token-major, and after
//     a cluster barrier CTA r sums tokens [r T / S, (r + 1) T / S) of all S
//     partials with ld.shared::cluster and runs the epilogue.  A second cluster
//     barrier keeps every CTA's shared memory alive until its peers have read
//     it.  No global workspace, no atomics, one launch.
//   * epilogues: none, + bias[n], + residual aux[t, n], SwiGLU over
//     interleaved (gate, up) weight rows; bf16 output, 16-byte stores.
// Warp roles: warp 0 (one thread) issues TMA tile loads (plain loads into this
// CTA's shared memory) into a 4-stage ring; warp 1 allocates TMEM and one of
// its threads issues the MMAs; warps 2-5 read TMEM.  All six warps join the
// reduction.  Every mbarrier wait is bounded (sm100_primitives.cuh); both
// cluster barriers are reached by every thread on every path, so a CTA that
// gave up still releases its peers.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "device_common.cuh"
#include "kernels.h"
#include "sm100_primitives.cuh"

namespace {

using namespace tb::sm100;

constexpr int kRows = 128;     // weight rows per tile (MMA M)
constexpr int kBK = 64;        // K per stage (one 128-byte swizzle row of bf16)
constexpr int kMaxT = 256;     // tokens per pass (MMA N at most 256)
constexpr int kStages = 4;
constexpr int kThreads = 192;  // warps 0 TMA, 1 MMA + TMEM, 2-5 TMEM readers
constexpr int kMaxSplits = 8;  // portable cluster size
constexpr int kWBytes = kRows * kBK * 2;             // 16 KB
constexpr int kXBytes = kMaxT * kBK * 2;             // 32 KB
constexpr int kStageBytes = kWBytes + kXBytes;       // 48 KB
constexpr int kBarOffset = kStages * kStageBytes;    // 192 KB; the partial [T][128] fp32 (<= 128 KB) reuses the ring
constexpr int kSmemBytes = kBarOffset + 256 + 1024;  // + barriers, + slack for 1024-byte alignment
constexpr uint32_t kTmemCols = 256;

struct DecArgs {
  int T, N, K, t_pad, kb_total;
  int epi;
  const float* bias;
  const __nv_bfloat16* aux;
  long long ld_aux;
  __nv_bfloat16* C;
  long long ldc;
  int* err;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t n;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(n));
  return n;
}
// Every thread of every CTA in the cluster; release / acquire order the
// shared-memory writes before the barrier against the peers' reads after it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The address of the same shared-memory location in cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(saddr), "r"(rank));
  return out;
}
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

__global__ void __launch_bounds__(kThreads, 1)
    gemm_decode_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, DecArgs p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOffset);
  uint64_t* empty = full + kStages;
  uint64_t* done = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = static_cast<int>(gridDim.x), split = static_cast<int>(blockIdx.x);
  const int n0 = static_cast<int>(blockIdx.y) * kRows;
  // balanced K ranges: every split gets at least one k-block (the host keeps S <= kb_total)
  const int kb0 = split * p.kb_total / S, kb1 = (split + 1) * p.kb_total / S;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch(&tmW);
    tma_prefetch(&tmX);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t x_bytes = static_cast<uint32_t>(p.t_pad) * kBK * 2;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------ TMA producer
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued_mask = 0, last_par = 0;  // per stage: issued at least once / parity of its last issue
    for (int kb = kb0; kb < kb1; ++kb) {
      if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) break;
      uint8_t* sw = smem + stage * kStageBytes;
      mbar_arrive_expect_tx(&full[stage], kWBytes + x_bytes);
      tma_load_2d(sw, &tmW, &full[stage], kb * kBK, n0);
      tma_load_2d(sw + kWBytes, &tmX, &full[stage], kb * kBK, 0);
      issued_mask |= 1u << stage;
      last_par = (last_par & ~(1u << stage)) | (phase << stage);
      if (++stage == kStages) {
        stage = 0;
        phase ^= 1;
      }
    }
    if (*abort_flag) {
      // copies still in flight land in this CTA's shared memory: let them finish
      for (int s = 0; s < kStages; ++s) {
        if (!(issued_mask >> s & 1u)) continue;
        const unsigned long long t0 = global_ns();
        while (!mbar_try_wait(&full[s], last_par >> s & 1u) && global_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------ MMA issuer
    const uint32_t idesc = idesc_bf16(kRows, p.t_pad, 0, 0);
    int stage = 0;
    uint32_t phase = 0;
    bool any = false;
    for (int kb = kb0; kb < kb1; ++kb) {
      if (!mbar_wait(&full[stage], phase, abort_flag)) break;
      tc_fence_after();
      const uint32_t sw = smem_u32(smem + stage * kStageBytes);
      const uint32_t sx = sw + kWBytes;
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk) {
        // both operands K-major: +32 bytes per K = 16 step inside the swizzle atom
        mma_f16(tmem_base, smem_desc_sw128(sw + kk * 32, 16, 1024), smem_desc_sw128(sx + kk * 32, 16, 1024), idesc,
                (kb > kb0 || kk > 0) ? 1u : 0u);
      }
      mma_commit(&empty[stage]);
      any = true;
      if (++stage == kStages) {
        stage = 0;
        phase ^= 1;
      }
    }
    // `done` completes once every MMA issued here has finished (at once if none was)
    if (any) mma_commit(done);
    else mbar_arrive(done);
  } else if (warp >= 2) {
    // ------------------------------------------------ TMEM -> shared memory (token-major partial)
    const int q = warp & 3;  // this warp's TMEM lane quarter
    const int row = q * 32 + lane;
    const bool ok = mbar_wait(done, 0, abort_flag);
    tc_fence_after();
    float* part = reinterpret_cast<float*>(smem);
    for (int c = 0; c < p.t_pad; c += 32) {
      float v[32];
      tmem_ld32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(c), v);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c + j < p.T) part[(c + j) * kRows + row] = ok ? v[j] : 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag && p.err) atomicCAS(p.err, 0, 1);

  // ------------------------------------------------ cluster reduction + epilogue
  cluster_sync();
  {
    const uint32_t r = cluster_rank(), ns = cluster_size();
    const int tc = (p.T + static_cast<int>(ns) - 1) / static_cast<int>(ns);
    const int t_lo = static_cast<int>(r) * tc, t_hi = min(p.T, t_lo + tc);
    const int items = max(0, t_hi - t_lo) * (kRows / 8);
    const uint32_t part_base = smem_u32(smem);
    for (int it = threadIdx.x; it < items; it += kThreads) {
      const int t = t_lo + it / (kRows / 8), g = it % (kRows / 8);
      const int n = n0 + g * 8;
      const uint32_t off = static_cast<uint32_t>((t * kRows + g * 8) * 4);
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (uint32_t s = 0; s < ns; ++s) {
        const uint32_t a = map_to_rank(part_base + off, s);
        const float4 x = ld_cluster_f4(a), y = ld_cluster_f4(a + 16);
        acc[0] += x.x;
        acc[1] += x.y;
        acc[2] += x.z;
        acc[3] += x.w;
        acc[4] += y.x;
        acc[5] += y.y;
        acc[6] += y.z;
        acc[7] += y.w;
      }
      if (n >= p.N) continue;
      if (p.epi == TB_EPI_SWIGLU) {
        // weight rows (2j, 2j + 1) are (gate, up) of output column j
        uint2 pk;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
        h[0] = __floats2bfloat162_rn(silu(acc[0]) * acc[1], silu(acc[2]) * acc[3]);
        h[1] = __floats2bfloat162_rn(silu(acc[4]) * acc[5], silu(acc[6]) * acc[7]);
        *reinterpret_cast<uint2*>(p.C + static_cast<long long>(t) * p.ldc + n / 2) = pk;
        continue;
      }
      if (p.epi == TB_EPI_BIAS) {
        const float4 b0 = *reinterpret_cast<const float4*>(p.bias + n);
        const float4 b1 = *reinterpret_cast<const float4*>(p.bias + n + 4);
        acc[0] += b0.x;
        acc[1] += b0.y;
        acc[2] += b0.z;
        acc[3] += b0.w;
        acc[4] += b1.x;
        acc[5] += b1.y;
        acc[6] += b1.z;
        acc[7] += b1.w;
      } else if (p.epi == TB_EPI_RESIDUAL) {
        const uint4 a = *reinterpret_cast<const uint4*>(p.aux + static_cast<long long>(t) * p.ld_aux + n);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&a);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h[j]);
          acc[2 * j] += f.x;
          acc[2 * j + 1] += f.y;
        }
      }
      uint4 pk;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
      *reinterpret_cast<uint4*>(p.C + static_cast<long long>(t) * p.ldc + n) = pk;
    }
  }
  // no CTA leaves (and frees its shared memory) while a peer may still read it
  cluster_sync();
}

// ---------------------------------------------------------------- host side
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

// bf16 row-major [rows, cols], leading dimension ld; box {64 cols, box_rows},
// 128-byte swizzle, zero fill out of bounds.
bool make_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long ld, int box_rows) {
  EncodeTiledFn f = encode_fn();
  if (!f) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {kBK, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t es[2] = {1, 1};
  return f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

int tb_gemm_decode_splits(int N, int K) {
  const int tiles = (N + kRows - 1) / kRows, kb = (K + kBK - 1) / kBK;
  int s = sm_count() / (tiles > 0 ? tiles : 1);
  if (s > kMaxSplits) s = kMaxSplits;
  if (s > kb) s = kb;
  return s < 1 ? 1 : s;
}

int tb_gemm_decode(const TbDecodeGemmArgs* a, cudaStream_t stream) {
  if (a == nullptr || a->T < 0 || a->N <= 0 || a->K <= 0) return static_cast<int>(cudaErrorInvalidValue);
  if (a->T == 0) return 0;
  const int epi = a->epi;
  if (epi != TB_EPI_NONE && epi != TB_EPI_BIAS && epi != TB_EPI_RESIDUAL && epi != TB_EPI_SWIGLU)
    return static_cast<int>(cudaErrorInvalidValue);
  // 16-byte rows for TMA; whole 8-column groups; 16-byte output stores (8-byte for SwiGLU's 4 columns)
  const bool sw = epi == TB_EPI_SWIGLU;
  if (a->N % 8 || a->K % 8 || a->ldw % 8 || a->ldx % 8 || a->ldc % (sw ? 4 : 8) || !aligned16(a->W) ||
      !aligned16(a->X) || (reinterpret_cast<uintptr_t>(a->C) & (sw ? 7 : 15)))
    return static_cast<int>(cudaErrorInvalidValue);
  if (epi == TB_EPI_BIAS && (a->bias == nullptr || !aligned16(a->bias))) return static_cast<int>(cudaErrorInvalidValue);
  if (epi == TB_EPI_RESIDUAL && (a->aux == nullptr || a->ld_aux % 8 || !aligned16(a->aux)))
    return static_cast<int>(cudaErrorInvalidValue);
  const int kb_total = (a->K + kBK - 1) / kBK;
  int S = a->splits > 0 ? a->splits : tb_gemm_decode_splits(a->N, a->K);
  if (S > kMaxSplits || S > kb_total) return static_cast<int>(cudaErrorInvalidValue);
  CUtensorMap tw;
  if (!make_map(&tw, a->W, a->N, a->K, a->ldw, kRows)) return static_cast<int>(cudaErrorInvalidValue);
  cudaError_t e = tb::ensure_dyn_smem(reinterpret_cast<const void*>(gemm_decode_kernel), kSmemBytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  const int tiles = (a->N + kRows - 1) / kRows;
  for (int t0 = 0; t0 < a->T; t0 += kMaxT) {
    const int T = a->T - t0 < kMaxT ? a->T - t0 : kMaxT;
    const int t_pad = (T + 15) / 16 * 16;
    CUtensorMap tx;
    const __nv_bfloat16* X = static_cast<const __nv_bfloat16*>(a->X) + static_cast<long long>(t0) * a->ldx;
    if (!make_map(&tx, X, T, a->K, a->ldx, t_pad)) return static_cast<int>(cudaErrorInvalidValue);
    DecArgs p{};
    p.T = T;
    p.N = a->N;
    p.K = a->K;
    p.t_pad = t_pad;
    p.kb_total = kb_total;
    p.epi = epi;
    p.bias = a->bias;
    p.aux = epi == TB_EPI_RESIDUAL ? static_cast<const __nv_bfloat16*>(a->aux) + static_cast<long long>(t0) * a->ld_aux
                                   : nullptr;
    p.ld_aux = a->ld_aux;
    p.C = static_cast<__nv_bfloat16*>(a->C) + static_cast<long long>(t0) * a->ldc;
    p.ldc = a->ldc;
    p.err = a->error;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S, tiles, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, gemm_decode_kernel, tw, tx, p);
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  return 0;
}
