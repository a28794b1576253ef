// Small-M ("decode") bf16 GEMM on tcgen05, weight-stationary, with the K
// split over a thread-block cluster and reduced through distributed shared
// memory.
//
//   C[T, N] = epilogue( X[T, K] . W[N, K]^T ),   T tokens (a few to a few hundred)
//
// At decode time T is the number of sequences in the batch and the weight is
// most of the traffic.  The general GEMM (gemm_tcgen05.cu) tiles the output as
// 128 tokens x BN weight rows; with few token tiles each SM streams a long
// K range of both operands, and per-SM load throughput (not DRAM) sets the
// time.  Here the operands swap roles and the work is cut finer:
//   * a CTA owns 256 weight rows (two M = 128 MMAs that share one token tile)
//     and a group of TG <= 128 tokens (the MMAs' N side), so one token tile
//     serves twice the weight rows and the weight crosses from DRAM once;
//   * K is split over a cluster of S CTAs (grid.x = S; grid.y = weight tiles,
//     grid.z = token groups): each CTA accumulates its K range in TMEM, copies
//     its [256 x TG] fp32 partial into its own shared memory token-major, and
//     after a cluster barrier CTA r sums tokens [r TG / S, (r + 1) TG / S) over
//     the S partials with ld.shared::cluster (all S loads in flight) and runs
//     the epilogue.  A second cluster barrier keeps each CTA's shared memory
//     alive until its peers have read it.  No global workspace, no atomics.
//   * epilogues: none, + bias[n], + residual aux[t, n], SwiGLU over
//     interleaved (gate, up) weight rows; bf16 output, 16-byte stores.
// The host picks (TG, S) from a per-SM traffic model under the number of
// clusters that fit on the GPU at once (cudaOccupancyMaxActiveClusters).
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
#include "pdl.cuh"
#include "sm100_primitives.cuh"

namespace {

using namespace tb::sm100;

constexpr int kRows = 256;     // weight rows per CTA (two MMAs of M = 128)
constexpr int kBK = 64;        // K per stage (one 128-byte swizzle row of bf16)
constexpr int kMaxTG = 128;    // tokens per CTA (the MMAs' N)
constexpr int kStages = 4;
constexpr int kThreads = 192;  // warps 0 TMA, 1 MMA + TMEM, 2-5 TMEM readers
constexpr int kMaxSplits = 8;  // portable cluster size
constexpr int kWBytes = kRows * kBK * 2;             // 32 KB
constexpr int kXBytes = kMaxTG * kBK * 2;            // 16 KB
constexpr int kStageBytes = kWBytes + kXBytes;       // 48 KB
constexpr int kBarOffset = kStages * kStageBytes;    // 192 KB; the partial [TG][256] fp32 (<= 128 KB) reuses the ring
constexpr int kSmemBytes = kBarOffset + 256 + 1024;  // + barriers, + slack for 1024-byte alignment
constexpr uint32_t kTmemCols = 256;                  // accumulator a at columns [128 a, 128 a + TG)

struct DecArgs {
  int T, N, K, tg, kb_total;
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
// Every thread of every CTA in the cluster; release / acquire order the
// shared-memory writes before the barrier against the peers' reads after it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The address of the same shared-memory location in cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t out;
  asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(saddr), "r"(rank));
  return out;
}
// Not volatile: the loads sit between the two cluster barriers (whose asm
// carries the memory clobber), and the compiler may issue them back to back.
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

// Sum over the S cluster partials of 8 consecutive fp32 at byte offset `off`:
// every load is issued before the first add.
template <int S>
__device__ __forceinline__ void sum_partials(uint32_t base, uint32_t off, float* acc) {
  float4 x[S], y[S];
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const uint32_t a = map_to_rank(base + off, static_cast<uint32_t>(s));
    x[s] = ld_cluster_f4(a);
    y[s] = ld_cluster_f4(a + 16);
  }
#pragma unroll
  for (int s = 0; s < S; ++s) {
    acc[0] += x[s].x;
    acc[1] += x[s].y;
    acc[2] += x[s].z;
    acc[3] += x[s].w;
    acc[4] += y[s].x;
    acc[5] += y[s].y;
    acc[6] += y[s].z;
    acc[7] += y[s].w;
  }
}

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
  const int tg = p.tg, t0 = static_cast<int>(blockIdx.z) * tg;
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

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------ TMA producer
    const uint32_t bytes = kWBytes + static_cast<uint32_t>(tg) * kBK * 2;
    // The weight is constant: the first ring's weight tiles load before the
    // wait for the preceding kernel (which may still be running under PDL);
    // the token tiles (its output) only after it.
    const int pre = min(kStages, kb1 - kb0);
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], bytes);
      tma_load_2d(smem + i * kStageBytes, &tmW, &full[i], (kb0 + i) * kBK, n0);
    }
    tb::pdl_wait();
    tb::pdl_trigger();
    for (int i = 0; i < pre; ++i) tma_load_2d(smem + i * kStageBytes + kWBytes, &tmX, &full[i], (kb0 + i) * kBK, t0);
    uint32_t issued_mask = (1u << pre) - 1u, last_par = 0;  // per stage: issued at least once / parity of its last issue
    int stage = pre % kStages;
    uint32_t phase = pre == kStages ? 1u : 0u;
    for (int kb = kb0 + pre; kb < kb1; ++kb) {
      if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) break;
      uint8_t* sw = smem + stage * kStageBytes;
      mbar_arrive_expect_tx(&full[stage], bytes);
      tma_load_2d(sw, &tmW, &full[stage], kb * kBK, n0);
      tma_load_2d(sw + kWBytes, &tmX, &full[stage], kb * kBK, t0);
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
        const unsigned long long w0 = global_ns();
        while (!mbar_try_wait(&full[s], last_par >> s & 1u) && global_ns() - w0 < 100000000ull) {
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------ MMA issuer: two M = 128 MMAs per K step share the token tile
    const uint32_t idesc = idesc_bf16(128, tg, 0, 0);
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
        // K-major operands: +32 bytes per K = 16 step inside the swizzle atom;
        // weight rows 128-255 start 128 rows x 128 bytes into the tile
        const uint64_t bd = smem_desc_sw128(sx + kk * 32, 16, 1024);
        const uint32_t acc = (kb > kb0 || kk > 0) ? 1u : 0u;
        mma_f16(tmem_base, smem_desc_sw128(sw + kk * 32, 16, 1024), bd, idesc, acc);
        mma_f16(tmem_base + 128, smem_desc_sw128(sw + 128 * 128 + kk * 32, 16, 1024), bd, idesc, acc);
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
    // ------------------------------------------------ TMEM -> shared memory (token-major partial [tg][256])
    const int q = warp & 3;  // this warp's TMEM lane quarter
    const bool ok = mbar_wait(done, 0, abort_flag);
    tc_fence_after();
    float* part = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int a = 0; a < 2; ++a) {
      const int row = a * 128 + q * 32 + lane;
      for (int c = 0; c < tg; c += 32) {
        float v[32];
        tmem_ld32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(a * 128 + c), v);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c + j < tg) part[(c + j) * kRows + row] = ok ? v[j] : 0.f;
      }
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
  tb::pdl_wait();  // the epilogue reads aux / bias and writes C: after the preceding kernel
  {
    const int r = static_cast<int>(cluster_rank());
    const int valid = min(tg, p.T - t0);  // real tokens of this group
    const int tc = (valid + S - 1) / S;
    const int t_lo = r * tc, t_hi = min(valid, t_lo + tc);
    constexpr int kGroups = kRows / 8;
    const int items = max(0, t_hi - t_lo) * kGroups;
    const uint32_t part_base = smem_u32(smem);
    for (int it = threadIdx.x; it < items; it += kThreads) {
      const int tl = t_lo + it / kGroups, g = it % kGroups;
      const int n = n0 + g * 8;
      const uint32_t off = static_cast<uint32_t>((tl * kRows + g * 8) * 4);
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      switch (S) {
        case 1: sum_partials<1>(part_base, off, acc); break;
        case 2: sum_partials<2>(part_base, off, acc); break;
        case 3: sum_partials<3>(part_base, off, acc); break;
        case 4: sum_partials<4>(part_base, off, acc); break;
        case 5: sum_partials<5>(part_base, off, acc); break;
        case 6: sum_partials<6>(part_base, off, acc); break;
        case 7: sum_partials<7>(part_base, off, acc); break;
        default: sum_partials<8>(part_base, off, acc); break;
      }
      if (n >= p.N) continue;
      const long long t = t0 + tl;
      if (p.epi == TB_EPI_SWIGLU) {
        // weight rows (2j, 2j + 1) are (gate, up) of output column j
        uint2 pk;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
        h[0] = __floats2bfloat162_rn(silu(acc[0]) * acc[1], silu(acc[2]) * acc[3]);
        h[1] = __floats2bfloat162_rn(silu(acc[4]) * acc[5], silu(acc[6]) * acc[7]);
        *reinterpret_cast<uint2*>(p.C + t * p.ldc + n / 2) = pk;
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
        const uint4 a = *reinterpret_cast<const uint4*>(p.aux + t * p.ld_aux + n);
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
      *reinterpret_cast<uint4*>(p.C + t * p.ldc + n) = pk;
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

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Clusters of size s that can be resident at once (one CTA per SM at this
// kernel's shared memory), per device.
int cluster_capacity(int s) {
  static std::mutex mu;
  static int cache[64][kMaxSplits + 1] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 0 || dev >= 64) dev = 0;
  int& c = cache[dev][s];
  if (c == 0) {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
    int n = 0;
    if (tb::ensure_dyn_smem(reinterpret_cast<const void*>(gemm_decode_kernel), kSmemBytes) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(s, 1, 1);
      cfg.blockDim = dim3(kThreads, 1, 1);
      cfg.dynamicSmemBytes = kSmemBytes;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = s;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, reinterpret_cast<const void*>(gemm_decode_kernel), &cfg) != cudaSuccess)
        n = 0;
      cudaGetLastError();
    }
    c = n > 0 ? n : sms / s;
  }
  return c;
}

struct DecPlan {
  int tg, splits;
};

// Per-SM load model: a CTA streams ceil(kb / S) k-blocks of (256 weight rows
// + TG token rows) x 128 bytes, and with S > 1 reads its share of the S fp32
// partials (256 x TG x 4 bytes, mostly remote); clusters beyond what fits at
// once run in further waves.  The cheapest (TG, S) wins.
DecPlan plan(int T, int N, int K, int splits) {
  const int tiles = (N + kRows - 1) / kRows, kb = (K + kBK - 1) / kBK;
  const int t16 = (T + 15) / 16 * 16;
  DecPlan best{t16 < kMaxTG ? t16 : kMaxTG, 1};
  double best_cost = 1e300;
  for (int tg = 16; tg <= kMaxTG; tg *= 2) {
    const int tgc = tg < t16 ? tg : t16;  // never wider than the (padded) token count
    const int groups = (T + tgc - 1) / tgc;
    const int s_lo = splits > 0 ? splits : 1, s_hi = splits > 0 ? splits : (kb < kMaxSplits ? kb : kMaxSplits);
    for (int s = s_lo; s <= s_hi; ++s) {
      const long long clusters = static_cast<long long>(tiles) * groups;
      const long long cap = cluster_capacity(s);
      const long long waves = (clusters + cap - 1) / cap;
      const double per_cta = static_cast<double>((kb + s - 1) / s) * (kWBytes + tgc * kBK * 2) +
                             (s > 1 ? 4.0 * kRows * tgc : 0.0) + 32768.0;  // + fixed setup, in bytes
      const double cost = waves * per_cta;
      if (cost < best_cost * 0.999) {
        best_cost = cost;
        best = DecPlan{tgc, s};
      }
    }
    if (tgc == t16) break;
  }
  return best;
}

}  // namespace

int tb_gemm_decode_splits(int T, int N, int K) { return plan(T, N, K, 0).splits; }

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
  if (a->splits < 0 || a->splits > kMaxSplits || a->splits > kb_total) return static_cast<int>(cudaErrorInvalidValue);
  cudaError_t e = tb::ensure_dyn_smem(reinterpret_cast<const void*>(gemm_decode_kernel), kSmemBytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  const DecPlan pl = plan(a->T, a->N, a->K, a->splits);
  CUtensorMap tw, tx;
  if (!make_map(&tw, a->W, a->N, a->K, a->ldw, kRows) || !make_map(&tx, a->X, a->T, a->K, a->ldx, pl.tg))
    return static_cast<int>(cudaErrorInvalidValue);
  DecArgs p{};
  p.T = a->T;
  p.N = a->N;
  p.K = a->K;
  p.tg = pl.tg;
  p.kb_total = kb_total;
  p.epi = epi;
  p.bias = a->bias;
  p.aux = static_cast<const __nv_bfloat16*>(a->aux);
  p.ld_aux = a->ld_aux;
  p.C = static_cast<__nv_bfloat16*>(a->C);
  p.ldc = a->ldc;
  p.err = a->error;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.splits, (a->N + kRows - 1) / kRows, (a->T + pl.tg - 1) / pl.tg);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = pl.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchAttribute attrs[2] = {attr[0], {}};
  if (tb::pdl_enabled()) {
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
  }
  cfg.attrs = attrs;
  e = cudaLaunchKernelEx(&cfg, gemm_decode_kernel, tw, tx, p);
  return static_cast<int>(e);
}
