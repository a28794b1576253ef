// Causal GQA attention for training and prefill (head_dim 128, bf16):
// FlashAttention-2-style forward (online softmax, O and log-sum-exp written),
// backward as two passes — dK/dV with the KV tile outer (no atomics: the query
// heads of a group are looped inside the CTA) and dQ with the query tile outer.
//
// Tiles of 64 queries x 64 keys, 4 warps (16 rows each), bf16 mma.sync
// m16n8k16 with fp32 accumulation, ldmatrix from XOR-swizzled shared memory
// (16-byte chunk c of row r lives at chunk c ^ (r & 7): conflict-free
// ldmatrix), cp.async double-buffered K/V streaming.  Attention is ~2% of the
// RLHF step's FLOPs at these sequence lengths (the projections and MLP are on
// the tcgen05 GEMM); this kernel keeps it off the critical path.
//
// q/k/v are addressed inside the fused QKV activation [B*T, ld]: head h of
// token t of sequence b at base + (b*T + t) * ld + h * 128.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "device_common.cuh"
#include "kernels.h"

namespace {

using bf16 = __nv_bfloat16;
constexpr int D = 128, BMQ = 64, BNK = 64, NT = 128;
constexpr int ROWB = D * 2;  // 256 bytes per row

__device__ __forceinline__ uint32_t saddr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// byte offset of (row, 16-byte chunk) inside a swizzled [rows x 128] bf16 tile
__device__ __forceinline__ int swz(int row, int chunk) { return row * ROWB + ((chunk ^ (row & 7)) << 4); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // zero-fill rows past the end
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr(dst)), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// rows [r0, r0+64) x 128 of a strided bf16 matrix -> swizzled smem tile
__device__ __forceinline__ void load_tile(uint8_t* tile, const bf16* base, long long ld, int r0, int rmax) {
  for (int i = threadIdx.x; i < 64 * 16; i += NT) {
    const int r = i >> 4, c = i & 15;
    const bool ok = r0 + r < rmax;
    const bf16* src = base + static_cast<long long>(ok ? r0 + r : 0) * ld + c * 8;
    cp_async16(tile + swz(r, c), src, ok);
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack2(float x, float y) {
  __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&h);
}

// A fragment (16 rows x 16 cols) at (r0, k0) of a swizzled row-major tile
__device__ __forceinline__ void load_a(uint32_t* a, const uint8_t* tile, int r0, int k0, int lane) {
  const int row = r0 + (lane & 7) + 8 * ((lane >> 3) & 1);
  const int chunk = (k0 >> 3) + (lane >> 4);
  ldsm_x4(a, saddr(tile + swz(row, chunk)));
}
// B fragments for two n-tiles (n0.., n0+8..) x k16 at k0, from a tile stored [n][k] (row = n)
__device__ __forceinline__ void load_b_nk(uint32_t* b, const uint8_t* tile, int n0, int k0, int lane) {
  const int row = n0 + (lane & 7) + 8 * (lane >> 4);
  const int chunk = (k0 >> 3) + ((lane >> 3) & 1);
  ldsm_x4(b, saddr(tile + swz(row, chunk)));  // b[0],b[1]: n-tile 0; b[2],b[3]: n-tile 1
}
// B fragments for two n-tiles x k16 at k0 from a tile stored [k][n] (row = k)
__device__ __forceinline__ void load_b_kn(uint32_t* b, const uint8_t* tile, int k0, int n0, int lane) {
  const int row = k0 + (lane & 7) + 8 * ((lane >> 3) & 1);
  const int chunk = (n0 >> 3) + (lane >> 4);
  ldsm_x4_t(b, saddr(tile + swz(row, chunk)));
}
// A fragment (16 rows x 16 cols) at (r0, k0) read transposed from a tile stored [k][r] (row = k)
__device__ __forceinline__ void load_a_t(uint32_t* a, const uint8_t* tile, int r0, int k0, int lane) {
  // matrices: (rows r0..7, k0..7), (r0+8.., k0..7), (r0.., k0+8..), (r0+8.., k0+8..)
  const int mat = lane >> 3;
  const int krow = k0 + (lane & 7) + 8 * (mat >> 1);
  const int chunk = (r0 >> 3) + (mat & 1);
  ldsm_x4_t(a, saddr(tile + swz(krow, chunk)));
}

// ============================================================ forward
__global__ void __launch_bounds__(NT) fa_fwd_kernel(const bf16* __restrict__ qb, const bf16* __restrict__ kb,
                                                    const bf16* __restrict__ vb, long long ld,
                                                    bf16* __restrict__ ob, long long ldo, float* __restrict__ lse,
                                                    int T, int Hq, int Hk, float scale) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* sQ = sm;
  uint8_t* sK = sm + 64 * ROWB;      // 2 stages
  uint8_t* sV = sK + 2 * 64 * ROWB;  // 2 stages
  const int qt = blockIdx.x, bh = blockIdx.y;
  const int b = bh / Hq, h = bh % Hq, hk = h / (Hq / Hk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long seq0 = static_cast<long long>(b) * T;
  const bf16* Q = qb + seq0 * ld + h * D;
  const bf16* K = kb + seq0 * ld + hk * D;
  const bf16* V = vb + seq0 * ld + hk * D;
  const int q0 = qt * BMQ;
  load_tile(sQ, Q, ld, q0, T);
  const int n_kv = min((q0 + BMQ + BNK - 1) / BNK, (T + BNK - 1) / BNK);  // causal: up to the diagonal
  load_tile(sK, K, ld, 0, T);
  load_tile(sV, V, ld, 0, T);
  cp_commit();
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float sl2 = scale * 1.4426950408889634f;  // scores in log2 units
  const int g = lane >> 2, t4 = lane & 3;
  const int row0 = q0 + warp * 16 + g, row1 = row0 + 8;
  uint32_t qa[8][4];
  for (int j = 0; j < n_kv; ++j) {
    if (j + 1 < n_kv) {
      load_tile(sK + ((j + 1) & 1) * 64 * ROWB, K, ld, (j + 1) * BNK, T);
      load_tile(sV + ((j + 1) & 1) * 64 * ROWB, V, ld, (j + 1) * BNK, T);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) load_a(qa[kk], sQ, warp * 16, kk * 16, lane);
    }
    const uint8_t* tk = sK + (j & 1) * 64 * ROWB;
    const uint8_t* tv = sV + (j & 1) * 64 * ROWB;
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        uint32_t bb[4];
        load_b_nk(bb, tk, n * 8, kk * 16, lane);
        mma16816(s[n], qa[kk], bb[0], bb[1]);
        mma16816(s[n + 1], qa[kk], bb[2], bb[3]);
      }
    }
    // scale, causal mask, online softmax (rows row0 and row1 of this thread)
    const int k0 = j * BNK;
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = k0 + n * 8 + 2 * t4 + (e & 1);
        const int row = e < 2 ? row0 : row1;
        float v = s[n][e] * sl2;
        if (col > row || col >= T) v = -INFINITY;
        s[n][e] = v;
      }
      mx0 = fmaxf(mx0, fmaxf(s[n][0], s[n][1]));
      mx1 = fmaxf(mx1, fmaxf(s[n][2], s[n][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float c0 = mx0 == -INFINITY ? 1.f : exp2f(m0 - mx0);
    const float c1 = mx1 == -INFINITY ? 1.f : exp2f(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      s[n][0] = mx0 == -INFINITY ? 0.f : exp2f(s[n][0] - mx0);
      s[n][1] = mx0 == -INFINITY ? 0.f : exp2f(s[n][1] - mx0);
      s[n][2] = mx1 == -INFINITY ? 0.f : exp2f(s[n][2] - mx1);
      s[n][3] = mx1 == -INFINITY ? 0.f : exp2f(s[n][3] - mx1);
      rs0 += s[n][0] + s[n][1];
      rs1 += s[n][2] + s[n][3];
    }
    l0 = l0 * c0 + rs0;
    l1 = l1 * c1 + rs1;
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      o[d][0] *= c0;
      o[d][1] *= c0;
      o[d][2] *= c1;
      o[d][3] *= c1;
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4] = {pack2(s[2 * kk][0], s[2 * kk][1]), pack2(s[2 * kk][2], s[2 * kk][3]),
                        pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]), pack2(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
      for (int d = 0; d < 16; d += 2) {
        uint32_t bb[4];
        load_b_kn(bb, tv, kk * 16, d * 8, lane);
        mma16816(o[d], pa, bb[0], bb[1]);
        mma16816(o[d + 1], pa, bb[2], bb[3]);
      }
    }
    __syncthreads();
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  bf16* O = ob + seq0 * ldo + h * D;
#pragma unroll
  for (int d = 0; d < 16; ++d) {
    const int col = d * 8 + 2 * t4;
    if (row0 < T)
      *reinterpret_cast<uint32_t*>(O + static_cast<long long>(row0) * ldo + col) = pack2(o[d][0] * inv0, o[d][1] * inv0);
    if (row1 < T)
      *reinterpret_cast<uint32_t*>(O + static_cast<long long>(row1) * ldo + col) = pack2(o[d][2] * inv1, o[d][3] * inv1);
  }
  if (lse != nullptr && t4 == 0) {
    // natural-log LSE of the scaled scores
    float* L = lse + (static_cast<long long>(b) * Hq + h) * T;
    if (row0 < T) L[row0] = (m0 + log2f(l0)) * 0.6931471805599453f;
    if (row1 < T) L[row1] = (m1 + log2f(l1)) * 0.6931471805599453f;
  }
}

// ============================================================ backward helpers
// delta[b, h, t] = sum_d dO[t, d] * O[t, d]
__global__ void fa_bwd_delta_kernel(const bf16* __restrict__ o, long long ldo, const bf16* __restrict__ dout,
                                    long long ldd, float* __restrict__ delta, int B, int T, int Hq) {
  const long long row = blockIdx.x * static_cast<long long>(blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= static_cast<long long>(B) * T * Hq) return;
  const int h = static_cast<int>(row % Hq);
  const long long bt = row / Hq;
  const int b = static_cast<int>(bt / T), t = static_cast<int>(bt % T);
  const bf16* op = o + bt * ldo + h * D + lane * 4;
  const bf16* dp = dout + bt * ldd + h * D + lane * 4;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) s += __bfloat162float(op[i]) * __bfloat162float(dp[i]);
#pragma unroll
  for (int k = 16; k > 0; k >>= 1) s += __shfl_xor_sync(0xffffffffu, s, k);
  if (lane == 0) delta[(static_cast<long long>(b) * Hq + h) * T + t] = s;
}

// ============================================================ backward: dK, dV
// CTA = (kv tile of 64 keys, b, kv head); warp w owns keys [16w, 16w+16).
// For every query head of the group and every query tile at/after the
// diagonal:  S^T = K Q^T,  P^T = exp(S^T - lse),  dV += P^T dO,
//            dP^T = V dO^T, dS^T = P^T (dP^T - delta),  dK += dS^T Q.
__global__ void __launch_bounds__(NT) fa_bwd_dkdv_kernel(const bf16* __restrict__ qb, const bf16* __restrict__ kb,
                                                         const bf16* __restrict__ vb, long long ld,
                                                         const bf16* __restrict__ dob, long long lddo,
                                                         const float* __restrict__ lse,
                                                         const float* __restrict__ delta, bf16* __restrict__ dkb,
                                                         bf16* __restrict__ dvb, long long lddkv, int T, int Hq,
                                                         int Hk, float scale) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* sK = sm;
  uint8_t* sV = sm + 64 * ROWB;
  uint8_t* sQ = sV + 64 * ROWB;   // 2 stages
  uint8_t* sdO = sQ + 2 * 64 * ROWB;  // 2 stages
  __shared__ float sL[2][64], sD[2][64];
  const int kt = blockIdx.x, bh = blockIdx.y;
  const int b = bh / Hk, hk = bh % Hk, G = Hq / Hk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const long long seq0 = static_cast<long long>(b) * T;
  const int k0 = kt * BNK;
  load_tile(sK, kb + seq0 * ld + hk * D, ld, k0, T);
  load_tile(sV, vb + seq0 * ld + hk * D, ld, k0, T);
  cp_commit();
  float dk[16][4], dv[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
  const int first_qt = k0 / BMQ, n_qt = (T + BMQ - 1) / BMQ;
  const int n_iter = G * (n_qt - first_qt);
  const float sl2 = scale * 1.4426950408889634f;
  auto issue = [&](int it, int stage) {
    const int hq = hk * G + it / (n_qt - first_qt);
    const int qt = first_qt + it % (n_qt - first_qt);
    load_tile(sQ + stage * 64 * ROWB, qb + seq0 * ld + hq * D, ld, qt * BMQ, T);
    load_tile(sdO + stage * 64 * ROWB, dob + seq0 * lddo + hq * D, lddo, qt * BMQ, T);
    for (int i = threadIdx.x; i < 64; i += NT) {
      const int tq = qt * BMQ + i;
      const long long idx = (static_cast<long long>(b) * Hq + hq) * T + tq;
      sL[stage][i] = tq < T ? lse[idx] * 1.4426950408889634f : 0.f;
      sD[stage][i] = tq < T ? delta[idx] : 0.f;
    }
  };
  if (n_iter > 0) issue(0, 0);
  cp_commit();
  for (int it = 0; it < n_iter; ++it) {
    const int stage = it & 1;
    if (it + 1 < n_iter) {
      __syncthreads();  // previous users of stage^1 are done
      issue(it + 1, stage ^ 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const int qt = first_qt + it % (n_qt - first_qt);
    const int q0 = qt * BMQ;
    const uint8_t* tq = sQ + stage * 64 * ROWB;
    const uint8_t* tdo = sdO + stage * 64 * ROWB;
    // S^T [16 keys x 64 queries] and dP^T
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
      st[n][0] = st[n][1] = st[n][2] = st[n][3] = dpt[n][0] = dpt[n][1] = dpt[n][2] = dpt[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t ka[4], va[4];
      load_a(ka, sK, warp * 16, kk * 16, lane);
      load_a(va, sV, warp * 16, kk * 16, lane);
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        uint32_t bq[4], bo[4];
        load_b_nk(bq, tq, n * 8, kk * 16, lane);
        load_b_nk(bo, tdo, n * 8, kk * 16, lane);
        mma16816(st[n], ka, bq[0], bq[1]);
        mma16816(st[n + 1], ka, bq[2], bq[3]);
        mma16816(dpt[n], va, bo[0], bo[1]);
        mma16816(dpt[n + 1], va, bo[2], bo[3]);
      }
    }
    const int key0 = k0 + warp * 16 + g, key1 = key0 + 8;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ql = n * 8 + 2 * t4 + (e & 1);
        const int key = e < 2 ? key0 : key1;
        const bool ok = (q0 + ql) >= key && (q0 + ql) < T && key < T;
        const float p = ok ? exp2f(st[n][e] * sl2 - sL[stage][ql]) : 0.f;
        st[n][e] = p;                                  // P^T
        dpt[n][e] = p * (dpt[n][e] - sD[stage][ql]);  // dS^T (unscaled)
      }
    }
    // dV += P^T dO ; dK += dS^T Q   (k = queries)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4] = {pack2(st[2 * kk][0], st[2 * kk][1]), pack2(st[2 * kk][2], st[2 * kk][3]),
                        pack2(st[2 * kk + 1][0], st[2 * kk + 1][1]), pack2(st[2 * kk + 1][2], st[2 * kk + 1][3])};
      uint32_t da[4] = {pack2(dpt[2 * kk][0], dpt[2 * kk][1]), pack2(dpt[2 * kk][2], dpt[2 * kk][3]),
                        pack2(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]), pack2(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3])};
#pragma unroll
      for (int d = 0; d < 16; d += 2) {
        uint32_t bo[4], bq[4];
        load_b_kn(bo, tdo, kk * 16, d * 8, lane);
        load_b_kn(bq, tq, kk * 16, d * 8, lane);
        mma16816(dv[d], pa, bo[0], bo[1]);
        mma16816(dv[d + 1], pa, bo[2], bo[3]);
        mma16816(dk[d], da, bq[0], bq[1]);
        mma16816(dk[d + 1], da, bq[2], bq[3]);
      }
    }
  }
  const int key0 = k0 + warp * 16 + g, key1 = key0 + 8;
  bf16* dK = dkb + seq0 * lddkv + hk * D;
  bf16* dV = dvb + seq0 * lddkv + hk * D;
#pragma unroll
  for (int d = 0; d < 16; ++d) {
    const int col = d * 8 + 2 * t4;
    if (key0 < T) {
      *reinterpret_cast<uint32_t*>(dK + static_cast<long long>(key0) * lddkv + col) = pack2(dk[d][0] * scale, dk[d][1] * scale);
      *reinterpret_cast<uint32_t*>(dV + static_cast<long long>(key0) * lddkv + col) = pack2(dv[d][0], dv[d][1]);
    }
    if (key1 < T) {
      *reinterpret_cast<uint32_t*>(dK + static_cast<long long>(key1) * lddkv + col) = pack2(dk[d][2] * scale, dk[d][3] * scale);
      *reinterpret_cast<uint32_t*>(dV + static_cast<long long>(key1) * lddkv + col) = pack2(dv[d][2], dv[d][3]);
    }
  }
}

// ============================================================ backward: dQ
// CTA = (query tile, b, q head); warp w owns query rows [16w, 16w+16).
//   S = Q K^T, P = exp(S - lse), dP = dO V^T, dS = P (dP - delta), dQ += dS K
__global__ void __launch_bounds__(NT) fa_bwd_dq_kernel(const bf16* __restrict__ qb, const bf16* __restrict__ kb,
                                                       const bf16* __restrict__ vb, long long ld,
                                                       const bf16* __restrict__ dob, long long lddo,
                                                       const float* __restrict__ lse, const float* __restrict__ delta,
                                                       bf16* __restrict__ dqb, long long lddq, int T, int Hq, int Hk,
                                                       float scale) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* sQ = sm;
  uint8_t* sdO = sm + 64 * ROWB;
  uint8_t* sK = sdO + 64 * ROWB;   // 2 stages
  uint8_t* sV = sK + 2 * 64 * ROWB;  // 2 stages
  const int qt = blockIdx.x, bh = blockIdx.y;
  const int b = bh / Hq, h = bh % Hq, hk = h / (Hq / Hk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
  const long long seq0 = static_cast<long long>(b) * T;
  const int q0 = qt * BMQ;
  const bf16* K = kb + seq0 * ld + hk * D;
  const bf16* V = vb + seq0 * ld + hk * D;
  load_tile(sQ, qb + seq0 * ld + h * D, ld, q0, T);
  load_tile(sdO, dob + seq0 * lddo + h * D, lddo, q0, T);
  load_tile(sK, K, ld, 0, T);
  load_tile(sV, V, ld, 0, T);
  cp_commit();
  const int row0 = q0 + warp * 16 + g, row1 = row0 + 8;
  const long long lrow = (static_cast<long long>(b) * Hq + h) * T;
  const float L0 = row0 < T ? lse[lrow + row0] * 1.4426950408889634f : 0.f;
  const float L1 = row1 < T ? lse[lrow + row1] * 1.4426950408889634f : 0.f;
  const float D0 = row0 < T ? delta[lrow + row0] : 0.f, D1 = row1 < T ? delta[lrow + row1] : 0.f;
  const float sl2 = scale * 1.4426950408889634f;
  float dq[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
  const int n_kv = min((q0 + BMQ + BNK - 1) / BNK, (T + BNK - 1) / BNK);
  for (int j = 0; j < n_kv; ++j) {
    if (j + 1 < n_kv) {
      load_tile(sK + ((j + 1) & 1) * 64 * ROWB, K, ld, (j + 1) * BNK, T);
      load_tile(sV + ((j + 1) & 1) * 64 * ROWB, V, ld, (j + 1) * BNK, T);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const uint8_t* tk = sK + (j & 1) * 64 * ROWB;
    const uint8_t* tv = sV + (j & 1) * 64 * ROWB;
    float s[8][4], dp[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = dp[n][0] = dp[n][1] = dp[n][2] = dp[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t qa[4], oa[4];
      load_a(qa, sQ, warp * 16, kk * 16, lane);
      load_a(oa, sdO, warp * 16, kk * 16, lane);
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        uint32_t bk[4], bv[4];
        load_b_nk(bk, tk, n * 8, kk * 16, lane);
        load_b_nk(bv, tv, n * 8, kk * 16, lane);
        mma16816(s[n], qa, bk[0], bk[1]);
        mma16816(s[n + 1], qa, bk[2], bk[3]);
        mma16816(dp[n], oa, bv[0], bv[1]);
        mma16816(dp[n + 1], oa, bv[2], bv[3]);
      }
    }
    const int kb0 = j * BNK;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = kb0 + n * 8 + 2 * t4 + (e & 1);
        const int row = e < 2 ? row0 : row1;
        const bool ok = col <= row && col < T && row < T;
        const float p = ok ? exp2f(s[n][e] * sl2 - (e < 2 ? L0 : L1)) : 0.f;
        s[n][e] = p * (dp[n][e] - (e < 2 ? D0 : D1));  // dS
      }
    }
    // dQ += dS K   (k = keys; K tile stored [key][d] -> row-major B)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t da[4] = {pack2(s[2 * kk][0], s[2 * kk][1]), pack2(s[2 * kk][2], s[2 * kk][3]),
                        pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]), pack2(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
      for (int d = 0; d < 16; d += 2) {
        uint32_t bb[4];
        load_b_kn(bb, tk, kk * 16, d * 8, lane);
        mma16816(dq[d], da, bb[0], bb[1]);
        mma16816(dq[d + 1], da, bb[2], bb[3]);
      }
    }
    __syncthreads();
  }
  bf16* dQ = dqb + seq0 * lddq + h * D;
#pragma unroll
  for (int d = 0; d < 16; ++d) {
    const int col = d * 8 + 2 * t4;
    if (row0 < T)
      *reinterpret_cast<uint32_t*>(dQ + static_cast<long long>(row0) * lddq + col) = pack2(dq[d][0] * scale, dq[d][1] * scale);
    if (row1 < T)
      *reinterpret_cast<uint32_t*>(dQ + static_cast<long long>(row1) * lddq + col) = pack2(dq[d][2] * scale, dq[d][3] * scale);
  }
}

}  // namespace

extern "C" {

int tb_flash_attn_fwd(const void* q, const void* k, const void* v, long long ld, void* o, long long ldo, float* lse,
                      int B, int T, int Hq, int Hk, float scale, cudaStream_t s) {
  if (B <= 0 || T <= 0) return 0;
  if (Hq % Hk || (ld % 8) || (ldo % 8)) return static_cast<int>(cudaErrorInvalidValue);
  const int smem = 5 * 64 * ROWB;
  tb::ensure_dyn_smem(reinterpret_cast<const void*>(fa_fwd_kernel), smem);
  dim3 grid((T + BMQ - 1) / BMQ, B * Hq);
  fa_fwd_kernel<<<grid, NT, smem, s>>>(static_cast<const bf16*>(q), static_cast<const bf16*>(k),
                                       static_cast<const bf16*>(v), ld, static_cast<bf16*>(o), ldo, lse, T, Hq, Hk,
                                       scale);
  return static_cast<int>(cudaGetLastError());
}

int tb_flash_attn_delta(const void* o, long long ldo, const void* dout, long long lddo, float* delta, int B, int T,
                        int Hq, cudaStream_t s) {
  if (B <= 0 || T <= 0) return 0;
  const long long rows = static_cast<long long>(B) * T * Hq;
  fa_bwd_delta_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, s>>>(
      static_cast<const bf16*>(o), ldo, static_cast<const bf16*>(dout), lddo, delta, B, T, Hq);
  return static_cast<int>(cudaGetLastError());
}

int tb_flash_attn_bwd(const void* q, const void* k, const void* v, long long ld, const void* o, long long ldo,
                      const void* dout, long long lddo, const float* lse, float* delta, void* dq, void* dk, void* dv,
                      long long lddqkv, int B, int T, int Hq, int Hk, float scale, cudaStream_t s) {
  if (B <= 0 || T <= 0) return 0;
  if (Hq % Hk || (ld % 8) || (lddqkv % 8) || (lddo % 8)) return static_cast<int>(cudaErrorInvalidValue);
  const long long rows = static_cast<long long>(B) * T * Hq;
  fa_bwd_delta_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, s>>>(
      static_cast<const bf16*>(o), ldo, static_cast<const bf16*>(dout), lddo, delta, B, T, Hq);
  const int smem = 6 * 64 * ROWB;
  tb::ensure_dyn_smem(reinterpret_cast<const void*>(fa_bwd_dkdv_kernel), smem);
  tb::ensure_dyn_smem(reinterpret_cast<const void*>(fa_bwd_dq_kernel), smem);
  dim3 g1((T + BNK - 1) / BNK, B * Hk);
  fa_bwd_dkdv_kernel<<<g1, NT, smem, s>>>(static_cast<const bf16*>(q), static_cast<const bf16*>(k),
                                          static_cast<const bf16*>(v), ld, static_cast<const bf16*>(dout), lddo, lse,
                                          delta, static_cast<bf16*>(dk), static_cast<bf16*>(dv), lddqkv, T, Hq, Hk,
                                          scale);
  dim3 g2((T + BMQ - 1) / BMQ, B * Hq);
  fa_bwd_dq_kernel<<<g2, NT, smem, s>>>(static_cast<const bf16*>(q), static_cast<const bf16*>(k),
                                        static_cast<const bf16*>(v), ld, static_cast<const bf16*>(dout), lddo, lse,
                                        delta, static_cast<bf16*>(dq), lddqkv, T, Hq, Hk, scale);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
