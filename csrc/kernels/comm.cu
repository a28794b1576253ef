// Collective kernels over NVLink peer memory (one process per GPU; every rank
// maps every peer's buffers through CUDA IPC, so a kernel addresses remote HBM
// with ordinary loads and stores).
//
//   tb_peer_allreduce       sum (or mean) of a buffer across ranks: rank r
//                           reduces slice r by reading it from every peer and
//                           writes the result into every peer's output.
//   tb_peer_scatter_copy    all-gather with a layout change: every rank writes
//                           row segments of its buffers into every rank's
//                           payload (the trainer -> rollout weight sync of a
//                           tensor-parallel trainer into full-model copies).
//   tb_peer_allreduce_adam  the data-parallel optimizer step in one kernel:
//                           reduce-scatter of the fp32 gradient (peer loads),
//                           Adam on the owned shard (ZeRO-1: the Adam moments
//                           are shard-sized arrays that exist only on the
//                           shard's owner), all-gather of
//                           the updated fp32 weights and their bf16 copy
//                           (peer stores).
//
// Synchronization: each rank owns a flag array in its peer buffer; a release
// store of the call's epoch into every peer's slot says "my inputs are ready",
// and an acquire spin (bounded) on all slots gates the reads.  The last block
// to finish (a local atomic counter) publishes the second flag ("my outputs
// are written into you") and waits for everyone else's before the kernel ends,
// so the next kernel on the stream sees complete weights.  Every wait gives up
// after a time budget and sets the error word instead of hanging; the host
// checks it.  The epoch lives in device memory so the kernel can be replayed
// from a CUDA graph.  No TMA or multicast is involved: peer traffic is plain
// 16-byte vector loads and stores.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstddef>

#include "device_common.cuh"
#include "kernels.h"

namespace {

constexpr int kBlock = 512;
constexpr unsigned long long kBudgetNs = 4000000000ull;  // 4 s

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Warp 0 (converged, all 32 lanes) stores `epoch` into every rank's flag at
// byte offset `off` of its header: lane p stores rank p's flag after its own
// system-scope fence (fence + relaxed store = a release).  One NVLink round
// trip for all ranks, where a release store per rank from one thread waits
// for each previous one to be performed.  The caller's __syncthreads orders
// the block's writes before the fences.
__device__ __forceinline__ void publish_all(const TbPeerTable& t, size_t off, unsigned epoch) {
  const int lane = threadIdx.x & 31;
  if (lane < t.world) {
    __threadfence_system();
    st_relaxed(reinterpret_cast<unsigned*>(static_cast<char*>(t.hdr[lane]) + off), epoch);
  }
  __syncwarp();
}

// Waits until flags[0..W) (local memory, written by peers) all reach `epoch`.
__device__ bool wait_all(const unsigned* flags, int W, unsigned epoch, int* err, int site,
                         unsigned long long budget_ns = kBudgetNs) {
  const unsigned long long t0 = now_ns();
  for (int p = 0; p < W; ++p) {
    while (ld_acquire(flags + p) < epoch) {
      if (*reinterpret_cast<volatile int*>(err) != 0) return false;
      if (now_ns() - t0 > budget_ns) {
        atomicCAS(err, 0, site);
        return false;
      }
      __nanosleep(100);
    }
  }
  return true;
}

// Blocks of the replicated-Adam step (one slice of the vector each; every
// rank runs the same grid, so block b of every rank owns the same slice).
constexpr int kRepBlocks = 148;

struct Hdr {
  unsigned flags_in[TB_MAX_PEERS];   // "peer p's inputs are ready" (epoch)
  unsigned flags_out[TB_MAX_PEERS];  // "peer p finished writing its outputs into me" (epoch)
  // replicated-Adam step, per block slice b (its own epoch sequence):
  unsigned rep_ready[kRepBlocks][TB_MAX_PEERS];  // "peer p's send slice b is ready"
  unsigned rep_read[kRepBlocks][TB_MAX_PEERS];   // "peer p has finished reading my send slice b"
};

// Slice [lo, hi) of n elements owned by `rank`, rounded to multiples of 4
// (the host computes the same split in tb_peer_owned_slice).
__host__ __device__ __forceinline__ void owned_slice(long long n, int rank, int W, long long& lo, long long& hi) {
  const long long n4 = (n + 3) / 4;
  const long long per = (n4 + W - 1) / W;
  const long long a = per * rank, b = per * (rank + 1);
  lo = (a < n4 ? a : n4) * 4;
  const long long h4 = (b < n4 ? b : n4) * 4;
  hi = h4 < n ? h4 : n;
}

__device__ void publish_and_finish(const TbPeerTable& t, unsigned epoch, unsigned* done_ctr, int* err) {
  // every block: make this block's peer stores visible, then count in
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    s_last = atomicAdd(done_ctr, 1u) == gridDim.x - 1 ? 1 : 0;  // the last block of this rank
  }
  __syncthreads();
  if (s_last && threadIdx.x < 32) {
    if (threadIdx.x == 0) *done_ctr = 0;
    publish_all(t, offsetof(Hdr, flags_out) + t.rank * sizeof(unsigned), epoch);
    if (threadIdx.x == 0) {
      wait_all(reinterpret_cast<Hdr*>(t.hdr[t.rank])->flags_out, t.world, epoch, err, 2);
      *t.epoch_ctr = epoch;  // next call uses epoch + 1
    }
  }
}

__device__ unsigned begin_call(const TbPeerTable& t, int* err, bool* ok) {
  const unsigned epoch = *t.epoch_ctr + 1;
  __shared__ int s_ok;
  if (threadIdx.x < 32) {
    // every block publishes "this rank's inputs are ready" (the same epoch,
    // idempotent), so no block waits on another block of its own grid being
    // scheduled: the only waits are on other ranks
    publish_all(t, offsetof(Hdr, flags_in) + t.rank * sizeof(unsigned), epoch);
    if (threadIdx.x == 0)
      s_ok = wait_all(reinterpret_cast<Hdr*>(t.hdr[t.rank])->flags_in, t.world, epoch, err, 1) ? 1 : 0;
  }
  __syncthreads();
  *ok = s_ok != 0;
  return epoch;
}

// Sum over the ranks of the float4 at element i of every rank's fp32 buffer
// at byte offset `off`.  All W peer loads are issued before the first add, so a
// call pays one NVLink round trip instead of W; the adds run in rank order, as
// a sequential loop would.
__device__ __forceinline__ float4 sum_peers4(const TbPeerTable& t, long long off, long long i) {
  float4 x[TB_MAX_PEERS];
#pragma unroll
  for (int p = 0; p < TB_MAX_PEERS; ++p)
    if (p < t.world)
      x[p] = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(static_cast<const char*>(t.base[p]) + off) + i);
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int p = 0; p < TB_MAX_PEERS; ++p) {
    if (p < t.world) {
      s.x += x[p].x;
      s.y += x[p].y;
      s.z += x[p].z;
      s.w += x[p].w;
    }
  }
  return s;
}

__global__ void __launch_bounds__(kBlock) allreduce_kernel(TbPeerTable t, long long in_off, long long out_off,
                                                           long long n, float scale, unsigned* done_ctr, int* err) {
  bool ok;
  const unsigned epoch = begin_call(t, err, &ok);
  if (ok) {
    long long lo, hi;
    owned_slice(n, t.rank, t.world, lo, hi);
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x * 4;
    for (long long i = lo + (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < hi; i += stride) {
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
      const bool full = i + 4 <= hi;
      if (full) {
        s = sum_peers4(t, in_off, i);
      } else {
        for (int p = 0; p < t.world; ++p) {
          const float* src = reinterpret_cast<const float*>(static_cast<const char*>(t.base[p]) + in_off) + i;
          s.x += src[0];
          if (i + 1 < hi) s.y += src[1];
          if (i + 2 < hi) s.z += src[2];
        }
      }
      s.x *= scale;
      s.y *= scale;
      s.z *= scale;
      s.w *= scale;
      for (int p = 0; p < t.world; ++p) {
        float* dst = reinterpret_cast<float*>(static_cast<char*>(t.base[p]) + out_off) + i;
        if (full) {
          *reinterpret_cast<float4*>(dst) = s;
        } else {
          dst[0] = s.x;
          if (i + 1 < hi) dst[1] = s.y;
          if (i + 2 < hi) dst[2] = s.z;
        }
      }
    }
  }
  publish_and_finish(t, epoch, done_ctr, err);
}

__device__ __forceinline__ float adam1(float& p, float g, float& m, float& v, const TbAdamParams& h, float bc1,
                                       float bc2) {
  m = h.beta1 * m + (1.f - h.beta1) * g;
  v = h.beta2 * v + (1.f - h.beta2) * g * g;
  p -= h.lr * ((m / bc1) / (sqrtf(v / bc2) + h.eps) + h.weight_decay * p);
  return p;
}

__global__ void __launch_bounds__(kBlock) allreduce_adam_kernel(TbPeerTable t, long long grad_off,
                                                                long long param_off, long long shadow_off,
                                                                long long n, float* m, float* v, TbAdamParams hp,
                                                                const long long* step_ptr, unsigned* done_ctr,
                                                                int* err) {
  bool ok;
  const unsigned epoch = begin_call(t, err, &ok);
  if (ok) {
    const long long step = (step_ptr ? *step_ptr : hp.step) + 1;
    const float bc1 = 1.f - powf(hp.beta1, static_cast<float>(step));
    const float bc2 = 1.f - powf(hp.beta2, static_cast<float>(step));
    long long lo, hi;
    owned_slice(n, t.rank, t.world, lo, hi);
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x * 4;
    const float gs = hp.grad_scale;
    for (long long i = lo + (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < hi; i += stride) {
      const int cnt = static_cast<int>(min(4LL, hi - i));
      float g[4] = {0.f, 0.f, 0.f, 0.f};
      if (cnt == 4) {
        const float4 x = sum_peers4(t, grad_off, i);
        g[0] = x.x;
        g[1] = x.y;
        g[2] = x.z;
        g[3] = x.w;
      } else {
        for (int p = 0; p < t.world; ++p) {
          const float* src = reinterpret_cast<const float*>(static_cast<const char*>(t.base[p]) + grad_off) + i;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (j < cnt) g[j] += src[j];
        }
      }
      // owner's fp32 master weights (local) -> Adam -> broadcast
      float* pl = reinterpret_cast<float*>(static_cast<char*>(t.base[t.rank]) + param_off) + i;
      float pv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (j < cnt) {
          pv[j] = pl[j];
          float mm = m[i - lo + j], vv = v[i - lo + j];  // moments: this rank's shard only
          adam1(pv[j], g[j] * gs, mm, vv, hp, bc1, bc2);
          m[i - lo + j] = mm;
          v[i - lo + j] = vv;
        }
      }
      __nv_bfloat162 b01 = __floats2bfloat162_rn(pv[0], pv[1]), b23 = __floats2bfloat162_rn(pv[2], pv[3]);
      for (int p = 0; p < t.world; ++p) {
        float* dp = reinterpret_cast<float*>(static_cast<char*>(t.base[p]) + param_off) + i;
        __nv_bfloat16* ds = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(t.base[p]) + shadow_off) + i;
        if (cnt == 4) {
          *reinterpret_cast<float4*>(dp) = make_float4(pv[0], pv[1], pv[2], pv[3]);
          reinterpret_cast<__nv_bfloat162*>(ds)[0] = b01;
          reinterpret_cast<__nv_bfloat162*>(ds)[1] = b23;
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (j < cnt) {
              dp[j] = pv[j];
              ds[j] = __float2bfloat16_rn(pv[j]);
            }
          }
        }
      }
    }
  }
  publish_and_finish(t, epoch, done_ctr, err);
}

// Data-parallel optimizer step with one handshake, for small vectors (the
// PPO minibatch step, ~0.6 MB, is latency-bound).  Every rank pulls every
// peer's whole gradient and runs Adam on the whole vector itself (full-size
// moments on every rank; the sum runs in rank order on every rank, so the
// ranks' weights stay bit-identical), so no updated weights cross NVLink and
// nothing waits for the peers at the end of the call.  Block b of every rank
// owns slice b:
//   1. wait until every peer has finished reading my send slice b of the
//      previous call (set long ago in practice: a local flag read);
//   2. copy my gradient slice into my send buffer (a snapshot, so the next
//      backward may overwrite the gradient while peers still read);
//   3. publish "slice b ready" into every peer, wait for every peer's;
//   4. sum the slice over the peers' send buffers, Adam, write the local fp32
//      weights and bf16 copy;
//   5. tell every peer "I have read your slice b".
// The epoch advances once per call (the last block to finish, locally).
__global__ void __launch_bounds__(kBlock) allreduce_adam_rep_kernel(TbPeerTable t, long long grad_off,
                                                                    long long send_off, long long param_off,
                                                                    long long shadow_off, long long n, float* m,
                                                                    float* v, TbAdamParams hp,
                                                                    const long long* step_ptr, unsigned* rep_epoch,
                                                                    unsigned* done_ctr, int* err) {
  const unsigned epoch = *rep_epoch + 1;
  const int b = blockIdx.x;
  Hdr* mine = reinterpret_cast<Hdr*>(t.hdr[t.rank]);
  const long long n4 = (n + 3) / 4, per = (n4 + gridDim.x - 1) / gridDim.x;
  const long long lo = min(n, b * per * 4), hi = min(n, (b + 1) * per * 4);
  const float* grad = reinterpret_cast<const float*>(static_cast<const char*>(t.base[t.rank]) + grad_off);
  float* send = reinterpret_cast<float*>(static_cast<char*>(t.base[t.rank]) + send_off);
  float* param = reinterpret_cast<float*>(static_cast<char*>(t.base[t.rank]) + param_off);
  __nv_bfloat16* shadow = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(t.base[t.rank]) + shadow_off);
  __shared__ int s_ok;
  // 1. my previous send slice has been read by everyone
  if (threadIdx.x == 0) s_ok = wait_all(mine->rep_read[b], t.world, epoch - 1, err, 21) ? 1 : 0;
  __syncthreads();
  bool ok = s_ok != 0;
  // 2. snapshot of my gradient slice
  if (ok) {
    for (long long i = lo + threadIdx.x * 4; i < hi; i += blockDim.x * 4) {
      if (i + 4 <= hi) {
        *reinterpret_cast<float4*>(send + i) = *reinterpret_cast<const float4*>(grad + i);
      } else {
        for (long long j = i; j < hi; ++j) send[j] = grad[j];
      }
    }
  }
  // 3. publish it; wait for everyone's
  __syncthreads();
  if (ok && threadIdx.x < 32) {
    publish_all(t, offsetof(Hdr, rep_ready) + (static_cast<size_t>(b) * TB_MAX_PEERS + t.rank) * sizeof(unsigned),
                epoch);
    if (threadIdx.x == 0) s_ok = wait_all(mine->rep_ready[b], t.world, epoch, err, 22) ? 1 : 0;
  }
  __syncthreads();
  ok = ok && s_ok != 0;
  // 4. reduce in rank order + Adam on the whole slice, local writes only
  if (ok) {
    const long long step = (step_ptr ? *step_ptr : hp.step) + 1;
    const float bc1 = 1.f - powf(hp.beta1, static_cast<float>(step));
    const float bc2 = 1.f - powf(hp.beta2, static_cast<float>(step));
    const float gs = hp.grad_scale;
    for (long long i = lo + threadIdx.x * 4; i < hi; i += blockDim.x * 4) {
      const int cnt = static_cast<int>(min(4LL, hi - i));
      float g[4] = {0.f, 0.f, 0.f, 0.f};
      if (cnt == 4) {
        const float4 x = sum_peers4(t, send_off, i);
        g[0] = x.x;
        g[1] = x.y;
        g[2] = x.z;
        g[3] = x.w;
      } else {
        for (int p = 0; p < t.world; ++p) {
          const float* src = reinterpret_cast<const float*>(static_cast<const char*>(t.base[p]) + send_off) + i;
          for (int j = 0; j < cnt; ++j) g[j] += src[j];
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (j < cnt) {
          float pv = param[i + j], mm = m[i + j], vv = v[i + j];
          adam1(pv, g[j] * gs, mm, vv, hp, bc1, bc2);
          param[i + j] = pv;
          m[i + j] = mm;
          v[i + j] = vv;
          shadow[i + j] = __float2bfloat16_rn(pv);
        }
      }
    }
  }
  // 5. done reading every peer's slice b
  __syncthreads();
  if (ok && threadIdx.x < 32)
    publish_all(t, offsetof(Hdr, rep_read) + (static_cast<size_t>(b) * TB_MAX_PEERS + t.rank) * sizeof(unsigned),
                epoch);
  if (threadIdx.x == 0) {
    // the last block of this rank advances the epoch (a local counter)
    __threadfence();
    if (atomicAdd(done_ctr, 1u) == gridDim.x - 1) {
      *done_ctr = 0;
      *rep_epoch = epoch;
    }
  }
}

// Scatter all-gather with a layout change (the trainer -> rollout weight sync
// of a tensor-parallel trainer with a full-model rollout copy on every rank).
// Segment k copies `rows` rows of `row_bytes` from this rank's source buffer
// (src[sel] + src_off, row stride src_ld) into the payload of every rank
// (peers != 0) or of this rank only (peers == 0, e.g. replicated tensors that
// every rank holds already), at dst_off with row stride dst_ld.  Work is
// flattened over the 16-byte vectors of all segments (vec_begin: exclusive
// prefix over the segments); a thread finds its segment by binary search and
// issues one local load and one store per destination rank, 4 vectors in
// flight.  The begin/finish handshakes are those of the other collectives
// here: no rank writes into a peer's copy before that peer has entered the
// call (its previous readers of the copy are done, by stream order), and no
// rank leaves before every peer's writes into its copy are complete.
__global__ void __launch_bounds__(kBlock) scatter_copy_kernel(TbPeerTable t, const char* __restrict__ src0,
                                                              const char* __restrict__ src1,
                                                              const TbCopySeg* __restrict__ segs, int nseg,
                                                              long long total_vecs, long long dst_base,
                                                              unsigned* done_ctr, int* err) {
  bool ok;
  const unsigned epoch = begin_call(t, err, &ok);
  if (ok) {
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    constexpr int kU = 4;
    for (long long v0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; v0 < total_vecs;
         v0 += stride * kU) {
      uint4 val[kU];
      long long dst[kU];
      int all[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const long long v = v0 + u * stride;
        dst[u] = -1;
        if (v >= total_vecs) continue;
        int lo = 0, hi = nseg - 1;  // last segment with vec_begin <= v
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (segs[mid].vec_begin <= v) lo = mid;
          else hi = mid - 1;
        }
        const TbCopySeg& g = segs[lo];
        const long long vpr = g.row_bytes >> 4;
        const long long e = v - g.vec_begin, row = e / vpr, col = e - row * vpr;
        const char* sp = (g.src_sel ? src1 : src0) + g.src_off + row * g.src_ld + col * 16;
        val[u] = *reinterpret_cast<const uint4*>(sp);
        dst[u] = dst_base + g.dst_off + row * g.dst_ld + col * 16;
        all[u] = g.peers;
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        if (dst[u] < 0) continue;
        if (all[u]) {
          for (int p = 0; p < t.world; ++p)
            *reinterpret_cast<uint4*>(static_cast<char*>(t.base[p]) + dst[u]) = val[u];
        } else {
          *reinterpret_cast<uint4*>(static_cast<char*>(t.base[t.rank]) + dst[u]) = val[u];
        }
      }
    }
  }
  publish_and_finish(t, epoch, done_ctr, err);
}

int grid_for(long long n, int world) {
  const long long per = (n / 4 + world) / world;
  long long g = (per + kBlock - 1) / kBlock;
  if (g > 148) g = 148;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

// The collectives' bounded wait on its own: one thread waits for flags[0..n)
// to reach `expect` for at most budget_ns, then records `site` in the error
// word and returns.  Lets a test make a wait run out (a flag that nothing
// sets) and check that the kernel ends with an error status instead of
// hanging, without a second rank.
__global__ void bounded_wait_probe_kernel(const unsigned* flags, int n, unsigned expect,
                                          unsigned long long budget_ns, int* err) {
  if (threadIdx.x == 0 && blockIdx.x == 0) wait_all(flags, n, expect, err, 99, budget_ns);
}

}  // namespace

extern "C" {

size_t tb_peer_header_bytes() { return sizeof(Hdr); }

void tb_peer_owned_slice(long long n, int rank, int world, long long* lo, long long* hi) {
  owned_slice(n, rank, world, *lo, *hi);
}

int tb_peer_allreduce(TbPeerTable t, long long in_off, long long out_off, long long n, float scale,
                      unsigned* done_ctr, int* err, cudaStream_t s) {
  if (t.world < 1 || t.world > TB_MAX_PEERS || (in_off & 15) || (out_off & 15)) return static_cast<int>(cudaErrorInvalidValue);
  allreduce_kernel<<<grid_for(n, t.world), kBlock, 0, s>>>(t, in_off, out_off, n, scale, done_ctr, err);
  return static_cast<int>(cudaGetLastError());
}

int tb_peer_allreduce_adam(TbPeerTable t, long long grad_off, long long param_off, long long shadow_off, long long n,
                           float* m, float* v, TbAdamParams hp, const long long* step_ptr, unsigned* done_ctr,
                           int* err, cudaStream_t s) {
  if (t.world < 1 || t.world > TB_MAX_PEERS || (grad_off & 15) || (param_off & 15) || (shadow_off & 7))
    return static_cast<int>(cudaErrorInvalidValue);
  allreduce_adam_kernel<<<grid_for(n, t.world), kBlock, 0, s>>>(t, grad_off, param_off, shadow_off, n, m, v, hp,
                                                                step_ptr, done_ctr, err);
  return static_cast<int>(cudaGetLastError());
}

int tb_peer_allreduce_adam_rep(TbPeerTable t, long long grad_off, long long send_off, long long param_off,
                               long long shadow_off, long long n, float* m, float* v, TbAdamParams hp,
                               const long long* step_ptr, unsigned* rep_epoch, unsigned* done_ctr, int* err,
                               cudaStream_t s) {
  if (t.world < 1 || t.world > TB_MAX_PEERS || n <= 0 || (grad_off & 15) || (send_off & 15) || (param_off & 15) ||
      (shadow_off & 7))
    return static_cast<int>(cudaErrorInvalidValue);
  // one float4 per thread where possible; the same grid on every rank (it depends on n only)
  long long g = ((n + 3) / 4 + kBlock - 1) / kBlock;
  if (g > kRepBlocks) g = kRepBlocks;
  allreduce_adam_rep_kernel<<<static_cast<int>(g), kBlock, 0, s>>>(t, grad_off, send_off, param_off, shadow_off, n, m,
                                                                   v, hp, step_ptr, rep_epoch, done_ctr, err);
  return static_cast<int>(cudaGetLastError());
}

int tb_peer_scatter_copy(TbPeerTable t, const void* src0, const void* src1, const TbCopySeg* segs, int nseg,
                         long long total_vecs, long long dst_base, unsigned* done_ctr, int* err, cudaStream_t s) {
  if (t.world < 1 || t.world > TB_MAX_PEERS || nseg <= 0 || total_vecs < 0 || (dst_base & 15) ||
      (reinterpret_cast<uintptr_t>(src0) & 15) || (reinterpret_cast<uintptr_t>(src1) & 15))
    return static_cast<int>(cudaErrorInvalidValue);
  long long g = (total_vecs + kBlock * 4 - 1) / (kBlock * 4);
  if (g > 4 * 148) g = 4 * 148;
  if (g < 1) g = 1;
  scatter_copy_kernel<<<static_cast<int>(g), kBlock, 0, s>>>(t, static_cast<const char*>(src0),
                                                              static_cast<const char*>(src1), segs, nseg, total_vecs,
                                                              dst_base, done_ctr, err);
  return static_cast<int>(cudaGetLastError());
}

int tb_bounded_wait_probe(const unsigned* flags, int n, unsigned expect, unsigned long long budget_ns, int* err,
                          cudaStream_t s) {
  if (n <= 0 || n > TB_MAX_PEERS) return static_cast<int>(cudaErrorInvalidValue);
  bounded_wait_probe_kernel<<<1, 32, 0, s>>>(flags, n, expect, budget_ns, err);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
