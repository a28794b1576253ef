// Replay-buffer kernels: batched ring push, uniform sampling and the
// prioritized sum-tree.
//
// Parity: the reference pushes and samples with one cudaMemcpy per field per
// row and draws indices on the host (turbol_vllm/src/replay_buffer/
// replay_buffer.cpp:55-149); its unused ring_buffer_push kernel reserves slots
// once per block (turbol_vllm/src/cuda/ring_buffer.cu:25).  Here one launch
// moves every field of a batch: the head is advanced on the host, rows wrap
// modulo the capacity, and each thread copies one 16-, 4- or 1-byte chunk of
// one row of one field (gridDim.y = field).  Sampling draws Philox indices and
// gathers in the same launch.  The prioritized tree follows the segment-tree
// design of docs/SPECIFICATION.md:841-864,982-1025 (the reference never
// implemented it).
#include <cuda_runtime.h>
#include <stdint.h>

#include "device_common.cuh"
#include "kernels.h"

namespace {

constexpr int kBlock = 256;

template <typename V>
__global__ void ring_copy_kernel(TbFieldSet fs, int rows, long long head, long long cap, const int* __restrict__ idx,
                                 int mode) {
  const TbField f = fs.f[blockIdx.y];
  const int vec = f.row_bytes / static_cast<int>(sizeof(V));
  const long long total = static_cast<long long>(rows) * vec;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = e / vec;
    const int c = static_cast<int>(e - r * vec);
    long long src_row, dst_row;
    if (mode == 0) {  // push: src row r -> ring slot (head + r) mod cap
      src_row = r;
      dst_row = (head + r) % cap;
    } else {  // gather: ring slot idx[r] -> dst row r
      src_row = idx[r];
      dst_row = r;
    }
    const V* s = reinterpret_cast<const V*>(static_cast<const char*>(f.src) + src_row * f.row_bytes);
    V* d = reinterpret_cast<V*>(static_cast<char*>(f.dst) + dst_row * f.row_bytes);
    d[c] = s[c];
  }
}

__global__ void sample_indices_kernel(int* __restrict__ idx, int n, long long size, unsigned long long seed,
                                      unsigned long long counter) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint4 r = tb::Philox::gen(seed, static_cast<uint32_t>(i), static_cast<uint32_t>(counter),
                                  static_cast<uint32_t>(counter >> 32), 0x52504C59u);
  idx[i] = static_cast<int>(tb::uniform_int(r.x, static_cast<uint32_t>(size)));
}

// Picks the widest vector width that every field of the set supports.
int vector_width(const TbFieldSet& fs, int nf) {
  int w = 16;
  for (int k = 0; k < nf; ++k) {
    const TbField& f = fs.f[k];
    const auto a = reinterpret_cast<uintptr_t>(f.src) | reinterpret_cast<uintptr_t>(f.dst);
    while (w > 1 && ((f.row_bytes % w) != 0 || (a % w) != 0)) w >>= 1;
  }
  return w >= 16 ? 16 : (w >= 4 ? 4 : 1);
}

int launch_ring_copy(const TbFieldSet& fs, int nf, int rows, long long head, long long cap, const int* idx, int mode,
                     cudaStream_t s) {
  if (rows <= 0 || nf <= 0) return 0;
  if (nf > TB_MAX_FIELDS) return static_cast<int>(cudaErrorInvalidValue);
  int max_row = 0;
  for (int k = 0; k < nf; ++k) max_row = max_row > fs.f[k].row_bytes ? max_row : fs.f[k].row_bytes;
  const int w = vector_width(fs, nf);
  const long long work = static_cast<long long>(rows) * (max_row / w);
  long long g = (work + kBlock - 1) / kBlock;
  if (g > 148 * 16) g = 148 * 16;  // grid-stride beyond 16 CTAs per SM
  if (g < 1) g = 1;
  dim3 grid(static_cast<unsigned>(g), nf);
  if (w == 16)
    ring_copy_kernel<uint4><<<grid, kBlock, 0, s>>>(fs, rows, head, cap, idx, mode);
  else if (w == 4)
    ring_copy_kernel<uint32_t><<<grid, kBlock, 0, s>>>(fs, rows, head, cap, idx, mode);
  else
    ring_copy_kernel<uint8_t><<<grid, kBlock, 0, s>>>(fs, rows, head, cap, idx, mode);
  return static_cast<int>(cudaGetLastError());
}

// ----------------------------------------------------------------------------
// Sum-tree (1-indexed heap of 2L floats; leaves at [L, 2L)).
// ----------------------------------------------------------------------------
__global__ void per_set_leaves_kernel(float* __restrict__ tree, long long L, const long long* __restrict__ idx,
                                      const float* __restrict__ prio, int n, float alpha, float eps,
                                      long long capacity, tb::ErrorWord* ew) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const long long k = idx[i];
  if (k < 0 || k >= capacity) {
    tb::report_error(ew, tb::kErrIndex, 20, static_cast<unsigned long long>(k));
    return;
  }
  tree[L + k] = powf(fabsf(prio[i]) + eps, alpha);
}

// Recomputes the parents, `level` steps above the leaves, of the touched
// leaves.  Siblings that share a parent write the same value, so duplicates
// are benign.
__global__ void per_propagate_kernel(float* __restrict__ tree, long long L, const long long* __restrict__ idx, int n,
                                     int level, long long capacity) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const long long k = idx[i];
  if (k < 0 || k >= capacity) return;
  const long long node = (L + k) >> level;
  tree[node] = tree[2 * node] + tree[2 * node + 1];
}

// Rebuilds one full level: parents [lo, 2*lo) from their children.
__global__ void per_rebuild_level_kernel(float* __restrict__ tree, long long lo) {
  for (long long j = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; j < lo;
       j += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long node = lo + j;
    tree[node] = tree[2 * node] + tree[2 * node + 1];
  }
}

// Stratified sampling: sample i draws u uniformly in [i, i+1) * total/n and
// descends the tree to the leaf whose prefix-sum interval holds u.
// IS weight w = (size * P(i))^-beta; weights are divided by the batch maximum
// in per_normalize_kernel.
__global__ void per_sample_kernel(const float* __restrict__ tree, long long L, long long size, int n, float beta,
                                  unsigned long long seed, unsigned long long counter, long long* __restrict__ out_idx,
                                  float* __restrict__ out_w, float* __restrict__ out_p, unsigned* __restrict__ wmax_bits) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  float w = 0.f;
  if (i < n) {
    const float total = tree[1];
    const float seg = total / static_cast<float>(n);
    const uint4 r = tb::Philox::gen(seed, static_cast<uint32_t>(i), static_cast<uint32_t>(counter),
                                    static_cast<uint32_t>(counter >> 32), 0x50455253u);
    float u = (static_cast<float>(i) + tb::u01(r.x)) * seg;
    long long node = 1;
    while (node < L) {
      const float left = tree[2 * node];
      if (u < left || tree[2 * node + 1] <= 0.f) {
        node = 2 * node;
      } else {
        u -= left;
        node = 2 * node + 1;
      }
    }
    long long leaf = node - L;
    if (leaf >= size) leaf = size - 1;  // rounding at the right edge
    const float p = tree[L + leaf] / total;
    w = powf(static_cast<float>(size) * p, -beta);
    out_idx[i] = leaf;
    out_w[i] = w;
    if (out_p) out_p[i] = p;
  }
  // positive floats order like their bit patterns
  float m = tb::warp_max(w);
  if ((threadIdx.x & 31) == 0 && m > 0.f) atomicMax(wmax_bits, __float_as_uint(m));
}

__global__ void per_normalize_kernel(float* __restrict__ w, int n, const unsigned* __restrict__ wmax_bits) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float m = __uint_as_float(*wmax_bits);
  w[i] = m > 0.f ? w[i] / m : 1.f;
}

}  // namespace

extern "C" {

int tb_ring_push(TbFieldSet fs, int nf, int rows, long long head, long long capacity, cudaStream_t s) {
  return launch_ring_copy(fs, nf, rows, head, capacity, nullptr, 0, s);
}

int tb_ring_gather(TbFieldSet fs, int nf, int rows, const int* idx, cudaStream_t s) {
  return launch_ring_copy(fs, nf, rows, 0, 1, idx, 1, s);
}

int tb_sample_indices(int* idx, int n, long long size, unsigned long long seed, unsigned long long counter,
                      cudaStream_t s) {
  if (n <= 0) return 0;
  if (size <= 0) return static_cast<int>(cudaErrorInvalidValue);
  sample_indices_kernel<<<(n + kBlock - 1) / kBlock, kBlock, 0, s>>>(idx, n, size, seed, counter);
  return static_cast<int>(cudaGetLastError());
}

int tb_per_update(float* tree, long long L, const long long* idx, const float* prio, int n, float alpha, float eps,
                  long long capacity, void* error_word, cudaStream_t s) {
  if (n <= 0) return 0;
  const int g = (n + kBlock - 1) / kBlock;
  per_set_leaves_kernel<<<g, kBlock, 0, s>>>(tree, L, idx, prio, n, alpha, eps, capacity,
                                             static_cast<tb::ErrorWord*>(error_word));
  int levels = 0;
  while ((1LL << levels) < L) ++levels;
  for (int lv = 1; lv <= levels; ++lv) {
    const long long width = L >> lv;  // nodes on this level
    if (width <= n) {
      // the touched set covers this level: rebuild it whole (cheaper, no duplicates)
      per_rebuild_level_kernel<<<static_cast<unsigned>((width + kBlock - 1) / kBlock), kBlock, 0, s>>>(tree, width);
    } else {
      per_propagate_kernel<<<g, kBlock, 0, s>>>(tree, L, idx, n, lv, capacity);
    }
  }
  return static_cast<int>(cudaGetLastError());
}

int tb_per_rebuild(float* tree, long long L, cudaStream_t s) {
  for (long long width = L >> 1; width >= 1; width >>= 1) {
    long long g = (width + kBlock - 1) / kBlock;
    if (g > 148 * 32) g = 148 * 32;
    per_rebuild_level_kernel<<<static_cast<unsigned>(g), kBlock, 0, s>>>(tree, width);
  }
  return static_cast<int>(cudaGetLastError());
}

int tb_per_sample(const float* tree, long long L, long long size, int n, float beta, unsigned long long seed,
                  unsigned long long counter, long long* out_idx, float* out_w, float* out_p, unsigned* wmax_scratch,
                  cudaStream_t s) {
  if (n <= 0) return 0;
  if (size <= 0) return static_cast<int>(cudaErrorInvalidValue);
  cudaMemsetAsync(wmax_scratch, 0, sizeof(unsigned), s);
  const int g = (n + kBlock - 1) / kBlock;
  per_sample_kernel<<<g, kBlock, 0, s>>>(tree, L, size, n, beta, seed, counter, out_idx, out_w, out_p, wmax_scratch);
  per_normalize_kernel<<<g, kBlock, 0, s>>>(out_w, n, wmax_scratch);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
