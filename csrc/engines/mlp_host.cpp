// The CPU trainer's PPO steps without autograd or per-operator dispatch: the
// forward of the actor and critic MLPs (tanh hidden layers), the
// clipped-surrogate PPO loss for a categorical actor with the value and
// entropy terms, the hand-written backward into the flat gradient, the update
// loop with Adam, and the CartPole rollout (forward, sampling, environment
// step).
//
// For the minibatches of a CPU PPO run (tens of rows, widths of 64-256) an
// ATen matrix product costs 7-15 us per call, mostly dispatch, allocation and
// thread-pool entry, against about 3 us of arithmetic; a step has ~16 of them
// plus the tanh passes.  Here every product is a register-tiled loop over
// native-width float vectors (GCC vector types), compiled three times
// (AVX-512, AVX2 + FMA, baseline x86-64 with SSE) and chosen once at run time
// from the CPU's features (TURBOL_HOST_ISA can name a narrower one).  tanh is
// a vectorized restatement through expm1 (below).  A large minibatch or
// rollout batch is split by rows over torch's intra-op thread count.
//
// Reference: turbol_vllm/src/policy/policy_engine.cpp:103-138 (the reference's
// PolicyEngine::Update: one autograd step of a linear Gaussian policy through
// libtorch); this file is the categorical MLP actor-critic PPO step of the CPU
// trainer.
#include <ATen/ATen.h>
#include <ATen/Parallel.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <system_error>
#include <thread>
#include <vector>

#include "turbol/engines.hpp"

namespace turbol {

namespace {

#define TB_INLINE static inline __attribute__((always_inline))
// Attributes of the AVX-512 and AVX2 entry points (see the end of this
// namespace); fp-contract=fast lets the compiler fuse the products'
// multiply-adds where the target has FMA (the rest of the host core is built
// without contraction).
#define TB_AVX512 __attribute__((target("avx512f,avx512vl,avx2,fma,prefer-vector-width=512"), optimize("fp-contract=fast")))
#define TB_AVX2 __attribute__((target("avx2,fma"), optimize("fp-contract=fast")))

// The vector values below never cross a call boundary (every helper is
// inlined into the per-instruction-set entry points), so the note that their
// by-value ABI depends on the instruction set does not apply.
#pragma GCC diagnostic ignored "-Wpsabi"

// Native vectors of W floats: 16 (one AVX-512 register), 8 (AVX2) or 4 (SSE),
// one width per instruction-set entry point below
template <int W>
struct Vec;
template <>
struct Vec<16> {
  typedef float f __attribute__((vector_size(64)));
  typedef int32_t i __attribute__((vector_size(64)));
};
template <>
struct Vec<8> {
  typedef float f __attribute__((vector_size(32)));
  typedef int32_t i __attribute__((vector_size(32)));
};
template <>
struct Vec<4> {
  typedef float f __attribute__((vector_size(16)));
  typedef int32_t i __attribute__((vector_size(16)));
};
constexpr int64_t kMaxLanes = 16;  // the widest W: row width of the padded scratch

template <int W>
TB_INLINE typename Vec<W>::f vload(const float* p) {
  typename Vec<W>::f v;
  __builtin_memcpy(&v, p, sizeof v);
  return v;
}
template <int W>
TB_INLINE void vstore(float* p, typename Vec<W>::f v) {
  __builtin_memcpy(p, &v, sizeof v);
}

// tanh.  tanh(x) = sign(x) * -m / (2 + m) with m = expm1(-2|x|), and
// expm1(z) = 2^k (q + 1) - 1 = 2^k q + (2^k - 1) with z = k ln2 + r,
// |r| <= ln2 / 2 (Cody and Waite's range reduction, ln2 split into a short
// high part and a correction) and q = expm1(r) from its Taylor series to r^7
// (truncation < 2e-8 relative).  For k = 0 the result is q itself, so small
// |x| keep full relative accuracy.  |x| >= 10 gives +-1 (tanh(10) rounds to 1
// in float).  Rounding to the nearest integer uses the 1.5 * 2^23 shift.
// Measured: max abs error 1.4e-7 against the fp64 tanh over [-5, 5].
constexpr float kLog2e = 1.44269504088896341f;
constexpr float kLn2Hi = 0.693145751953125f;      // 0x3f317200: ln2 rounded to 16 significant bits
constexpr float kLn2Lo = 1.42860682030941723e-6f;  // ln2 - kLn2Hi
constexpr float kShift = 12582912.f;               // 1.5 * 2^23

template <int W>
TB_INLINE typename Vec<W>::f tanh_v(typename Vec<W>::f x) {
  using vf = typename Vec<W>::f;
  using vi = typename Vec<W>::i;
  const vi bits = __builtin_bit_cast(vi, x);
  const vi sign = bits & INT32_MIN;
  vf z = -2.f * __builtin_bit_cast(vf, vi(bits & INT32_MAX));
  z = z < -20.f ? vf{} - 20.f : z;
  const vf kf = (z * kLog2e + kShift) - kShift;  // nearest integer, in [-29, 0]
  const vf r = (z - kf * kLn2Hi) - kf * kLn2Lo;
  vf q = vf{} + 1.f / 5040.f;
  q = q * r + 1.f / 720.f;
  q = q * r + 1.f / 120.f;
  q = q * r + 1.f / 24.f;
  q = q * r + 1.f / 6.f;
  q = q * r + 0.5f;
  q = q * r + 1.f;
  q = q * r;
  const vf s = __builtin_bit_cast(vf, vi((__builtin_convertvector(kf, vi) + 127) << 23));  // 2^k, normal for k >= -29
  const vf m = s * q + (s - 1.f);
  const vf t = -m / (2.f + m);
  return __builtin_bit_cast(vf, vi(__builtin_bit_cast(vi, t) ^ sign));
}

template <int W>
TB_INLINE void tanh_inplace(float* v, int64_t n) {
  int64_t j = 0;
  for (; j + W <= n; j += W) vstore<W>(v + j, tanh_v<W>(vload<W>(v + j)));
  if (j < n) {
    float tmp[W] = {};
    __builtin_memcpy(tmp, v + j, sizeof(float) * (n - j));
    vstore<W>(tmp, tanh_v<W>(vload<W>(tmp)));
    __builtin_memcpy(v + j, tmp, sizeof(float) * (n - j));
  }
}

// How a product's output tile starts: zeros, the bias row, or the output's current values.
enum class Init { kZero, kBias, kAccumulate };

// C[0:R, 0:W*V] = init + sum_k A(r, k) B[k, 0:W*V], A(r, k) = A[r * sam + k * sak];
// the R x V accumulators stay in registers for the whole k loop.
template <int W, int R, int V>
TB_INLINE void gemm_tile(const float* A, int64_t sam, int64_t sak, const float* Bm, int64_t ldb, int64_t K, float* C,
                         int64_t ldc, const float* bias, Init init) {
  using vf = typename Vec<W>::f;
  vf acc[R][V];
#pragma GCC unroll 8
  for (int r = 0; r < R; ++r)
#pragma GCC unroll 2
    for (int v = 0; v < V; ++v)
      acc[r][v] = init == Init::kAccumulate ? vload<W>(C + r * ldc + v * W)
                  : init == Init::kBias     ? vload<W>(bias + v * W)
                                            : vf{};
  for (int64_t k = 0; k < K; ++k) {
    vf b[V];
#pragma GCC unroll 2
    for (int v = 0; v < V; ++v) b[v] = vload<W>(Bm + k * ldb + v * W);
#pragma GCC unroll 8
    for (int r = 0; r < R; ++r) {
      const float a = A[r * sam + k * sak];
#pragma GCC unroll 2
      for (int v = 0; v < V; ++v) acc[r][v] += a * b[v];
    }
  }
#pragma GCC unroll 8
  for (int r = 0; r < R; ++r)
#pragma GCC unroll 2
    for (int v = 0; v < V; ++v) vstore<W>(C + r * ldc + v * W, acc[r][v]);
}

// Row blocks of 8 with AVX-512 (16 accumulators + 2 operands of its 32
// registers), else 4 (8 + 2 of 16), then single rows.
template <int W, int V>
TB_INLINE void gemm_rows(int64_t M, int64_t K, const float* A, int64_t sam, int64_t sak, const float* Bm, int64_t ldb,
                         float* C, int64_t ldc, const float* bias, Init init) {
  int64_t m = 0;
  if constexpr (W == 16)
    for (; m + 8 <= M; m += 8) gemm_tile<W, 8, V>(A + m * sam, sam, sak, Bm, ldb, K, C + m * ldc, ldc, bias, init);
  for (; m + 4 <= M; m += 4) gemm_tile<W, 4, V>(A + m * sam, sam, sak, Bm, ldb, K, C + m * ldc, ldc, bias, init);
  for (; m < M; ++m) gemm_tile<W, 1, V>(A + m * sam, sam, sak, Bm, ldb, K, C + m * ldc, ldc, bias, init);
}

// C[M, N] = init + A[M, K] B[K, N] with A(m, k) = A[m * sam + k * sak] (any
// strides: a plain, a transposed or a strided operand), B's rows ldb apart and
// C's rows ldc apart.  Column blocks of 2W, then W; the columns past the last
// multiple of W go through W-wide zero-padded copies (pb: K x W floats,
// pc: M x W floats).
template <int W>
TB_INLINE void gemm(int64_t M, int64_t N, int64_t K, const float* A, int64_t sam, int64_t sak, const float* Bm,
                    int64_t ldb, float* C, int64_t ldc, const float* bias, Init init, float* pb, float* pc) {
  int64_t n = 0;
  for (; n + 2 * W <= N; n += 2 * W)
    gemm_rows<W, 2>(M, K, A, sam, sak, Bm + n, ldb, C + n, ldc, bias ? bias + n : nullptr, init);
  for (; n + W <= N; n += W)
    gemm_rows<W, 1>(M, K, A, sam, sak, Bm + n, ldb, C + n, ldc, bias ? bias + n : nullptr, init);
  if (n == N) return;
  const int64_t w = N - n;
  for (int64_t k = 0; k < K; ++k) {
    float* row = pb + k * W;
    for (int64_t j = 0; j < W; ++j) row[j] = j < w ? Bm[k * ldb + n + j] : 0.f;
  }
  float pbias[W] = {};
  if (bias)
    for (int64_t j = 0; j < w; ++j) pbias[j] = bias[n + j];
  if (init == Init::kAccumulate)
    for (int64_t m = 0; m < M; ++m)
      for (int64_t j = 0; j < W; ++j) pc[m * W + j] = j < w ? C[m * ldc + n + j] : 0.f;
  gemm_rows<W, 1>(M, K, A, sam, sak, pb, W, pc, W, pbias, init);
  for (int64_t m = 0; m < M; ++m)
    for (int64_t j = 0; j < w; ++j) C[m * ldc + n + j] = pc[m * W + j];
}

// Allocator for the workspace vectors: 64-byte (cache-line) aligned, so that
// a vector load of a row that starts at a multiple of 16 floats stays in one line.
template <typename T>
struct LineAllocator {
  using value_type = T;
  LineAllocator() = default;
  template <typename U>
  LineAllocator(const LineAllocator<U>&) {}
  T* allocate(size_t n) { return static_cast<T*>(::operator new(n * sizeof(T), std::align_val_t(64))); }
  void deallocate(T* p, size_t) { ::operator delete(p, std::align_val_t(64)); }
  template <typename U>
  bool operator==(const LineAllocator<U>&) const { return true; }
  template <typename U>
  bool operator!=(const LineAllocator<U>&) const { return false; }
};
using Buf = std::vector<float, LineAllocator<float>>;

struct Mlp {
  std::vector<int64_t> dims;  // widths dims[0] -> ... -> dims[L]
  std::vector<int64_t> woff;  // per layer: offset of W [out, in] in the flat buffers (b follows W)
};

Mlp mlp_layout(const std::vector<int64_t>& dims, int64_t* off) {
  Mlp m{dims, {}};
  for (size_t l = 0; l + 1 < dims.size(); ++l) {
    m.woff.push_back(*off);
    *off += dims[l + 1] * (dims[l] + 1);
  }
  return m;
}

// Buffers of one minibatch step (or one rollout step), sized once for B rows and reused.
struct Workspace {
  int64_t B = 0;
  Buf x;                   // [B, dims[0]] gathered observations
  std::vector<Buf> ha, hc;  // per layer: output [B, dims[l + 1]] (tanh applied on hidden layers)
  Buf d0, d1, wt;          // gradient ping-pong [B, max width], W^T of one layer
  Buf pb, pc;              // W-wide padded operand / output of a product's last columns

  void size_for(const Mlp& a, const Mlp& c, int64_t rows) {
    B = rows;
    int64_t wmax = 0, wt_max = 0;
    for (const Mlp* m : {&a, &c})
      for (size_t l = 0; l < m->dims.size(); ++l) {
        wmax = std::max(wmax, m->dims[l]);
        if (l + 1 < m->dims.size()) wt_max = std::max(wt_max, m->dims[l] * m->dims[l + 1]);
      }
    x.assign(static_cast<size_t>(rows * a.dims[0]), 0.f);
    auto make = [&](const Mlp& m, std::vector<Buf>* h) {
      h->clear();
      for (size_t l = 0; l + 1 < m.dims.size(); ++l) h->emplace_back(static_cast<size_t>(rows * m.dims[l + 1]));
    };
    make(a, &ha);
    make(c, &hc);
    d0.assign(static_cast<size_t>(rows * wmax), 0.f);
    d1.assign(static_cast<size_t>(rows * wmax), 0.f);
    wt.assign(static_cast<size_t>(wt_max), 0.f);
    const int64_t mk = std::max(rows, wmax);  // the largest M and K of the step's products
    pb.assign(static_cast<size_t>(mk * kMaxLanes), 0.f);
    pc.assign(static_cast<size_t>(mk * kMaxLanes), 0.f);
  }
};

// h[l] = tanh(h[l - 1] W_l^T + b_l) (no tanh on the last layer), h[-1] = x
template <int W>
TB_INLINE void mlp_forward(const Mlp& m, const float* p, const float* x, Workspace* ws,
                           std::vector<Buf>* h) {
  const size_t L = m.dims.size() - 1;
  const int64_t B = ws->B;
  const float* in = x;
  for (size_t l = 0; l < L; ++l) {
    const int64_t ni = m.dims[l], no = m.dims[l + 1];
    const float* Wl = p + m.woff[l];
    // W^T in 16 x 16 blocks: a plain column-order copy writes rows of wt
    // no floats apart and evicts its own lines (6x slower at 256 x 256)
    float* wt = ws->wt.data();
    for (int64_t o0 = 0; o0 < no; o0 += 16)
      for (int64_t k0 = 0; k0 < ni; k0 += 16) {
        const int64_t oe = std::min(o0 + 16, no), ke = std::min(k0 + 16, ni);
        for (int64_t o = o0; o < oe; ++o)
          for (int64_t k = k0; k < ke; ++k) wt[k * no + o] = Wl[o * ni + k];
      }
    float* y = (*h)[l].data();
    gemm<W>(B, no, ni, in, ni, 1, wt, no, y, no, Wl + no * ni, Init::kBias, ws->pb.data(), ws->pc.data());
    if (l + 1 < L) tanh_inplace<W>(y, B * no);
    in = y;
  }
}

// Backward from d(output), which is in ws->d0 ([B, dims[L]]); d0 / d1 are clobbered.
// Per layer: gb += column sums of dy, gW += dy^T input, dx = dy W, then dx *= 1 - h^2.
template <int W>
TB_INLINE void mlp_backward(const Mlp& m, const float* p, float* g, const float* x, Workspace* ws,
                            const std::vector<Buf>& h) {
  const int64_t B = ws->B;
  float* d = ws->d0.data();
  float* dn = ws->d1.data();
  for (size_t l = m.dims.size() - 1; l-- > 0;) {
    const int64_t ni = m.dims[l], no = m.dims[l + 1];
    const float* input = l == 0 ? x : h[l - 1].data();
    const float* Wl = p + m.woff[l];
    float* gW = g + m.woff[l];
    float* gb = gW + no * ni;
    for (int64_t i = 0; i < B; ++i)
      for (int64_t o = 0; o < no; ++o) gb[o] += d[i * no + o];
    gemm<W>(no, ni, B, d, 1, no, input, ni, gW, ni, nullptr, Init::kAccumulate, ws->pb.data(), ws->pc.data());
    if (l == 0) break;
    gemm<W>(B, ni, no, d, no, 1, Wl, ni, dn, ni, nullptr, Init::kZero, ws->pb.data(), ws->pc.data());
    const float* hp = h[l - 1].data();
    for (int64_t e = 0; e < B * ni; ++e) dn[e] *= 1.f - hp[e] * hp[e];
    std::swap(d, dn);
  }
}

struct LossArgs {
  const int* act;
  const float *old_logp, *adv, *ret;
  int64_t n_all;
  float clip, vf_coef, ent_coef;
};

// Forward, loss and backward for the rows idx[0:ws->B] of a minibatch whose
// loss is averaged with inv_b (1 / its row count, which may be more rows than
// this call's when threads share the minibatch); adds the gradient into g and
// the loss statistics to st[0:6].
// Inlined (like every helper above) into the per-instruction-set entry points
// below, so that it is compiled for their targets.
template <int W>
TB_INLINE Status minibatch_step(const Mlp& a, const Mlp& c, const float* p, float* g, const float* obs,
                                int64_t obs_rows, const int64_t* idx, const LossArgs& la, Workspace* ws, float inv_b,
                                float* st) {
  const int64_t B = ws->B, O = a.dims[0], A = a.dims.back();
  for (int64_t i = 0; i < B; ++i) {
    const int64_t row = idx[i];
    if (row < 0 || row >= obs_rows || row >= la.n_all)
      return Status::InvalidArgument("ppo minibatch: row index out of range");
    std::memcpy(ws->x.data() + i * O, obs + row * O, sizeof(float) * O);
  }
  mlp_forward<W>(a, p, ws->x.data(), ws, &ws->ha);
  mlp_forward<W>(c, p, ws->x.data(), ws, &ws->hc);
  const float* L = ws->ha.back().data();
  const float* V = ws->hc.back().data();
  float* dL = ws->d0.data();
  double s_pg = 0, s_v = 0, s_ent = 0, s_kl = 0, s_clip = 0;
  std::vector<float> lsm(A), pr(A);
  for (int64_t i = 0; i < B; ++i) {
    const float* li = L + i * A;
    float mx = li[0];
    for (int64_t j = 1; j < A; ++j) mx = std::max(mx, li[j]);
    float se = 0.f;
    for (int64_t j = 0; j < A; ++j) se += std::exp(li[j] - mx);
    const float lse = mx + std::log(se);
    float ent = 0.f;
    for (int64_t j = 0; j < A; ++j) {
      lsm[j] = li[j] - lse;
      pr[j] = std::exp(lsm[j]);
      ent -= pr[j] * lsm[j];
    }
    const int64_t row = idx[i];
    const int act = la.act[row];
    if (act < 0 || act >= A) return Status::InvalidArgument("ppo minibatch: action out of range");
    const float adv = la.adv[row];
    const float logp = lsm[act], dlp = logp - la.old_logp[row], ratio = std::exp(dlp);
    const float unc = ratio * adv, clp = std::min(std::max(ratio, 1.f - la.clip), 1.f + la.clip) * adv;
    const float pg = -std::min(unc, clp);
    // d pg / d logp = -ratio * adv where the unclipped term is the minimum (or the ratio is inside the clip range)
    const float g_lp = (unc <= clp || (ratio > 1.f - la.clip && ratio < 1.f + la.clip)) ? -unc * inv_b : 0.f;
    // d(-ent_coef * mean(ent)) / d logits_j = ent_coef / B * p_j (log p_j + ent)
    for (int64_t j = 0; j < A; ++j)
      dL[i * A + j] = g_lp * ((j == act ? 1.f : 0.f) - pr[j]) + la.ent_coef * inv_b * pr[j] * (lsm[j] + ent);
    const float dv = V[i] - la.ret[row];
    s_pg += pg;
    s_v += 0.5f * dv * dv;
    s_ent += ent;
    s_kl += (ratio - 1.f) - dlp;
    s_clip += std::fabs(ratio - 1.f) > la.clip ? 1.0 : 0.0;
  }
  mlp_backward<W>(a, p, g, ws->x.data(), ws, ws->ha);
  float* dV = ws->d0.data();
  for (int64_t i = 0; i < B; ++i) dV[i] = la.vf_coef * (V[i] - la.ret[idx[i]]) * inv_b;
  mlp_backward<W>(c, p, g, ws->x.data(), ws, ws->hc);
  st[0] += static_cast<float>(s_pg);
  st[1] += static_cast<float>(s_v);
  st[2] += static_cast<float>(s_ent);
  st[3] += static_cast<float>(s_kl);
  st[4] += static_cast<float>(s_clip);
  st[5] += static_cast<float>(B);
  return Status::Ok();
}

// One thread's share of a minibatch: rows idx[0:ws->B], gradient added into
// g, statistics into st.
struct Chunk {
  const Mlp* a;
  const Mlp* c;
  const float* p;
  float* g;
  const float* obs;
  int64_t obs_rows;
  const int64_t* idx;
  const LossArgs* la;
  Workspace* ws;
  float inv_b;
  float st[6];
  Status status;
};

template <int W>
TB_INLINE void run_chunk(Chunk* k) {
  k->status = minibatch_step<W>(*k->a, *k->c, k->p, k->g, k->obs, k->obs_rows, k->idx, *k->la, k->ws, k->inv_b, k->st);
}
// thread entry points, compiled for their instruction set like the callers
TB_AVX512 void chunk_avx512(Chunk* k) { run_chunk<16>(k); }
TB_AVX2 void chunk_avx2(Chunk* k) { run_chunk<8>(k); }
void chunk_base(Chunk* k) { run_chunk<4>(k); }

// Runs fn on every chunk: chunks 1.. on threads of their own, chunk 0 on the
// calling thread, then joins.  A chunk whose thread cannot be started (the
// process is out of threads) runs on the calling thread instead, so no
// started thread is ever left unjoined.
template <typename C>
void run_chunks(void (*fn)(C*), std::vector<C>& ch) {
  std::vector<std::thread> th;
  th.reserve(ch.size());
  size_t started = 1;
  try {
    for (; started < ch.size(); ++started) th.emplace_back(fn, &ch[started]);
  } catch (const std::system_error&) {
    // the rest run below
  }
  fn(&ch[0]);
  for (size_t k = started; k < ch.size(); ++k) fn(&ch[k]);
  for (auto& x : th) x.join();
}

// Multiply-adds per row of a minibatch step: the forward and the two backward
// products of every layer of both networks.
int64_t macs_per_row(const Mlp& a, const Mlp& c) {
  int64_t s = 0;
  for (const Mlp* m : {&a, &c})
    for (size_t l = 0; l + 1 < m->dims.size(); ++l) s += 3 * m->dims[l] * m->dims[l + 1];
  return s;
}

// Threads for a minibatch of `rows`: at most torch's intra-op thread count,
// each with at least 4 M multiply-adds (~60 us, well above the cost of
// starting a thread) and 8 rows; small minibatches (a CartPole MLP 64-64 at
// 64 rows is 1.7 M) stay on the calling thread.  TURBOL_HOST_THREAD_MACS,
// read once per process, replaces the 4 M (the sanitizer tests lower it to
// split small batches).
int threads_for(int64_t rows, int64_t per_row) {
  static const int64_t min_macs = [] {
    const char* e = std::getenv("TURBOL_HOST_THREAD_MACS");
    const long long v = e ? std::atoll(e) : 0;
    return v > 0 ? static_cast<int64_t>(v) : int64_t{4} << 20;
  }();
  const int64_t p =
      std::min<int64_t>({static_cast<int64_t>(at::get_num_threads()), rows * per_row / min_macs, rows / 8});
  return p < 1 ? 1 : static_cast<int>(p);
}

// The update loop (epochs x minibatches of perms, Adam after each when adam)
// for one instruction set.  A large minibatch is split by rows over threads,
// each with its own workspace and gradient buffer; the buffers are summed
// into g (the sum's order depends on the thread count, not on timing).
template <int W>
TB_INLINE Status update_loop(const Mlp& a, const Mlp& c, float* p, float* g, float* m1, float* m2, int64_t n,
                             int64_t* step, const float* obs, int64_t obs_rows, const int64_t* perms, int64_t epochs,
                             int64_t rows, int64_t minibatch, bool adam, const LossArgs& la, float lr, float b1,
                             float b2, float eps, float wd, float* st) {
  const int P0 = threads_for(minibatch, macs_per_row(a, c));
  const int64_t per = (minibatch + P0 - 1) / P0;
  const int P = static_cast<int>((minibatch + per - 1) / per);  // chunks that hold rows
  std::vector<Workspace> ws(P);
  for (auto& w : ws) w.size_for(a, c, per);
  std::vector<Buf> gbuf(P - 1, Buf(static_cast<size_t>(n)));
  void (*const fn)(Chunk*) = W == 16 ? chunk_avx512 : (W == 8 ? chunk_avx2 : chunk_base);
  const float inv_b = 1.f / static_cast<float>(minibatch);
  const int64_t n_mb = rows / minibatch;
  for (int64_t e = 0; e < epochs; ++e)
    for (int64_t k = 0; k < n_mb; ++k) {
      if (adam) std::fill(g, g + n, 0.f);
      const int64_t* idx = perms + e * rows + k * minibatch;
      if (P == 1) {
        ws[0].B = minibatch;
        TURBOL_RETURN_IF_ERROR(minibatch_step<W>(a, c, p, g, obs, obs_rows, idx, la, &ws[0], inv_b, st));
      } else {
        std::vector<Chunk> ch(P);
        for (int t = 0; t < P; ++t) {
          const int64_t r0 = t * per, r1 = std::min(minibatch, r0 + per);
          ws[t].B = r1 - r0;
          float* gt = t == 0 ? g : gbuf[t - 1].data();
          if (t > 0) std::fill(gt, gt + n, 0.f);
          ch[t] = Chunk{&a, &c, p, gt, obs, obs_rows, idx + r0, &la, &ws[t], inv_b, {0, 0, 0, 0, 0, 0}, Status::Ok()};
        }
        run_chunks(fn, ch);
        for (int t = 0; t < P; ++t) {
          TURBOL_RETURN_IF_ERROR(ch[t].status);
          for (int j = 0; j < 6; ++j) st[j] += ch[t].st[j];
          if (t > 0)
            for (int64_t i = 0; i < n; ++i) g[i] += gbuf[t - 1][i];
        }
      }
      if (adam) AdamHost(p, g, m1, m2, n, ++*step, lr, b1, b2, eps, wd, 1.f);
    }
  return Status::Ok();
}

struct RolloutArgs {
  GPUEnvironment* env;
  float *obs, *logp, *val, *rew;
  int* act;
  uint8_t* done;
  int64_t T, N;
  uint64_t seed, counter;
};

// One thread's rows [row0, row0 + ws->B) of a rollout step: the critic's
// values of the observations ob (rows of the whole batch) and, unless
// values_only, the actor's action and its log-probability.  A row's result
// depends on its own data only (the Philox key is the global env index), so
// any split over threads gives the same rollout.
struct RolloutChunk {
  const Mlp* a;
  const Mlp* c;
  const float* p;
  const float* ob;
  int64_t row0;
  Workspace* ws;
  int* act;
  float* logp;
  float* val;
  bool values_only;
  uint64_t seed;
  uint32_t t, ctr_lo, ctr_hi;
};

template <int W>
TB_INLINE void rollout_rows(RolloutChunk* k) {
  const Mlp& a = *k->a;
  Workspace* ws = k->ws;
  const int64_t O = a.dims[0], A = a.dims.back(), n = ws->B, r0 = k->row0;
  const float* ob = k->ob + r0 * O;
  mlp_forward<W>(*k->c, k->p, ob, ws, &ws->hc);
  const float* V = ws->hc.back().data();
  for (int64_t i = 0; i < n; ++i) k->val[r0 + i] = V[i];
  if (k->values_only) return;
  mlp_forward<W>(a, k->p, ob, ws, &ws->ha);
  const float* L = ws->ha.back().data();
  for (int64_t i = 0; i < n; ++i) {
    const float* li = L + i * A;
    float mx = li[0];
    for (int64_t j = 1; j < A; ++j) mx = std::max(mx, li[j]);
    float se = 0.f;
    for (int64_t j = 0; j < A; ++j) se += std::exp(li[j] - mx);
    const float lse = mx + std::log(se);
    // inverse CDF of the softmax at u in [0, 1): the first action whose
    // cumulative probability passes u (the last one if rounding leaves the sum below u)
    const uint32_t w =
        static_cast<uint32_t>(HostPhiloxWord(k->seed, static_cast<uint32_t>(r0 + i), k->t, k->ctr_lo, k->ctr_hi, 0));
    const float u = static_cast<float>(w >> 8) * (1.0f / 16777216.0f);
    int64_t pick = A - 1;
    float cum = 0.f;
    for (int64_t j = 0; j < A; ++j) {
      cum += std::exp(li[j] - lse);
      if (u < cum) {
        pick = j;
        break;
      }
    }
    k->act[r0 + i] = static_cast<int>(pick);
    k->logp[r0 + i] = li[pick] - lse;
  }
}
// thread entry points, compiled for their instruction set like the callers
TB_AVX512 void rchunk_avx512(RolloutChunk* k) { rollout_rows<16>(k); }
TB_AVX2 void rchunk_avx2(RolloutChunk* k) { rollout_rows<8>(k); }
void rchunk_base(RolloutChunk* k) { rollout_rows<4>(k); }

// The CPU CartPole rollout for one instruction set (see PpoCartPoleRolloutHost).
// Each step's forward and sampling are split by rows over threads when the
// batch is large (threads_for on the forward's multiply-adds); the
// environment step stays on the calling thread.
template <int W>
TB_INLINE Status rollout_loop(const Mlp& a, const Mlp& c, const float* p, const RolloutArgs& r) {
  const int64_t O = a.dims[0], N = r.N;
  const int P0 = threads_for(N, macs_per_row(a, c) / 3);
  const int64_t per = (N + P0 - 1) / P0;
  const int P = static_cast<int>((N + per - 1) / per);
  std::vector<Workspace> ws(P);
  for (auto& w : ws) w.size_for(a, c, per);
  Buf last(static_cast<size_t>(N * O));  // the observations after the last step (values only)
  void (*const fn)(RolloutChunk*) = W == 16 ? rchunk_avx512 : (W == 8 ? rchunk_avx2 : rchunk_base);
  const float* state = r.env->StateTensor().data_ptr<float>();
  const uint32_t ctr_lo = static_cast<uint32_t>(r.counter), ctr_hi = static_cast<uint32_t>(r.counter >> 32);
  std::vector<RolloutChunk> ch(P);
  for (int64_t t = 0; t <= r.T; ++t) {
    float* ob = t < r.T ? r.obs + t * N * O : last.data();
    std::memcpy(ob, state, sizeof(float) * N * O);
    int* act = r.act + t * N;
    for (int k = 0; k < P; ++k) {
      const int64_t r0 = k * per;
      ws[k].B = std::min(N, r0 + per) - r0;
      ch[k] = RolloutChunk{&a, &c, p, ob, r0, &ws[k], act, r.logp + t * N, r.val + t * N, t == r.T, r.seed,
                           static_cast<uint32_t>(t), ctr_lo, ctr_hi};
    }
    run_chunks(fn, ch);
    if (t == r.T) break;
    TURBOL_RETURN_IF_ERROR(r.env->StepCartPoleHost(act, r.rew + t * N, r.done + t * N));
  }
  return Status::Ok();
}

#define TB_UPDATE_ARGS                                                                                              \
  const Mlp &a, const Mlp &c, float *p, float *g, float *m1, float *m2, int64_t n, int64_t *step, const float *obs, \
      int64_t obs_rows, const int64_t *perms, int64_t epochs, int64_t rows, int64_t minibatch, bool adam,            \
      const LossArgs &la, float lr, float b1, float b2, float eps, float wd, float *st
#define TB_UPDATE_PASS a, c, p, g, m1, m2, n, step, obs, obs_rows, perms, epochs, rows, minibatch, adam, la, lr, b1, b2, eps, wd, st
#define TB_ROLLOUT_ARGS const Mlp &a, const Mlp &c, const float *p, const RolloutArgs &r

// One entry point per instruction set, chosen at run time, not through an
// ifunc, which would run while the loader relocates the library (before a
// sanitizer runtime has started).

TB_AVX512 Status update_avx512(TB_UPDATE_ARGS) { return update_loop<16>(TB_UPDATE_PASS); }
TB_AVX2 Status update_avx2(TB_UPDATE_ARGS) { return update_loop<8>(TB_UPDATE_PASS); }
Status update_base(TB_UPDATE_ARGS) { return update_loop<4>(TB_UPDATE_PASS); }
TB_AVX512 Status rollout_avx512(TB_ROLLOUT_ARGS) { return rollout_loop<16>(a, c, p, r); }
TB_AVX2 Status rollout_avx2(TB_ROLLOUT_ARGS) { return rollout_loop<8>(a, c, p, r); }
Status rollout_base(TB_ROLLOUT_ARGS) { return rollout_loop<4>(a, c, p, r); }

struct Impl {
  Status (*update)(TB_UPDATE_ARGS);
  Status (*rollout)(TB_ROLLOUT_ARGS);
};

// The entry points for this CPU, chosen on first use: the widest instruction
// set it has, or a narrower one named by TURBOL_HOST_ISA (avx512, avx2, base).
const Impl& impl() {
  static const Impl fns = [] {
    __builtin_cpu_init();
    const char* want = std::getenv("TURBOL_HOST_ISA");
    const std::string w = want ? want : "";
    const bool avx512 =
        __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512vl") && __builtin_cpu_supports("fma");
    const bool avx2 = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
    if (avx512 && (w.empty() || w == "avx512")) return Impl{update_avx512, rollout_avx512};
    if (avx2 && w != "base") return Impl{update_avx2, rollout_avx2};
    return Impl{update_base, rollout_base};
  }();
  return fns;
}

Status check_inputs(const at::Tensor& flat, const at::Tensor& grad, const std::vector<int64_t>& dims_a,
                    const std::vector<int64_t>& dims_c, const at::Tensor& obs, const at::Tensor& act,
                    const at::Tensor& old_logp, const at::Tensor& adv, const at::Tensor& ret, const at::Tensor& stats) {
  if (dims_a.size() < 2 || dims_c.size() < 2 || dims_a.front() != dims_c.front() || dims_c.back() != 1)
    return Status::InvalidArgument("ppo minibatch: actor / critic widths");
  for (const auto* d : {&dims_a, &dims_c})
    for (int64_t w : *d)
      if (w <= 0) return Status::InvalidArgument("ppo minibatch: widths must be positive");
  int64_t need = 0;
  for (const auto* d : {&dims_a, &dims_c})
    for (size_t l = 0; l + 1 < d->size(); ++l) need += (*d)[l + 1] * ((*d)[l] + 1);
  if (flat.numel() < need || grad.numel() < need || flat.scalar_type() != at::kFloat ||
      grad.scalar_type() != at::kFloat || !flat.is_contiguous() || !grad.is_contiguous())
    return Status::InvalidArgument("ppo minibatch: flat parameters / gradient");
  if (stats.numel() < 6 || stats.scalar_type() != at::kFloat || !stats.is_contiguous())
    return Status::InvalidArgument("ppo minibatch: stats must be fp32 [6]");
  if (obs.scalar_type() != at::kFloat || !obs.is_contiguous() || obs.dim() != 2 || obs.size(1) != dims_a.front())
    return Status::InvalidArgument("ppo minibatch: observations must be contiguous fp32 [rows, obs_dim]");
  if (act.scalar_type() != at::kInt || old_logp.scalar_type() != at::kFloat || adv.scalar_type() != at::kFloat ||
      ret.scalar_type() != at::kFloat || !act.is_contiguous() || !old_logp.is_contiguous() || !adv.is_contiguous() ||
      !ret.is_contiguous())
    return Status::InvalidArgument("ppo minibatch: int32 actions, fp32 log-probs / advantages / returns");
  if (old_logp.numel() < act.numel() || adv.numel() < act.numel() || ret.numel() < act.numel())
    return Status::InvalidArgument("ppo minibatch: log-probs / advantages / returns shorter than the actions");
  return Status::Ok();
}

LossArgs loss_args(const at::Tensor& act, const at::Tensor& old_logp, const at::Tensor& adv, const at::Tensor& ret,
                   float clip, float vf_coef, float ent_coef) {
  return LossArgs{act.data_ptr<int>(), old_logp.data_ptr<float>(), adv.data_ptr<float>(), ret.data_ptr<float>(),
                  act.numel(), clip, vf_coef, ent_coef};
}

}  // namespace

Status PpoCategoricalMinibatchHost(const at::Tensor& flat, const at::Tensor& grad, const std::vector<int64_t>& dims_a,
                                   const std::vector<int64_t>& dims_c, const at::Tensor& obs, const at::Tensor& act,
                                   const at::Tensor& old_logp, const at::Tensor& adv, const at::Tensor& ret,
                                   const at::Tensor& idx, float clip, float vf_coef, float ent_coef,
                                   const at::Tensor& stats) {
  TURBOL_RETURN_IF_ERROR(check_inputs(flat, grad, dims_a, dims_c, obs, act, old_logp, adv, ret, stats));
  if (idx.scalar_type() != at::kLong || !idx.is_contiguous() || idx.dim() != 1 || idx.numel() == 0)
    return Status::InvalidArgument("ppo minibatch: rows must be a non-empty contiguous int64 vector");
  int64_t off = 0;
  const Mlp a = mlp_layout(dims_a, &off);
  const Mlp c = mlp_layout(dims_c, &off);
  int64_t step = 0;
  const int64_t B = idx.numel();
  return impl().update(a, c, flat.data_ptr<float>(), grad.data_ptr<float>(), nullptr, nullptr, flat.numel(), &step,
                       obs.data_ptr<float>(), obs.size(0), idx.data_ptr<int64_t>(), 1, B, B, false,
                       loss_args(act, old_logp, adv, ret, clip, vf_coef, ent_coef), 0.f, 0.f, 0.f, 0.f, 0.f,
                       stats.data_ptr<float>());
}

int64_t PpoCategoricalUpdateHost(const at::Tensor& flat, const at::Tensor& grad, const at::Tensor& m,
                                  const at::Tensor& v, int64_t step, const std::vector<int64_t>& dims_a,
                                  const std::vector<int64_t>& dims_c, const at::Tensor& obs, const at::Tensor& act,
                                  const at::Tensor& old_logp, const at::Tensor& adv, const at::Tensor& ret,
                                  const at::Tensor& perms, int64_t minibatch, float clip, float vf_coef,
                                  float ent_coef, float lr, float b1, float b2, float eps, float wd,
                                  const at::Tensor& stats, Status* st) {
  *st = check_inputs(flat, grad, dims_a, dims_c, obs, act, old_logp, adv, ret, stats);
  if (!st->ok()) return step;
  if (perms.dim() != 2 || perms.scalar_type() != at::kLong || !perms.is_contiguous() || minibatch <= 0 ||
      minibatch > perms.size(1) || m.numel() != flat.numel() || v.numel() != flat.numel() ||
      m.scalar_type() != at::kFloat || v.scalar_type() != at::kFloat || !m.is_contiguous() || !v.is_contiguous()) {
    *st = Status::InvalidArgument("ppo update: perms [epochs, rows] int64, moments like the parameters");
    return step;
  }
  int64_t off = 0;
  const Mlp a = mlp_layout(dims_a, &off);
  const Mlp c = mlp_layout(dims_c, &off);
  *st = impl().update(a, c, flat.data_ptr<float>(), grad.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                      flat.numel(), &step, obs.data_ptr<float>(), obs.size(0), perms.data_ptr<int64_t>(),
                      perms.size(0), perms.size(1), minibatch, true,
                      loss_args(act, old_logp, adv, ret, clip, vf_coef, ent_coef), lr, b1, b2, eps, wd,
                      stats.data_ptr<float>());
  return step;
}

Status PpoCartPoleRolloutHost(GPUEnvironment* env, const at::Tensor& flat, const std::vector<int64_t>& dims_a,
                              const std::vector<int64_t>& dims_c, const at::Tensor& obs_buf, const at::Tensor& act_buf,
                              const at::Tensor& logp_buf, const at::Tensor& val_buf, const at::Tensor& rew_buf,
                              const at::Tensor& done_buf, uint64_t seed, uint64_t counter) {
  if (!env || env->type() != EnvType::kCartPole || env->device().is_cuda())
    return Status::InvalidArgument("ppo rollout: a CPU CartPole environment");
  if (dims_a.size() < 2 || dims_c.size() < 2 || dims_a.front() != 4 || dims_c.front() != 4 || dims_a.back() != 2 ||
      dims_c.back() != 1)
    return Status::InvalidArgument("ppo rollout: actor 4 -> ... -> 2, critic 4 -> ... -> 1");
  int64_t need = 0;
  for (const auto* d : {&dims_a, &dims_c})
    for (size_t l = 0; l + 1 < d->size(); ++l) {
      if ((*d)[l + 1] <= 0) return Status::InvalidArgument("ppo rollout: widths must be positive");
      need += (*d)[l + 1] * ((*d)[l] + 1);
    }
  if (flat.numel() < need || flat.scalar_type() != at::kFloat || !flat.is_contiguous() || flat.is_cuda())
    return Status::InvalidArgument("ppo rollout: flat parameters");
  const int64_t N = env->NumEnvs();
  if (obs_buf.dim() != 3 || obs_buf.size(1) != N || obs_buf.size(2) != 4)
    return Status::InvalidArgument("ppo rollout: obs_buf must be [T, num_envs, 4]");
  const int64_t T = obs_buf.size(0);
  for (const at::Tensor* b : {&obs_buf, &act_buf, &logp_buf, &val_buf, &rew_buf, &done_buf})
    if (!b->is_contiguous() || b->is_cuda()) return Status::InvalidArgument("ppo rollout: contiguous CPU buffers");
  if (obs_buf.scalar_type() != at::kFloat || logp_buf.scalar_type() != at::kFloat ||
      val_buf.scalar_type() != at::kFloat || rew_buf.scalar_type() != at::kFloat ||
      act_buf.scalar_type() != at::kInt || done_buf.element_size() != 1)
    return Status::InvalidArgument("ppo rollout: fp32 obs / log-prob / value / reward, int32 actions, byte dones");
  if (act_buf.numel() != T * N || logp_buf.numel() != T * N || rew_buf.numel() != T * N ||
      done_buf.numel() != T * N || val_buf.numel() != (T + 1) * N)
    return Status::InvalidArgument("ppo rollout: buffers [T, N] (values [T + 1, N])");
  int64_t off = 0;
  const Mlp a = mlp_layout(dims_a, &off);
  const Mlp c = mlp_layout(dims_c, &off);
  const RolloutArgs r{env, obs_buf.data_ptr<float>(), logp_buf.data_ptr<float>(), val_buf.data_ptr<float>(),
                      rew_buf.data_ptr<float>(), act_buf.data_ptr<int>(), static_cast<uint8_t*>(done_buf.data_ptr()),
                      T, N, seed, counter};
  return impl().rollout(a, c, flat.data_ptr<float>(), r);
}

}  // namespace turbol
