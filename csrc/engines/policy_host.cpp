// Host (CPU) versions of the linear Gaussian policy's fused steps, of the
// Adam update and of GAE: the same math as csrc/kernels/policy.cu, optim.cu
// and advantage.cu, one pass in plain loops, so the CPU paths pay no
// per-operator framework dispatch.
//
//   mean = tanh(W_a x + b_a) [A],   value = W_c x + b_c
//   parameter layout (flat fp32): W_a [A, O], b_a [A], W_c [O], b_c
#include <math.h>

#include <ATen/Parallel.h>

#include <algorithm>
#include <cmath>
#include <system_error>
#include <thread>
#include <vector>

#include "turbol/engines.hpp"

namespace turbol {

namespace {

constexpr float kPi = 3.14159265358979323846f;

void philox4(uint64_t seed, uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t* out) {
  uint32_t c[4] = {c0, c1, c2, c3};
  uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = static_cast<uint64_t>(0xD2511F53u) * c[0];
    const uint64_t p1 = static_cast<uint64_t>(0xCD9E8D57u) * c[2];
    const uint32_t n0 = static_cast<uint32_t>(p1 >> 32) ^ c[1] ^ k0;
    const uint32_t n2 = static_cast<uint32_t>(p0 >> 32) ^ c[3] ^ k1;
    c[1] = static_cast<uint32_t>(p1);
    c[3] = static_cast<uint32_t>(p0);
    c[0] = n0;
    c[2] = n2;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  for (int i = 0; i < 4; ++i) out[i] = c[i];
}

// tanh through one exp: tanh(z) = sign(z) (1 - e^{-2|z|}) / (1 + e^{-2|z|}) (no overflow for large |z|)
inline float tanh_exp(float z) {
  const float e = std::exp(-2.f * std::fabs(z));
  return std::copysign((1.f - e) / (1.f + e), z);
}

float u01(uint32_t x) { return static_cast<float>(x >> 8) * (1.0f / 16777216.0f); }
float u01_open(uint32_t x) { return (static_cast<float>(x >> 8) + 0.5f) * (1.0f / 16777216.0f); }

Status check_dims(int N, int O, int A) {
  if (N < 0 || O <= 0 || A <= 0) return Status::InvalidArgument("linear Gaussian policy: bad dimensions");
  return Status::Ok();
}

}  // namespace

Status LinGaussActHost(const float* x, const float* p, float* act, float* logp, int N, int O, int A, float stdv,
                       uint64_t seed, uint32_t counter) {
  TURBOL_RETURN_IF_ERROR(check_dims(N, O, A));
  const float var = stdv * stdv, c = -0.5f * std::log(2.f * kPi * var);
  const float* W = p;
  const float* b = p + static_cast<size_t>(A) * O;
  for (int64_t row = 0; row < N; ++row) {
    const float* xr = x + static_cast<size_t>(row) * O;
    float* ar = act + static_cast<size_t>(row) * A;
    float lp = 0.f;
    for (int j0 = 0; j0 < A; j0 += 2) {
      // two standard normals (Box-Muller) from the Philox block of (row, j0, call)
      uint32_t r[4];
      philox4(seed, static_cast<uint32_t>(row), static_cast<uint32_t>(j0), counter, 0u, r);
      const float rad = std::sqrt(-2.f * std::log(u01_open(r[0])));
      float sn, cs;
      sincosf(2.f * kPi * u01(r[1]), &sn, &cs);
      const float nz[2] = {rad * cs, rad * sn};
      for (int t = 0; t < 2 && j0 + t < A; ++t) {
        const int j = j0 + t;
        float z = b[j];
        const float* wj = W + static_cast<size_t>(j) * O;
        for (int k = 0; k < O; ++k) z += wj[k] * xr[k];
        const float m = tanh_exp(z);
        const float a = std::min(1.f, std::max(-1.f, m + stdv * nz[t]));
        ar[j] = a;
        lp += -0.5f * (a - m) * (a - m) / var + c;
      }
    }
    logp[row] = lp;
  }
  return Status::Ok();
}

Status LinGaussGradHost(const float* batch, int row_w, const float* p, float* g, int N, int O, int A, float stdv,
                        float clip, float vf_coef, bool has_old) {
  TURBOL_RETURN_IF_ERROR(check_dims(N, O, A));
  if (row_w < O + A + 2 + (has_old ? 1 : 0)) return Status::InvalidArgument("linear Gaussian policy: row too narrow");
  if (N == 0) return Status::Ok();
  const float var = stdv * stdv, c = -0.5f * std::log(2.f * kPi * var);
  const float inv_n = 1.f / static_cast<float>(N);
  const float* Wa = p;
  const float* ba = Wa + static_cast<size_t>(A) * O;
  const float* Wc = ba + A;
  const float bc = Wc[O];
  float* gWa = g;
  float* gba = gWa + static_cast<size_t>(A) * O;
  float* gWc = gba + A;
  float* gbc = gWc + O;
  std::vector<float> m(A);
  for (int row = 0; row < N; ++row) {
    const float* r = batch + static_cast<size_t>(row) * row_w;
    const float* xr = r;
    const float* a = r + O;
    const float adv = r[O + A], ret = r[O + A + 1];
    float lp = 0.f;
    for (int j = 0; j < A; ++j) {
      float z = ba[j];
      const float* wj = Wa + static_cast<size_t>(j) * O;
      for (int k = 0; k < O; ++k) z += wj[k] * xr[k];
      m[j] = std::tanh(z);
      lp += -0.5f * (a[j] - m[j]) * (a[j] - m[j]) / var + c;
    }
    const float old = has_old ? r[O + A + 2] : lp;
    const float ratio = std::exp(lp - old);
    const float unc = ratio * adv, clp = std::min(std::max(ratio, 1.f - clip), 1.f + clip) * adv;
    // d(-min(unclipped, clipped)) / d logp: nonzero where the unclipped term is the minimum or the ratio is inside
    const float g_lp = (unc <= clp || (ratio > 1.f - clip && ratio < 1.f + clip)) ? -unc * inv_n : 0.f;
    for (int j = 0; j < A; ++j) {
      const float gz = g_lp * (a[j] - m[j]) / var * (1.f - m[j] * m[j]);
      float* gj = gWa + static_cast<size_t>(j) * O;
      for (int k = 0; k < O; ++k) gj[k] += gz * xr[k];
      gba[j] += gz;
    }
    // value head: vf * mean((v - ret)^2)
    float v = bc;
    for (int k = 0; k < O; ++k) v += Wc[k] * xr[k];
    const float gv = vf_coef * 2.f * (v - ret) * inv_n;
    for (int k = 0; k < O; ++k) gWc[k] += gv * xr[k];
    *gbc += gv;
  }
  return Status::Ok();
}

namespace {

// One Adam pass; inlined into the per-instruction-set entry points below.
// Distinct arrays (restrict), the bias corrections as multiplications, IEEE
// square root and divide; the host core is built without math errno, so the
// square root vectorizes (0.23 G elements/s with errno, 1.2-1.7 G without).
static inline __attribute__((always_inline)) void adam_body(float* __restrict__ p, const float* __restrict__ g,
                                                            float* __restrict__ m, float* __restrict__ v, int64_t n,
                                                            float lr, float b1, float b2, float eps, float wd,
                                                            float grad_scale, float ibc1, float ibc2) {
  for (int64_t i = 0; i < n; ++i) {
    const float gi = g[i] * grad_scale;
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    p[i] -= lr * ((mi * ibc1) / (__builtin_sqrtf(vi * ibc2) + eps) + wd * p[i]);
  }
}

#define TB_ADAM_ARGS                                                                                               \
  float *__restrict__ p, const float *__restrict__ g, float *__restrict__ m, float *__restrict__ v, int64_t n, \
      float lr, float b1, float b2, float eps, float wd, float grad_scale, float ibc1, float ibc2
#define TB_ADAM_PASS p, g, m, v, n, lr, b1, b2, eps, wd, grad_scale, ibc1, ibc2

// Chosen at run time rather than through an ifunc (target_clones): an ifunc
// resolver runs while the loader relocates the library, before a sanitizer
// runtime has started.
__attribute__((target("avx512f,avx512vl,avx2,fma"))) void adam_avx512(TB_ADAM_ARGS) { adam_body(TB_ADAM_PASS); }
__attribute__((target("avx2,fma"))) void adam_avx2(TB_ADAM_ARGS) { adam_body(TB_ADAM_PASS); }
void adam_base(TB_ADAM_ARGS) { adam_body(TB_ADAM_PASS); }

using AdamFn = void (*)(TB_ADAM_ARGS);

AdamFn adam_fn() {
  static const AdamFn fn = [] {
    __builtin_cpu_init();
    if (__builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512vl")) return adam_avx512;
    if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) return adam_avx2;
    return adam_base;
  }();
  return fn;
}

}  // namespace

void AdamHost(float* p, const float* g, float* m, float* v, int64_t n, int64_t step, float lr, float b1, float b2,
              float eps, float wd, float grad_scale) {
  const float ibc1 = 1.f / (1.f - std::pow(b1, static_cast<float>(step)));
  const float ibc2 = 1.f / (1.f - std::pow(b2, static_cast<float>(step)));
  adam_fn()(p, g, m, v, n, lr, b1, b2, eps, wd, grad_scale, ibc1, ibc2);
}

namespace {

// The backward sweep over environments [n0, n1) (vectorizable over them);
// adds the sum and sum of squares of their advantages into s[0], s[1].
void gae_columns(const float* rewards, const float* values, const uint8_t* dones, float* adv, float* ret, int T,
                 int N, int n0, int n1, float gamma, float gl, bool want_stats, double* s) {
  std::vector<float> last(static_cast<size_t>(n1 - n0), 0.f);
  double s1 = 0.0, s2 = 0.0;
  for (int t = T - 1; t >= 0; --t) {
    const size_t o = static_cast<size_t>(t) * N + n0;
    const float* r = rewards + o;
    const float* v0 = values + o;
    const float* v1 = v0 + N;
    const uint8_t* d = dones + o;
    float* a = adv + o;
    float* rt = ret + o;
    for (int n = 0; n < n1 - n0; ++n) {
      const float nd = d[n] ? 0.f : 1.f;
      const float delta = r[n] + gamma * nd * v1[n] - v0[n];
      const float l = delta + gl * nd * last[n];
      last[n] = l;
      a[n] = l;
      rt[n] = l + v0[n];
    }
    if (want_stats)
      for (int n = 0; n < n1 - n0; ++n) {
        s1 += a[n];
        s2 += static_cast<double>(a[n]) * a[n];
      }
  }
  s[0] += s1;
  s[1] += s2;
}

}  // namespace

// Environments are independent columns of the sweep: a large [T, N] is split
// by column blocks (multiples of 64) over torch's intra-op threads, at least
// 1 M elements each; a block whose thread cannot be started runs on the
// calling thread.  The statistics add up block by block in block order.
Status GaeHost(const float* rewards, const float* values, const uint8_t* dones, float* adv, float* ret, int T, int N,
               float gamma, float lam, double* stats) {
  if (T < 0 || N < 0) return Status::InvalidArgument("gae: bad dimensions");
  const float gl = static_cast<float>(static_cast<double>(gamma) * lam);
  const int64_t work = static_cast<int64_t>(T) * N;
  const int P = static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>({static_cast<int64_t>(at::get_num_threads()), work >> 20, N / 64})));
  const int per = P == 1 ? N : (N / P + 63) / 64 * 64;
  const int blocks = P == 1 ? 1 : (N + per - 1) / per;
  std::vector<double> s(2 * static_cast<size_t>(blocks), 0.0);
  auto run = [&](int k) {
    const int n0 = k * per, n1 = std::min(N, n0 + per);
    gae_columns(rewards, values, dones, adv, ret, T, N, n0, n1, gamma, gl, stats != nullptr, &s[2 * k]);
  };
  std::vector<std::thread> th;
  th.reserve(blocks);
  int started = 1;
  try {
    for (; started < blocks; ++started) th.emplace_back(run, started);
  } catch (const std::system_error&) {
    // the rest run below
  }
  run(0);
  for (int k = started; k < blocks; ++k) run(k);
  for (auto& x : th) x.join();
  if (stats)
    for (int k = 0; k < blocks; ++k) {
      stats[0] += s[2 * k];
      stats[1] += s[2 * k + 1];
    }
  return Status::Ok();
}

}  // namespace turbol
