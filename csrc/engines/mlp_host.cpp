// One PPO minibatch step of the CPU trainer without autograd: the forward of
// the actor and critic MLPs (tanh hidden layers), the clipped-surrogate PPO
// loss for a categorical actor with the value and entropy terms, and the
// hand-written backward into the flat gradient.  The matrix products go
// through ATen (MKL); the loss and its gradient are one loop over the rows.
// For minibatches of tens of rows the autograd graph and the per-operator
// dispatch of the Python path cost several times the arithmetic.
#include <ATen/ATen.h>
#include <c10/core/InferenceMode.h>

#include <algorithm>
#include <cmath>
#include <vector>

#include "turbol/engines.hpp"

namespace turbol {

namespace {

struct Net {
  std::vector<at::Tensor> W, b, gW, gb;  // per layer: weight [out, in], bias [out] and their gradient views
};

// Views of one MLP (widths dims[0] -> ... -> dims[L]) at *off of the flat buffers.
Net net_views(const at::Tensor& flat, const at::Tensor& grad, const std::vector<int64_t>& dims, int64_t* off) {
  Net n;
  for (size_t l = 0; l + 1 < dims.size(); ++l) {
    const int64_t in = dims[l], out = dims[l + 1];
    n.W.push_back(flat.narrow(0, *off, out * in).view({out, in}));
    n.gW.push_back(grad.narrow(0, *off, out * in).view({out, in}));
    *off += out * in;
    n.b.push_back(flat.narrow(0, *off, out));
    n.gb.push_back(grad.narrow(0, *off, out));
    *off += out;
  }
  return n;
}

// Forward; acts[l] is the input of layer l (acts[0] = x), tanh after every layer but the last.
at::Tensor forward(const Net& n, const at::Tensor& x, std::vector<at::Tensor>* acts) {
  at::Tensor h = x;
  const size_t L = n.W.size();
  for (size_t l = 0; l < L; ++l) {
    acts->push_back(h);
    h = at::addmm(n.b[l], h, n.W[l].t());
    if (l + 1 < L) h.tanh_();
  }
  return h;
}

// Backward from d(output) (contiguous [B, out]); weight gradients are added
// by the matrix product, bias gradients and the tanh derivative in plain loops.
void backward(const Net& n, const std::vector<at::Tensor>& acts, at::Tensor d) {
  for (size_t l = n.W.size(); l-- > 0;) {
    const int64_t B = d.size(0), out = d.size(1);
    n.gW[l].addmm_(d.t(), acts[l]);
    const float* dp = d.data_ptr<float>();
    float* gb = n.gb[l].data_ptr<float>();
    for (int64_t i = 0; i < B; ++i)
      for (int64_t j = 0; j < out; ++j) gb[j] += dp[i * out + j];
    if (l == 0) break;
    const at::Tensor& h = acts[l];  // tanh output of layer l - 1, contiguous [B, in]
    d = at::mm(d, n.W[l]);
    float* q = d.data_ptr<float>();
    const float* hp = h.data_ptr<float>();
    const int64_t cnt = d.numel();
    for (int64_t e = 0; e < cnt; ++e) q[e] *= 1.f - hp[e] * hp[e];
  }
}

}  // namespace

Status PpoCategoricalMinibatchHost(const at::Tensor& flat, const at::Tensor& grad, const std::vector<int64_t>& dims_a,
                                   const std::vector<int64_t>& dims_c, const at::Tensor& obs, const at::Tensor& act,
                                   const at::Tensor& old_logp, const at::Tensor& adv, const at::Tensor& ret,
                                   const at::Tensor& idx, float clip, float vf_coef, float ent_coef,
                                   const at::Tensor& stats) {
  if (dims_a.size() < 2 || dims_c.size() < 2 || dims_a.front() != dims_c.front() || dims_c.back() != 1)
    return Status::InvalidArgument("ppo minibatch: actor / critic widths");
  int64_t need = 0;
  for (const auto* d : {&dims_a, &dims_c})
    for (size_t l = 0; l + 1 < d->size(); ++l) need += (*d)[l + 1] * ((*d)[l] + 1);
  if (flat.numel() < need || grad.numel() < need || flat.scalar_type() != at::kFloat ||
      grad.scalar_type() != at::kFloat || !flat.is_contiguous() || !grad.is_contiguous())
    return Status::InvalidArgument("ppo minibatch: flat parameters / gradient");
  if (stats.numel() < 6 || stats.scalar_type() != at::kFloat)
    return Status::InvalidArgument("ppo minibatch: stats must be fp32 [6]");
  c10::InferenceMode no_grad;
  int64_t off = 0;
  const Net an = net_views(flat, grad, dims_a, &off);
  const Net cn = net_views(flat, grad, dims_c, &off);
  const at::Tensor x = obs.index_select(0, idx).contiguous();
  std::vector<at::Tensor> aa, ca;
  const at::Tensor logits = forward(an, x, &aa).contiguous();
  const at::Tensor value = forward(cn, x, &ca).contiguous();
  const int64_t B = x.size(0), A = dims_a.back();
  if (act.scalar_type() != at::kInt || old_logp.scalar_type() != at::kFloat || adv.scalar_type() != at::kFloat ||
      ret.scalar_type() != at::kFloat || !act.is_contiguous() || !old_logp.is_contiguous() || !adv.is_contiguous() ||
      !ret.is_contiguous() || idx.scalar_type() != at::kLong || !idx.is_contiguous())
    return Status::InvalidArgument("ppo minibatch: int32 actions, fp32 log-probs / advantages / returns, int64 rows");
  at::Tensor dlogits = at::empty({B, A}, logits.options());
  at::Tensor dvalue = at::empty({B, 1}, logits.options());
  const float* L = logits.data_ptr<float>();
  const float* V = value.data_ptr<float>();
  const int64_t* rows = idx.data_ptr<int64_t>();
  const int64_t n_all = act.numel();
  const int* act_all = act.data_ptr<int>();
  const float* olp_all = old_logp.data_ptr<float>();
  const float* adv_all = adv.data_ptr<float>();
  const float* ret_all = ret.data_ptr<float>();
  float* dL = dlogits.data_ptr<float>();
  float* dV = dvalue.data_ptr<float>();
  const float inv_b = 1.f / static_cast<float>(B);
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
    const int64_t row = rows[i];
    if (row < 0 || row >= n_all) return Status::InvalidArgument("ppo minibatch: row index out of range");
    const int a = act_all[row];
    if (a < 0 || a >= A) return Status::InvalidArgument("ppo minibatch: action out of range");
    const float adv_i = adv_all[row];
    const float logp = lsm[a], d = logp - olp_all[row], ratio = std::exp(d);
    const float unc = ratio * adv_i, clp = std::min(std::max(ratio, 1.f - clip), 1.f + clip) * adv_i;
    const float pg = -std::min(unc, clp);
    // d pg / d logp = -ratio * adv where the unclipped term is the minimum (or the ratio is inside the clip range)
    const float g_lp = (unc <= clp || (ratio > 1.f - clip && ratio < 1.f + clip)) ? -unc * inv_b : 0.f;
    // d(-ent_coef * mean(ent)) / d logits_j = ent_coef / B * p_j (log p_j + ent)
    for (int64_t j = 0; j < A; ++j)
      dL[i * A + j] = g_lp * ((j == a ? 1.f : 0.f) - pr[j]) + ent_coef * inv_b * pr[j] * (lsm[j] + ent);
    const float dv = V[i] - ret_all[row];
    dV[i] = vf_coef * dv * inv_b;
    s_pg += pg;
    s_v += 0.5f * dv * dv;
    s_ent += ent;
    s_kl += (ratio - 1.f) - d;
    s_clip += std::fabs(ratio - 1.f) > clip ? 1.0 : 0.0;
  }
  backward(an, aa, dlogits);
  backward(cn, ca, dvalue);
  float* st = stats.data_ptr<float>();
  st[0] += static_cast<float>(s_pg);
  st[1] += static_cast<float>(s_v);
  st[2] += static_cast<float>(s_ent);
  st[3] += static_cast<float>(s_kl);
  st[4] += static_cast<float>(s_clip);
  st[5] += static_cast<float>(B);
  return Status::Ok();
}

int64_t PpoCategoricalUpdateHost(const at::Tensor& flat, const at::Tensor& grad, const at::Tensor& m,
                                  const at::Tensor& v, int64_t step, const std::vector<int64_t>& dims_a,
                                  const std::vector<int64_t>& dims_c, const at::Tensor& obs, const at::Tensor& act,
                                  const at::Tensor& old_logp, const at::Tensor& adv, const at::Tensor& ret,
                                  const at::Tensor& perms, int64_t minibatch, float clip, float vf_coef,
                                  float ent_coef, float lr, float b1, float b2, float eps, float wd,
                                  const at::Tensor& stats, Status* st) {
  *st = Status::Ok();
  if (perms.dim() != 2 || perms.scalar_type() != at::kLong || !perms.is_contiguous() || minibatch <= 0 ||
      m.numel() != flat.numel() || v.numel() != flat.numel() || m.scalar_type() != at::kFloat ||
      v.scalar_type() != at::kFloat || !m.is_contiguous() || !v.is_contiguous()) {
    *st = Status::InvalidArgument("ppo update: perms [epochs, rows] int64, moments like the parameters");
    return step;
  }
  const int64_t rows = perms.size(1), n_mb = rows / minibatch;
  float* g = grad.data_ptr<float>();
  const int64_t n = flat.numel();
  for (int64_t e = 0; e < perms.size(0); ++e) {
    const at::Tensor pe = perms[e];
    for (int64_t k = 0; k < n_mb; ++k) {
      std::fill(g, g + n, 0.f);
      *st = PpoCategoricalMinibatchHost(flat, grad, dims_a, dims_c, obs, act, old_logp, adv, ret,
                                        pe.narrow(0, k * minibatch, minibatch), clip, vf_coef, ent_coef, stats);
      if (!st->ok()) return step;
      AdamHost(flat.data_ptr<float>(), g, m.data_ptr<float>(), v.data_ptr<float>(), n, ++step, lr, b1, b2, eps, wd,
               1.f);
    }
  }
  return step;
}

}  // namespace turbol
