// RewardEngine: rule scores, hash reward, masked KL, adaptive KL coefficient,
// batch normalization and Welford running statistics.  String scoring runs on
// the host (the strings live there); token scoring and KL run as kernels when
// the tensors are on the GPU.
#include <ATen/ATen.h>

#include <algorithm>
#include <cmath>

#include "turbol/engines.hpp"

namespace turbol {

Status RewardEngine::Initialize() {
  initialized_ = true;
  mean_ = 0.0;
  m2_ = 0.0;
  count_ = 0;
  return Status::Ok();
}

Status RewardEngine::Normalize(at::Tensor& r) {
  if (r.numel() == 0) return Status::Ok();
  if (r.is_cuda())
    return FromCuda(tb_normalize_rewards(r.data_ptr<float>(), static_cast<int>(r.numel()), cfg_.whiten ? 1 : 0,
                                         1e-8f, StreamFor(r)),
                    "normalize_rewards");
  const double mean = r.mean().item<double>();
  r.sub_(mean);
  if (cfg_.whiten) {
    const double sd = std::sqrt(r.pow(2).mean().item<double>());
    r.div_(sd + 1e-8);
  }
  return Status::Ok();
}

Status RewardEngine::ScoreBatch(const std::vector<std::string>& responses, const std::optional<Tensor>& ref_logprobs,
                                RewardResult* out) {
  (void)ref_logprobs;
  if (!initialized_) return Status::InvalidArgument("RewardEngine not initialized");
  if (!out) return Status::InvalidArgument("result pointer is null");
  const int64_t B = static_cast<int64_t>(responses.size());
  at::Tensor rule = at::empty({B}, at::kFloat);
  for (int64_t i = 0; i < B; ++i) {
    const std::string& s = responses[i];
    float v = 0.f;
    if (!s.empty() && s.back() == '.') v += cfg_.format_bonus;
    const float d = static_cast<float>(static_cast<long long>(s.size()) - cfg_.target_length);
    v += cfg_.length_penalty * d * d;
    rule.data_ptr<float>()[i] = v;
  }
  at::Tensor total = rule.clamp(-cfg_.reward_clip, cfg_.reward_clip);
  const at::Device dev = cfg_.device.torch();
  rule = rule.to(dev);
  total = total.to(dev).contiguous();
  if (cfg_.normalize) TURBOL_RETURN_IF_ERROR(Normalize(total));
  out->rule_scores = Tensor(rule);
  out->total = Tensor(total);
  out->model_scores = Tensor(at::zeros({B}, at::TensorOptions().dtype(at::kFloat).device(dev)));
  out->kl_penalties = Tensor(at::zeros({B}, at::TensorOptions().dtype(at::kFloat).device(dev)));
  return Status::Ok();
}

Status RewardEngine::ScoreTokens(const Tensor& token_ids, const Tensor& masks, const std::optional<Tensor>& logprobs,
                                 const std::optional<Tensor>& ref_logprobs, RewardResult* out) {
  if (!initialized_) return Status::InvalidArgument("RewardEngine not initialized");
  if (!out) return Status::InvalidArgument("result pointer is null");
  if (token_ids.shape().size() != 2) return Status::InvalidArgument("token_ids must be [B, T]");
  const int B = static_cast<int>(token_ids.shape()[0]), T = static_cast<int>(token_ids.shape()[1]);
  const at::Device dev = token_ids.torch().device();
  auto f32 = at::TensorOptions().dtype(at::kFloat).device(dev);
  at::Tensor ids = token_ids.torch().to(at::kInt).contiguous();
  at::Tensor mask = masks.defined() ? masks.torch().to(f32).contiguous() : at::ones({B, T}, f32);
  at::Tensor lens = (mask > 0.5f).sum(1).to(at::kInt).contiguous();
  at::Tensor rule = at::empty({B}, f32), total = at::empty({B}, f32);
  if (dev.is_cuda()) {
    TURBOL_RETURN_IF_ERROR(FromCuda(
        tb_rule_reward(ids.data_ptr<int>(), lens.data_ptr<int>(), B, T, cfg_.period_token_id, cfg_.format_bonus,
                       cfg_.length_penalty, cfg_.target_length, cfg_.reward_clip, rule.data_ptr<float>(),
                       total.data_ptr<float>(), StreamFor(ids)),
        "rule_reward"));
  } else {
    for (int i = 0; i < B; ++i) {
      const int L = std::min(lens.data_ptr<int>()[i], T);
      float s = 0.f;
      if (L > 0 && ids.data_ptr<int>()[static_cast<size_t>(i) * T + L - 1] == cfg_.period_token_id)
        s += cfg_.format_bonus;
      const float d = static_cast<float>(L - cfg_.target_length);
      s += cfg_.length_penalty * d * d;
      rule.data_ptr<float>()[i] = s;
      total.data_ptr<float>()[i] = std::max(-cfg_.reward_clip, std::min(cfg_.reward_clip, s));
    }
  }
  at::Tensor kl = at::zeros({B}, f32);
  if (logprobs.has_value() && ref_logprobs.has_value()) {
    TURBOL_RETURN_IF_ERROR(ComputeKLPenalty(logprobs->torch(), ref_logprobs->torch(), mask, &kl));
    total.sub_(kl);
  }
  if (cfg_.normalize) TURBOL_RETURN_IF_ERROR(Normalize(total));
  out->rule_scores = Tensor(rule);
  out->total = Tensor(total);
  out->model_scores = Tensor(at::zeros({B}, f32));
  out->kl_penalties = Tensor(kl);
  return Status::Ok();
}

Status RewardEngine::HashReward(const at::Tensor& token_ids, const at::Tensor& lengths, at::Tensor* out) {
  if (token_ids.dim() != 2) return Status::InvalidArgument("token_ids must be [B, T]");
  const int B = static_cast<int>(token_ids.size(0)), T = static_cast<int>(token_ids.size(1));
  at::Tensor ids = token_ids.to(at::kInt).contiguous();
  at::Tensor lens = lengths.defined() ? lengths.to(ids.options()).contiguous() : at::full({B}, T, ids.options());
  at::Tensor r = at::empty({B}, ids.options().dtype(at::kFloat));
  if (ids.is_cuda()) {
    TURBOL_RETURN_IF_ERROR(FromCuda(
        tb_hash_reward(ids.data_ptr<int>(), lens.data_ptr<int>(), B, T, r.data_ptr<float>(), StreamFor(ids)),
        "hash_reward"));
  } else {
    for (int i = 0; i < B; ++i) {
      uint64_t h = 0xcbf29ce484222325ull;
      const int L = std::min(lens.data_ptr<int>()[i], T);
      for (int t = 0; t < L; ++t) {
        uint32_t w = static_cast<uint32_t>(ids.data_ptr<int>()[static_cast<size_t>(i) * T + t]);
        for (int b = 0; b < 4; ++b) {
          h ^= (w & 0xffu);
          h *= 0x100000001b3ull;
          w >>= 8;
        }
      }
      r.data_ptr<float>()[i] = static_cast<float>(h % 1000ull) / 1000.0f;
    }
  }
  *out = r;
  return Status::Ok();
}

Status RewardEngine::ComputeKLPenalty(const at::Tensor& logprobs, const at::Tensor& ref_logprobs,
                                      const at::Tensor& masks, at::Tensor* out) {
  if (logprobs.dim() != 2 || ref_logprobs.sizes() != logprobs.sizes())
    return Status::InvalidArgument("logprobs/ref_logprobs must both be [B, T]");
  const int B = static_cast<int>(logprobs.size(0)), T = static_cast<int>(logprobs.size(1));
  at::Tensor lp = logprobs.to(at::kFloat).contiguous(), ref = ref_logprobs.to(lp.options()).contiguous();
  at::Tensor m = masks.defined() ? masks.to(lp.options()).contiguous() : at::ones_like(lp);
  at::Tensor kl = at::empty({B}, lp.options());
  if (lp.is_cuda()) {
    TURBOL_RETURN_IF_ERROR(FromCuda(tb_masked_kl(lp.data_ptr<float>(), ref.data_ptr<float>(), m.data_ptr<float>(), B,
                                                 T, kl_coef_, cfg_.k3_kl ? 1 : 0, kl.data_ptr<float>(), StreamFor(lp)),
                                    "masked_kl"));
  } else {
    at::Tensor d = lp - ref;
    at::Tensor est = cfg_.k3_kl ? (at::exp(-d) + d - 1.0) : d;
    at::Tensor valid = (m > 0.5f).to(at::kFloat);
    at::Tensor cnt = valid.sum(1);
    kl = at::where(cnt > 0, (est * valid).sum(1) / cnt.clamp_min(1.0) * kl_coef_, at::zeros_like(cnt));
  }
  *out = kl;
  return Status::Ok();
}

Status RewardEngine::UpdateAdaptiveKL(float observed_kl) {
  if (!cfg_.adaptive_kl) return Status::Ok();
  kl_coef_ = std::max(0.0f, kl_coef_ + cfg_.kl_adapt_rate * (observed_kl - cfg_.kl_target));
  return Status::Ok();
}

Status RewardEngine::UpdateStats(const Tensor& rewards) {
  at::Tensor r = rewards.torch().to(at::kCPU).to(at::kDouble).reshape({-1});
  const double* p = r.data_ptr<double>();
  for (int64_t i = 0; i < r.numel(); ++i) {
    ++count_;
    const double d = p[i] - mean_;
    mean_ += d / static_cast<double>(count_);
    m2_ += d * (p[i] - mean_);
  }
  return Status::Ok();
}

}  // namespace turbol
