// GPUEnvironment, RingBuffer and PrioritizedReplayBuffer.
#include <ATen/ATen.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <stdexcept>

#include "turbol/engines.hpp"

namespace turbol {

// Host Philox4x32-10 (same rounds/constants as the device generator in
// csrc/kernels/device_common.cuh); returns word `which` of the 4-word block.
uint64_t HostPhiloxWord(uint64_t seed, uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, int which) {
  uint32_t c[4] = {c0, c1, c2, c3};
  uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = static_cast<uint64_t>(0xD2511F53u) * c[0];
    const uint64_t p1 = static_cast<uint64_t>(0xCD9E8D57u) * c[2];
    const uint32_t hi0 = static_cast<uint32_t>(p0 >> 32), lo0 = static_cast<uint32_t>(p0);
    const uint32_t hi1 = static_cast<uint32_t>(p1 >> 32), lo1 = static_cast<uint32_t>(p1);
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n1 = lo1, n2 = hi0 ^ c[3] ^ k1, n3 = lo0;
    c[0] = n0;
    c[1] = n1;
    c[2] = n2;
    c[3] = n3;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c[which & 3];
}

namespace {

// Word 0 of Philox4x32-10 for counters (c0 + j, c1, c2, c3), j < 8, written as
// independent lanes so the compiler can vectorize the rounds (the same values
// as HostPhiloxWord(seed, c0 + j, c1, c2, c3, 0)).
void host_philox_word0_x8(uint64_t seed, uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t* out) {
  constexpr int L = 8;
  uint32_t x0[L], x1[L], x2[L], x3[L];
  for (int j = 0; j < L; ++j) {
    x0[j] = c0 + static_cast<uint32_t>(j);
    x1[j] = c1;
    x2[j] = c2;
    x3[j] = c3;
  }
  uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
  for (int r = 0; r < 10; ++r) {
    for (int j = 0; j < L; ++j) {
      const uint64_t p0 = static_cast<uint64_t>(0xD2511F53u) * x0[j];
      const uint64_t p1 = static_cast<uint64_t>(0xCD9E8D57u) * x2[j];
      const uint32_t n0 = static_cast<uint32_t>(p1 >> 32) ^ x1[j] ^ k0;
      const uint32_t n2 = static_cast<uint32_t>(p0 >> 32) ^ x3[j] ^ k1;
      x1[j] = static_cast<uint32_t>(p1);
      x3[j] = static_cast<uint32_t>(p0);
      x0[j] = n0;
      x2[j] = n2;
    }
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  for (int j = 0; j < L; ++j) out[j] = x0[j];
}

float host_u01(uint32_t x) { return static_cast<float>(x >> 8) * (1.0f / 16777216.0f); }

float ref_reset_unit(unsigned i, unsigned d, unsigned seed) {
  unsigned h = seed ^ (i * 73856093u) ^ (d * 19349663u);
  h ^= h >> 13;
  h *= 2654435761u;
  h ^= h >> 16;
  return static_cast<float>(h & 0xFFFFu) / 65535.0f;
}

void cartpole_initial(uint64_t seed, unsigned env, unsigned ep, float range, float* s) {
  for (int k = 0; k < 4; ++k) {
    const uint32_t w = static_cast<uint32_t>(HostPhiloxWord(seed, env, ep, 0x43504F4Cu, 0, k));
    s[k] = (host_u01(w) * 2.f - 1.f) * range;
  }
}

bool cartpole_physics(float* s, int action, const CartPoleConfig& p) {
  const float total_mass = p.masscart + p.masspole;
  const float pml = p.masspole * p.length;
  const float force = action == 1 ? p.force_mag : -p.force_mag;
  const float sin_t = std::sin(s[2]), cos_t = std::cos(s[2]);
  const float temp = (force + pml * s[3] * s[3] * sin_t) / total_mass;
  const float tacc = (p.gravity * sin_t - cos_t * temp) / (p.length * (4.0f / 3.0f - p.masspole * cos_t * cos_t / total_mass));
  const float xacc = temp - pml * tacc * cos_t / total_mass;
  s[0] += p.tau * s[1];
  s[1] += p.tau * xacc;
  s[2] += p.tau * s[3];
  s[3] += p.tau * tacc;
  return s[0] < -p.x_threshold || s[0] > p.x_threshold || s[2] < -p.theta_threshold || s[2] > p.theta_threshold;
}

Status check_cuda(int err, const char* what) { return FromCuda(err, what); }

// int32 action indices for CartPole from int32/int64 [N], float [N] (rounded)
// or float [N, A] (argmax).
at::Tensor discrete_actions(const at::Tensor& a, int n) {
  at::Tensor x = a;
  if (x.dim() == 2) x = x.argmax(1);
  else if (x.is_floating_point()) x = x.round();
  x = x.reshape({-1});
  if (x.numel() != n) throw std::invalid_argument("action has wrong number of elements");
  return x.to(at::kInt).contiguous();
}

}  // namespace

// ============================================================================
// GPUEnvironment
// ============================================================================
GPUEnvironment::GPUEnvironment(int num_envs, int obs_dim, int act_dim, Device device, EnvType type, uint64_t seed)
    : num_envs_(num_envs), obs_dim_(obs_dim), act_dim_(act_dim), device_(device), type_(type), seed_(seed),
      rng_(static_cast<std::mt19937::result_type>(seed)) {
  if (num_envs <= 0 || obs_dim <= 0 || act_dim <= 0) throw std::invalid_argument("GPUEnvironment dims must be positive");
  if (type == EnvType::kCartPole && (obs_dim != 4 || act_dim != 2))
    throw std::invalid_argument("CartPole has obs_dim 4 and act_dim 2");
  states_ = Tensor(Shape({num_envs, obs_dim}), DataType::kFloat32, device);
  ep_len_ = Tensor(Shape({num_envs}), DataType::kInt32, device);
  ep_ret_ = Tensor(Shape({num_envs}), DataType::kFloat32, device);
  ep_count_ = Tensor(Shape({num_envs}), DataType::kInt32, device);
  stats_ = Tensor(Shape({4}), DataType::kFloat32, device);
  Status st = Reset();
  if (!st.ok()) throw std::runtime_error(st.ToString());
}

Status GPUEnvironment::Reset() {
  if (type_ == EnvType::kLinear) {
    const unsigned seed = static_cast<unsigned>(rng_());
    if (device_.is_cuda()) {
      auto& s = states_.torch();
      return check_cuda(tb_env_linear_reset(s.data_ptr<float>(), num_envs_, obs_dim_, seed, StreamFor(s)),
                        "env_linear_reset");
    }
    float* s = states_.data<float>();
    for (int i = 0; i < num_envs_; ++i)
      for (int d = 0; d < obs_dim_; ++d) {
        const float u = ref_reset_unit(i, d, seed);
        s[static_cast<size_t>(i) * obs_dim_ + d] = (u * 2.0f - 1.0f) * 0.1f;
      }
    return Status::Ok();
  }
  stats_.torch().zero_();
  if (device_.is_cuda()) {
    auto& s = states_.torch();
    return check_cuda(tb_cartpole_reset(s.data_ptr<float>(), ep_len_.data<int>(), ep_ret_.data<float>(),
                                        reinterpret_cast<unsigned*>(ep_count_.data<int>()), num_envs_, seed_,
                                        cp_.init_range, StreamFor(s)),
                      "cartpole_reset");
  }
  float* s = states_.data<float>();
  for (int i = 0; i < num_envs_; ++i) {
    cartpole_initial(seed_, i, 0, cp_.init_range, s + 4 * static_cast<size_t>(i));
    ep_len_.data<int>()[i] = 0;
    ep_ret_.data<float>()[i] = 0.f;
    ep_count_.data<int>()[i] = 0;
  }
  return Status::Ok();
}

Status GPUEnvironment::Step(const Tensor& action, Tensor* obs, Tensor* reward, Tensor* done) {
  if (!obs || !reward || !done) return Status::InvalidArgument("Step output tensors must be non-null");
  if (!action.defined()) return Status::InvalidArgument("action is empty");
  if (action.device() != device_) return Status::InvalidArgument("action device must match environment device");
  at::Tensor o = at::empty({num_envs_, obs_dim_}, at::TensorOptions().dtype(at::kFloat).device(device_.torch()));
  at::Tensor r = at::empty({num_envs_}, o.options());
  at::Tensor d = at::empty({num_envs_}, o.options().dtype(at::kBool));
  TURBOL_RETURN_IF_ERROR(StepInto(action.torch(), o, r, d));
  *obs = Tensor(o);
  *reward = Tensor(r);
  *done = Tensor(d);
  return Status::Ok();
}

Status GPUEnvironment::StepInto(const at::Tensor& action, at::Tensor& obs, at::Tensor& reward, at::Tensor& done) {
  if (obs.numel() != static_cast<int64_t>(num_envs_) * obs_dim_ || reward.numel() != num_envs_ ||
      done.numel() != num_envs_)
    return Status::InvalidArgument("StepInto: output shapes do not match the environment");
  if (!obs.is_contiguous() || !reward.is_contiguous() || !done.is_contiguous())
    return Status::InvalidArgument("StepInto: outputs must be contiguous");
  if (done.element_size() != 1) return Status::InvalidArgument("StepInto: done must be bool/uint8");
  at::Tensor& s = states_.torch();
  if (type_ == EnvType::kLinear) {
    if (action.scalar_type() != at::kFloat) return Status::InvalidArgument("action must be Float32");
    if (action.numel() != static_cast<int64_t>(num_envs_) * act_dim_)
      return Status::InvalidArgument("action has wrong number of elements");
    at::Tensor a = action.contiguous();
    if (device_.is_cuda()) {
      const int e = tb_env_linear_step(s.data_ptr<float>(), a.data_ptr<float>(), s.data_ptr<float>(),
                                       reward.data_ptr<float>(), static_cast<uint8_t*>(done.data_ptr()), num_envs_,
                                       obs_dim_, act_dim_, decay_, force_, done_threshold_, StreamFor(s));
      TURBOL_RETURN_IF_ERROR(check_cuda(e, "env_linear_step"));
      obs.view({num_envs_, obs_dim_}).copy_(s, /*non_blocking=*/true);
      return Status::Ok();
    }
    if (obs.scalar_type() != at::kFloat || reward.scalar_type() != at::kFloat)
      return Status::InvalidArgument("StepInto: obs and reward must be Float32");
    float* st = s.data_ptr<float>();
    const float* ap = a.data_ptr<float>();
    float* rp = reward.data_ptr<float>();
    auto* dp = static_cast<uint8_t*>(done.data_ptr());
    float* op = obs.data_ptr<float>();
    const int O = obs_dim_, A = act_dim_;
    const float decay = decay_, force = force_, thr = done_threshold_;
    // Rounded like the device kernel (and the reference): each product and
    // sum once, in this order, no fused multiply-add (the host core is built
    // with -ffp-contract=off); the reward sums the squares in dimension order.
    for (int i = 0; i < num_envs_; ++i) {
      float* x = st + static_cast<size_t>(i) * O;
      const float* ai = ap + static_cast<size_t>(i) * A;
      float* oi = op + static_cast<size_t>(i) * O;
      float cost = 0.f;
      for (int k = 0; k < O; ++k) {
        const float t1 = decay * x[k];
        const float t2 = force * ai[k < A ? k : A - 1];
        const float v = t1 + t2;
        x[k] = v;
        oi[k] = v;
        const float sq = v * v;
        cost = cost + sq;
      }
      rp[i] = -cost;
      dp[i] = std::fabs(x[0]) > thr ? 1 : 0;
    }
    return Status::Ok();
  }
  // CartPole
  at::Tensor a;
  try {
    a = discrete_actions(action, num_envs_);
  } catch (const std::exception& e) {
    return Status::InvalidArgument(e.what());
  }
  if (device_.is_cuda()) {
    const int e = tb_cartpole_step(s.data_ptr<float>(), a.data_ptr<int>(), obs.data_ptr<float>(),
                                   reward.data_ptr<float>(), static_cast<uint8_t*>(done.data_ptr()),
                                   ep_len_.data<int>(), ep_ret_.data<float>(),
                                   reinterpret_cast<unsigned*>(ep_count_.data<int>()), stats_.data<float>(), num_envs_,
                                   seed_, cp_.params(), StreamFor(s));
    return check_cuda(e, "cartpole_step");
  }
  TURBOL_RETURN_IF_ERROR(StepCartPoleHost(a.data_ptr<int>(), reward.data_ptr<float>(),
                                          static_cast<uint8_t*>(done.data_ptr())));
  obs.view({num_envs_, 4}).copy_(s);
  return Status::Ok();
}

Status GPUEnvironment::StepCartPoleHost(const int* action, float* reward, uint8_t* done) {
  if (type_ != EnvType::kCartPole || device_.is_cuda())
    return Status::InvalidArgument("StepCartPoleHost: a CPU CartPole environment");
  float* st = states_.torch().data_ptr<float>();
  float* stats = stats_.data<float>();
  int* ep_len = ep_len_.data<int>();
  float* ep_ret = ep_ret_.data<float>();
  int* ep_count = ep_count_.data<int>();
  for (int i = 0; i < num_envs_; ++i) {
    float* x = st + 4 * static_cast<size_t>(i);
    const bool term = cartpole_physics(x, action[i], cp_);
    const int len = ep_len[i] + 1;
    const float ret = ep_ret[i] + 1.f;
    const bool fin = term || len >= cp_.max_steps;
    if (fin) {
      const unsigned e = static_cast<unsigned>(ep_count[i]) + 1;
      ep_count[i] = static_cast<int>(e);
      cartpole_initial(seed_, i, e, cp_.init_range, x);
      ep_len[i] = 0;
      ep_ret[i] = 0.f;
      stats[0] += ret;
      stats[1] += 1.f;
      stats[2] += static_cast<float>(len);
    } else {
      ep_len[i] = len;
      ep_ret[i] = ret;
    }
    reward[i] = 1.f;
    done[i] = fin ? 1 : 0;
  }
  return Status::Ok();
}

std::vector<double> GPUEnvironment::TakeEpisodeStats() {
  at::Tensor h = stats_.torch().to(at::kCPU).to(at::kDouble);
  stats_.torch().zero_();
  auto* p = h.data_ptr<double>();
  return {p[0], p[1], p[2]};
}

// ============================================================================
// RingBuffer
// ============================================================================
RingBuffer::RingBuffer(int64_t capacity, int obs_dim, int act_dim, Device device, uint64_t seed)
    : capacity_(capacity), obs_dim_(obs_dim), act_dim_(act_dim), device_(device), seed_(seed), host_rng_(seed) {
  if (capacity <= 0 || obs_dim <= 0 || act_dim <= 0) throw std::invalid_argument("RingBuffer dims must be positive");
  obs_ = Tensor(Shape({capacity, obs_dim}), DataType::kFloat32, device);
  act_ = Tensor(Shape({capacity, act_dim}), DataType::kFloat32, device);
  rew_ = Tensor(Shape({capacity}), DataType::kFloat32, device);
  done_ = Tensor(Shape({capacity}), DataType::kBool, device);
}

Status RingBuffer::Push(const Tensor& obs, const Tensor& act, const Tensor& reward, bool done) {
  if (obs.numel() < obs_dim_) return Status::InvalidArgument("obs too small");
  if (act.numel() < act_dim_) return Status::InvalidArgument("act too small");
  if (reward.numel() < 1) return Status::InvalidArgument("reward empty");
  auto opts = at::TensorOptions().device(device_.torch());
  at::Tensor o = obs.torch().reshape({-1}).narrow(0, 0, obs_dim_).to(opts.dtype(at::kFloat)).reshape({1, obs_dim_});
  at::Tensor a = act.torch().reshape({-1}).narrow(0, 0, act_dim_).to(opts.dtype(at::kFloat)).reshape({1, act_dim_});
  at::Tensor r = reward.torch().reshape({-1}).narrow(0, 0, 1).to(opts.dtype(at::kFloat));
  at::Tensor d = at::full({1}, done, opts.dtype(at::kBool));
  return PushBatch(Tensor(o), Tensor(a), Tensor(r), Tensor(d));
}

Status RingBuffer::PushBatch(const Tensor& obs, const Tensor& act, const Tensor& reward, const Tensor& done) {
  if (!obs.defined() || obs.shape().size() == 0) return Status::InvalidArgument("empty batch");
  int64_t B = obs.shape()[0];
  if (B <= 0) return Status::InvalidArgument("empty batch");
  if (obs.numel() < B * obs_dim_) return Status::InvalidArgument("obs batch dims mismatch");
  if (act.numel() < B * act_dim_) return Status::InvalidArgument("act batch dims mismatch");
  if (reward.numel() < B || done.numel() < B) return Status::InvalidArgument("reward/done batch mismatch");
  auto opts = at::TensorOptions().device(device_.torch());
  // inputs already of the buffer's dtype, device and layout are used as they
  // are (no conversion ops on the hot path)
  auto as = [&](const Tensor& t, int64_t n, at::ScalarType dt) {
    const at::Tensor& x = t.torch();
    if (x.scalar_type() == dt && x.device() == device_.torch() && x.is_contiguous() && x.numel() >= n) return x;
    return x.reshape({-1}).narrow(0, 0, n).to(opts.dtype(dt)).contiguous();
  };
  at::Tensor o = as(obs, B * obs_dim_, at::kFloat);
  at::Tensor a = as(act, B * act_dim_, at::kFloat);
  at::Tensor r = as(reward, B, at::kFloat);
  at::Tensor d = as(done, B, at::kBool);
  // Only the last `capacity` rows survive a push larger than the ring.
  int64_t skip = 0;
  if (B > capacity_) {
    skip = B - capacity_;
    head_ = (head_ + skip) % capacity_;
    B = capacity_;
  }
  const int64_t first = head_;
  if (device_.is_cuda()) {
    TbFieldSet fs{};
    fs.f[0] = TbField{o.data_ptr<float>() + skip * obs_dim_, obs_.data(), static_cast<int>(obs_dim_ * 4)};
    fs.f[1] = TbField{a.data_ptr<float>() + skip * act_dim_, act_.data(), static_cast<int>(act_dim_ * 4)};
    fs.f[2] = TbField{r.data_ptr<float>() + skip, rew_.data(), 4};
    fs.f[3] = TbField{static_cast<uint8_t*>(d.data_ptr()) + skip, done_.data(), 1};
    TURBOL_RETURN_IF_ERROR(
        check_cuda(tb_ring_push(fs, 4, static_cast<int>(B), head_, capacity_, StreamFor(o)), "ring_push"));
  } else {
    // at most two contiguous runs of slots (before and after the wrap)
    float* bo = obs_.data<float>();
    float* ba = act_.data<float>();
    float* br = rew_.data<float>();
    bool* bd = done_.data<bool>();
    const float* so = o.data_ptr<float>() + skip * obs_dim_;
    const float* sa = a.data_ptr<float>() + skip * act_dim_;
    const float* sr = r.data_ptr<float>() + skip;
    const bool* sd = d.data_ptr<bool>() + skip;
    int64_t done_rows = 0;
    while (done_rows < B) {
      const int64_t slot = (head_ + done_rows) % capacity_;
      const int64_t n = std::min(B - done_rows, capacity_ - slot);
      std::memcpy(bo + slot * obs_dim_, so + done_rows * obs_dim_, static_cast<size_t>(n * obs_dim_) * 4);
      std::memcpy(ba + slot * act_dim_, sa + done_rows * act_dim_, static_cast<size_t>(n * act_dim_) * 4);
      std::memcpy(br + slot, sr + done_rows, static_cast<size_t>(n) * 4);
      std::memcpy(bd + slot, sd + done_rows, static_cast<size_t>(n));
      done_rows += n;
    }
  }
  head_ = (head_ + B) % capacity_;
  size_ = std::min(capacity_, size_ + B);
  OnPushed(first, B);
  return Status::Ok();
}

at::Tensor RingBuffer::SampleIndices(int batch_size) {
  auto opts = at::TensorOptions().dtype(at::kInt).device(device_.torch());
  at::Tensor idx = at::empty({batch_size}, opts);
  const uint64_t ctr = sample_counter_++;
  if (device_.is_cuda()) {
    const int e = tb_sample_indices(idx.data_ptr<int>(), batch_size, size_, seed_, ctr, StreamFor(idx));
    if (e != 0) throw std::runtime_error("sample_indices failed");
  } else {
    int* ip = idx.data_ptr<int>();
    const uint64_t n = static_cast<uint64_t>(size_);
    uint32_t w[8];
    for (int i0 = 0; i0 < batch_size; i0 += 8) {
      host_philox_word0_x8(seed_, static_cast<uint32_t>(i0), static_cast<uint32_t>(ctr),
                           static_cast<uint32_t>(ctr >> 32), 0x52504C59u, w);
      for (int j = 0; j < 8 && i0 + j < batch_size; ++j)
        ip[i0 + j] = static_cast<int>((static_cast<uint64_t>(w[j]) * n) >> 32);
    }
  }
  return idx;
}

Status RingBuffer::Gather(const at::Tensor& idx_in, Tensor* obs, Tensor* act, Tensor* reward, Tensor* done) {
  if (!obs || !act || !reward || !done) return Status::InvalidArgument("null output pointer");
  at::Tensor idx = idx_in.scalar_type() == at::kInt && idx_in.device() == device_.torch() && idx_in.is_contiguous()
                      ? idx_in
                      : idx_in.to(at::TensorOptions().dtype(at::kInt).device(device_.torch())).contiguous();
  const int64_t B = idx.numel();
  auto opts = at::TensorOptions().device(device_.torch());
  at::Tensor o = at::empty({B, obs_dim_}, opts.dtype(at::kFloat));
  at::Tensor a = at::empty({B, act_dim_}, opts.dtype(at::kFloat));
  at::Tensor r = at::empty({B}, opts.dtype(at::kFloat));
  at::Tensor d = at::empty({B}, opts.dtype(at::kBool));
  if (device_.is_cuda()) {
    TbFieldSet fs{};
    fs.f[0] = TbField{obs_.data(), o.data_ptr(), static_cast<int>(obs_dim_ * 4)};
    fs.f[1] = TbField{act_.data(), a.data_ptr(), static_cast<int>(act_dim_ * 4)};
    fs.f[2] = TbField{rew_.data(), r.data_ptr(), 4};
    fs.f[3] = TbField{done_.data(), d.data_ptr(), 1};
    TURBOL_RETURN_IF_ERROR(
        check_cuda(tb_ring_gather(fs, 4, static_cast<int>(B), idx.data_ptr<int>(), StreamFor(o)), "ring_gather"));
  } else {
    const int* ip = idx.data_ptr<int>();
    const float* bo = obs_.data<float>();
    const float* ba = act_.data<float>();
    const float* br = rew_.data<float>();
    const bool* bd = done_.data<bool>();
    float* po = o.data_ptr<float>();
    float* pa = a.data_ptr<float>();
    float* pr = r.data_ptr<float>();
    bool* pd = d.data_ptr<bool>();
    const size_t ob = static_cast<size_t>(obs_dim_) * 4, ab = static_cast<size_t>(act_dim_) * 4;
    for (int64_t i = 0; i < B; ++i) {
      const int64_t s = ip[i];
      if (s < 0 || s >= capacity_) return Status::InvalidArgument("gather index out of range");
      std::memcpy(po + i * obs_dim_, bo + s * obs_dim_, ob);
      std::memcpy(pa + i * act_dim_, ba + s * act_dim_, ab);
      pr[i] = br[s];
      pd[i] = bd[s];
    }
  }
  *obs = Tensor(o);
  *act = Tensor(a);
  *reward = Tensor(r);
  *done = Tensor(d);
  return Status::Ok();
}

Status RingBuffer::Sample(int batch_size, Tensor* obs, Tensor* act, Tensor* reward, Tensor* done) {
  if (!obs || !act || !reward || !done) return Status::InvalidArgument("null output pointer");
  if (size_ == 0) return Status::InvalidArgument("Buffer is empty");
  if (batch_size <= 0) return Status::InvalidArgument("batch_size must be > 0");
  if (device_.is_cuda()) return Gather(SampleIndices(batch_size), obs, act, reward, done);
  // host: the indices of SampleIndices (same Philox stream and counter),
  // drawn 8 at a time and copied straight into the outputs
  const int64_t B = batch_size;
  auto opts = at::TensorOptions().device(device_.torch());
  at::Tensor o = at::empty({B, obs_dim_}, opts.dtype(at::kFloat));
  at::Tensor a = at::empty({B, act_dim_}, opts.dtype(at::kFloat));
  at::Tensor r = at::empty({B}, opts.dtype(at::kFloat));
  at::Tensor d = at::empty({B}, opts.dtype(at::kBool));
  const uint64_t ctr = sample_counter_++;
  const uint64_t n = static_cast<uint64_t>(size_);
  const float* bo = obs_.data<float>();
  const float* ba = act_.data<float>();
  const float* br = rew_.data<float>();
  const bool* bd = done_.data<bool>();
  float* po = o.data_ptr<float>();
  float* pa = a.data_ptr<float>();
  float* pr = r.data_ptr<float>();
  bool* pd = d.data_ptr<bool>();
  const size_t ob = static_cast<size_t>(obs_dim_) * 4, ab = static_cast<size_t>(act_dim_) * 4;
  uint32_t w[8];
  for (int64_t i0 = 0; i0 < B; i0 += 8) {
    host_philox_word0_x8(seed_, static_cast<uint32_t>(i0), static_cast<uint32_t>(ctr), static_cast<uint32_t>(ctr >> 32),
                         0x52504C59u, w);
    for (int j = 0; j < 8 && i0 + j < B; ++j) {
      const int64_t i = i0 + j, src = static_cast<int64_t>((static_cast<uint64_t>(w[j]) * n) >> 32);
      std::memcpy(po + i * obs_dim_, bo + src * obs_dim_, ob);
      std::memcpy(pa + i * act_dim_, ba + src * act_dim_, ab);
      pr[i] = br[src];
      pd[i] = bd[src];
    }
  }
  *obs = Tensor(o);
  *act = Tensor(a);
  *reward = Tensor(r);
  *done = Tensor(d);
  return Status::Ok();
}

// ============================================================================
// PrioritizedReplayBuffer
// ============================================================================
PrioritizedReplayBuffer::PrioritizedReplayBuffer(int64_t capacity, int obs_dim, int act_dim, float alpha, float beta,
                                                 float eps, Device device, uint64_t seed)
    : RingBuffer(capacity, obs_dim, act_dim, device, seed), alpha_(alpha), beta_(beta), eps_(eps) {
  leaves_ = 1;
  while (leaves_ < capacity) leaves_ <<= 1;
  auto opts = at::TensorOptions().device(device.torch());
  tree_ = at::zeros({2 * leaves_}, opts.dtype(at::kFloat));
  wmax_ = at::zeros({1}, opts.dtype(at::kInt));
  error_ = at::zeros({4}, opts.dtype(at::kInt));
}

void PrioritizedReplayBuffer::OnPushed(int64_t first_slot, int64_t n) {
  auto opts = at::TensorOptions().device(device_.torch());
  at::Tensor idx = at::arange(first_slot, first_slot + n, opts.dtype(at::kLong)).remainder_(capacity_);
  at::Tensor pr = at::full({n}, max_priority_, opts.dtype(at::kFloat));
  Status st = UpdatePriorities(idx, pr);
  if (!st.ok()) throw std::runtime_error(st.ToString());
}

Status PrioritizedReplayBuffer::UpdatePriorities(const at::Tensor& indices, const at::Tensor& priorities) {
  auto opts = at::TensorOptions().device(device_.torch());
  at::Tensor idx = indices.to(opts.dtype(at::kLong)).contiguous().reshape({-1});
  at::Tensor pr = priorities.to(opts.dtype(at::kFloat)).contiguous().reshape({-1});
  if (idx.numel() != pr.numel()) return Status::InvalidArgument("indices/priorities size mismatch");
  const int n = static_cast<int>(idx.numel());
  if (n == 0) return Status::Ok();
  // Track the running max priority on the host (new samples enter at it).
  const float mx = pr.abs().max().item<float>();
  max_priority_ = std::max(max_priority_, mx);
  if (device_.is_cuda()) {
    return check_cuda(tb_per_update(tree_.data_ptr<float>(), leaves_, reinterpret_cast<const long long*>(idx.data_ptr<int64_t>()), pr.data_ptr<float>(), n,
                                    alpha_, eps_, capacity_, error_.data_ptr(), StreamFor(tree_)),
                      "per_update");
  }
  float* t = tree_.data_ptr<float>();
  const int64_t* ip = idx.data_ptr<int64_t>();
  const float* pp = pr.data_ptr<float>();
  for (int i = 0; i < n; ++i) {
    if (ip[i] < 0 || ip[i] >= capacity_) return Status::InvalidArgument("priority index out of range");
    t[leaves_ + ip[i]] = std::pow(std::fabs(pp[i]) + eps_, alpha_);
  }
  for (int i = 0; i < n; ++i)
    for (int64_t node = (leaves_ + ip[i]) >> 1; node >= 1; node >>= 1) t[node] = t[2 * node] + t[2 * node + 1];
  return Status::Ok();
}

double PrioritizedReplayBuffer::TotalPriority() const { return tree_[1].item<double>(); }

Status PrioritizedReplayBuffer::SamplePrioritized(int batch_size, float beta, Tensor* obs, Tensor* act, Tensor* reward,
                                                  Tensor* done, at::Tensor* indices, at::Tensor* weights) {
  if (size_ == 0) return Status::InvalidArgument("Buffer is empty");
  if (batch_size <= 0) return Status::InvalidArgument("batch_size must be > 0");
  auto opts = at::TensorOptions().device(device_.torch());
  at::Tensor idx = at::empty({batch_size}, opts.dtype(at::kLong));
  at::Tensor w = at::empty({batch_size}, opts.dtype(at::kFloat));
  const uint64_t ctr = sample_counter_++;
  if (device_.is_cuda()) {
    TURBOL_RETURN_IF_ERROR(check_cuda(
        tb_per_sample(tree_.data_ptr<float>(), leaves_, size_, batch_size, beta, seed_, ctr, reinterpret_cast<long long*>(idx.data_ptr<int64_t>()),
                      w.data_ptr<float>(), nullptr, reinterpret_cast<unsigned*>(wmax_.data_ptr<int>()),
                      StreamFor(tree_)),
        "per_sample"));
  } else {
    const float* t = tree_.data_ptr<float>();
    const float total = t[1];
    const float seg = total / static_cast<float>(batch_size);
    float wmax = 0.f;
    for (int i = 0; i < batch_size; ++i) {
      const uint32_t r = static_cast<uint32_t>(HostPhiloxWord(seed_, i, static_cast<uint32_t>(ctr),
                                                              static_cast<uint32_t>(ctr >> 32), 0x50455253u, 0));
      float u = (static_cast<float>(i) + host_u01(r)) * seg;
      int64_t node = 1;
      while (node < leaves_) {
        const float left = t[2 * node];
        if (u < left || t[2 * node + 1] <= 0.f) {
          node = 2 * node;
        } else {
          u -= left;
          node = 2 * node + 1;
        }
      }
      int64_t leaf = node - leaves_;
      if (leaf >= size_) leaf = size_ - 1;
      const float p = t[leaves_ + leaf] / total;
      const float wi = std::pow(static_cast<float>(size_) * p, -beta);
      idx.data_ptr<int64_t>()[i] = leaf;
      w.data_ptr<float>()[i] = wi;
      wmax = std::max(wmax, wi);
    }
    if (wmax > 0.f) w.div_(wmax);
  }
  TURBOL_RETURN_IF_ERROR(Gather(idx, obs, act, reward, done));
  *indices = idx;
  *weights = w;
  return Status::Ok();
}

}  // namespace turbol
