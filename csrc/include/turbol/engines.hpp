// RL engines of the host runtime: GPUEnvironment, RingBuffer,
// PrioritizedReplayBuffer and RewardEngine.  Device work goes to the kernels
// in csrc/kernels on the current torch stream; CPU instances run the same math
// on the host (they are also the oracles the kernel tests compare against).
//
// Parity (reference file:line):
//   GPUEnvironment  turbol_vllm/include/turbol/env/gpu_environment.hpp:18-64,
//                   src/env/gpu_environment.cpp:35-142 (linear env, seed 42)
//   RingBuffer      turbol_vllm/include/turbol/replay_buffer/ring_buffer.hpp:20-65,
//                   src/replay_buffer/replay_buffer.cpp:6-154
//   RewardEngine    turbol_vllm/include/turbol/reward/reward_engine.hpp:28-122,
//                   src/reward/reward_engine.cpp:11-189
#pragma once

#include <optional>
#include <random>
#include <string>
#include <vector>

#include "turbol/common.hpp"
#include "kernels.h"

namespace turbol {

uint64_t HostPhiloxWord(uint64_t seed, uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, int which);

// Host versions of the linear Gaussian policy's fused act / gradient passes
// and of the Adam step (csrc/engines/policy_host.cpp); flat fp32 parameters
// W_a [A, O], b_a [A], W_c [O], b_c.  The gradient is added into `grad`.
Status LinGaussActHost(const float* x, const float* params, float* act, float* logp, int N, int O, int A, float stdv,
                       uint64_t seed, uint32_t counter);
Status LinGaussGradHost(const float* batch, int row_w, const float* params, float* grad, int N, int O, int A,
                        float stdv, float clip, float vf_coef, bool has_old);
void AdamHost(float* p, const float* g, float* m, float* v, int64_t n, int64_t step, float lr, float b1, float b2,
              float eps, float wd, float grad_scale);
// One PPO minibatch step of an actor-critic MLP pair on the host
// (csrc/engines/mlp_host.cpp): actor widths dims_a (obs -> ... -> actions,
// categorical), critic widths dims_c (obs -> ... -> 1), tanh hidden layers,
// parameters laid out layer by layer (W [out, in], b [out]), actor first.
// Rows idx of the rollout tensors; gradients added into grad; stats (fp32
// [6]) += policy-loss sum, value-loss sum, entropy sum, approximate-KL sum,
// clipped count and row count.
Status PpoCategoricalMinibatchHost(const at::Tensor& flat, const at::Tensor& grad, const std::vector<int64_t>& dims_a,
                                   const std::vector<int64_t>& dims_c, const at::Tensor& obs, const at::Tensor& act,
                                   const at::Tensor& old_logp, const at::Tensor& adv, const at::Tensor& ret,
                                   const at::Tensor& idx, float clip, float vf_coef, float ent_coef,
                                   const at::Tensor& stats);
// A whole PPO update on the host: for every epoch e and minibatch k, the rows
// perms[e, k*minibatch : (k+1)*minibatch] go through
// PpoCategoricalMinibatchHost and one Adam step (moments m, v; the step
// counter continues from `step`).  Returns the last step number.
int64_t PpoCategoricalUpdateHost(const at::Tensor& flat, const at::Tensor& grad, const at::Tensor& m,
                                  const at::Tensor& v, int64_t step, const std::vector<int64_t>& dims_a,
                                  const std::vector<int64_t>& dims_c, const at::Tensor& obs, const at::Tensor& act,
                                  const at::Tensor& old_logp, const at::Tensor& adv, const at::Tensor& ret,
                                  const at::Tensor& perms, int64_t minibatch, float clip, float vf_coef,
                                  float ent_coef, float lr, float b1, float b2, float eps, float wd,
                                  const at::Tensor& stats, Status* st);
// GAE over [T, N] (values [T + 1, N], dones as bytes): advantages and returns
// in one backward sweep; stats (optional, float64 [2]) += sum and sum of
// squares of the advantages.
Status GaeHost(const float* rewards, const float* values, const uint8_t* dones, float* adv, float* ret, int T, int N,
               float gamma, float lam, double* stats);

// ---------------------------------------------------------------------------
enum class EnvType { kLinear, kCartPole };

struct CartPoleConfig {
  float gravity = 9.8f, masscart = 1.0f, masspole = 0.1f, length = 0.5f, force_mag = 10.0f, tau = 0.02f;
  float x_threshold = 2.4f, theta_threshold = 12.0f * 2.0f * 3.14159265358979f / 360.0f, init_range = 0.05f;
  int max_steps = 500;
  TbCartPoleParams params() const {
    return TbCartPoleParams{gravity, masscart, masspole, length, force_mag, tau,
                            x_threshold, theta_threshold, init_range, max_steps};
  }
};

class GPUEnvironment {
 public:
  GPUEnvironment(int num_envs = 1, int obs_dim = 4, int act_dim = 2, Device device = Device::CPU(),
                 EnvType type = EnvType::kLinear, uint64_t seed = 42);

  Status Reset();
  // Returns freshly allocated obs [N, obs_dim] f32, reward [N] f32, done [N] bool.
  Status Step(const Tensor& action, Tensor* obs, Tensor* reward, Tensor* done);
  // Writes into caller-owned tensors of the right shape/dtype (no allocation).
  Status StepInto(const at::Tensor& action, at::Tensor& obs, at::Tensor& reward, at::Tensor& done);
  // CPU CartPole only: one step from int32 actions [N] on raw pointers; the
  // state advances in place (finished episodes reset), reward / done [N] are
  // written, episode statistics accumulate.  No observation copy.
  Status StepCartPoleHost(const int* action, float* reward, uint8_t* done);
  Tensor Observe() const { return states_.Clone(); }
  // The live state tensor (CartPole: [N, 4]); used by the fused PPO rollout.
  at::Tensor& StateTensor() { return states_.torch(); }
  at::Tensor& EpLen() { return ep_len_.torch(); }
  at::Tensor& EpRet() { return ep_ret_.torch(); }
  at::Tensor& EpCount() { return ep_count_.torch(); }
  at::Tensor& StatsTensor() { return stats_.torch(); }
  // Returns {sum of finished-episode returns, episodes finished, sum of lengths}
  // since the last call, and clears the accumulator.
  std::vector<double> TakeEpisodeStats();

  int NumEnvs() const { return num_envs_; }
  int ObsDim() const { return obs_dim_; }
  int ActDim() const { return act_dim_; }
  Shape ObsShape() const { return Shape({num_envs_, obs_dim_}); }
  Shape ActionShape() const { return type_ == EnvType::kCartPole ? Shape({num_envs_}) : Shape({num_envs_, act_dim_}); }
  Device device() const { return device_; }
  EnvType type() const { return type_; }
  uint64_t seed() const { return seed_; }
  float decay() const { return decay_; }
  float force() const { return force_; }
  float done_threshold() const { return done_threshold_; }
  CartPoleConfig& cartpole() { return cp_; }

 private:
  int num_envs_, obs_dim_, act_dim_;
  Device device_;
  EnvType type_;
  uint64_t seed_;
  std::mt19937 rng_;
  Tensor states_, ep_len_, ep_ret_, ep_count_, stats_;
  float decay_ = 0.99f, force_ = 0.1f, done_threshold_ = 5.0f;
  CartPoleConfig cp_;
};

// ---------------------------------------------------------------------------
class RingBuffer {
 public:
  RingBuffer(int64_t capacity, int obs_dim, int act_dim, Device device = Device::CPU(), uint64_t seed = 0);
  virtual ~RingBuffer() = default;

  Status Push(const Tensor& obs, const Tensor& act, const Tensor& reward, bool done);
  Status PushBatch(const Tensor& obs, const Tensor& act, const Tensor& reward, const Tensor& done);
  // Uniform with replacement; outputs are (re)allocated on the buffer's device.
  Status Sample(int batch_size, Tensor* obs, Tensor* act, Tensor* reward, Tensor* done);
  // Gathers the given slots (int32 on the buffer's device) into new tensors.
  Status Gather(const at::Tensor& idx, Tensor* obs, Tensor* act, Tensor* reward, Tensor* done);
  at::Tensor SampleIndices(int batch_size);

  int64_t Size() const { return size_; }
  int64_t Capacity() const { return capacity_; }
  int64_t Head() const { return head_; }
  Device device() const { return device_; }
  void Clear() {
    head_ = 0;
    size_ = 0;
  }
  at::Tensor& Observations() { return obs_.torch(); }
  at::Tensor& Actions() { return act_.torch(); }
  at::Tensor& Rewards() { return rew_.torch(); }
  at::Tensor& Dones() { return done_.torch(); }

 protected:
  // Called after rows [head, head + n) (mod capacity) were written.
  virtual void OnPushed(int64_t first_slot, int64_t n) {}
  int64_t capacity_;
  int obs_dim_, act_dim_;
  Device device_;
  uint64_t seed_;
  uint64_t sample_counter_ = 0;
  std::mt19937_64 host_rng_;
  int64_t head_ = 0, size_ = 0;
  Tensor obs_, act_, rew_, done_;
};

class PrioritizedReplayBuffer : public RingBuffer {
 public:
  PrioritizedReplayBuffer(int64_t capacity, int obs_dim, int act_dim, float alpha = 0.6f, float beta = 0.4f,
                          float eps = 1e-6f, Device device = Device::CPU(), uint64_t seed = 0);
  // Stratified proportional sampling; returns slot indices (int64) and
  // IS weights normalized by the batch maximum.
  Status SamplePrioritized(int batch_size, float beta, Tensor* obs, Tensor* act, Tensor* reward, Tensor* done,
                           at::Tensor* indices, at::Tensor* weights);
  Status UpdatePriorities(const at::Tensor& indices, const at::Tensor& priorities);
  double TotalPriority() const;
  at::Tensor& Tree() { return tree_; }
  int64_t Leaves() const { return leaves_; }
  float alpha() const { return alpha_; }
  float beta() const { return beta_; }

 protected:
  void OnPushed(int64_t first_slot, int64_t n) override;

 private:
  float alpha_, beta_, eps_;
  float max_priority_ = 1.0f;
  int64_t leaves_;
  at::Tensor tree_;   // [2 * leaves] f32
  at::Tensor wmax_;   // [1] u32 scratch
  at::Tensor error_;  // device error word
};

// ---------------------------------------------------------------------------
enum class RewardMode { kScalar, kPerToken };

struct RewardConfig {
  float kl_coef = 0.01f;
  float kl_target = 0.1f;
  bool adaptive_kl = false;
  float kl_adapt_rate = 0.01f;
  bool normalize = true;
  bool whiten = false;  // divide by the batch std as well as centring
  float reward_clip = 10.0f;
  float gamma = 1.0f;
  RewardMode mode = RewardMode::kScalar;
  Device device = Device::CPU();
  float format_bonus = 0.1f;
  float length_penalty = -0.01f;
  int target_length = 256;
  int period_token_id = 46;  // byte-level id of '.' under the ByteTokenizer's raw-byte mapping
  bool k3_kl = false;
};

struct RewardResult {
  Tensor total, model_scores, kl_penalties, rule_scores;
};

class RewardEngine {
 public:
  explicit RewardEngine(const RewardConfig& cfg) : cfg_(cfg), kl_coef_(cfg.kl_coef) {}
  Status Initialize();
  Status ScoreBatch(const std::vector<std::string>& responses, const std::optional<Tensor>& ref_logprobs,
                    RewardResult* out);
  // Token path: token_ids [B, T] int32, masks [B, T] (1 = valid), optional
  // policy/ref log-probs [B, T] for the KL term.
  Status ScoreTokens(const Tensor& token_ids, const Tensor& masks, const std::optional<Tensor>& logprobs,
                     const std::optional<Tensor>& ref_logprobs, RewardResult* out);
  // reward = (FNV-1a-64(ids[:len]) mod 1000) / 1000.
  Status HashReward(const at::Tensor& token_ids, const at::Tensor& lengths, at::Tensor* out);
  Status ComputeKLPenalty(const at::Tensor& logprobs, const at::Tensor& ref_logprobs, const at::Tensor& masks,
                          at::Tensor* out);
  Status UpdateAdaptiveKL(float observed_kl);
  Status UpdateStats(const Tensor& rewards);
  float CurrentKLCoef() const { return kl_coef_; }
  const RewardConfig& config() const { return cfg_; }
  double RunningMean() const { return mean_; }
  double RunningVar() const { return count_ ? m2_ / static_cast<double>(count_) : 1.0; }
  int64_t RunningCount() const { return count_; }

 private:
  Status Normalize(at::Tensor& r);
  RewardConfig cfg_;
  bool initialized_ = false;
  float kl_coef_;
  double mean_ = 0.0, m2_ = 0.0;
  int64_t count_ = 0;
};

// The CPU PPO rollout on CartPole in one call: T steps of (record the state in
// obs_buf[t], actor / critic forward of the categorical MLP policy, an action
// drawn from the softmax by inverse CDF with the Philox uniform of
// (seed; env, t, counter), its log-probability and the value into act_buf[t],
// logp_buf[t], val_buf[t], then one host CartPole step into rew_buf[t],
// done_buf[t]), and the value of the final state into val_buf[T].  Layout of
// flat and the widths as for PpoCategoricalMinibatchHost.
Status PpoCartPoleRolloutHost(GPUEnvironment* env, const at::Tensor& flat, const std::vector<int64_t>& dims_a,
                              const std::vector<int64_t>& dims_c, const at::Tensor& obs_buf, const at::Tensor& act_buf,
                              const at::Tensor& logp_buf, const at::Tensor& val_buf, const at::Tensor& rew_buf,
                              const at::Tensor& done_buf, uint64_t seed, uint64_t counter);

}  // namespace turbol
