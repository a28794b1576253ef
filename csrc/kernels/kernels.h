// C ABI of the turbol_b200 CUDA kernels.  Every launcher takes raw device
// pointers and a stream, launches on that stream, never synchronizes, and
// returns a cudaError_t as int (0 = success).  Host engines (C++) and the torch
// op bindings call these; no launcher allocates device memory — scratch, when a
// kernel needs it, is passed in by the caller.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// ---------------- environments ----------------
typedef struct {
  float gravity, masscart, masspole, length, force_mag, tau;
  float x_threshold, theta_threshold, init_range;
  int max_steps;
} TbCartPoleParams;

int tb_env_linear_reset(float* state, int n, int d, unsigned seed, cudaStream_t s);
int tb_env_linear_step(const float* state, const float* action, float* next_state, float* reward, uint8_t* done,
                       int n, int d, int a, float decay, float force, float thr, cudaStream_t s);
int tb_cartpole_reset(float* state, int* ep_len, float* ep_ret, unsigned* ep_count, int n, unsigned long long seed,
                      float init_range, cudaStream_t s);
int tb_cartpole_step(float* state, const int* action, float* obs_out, float* reward, uint8_t* done, int* ep_len,
                     float* ep_ret, unsigned* ep_count, float* stats, int n, unsigned long long seed,
                     TbCartPoleParams p, cudaStream_t s);
int tb_ppo_cartpole_act_step(const float* logits, int A, const float* values, float* state, int* ep_len,
                             float* ep_ret, unsigned* ep_count, float* stats, float* obs_buf, int* act_buf,
                             float* logp_buf, float* val_buf, float* rew_buf, uint8_t* done_buf,
                             const long long* iter_ptr, int t, int n, unsigned long long policy_seed,
                             unsigned long long env_seed, TbCartPoleParams p, cudaStream_t s);

// ---------------- replay ----------------
#define TB_MAX_FIELDS 8
typedef struct {
  const void* src;
  void* dst;
  int row_bytes;
} TbField;
typedef struct {
  TbField f[TB_MAX_FIELDS];
} TbFieldSet;

int tb_ring_push(TbFieldSet fs, int nf, int rows, long long head, long long capacity, cudaStream_t s);
int tb_ring_gather(TbFieldSet fs, int nf, int rows, const int* idx, cudaStream_t s);
int tb_sample_indices(int* idx, int n, long long size, unsigned long long seed, unsigned long long counter,
                      cudaStream_t s);
int tb_per_update(float* tree, long long L, const long long* idx, const float* prio, int n, float alpha, float eps,
                  long long capacity, void* error_word, cudaStream_t s);
int tb_per_rebuild(float* tree, long long L, cudaStream_t s);
int tb_per_sample(const float* tree, long long L, long long size, int n, float beta, unsigned long long seed,
                  unsigned long long counter, long long* out_idx, float* out_w, float* out_p, unsigned* wmax_scratch,
                  cudaStream_t s);

// ---------------- advantages ----------------
int tb_gae_chunks_for(int T, int N);
size_t tb_gae_scratch_bytes(int T, int N);
int tb_gae(const float* rew, const float* val, const uint8_t* done, float* adv, float* ret, double* stats,
           float* scratch, int T, int N, float gamma, float lam, cudaStream_t s);
int tb_grpo_advantage(const float* rewards, float* adv, int groups, int G, float eps, int scale_by_std,
                      cudaStream_t s);

// ---------------- PPO ----------------
int tb_ppo_gather(const float* obs, int obs_dim, const int* act, const float* logp, const float* adv, const float* ret,
                  const float* val, const double* adv_stats, float* o_obs, int* o_act, float* o_logp, float* o_adv,
                  float* o_ret, float* o_val, int total, int mb_size, int n_mb, const long long* step_ptr,
                  const long long* iter_ptr, long long step_imm, unsigned long long seed, int normalize,
                  cudaStream_t s);
int tb_ppo_loss(const float* logits, int A, const float* value, const int* act, const float* old_logp,
                const float* adv, const float* ret, const float* old_val, float* dlogits, float* dvalue, float* stats,
                int B, float clip, float vclip, float vf_coef, float ent_coef, cudaStream_t s);
int tb_counter_add(long long* counter, long long v, cudaStream_t s);

// ---------------- optimizer / elementwise ----------------
typedef struct {
  float lr, beta1, beta2, eps, weight_decay, grad_scale, max_grad_norm;
  long long step;  // used when step_ptr is null
} TbAdamParams;

int tb_adam(float* p, const float* g, float* m, float* v, void* p_bf16, long long n, TbAdamParams hp,
            const long long* step_ptr, const float* gnorm_sq, cudaStream_t s);
int tb_sumsq(const float* x, long long n, float* out, cudaStream_t s);
int tb_elementwise(float* out, const float* x, const float* y, long long n, float a, int op, cudaStream_t s);

// ---------------- rewards ----------------
int tb_hash_reward(const int* ids, const int* lens, int B, int T, float* out, cudaStream_t s);
int tb_rule_reward(const int* ids, const int* lens, int B, int T, int period_id, float format_bonus,
                   float length_penalty, int target_len, float clip, float* rule, float* total, cudaStream_t s);
int tb_masked_kl(const float* lp, const float* ref, const float* mask, int B, int T, float coef, int k3, float* out,
                 cudaStream_t s);
int tb_normalize_rewards(float* r, int B, int whiten, float eps, cudaStream_t s);

#ifdef __cplusplus
}
#endif
