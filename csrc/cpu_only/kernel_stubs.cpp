// Kernel launchers of the host core, for the CPU-only build (TURBOL_CUDA=0).
//
// The engines call these only on their CUDA branches, which a CPU-only build
// cannot reach (it has no CUDA tensors); each returns cudaErrorNoDevice so a
// call that got here by mistake fails as a Status instead of at link time.
// The normal build links the real launchers from csrc/kernels/*.cu instead.
#include "kernels.h"

extern "C" {

int tb_cartpole_reset(float* state, int* ep_len, float* ep_ret, unsigned* ep_count, int n, unsigned long long seed, float init_range, cudaStream_t s) {
  return static_cast<int>(cudaErrorNoDevice);
}

int tb_cartpole_step(float* state, const int* action, float* obs_out, float* reward, uint8_t* done, int* ep_len, float* ep_ret, unsigned* ep_count, float* stats, int n, unsigned long long seed, TbCartPoleParams p, cudaStream_t s) {
  return static_cast<int>(cudaErrorNoDevice);
}

int tb_elementwise(float* out, const float* x, const float* y, long long n, float a, int op, cudaStream_t s) {
  return static_cast<int>(cudaErrorNoDevice);
}

int tb_env_linear_reset(float* state, int n, int d, unsigned seed, cudaStream_t s) {
  return static_cast<int>(cudaErrorNoDevice);
}

int tb_env_linear_step(const float* state, const float* action, float* next_state, float* reward, uint8_t* done, int n, int d, int a, float decay, float force, float thr, cudaStream_t s) {
  return static_cast<int>(cudaErrorNoDevice);
}

int tb_hash_reward(const int* ids, const int* lens, int B, int T, float* out, cudaStream_t s) {
  return static_cast<int>(cudaErrorNoDevice);
}

int tb_masked_kl(const float* lp, const float* ref, const float* mask, int B, int T, float coef, int k3, float* out, cudaStream_t s) {
  return static_cast<int>(cudaErrorNoDevice);
}

int tb_normalize_rewards(float* r, int B, int whiten, float eps, cudaStream_t s) {
  return static_cast<int>(cudaErrorNoDevice);
}

int tb_per_sample(const float* tree, long long L, long long size, int n, float beta, unsigned long long seed, unsigned long long counter, long long* out_idx, float* out_w, float* out_p, unsigned* wmax_scratch, cudaStream_t s) {
  return static_cast<int>(cudaErrorNoDevice);
}

int tb_per_update(float* tree, long long L, const long long* idx, const float* prio, int n, float alpha, float eps, long long capacity, void* error_word, cudaStream_t s) {
  return static_cast<int>(cudaErrorNoDevice);
}

int tb_ring_gather(TbFieldSet fs, int nf, int rows, const int* idx, cudaStream_t s) {
  return static_cast<int>(cudaErrorNoDevice);
}

int tb_ring_push(TbFieldSet fs, int nf, int rows, long long head, long long capacity, cudaStream_t s) {
  return static_cast<int>(cudaErrorNoDevice);
}

int tb_rule_reward(const int* ids, const int* lens, int B, int T, int period_id, float format_bonus, float length_penalty, int target_len, float clip, float* rule, float* total, cudaStream_t s) {
  return static_cast<int>(cudaErrorNoDevice);
}

int tb_sample_indices(int* idx, int n, long long size, unsigned long long seed, unsigned long long counter, cudaStream_t s) {
  return static_cast<int>(cudaErrorNoDevice);
}

}  // extern "C"
