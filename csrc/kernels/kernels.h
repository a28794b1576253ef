// C ABI of the turbol_b200 CUDA kernels.  Every launcher takes raw device
// pointers and a stream, launches on that stream, never synchronizes, and
// returns a cudaError_t as int (0 = success).  Host engines (C++) and the torch
// op bindings call these; no launcher allocates device memory — scratch, when a
// kernel needs it, is passed in by the caller.
#pragma once

#if !defined(TURBOL_CUDA) || TURBOL_CUDA
#include <cuda_runtime.h>
#else
#include "turbol/cuda_compat.hpp"  // CPU-only build of the host core: runtime types only
#endif
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
int tb_pad_obs_bf16(const float* state, void* out, int n, cudaStream_t s);  // [n,4] f32 -> [n,8] bf16
// logits [n, ldl] (first A used), values [n, ldv] (column 0); obs_bf16 (nullable) [n, 8]
int tb_ppo_cartpole_act_step(const float* logits, int A, int ldl, const float* values, int ldv, float* state,
                             void* obs_bf16, int* ep_len,
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
                  float* o_ret, float* o_val, void* o_obs_bf16, int total, int mb_size, int n_mb,
                  const long long* step_ptr, const long long* iter_ptr, long long step_imm, unsigned long long seed,
                  int normalize, cudaStream_t s);
int tb_ppo_loss_padded(const float* logits, int ldl, int A, const float* value, int ldv, const int* act,
                       const float* old_logp, const float* adv, const float* ret, void* dlog_bf16, void* dval_bf16,
                       int ldd, float* stats, int B, float clip, float vf_coef, float ent_coef, float* db_log,
                       float* db_val, cudaStream_t s);
int tb_colsum_bf16(const void* x, long long ld, int rows, int cols, float* out, int accumulate, cudaStream_t s);
// First MLP layer with 8 (padded) input features: y = act(x . W^T + b), act 0
// none / 1 tanh; x bf16 [M, 8], W bf16 [N, 8] (N % 8 == 0, N <= 1024), y bf16.
// Linear Gaussian actor-critic (params: W_a [A, O], b_a [A], W_c [O], b_c):
// sampling with log-density, and the PPO + value-loss gradient accumulated
// into grad (caller zeroes it).  O <= 64, A <= 16.
int tb_lin_gauss_act(const float* x, const float* params, float* act, float* logp, int N, int O, int A, float stdv,
                     uint64_t seed, uint32_t counter, cudaStream_t s);
int tb_lin_gauss_grad(const float* batch, int row_w, const float* params, float* grad, int N, int O, int A,
                      float stdv, float clip, float vf_coef, int has_old, cudaStream_t s);
int tb_dense_k8_fwd(const void* x, long long ldx, const void* W, const float* bias, void* y, long long ldy, int M,
                    int N, int act, cudaStream_t s);
// Same, with the rows per CTA given (0: automatic).
int tb_dense_k8_fwd_rows(const void* x, long long ldx, const void* W, const float* bias, void* y, long long ldy,
                         int M, int N, int act, int rows_hint, cudaStream_t s);
// dW[N, 8] (fp32) = (or += with accumulate) dz[M, N]^T . x[M, 8] (bf16 inputs).
// out = A^T X over M rows for 8-wide X (the weight gradient of a layer with 8
// input or output features), A bf16 [M, N<=512], X bf16 [M, 8 * N/xblock]:
// A's column block b pairs with X's columns [8b, 8b+8); out[(j, k)] at
// j*os_j + k*os_k + b*os_blk, fp32, stored (or added with accumulate).
// scratch: tb_skinny8_scratch_floats(N) floats for the per-CTA partials.
size_t tb_skinny8_scratch_floats(int N);
int tb_skinny8_wgrad(const void* A, long long lda, const void* X, long long ldx, int xblock, float* out,
                     long long os_j, long long os_k, long long os_blk, int M, int N, int accumulate, float* scratch,
                     size_t scratch_floats, cudaStream_t s);
// dZ = (dOut_b W_b) * (1 - H^2) per head b (8 outputs per head, xblock hidden
// columns per head) and db (+)= column sums of dZ: the backward of an output
// layer with 8 outputs per head into a tanh layer.  scratch as above.
int tb_mlp_head_dz(const void* dout, long long ldd, const void* H, long long ldh, const void* W, long long ldw,
                   int xblock, void* dz, long long ldz, float* db, int M, int N, int accumulate, float* scratch,
                   size_t scratch_floats, cudaStream_t s);
// out[r, 8b + k] = bias[8b + k] + H[r, head b's xblock columns] . W[8b + k, same]:
// an output layer with 8 outputs per head (fp32 out, row stride ldo); xblock a
// power of two in [64, 256].
int tb_mlp_head_fwd(const void* H, long long ldh, const void* W, long long ldw, const float* bias, float* out,
                    long long ldo, int xblock, int heads, int M, cudaStream_t s);
int tb_dense_k8_wgrad(const void* dz, long long ldz, const void* x, long long ldx, float* dW, int M, int N,
                      int accumulate, cudaStream_t s);
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

// ---------------- tensor-core GEMM (tcgen05) ----------------
enum {
  TB_EPI_NONE = 0,
  TB_EPI_BIAS = 1,
  TB_EPI_BIAS_TANH = 2,
  TB_EPI_BIAS_SILU = 3,
  TB_EPI_TANH_BWD = 4,  // C = acc * (1 - aux^2)   (aux = saved tanh output)
  TB_EPI_RESIDUAL = 5,  // C = acc + aux
  TB_EPI_SWIGLU = 6,    // interleaved gate/up columns -> C[:, j] = silu(acc[2j]) * acc[2j+1]
                        // (C2, optional: the raw interleaved gate/up accumulator, bf16 [M, N])
  TB_EPI_SWIGLU_BWD = 7,  // acc = d out of out = silu(g) * u; aux = interleaved (g, u) bf16 [M, 2N];
                          // C = interleaved (d g, d u) bf16 [M, 2N]
};
#define TB_GEMM_ERR_TIMEOUT 2
typedef struct {
  const void* A;  // bf16; a_mn = 0: [M, K] (row stride lda), a_mn = 1: [K, M] (row stride lda)
  long long lda;
  int a_mn;
  const void* B;  // bf16; b_mn = 0: [N, K] (row stride ldb), b_mn = 1: [K, N]
  long long ldb;
  int b_mn;
  void* C;  // [M, N] row stride ldc; bf16 or fp32
  long long ldc;
  int c_fp32;
  int c_accumulate;  // C += result (fp32 atomics)
  int M, N, K;
  const float* bias;  // [N] fp32 (EPI_BIAS*)
  const void* aux;    // bf16 [M, N] row stride ld_aux (EPI_TANH_BWD / EPI_RESIDUAL)
  long long ld_aux;
  int epi;
  float alpha;  // 0 or 1 = no scaling
  int split_k;  // 0 = automatic (fp32 output, no nonlinear epilogue)
  int bn_hint;  // 0 = automatic, else 64, 128 or 256
  int* error;   // optional device int: set to TB_GEMM_ERR_TIMEOUT if a wait ran out
  // Optional split-K scratch (else atomics into an fp32 C).  Layout: 32 KB of
  // arrival counters, then the fp32 partials.  Zero-fill it before its first
  // use; every call that completes leaves the counters zero again.  Calls that
  // may overlap on the GPU need separate workspaces.
  void* workspace;
  size_t workspace_bytes;
  float* colsum;           // optional [N] fp32: column sums of the output (e.g. a bias gradient)
  void* C2;                // EPI_SWIGLU, optional bf16 [M, N]: also receives the raw gate/up accumulator
  long long ldc2;
  // Block-diagonal B (0 = off): B holds N / kgroup square diagonal blocks of
  // kgroup x kgroup (zeros elsewhere), so output column n only needs the K range
  // [g * kgroup, (g + 1) * kgroup) with g = n / kgroup; the kernel skips the rest.
  // Needs K == N and kgroup a multiple of 64 that divides N.
  int kgroup;
  // With kgroup: B holds the diagonal blocks only, packed along its inner
  // dimension (K-major: [N, kgroup], row n = block g's row; MN-major:
  // [K, kgroup], row k = block g's row), ldb >= kgroup.
  int kgroup_packed;
} TbGemmArgs;

int tb_gemm_bf16(const TbGemmArgs* args, cudaStream_t s);

// Small-M GEMM for decode (gemm_decode.cu): C[T, N] = epi(X[T, K] . W[N, K]^T)
// with the weight as the tensor cores' M side and K split over a thread-block
// cluster (reduced through distributed shared memory).  bf16 operands and
// output; epi is TB_EPI_NONE, TB_EPI_BIAS (fp32 [N]), TB_EPI_RESIDUAL (aux bf16
// [T, N]) or TB_EPI_SWIGLU (interleaved gate / up rows of W, C [T, N / 2]).
// N, K and every leading dimension a multiple of 8, base pointers 16-byte
// aligned; any T.
typedef struct {
  const void* X;
  long long ldx;
  const void* W;
  long long ldw;
  void* C;
  long long ldc;
  int T, N, K;
  int epi;
  const float* bias;
  const void* aux;
  long long ld_aux;
  int splits;  // 0: automatic (fill the SMs, at most 8 per cluster)
  int* error;  // optional: set when a wait ran out
} TbDecodeGemmArgs;

int tb_gemm_decode(const TbDecodeGemmArgs* args, cudaStream_t s);
// The automatic split count (cluster size) for T tokens and an [N, K] weight.
int tb_gemm_decode_splits(int T, int N, int K);
// PPO output layer + clipped loss + output-layer backward in one pass over the
// hidden activations H2 = [H2a | H2c] (bf16 [M, 2H]); categorical actor with A
// actions.  W3 bf16 [>= crow + 1, 2H] (actor rows 0..A-1 over columns [0, H),
// the critic row `crow` over [H, 2H)), b3 fp32.  Writes dZ2 (bf16 [M, 2H]),
// the gradients of b2, W3 (actor rows and the critic row) and b3 (written, not
// accumulated), and adds [pg, v, entropy, kl, clipfrac, rows] into stats.
// part: scratch of tb_ppo_head_part_numel(H, A, parts) floats.
typedef struct {
  const void* H2;
  long long ldh;
  const void* W3;
  long long ldw;
  const float* b3;
  int crow;
  const int* act;
  const float* old_logp;
  const float* adv;
  const float* ret;
  void* dz;
  long long ldz;
  float* g_w3;
  long long ldgw;
  float* g_b3;
  float* g_b2;
  float* stats;
  float* part;
  int parts;  // CTAs (each writes one partial row)
  int M, H, A;
  float clip, vf_coef, ent_coef;
} TbPpoHeadArgs;
int tb_ppo_head(const TbPpoHeadArgs* args, cudaStream_t s);
long long tb_ppo_head_part_numel(int H, int A, int parts);
int tb_ppo_head_default_parts(int H, int A);  // CTAs for one resident wave on this device

size_t tb_gemm_workspace_bytes(int M, int N, int K);

// ---------------- transformer ops ----------------
int tb_rmsnorm_fwd(const void* x, const float* w, void* y, float* rstd, int T, int D, float eps, cudaStream_t s);
int tb_rmsnorm_bwd(const void* dy, const void* x, const float* w, const float* rstd, void* dx, const void* dx_add,
                   float* dw, int T, int D, cudaStream_t s);
// Same; with a workspace of tb_rmsnorm_bwd_ws_floats(D) floats the blocks'
// weight-gradient partials are summed by a second pass instead of contended
// global atomics (dw still accumulates: dw += sum).
size_t tb_rmsnorm_bwd_ws_floats(int D);
int tb_rmsnorm_bwd_ws(const void* dy, const void* x, const float* w, const float* rstd, void* dx, const void* dx_add,
                      float* dw, int T, int D, float* ws, size_t ws_floats, cudaStream_t s);
int tb_rope(void* qkv, long long ld, const int* pos, const void* table, int T, int n_rot_heads, int D, int inverse,
            cudaStream_t s);
int tb_embed_fwd(const int* ids, const void* W, void* out, int T, int D, int V, int* err, cudaStream_t s);
int tb_embed_bwd(const int* ids, const void* dout, float* dW, int T, int D, int V, cudaStream_t s);
int tb_swiglu_bwd(const void* gu, const void* dh, void* dgu, long long T, int F, cudaStream_t s);
int tb_swiglu_fwd(const void* gu, void* act, long long T, int F, cudaStream_t s);
int tb_kv_write(const void* qkv, long long ld, int k_off, int v_off, const int* seq_of_token, const int* pos,
                const int* block_table, int max_blocks, void* kc, void* vc, int T, int Hk, int D, int bs,
                cudaStream_t s);
// RoPE (in place on the q and k heads of fused QKV rows, k / v at columns
// Hq*D and (Hq+Hk)*D) and the paged-cache write of the rotated k and of v, in
// one launch.
int tb_rope_kv_write(void* qkv, long long ld, const int* pos, const void* table, int Hq, int Hk, int D,
                     const int* seq_of_token, const int* block_table, int max_blocks, void* kc, void* vc, int T, int bs,
                     cudaStream_t s);
int tb_decode_attention(const void* q, long long ldq, const void* kc, const void* vc, const int* block_table,
                        int max_blocks, const int* ctx_len, void* out, long long ldo, int B, int Hq, int Hk, int D,
                        int bs, float scale, cudaStream_t s);
// The same with each (sequence, KV head) context split into n_split chunks
// run by separate CTAs (head dim 128, 16-token blocks, <= 8 query heads per
// KV head); the last chunk to finish merges the partials.  part: fp32
// scratch of tb_decode_attention_part_floats(); counters: B * Hk ints, zero
// before the first call and left zero by every call.
int tb_decode_attention_split(const void* q, long long ldq, const void* kc, const void* vc, const int* block_table,
                              int max_blocks, const int* ctx_len, void* out, long long ldo, int B, int Hq, int Hk,
                              int D, int bs, float scale, int n_split, float* part, int* counters, cudaStream_t s);
// Chunks per context that fill the SMs' resident CTA slots in the fewest
// waves (for long contexts), 1..8.
int tb_decode_attention_splits(int B, int Hk);
size_t tb_decode_attention_part_floats(int B, int Hq, int Hk, int n_split);
// seed_ptr / temp_ptr (optional) override seed / temperature from device
// memory, so a captured CUDA graph can be replayed with new values.
int tb_sample(const void* logits, long long ld, int B, int V, float temperature, unsigned long long seed,
              const long long* step_ptr, long long step_imm, int* out_tok, float* out_logp, int* tok_mat,
              float* lp_mat, int ld_mat, const unsigned long long* seed_ptr, const float* temp_ptr, cudaStream_t s);
// Sampling with top-k (k <= 0: off), top-p (p >= 1: off) and an end-of-sequence
// stop (eos_id < 0: off; then done [B] flags, lengths [B] and the n_done
// counter are updated).  The returned log-prob is under the full tempered
// softmax.
int tb_sample_filtered(const void* logits, long long ld, int B, int V, float temperature, int top_k, float top_p,
                       unsigned long long seed, const long long* step_ptr, long long step_imm, int* out_tok,
                       float* out_logp, int* tok_mat, float* lp_mat, int ld_mat, const unsigned long long* seed_ptr,
                       const float* temp_ptr, int eos_id, int pad_id, unsigned char* done, int* lengths, int* n_done,
                       cudaStream_t s);
int tb_logprob(void* logits, long long ld, int T, int V, const int* target, float* logp, const float* dlogp,
               float inv_temp, cudaStream_t s);
int tb_grpo_loss(const float* lp, const float* old_lp, const float* ref_lp, const float* adv, const float* mask,
                 float* dlp, float* stats, int B, int T, float clip, float beta, float inv_total_seqs,
                 cudaStream_t s);
// Clipped PPO policy loss + clipped value loss per token (RLHF with a value
// head), forward and backward: dlp, dv = d loss / d (lp, v), loss = norm *
// (sum pg + vf_coef sum vf); stats (nullable) += {pg * norm, vf * norm,
// clipped tokens, tokens}.  All arrays fp32 [R].
int tb_ppo_token_loss(const float* lp, const float* old_lp, const float* adv, const float* v, const float* old_v,
                      const float* ret, float* dlp, float* dv, float* stats, long long R, float clip, float vclip,
                      float vf_coef, float norm, cudaStream_t s);
int tb_flash_attn_fwd(const void* q, const void* k, const void* v, long long ld, void* o, long long ldo, float* lse,
                      int B, int T, int Hq, int Hk, float scale, cudaStream_t s);
// Same contract on tcgen05 tensor cores (TMA + TMEM); err (nullable) gets site
// 21 when a bounded wait ran out.
int tb_flash_attn_fwd_tc(const void* q, const void* k, const void* v, long long ld, void* o, long long ldo, float* lse,
                         int B, int T, int Hq, int Hk, float scale, int* err, cudaStream_t s);
int tb_flash_attn_bwd(const void* q, const void* k, const void* v, long long ld, const void* o, long long ldo,
                      const void* dout, long long lddo, const float* lse, float* delta, void* dq, void* dk, void* dv,
                      long long lddqkv, int B, int T, int Hq, int Hk, float scale, cudaStream_t s);
// delta[b, h, t] = sum_d dO[t, h, d] * O[t, h, d] (the backward's row term)
int tb_flash_attn_delta(const void* o, long long ldo, const void* dout, long long lddo, float* delta, int B, int T,
                        int Hq, cudaStream_t s);
// Backward on tcgen05: delta, dK/dV (KV tile outer) and dQ (query tile outer).
// ws (nullable, tb_flash_attn_bwd_ws_bytes) lets the dK/dV pass split a GQA
// group over CTAs and sum in fp32; err (nullable) gets site 22/23 on a timeout.
size_t tb_flash_attn_bwd_ws_bytes(int B, int T, int Hk);
int tb_flash_attn_bwd_tc(const void* q, const void* k, const void* v, long long ld, const void* o, long long ldo,
                         const void* dout, long long lddo, const float* lse, float* delta, void* dq, void* dk,
                         void* dv, long long lddqkv, int B, int T, int Hq, int Hk, float scale, float* ws,
                         size_t ws_bytes, int* err, cudaStream_t s);

// ---------------- NVLink peer-memory collectives ----------------
#define TB_MAX_PEERS 8
typedef struct {
  void* base[TB_MAX_PEERS];  // every rank's symmetric buffer, mapped into this process
  void* hdr[TB_MAX_PEERS];   // every rank's flag header (inside its buffer)
  unsigned* epoch_ctr;       // local: epoch of the last completed call
  int rank, world;
} TbPeerTable;

size_t tb_peer_header_bytes(void);
// Data-parallel Adam with one handshake for small vectors: every rank pulls
// every peer's whole gradient (snapshotted into its send buffer at send_off)
// and runs Adam on the whole vector (m, v full-size on every rank); only
// local weights are written.  rep_epoch: the step's own epoch counter.
int tb_peer_allreduce_adam_rep(TbPeerTable t, long long grad_off, long long send_off, long long param_off,
                               long long shadow_off, long long n, float* m, float* v, TbAdamParams hp,
                               const long long* step_ptr, unsigned* rep_epoch, unsigned* done_ctr, int* err,
                               cudaStream_t s);
// One row-segment copy of tb_peer_scatter_copy (all sizes and offsets in bytes,
// multiples of 16).
typedef struct {
  long long vec_begin;  // first 16-byte vector of this segment in the flattened work (exclusive prefix)
  long long src_off, src_ld;
  long long dst_off, dst_ld;  // relative to dst_base in every rank's payload
  long long rows, row_bytes;
  int src_sel;  // 0: src0, 1: src1
  int peers;    // 1: write into every rank, 0: this rank only
} TbCopySeg;
// Every rank copies its segments (segs: device array, sorted by vec_begin) from
// its local src0 / src1 into the payloads of all ranks (or only its own),
// between the begin / finish handshakes of the peer collectives.
int tb_peer_scatter_copy(TbPeerTable t, const void* src0, const void* src1, const TbCopySeg* segs, int nseg,
                         long long total_vecs, long long dst_base, unsigned* done_ctr, int* err, cudaStream_t s);
// The peer collectives' bounded flag wait, alone: waits up to budget_ns for
// flags[0..n) >= expect, then sets *err = 99 (site code) and returns.
int tb_bounded_wait_probe(const unsigned* flags, int n, unsigned expect, unsigned long long budget_ns, int* err,
                          cudaStream_t s);

// ---- tensor parallelism: collectives fused into the tcgen05 GEMM -----------
// Symmetric layout per rank (mapped into every peer): a header of
// tb_tp_header_bytes() (flags) and a data region of two parity halves.
typedef struct {
  int rank, world, rows_per_rank;  // rows_per_rank: a multiple of 128
  unsigned* epoch_ctr;             // device counter: epoch of this op's previous call (one per op)
  unsigned* done_ctr;              // device counter, zero-initialized (one per op)
  void* hdr[TB_MAX_PEERS];         // every rank's header
  void* data[TB_MAX_PEERS];        // every rank's data region
  long long parity_bytes;          // bytes of one parity half of a data region
  int* err;                        // device error word (a nonzero site after a timed-out wait)
  unsigned* rs_target;             // reduce-scatter only: device [2] arrival targets, zero-initialized
  void* gather_out;                // all-gather only, optional: bf16 [M, K] receives the gathered A
  long long ld_gather;             // its row stride (elements, a multiple of 8)
} TbTpComm;
size_t tb_tp_header_bytes(void);
// C[M, N] = gather_rows(A) . B^T with A this rank's rows [rows_per_rank, K]
// (a->A, a->lda) and M = world * rows_per_rank; the other ranks' rows arrive by
// peer stores into this rank's data region (needs 2 * M * K * 2 bytes) while
// the tiles of the local rows are computed.  Epilogues as tb_gemm_bf16.
// With c->gather_out set, the gathered A [M, K] is also written there (for the
// weight gradient of a column-parallel layer, or of a row-parallel layer's
// backward), at the end of the same kernel.
int tb_tp_ag_gemm(const TbTpComm* c, const TbGemmArgs* a, cudaStream_t s);
// out[rows_per_rank, N] = (sum over ranks of A_r . B_r^T)[this rank's rows]
// (+ bias) (+ residual): each GEMM tile is stored (bf16) into the receive slot
// of the rank that owns its rows; a finishing kernel sums the slots.  The
// data region needs 2 * M * N * 2 bytes.
int tb_tp_gemm_rs(const TbTpComm* c, const TbGemmArgs* a, void* out, long long ldo, const float* bias,
                  const void* residual, long long ld_res, cudaStream_t s);
// out[i] = scale * sum_p in_p[i] for fp32 buffers at byte offsets in_off/out_off
// of every rank's symmetric buffer (in-place when in_off == out_off).
int tb_peer_allreduce(TbPeerTable t, long long in_off, long long out_off, long long n, float scale,
                      unsigned* done_ctr, int* err, cudaStream_t s);
// grad (fp32) reduce-scatter -> Adam on the owned shard -> fp32 weights and
// bf16 copy written into every rank's buffer.  m and v hold the owned shard
// only: element i of the owned slice [lo, hi) is m[i - lo].
void tb_peer_owned_slice(long long n, int rank, int world, long long* lo, long long* hi);
int tb_peer_allreduce_adam(TbPeerTable t, long long grad_off, long long param_off, long long shadow_off, long long n,
                           float* m, float* v, TbAdamParams hp, const long long* step_ptr, unsigned* done_ctr,
                           int* err, cudaStream_t s);

#ifdef __cplusplus
}
#endif
