// torch-tensor entry points of the RL kernels (turbol_b200.turbol_core.ops).
// Each op checks device, dtype, contiguity and shapes, then launches on the
// current torch CUDA stream; errors raise.  No op allocates scratch behind the
// caller's back except where the output itself is returned.
#include <pybind11/pybind11.h>
#include <torch/extension.h>

#include "kernels.h"
#include "turbol/common.hpp"

namespace py = pybind11;

namespace {

#define TB_CHECK(cond, msg)                                  \
  do {                                                       \
    if (!(cond)) throw std::invalid_argument(std::string(msg)); \
  } while (0)

void cuda_ok(int e, const char* what) {
  if (e != 0) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(static_cast<cudaError_t>(e)));
}

void need(const at::Tensor& t, at::ScalarType dt, const char* name) {
  TB_CHECK(t.defined(), std::string(name) + " is undefined");
  TB_CHECK(t.is_cuda(), std::string(name) + " must be a CUDA tensor");
  TB_CHECK(t.scalar_type() == dt, std::string(name) + " has the wrong dtype");
  TB_CHECK(t.is_contiguous(), std::string(name) + " must be contiguous");
}

cudaStream_t stream_of(const at::Tensor& t) { return turbol::StreamFor(t); }

// A row-major 2-D block (unit column stride, any row stride), e.g. a column
// block of a wider buffer; 1-D tensors must be contiguous.
void need_rows(const at::Tensor& t, at::ScalarType dt, const char* name) {
  TB_CHECK(t.defined() && t.is_cuda() && t.scalar_type() == dt, std::string(name) + ": wrong device or dtype");
  TB_CHECK((t.dim() == 2 && t.stride(1) == 1) || (t.dim() == 1 && t.is_contiguous()),
           std::string(name) + " must have unit column stride");
}

TbCartPoleParams cp_params(py::dict d) {
  TbCartPoleParams p{9.8f, 1.0f, 0.1f, 0.5f, 10.0f, 0.02f, 2.4f, 12.0f * 2.0f * 3.14159265358979f / 360.0f, 0.05f, 500};
  if (d.contains("gravity")) p.gravity = d["gravity"].cast<float>();
  if (d.contains("masscart")) p.masscart = d["masscart"].cast<float>();
  if (d.contains("masspole")) p.masspole = d["masspole"].cast<float>();
  if (d.contains("length")) p.length = d["length"].cast<float>();
  if (d.contains("force_mag")) p.force_mag = d["force_mag"].cast<float>();
  if (d.contains("tau")) p.tau = d["tau"].cast<float>();
  if (d.contains("x_threshold")) p.x_threshold = d["x_threshold"].cast<float>();
  if (d.contains("theta_threshold")) p.theta_threshold = d["theta_threshold"].cast<float>();
  if (d.contains("init_range")) p.init_range = d["init_range"].cast<float>();
  if (d.contains("max_steps")) p.max_steps = d["max_steps"].cast<int>();
  return p;
}

}  // namespace

void register_kernel_ops(py::module_& m) {
  // ---------------- environments ----------------
  m.def("cartpole_reset",
        [](at::Tensor state, at::Tensor ep_len, at::Tensor ep_ret, at::Tensor ep_count, uint64_t seed, float range) {
          need(state, at::kFloat, "state");
          need(ep_len, at::kInt, "ep_len");
          need(ep_ret, at::kFloat, "ep_ret");
          need(ep_count, at::kInt, "ep_count");
          const int n = static_cast<int>(ep_len.numel());
          TB_CHECK(state.numel() == 4LL * n, "state must be [N, 4]");
          cuda_ok(tb_cartpole_reset(state.data_ptr<float>(), ep_len.data_ptr<int>(), ep_ret.data_ptr<float>(),
                                    reinterpret_cast<unsigned*>(ep_count.data_ptr<int>()), n, seed, range,
                                    stream_of(state)),
                  "cartpole_reset");
        },
        py::arg("state"), py::arg("ep_len"), py::arg("ep_ret"), py::arg("ep_count"), py::arg("seed"),
        py::arg("init_range") = 0.05f);

  m.def("pad_obs_bf16", [](at::Tensor state, at::Tensor out) {
    need(state, at::kFloat, "state");
    need(out, at::kBFloat16, "out");
    const int n = static_cast<int>(state.size(0));
    TB_CHECK(state.numel() == 4LL * n && out.numel() == 8LL * n, "pad_obs_bf16: [N,4] -> [N,8]");
    cuda_ok(tb_pad_obs_bf16(state.data_ptr<float>(), out.data_ptr(), n, stream_of(state)), "pad_obs_bf16");
  });

  // logits [N, ldl] (first A columns used), values [N, ldv] (column 0);
  // obs_bf16 (optional) receives the next observation as bf16 [N, 8].
  m.def("ppo_cartpole_act_step",
        [](at::Tensor logits, int A, at::Tensor values, at::Tensor state, py::object obs_bf16, at::Tensor ep_len,
           at::Tensor ep_ret, at::Tensor ep_count, at::Tensor stats, at::Tensor obs_buf, at::Tensor act_buf,
           at::Tensor logp_buf, at::Tensor val_buf, at::Tensor rew_buf, at::Tensor done_buf, py::object iter_ptr,
           int t, uint64_t policy_seed, uint64_t env_seed, py::dict params) {
          need_rows(logits, at::kFloat, "logits");
          need_rows(values, at::kFloat, "values");
          need(state, at::kFloat, "state");
          need(obs_buf, at::kFloat, "obs_buf");
          need(act_buf, at::kInt, "act_buf");
          need(logp_buf, at::kFloat, "logp_buf");
          need(val_buf, at::kFloat, "val_buf");
          need(rew_buf, at::kFloat, "rew_buf");
          TB_CHECK(done_buf.is_cuda() && done_buf.element_size() == 1 && done_buf.is_contiguous(), "done_buf u8");
          const int n = static_cast<int>(state.size(0));
          TB_CHECK(logits.dim() == 2 && logits.size(0) == n && logits.size(1) >= A && logits.stride(1) == 1,
                   "logits [N, >=A]");
          TB_CHECK(values.size(0) == n && (values.dim() == 1 || values.stride(1) == 1), "values batch mismatch");
          TB_CHECK(obs_buf.dim() == 3 && obs_buf.size(1) == n && t >= 0 && t < obs_buf.size(0), "obs_buf [T, N, 4]");
          const int ldv = values.dim() == 2 ? static_cast<int>(values.stride(0)) : 1;
          void* ob = nullptr;
          if (!obs_bf16.is_none()) {
            at::Tensor x = obs_bf16.cast<at::Tensor>();
            need(x, at::kBFloat16, "obs_bf16");
            TB_CHECK(x.numel() == 8LL * n, "obs_bf16 [N, 8]");
            ob = x.data_ptr();
          }
          const long long* ip = nullptr;
          if (!iter_ptr.is_none()) {
            at::Tensor it = iter_ptr.cast<at::Tensor>();
            need(it, at::kLong, "iter");
            ip = reinterpret_cast<const long long*>(it.data_ptr<int64_t>());
          }
          cuda_ok(tb_ppo_cartpole_act_step(
                      logits.data_ptr<float>(), A, static_cast<int>(logits.stride(0)), values.data_ptr<float>(), ldv,
                      state.data_ptr<float>(), ob, ep_len.data_ptr<int>(), ep_ret.data_ptr<float>(),
                      reinterpret_cast<unsigned*>(ep_count.data_ptr<int>()), stats.data_ptr<float>(),
                      obs_buf.data_ptr<float>(), act_buf.data_ptr<int>(), logp_buf.data_ptr<float>(),
                      val_buf.data_ptr<float>(), rew_buf.data_ptr<float>(),
                      static_cast<uint8_t*>(done_buf.data_ptr()), ip, t, n, policy_seed, env_seed, cp_params(params),
                      stream_of(state)),
                  "ppo_cartpole_act_step");
        });

  // ---------------- replay ----------------
  m.def("sample_indices",
        [](int64_t n, int64_t size, uint64_t seed, uint64_t counter, at::Device dev) {
          at::Tensor idx = at::empty({n}, at::TensorOptions().dtype(at::kInt).device(dev));
          cuda_ok(tb_sample_indices(idx.data_ptr<int>(), static_cast<int>(n), size, seed, counter, stream_of(idx)),
                  "sample_indices");
          return idx;
        });

  // Pushes rows of several tensors (each [B, ...], same B) into ring tensors
  // ([cap, ...]) at slots (head + i) mod cap, in one launch.
  m.def("ring_push",
        [](std::vector<at::Tensor> src, std::vector<at::Tensor> dst, int64_t head) {
          TB_CHECK(src.size() == dst.size() && !src.empty() && src.size() <= TB_MAX_FIELDS, "field count");
          const int64_t B = src[0].size(0), cap = dst[0].size(0);
          TbFieldSet fs{};
          for (size_t k = 0; k < src.size(); ++k) {
            TB_CHECK(src[k].is_cuda() && dst[k].is_cuda() && src[k].is_contiguous() && dst[k].is_contiguous(),
                     "ring_push needs contiguous CUDA tensors");
            TB_CHECK(src[k].size(0) == B && dst[k].size(0) == cap, "ring_push row count mismatch");
            TB_CHECK(src[k].scalar_type() == dst[k].scalar_type(), "ring_push dtype mismatch");
            const int64_t rb = src[k].numel() / std::max<int64_t>(B, 1) * src[k].element_size();
            TB_CHECK(rb == dst[k].numel() / cap * dst[k].element_size(), "ring_push row size mismatch");
            fs.f[k] = TbField{src[k].data_ptr(), dst[k].data_ptr(), static_cast<int>(rb)};
          }
          cuda_ok(tb_ring_push(fs, static_cast<int>(src.size()), static_cast<int>(B), head, cap, stream_of(src[0])),
                  "ring_push");
        });

  m.def("ring_gather",
        [](std::vector<at::Tensor> src, std::vector<at::Tensor> dst, at::Tensor idx) {
          TB_CHECK(src.size() == dst.size() && !src.empty() && src.size() <= TB_MAX_FIELDS, "field count");
          need(idx, at::kInt, "idx");
          const int64_t B = idx.numel();
          TbFieldSet fs{};
          for (size_t k = 0; k < src.size(); ++k) {
            TB_CHECK(src[k].is_contiguous() && dst[k].is_contiguous() && dst[k].size(0) == B, "ring_gather shapes");
            const int64_t rb = dst[k].numel() / std::max<int64_t>(B, 1) * dst[k].element_size();
            fs.f[k] = TbField{src[k].data_ptr(), dst[k].data_ptr(), static_cast<int>(rb)};
          }
          cuda_ok(tb_ring_gather(fs, static_cast<int>(src.size()), static_cast<int>(B), idx.data_ptr<int>(),
                                 stream_of(idx)),
                  "ring_gather");
        });

  m.def("per_update",
        [](at::Tensor tree, at::Tensor idx, at::Tensor prio, float alpha, float eps, int64_t capacity) {
          need(tree, at::kFloat, "tree");
          need(idx, at::kLong, "idx");
          need(prio, at::kFloat, "prio");
          const int64_t L = tree.numel() / 2;
          cuda_ok(tb_per_update(tree.data_ptr<float>(), L, reinterpret_cast<const long long*>(idx.data_ptr<int64_t>()), prio.data_ptr<float>(),
                                static_cast<int>(idx.numel()), alpha, eps, capacity, nullptr, stream_of(tree)),
                  "per_update");
        });

  m.def("per_rebuild", [](at::Tensor tree) {
    need(tree, at::kFloat, "tree");
    cuda_ok(tb_per_rebuild(tree.data_ptr<float>(), tree.numel() / 2, stream_of(tree)), "per_rebuild");
  });

  m.def("per_sample",
        [](at::Tensor tree, int64_t size, int64_t n, float beta, uint64_t seed, uint64_t counter) {
          need(tree, at::kFloat, "tree");
          auto o = tree.options();
          at::Tensor idx = at::empty({n}, o.dtype(at::kLong));
          at::Tensor w = at::empty({n}, o.dtype(at::kFloat));
          at::Tensor p = at::empty({n}, o.dtype(at::kFloat));
          at::Tensor mx = at::empty({1}, o.dtype(at::kInt));
          cuda_ok(tb_per_sample(tree.data_ptr<float>(), tree.numel() / 2, size, static_cast<int>(n), beta, seed,
                                counter, reinterpret_cast<long long*>(idx.data_ptr<int64_t>()), w.data_ptr<float>(), p.data_ptr<float>(),
                                reinterpret_cast<unsigned*>(mx.data_ptr<int>()), stream_of(tree)),
                  "per_sample");
          return py::make_tuple(idx, w, p);
        });

  // ---------------- advantages ----------------
  m.def("gae_scratch_numel", [](int T, int N) { return static_cast<int64_t>(tb_gae_scratch_bytes(T, N) / 4); });
  m.def("gae",
        [](at::Tensor rew, at::Tensor val, at::Tensor done, at::Tensor adv, at::Tensor ret, py::object stats,
           py::object scratch, float gamma, float lam) {
          need(rew, at::kFloat, "rewards");
          need(val, at::kFloat, "values");
          need(adv, at::kFloat, "advantages");
          need(ret, at::kFloat, "returns");
          TB_CHECK(done.is_cuda() && done.element_size() == 1 && done.is_contiguous(), "done must be bool/u8");
          TB_CHECK(rew.dim() == 2, "rewards must be [T, N]");
          const int T = static_cast<int>(rew.size(0)), N = static_cast<int>(rew.size(1));
          TB_CHECK(val.numel() == static_cast<int64_t>(T + 1) * N, "values must be [T+1, N]");
          TB_CHECK(done.numel() == static_cast<int64_t>(T) * N && adv.numel() == rew.numel() &&
                       ret.numel() == rew.numel(),
                   "shape mismatch");
          double* sp = nullptr;
          if (!stats.is_none()) {
            at::Tensor s = stats.cast<at::Tensor>();
            need(s, at::kDouble, "stats");
            sp = s.data_ptr<double>();
          }
          at::Tensor scr;
          const size_t need_bytes = tb_gae_scratch_bytes(T, N);
          if (need_bytes > 0) {
            if (!scratch.is_none()) {
              scr = scratch.cast<at::Tensor>();
              need(scr, at::kFloat, "scratch");
              TB_CHECK(static_cast<size_t>(scr.numel()) * 4 >= need_bytes, "scratch too small");
            } else {
              scr = at::empty({static_cast<int64_t>(need_bytes / 4)}, rew.options());
            }
          }
          cuda_ok(tb_gae(rew.data_ptr<float>(), val.data_ptr<float>(), static_cast<const uint8_t*>(done.data_ptr()),
                         adv.data_ptr<float>(), ret.data_ptr<float>(), sp,
                         scr.defined() ? scr.data_ptr<float>() : nullptr, T, N, gamma, lam, stream_of(rew)),
                  "gae");
        },
        py::arg("rewards"), py::arg("values"), py::arg("dones"), py::arg("advantages"), py::arg("returns"),
        py::arg("stats") = py::none(), py::arg("scratch") = py::none(), py::arg("gamma") = 0.99f,
        py::arg("lam") = 0.95f);

  m.def("grpo_advantage",
        [](at::Tensor rewards, int G, float eps, bool scale_by_std) {
          need(rewards, at::kFloat, "rewards");
          TB_CHECK(G > 0 && rewards.numel() % G == 0, "rewards must be a multiple of the group size");
          at::Tensor adv = at::empty_like(rewards);
          cuda_ok(tb_grpo_advantage(rewards.data_ptr<float>(), adv.data_ptr<float>(),
                                    static_cast<int>(rewards.numel() / G), G, eps, scale_by_std ? 1 : 0,
                                    stream_of(rewards)),
                  "grpo_advantage");
          return adv;
        },
        py::arg("rewards"), py::arg("group_size"), py::arg("eps") = 1e-4f, py::arg("scale_by_std") = true);

  // ---------------- PPO ----------------
  m.def("ppo_gather",
        [](at::Tensor obs, at::Tensor act, at::Tensor logp, at::Tensor adv, at::Tensor ret, at::Tensor val,
           py::object adv_stats, at::Tensor o_obs, at::Tensor o_act, at::Tensor o_logp, at::Tensor o_adv,
           at::Tensor o_ret, py::object o_val, int n_mb, py::object step_ptr, py::object iter_ptr, int64_t step,
           uint64_t seed, bool normalize, py::object o_obs_bf16) {
          need(obs, at::kFloat, "obs");
          need(act, at::kInt, "act");
          const int total = static_cast<int>(act.numel());
          const int obs_dim = static_cast<int>(obs.numel() / total);
          const int mb = static_cast<int>(o_act.numel());
          const double* sp = nullptr;
          if (!adv_stats.is_none()) sp = adv_stats.cast<at::Tensor>().data_ptr<double>();
          float* ov = o_val.is_none() ? nullptr : o_val.cast<at::Tensor>().data_ptr<float>();
          void* ob = o_obs_bf16.is_none() ? nullptr : o_obs_bf16.cast<at::Tensor>().data_ptr();
          float* oo = o_obs.numel() > 0 ? o_obs.data_ptr<float>() : nullptr;
          const long long* stp = step_ptr.is_none()
                                     ? nullptr
                                     : reinterpret_cast<const long long*>(step_ptr.cast<at::Tensor>().data_ptr<int64_t>());
          const long long* itp = iter_ptr.is_none()
                                     ? nullptr
                                     : reinterpret_cast<const long long*>(iter_ptr.cast<at::Tensor>().data_ptr<int64_t>());
          cuda_ok(tb_ppo_gather(obs.data_ptr<float>(), obs_dim, act.data_ptr<int>(), logp.data_ptr<float>(),
                                adv.data_ptr<float>(), ret.data_ptr<float>(), val.data_ptr<float>(), sp,
                                oo, o_act.data_ptr<int>(), o_logp.data_ptr<float>(), o_adv.data_ptr<float>(),
                                o_ret.data_ptr<float>(), ov, ob, total, mb, n_mb, stp, itp, step, seed,
                                normalize ? 1 : 0, stream_of(obs)),
                  "ppo_gather");
        },
        py::arg("obs"), py::arg("act"), py::arg("logp"), py::arg("adv"), py::arg("ret"), py::arg("val"),
        py::arg("adv_stats"), py::arg("o_obs"), py::arg("o_act"), py::arg("o_logp"), py::arg("o_adv"),
        py::arg("o_ret"), py::arg("o_val"), py::arg("n_mb"), py::arg("step_ptr"), py::arg("iter_ptr"),
        py::arg("step"), py::arg("seed"), py::arg("normalize"), py::arg("o_obs_bf16") = py::none());

  m.def("ppo_loss_padded",
        [](at::Tensor logits, int A, at::Tensor value, at::Tensor act, at::Tensor old_logp, at::Tensor adv,
           at::Tensor ret, at::Tensor dlog, at::Tensor dval, py::object stats, float clip, float vf_coef,
           float ent_coef, py::object db_log, py::object db_val) {
          // logits / value / dlog / dval may be column blocks of wider row-major buffers
          auto rows = [](const at::Tensor& t, at::ScalarType dt, const char* n) {
            TB_CHECK(t.is_cuda() && t.scalar_type() == dt && t.dim() == 2 && t.stride(1) == 1, n);
          };
          rows(logits, at::kFloat, "logits: fp32 [B, >=A] with unit column stride");
          rows(value, at::kFloat, "value: fp32 [B, >=1] with unit column stride");
          rows(dlog, at::kBFloat16, "dlog: bf16 [B, 8] with unit column stride");
          rows(dval, at::kBFloat16, "dval: bf16 [B, 8] with unit column stride");
          need(act, at::kInt, "act");
          const int B = static_cast<int>(act.numel());
          TB_CHECK(logits.size(0) == B && dlog.size(0) == B && dval.size(0) == B && dlog.size(1) >= 8 &&
                       dval.size(1) >= 8 && dlog.stride(0) == dval.stride(0), "padded loss shapes");
          float* sp = stats.is_none() ? nullptr : stats.cast<at::Tensor>().data_ptr<float>();
          cuda_ok(tb_ppo_loss_padded(logits.data_ptr<float>(), static_cast<int>(logits.stride(0)), A,
                                     value.data_ptr<float>(), static_cast<int>(value.stride(0)), act.data_ptr<int>(),
                                     old_logp.data_ptr<float>(), adv.data_ptr<float>(), ret.data_ptr<float>(),
                                     dlog.data_ptr(), dval.data_ptr(), static_cast<int>(dlog.stride(0)), sp, B, clip,
                                     vf_coef, ent_coef,
                                     db_log.is_none() ? nullptr : db_log.cast<at::Tensor>().data_ptr<float>(),
                                     db_val.is_none() ? nullptr : db_val.cast<at::Tensor>().data_ptr<float>(),
                                     stream_of(logits)),
                  "ppo_loss_padded");
        },
        py::arg("logits"), py::arg("A"), py::arg("value"), py::arg("act"), py::arg("old_logp"), py::arg("adv"),
        py::arg("ret"), py::arg("dlog"), py::arg("dval"), py::arg("stats"), py::arg("clip"), py::arg("vf_coef"),
        py::arg("ent_coef"), py::arg("db_log") = py::none(), py::arg("db_val") = py::none());

  m.def("colsum_bf16", [](at::Tensor x, at::Tensor out, bool accumulate) {
    TB_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "colsum: bf16 2-D");
    need(out, at::kFloat, "out");
    TB_CHECK(out.numel() == x.size(1), "colsum: out [cols]");
    cuda_ok(tb_colsum_bf16(x.data_ptr(), x.stride(0), static_cast<int>(x.size(0)), static_cast<int>(x.size(1)),
                           out.data_ptr<float>(), accumulate ? 1 : 0, stream_of(x)),
            "colsum_bf16");
  }, py::arg("x"), py::arg("out"), py::arg("accumulate") = false);

  m.def(
      "lin_gauss_act",
      [](at::Tensor x, at::Tensor params, at::Tensor act, at::Tensor logp, int O, int A, float stdv, uint64_t seed,
         uint32_t counter) {
        need(x, at::kFloat, "x");
        need(params, at::kFloat, "params");
        need(act, at::kFloat, "act");
        need(logp, at::kFloat, "logp");
        TB_CHECK(x.numel() % O == 0 && act.numel() == x.numel() / O * A && logp.numel() == x.numel() / O,
                 "lin_gauss_act: shapes");
        cuda_ok(tb_lin_gauss_act(x.data_ptr<float>(), params.data_ptr<float>(), act.data_ptr<float>(),
                                 logp.data_ptr<float>(), static_cast<int>(x.numel() / O), O, A, stdv, seed, counter,
                                 stream_of(x)),
                "lin_gauss_act");
      },
      py::arg("x"), py::arg("params"), py::arg("act"), py::arg("logp"), py::arg("O"), py::arg("A"), py::arg("std"),
      py::arg("seed"), py::arg("counter"));
  m.def(
      "lin_gauss_grad",
      [](at::Tensor batch, at::Tensor params, at::Tensor grad, int O, int A, float stdv, float clip, float vf_coef,
         bool has_old) {
        need(batch, at::kFloat, "batch");
        need(params, at::kFloat, "params");
        need(grad, at::kFloat, "grad");
        TB_CHECK(batch.dim() == 2, "lin_gauss_grad: batch [N, row]");
        cuda_ok(tb_lin_gauss_grad(batch.data_ptr<float>(), static_cast<int>(batch.size(1)), params.data_ptr<float>(),
                                  grad.data_ptr<float>(), static_cast<int>(batch.size(0)), O, A, stdv, clip, vf_coef,
                                  has_old ? 1 : 0, stream_of(batch)),
                "lin_gauss_grad");
      },
      py::arg("batch"), py::arg("params"), py::arg("grad"), py::arg("O"), py::arg("A"), py::arg("std"),
      py::arg("clip"), py::arg("vf_coef"), py::arg("has_old"));

  m.def("dense_k8_fwd", [](at::Tensor x, at::Tensor W, py::object bias, at::Tensor y, bool tanh_act, int rows) {
    TB_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.size(1) == 8 && x.stride(1) == 1,
             "dense_k8_fwd: x bf16 [M, 8]");
    TB_CHECK(W.scalar_type() == at::kBFloat16 && W.is_contiguous() && W.dim() == 2 && W.size(1) == 8,
             "dense_k8_fwd: W bf16 [N, 8] contiguous");
    TB_CHECK(y.scalar_type() == at::kBFloat16 && y.dim() == 2 && y.size(0) == x.size(0) && y.size(1) == W.size(0) &&
                 y.stride(1) == 1, "dense_k8_fwd: y bf16 [M, N]");
    const float* bp = nullptr;
    at::Tensor bt;
    if (!bias.is_none()) {
      bt = bias.cast<at::Tensor>();
      need(bt, at::kFloat, "bias");
      bp = bt.data_ptr<float>();
    }
    cuda_ok(tb_dense_k8_fwd_rows(x.data_ptr(), x.stride(0), W.data_ptr(), bp, y.data_ptr(), y.stride(0),
                                 static_cast<int>(x.size(0)), static_cast<int>(W.size(0)), tanh_act ? 1 : 0, rows,
                                 stream_of(x)),
            "dense_k8_fwd");
  }, py::arg("x"), py::arg("W"), py::arg("bias"), py::arg("y"), py::arg("tanh") = true, py::arg("rows") = 0);
  m.def("ppo_head_parts", [](int H, int A) { return tb_ppo_head_default_parts(H, A); });
  m.def("ppo_head_part_numel", [](int H, int A, int parts) { return static_cast<int64_t>(tb_ppo_head_part_numel(H, A, parts)); });
  // fused output layer + clipped PPO loss + output-layer backward (see ppo_head.cu)
  m.def("ppo_head", [](at::Tensor h2, at::Tensor W3, at::Tensor b3, int crow, int A, at::Tensor act, at::Tensor old_logp,
                       at::Tensor adv, at::Tensor ret, at::Tensor dz, at::Tensor g_w3, at::Tensor g_b3, at::Tensor g_b2,
                       py::object stats, at::Tensor part, int parts, float clip, float vf_coef, float ent_coef) {
    for (auto* t : {&h2, &W3, &dz})
      TB_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 2 && t->stride(1) == 1,
               "ppo_head: h2, W3, dz must be bf16 2-D CUDA tensors with a contiguous last dim");
    const int64_t M = h2.size(0), N = h2.size(1);
    TB_CHECK(N % 2 == 0 && dz.size(0) == M && dz.size(1) == N && W3.size(1) == N && W3.size(0) > crow,
             "ppo_head: h2/dz [M, 2H], W3 [> crow, 2H]");
    for (auto* t : {&b3, &g_w3, &g_b3, &g_b2, &old_logp, &adv, &ret, &part}) need(*t, at::kFloat, "ppo_head fp32 operand");
    need(act, at::kInt, "act");
    TB_CHECK(g_w3.dim() == 2 && g_w3.size(1) == N && g_w3.size(0) > crow && g_w3.stride(1) == 1 && g_b2.numel() == N &&
                 g_b3.numel() > crow && b3.numel() > crow && act.numel() >= M && old_logp.numel() >= M &&
                 adv.numel() >= M && ret.numel() >= M,
             "ppo_head: gradient / input shapes");
    TB_CHECK(part.numel() >= tb_ppo_head_part_numel(static_cast<int>(N / 2), A, parts), "ppo_head: part too small");
    float* sp = nullptr;
    if (!stats.is_none()) {
      at::Tensor st = stats.cast<at::Tensor>();
      need(st, at::kFloat, "stats");
      TB_CHECK(st.numel() >= 6, "ppo_head: stats [>= 6]");
      sp = st.data_ptr<float>();
    }
    TbPpoHeadArgs a{};
    a.H2 = h2.data_ptr();
    a.ldh = h2.stride(0);
    a.W3 = W3.data_ptr();
    a.ldw = W3.stride(0);
    a.b3 = b3.data_ptr<float>();
    a.crow = crow;
    a.act = act.data_ptr<int>();
    a.old_logp = old_logp.data_ptr<float>();
    a.adv = adv.data_ptr<float>();
    a.ret = ret.data_ptr<float>();
    a.dz = dz.data_ptr();
    a.ldz = dz.stride(0);
    a.g_w3 = g_w3.data_ptr<float>();
    a.ldgw = g_w3.stride(0);
    a.g_b3 = g_b3.data_ptr<float>();
    a.g_b2 = g_b2.data_ptr<float>();
    a.stats = sp;
    a.part = part.data_ptr<float>();
    a.parts = parts;
    a.M = static_cast<int>(M);
    a.H = static_cast<int>(N / 2);
    a.A = A;
    a.clip = clip;
    a.vf_coef = vf_coef;
    a.ent_coef = ent_coef;
    cuda_ok(tb_ppo_head(&a, stream_of(h2)), "ppo_head");
  }, py::arg("h2"), py::arg("W3"), py::arg("b3"), py::arg("crow"), py::arg("A"), py::arg("act"), py::arg("old_logp"),
     py::arg("adv"), py::arg("ret"), py::arg("dz"), py::arg("g_w3"), py::arg("g_b3"), py::arg("g_b2"),
     py::arg("stats"), py::arg("part"), py::arg("parts"), py::arg("clip"), py::arg("vf_coef"), py::arg("ent_coef"));
  m.def("skinny8_scratch_numel", [](int N) { return static_cast<int64_t>(tb_skinny8_scratch_floats(N)); });
  // out (fp32, contiguous) = A^T X for 8-wide X blocks (+= with accumulate); scratch fp32 per-CTA partials
  m.def("skinny8_wgrad", [](at::Tensor A, at::Tensor X, at::Tensor out, int xblock, int64_t os_j, int64_t os_k,
                            int64_t os_blk, bool accumulate, at::Tensor scratch) {
    TB_CHECK(A.is_cuda() && A.scalar_type() == at::kBFloat16 && A.dim() == 2 && A.stride(1) == 1,
             "skinny8_wgrad: A bf16 [M, N]");
    TB_CHECK(X.is_cuda() && X.scalar_type() == at::kBFloat16 && X.dim() == 2 && X.stride(1) == 1 &&
                 X.size(0) == A.size(0) && xblock > 0 && A.size(1) % xblock == 0 &&
                 X.size(1) >= 8 * (A.size(1) / xblock),
             "skinny8_wgrad: X bf16 [M, 8 * N / xblock]");
    need(out, at::kFloat, "out");
    need(scratch, at::kFloat, "scratch");
    TB_CHECK(out.is_contiguous() && scratch.is_contiguous(), "skinny8_wgrad: contiguous out and scratch");
    const int64_t N = A.size(1), nb = N / xblock;
    const int64_t last = (N - 1) * os_j + 7 * os_k + (nb - 1) * os_blk;
    TB_CHECK(os_j >= 0 && os_k >= 0 && os_blk >= 0 && last < out.numel(), "skinny8_wgrad: out too small");
    cuda_ok(tb_skinny8_wgrad(A.data_ptr(), A.stride(0), X.data_ptr(), X.stride(0), xblock, out.data_ptr<float>(), os_j,
                             os_k, os_blk, static_cast<int>(A.size(0)), static_cast<int>(N), accumulate ? 1 : 0,
                             scratch.data_ptr<float>(), static_cast<size_t>(scratch.numel()), stream_of(A)),
            "skinny8_wgrad");
  }, py::arg("A"), py::arg("X"), py::arg("out"), py::arg("xblock"), py::arg("os_j"), py::arg("os_k"),
     py::arg("os_blk"), py::arg("accumulate"), py::arg("scratch"));
  // dz = (dout W per head) * (1 - h^2); db (fp32 [N]) = column sums of dz (+= with accumulate)
  m.def("mlp_head_dz", [](at::Tensor dout, at::Tensor h, at::Tensor W, int xblock, at::Tensor dz, at::Tensor db,
                          bool accumulate, at::Tensor scratch) {
    for (auto* t : {&dout, &h, &W, &dz})
      TB_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 2 && t->stride(1) == 1,
               "mlp_head_dz: bf16 2-D CUDA tensors with a contiguous last dim");
    const int64_t M = h.size(0), N = h.size(1);
    TB_CHECK(xblock > 0 && N % xblock == 0 && dz.size(0) == M && dz.size(1) == N && dout.size(0) == M &&
                 dout.size(1) >= 8 * (N / xblock) && W.size(0) >= 8 * (N / xblock) && W.size(1) == N,
             "mlp_head_dz: shapes (dout [M, 8 heads], h/dz [M, N], W [8 heads, N])");
    need(db, at::kFloat, "db");
    need(scratch, at::kFloat, "scratch");
    TB_CHECK(db.is_contiguous() && db.numel() == N && scratch.is_contiguous(), "mlp_head_dz: db fp32 [N]");
    cuda_ok(tb_mlp_head_dz(dout.data_ptr(), dout.stride(0), h.data_ptr(), h.stride(0), W.data_ptr(), W.stride(0),
                           xblock, dz.data_ptr(), dz.stride(0), db.data_ptr<float>(), static_cast<int>(M),
                           static_cast<int>(N), accumulate ? 1 : 0, scratch.data_ptr<float>(),
                           static_cast<size_t>(scratch.numel()), stream_of(h)),
            "mlp_head_dz");
  }, py::arg("dout"), py::arg("h"), py::arg("W"), py::arg("xblock"), py::arg("dz"), py::arg("db"),
     py::arg("accumulate"), py::arg("scratch"));
  // out (fp32 [M, >= 8 heads]) = h W^T + bias per head (8 outputs per head, xblock hidden columns each)
  m.def("mlp_head_fwd", [](at::Tensor h, at::Tensor W, py::object bias, int xblock, at::Tensor out) {
    TB_CHECK(h.is_cuda() && h.scalar_type() == at::kBFloat16 && h.dim() == 2 && h.stride(1) == 1 &&
                 W.scalar_type() == at::kBFloat16 && W.dim() == 2 && W.stride(1) == 1 && W.size(1) == h.size(1) &&
                 xblock > 0 && h.size(1) % xblock == 0,
             "mlp_head_fwd: h bf16 [M, N], W bf16 [8 heads, N]");
    const int heads = static_cast<int>(h.size(1) / xblock);
    TB_CHECK(W.size(0) >= 8 * heads, "mlp_head_fwd: W needs 8 rows per head");
    need(out, at::kFloat, "out");
    TB_CHECK(out.dim() == 2 && out.stride(1) == 1 && out.size(0) == h.size(0) && out.size(1) >= 8 * heads,
             "mlp_head_fwd: out fp32 [M, 8 heads]");
    const float* b = nullptr;
    at::Tensor bt;
    if (!bias.is_none()) {
      bt = bias.cast<at::Tensor>();
      need(bt, at::kFloat, "bias");
      TB_CHECK(bt.numel() >= 8 * heads, "mlp_head_fwd: bias fp32 [8 heads]");
      b = bt.data_ptr<float>();
    }
    cuda_ok(tb_mlp_head_fwd(h.data_ptr(), h.stride(0), W.data_ptr(), W.stride(0), b, out.data_ptr<float>(),
                            out.stride(0), xblock, heads, static_cast<int>(h.size(0)), stream_of(h)),
            "mlp_head_fwd");
  }, py::arg("h"), py::arg("W"), py::arg("bias"), py::arg("xblock"), py::arg("out"));
  m.def("dense_k8_wgrad", [](at::Tensor dz, at::Tensor x, at::Tensor dW, bool accumulate) {
    TB_CHECK(dz.is_cuda() && dz.scalar_type() == at::kBFloat16 && dz.dim() == 2 && dz.stride(1) == 1,
             "dense_k8_wgrad: dz bf16 [M, N]");
    TB_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.size(1) == 8 && x.size(0) == dz.size(0) &&
                 x.stride(1) == 1, "dense_k8_wgrad: x bf16 [M, 8]");
    need(dW, at::kFloat, "dW");
    TB_CHECK(dW.numel() == dz.size(1) * 8, "dense_k8_wgrad: dW fp32 [N, 8]");
    cuda_ok(tb_dense_k8_wgrad(dz.data_ptr(), dz.stride(0), x.data_ptr(), x.stride(0), dW.data_ptr<float>(),
                              static_cast<int>(dz.size(0)), static_cast<int>(dz.size(1)), accumulate ? 1 : 0,
                              stream_of(dz)),
            "dense_k8_wgrad");
  }, py::arg("dz"), py::arg("x"), py::arg("dW"), py::arg("accumulate") = false);

  m.def("ppo_loss",
        [](at::Tensor logits, at::Tensor value, at::Tensor act, at::Tensor old_logp, at::Tensor adv, at::Tensor ret,
           py::object old_val, at::Tensor dlogits, at::Tensor dvalue, py::object stats, float clip, float vclip,
           float vf_coef, float ent_coef) {
          need(logits, at::kFloat, "logits");
          need(value, at::kFloat, "value");
          need(act, at::kInt, "act");
          need(dlogits, at::kFloat, "dlogits");
          need(dvalue, at::kFloat, "dvalue");
          const int B = static_cast<int>(act.numel());
          const int A = static_cast<int>(logits.numel() / B);
          const float* ov = old_val.is_none() ? nullptr : old_val.cast<at::Tensor>().data_ptr<float>();
          float* sp = stats.is_none() ? nullptr : stats.cast<at::Tensor>().data_ptr<float>();
          cuda_ok(tb_ppo_loss(logits.data_ptr<float>(), A, value.data_ptr<float>(), act.data_ptr<int>(),
                              old_logp.data_ptr<float>(), adv.data_ptr<float>(), ret.data_ptr<float>(), ov,
                              dlogits.data_ptr<float>(), dvalue.data_ptr<float>(), sp, B, clip, vclip, vf_coef,
                              ent_coef, stream_of(logits)),
                  "ppo_loss");
        });

  m.def("counter_add", [](at::Tensor c, int64_t v) {
    need(c, at::kLong, "counter");
    cuda_ok(tb_counter_add(reinterpret_cast<long long*>(c.data_ptr<int64_t>()), v, stream_of(c)), "counter_add");
  });

  // ---------------- optimizer / elementwise ----------------
  m.def("adam",
        [](at::Tensor p, at::Tensor g, at::Tensor m1, at::Tensor m2, py::object p_bf16, float lr, float b1, float b2,
           float eps, float wd, float grad_scale, float max_norm, py::object step_ptr, int64_t step,
           py::object gnorm_sq) {
          need(p, at::kFloat, "param");
          need(g, at::kFloat, "grad");
          need(m1, at::kFloat, "exp_avg");
          need(m2, at::kFloat, "exp_avg_sq");
          TB_CHECK(g.numel() == p.numel() && m1.numel() == p.numel() && m2.numel() == p.numel(), "adam sizes");
          void* pb = nullptr;
          if (!p_bf16.is_none()) {
            at::Tensor b = p_bf16.cast<at::Tensor>();
            need(b, at::kBFloat16, "p_bf16");
            TB_CHECK(b.numel() == p.numel(), "p_bf16 size");
            pb = b.data_ptr();
          }
          const long long* sp = step_ptr.is_none()
                                    ? nullptr
                                    : reinterpret_cast<const long long*>(step_ptr.cast<at::Tensor>().data_ptr<int64_t>());
          const float* gn = gnorm_sq.is_none() ? nullptr : gnorm_sq.cast<at::Tensor>().data_ptr<float>();
          TbAdamParams hp{lr, b1, b2, eps, wd, grad_scale, max_norm, step};
          cuda_ok(tb_adam(p.data_ptr<float>(), g.data_ptr<float>(), m1.data_ptr<float>(), m2.data_ptr<float>(), pb,
                          p.numel(), hp, sp, gn, stream_of(p)),
                  "adam");
        },
        py::arg("param"), py::arg("grad"), py::arg("exp_avg"), py::arg("exp_avg_sq"), py::arg("param_bf16") = py::none(),
        py::arg("lr") = 3e-4f, py::arg("beta1") = 0.9f, py::arg("beta2") = 0.999f, py::arg("eps") = 1e-8f,
        py::arg("weight_decay") = 0.0f, py::arg("grad_scale") = 1.0f, py::arg("max_grad_norm") = 0.0f,
        py::arg("step_ptr") = py::none(), py::arg("step") = 0, py::arg("gnorm_sq") = py::none());

  m.def("sumsq", [](at::Tensor x, at::Tensor out) {
    need(x, at::kFloat, "x");
    need(out, at::kFloat, "out");
    cuda_ok(tb_sumsq(x.data_ptr<float>(), x.numel(), out.data_ptr<float>(), stream_of(x)), "sumsq");
  });

  m.def("elementwise",
        [](at::Tensor out, py::object x, py::object y, float a, int op) {
          need(out, at::kFloat, "out");
          const float* xp = x.is_none() ? nullptr : x.cast<at::Tensor>().data_ptr<float>();
          const float* yp = y.is_none() ? nullptr : y.cast<at::Tensor>().data_ptr<float>();
          cuda_ok(tb_elementwise(out.data_ptr<float>(), xp, yp, out.numel(), a, op, stream_of(out)), "elementwise");
        });

  // ---------------- rewards ----------------
  m.def("hash_reward", [](at::Tensor ids, at::Tensor lens) {
    need(ids, at::kInt, "ids");
    need(lens, at::kInt, "lens");
    at::Tensor out = at::empty({ids.size(0)}, ids.options().dtype(at::kFloat));
    cuda_ok(tb_hash_reward(ids.data_ptr<int>(), lens.data_ptr<int>(), static_cast<int>(ids.size(0)),
                           static_cast<int>(ids.size(1)), out.data_ptr<float>(), stream_of(ids)),
            "hash_reward");
    return out;
  });
}
