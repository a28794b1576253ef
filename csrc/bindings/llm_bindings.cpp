// torch-tensor entry points of the tensor-core GEMM and the LLM kernels.
#include <pybind11/pybind11.h>
#include <torch/extension.h>

#include "kernels.h"
#include "turbol/common.hpp"

namespace py = pybind11;

namespace {

void chk(bool c, const std::string& m) {
  if (!c) throw std::invalid_argument(m);
}
void cuda_ok(int e, const char* what) {
  if (e != 0) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(static_cast<cudaError_t>(e)));
}

// C = epi(A . B^T) with A [M,K] (a_mn=0) or [K,M] (a_mn=1), B [N,K] (b_mn=0) or [K,N] (b_mn=1).
void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor C, bool a_mn, bool b_mn, py::object bias,
          py::object aux, int epi, bool accumulate, float alpha, int split_k, int bn, py::object err,
          py::object workspace, py::object colsum, py::object c2, int kgroup) {
  chk(A.is_cuda() && B.is_cuda() && C.is_cuda(), "gemm: CUDA tensors required");
  chk(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm: A and B must be bfloat16");
  chk(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "gemm: 2-D operands");
  chk(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "gemm: last dim must be contiguous");
  const int64_t M = a_mn ? A.size(1) : A.size(0);
  const int64_t K = a_mn ? A.size(0) : A.size(1);
  // kgroup with B's inner dimension one block wide: B holds only the diagonal
  // blocks, packed side by side (then N == K, the outer dimension of B)
  const bool packed = kgroup > 0 && B.size(1) == kgroup && B.size(0) == K && K > kgroup;
  const int64_t N = packed ? K : (b_mn ? B.size(1) : B.size(0));
  const int64_t Kb = packed ? K : (b_mn ? B.size(0) : B.size(1));
  chk(K == Kb, "gemm: K mismatch");
  const int64_t nc = epi == TB_EPI_SWIGLU ? N / 2 : (epi == TB_EPI_SWIGLU_BWD ? 2 * N : N);
  chk(C.size(0) == M && C.size(1) == nc, "gemm: C shape mismatch");
  chk(C.scalar_type() == at::kFloat || C.scalar_type() == at::kBFloat16, "gemm: C must be fp32 or bf16");
  TbGemmArgs a{};
  a.A = A.data_ptr();
  a.lda = A.stride(0);
  a.a_mn = a_mn;
  a.B = B.data_ptr();
  a.ldb = B.stride(0);
  a.b_mn = b_mn;
  a.C = C.data_ptr();
  a.ldc = C.stride(0);
  a.c_fp32 = C.scalar_type() == at::kFloat;
  a.c_accumulate = accumulate;
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  at::Tensor b, x;
  if (!bias.is_none()) {
    b = bias.cast<at::Tensor>();
    chk(b.scalar_type() == at::kFloat && b.is_contiguous() && b.numel() == N, "gemm: bias must be fp32 [N]");
    a.bias = b.data_ptr<float>();
  }
  if (!aux.is_none()) {
    x = aux.cast<at::Tensor>();
    chk(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1 && x.size(0) == M &&
            x.size(1) == (epi == TB_EPI_SWIGLU_BWD ? 2 * N : N),
        "gemm: aux must be bf16 [M, N] ([M, 2N] interleaved gate/up for EPI_SWIGLU_BWD)");
    a.aux = x.data_ptr();
    a.ld_aux = x.stride(0);
  }
  a.epi = epi;
  a.alpha = alpha;
  a.split_k = split_k;
  a.bn_hint = bn;
  a.kgroup = kgroup;
  a.kgroup_packed = packed ? 1 : 0;
  if (!err.is_none()) a.error = err.cast<at::Tensor>().data_ptr<int>();
  at::Tensor ws, cs;
  if (!workspace.is_none()) {
    ws = workspace.cast<at::Tensor>();
    chk(ws.is_cuda() && ws.is_contiguous(), "gemm: workspace must be a contiguous CUDA tensor");
    a.workspace = ws.data_ptr();
    a.workspace_bytes = ws.nbytes();
  }
  if (!colsum.is_none()) {
    cs = colsum.cast<at::Tensor>();
    chk(cs.scalar_type() == at::kFloat && cs.is_contiguous() && cs.numel() == N, "gemm: colsum must be fp32 [N]");
    a.colsum = cs.data_ptr<float>();
  }
  at::Tensor raw;
  if (!c2.is_none()) {
    raw = c2.cast<at::Tensor>();
    chk(epi == TB_EPI_SWIGLU && raw.is_cuda() && raw.scalar_type() == at::kBFloat16 && raw.dim() == 2 &&
            raw.stride(1) == 1 && raw.size(0) == M && raw.size(1) == N,
        "gemm: c2 (EPI_SWIGLU only) must be bf16 [M, N]");
    a.C2 = raw.data_ptr();
    a.ldc2 = raw.stride(0);
  }
  cuda_ok(tb_gemm_bf16(&a, turbol::StreamFor(C)), "gemm_bf16");
}

// Decode-shaped GEMM (few tokens, weight-stationary, cluster split-K).
void gemm_decode(const at::Tensor& X, const at::Tensor& W, at::Tensor C, py::object bias, py::object aux, int epi,
                 int splits, py::object err) {
  chk(X.is_cuda() && W.is_cuda() && C.is_cuda(), "gemm_decode: CUDA tensors required");
  chk(X.scalar_type() == at::kBFloat16 && W.scalar_type() == at::kBFloat16 && C.scalar_type() == at::kBFloat16,
      "gemm_decode: bf16 X, W and C");
  chk(X.dim() == 2 && W.dim() == 2 && C.dim() == 2 && X.stride(1) == 1 && W.stride(1) == 1 && C.stride(1) == 1,
      "gemm_decode: 2-D operands with a contiguous last dim");
  chk(X.size(1) == W.size(1), "gemm_decode: K mismatch");
  const int64_t T = X.size(0), N = W.size(0);
  chk(C.size(0) == T && C.size(1) == (epi == TB_EPI_SWIGLU ? N / 2 : N), "gemm_decode: C shape mismatch");
  TbDecodeGemmArgs a{};
  a.X = X.data_ptr();
  a.ldx = X.stride(0);
  a.W = W.data_ptr();
  a.ldw = W.stride(0);
  a.C = C.data_ptr();
  a.ldc = C.stride(0);
  a.T = static_cast<int>(T);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(X.size(1));
  a.epi = epi;
  a.splits = splits;
  at::Tensor b, x;
  if (!bias.is_none()) {
    b = bias.cast<at::Tensor>();
    chk(b.is_cuda() && b.scalar_type() == at::kFloat && b.is_contiguous() && b.numel() == N,
        "gemm_decode: bias must be fp32 [N]");
    a.bias = b.data_ptr<float>();
  }
  if (!aux.is_none()) {
    x = aux.cast<at::Tensor>();
    chk(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1 && x.size(0) == T &&
            x.size(1) == N,
        "gemm_decode: aux must be bf16 [T, N]");
    a.aux = x.data_ptr();
    a.ld_aux = x.stride(0);
  }
  if (!err.is_none()) a.error = err.cast<at::Tensor>().data_ptr<int>();
  cuda_ok(tb_gemm_decode(&a, turbol::StreamFor(C)), "gemm_decode");
}

}  // namespace

void register_llm_ops(py::module_& m) {
  m.def("gemm_decode", &gemm_decode, py::arg("X"), py::arg("W"), py::arg("C"), py::arg("bias") = py::none(),
        py::arg("aux") = py::none(), py::arg("epi") = 0, py::arg("splits") = 0, py::arg("error") = py::none(),
        "C = epi(X W^T) for few tokens: weight-stationary tcgen05 GEMM, K split over a cluster");
  m.def("gemm_decode_splits", &tb_gemm_decode_splits, py::arg("T"), py::arg("N"), py::arg("K"));
  m.def("gemm", &gemm, py::arg("A"), py::arg("B"), py::arg("C"), py::arg("a_mn") = false, py::arg("b_mn") = false,
        py::arg("bias") = py::none(), py::arg("aux") = py::none(), py::arg("epi") = 0, py::arg("accumulate") = false,
        py::arg("alpha") = 1.0f, py::arg("split_k") = 0, py::arg("bn") = 0, py::arg("error") = py::none(),
        py::arg("workspace") = py::none(), py::arg("colsum") = py::none(), py::arg("c2") = py::none(),
        py::arg("kgroup") = 0);
  m.def("gemm_workspace_numel", [](int M, int N, int K) {
    return static_cast<int64_t>(tb_gemm_workspace_bytes(M, N, K) / 4);
  });
  // ---------------- transformer ops (all launch on the current stream) ----------------
  auto bf16_2d = [](const at::Tensor& t, const char* n) {
    chk(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.stride(1) == 1,
        std::string(n) + ": bf16 2-D CUDA tensor with contiguous rows");
  };
  auto f32c = [](const at::Tensor& t, const char* n) {
    chk(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous(), std::string(n) + ": contiguous fp32");
  };
  auto i32c = [](const at::Tensor& t, const char* n) {
    chk(t.is_cuda() && t.scalar_type() == at::kInt && t.is_contiguous(), std::string(n) + ": contiguous int32");
  };
  m.def("rmsnorm_fwd", [=](at::Tensor x, at::Tensor w, at::Tensor y, py::object rstd, float eps) {
    bf16_2d(x, "x");
    bf16_2d(y, "y");
    f32c(w, "w");
    chk(x.is_contiguous() && y.is_contiguous(), "rmsnorm: contiguous rows");
    float* r = rstd.is_none() ? nullptr : rstd.cast<at::Tensor>().data_ptr<float>();
    cuda_ok(tb_rmsnorm_fwd(x.data_ptr(), w.data_ptr<float>(), y.data_ptr(), r, static_cast<int>(x.size(0)),
                           static_cast<int>(x.size(1)), eps, turbol::StreamFor(x)),
            "rmsnorm_fwd");
  }, py::arg("x"), py::arg("w"), py::arg("y"), py::arg("rstd") = py::none(), py::arg("eps") = 1e-6f);
  m.def("rmsnorm_bwd_ws_numel", [](int D) { return static_cast<int64_t>(tb_rmsnorm_bwd_ws_floats(D)); });
  // ws (optional fp32, rmsnorm_bwd_ws_numel(D)): weight-gradient partials summed by a second pass
  m.def("rmsnorm_bwd", [=](at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd, at::Tensor dx,
                           py::object dx_add, at::Tensor dw, py::object ws) {
    bf16_2d(dy, "dy");
    bf16_2d(x, "x");
    bf16_2d(dx, "dx");
    f32c(w, "w");
    f32c(rstd, "rstd");
    f32c(dw, "dw");
    const void* add = dx_add.is_none() ? nullptr : dx_add.cast<at::Tensor>().data_ptr();
    float* wsp = nullptr;
    size_t wsn = 0;
    at::Tensor wst;
    if (!ws.is_none()) {
      wst = ws.cast<at::Tensor>();
      f32c(wst, "ws");
      wsp = wst.data_ptr<float>();
      wsn = static_cast<size_t>(wst.numel());
    }
    cuda_ok(tb_rmsnorm_bwd_ws(dy.data_ptr(), x.data_ptr(), w.data_ptr<float>(), rstd.data_ptr<float>(),
                              dx.data_ptr(), add, dw.data_ptr<float>(), static_cast<int>(x.size(0)),
                              static_cast<int>(x.size(1)), wsp, wsn, turbol::StreamFor(x)),
            "rmsnorm_bwd");
  }, py::arg("dy"), py::arg("x"), py::arg("w"), py::arg("rstd"), py::arg("dx"), py::arg("dx_add"), py::arg("dw"),
     py::arg("ws") = py::none());
  m.def("rope", [=](at::Tensor qkv, at::Tensor pos, at::Tensor table, int n_rot_heads, int head_dim, bool inverse) {
    bf16_2d(qkv, "qkv");
    i32c(pos, "pos");
    f32c(table, "table");
    chk(pos.numel() == qkv.size(0), "rope: one position per row");
    cuda_ok(tb_rope(qkv.data_ptr(), qkv.stride(0), pos.data_ptr<int>(), table.data_ptr<float>(),
                    static_cast<int>(qkv.size(0)), n_rot_heads, head_dim, inverse ? 1 : 0, turbol::StreamFor(qkv)),
            "rope");
  }, py::arg("qkv"), py::arg("pos"), py::arg("table"), py::arg("n_rot_heads"), py::arg("head_dim"),
     py::arg("inverse") = false);
  m.def("embed_fwd", [=](at::Tensor ids, at::Tensor W, at::Tensor out, py::object err) {
    i32c(ids, "ids");
    bf16_2d(W, "W");
    bf16_2d(out, "out");
    int* e = err.is_none() ? nullptr : err.cast<at::Tensor>().data_ptr<int>();
    cuda_ok(tb_embed_fwd(ids.data_ptr<int>(), W.data_ptr(), out.data_ptr(), static_cast<int>(ids.numel()),
                         static_cast<int>(W.size(1)), static_cast<int>(W.size(0)), e, turbol::StreamFor(ids)),
            "embed_fwd");
  }, py::arg("ids"), py::arg("W"), py::arg("out"), py::arg("error") = py::none());
  m.def("embed_bwd", [=](at::Tensor ids, at::Tensor dout, at::Tensor dW) {
    i32c(ids, "ids");
    bf16_2d(dout, "dout");
    f32c(dW, "dW");
    cuda_ok(tb_embed_bwd(ids.data_ptr<int>(), dout.data_ptr(), dW.data_ptr<float>(), static_cast<int>(ids.numel()),
                         static_cast<int>(dout.size(1)), static_cast<int>(dW.size(0)), turbol::StreamFor(ids)),
            "embed_bwd");
  });
  m.def("swiglu_bwd", [=](at::Tensor gu, at::Tensor dh, at::Tensor dgu) {
    bf16_2d(gu, "gu");
    bf16_2d(dh, "dh");
    bf16_2d(dgu, "dgu");
    chk(gu.is_contiguous() && dh.is_contiguous() && dgu.is_contiguous(), "swiglu_bwd: contiguous");
    cuda_ok(tb_swiglu_bwd(gu.data_ptr(), dh.data_ptr(), dgu.data_ptr(), gu.size(0), static_cast<int>(dh.size(1)),
                          turbol::StreamFor(gu)),
            "swiglu_bwd");
  });
  m.def("swiglu_fwd", [=](at::Tensor gu, at::Tensor act) {
    bf16_2d(gu, "gu");
    bf16_2d(act, "act");
    chk(gu.is_contiguous() && act.is_contiguous() && gu.size(1) == 2 * act.size(1), "swiglu_fwd: [T,2F] -> [T,F]");
    cuda_ok(tb_swiglu_fwd(gu.data_ptr(), act.data_ptr(), gu.size(0), static_cast<int>(act.size(1)),
                          turbol::StreamFor(gu)),
            "swiglu_fwd");
  });
  m.def("kv_write", [=](at::Tensor qkv, int k_off, int v_off, at::Tensor seq_of_token, at::Tensor pos,
                        at::Tensor block_table, at::Tensor kc, at::Tensor vc, int Hk, int D, int bs) {
    bf16_2d(qkv, "qkv");
    i32c(seq_of_token, "seq_of_token");
    i32c(pos, "pos");
    i32c(block_table, "block_table");
    cuda_ok(tb_kv_write(qkv.data_ptr(), qkv.stride(0), k_off, v_off, seq_of_token.data_ptr<int>(), pos.data_ptr<int>(),
                        block_table.data_ptr<int>(), static_cast<int>(block_table.size(1)), kc.data_ptr(),
                        vc.data_ptr(), static_cast<int>(qkv.size(0)), Hk, D, bs, turbol::StreamFor(qkv)),
            "kv_write");
  });
  m.def("rope_kv_write", [=](at::Tensor qkv, at::Tensor pos, at::Tensor table, int Hq, int Hk, int D,
                             at::Tensor seq_of_token, at::Tensor block_table, at::Tensor kc, at::Tensor vc, int bs) {
    bf16_2d(qkv, "qkv");
    i32c(pos, "pos");
    f32c(table, "table");
    i32c(seq_of_token, "seq_of_token");
    i32c(block_table, "block_table");
    chk(pos.numel() == qkv.size(0) && seq_of_token.numel() == qkv.size(0), "rope_kv_write: one position per row");
    chk(qkv.size(1) >= static_cast<int64_t>(Hq + 2 * Hk) * D, "rope_kv_write: qkv narrower than (Hq + 2 Hk) D");
    chk(kc.scalar_type() == at::kBFloat16 && vc.scalar_type() == at::kBFloat16 && kc.is_contiguous() &&
            vc.is_contiguous(), "rope_kv_write: bf16 contiguous caches");
    cuda_ok(tb_rope_kv_write(qkv.data_ptr(), qkv.stride(0), pos.data_ptr<int>(), table.data_ptr<float>(), Hq, Hk, D,
                             seq_of_token.data_ptr<int>(), block_table.data_ptr<int>(),
                             static_cast<int>(block_table.size(1)), kc.data_ptr(), vc.data_ptr(),
                             static_cast<int>(qkv.size(0)), bs, turbol::StreamFor(qkv)),
            "rope_kv_write");
  });
  m.def("decode_attention", [=](at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor block_table,
                                at::Tensor ctx_len, at::Tensor out, int Hq, int Hk, int D, int bs, float scale,
                                int n_split, py::object part, py::object counters) {
    bf16_2d(q, "q");
    bf16_2d(out, "out");
    i32c(block_table, "block_table");
    i32c(ctx_len, "ctx_len");
    const int B = static_cast<int>(ctx_len.numel());
    float* pp = nullptr;
    int* cp = nullptr;
    at::Tensor pt, ct;
    if (n_split > 1) {
      chk(!part.is_none() && !counters.is_none(), "decode_attention: n_split > 1 needs part and counters");
      pt = part.cast<at::Tensor>();
      ct = counters.cast<at::Tensor>();
      f32c(pt, "part");
      i32c(ct, "counters");
      chk(static_cast<size_t>(pt.numel()) >= tb_decode_attention_part_floats(B, Hq, Hk, n_split) &&
              ct.numel() >= static_cast<int64_t>(B) * Hk,
          "decode_attention: part / counters too small");
      pp = pt.data_ptr<float>();
      cp = ct.data_ptr<int>();
    }
    cuda_ok(tb_decode_attention_split(q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(),
                                      block_table.data_ptr<int>(), static_cast<int>(block_table.size(1)),
                                      ctx_len.data_ptr<int>(), out.data_ptr(), out.stride(0), B, Hq, Hk, D, bs, scale,
                                      n_split, pp, cp, turbol::StreamFor(q)),
            "decode_attention");
  }, py::arg("q"), py::arg("kc"), py::arg("vc"), py::arg("block_table"), py::arg("ctx_len"), py::arg("out"),
     py::arg("Hq"), py::arg("Hk"), py::arg("D"), py::arg("bs"), py::arg("scale"), py::arg("n_split") = 1,
     py::arg("part") = py::none(), py::arg("counters") = py::none());
  m.def("decode_attention_splits", &tb_decode_attention_splits, py::arg("B"), py::arg("Hk"));
  m.def("decode_attention_part_numel", [](int B, int Hq, int Hk, int n_split) {
    return static_cast<int64_t>(tb_decode_attention_part_floats(B, Hq, Hk, n_split));
  });
  m.def("sample", [=](at::Tensor logits, float temperature, uint64_t seed, py::object step_ptr, int64_t step,
                      at::Tensor out_tok, py::object out_logp, py::object tok_mat, py::object lp_mat,
                      py::object seed_t, py::object temp_t) {
    bf16_2d(logits, "logits");
    i32c(out_tok, "out_tok");
    const long long* sp = step_ptr.is_none()
                              ? nullptr
                              : reinterpret_cast<const long long*>(step_ptr.cast<at::Tensor>().data_ptr<int64_t>());
    float* lp = out_logp.is_none() ? nullptr : out_logp.cast<at::Tensor>().data_ptr<float>();
    int* tm = nullptr;
    float* lm = nullptr;
    int ldm = 0;
    if (!tok_mat.is_none()) {
      at::Tensor t = tok_mat.cast<at::Tensor>();
      i32c(t, "tok_mat");
      chk(t.dim() == 2 && t.size(0) == logits.size(0), "tok_mat [B, steps]");
      tm = t.data_ptr<int>();
      ldm = static_cast<int>(t.size(1));
    }
    if (!lp_mat.is_none()) {
      at::Tensor t = lp_mat.cast<at::Tensor>();
      f32c(t, "lp_mat");
      chk(t.dim() == 2 && t.size(0) == logits.size(0) && (ldm == 0 || t.size(1) == ldm), "lp_mat [B, steps]");
      lm = t.data_ptr<float>();
      ldm = static_cast<int>(t.size(1));
    }
    const unsigned long long* sd = nullptr;
    const float* tp = nullptr;
    if (!seed_t.is_none()) {
      at::Tensor t = seed_t.cast<at::Tensor>();
      chk(t.is_cuda() && t.scalar_type() == at::kLong && t.numel() >= 1, "seed_t: int64 CUDA tensor");
      sd = reinterpret_cast<const unsigned long long*>(t.data_ptr<int64_t>());
    }
    if (!temp_t.is_none()) {
      at::Tensor t = temp_t.cast<at::Tensor>();
      f32c(t, "temp_t");
      tp = t.data_ptr<float>();
    }
    cuda_ok(tb_sample(logits.data_ptr(), logits.stride(0), static_cast<int>(logits.size(0)),
                      static_cast<int>(logits.size(1)), temperature, seed, sp, step, out_tok.data_ptr<int>(), lp, tm,
                      lm, ldm, sd, tp, turbol::StreamFor(logits)),
            "sample");
  }, py::arg("logits"), py::arg("temperature"), py::arg("seed"), py::arg("step_ptr"), py::arg("step"),
     py::arg("out_tok"), py::arg("out_logp") = py::none(), py::arg("tok_mat") = py::none(),
     py::arg("lp_mat") = py::none(), py::arg("seed_t") = py::none(), py::arg("temp_t") = py::none());
  m.def("sample_filtered", [=](at::Tensor logits, float temperature, int top_k, float top_p, uint64_t seed,
                               py::object step_ptr, int64_t step, at::Tensor out_tok, py::object out_logp,
                               py::object tok_mat, py::object lp_mat, py::object seed_t, py::object temp_t,
                               int eos_id, int pad_id, py::object done, py::object lengths, py::object n_done) {
    bf16_2d(logits, "logits");
    i32c(out_tok, "out_tok");
    const int B = static_cast<int>(logits.size(0));
    auto ptr_i64 = [](py::object o) -> const long long* {
      return o.is_none() ? nullptr : reinterpret_cast<const long long*>(o.cast<at::Tensor>().data_ptr<int64_t>());
    };
    float* lp = out_logp.is_none() ? nullptr : out_logp.cast<at::Tensor>().data_ptr<float>();
    int* tm = nullptr;
    float* lm = nullptr;
    int ldm = 0;
    if (!tok_mat.is_none()) {
      at::Tensor t = tok_mat.cast<at::Tensor>();
      i32c(t, "tok_mat");
      chk(t.dim() == 2 && t.size(0) == B, "tok_mat [B, steps]");
      tm = t.data_ptr<int>();
      ldm = static_cast<int>(t.size(1));
    }
    if (!lp_mat.is_none()) {
      at::Tensor t = lp_mat.cast<at::Tensor>();
      f32c(t, "lp_mat");
      chk(t.dim() == 2 && t.size(0) == B && (ldm == 0 || t.size(1) == ldm), "lp_mat [B, steps]");
      lm = t.data_ptr<float>();
      ldm = static_cast<int>(t.size(1));
    }
    const float* tp = nullptr;
    if (!temp_t.is_none()) {
      at::Tensor t = temp_t.cast<at::Tensor>();
      f32c(t, "temp_t");
      tp = t.data_ptr<float>();
    }
    unsigned char* dn = nullptr;
    int* len = nullptr;
    int* nd = nullptr;
    if (eos_id >= 0) {
      chk(!done.is_none() && !n_done.is_none(), "sample_filtered: eos_id needs done and n_done tensors");
      at::Tensor d = done.cast<at::Tensor>();
      chk(d.is_cuda() && d.scalar_type() == at::kByte && d.numel() >= B && d.is_contiguous(), "done: uint8 [B]");
      dn = d.data_ptr<uint8_t>();
      at::Tensor c = n_done.cast<at::Tensor>();
      i32c(c, "n_done");
      nd = c.data_ptr<int>();
      if (!lengths.is_none()) {
        at::Tensor l = lengths.cast<at::Tensor>();
        i32c(l, "lengths");
        chk(l.numel() >= B, "lengths [B]");
        len = l.data_ptr<int>();
      }
    }
    if (!seed_t.is_none()) {
      at::Tensor t = seed_t.cast<at::Tensor>();
      chk(t.is_cuda() && t.scalar_type() == at::kLong && t.numel() >= 1, "seed_t: int64 CUDA tensor");
    }
    cuda_ok(tb_sample_filtered(logits.data_ptr(), logits.stride(0), B, static_cast<int>(logits.size(1)), temperature,
                               top_k, top_p, seed, ptr_i64(step_ptr), step, out_tok.data_ptr<int>(), lp, tm, lm, ldm,
                               reinterpret_cast<const unsigned long long*>(ptr_i64(seed_t)), tp, eos_id, pad_id, dn,
                               len, nd, turbol::StreamFor(logits)),
            "sample_filtered");
  }, py::arg("logits"), py::arg("temperature"), py::arg("top_k"), py::arg("top_p"), py::arg("seed"),
     py::arg("step_ptr"), py::arg("step"), py::arg("out_tok"), py::arg("out_logp") = py::none(),
     py::arg("tok_mat") = py::none(), py::arg("lp_mat") = py::none(), py::arg("seed_t") = py::none(),
     py::arg("temp_t") = py::none(), py::arg("eos_id") = -1, py::arg("pad_id") = 0, py::arg("done") = py::none(),
     py::arg("lengths") = py::none(), py::arg("n_done") = py::none());
  m.def("logprob", [=](at::Tensor logits, at::Tensor target, py::object logp, py::object dlogp, float inv_temp) {
    bf16_2d(logits, "logits");
    i32c(target, "target");
    float* lp = logp.is_none() ? nullptr : logp.cast<at::Tensor>().data_ptr<float>();
    const float* dl = dlogp.is_none() ? nullptr : dlogp.cast<at::Tensor>().data_ptr<float>();
    cuda_ok(tb_logprob(logits.data_ptr(), logits.stride(0), static_cast<int>(logits.size(0)),
                       static_cast<int>(logits.size(1)), target.data_ptr<int>(), lp, dl, inv_temp,
                       turbol::StreamFor(logits)),
            "logprob");
  }, py::arg("logits"), py::arg("target"), py::arg("logp") = py::none(), py::arg("dlogp") = py::none(),
     py::arg("inv_temp") = 1.0f);
  m.def("grpo_loss", [=](at::Tensor lp, at::Tensor old_lp, py::object ref_lp, at::Tensor adv, at::Tensor mask,
                         at::Tensor dlp, py::object stats, float clip, float beta, float inv_total_seqs) {
    f32c(lp, "lp");
    f32c(old_lp, "old_lp");
    f32c(adv, "adv");
    f32c(mask, "mask");
    f32c(dlp, "dlp");
    chk(lp.dim() == 2, "grpo_loss: lp [B, T]");
    const float* rl = ref_lp.is_none() ? nullptr : ref_lp.cast<at::Tensor>().data_ptr<float>();
    float* st = stats.is_none() ? nullptr : stats.cast<at::Tensor>().data_ptr<float>();
    cuda_ok(tb_grpo_loss(lp.data_ptr<float>(), old_lp.data_ptr<float>(), rl, adv.data_ptr<float>(),
                         mask.data_ptr<float>(), dlp.data_ptr<float>(), st, static_cast<int>(lp.size(0)),
                         static_cast<int>(lp.size(1)), clip, beta, inv_total_seqs, turbol::StreamFor(lp)),
            "grpo_loss");
  });
  m.def("ppo_token_loss", [=](at::Tensor lp, at::Tensor old_lp, at::Tensor adv, at::Tensor v, at::Tensor old_v,
                              at::Tensor ret, at::Tensor dlp, at::Tensor dv, py::object stats, float clip, float vclip,
                              float vf_coef, float norm) {
    for (auto* t : {&lp, &old_lp, &adv, &v, &old_v, &ret, &dlp, &dv}) f32c(*t, "ppo_token_loss");
    const long long R = lp.numel();
    for (auto* t : {&old_lp, &adv, &v, &old_v, &ret, &dlp, &dv})
      chk(t->numel() == R, "ppo_token_loss: every array has the same number of tokens");
    float* st = stats.is_none() ? nullptr : stats.cast<at::Tensor>().data_ptr<float>();
    cuda_ok(tb_ppo_token_loss(lp.data_ptr<float>(), old_lp.data_ptr<float>(), adv.data_ptr<float>(),
                              v.data_ptr<float>(), old_v.data_ptr<float>(), ret.data_ptr<float>(),
                              dlp.data_ptr<float>(), dv.data_ptr<float>(), st, R, clip, vclip, vf_coef, norm,
                              turbol::StreamFor(lp)),
            "ppo_token_loss");
  });
  m.def(
      "flash_attn_fwd",
      [=](at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, py::object lse, int B, int T, int Hq, int Hk,
          float scale, const std::string& impl, py::object err) {
        bf16_2d(q, "q");
        bf16_2d(o, "o");
        chk(q.stride(0) == k.stride(0) && q.stride(0) == v.stride(0), "flash_attn: q/k/v share the row stride");
        float* l = lse.is_none() ? nullptr : lse.cast<at::Tensor>().data_ptr<float>();
        if (impl == "tc") {
          int* e = err.is_none() ? nullptr : err.cast<at::Tensor>().data_ptr<int>();
          cuda_ok(tb_flash_attn_fwd_tc(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(0), o.data_ptr(),
                                       o.stride(0), l, B, T, Hq, Hk, scale, e, turbol::StreamFor(q)),
                  "flash_attn_fwd");
        } else {
          chk(impl == "mma", "flash_attn_fwd: impl is 'tc' (tcgen05) or 'mma' (mma.sync)");
          cuda_ok(tb_flash_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(0), o.data_ptr(), o.stride(0),
                                    l, B, T, Hq, Hk, scale, turbol::StreamFor(q)),
                  "flash_attn_fwd");
        }
      },
      py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("lse"), py::arg("B"), py::arg("T"),
      py::arg("Hq"), py::arg("Hk"), py::arg("scale"), py::arg("impl") = "tc", py::arg("err") = py::none());
  m.def(
      "flash_attn_bwd",
      [=](at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor dout, at::Tensor lse, at::Tensor delta,
          at::Tensor dq, at::Tensor dk, at::Tensor dv, int B, int T, int Hq, int Hk, float scale,
          const std::string& impl, py::object ws, py::object err) {
        chk(dq.stride(0) == dk.stride(0) && dq.stride(0) == dv.stride(0), "flash_attn_bwd: dq/dk/dv share the stride");
        if (impl == "tc") {
          float* w = nullptr;
          size_t wb = 0;
          if (!ws.is_none()) {
            at::Tensor wt = ws.cast<at::Tensor>();
            chk(wt.is_cuda() && wt.scalar_type() == at::kFloat && wt.is_contiguous(), "flash_attn_bwd: ws fp32");
            w = wt.data_ptr<float>();
            wb = static_cast<size_t>(wt.numel()) * sizeof(float);
          }
          int* e = err.is_none() ? nullptr : err.cast<at::Tensor>().data_ptr<int>();
          cuda_ok(tb_flash_attn_bwd_tc(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(0), o.data_ptr(),
                                       o.stride(0), dout.data_ptr(), dout.stride(0), lse.data_ptr<float>(),
                                       delta.data_ptr<float>(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                                       dq.stride(0), B, T, Hq, Hk, scale, w, wb, e, turbol::StreamFor(q)),
                  "flash_attn_bwd");
        } else {
          chk(impl == "mma", "flash_attn_bwd: impl is 'tc' (tcgen05) or 'mma' (mma.sync)");
          cuda_ok(tb_flash_attn_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(0), o.data_ptr(), o.stride(0),
                                    dout.data_ptr(), dout.stride(0), lse.data_ptr<float>(), delta.data_ptr<float>(),
                                    dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dq.stride(0), B, T, Hq, Hk, scale,
                                    turbol::StreamFor(q)),
                  "flash_attn_bwd");
        }
      },
      py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("dout"), py::arg("lse"), py::arg("delta"),
      py::arg("dq"), py::arg("dk"), py::arg("dv"), py::arg("B"), py::arg("T"), py::arg("Hq"), py::arg("Hk"),
      py::arg("scale"), py::arg("impl") = "tc", py::arg("ws") = py::none(), py::arg("err") = py::none());
  m.def("flash_attn_bwd_ws_numel", [](int B, int T, int Hk) {
    return static_cast<int64_t>(tb_flash_attn_bwd_ws_bytes(B, T, Hk) / sizeof(float));
  });

  m.attr("EPI_NONE") = static_cast<int>(TB_EPI_NONE);
  m.attr("EPI_BIAS") = static_cast<int>(TB_EPI_BIAS);
  m.attr("EPI_BIAS_TANH") = static_cast<int>(TB_EPI_BIAS_TANH);
  m.attr("EPI_BIAS_SILU") = static_cast<int>(TB_EPI_BIAS_SILU);
  m.attr("EPI_TANH_BWD") = static_cast<int>(TB_EPI_TANH_BWD);
  m.attr("EPI_RESIDUAL") = static_cast<int>(TB_EPI_RESIDUAL);
  m.attr("EPI_SWIGLU") = static_cast<int>(TB_EPI_SWIGLU);
  m.attr("EPI_SWIGLU_BWD") = static_cast<int>(TB_EPI_SWIGLU_BWD);
}
