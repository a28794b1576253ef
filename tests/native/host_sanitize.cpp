// Host-side race and memory checks of the native core (built with
// -fsanitize=address,undefined and, separately, -fsanitize=thread by
// tests/test_sanitizers.py; no GPU is used).  Each section drives one
// component the way the Python bindings do, with the concurrency the
// framework allows: the profiler from several threads with exports running
// alongside (the reference's ExportJSON re-locked its own mutex,
// turbol_vllm/src/profiler/profiler.cpp:192-200), the TCP rendezvous store
// with a server thread per client, the KV block allocator through many
// allocate/append/free cycles, the file formats (Config, TFRecord event
// files, Prometheus text, JSONL datasets) through write/read round trips, and
// the CPU trainer's host engines (CartPole rollout, PPO minibatch step and
// update with Adam, GAE) on sizes that are not multiples of the vector tiles,
// from two threads at once.
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <string>
#include <thread>
#include <vector>

#include <ATen/ATen.h>
#include <ATen/CPUGeneratorImpl.h>
#include <ATen/Parallel.h>

#include "kernels.h"
#include "turbol/config.hpp"
#include "turbol/engines.hpp"
#include "turbol/observability.hpp"
#include "turbol/runtime.hpp"

// The sanitizer build links no kernels: the launchers come from the CPU-only
// build's stubs (csrc/cpu_only/kernel_stubs.cpp), which CPU tensors never reach.

using namespace turbol;

static int g_fail = 0;
#define EXPECT(c)                                                   \
  do {                                                             \
    if (!(c)) {                                                    \
      std::fprintf(stderr, "EXPECT failed %s:%d: %s\n", __FILE__, __LINE__, #c); \
      ++g_fail;                                                    \
    }                                                              \
  } while (0)

static void config_roundtrip(const std::string& dir) {
  Config c;
  c.SetString("model", "qwen2-1.5b");
  c.SetInt("num_envs", 65536);
  c.SetFloat("lr", 3e-4);
  c.SetBool("fused", true);
  const std::string p = dir + "/cfg.txt";
  EXPECT(c.Save(p).ok());
  Config d;
  EXPECT(d.Load(p).ok());
  EXPECT(d.GetInt("num_envs", 0) == 65536 && d.GetBool("fused", false) && d.GetString("model", "") == "qwen2-1.5b");
}

static void profiler_threads(const std::string& dir) {
  ProfilerConfig pc;
  pc.enable_cuda_timing = false;
  Profiler prof(pc);
  prof.Enable();
  std::atomic<bool> done{false};
  std::vector<std::thread> ts;
  for (int t = 0; t < 4; ++t)
    ts.emplace_back([&prof, t] {
      for (int i = 0; i < 300; ++i) {
        SpanID a = prof.BeginSpan("outer" + std::to_string(t));
        SpanID b = prof.BeginSpan("inner");
        prof.RecordComm("allreduce", 1 << 20, 0.01);
        prof.EndSpan(b);
        prof.EndSpan(a);
      }
    });
  std::thread exporter([&] {
    int n = 0;
    while (!done.load()) {
      EXPECT(prof.ExportJSON(dir + "/stats.json").ok());
      (void)prof.GetStats();
      (void)prof.Summary();
      ++n;
      // exports walk every span under the profiler's lock; back to back they
      // can starve the recording threads (minutes under a sanitizer)
      std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    EXPECT(n > 0);
  });
  for (auto& t : ts) t.join();
  done = true;
  exporter.join();
  EXPECT(prof.GetAllSpans().size() == 4u * 300u * 2u);
  EXPECT(prof.ExportChromeTrace(dir + "/trace.json").ok());
  prof.Disable();
}

static void writers(const std::string& dir) {
  {
    TensorBoardWriter tb(dir);
    std::vector<float> h(1000);
    for (int i = 0; i < 1000; ++i) h[i] = static_cast<float>(i % 37) * 0.5f;
    std::vector<std::thread> ts;
    for (int t = 0; t < 3; ++t)
      ts.emplace_back([&tb, &h, t] {
        for (int s = 0; s < 200; ++s) tb.AddScalar("loss/" + std::to_string(t), 1.0f / (s + 1), s);
        tb.AddHistogram("h", h.data(), static_cast<int64_t>(h.size()), t);
        tb.AddText("note", "step text", t);
      });
    for (auto& t : ts) t.join();
    tb.Flush();
  }
  PrometheusWriter pw(dir + "/metrics.prom");
  for (int i = 0; i < 50; ++i) {
    Labels l;
    l.kv["rank"] = "0";
    pw.WriteCounter("env_steps_total", 1000.0 * i, l);
    pw.WriteGauge("reward_mean", 0.5);
  }
  pw.Flush();
}

static void tcp_store() {
  TcpStore server("127.0.0.1", 0, true, 5000);
  const int port = server.port();
  EXPECT(port > 0);
  const int world = 4;
  std::vector<std::thread> ts;
  std::atomic<int> ok{0};
  for (int r = 0; r < world; ++r)
    ts.emplace_back([&, r] {
      TcpStore c("127.0.0.1", port, false, 5000);
      bool good = c.Set("key" + std::to_string(r), "v" + std::to_string(r)).ok();
      int64_t res = 0;
      for (int i = 0; i < 20; ++i) good = good && c.Add("counter", 1, &res).ok();
      good = good && c.Barrier("b0", world, 5000).ok();
      std::string v;
      good = good && c.Get("key" + std::to_string((r + 1) % world), &v, 5000).ok() &&
             v == "v" + std::to_string((r + 1) % world);
      good = good && c.Barrier("b1", world, 5000).ok();
      if (good) ok.fetch_add(1);
    });
  for (auto& t : ts) t.join();
  EXPECT(ok.load() == world);
  std::string v;
  EXPECT(server.Get("counter", &v, 1000).ok() && v == "80");
  // a missing key times out with a status, not a hang
  EXPECT(server.Get("never_set", &v, 50).code() == StatusCode::kTimeout);
}

static void kv_blocks() {
  KVBlockManager kv(257, 16);
  for (int round = 0; round < 20; ++round) {
    for (int s = 0; s < 16; ++s) EXPECT(kv.Allocate(round * 100 + s, 200).ok());
    for (int s = 0; s < 16; ++s)
      for (int t = 0; t < 20; ++t) EXPECT(kv.AppendToken(round * 100 + s).ok());
    EXPECT(kv.BlockTable(round * 100 + 3).size() == static_cast<size_t>(kv.BlocksFor(220)));
    for (int s = 0; s < 16; ++s) EXPECT(kv.Free(round * 100 + s).ok());
    EXPECT(kv.NumFree() == 257);
  }
  EXPECT(!kv.Allocate(1, 257 * 16 + 1).ok());  // more than the pool: refused
}

static void schedules_tokenizer_dataset(const std::string& dir) {
  for (int S = 1; S <= 8; ++S)
    for (int s = 0; s < S; ++s) {
      auto ops = PipelineSchedule::OneFOneB(S, s, 8);
      EXPECT(ops.size() == 16u);
      EXPECT(PipelineSchedule::PeakActivations(ops) <= S - s);
    }
  ByteTokenizer tok;
  const std::string text = "GRPO on B200: \xce\xbb = 0.95 \xe2\x9c\x93";
  EXPECT(tok.Decode(tok.Encode(text, true, true)) == text);
  const std::string p = dir + "/data.jsonl";
  {
    std::ofstream f(p);
    for (int i = 0; i < 64; ++i)
      f << "{\"prompt\": \"question " << i << " \\\"quoted\\\"\", \"chosen\": \"yes\", \"rejected\": \"no\"}\n";
  }
  DatasetConfig dc;
  dc.data_paths = {p};
  dc.batch_size = 8;
  dc.max_seq_length = 32;
  Dataset ds(dc);
  EXPECT(ds.Initialize().ok());
  int batches = 0;
  PreprocessedBatch b;
  while (ds.HasNext() && ds.NextBatch(&b).ok()) ++batches;
  EXPECT(batches == 8);
}

// One CPU PPO iteration through the host engines: rollout on CartPole, GAE,
// the update (epochs x minibatches with Adam), one stand-alone minibatch step,
// and a rejected call (a row index past the data) that must not read it.
static void ppo_host_iteration(uint64_t seed) {
  const int N = 37, T = 5, B = T * N, MB = 37;
  const std::vector<int64_t> dims_a{4, 20, 37, 2}, dims_c{4, 20, 37, 1};
  int64_t n = 0;
  for (const auto* d : {&dims_a, &dims_c})
    for (size_t l = 0; l + 1 < d->size(); ++l) n += (*d)[l + 1] * ((*d)[l] + 1);
  // a generator of this thread's own: the global one is shared state
  const at::Generator gen = at::detail::createCPUGenerator(seed);
  const at::Tensor flat = at::randn({n}, gen) * 0.2, grad = at::zeros({n}), m = at::zeros({n}), v = at::zeros({n});
  GPUEnvironment env(N, 4, 2, Device::CPU(), EnvType::kCartPole, seed);
  const auto i32 = at::TensorOptions().dtype(at::kInt), u8 = at::TensorOptions().dtype(at::kByte);
  const at::Tensor obs = at::zeros({T, N, 4}), act = at::zeros({T, N}, i32), logp = at::zeros({T, N}),
                   val = at::zeros({T + 1, N}), rew = at::zeros({T, N}), done = at::zeros({T, N}, u8);
  EXPECT(PpoCartPoleRolloutHost(&env, flat, dims_a, dims_c, obs, act, logp, val, rew, done, seed, 0).ok());
  EXPECT(act.min().item<int>() >= 0 && act.max().item<int>() <= 1 && at::all(logp <= 0).item<bool>());
  const at::Tensor adv = at::zeros({T, N}), ret = at::zeros({T, N});
  double st2[2] = {0, 0};
  EXPECT(GaeHost(rew.data_ptr<float>(), val.data_ptr<float>(), done.data_ptr<uint8_t>(), adv.data_ptr<float>(),
                 ret.data_ptr<float>(), T, N, 0.99f, 0.95f, st2)
             .ok());
  const at::Tensor perms = at::stack({at::randperm(B, gen), at::randperm(B, gen)});
  const at::Tensor stats = at::zeros({8});
  Status st;
  const int64_t last = PpoCategoricalUpdateHost(flat, grad, m, v, 0, dims_a, dims_c, obs.view({B, 4}),
                                                act.view({B}), logp.view({B}), adv.view({B}), ret.view({B}), perms,
                                                MB, 0.2f, 0.5f, 0.01f, 3e-4f, 0.9f, 0.999f, 1e-5f, 0.f, stats, &st);
  EXPECT(st.ok() && last == 2 * (B / MB) && stats[5].item<float>() == 2.f * B);
  const at::Tensor idx = at::randperm(B, gen).narrow(0, 0, 13);
  EXPECT(PpoCategoricalMinibatchHost(flat, grad, dims_a, dims_c, obs.view({B, 4}), act.view({B}), logp.view({B}),
                                     adv.view({B}), ret.view({B}), idx, 0.2f, 0.5f, 0.01f, stats)
             .ok());
  const at::Tensor bad = at::full({3}, static_cast<int64_t>(B));
  EXPECT(!PpoCategoricalMinibatchHost(flat, grad, dims_a, dims_c, obs.view({B, 4}), act.view({B}), logp.view({B}),
                                      adv.view({B}), ret.view({B}), bad, 0.2f, 0.5f, 0.01f, stats)
              .ok());
  EXPECT(at::all(at::isfinite(flat)).item<bool>());
}

static void ppo_host_threads() {
  std::thread a(ppo_host_iteration, 11), b(ppo_host_iteration, 12);
  a.join();
  b.join();
}

// A minibatch and a rollout batch split by rows over threads (per-thread
// workspaces and gradient buffers, summed after the join): main lowers the
// work per thread (TURBOL_HOST_THREAD_MACS) so that these small batches
// split; every tensor is made before the thread count is raised, so only the
// core's own threads run while it is 4.
static void ppo_host_split() {
  const int B = 67, N = 70, T = 2;
  const std::vector<int64_t> dims_a{4, 16, 24, 2}, dims_c{4, 16, 24, 1};
  int64_t n = 0;
  for (const auto* d : {&dims_a, &dims_c})
    for (size_t l = 0; l + 1 < d->size(); ++l) n += (*d)[l + 1] * ((*d)[l] + 1);
  const at::Generator gen = at::detail::createCPUGenerator(21);
  const at::Tensor flat = at::randn({n}, gen) * 0.1, grad = at::zeros({n}), m = at::zeros({n}), v = at::zeros({n});
  const at::Tensor obs = at::randn({B, 4}, gen), logp = at::randn({B}, gen) * 0.1 - 0.7, adv = at::randn({B}, gen),
                   ret = at::randn({B}, gen), stats = at::zeros({8});
  const at::Tensor act = at::randint(0, 2, {B}, gen, at::TensorOptions().dtype(at::kInt));
  const at::Tensor perms = at::randperm(B, gen).view({1, B});
  GPUEnvironment env(N, 4, 2, Device::CPU(), EnvType::kCartPole, 21);
  const at::Tensor ro = at::zeros({T, N, 4}), ra = at::zeros({T, N}, at::TensorOptions().dtype(at::kInt)),
                   rl = at::zeros({T, N}), rv = at::zeros({T + 1, N}), rr = at::zeros({T, N}),
                   rd = at::zeros({T, N}, at::TensorOptions().dtype(at::kByte));
  const int GT = 40, GN = 64 * 1024;  // GAE over 2.6 M elements: split into column blocks
  const at::Tensor gr = at::randn({GT, GN}, gen), gv = at::randn({GT + 1, GN}, gen),
                   gd = at::zeros({GT, GN}, at::TensorOptions().dtype(at::kByte)), ga = at::empty({GT, GN}),
                   gret = at::empty({GT, GN});
  double gs[2] = {0, 0};
  const int prev = at::get_num_threads();
  at::set_num_threads(4);
  Status st;
  const int64_t last = PpoCategoricalUpdateHost(flat, grad, m, v, 0, dims_a, dims_c, obs, act, logp, adv, ret, perms,
                                                B, 0.2f, 0.5f, 0.01f, 3e-4f, 0.9f, 0.999f, 1e-5f, 0.f, stats, &st);
  const Status rs = PpoCartPoleRolloutHost(&env, flat, dims_a, dims_c, ro, ra, rl, rv, rr, rd, 21, 0);
  const Status gst = GaeHost(gr.data_ptr<float>(), gv.data_ptr<float>(), gd.data_ptr<uint8_t>(), ga.data_ptr<float>(),
                             gret.data_ptr<float>(), GT, GN, 0.99f, 0.95f, gs);
  at::set_num_threads(prev);
  EXPECT(gst.ok() && std::isfinite(gs[0]) && gs[1] > 0 && at::all(at::isfinite(gret)).item<bool>());
  EXPECT(st.ok() && last == 1 && stats[5].item<float>() == static_cast<float>(B));
  EXPECT(rs.ok() && at::all(at::isfinite(flat)).item<bool>() && at::all(at::isfinite(rv)).item<bool>());
}

int main(int argc, char** argv) {
  // small batches split over threads in ppo_host_split (read once, before any host-engine call)
  setenv("TURBOL_HOST_THREAD_MACS", "16384", 1);
  const std::string dir = argc > 1 ? argv[1] : "/tmp";
  // each section's wall time goes to stdout (instrumented code is slow; this shows where)
  auto section = [](const char* name, auto&& fn) {
    const auto t0 = std::chrono::steady_clock::now();
    fn();
    std::printf("%-28s %8.2f s\n", name,
                std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
    std::fflush(stdout);
  };
  section("config", [&] { config_roundtrip(dir); });
  section("profiler threads", [&] { profiler_threads(dir); });
  section("writers", [&] { writers(dir); });
  section("tcp store", [] { tcp_store(); });
  section("kv blocks", [] { kv_blocks(); });
  section("schedules/tokenizer/dataset", [&] { schedules_tokenizer_dataset(dir); });
  section("ppo host (two threads)", [] { ppo_host_threads(); });
  section("ppo host (split batches)", [] { ppo_host_split(); });
  if (g_fail) {
    std::fprintf(stderr, "%d checks failed\n", g_fail);
    return 1;
  }
  std::printf("HOST_SANITIZE_OK\n");
  return 0;
}
