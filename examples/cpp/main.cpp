// Native C++ demo of the framework's core (the counterpart of the reference's
// turbol_vllm/examples/main.cpp:9-59): builds the runtime, tensors, an
// environment, a replay buffer, the reward engine, the config store, the
// profiler and the distributed trainer from C++ only, steps the environment through its public API and
// prints what it did.  Runs on CPU, or on the GPU when one is present.
//
//   make -C examples/cpp && ./examples/cpp/turbol_demo [cpu|cuda]
#include <cstdio>
#include <string>

#include "turbol/common.hpp"
#include "turbol/config.hpp"
#include "turbol/distributed.hpp"
#include "turbol/engines.hpp"
#include "turbol/observability.hpp"
#include "turbol/runtime.hpp"

using namespace turbol;

static int fail(const char* what, const Status& s) {
  std::printf("FAILED: %s: %s\n", what, s.ToString().c_str());
  return 1;
}

int main(int argc, char** argv) {
  const bool want_cuda = argc > 1 ? std::string(argv[1]) == "cuda" : GetCudaDeviceCount() > 0;
  const Device dev = want_cuda ? Device::CUDA(0) : Device::CPU();
  std::printf("=== turbol_b200 native demo (device %s) ===\n", dev.ToString().c_str());

  std::printf("\n1. Core engine\n");
  auto& engine = CoreEngine::Instance();
  if (want_cuda) {
    Status s = engine.Initialize(0, 4);
    if (!s.ok()) return fail("CoreEngine::Initialize", s);
  }
  engine.RegisterModule("demo");
  std::printf("   modules registered: %zu\n", engine.ListModules().size());

  std::printf("\n2. Tensor\n");
  Tensor t(Shape({10, 20}), DataType::kFloat32, dev);
  Status s = TensorUtils::Fill(&t, 1.5f);
  if (!s.ok()) return fail("TensorUtils::Fill", s);
  std::printf("   [10, 20] float32: %zu bytes, filled with 1.5\n", t.size_bytes());

  std::printf("\n3. Environment (CartPole, 1024 envs)\n");
  GPUEnvironment env(1024, 4, 2, dev, EnvType::kCartPole, 7);
  Tensor action(Shape({1024}), DataType::kInt32, dev);
  Tensor obs, reward, done;
  long finished = 0;
  for (int step = 0; step < 200; ++step) {
    action.torch().random_(0, 2);
    s = env.Step(action, &obs, &reward, &done);
    if (!s.ok()) return fail("GPUEnvironment::Step", s);
    finished += done.torch().sum().item<long>();
  }
  const auto stats = env.TakeEpisodeStats();
  std::printf("   200 steps x 1024 envs, %ld episodes finished, mean return %.2f\n", finished,
              stats[1] > 0 ? stats[0] / stats[1] : 0.0);

  std::printf("\n4. Replay buffer\n");
  RingBuffer buffer(4096, 4, 1, dev, 3);
  Tensor act(Shape({1024, 1}), DataType::kFloat32, dev);
  s = buffer.PushBatch(obs, act, reward, done);
  if (!s.ok()) return fail("RingBuffer::PushBatch", s);
  Tensor so, sa, sr, sd;
  s = buffer.Sample(256, &so, &sa, &sr, &sd);
  if (!s.ok()) return fail("RingBuffer::Sample", s);
  std::printf("   capacity %lld, size %lld, sampled %lld rows\n", static_cast<long long>(buffer.Capacity()),
              static_cast<long long>(buffer.Size()), static_cast<long long>(so.shape()[0]));

  std::printf("\n5. Reward engine\n");
  RewardConfig rc;
  rc.normalize = false;
  RewardEngine rewards(rc);
  s = rewards.Initialize();
  if (!s.ok()) return fail("RewardEngine::Initialize", s);
  RewardResult rr;
  s = rewards.ScoreBatch({"A short answer.", "no period"}, std::nullopt, &rr);
  if (!s.ok()) return fail("RewardEngine::ScoreBatch", s);
  const at::Tensor tot = rr.total.torch().to(at::kCPU).to(at::kFloat);
  std::printf("   rule rewards: %.3f %.3f\n", tot[0].item<float>(), tot[1].item<float>());

  std::printf("\n6. Config and profiler\n");
  Config cfg;
  cfg.SetInt("num_envs", 1024);
  Profiler prof;
  prof.Enable();
  {
    Profiler::Guard g(&prof, "demo_span", "demo");
  }
  std::printf("   config num_envs=%lld, profiler spans=%zu\n", cfg.GetInt("num_envs", 0), prof.GetAllSpans().size());

  std::printf("\n7. Distributed trainer (one process: a group of one)\n");
  distributed::DistributedConfig dcfg;
  distributed::DistributedTrainer dist(dcfg);
  s = dist.Initialize();
  if (!s.ok()) return fail("DistributedTrainer::Initialize", s);
  s = dist.AllReduce(&t, "mean");
  if (!s.ok()) return fail("DistributedTrainer::AllReduce", s);
  std::printf("   rank %d of %d, all-reduce(mean) ok\n", dist.GetRank(), dist.GetWorldSize());
  dist.Shutdown();

  if (want_cuda) {
    const auto mem = GetCudaMemoryInfo(0);
    std::printf("\n[CUDA] %zu MB used / %zu MB total\n", mem.used() >> 20, mem.total >> 20);
  }
  std::printf("\n=== demo finished ===\n");
  return 0;
}
