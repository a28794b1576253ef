"""turbol_b200 — a Blackwell-native (B200, sm_100a) RL / RLHF framework.

Drop-in for the reference's ``import turbol`` API (turbol_vllm/python/turbol/
__init__.py:10-211): ``import turbol_b200 as turbol`` gives Tensor,
GPUEnvironment, RingBuffer, PolicyEngine, Config, RolloutConfig/RolloutEngine,
RewardConfig/RewardEngine/RewardResult, DistributedConfig/DistributedTrainer,
Profiler/ProfilerGuard/ProfilerConfig, TensorBoardWriter, PrometheusWriter,
Labels, get_version, get_device_count, get_memory_info, make, from_torch,
to_torch, register_env, get_build_info and the vLLM wrapper names.

The package is named ``turbol_b200`` (not ``turbol``) so it can be imported
side by side with the reference build used as the baseline arm.
"""
from __future__ import annotations

__version__ = "1.0.0"

from typing import Any, Callable, Dict, Optional

import torch

from ._native import core as _core_fn
from .utils.device import device_str as _device_str, parse_device as _parse_device

turbol_core = _core_fn()

Status = turbol_core.Status
StatusCode = turbol_core.StatusCode
Shape = turbol_core.Shape
Tensor = turbol_core.Tensor
GPUEnvironment = turbol_core.GPUEnvironment
CartPoleConfig = turbol_core.CartPoleConfig
RingBuffer = turbol_core.RingBuffer
PrioritizedReplayBuffer = turbol_core.PrioritizedReplayBuffer
Config = turbol_core.Config
RewardConfig = turbol_core.RewardConfig
RewardResult = turbol_core.RewardResult
RewardEngine = turbol_core.RewardEngine
SpanID = turbol_core.SpanID
Profiler = turbol_core.Profiler
ProfilerGuard = turbol_core.ProfilerGuard
ProfilerConfig = turbol_core.ProfilerConfig
AggregatedStats = turbol_core.AggregatedStats
TensorBoardWriter = turbol_core.TensorBoardWriter
PrometheusWriter = turbol_core.PrometheusWriter
Labels = turbol_core.Labels
CoreEngine = turbol_core.CoreEngine
TensorUtils = turbol_core.TensorUtils
ByteTokenizer = turbol_core.ByteTokenizer
Dataset = turbol_core.Dataset
DatasetConfig = turbol_core.DatasetConfig
DataSample = turbol_core.DataSample
TcpStore = turbol_core.TcpStore
PipelineSchedule = turbol_core.PipelineSchedule
KVBlockManager = turbol_core.KVBlockManager

get_version = turbol_core.get_version
get_device_count = turbol_core.get_device_count
get_memory_info = turbol_core.get_memory_info

from .rl.policy import PolicyEngine  # noqa: E402

_LAZY = {
    "RolloutConfig": ("turbol_b200.rl.rollout", "RolloutConfig"),
    "RolloutEngine": ("turbol_b200.rl.rollout", "RolloutEngine"),
    "DistributedConfig": ("turbol_b200.parallel.dist", "DistributedConfig"),
    "DistributedTrainer": ("turbol_b200.parallel.dist", "DistributedTrainer"),
    "PPOConfig": ("turbol_b200.rl.ppo", "PPOConfig"),
    "PPOTrainer": ("turbol_b200.rl.ppo", "PPOTrainer"),
    "GRPOConfig": ("turbol_b200.rl.grpo", "GRPOConfig"),
    "GRPOTrainer": ("turbol_b200.rl.grpo", "GRPOTrainer"),
    "VLLMInferenceEngine": ("turbol_b200.vllm_inference", "VLLMInferenceEngine"),
    "VLLMInferenceConfig": ("turbol_b200.vllm_inference", "VLLMInferenceConfig"),
    "DEEPSEEK_MODELS": ("turbol_b200.vllm_inference", "DEEPSEEK_MODELS"),
    "vllm_available": ("turbol_b200.vllm_inference", "vllm_available"),
    "save_checkpoint": ("turbol_b200.utils.checkpoint", "save_checkpoint"),
    "load_checkpoint": ("turbol_b200.utils.checkpoint", "load_checkpoint"),
}


def __getattr__(name):
    if name in _LAZY:
        import importlib

        mod, attr = _LAZY[name]
        val = getattr(importlib.import_module(mod), attr)
        globals()[name] = val
        return val
    raise AttributeError(name)


__all__ = [
    "Tensor", "GPUEnvironment", "RingBuffer", "PrioritizedReplayBuffer", "PolicyEngine", "Config",
    "RolloutConfig", "RolloutEngine", "RewardConfig", "RewardEngine", "RewardResult", "DistributedConfig",
    "DistributedTrainer", "VLLMInferenceEngine", "VLLMInferenceConfig", "DEEPSEEK_MODELS", "vllm_available",
    "Profiler", "ProfilerGuard", "ProfilerConfig", "TensorBoardWriter", "PrometheusWriter", "Labels",
    "get_version", "get_device_count", "get_memory_info", "make", "from_torch", "to_torch", "register_env",
    "get_build_info", "PPOConfig", "PPOTrainer", "GRPOConfig", "GRPOTrainer",
]

# --------------------------------------------------------------------------
# environments registry (consulted by make(); the reference's registry is
# write-only, turbol_vllm/python/turbol/__init__.py:122-145,195-197)
# --------------------------------------------------------------------------
_ENV_REGISTRY: Dict[str, Callable[..., Any]] = {}


def register_env(name: str, factory_fn: Callable[..., Any]):
    """Registers ``factory_fn(num_envs=..., device=..., **kwargs)`` under ``name``."""
    _ENV_REGISTRY[name] = factory_fn


def make(env_name: str = "LinearEnv", num_envs: int = 256, device: str = "cuda:0", **kwargs):
    """Creates a vectorized environment: "LinearEnv", "CartPole"/"CartPole-v1",
    or any name registered with :func:`register_env`."""
    dev = _device_str(device)
    if dev.startswith("cuda") and not torch.cuda.is_available():
        dev = "cpu"
    if env_name in _ENV_REGISTRY:
        return _ENV_REGISTRY[env_name](num_envs=num_envs, device=dev, **kwargs)
    seed = kwargs.pop("seed", 42)
    if env_name in ("CartPole", "CartPole-v1", "cartpole"):
        return GPUEnvironment(num_envs=num_envs, obs_dim=4, act_dim=2, device=dev, env_type="cartpole", seed=seed)
    if env_name in ("LinearEnv", "linear"):
        return GPUEnvironment(num_envs=num_envs, obs_dim=kwargs.pop("obs_dim", 4), act_dim=kwargs.pop("act_dim", 2),
                              device=dev, env_type="linear", seed=seed)
    raise ValueError(f"unknown environment {env_name!r}; registered: {sorted(_ENV_REGISTRY)}")


def from_torch(tt: torch.Tensor, device: Optional[str] = None) -> Tensor:
    """torch.Tensor -> Tensor.  Zero-copy when already on the target device and
    contiguous (the Tensor adopts the torch storage); otherwise one copy."""
    if device is not None:
        tt = tt.to(_parse_device(device))
    return Tensor.from_torch(tt.contiguous())


def to_torch(t: Tensor) -> torch.Tensor:
    """Tensor -> torch.Tensor sharing the same storage (CPU and CUDA)."""
    return t.torch()


def get_build_info() -> Dict[str, Any]:
    n = get_device_count()
    return {
        "version": __version__,
        "cuda_available": n > 0,
        "num_devices": n,
        "torch_version": torch.__version__,
        "arch": turbol_core.built_for(),
    }
