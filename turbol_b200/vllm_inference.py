"""Optional vLLM-backed text generation with the reference's Python surface.

Reference: turbol_vllm/python/turbol/vllm_inference.py (presets :51-77,
``vllm_available`` :80-86, ``VLLMInferenceConfig`` :93-120,
``VLLMInferenceEngine`` :127-236).  Behaviour kept:

* nothing heavy happens at construction; the ``vllm`` import and the model load
  happen on the first real generation;
* without vLLM (or before a model is loaded) and with ``fallback_to_echo``,
  ``generate`` / ``generate_batch`` return ``"[VLLMInferenceEngine] " + prompt``;
  with ``fallback_to_echo=False`` they raise ``RuntimeError`` naming vllm;
* preset keys resolve to Hugging Face repo ids; local paths and full ids pass
  through; presets marked ``chat`` use the tokenizer's chat template.

Addition: ``backend="native"`` routes generation through this package's own
decode engine (:class:`turbol_b200.rl.rollout.RolloutEngine`: paged KV cache,
tensor-core GEMMs, CUDA-graph decode) on a random-init model of the preset's
architecture shape, for machines without vLLM or without the weights.  vLLM is
never on a hot path of this package.
"""
from __future__ import annotations

import importlib.util
import os
from dataclasses import dataclass
from typing import List, Optional, Sequence

ECHO_PREFIX = "[VLLMInferenceEngine] "

# Small DeepSeek presets, smallest first.  ``shape`` names the architecture the
# native backend instantiates for a preset.
DEEPSEEK_MODELS: dict = {
    "deepseek-r1-distill-qwen-1.5b": {"repo": "deepseek-ai/DeepSeek-R1-Distill-Qwen-1.5B", "params": "1.5B",
                                      "chat": True, "shape": "qwen2-1.5b"},
    "deepseek-r1-distill-qwen-7b": {"repo": "deepseek-ai/DeepSeek-R1-Distill-Qwen-7B", "params": "7B",
                                    "chat": True, "shape": "tiny"},
    "deepseek-r1-distill-llama-8b": {"repo": "deepseek-ai/DeepSeek-R1-Distill-Llama-8B", "params": "8B",
                                     "chat": True, "shape": "llama3-8b"},
    "deepseek-v2-lite": {"repo": "deepseek-ai/DeepSeek-V2-Lite", "params": "15.7B (MoE, ~2.4B active)",
                         "chat": True, "shape": "tiny"},
    "deepseek-llm-7b-chat": {"repo": "deepseek-ai/deepseek-llm-7b-chat", "params": "7B", "chat": True,
                             "shape": "tiny"},
}


def vllm_available() -> bool:
    """True if the ``vllm`` package is installed (checked without importing it)."""
    try:
        return importlib.util.find_spec("vllm") is not None
    except (ImportError, ValueError):
        return False


@dataclass
class VLLMInferenceConfig:
    model: str = "deepseek-r1-distill-qwen-1.5b"  # preset key, Hugging Face repo id, or local path
    tensor_parallel_size: int = 1
    max_new_tokens: int = 256
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    max_batch_size: int = 256
    dtype: str = "auto"
    trust_remote_code: bool = True
    use_chat_template: bool = False
    gpu_memory_utilization: float = 0.90
    max_model_len: int = 8192
    fallback_to_echo: bool = True
    backend: str = "vllm"  # "vllm" | "native"
    device: str = "cuda:0"
    seed: int = 0

    def resolve_model(self) -> str:
        if os.path.exists(self.model):
            return self.model
        preset = DEEPSEEK_MODELS.get(self.model)
        return preset["repo"] if preset else self.model

    def uses_chat_template(self) -> bool:
        preset = DEEPSEEK_MODELS.get(self.model, {})
        return bool(self.use_chat_template or preset.get("chat", False))

    def native_shape(self) -> str:
        return DEEPSEEK_MODELS.get(self.model, {}).get("shape", "tiny")


class VLLMInferenceEngine:
    def __init__(self, config: Optional[VLLMInferenceConfig] = None):
        self.config = config or VLLMInferenceConfig()
        self._llm = None
        self._params = None
        self._native = None
        self._error: Optional[BaseException] = None

    # ------------------------------------------------------------ state
    def is_available(self) -> bool:
        """True once a model (vLLM or native) is loaded."""
        return self._llm is not None or self._native is not None

    def availability_error(self) -> Optional[str]:
        if self.is_available():
            return None
        if self.config.backend == "vllm" and not vllm_available():
            return "vllm package is not installed"
        if self._error is not None:
            return f"model load failed: {self._error}"
        return "model not loaded yet"

    def load(self) -> None:
        """Loads the model now (otherwise the first generation without echo does)."""
        if self.is_available():
            return
        if self._error is not None:
            raise RuntimeError(self.availability_error())
        c = self.config
        if c.backend == "native":
            try:
                from .rl.rollout import RolloutConfig, RolloutEngine

                eng = RolloutEngine(RolloutConfig(inference_backend="native", model=c.native_shape(),
                                                  max_new_tokens=c.max_new_tokens, temperature=c.temperature,
                                                  max_batch_size=c.max_batch_size, device=c.device, seed=c.seed))
                st = eng.initialize()
                if not st.ok() or not eng.is_native_available():
                    raise RuntimeError(f"native engine unavailable: {st}")
                self._native = eng
            except Exception as e:  # no GPU, no build, ...
                self._error = e
                raise RuntimeError(self.availability_error()) from e
            return
        if not vllm_available():
            raise RuntimeError("vllm is not installed; install it, use backend='native', or keep "
                               "fallback_to_echo=True for the echo backend")
        try:
            from vllm import LLM, SamplingParams

            self._llm = LLM(model=c.resolve_model(), tensor_parallel_size=c.tensor_parallel_size, dtype=c.dtype,
                            trust_remote_code=c.trust_remote_code, gpu_memory_utilization=c.gpu_memory_utilization,
                            max_model_len=c.max_model_len)
            self._params = SamplingParams(temperature=c.temperature, top_p=c.top_p,
                                          top_k=c.top_k if c.top_k > 0 else -1, max_tokens=c.max_new_tokens)
        except Exception as e:  # weights missing, out of memory, driver mismatch ...
            self._error = e
            raise RuntimeError(self.availability_error()) from e

    # ------------------------------------------------------------ generation
    def _chat(self, prompt: str) -> str:
        if self._llm is None or not self.config.uses_chat_template():
            return prompt
        tok = self._llm.get_tokenizer()
        return tok.apply_chat_template([{"role": "user", "content": prompt}], tokenize=False,
                                       add_generation_prompt=True)

    def generate(self, prompt: str) -> str:
        return self.generate_batch([prompt])[0]

    def generate_batch(self, prompts: Sequence[str]) -> List[str]:
        prompts = list(prompts)
        if not prompts:
            return []
        if not self.is_available():
            if self.config.backend == "native" and self._error is None:
                try:  # the native engine is cheap to bring up: try it before echoing
                    self.load()
                except RuntimeError:
                    if not self.config.fallback_to_echo:
                        raise
            if not self.is_available():
                if self.config.fallback_to_echo:
                    return [ECHO_PREFIX + p for p in prompts]
                self.load()
        if self._native is not None:
            return list(self._native.generate_batch(prompts))
        outs = self._llm.generate([self._chat(p) for p in prompts], self._params, use_tqdm=False)
        return [o.outputs[0].text for o in outs]


__all__ = ["DEEPSEEK_MODELS", "vllm_available", "VLLMInferenceConfig", "VLLMInferenceEngine"]
