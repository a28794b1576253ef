"""vLLM wrapper: presets, config resolution, echo fallback (no model weights
needed), and the failure path without fallback."""
import pytest

from turbol_b200.vllm_inference import DEEPSEEK_MODELS, VLLMInferenceConfig, VLLMInferenceEngine, vllm_available


def test_presets():
    for k in ("deepseek-r1-distill-qwen-1.5b", "deepseek-r1-distill-qwen-7b", "deepseek-v2-lite"):
        assert k in DEEPSEEK_MODELS
    assert DEEPSEEK_MODELS["deepseek-r1-distill-qwen-1.5b"]["repo"].startswith("deepseek-ai/")


def test_config_resolution(tmp_path):
    c = VLLMInferenceConfig(model="deepseek-r1-distill-qwen-1.5b")
    assert c.resolve_model() == "deepseek-ai/DeepSeek-R1-Distill-Qwen-1.5B" and c.uses_chat_template()
    assert VLLMInferenceConfig(model="org/custom").resolve_model() == "org/custom"
    assert VLLMInferenceConfig(model=str(tmp_path)).resolve_model() == str(tmp_path)
    d = VLLMInferenceConfig()
    assert (d.tensor_parallel_size, d.temperature, d.top_k, d.max_batch_size) == (1, 1.0, -1, 256)
    assert d.max_new_tokens > 0


def test_echo_fallback():
    e = VLLMInferenceEngine()
    assert e.generate("hello") == "[VLLMInferenceEngine] hello"
    assert e.generate_batch(["a", "b"]) == ["[VLLMInferenceEngine] a", "[VLLMInferenceEngine] b"]
    assert e.generate_batch([]) == []
    assert not e.is_available()


def test_no_fallback_raises_without_vllm():
    if vllm_available():
        pytest.skip("vllm is installed: this would load a model")
    e = VLLMInferenceEngine(VLLMInferenceConfig(fallback_to_echo=False))
    with pytest.raises(RuntimeError, match="vllm"):
        e.generate("hello")


def test_native_backend_without_gpu_echoes():
    import torch

    if torch.cuda.is_available():
        pytest.skip("covered by the GPU test")
    e = VLLMInferenceEngine(VLLMInferenceConfig(backend="native"))
    out = e.generate("x")
    assert isinstance(out, str)


@pytest.mark.gpu
def test_native_backend_generates(dev):
    e = VLLMInferenceEngine(VLLMInferenceConfig(model="tiny-random", backend="native", max_new_tokens=8,
                                                max_batch_size=4))
    outs = e.generate_batch(["hi", "there"])
    assert e.is_available() and len(outs) == 2 and all(isinstance(o, str) for o in outs)
