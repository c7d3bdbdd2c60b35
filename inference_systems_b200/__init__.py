"""B200-native serving engine for Qwen3.5 hybrid (Gated DeltaNet + attention) and Qwen3 models.

Public API (parity: ``nanovllm/__init__.py:1-3``): ``LLM``, ``SamplingParams``,
``AsyncLLMEngine``, ``RequestStream``, ``StreamOutput``.
"""

from inference_systems_b200.sampling_params import SamplingParams

__version__ = "0.1.0"


def __getattr__(name):
    if name == "LLM":
        from inference_systems_b200.llm import LLM
        return LLM
    if name in ("AsyncLLMEngine", "RequestStream", "StreamOutput"):
        from inference_systems_b200 import async_llm
        return getattr(async_llm, name)
    raise AttributeError(name)


__all__ = ["LLM", "SamplingParams", "AsyncLLMEngine", "RequestStream", "StreamOutput"]
