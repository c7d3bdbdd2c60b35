"""``LLM`` -- the synchronous public entry point (parity: ``nanovllm/llm.py:4-5``)."""

from inference_systems_b200.engine.llm_engine import LLMEngine


class LLM(LLMEngine):
    pass
