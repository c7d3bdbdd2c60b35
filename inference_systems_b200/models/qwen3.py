"""Dense Qwen3 causal LM (parity: ``nanovllm/models/qwen3.py:14-216``).

Shares the decoder body with the hybrid model; every layer is full attention
with merged q|k|v, per-head q/k RMSNorm (plain weights), full-width RoPE.
"""

from inference_systems_b200.models.qwen3_5 import Qwen3ForCausalLM

__all__ = ["Qwen3ForCausalLM"]
