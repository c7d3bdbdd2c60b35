"""Model-config normalisation and model factory.

Parity: the reference normalises Hugging Face configs in
``nanovllm/models/registry.py:25-88`` (text sub-config extraction, multimodal
wrapper mapped to the text runtime, ``layer_types`` validation) and builds the
model in ``registry.py:91-100``.  The capability record below carries the same
facts; the factory builds this package's models.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any


@dataclass(frozen=True, slots=True)
class ModelCapabilities:
    architecture: str
    model_type: str
    layer_types: tuple[str, ...]
    full_attention_layer_indices: tuple[int, ...]
    linear_attention_layer_indices: tuple[int, ...]
    has_recurrent_state: bool
    supports_mrope: bool
    mtp_num_hidden_layers: int

    @property
    def is_hybrid(self) -> bool:
        return bool(self.linear_attention_layer_indices)

    @property
    def num_layers(self) -> int:
        return len(self.layer_types)


_LAYER_KINDS = {"full_attention", "linear_attention", "sliding_attention"}


def _get(cfg: Any, name: str, default=None):
    if isinstance(cfg, dict):
        return cfg.get(name, default)
    return getattr(cfg, name, default)


def normalize_hf_config(full_config: Any) -> tuple[Any, ModelCapabilities]:
    """Return ``(text_config, capabilities)`` for a Qwen3 / Qwen3.5 config.

    A multimodal Qwen3.5 wrapper (``model_type == "qwen3_5"`` with a
    ``text_config``) maps to the text-only causal LM; vision weights are not
    part of this runtime.
    """
    text_config = _get(full_config, "text_config", None) or full_config
    archs = _get(full_config, "architectures", None) or _get(text_config, "architectures", None)
    model_type = _get(text_config, "model_type", None) or _get(full_config, "model_type", "")
    outer_type = _get(full_config, "model_type", "")
    if model_type == "qwen3_5_text" or outer_type == "qwen3_5" or model_type == "qwen3_5":
        architecture = archs[0] if archs else "Qwen3_5ForCausalLM"
        if architecture == "Qwen3_5ForConditionalGeneration":
            architecture = "Qwen3_5ForCausalLM"
    elif model_type == "qwen3":
        architecture = archs[0] if archs else "Qwen3ForCausalLM"
    else:
        raise ValueError(f"unsupported model_type: {model_type!r}")

    num_layers = int(_get(text_config, "num_hidden_layers"))
    raw = _get(text_config, "layer_types", None)
    if raw is None:
        layer_types = ("full_attention",) * num_layers
    else:
        layer_types = tuple(raw)
        if len(layer_types) != num_layers:
            raise ValueError(f"layer_types has {len(layer_types)} entries for {num_layers} layers")
    unknown = sorted(set(layer_types) - _LAYER_KINDS)
    if unknown:
        raise ValueError(f"unsupported layer types: {unknown}")
    full = tuple(i for i, t in enumerate(layer_types) if t != "linear_attention")
    linear = tuple(i for i, t in enumerate(layer_types) if t == "linear_attention")
    rope = _get(text_config, "rope_parameters", None) or {}
    caps = ModelCapabilities(
        architecture=architecture,
        model_type=model_type,
        layer_types=layer_types,
        full_attention_layer_indices=full,
        linear_attention_layer_indices=linear,
        has_recurrent_state=bool(linear),
        supports_mrope=bool(rope.get("mrope_interleaved", False) or rope.get("mrope_section")),
        mtp_num_hidden_layers=int(_get(text_config, "mtp_num_hidden_layers", 0) or 0),
    )
    return text_config, caps


def create_model(text_config: Any, caps: ModelCapabilities, *, tp_rank: int = 0, tp_size: int = 1):
    if caps.architecture == "Qwen3_5ForCausalLM":
        from inference_systems_b200.models.qwen3_5 import Qwen3_5ForCausalLM

        return Qwen3_5ForCausalLM(text_config, caps, tp_rank=tp_rank, tp_size=tp_size)
    if caps.architecture == "Qwen3ForCausalLM":
        from inference_systems_b200.models.qwen3 import Qwen3ForCausalLM

        return Qwen3ForCausalLM(text_config, caps, tp_rank=tp_rank, tp_size=tp_size)
    raise ValueError(f"unsupported architecture: {caps.architecture!r}")
