"""Model families: Hugging Face config normalisation and the model factory.

Behavioural parity with ``nanovllm/models/registry.py:9-100``: a Qwen3 or
Qwen3.5 Hugging Face config (including the multimodal Qwen3.5 wrapper, whose
text part is served) becomes a text config plus a ``ModelCapabilities`` record
(the capability fields are the reference's), and the factory builds the model.

Design: each supported family is one ``ModelFamily`` row -- the ``model_type``
values it accepts, the architecture names it answers to (with aliases that map
a wrapper architecture to the text runtime) and how its layers are laid out.
Normalisation is a lookup in that table followed by one layer-plan check, so
adding a family is adding a row.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable


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


def _field(cfg: Any, name: str, default=None):
    return cfg.get(name, default) if isinstance(cfg, dict) else getattr(cfg, name, default)


def _build_qwen3_5(cfg, caps, tp_rank, tp_size):
    from inference_systems_b200.models.qwen3_5 import Qwen3_5ForCausalLM
    return Qwen3_5ForCausalLM(cfg, caps, tp_rank=tp_rank, tp_size=tp_size)


def _build_qwen3(cfg, caps, tp_rank, tp_size):
    from inference_systems_b200.models.qwen3 import Qwen3ForCausalLM
    return Qwen3ForCausalLM(cfg, caps, tp_rank=tp_rank, tp_size=tp_size)


@dataclass(frozen=True)
class ModelFamily:
    architecture: str                       # the causal-LM runtime this package builds
    model_types: frozenset[str]             # text or wrapper ``model_type`` values that select it
    architecture_aliases: frozenset[str]    # checkpoint architectures served by this runtime
    default_layer_type: str                 # layer kind when the config has no ``layer_types``
    build: Callable


FAMILIES = (
    ModelFamily("Qwen3_5ForCausalLM", frozenset({"qwen3_5_text", "qwen3_5"}),
                frozenset({"Qwen3_5ForCausalLM", "Qwen3_5ForConditionalGeneration"}), "full_attention", _build_qwen3_5),
    ModelFamily("Qwen3ForCausalLM", frozenset({"qwen3"}), frozenset({"Qwen3ForCausalLM"}), "full_attention",
                _build_qwen3),
)
_LAYER_KINDS = frozenset({"full_attention", "linear_attention", "sliding_attention"})


def _family(model_type: str, outer_type: str) -> ModelFamily:
    for fam in FAMILIES:
        if model_type in fam.model_types or outer_type in fam.model_types:
            return fam
    raise ValueError(f"unsupported model_type: {model_type!r}")


def _layer_plan(text_config: Any, fam: ModelFamily) -> tuple[str, ...]:
    n = int(_field(text_config, "num_hidden_layers"))
    declared = _field(text_config, "layer_types", None)
    plan = (fam.default_layer_type,) * n if declared is None else tuple(declared)
    if len(plan) != n:
        raise ValueError(f"layer_types has {len(plan)} entries for {n} layers")
    unknown = sorted(set(plan) - _LAYER_KINDS)
    if unknown:
        raise ValueError(f"unsupported layer types: {unknown}")
    return plan


def normalize_hf_config(full_config: Any) -> tuple[Any, ModelCapabilities]:
    """``(text_config, capabilities)`` of a Qwen3 / Qwen3.5 config (a multimodal wrapper maps to its
    text-only causal LM; vision weights are not part of this runtime)."""
    text_config = _field(full_config, "text_config", None) or full_config
    outer_type = _field(full_config, "model_type", "") or ""
    model_type = _field(text_config, "model_type", None) or outer_type
    fam = _family(model_type, outer_type)
    archs = _field(full_config, "architectures", None) or _field(text_config, "architectures", None) or []
    declared = archs[0] if archs else fam.architecture
    architecture = fam.architecture if declared in fam.architecture_aliases else declared
    plan = _layer_plan(text_config, fam)
    rope = _field(text_config, "rope_parameters", None) or {}
    linear = tuple(i for i, kind in enumerate(plan) if kind == "linear_attention")
    caps = ModelCapabilities(
        architecture=architecture,
        model_type=model_type,
        layer_types=plan,
        full_attention_layer_indices=tuple(i for i in range(len(plan)) if i not in set(linear)),
        linear_attention_layer_indices=linear,
        has_recurrent_state=bool(linear),
        supports_mrope=bool(rope.get("mrope_interleaved") or rope.get("mrope_section")),
        mtp_num_hidden_layers=int(_field(text_config, "mtp_num_hidden_layers", 0) or 0),
    )
    return text_config, caps


def create_model(text_config: Any, caps: ModelCapabilities, *, tp_rank: int = 0, tp_size: int = 1):
    for fam in FAMILIES:
        if fam.architecture == caps.architecture:
            return fam.build(text_config, caps, tp_rank, tp_size)
    raise ValueError(f"unsupported architecture: {caps.architecture!r}")
