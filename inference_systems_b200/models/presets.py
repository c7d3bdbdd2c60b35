"""Named model shapes and random-init checkpoint writer.

The shapes are the public Qwen3.5 / Qwen3 text configurations that the
reference serves (the reference's own docs recover the 0.8B dims:
``docs/qwen35-08b-validation-report.md:20``, ``docs/mtp-phase-profiling.md:143-144``,
``cuda_kernels/gemm/src/gemm_bench.cu:45-57``).  ``tiny`` is the 4-layer CPU
oracle shape.  ``write_random_checkpoint`` produces a Hugging-Face-layout
directory (``config.json`` + ``model.safetensors``) with N(0, 0.02) weights,
zero-centred norms at zero, gated-norm weights at one, ``A_log = 0`` and
``dt_bias = 1`` -- the same initialisation rule the reference's GPU tests use
for their tiny checkpoints (``tests/test_qwen35_model_runner_e2e.py:64-123``).
"""

from __future__ import annotations

import copy
import json
import os
from typing import Any

import torch


def _hybrid_layer_types(n: int, interval: int = 4) -> list[str]:
    return ["full_attention" if (i + 1) % interval == 0 else "linear_attention" for i in range(n)]


_QWEN35_COMMON = {
    "model_type": "qwen3_5_text",
    "architectures": ["Qwen3_5ForCausalLM"],
    "hidden_act": "silu",
    "rms_norm_eps": 1e-6,
    "attention_bias": False,
    "linear_conv_kernel_dim": 4,
    "rope_parameters": {
        "rope_type": "default",
        "rope_theta": 10_000_000,
        "partial_rotary_factor": 0.25,
    },
    "dtype": "bfloat16",
    "eos_token_id": 248044,
    "mtp_num_hidden_layers": 1,
}

PRESETS: dict[str, dict[str, Any]] = {
    # the CPU oracle shape (4 layers, hidden 256)
    "tiny": {
        **_QWEN35_COMMON,
        "vocab_size": 1024,
        "hidden_size": 256,
        "intermediate_size": 512,
        "num_hidden_layers": 4,
        "layer_types": ["linear_attention"] * 3 + ["full_attention"],
        "num_attention_heads": 4,
        "num_key_value_heads": 2,
        "head_dim": 64,
        "linear_num_key_heads": 4,
        "linear_num_value_heads": 4,
        "linear_key_head_dim": 64,
        "linear_value_head_dim": 64,
        "max_position_embeddings": 4096,
        "tie_word_embeddings": True,
        "eos_token_id": 1023,
        "dtype": "float32",
    },
    # Same as tiny but with head dims of the real family (128 GDN / 256 attn),
    # used by GPU kernel tests that need production head sizes on a small model.
    "tiny_hd": {
        **_QWEN35_COMMON,
        "vocab_size": 4096,
        "hidden_size": 512,
        "intermediate_size": 1024,
        "num_hidden_layers": 4,
        "layer_types": ["linear_attention"] * 3 + ["full_attention"],
        "num_attention_heads": 4,
        "num_key_value_heads": 2,
        "head_dim": 256,
        "linear_num_key_heads": 4,
        "linear_num_value_heads": 4,
        "linear_key_head_dim": 128,
        "linear_value_head_dim": 128,
        "max_position_embeddings": 8192,
        "tie_word_embeddings": True,
        "eos_token_id": 4095,
    },
    "qwen3_5-0.8b": {
        **_QWEN35_COMMON,
        "vocab_size": 248320,
        "hidden_size": 1024,
        "intermediate_size": 3584,
        "num_hidden_layers": 24,
        "layer_types": _hybrid_layer_types(24),
        "num_attention_heads": 8,
        "num_key_value_heads": 2,
        "head_dim": 256,
        "linear_num_key_heads": 16,
        "linear_num_value_heads": 16,
        "linear_key_head_dim": 128,
        "linear_value_head_dim": 128,
        "max_position_embeddings": 262144,
        "tie_word_embeddings": True,
    },
    "qwen3_5-9b": {
        **_QWEN35_COMMON,
        "vocab_size": 248320,
        "hidden_size": 4096,
        "intermediate_size": 12288,
        "num_hidden_layers": 32,
        "layer_types": _hybrid_layer_types(32),
        "num_attention_heads": 16,
        "num_key_value_heads": 4,
        "head_dim": 256,
        "linear_num_key_heads": 16,
        "linear_num_value_heads": 32,
        "linear_key_head_dim": 128,
        "linear_value_head_dim": 128,
        "max_position_embeddings": 262144,
        "tie_word_embeddings": False,
    },
    "qwen3_5-27b": {
        **_QWEN35_COMMON,
        "vocab_size": 248320,
        "hidden_size": 5120,
        "intermediate_size": 17408,
        "num_hidden_layers": 64,
        "layer_types": _hybrid_layer_types(64),
        "num_attention_heads": 24,
        "num_key_value_heads": 4,
        "head_dim": 256,
        "linear_num_key_heads": 16,
        "linear_num_value_heads": 48,
        "linear_key_head_dim": 128,
        "linear_value_head_dim": 128,
        "max_position_embeddings": 262144,
        "tie_word_embeddings": False,
    },
    # Dense Qwen3 (the reference's second family, ``nanovllm/models/qwen3.py``).
    "qwen3-0.6b": {
        "model_type": "qwen3",
        "architectures": ["Qwen3ForCausalLM"],
        "vocab_size": 151936,
        "hidden_size": 1024,
        "intermediate_size": 3072,
        "num_hidden_layers": 28,
        "num_attention_heads": 16,
        "num_key_value_heads": 8,
        "head_dim": 128,
        "hidden_act": "silu",
        "rms_norm_eps": 1e-6,
        "attention_bias": False,
        "rope_theta": 1_000_000,
        "max_position_embeddings": 40960,
        "tie_word_embeddings": True,
        "dtype": "bfloat16",
        "eos_token_id": 151645,
    },
    "qwen3-tiny": {
        "model_type": "qwen3",
        "architectures": ["Qwen3ForCausalLM"],
        "vocab_size": 1024,
        "hidden_size": 256,
        "intermediate_size": 512,
        "num_hidden_layers": 2,
        "num_attention_heads": 4,
        "num_key_value_heads": 2,
        "head_dim": 64,
        "hidden_act": "silu",
        "rms_norm_eps": 1e-6,
        "attention_bias": False,
        "rope_theta": 1_000_000,
        "max_position_embeddings": 4096,
        "tie_word_embeddings": True,
        "dtype": "float32",
        "eos_token_id": 1023,
    },
}


def preset(name: str, **overrides) -> dict[str, Any]:
    if name not in PRESETS:
        raise KeyError(f"unknown preset {name!r}; choose from {sorted(PRESETS)}")
    cfg = copy.deepcopy(PRESETS[name])
    cfg.update(overrides)
    if "num_hidden_layers" in overrides and "layer_types" not in overrides and "layer_types" in cfg:
        cfg["layer_types"] = _hybrid_layer_types(cfg["num_hidden_layers"])
    return cfg


def write_config(path: str, cfg: dict[str, Any]) -> None:
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=2)


def random_state_dict(cfg: dict[str, Any], *, seed: int = 0, dtype: torch.dtype | None = None,
                      include_mtp: bool = True, std: float = 0.02) -> dict[str, torch.Tensor]:
    """Random-init HF-named tensors for ``cfg`` (N(0, std) for matrices)."""
    from inference_systems_b200.models.weights import hf_parameter_shapes

    if dtype is None:
        dtype = torch.float32 if cfg.get("dtype") == "float32" else torch.bfloat16
    gen = torch.Generator().manual_seed(seed)
    out: dict[str, torch.Tensor] = {}
    for name, (shape, kind) in hf_parameter_shapes(cfg, include_mtp=include_mtp).items():
        if kind == "matrix":
            t = torch.empty(shape, dtype=torch.float32).normal_(0.0, std, generator=gen)
        elif kind == "zero_norm":
            t = torch.zeros(shape)
        elif kind == "one_norm":
            t = torch.ones(shape)
        elif kind == "a_log":
            t = torch.zeros(shape)
        elif kind == "dt_bias":
            t = torch.ones(shape)
        else:  # pragma: no cover
            raise AssertionError(kind)
        keep_fp32 = kind == "a_log"
        out[name] = t if keep_fp32 else t.to(dtype)
    return out


def write_random_checkpoint(path: str, cfg: dict[str, Any] | str, *, seed: int = 0,
                            include_mtp: bool = True, dtype: torch.dtype | None = None) -> str:
    """Write ``config.json`` + ``model.safetensors`` of random weights."""
    from safetensors.torch import save_file

    if isinstance(cfg, str):
        cfg = preset(cfg)
    write_config(path, cfg)
    sd = random_state_dict(cfg, seed=seed, dtype=dtype, include_mtp=include_mtp)
    save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(path, "model.safetensors"))
    return path
