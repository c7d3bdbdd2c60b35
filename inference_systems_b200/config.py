"""Engine configuration.

Parity: flag names, defaults and validation rules follow the reference's
``nanovllm/config.py:8-65`` (fields) and ``:67-224`` (validation) so a
reference user can pass the same keyword arguments.  Additional fields used
only by this engine are grouped at the end of the dataclass.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from typing import Any

import torch

from inference_systems_b200.models.registry import ModelCapabilities, normalize_hf_config


class HFConfig(dict):
    """Attribute view over a ``config.json`` dictionary (nested ``text_config`` too)."""

    def __getattr__(self, name):
        try:
            value = self[name]
        except KeyError as exc:
            raise AttributeError(name) from exc
        if isinstance(value, dict) and not isinstance(value, HFConfig):
            value = HFConfig(value)
            self[name] = value
        return value

    def __setattr__(self, name, value):
        self[name] = value

    @property
    def torch_dtype(self) -> torch.dtype:
        name = self.get("dtype") or self.get("torch_dtype") or "bfloat16"
        return {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}[name]


def load_hf_config(model: str | dict) -> HFConfig:
    if isinstance(model, dict):
        return HFConfig(json.loads(json.dumps(model)))
    path = os.path.join(model, "config.json")
    with open(path) as f:
        return HFConfig(json.load(f))


def _text_defaults(text: HFConfig) -> None:
    """Fill Qwen3.5 text defaults that public configs may omit."""
    if text.get("model_type") in ("qwen3_5_text", "qwen3_5"):
        rope = text.get("rope_parameters") or {}
        rope.setdefault("rope_theta", text.get("rope_theta", 10_000_000))
        rope.setdefault("partial_rotary_factor", text.get("partial_rotary_factor", 0.25))
        text["rope_parameters"] = rope
        text.setdefault("linear_conv_kernel_dim", 4)
        text.setdefault("head_dim", 256)
        if text.get("layer_types") is None:
            interval = text.get("full_attention_interval", 4)
            text["layer_types"] = [
                "full_attention" if (i + 1) % interval == 0 else "linear_attention"
                for i in range(text["num_hidden_layers"])
            ]
    text.setdefault("max_position_embeddings", 4096)
    text.setdefault("rms_norm_eps", 1e-6)
    text.setdefault("tie_word_embeddings", False)
    text.setdefault("attention_bias", False)
    if "head_dim" not in text:
        text["head_dim"] = text["hidden_size"] // text["num_attention_heads"]


@dataclass(slots=True)
class Config:
    model: Any
    max_num_batched_tokens: int = 16384
    max_num_seqs: int = 512
    max_model_len: int = 4096
    gpu_memory_utilization: float = 0.9
    tensor_parallel_size: int = 1
    enforce_eager: bool = False
    scheduling_policy: str = "prefill_first"
    waiting_admission_policy: str = "fcfs"
    preemption_policy: str = "lifo"
    hybrid_scheduler_candidate_window: int = 8
    hybrid_scheduler_aging_tokens_per_ms: float = 0.5
    hybrid_scheduler_max_wait_ms: float = 200.0
    hybrid_scheduler_min_saved_tokens: int = 16
    hybrid_scheduler_preemption_penalty: float = 128.0
    hybrid_scheduler_score_source: str = "joint"
    hybrid_scheduler_enable_aging: bool = True
    hybrid_scheduler_enable_hysteresis: bool = True
    hybrid_scheduler_enable_sticky_recovery: bool = True
    enable_scheduler_profiling: bool = False
    scheduler_decision_history_size: int = 4096
    scheduler_target_ttft_ms: float = 200.0
    scheduler_target_tpot_ms: float = 50.0
    slo_prefill_priority_threshold: float = 0.8
    slo_min_prefill_tokens: int = 64
    slo_kv_pressure_threshold: float = 0.9
    slo_queue_pressure_threshold: int = 3
    slo_latency_safety_margin_ms: float = 5.0
    scheduler_ewma_alpha: float = 0.2
    enable_prefix_cache: bool = True
    enable_chunked_prefill: bool = True
    request_metrics_history_size: int = 1024
    full_hf_config: Any = None
    hf_config: Any = None
    model_capabilities: ModelCapabilities | None = None
    eos: int = -1
    kvcache_block_size: int = 256
    prefix_match_unit: int | None = None
    num_kvcache_blocks: int = -1
    max_num_kvcache_blocks: int | None = None
    max_num_state_slots: int = 1
    num_speculative_tokens: int = 0
    speculative_parallel_verify: bool = True
    enable_mtp_phase_profiling: bool = False
    enable_mtp_replay_ssm: bool | None = None  # None: replay records whenever MTP is on
    gdn_decode_backend: str = "auto"
    enable_hybrid_prefix_cache: bool = False
    hybrid_prefix_checkpoint_interval_blocks: int = 8
    hybrid_prefix_checkpoint_interval_tokens: int | None = None
    hybrid_prefix_checkpoint_memory_bytes: int = 0
    hybrid_prefix_checkpoint_dtype: str = "fp32"
    hybrid_prefix_promotion_min_sightings: int = 2
    hybrid_prefix_retention_policy: str = "periodic"
    hybrid_prefix_eviction_policy: str = "lru"
    enable_hybrid_internal_checkpoints: bool = False
    hybrid_prefix_checkpoint_bytes_per_slot: int = field(default=0, init=False)
    # ---- fields specific to this engine ---------------------------------
    load_format: str = "auto"            # "auto": safetensors in ``model``; "dummy": random init
    device: str = "auto"                 # "auto" -> cuda when available, else cpu
    dtype: str | None = None             # override the checkpoint dtype
    seed: int = 0
    max_cudagraph_batch_size: int = 256
    mtp_synthetic_acceptance: float | None = None  # benchmark hook: seeded draft agreement
    dist_port: int = 29533
    dist_timeout_s: float = 120.0

    def __post_init__(self):
        if not isinstance(self.model, dict):
            assert os.path.isdir(self.model), f"model directory not found: {self.model}"
        assert self.kvcache_block_size % 256 == 0
        if self.prefix_match_unit is None:
            self.prefix_match_unit = self.kvcache_block_size
        if self.prefix_match_unit <= 0:
            raise ValueError("prefix_match_unit must be positive")
        if self.kvcache_block_size % self.prefix_match_unit:
            raise ValueError("kvcache_block_size must be divisible by prefix_match_unit")
        assert 1 <= self.tensor_parallel_size <= 8
        assert self.scheduling_policy in ("prefill_first", "decode_first", "slo_aware")
        if self.waiting_admission_policy not in ("fcfs", "hybrid_state_aware"):
            raise ValueError("unsupported waiting admission policy")
        if self.preemption_policy not in ("lifo", "recompute_aware"):
            raise ValueError("unsupported preemption policy")
        if self.hybrid_scheduler_candidate_window <= 0:
            raise ValueError("candidate window must be positive")
        if self.hybrid_scheduler_aging_tokens_per_ms < 0:
            raise ValueError("aging factor must be non-negative")
        if self.hybrid_scheduler_max_wait_ms <= 0:
            raise ValueError("maximum wait must be positive")
        if self.hybrid_scheduler_min_saved_tokens < 0:
            raise ValueError("minimum saved tokens must be non-negative")
        if self.hybrid_scheduler_preemption_penalty < 0:
            raise ValueError("preemption penalty must be non-negative")
        if self.hybrid_scheduler_score_source not in ("joint", "kv_only"):
            raise ValueError("scheduler score source must be joint or kv_only")
        if self.scheduler_decision_history_size < 0:
            raise ValueError("scheduler decision history size cannot be negative")
        assert self.scheduler_target_ttft_ms > 0
        assert self.scheduler_target_tpot_ms > 0
        assert self.slo_prefill_priority_threshold > 0
        assert self.slo_min_prefill_tokens > 0
        assert 0 < self.slo_kv_pressure_threshold <= 1
        assert self.slo_queue_pressure_threshold > 0
        assert self.slo_latency_safety_margin_ms >= 0
        assert 0 < self.scheduler_ewma_alpha <= 1
        assert self.request_metrics_history_size >= 0
        assert self.max_num_kvcache_blocks is None or self.max_num_kvcache_blocks > 0
        assert self.max_num_state_slots > 0
        assert 0 <= self.num_speculative_tokens <= 8
        if self.gdn_decode_backend not in ("torch", "cuda", "auto"):
            raise ValueError("gdn_decode_backend must be torch, cuda, or auto")
        # GDN runs on this engine's sm_100a kernels on GPUs and on the PyTorch recurrence on CPUs;
        # there is no second implementation to switch to on either device.
        on_cuda = (self.device or ("cuda" if torch.cuda.is_available() else "cpu")) == "cuda"
        if on_cuda and self.gdn_decode_backend == "torch":
            raise ValueError("gdn_decode_backend='torch' is not available on GPUs: GDN runs on the sm_100a "
                             "kernels (use 'auto' or 'cuda')")
        if not on_cuda and self.gdn_decode_backend == "cuda":
            raise ValueError("gdn_decode_backend='cuda' needs a CUDA device (use 'auto' or 'torch' on CPU)")
        if not self.speculative_parallel_verify:
            raise ValueError("sequential speculative verification is not provided: the one-pass verify "
                             "(speculative_parallel_verify=True) is lossless and does strictly less work")
        assert self.hybrid_prefix_checkpoint_interval_blocks > 0
        if self.hybrid_prefix_checkpoint_interval_tokens is not None:
            if self.hybrid_prefix_checkpoint_interval_tokens <= 0:
                raise ValueError("checkpoint token interval must be positive")
            if self.hybrid_prefix_checkpoint_interval_tokens % self.prefix_match_unit:
                raise ValueError("checkpoint token interval must align to prefix_match_unit")
        assert self.hybrid_prefix_checkpoint_memory_bytes >= 0
        if self.hybrid_prefix_checkpoint_dtype not in ("fp32", "bf16", "int8"):
            raise ValueError("hybrid prefix checkpoint dtype must be fp32, bf16, or int8")
        if self.hybrid_prefix_promotion_min_sightings < 2:
            raise ValueError("hybrid prefix promotion requires at least two sightings")
        if self.hybrid_prefix_retention_policy not in ("periodic", "adaptive"):
            raise ValueError("unsupported hybrid prefix retention policy")
        if self.hybrid_prefix_eviction_policy not in ("lru", "cost_aware"):
            raise ValueError("unsupported hybrid prefix eviction policy")
        if self.load_format not in ("auto", "dummy"):
            raise ValueError("load_format must be auto or dummy")
        if self.device == "auto":
            self.device = "cuda" if torch.cuda.is_available() else "cpu"

        self.full_hf_config = load_hf_config(self.model)
        text, caps = normalize_hf_config(self.full_hf_config)
        text = HFConfig(text)
        _text_defaults(text)
        if self.dtype is not None:
            text["dtype"] = self.dtype
        self.hf_config = text
        self.model_capabilities = caps
        if self.num_speculative_tokens:
            if not caps.has_recurrent_state:
                raise ValueError("native MTP currently requires Qwen3.5 hybrid state")
            if caps.mtp_num_hidden_layers != 1:
                raise ValueError("native MTP requires exactly one checkpoint MTP layer")
        if self.enable_mtp_replay_ssm is True:
            if not self.num_speculative_tokens:
                raise ValueError("MTP ReplaySSM requires speculative decoding")
            if not self.speculative_parallel_verify:
                raise ValueError("MTP ReplaySSM requires parallel verification")
        if self.enable_hybrid_prefix_cache:
            if self.enable_hybrid_internal_checkpoints and self.max_num_seqs != 1:
                raise ValueError("internal hybrid checkpoints currently require max_num_seqs=1")
            if not self.enable_prefix_cache:
                raise ValueError("hybrid prefix cache requires prefix caching enabled")
            if not caps.has_recurrent_state:
                raise ValueError("hybrid prefix cache requires recurrent model state")
            if self.num_speculative_tokens:
                raise ValueError("hybrid prefix cache MVP does not yet support MTP")
            if self.hybrid_prefix_checkpoint_memory_bytes <= 0:
                raise ValueError("hybrid prefix cache requires a positive checkpoint byte budget")
            self.hybrid_prefix_checkpoint_bytes_per_slot = checkpoint_bytes_per_slot(
                text, caps, self.tensor_parallel_size, self.hybrid_prefix_checkpoint_dtype
            )
            if self.hybrid_prefix_checkpoint_memory_bytes < self.hybrid_prefix_checkpoint_bytes_per_slot:
                raise ValueError(
                    "hybrid prefix checkpoint budget is smaller than one checkpoint "
                    f"({self.hybrid_prefix_checkpoint_bytes_per_slot} bytes)"
                )
        self.max_model_len = min(self.max_model_len, int(text.max_position_embeddings))
        if self.eos == -1:
            eos = text.get("eos_token_id", self.full_hf_config.get("eos_token_id", -1))
            if isinstance(eos, list):
                eos = eos[0] if eos else -1
            self.eos = -1 if eos is None else int(eos)

    @property
    def torch_dtype(self) -> torch.dtype:
        return self.hf_config.torch_dtype


def checkpoint_bytes_per_slot(text, caps: ModelCapabilities, tp: int, dtype: str) -> int:
    """Bytes of one GDN prefix checkpoint per rank (recurrent + scales + conv)."""
    n_lin = len(caps.linear_attention_layer_indices)
    hk = text.linear_num_key_heads // tp
    hv = text.linear_num_value_heads // tp
    dk = text.linear_key_head_dim
    dv = text.linear_value_head_dim
    conv_dim = 2 * hk * dk + hv * dv
    rec_elems = n_lin * hv * dk * dv
    conv_bytes = n_lin * conv_dim * (text.linear_conv_kernel_dim - 1) * text.torch_dtype.itemsize
    if dtype == "fp32":
        rec, scale = rec_elems * 4, 0
    elif dtype == "bf16":
        rec, scale = rec_elems * 2, 0
    else:
        rec, scale = rec_elems, n_lin * hv * dk * 4
    return rec + scale + conv_bytes
