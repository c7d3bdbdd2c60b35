"""Checkpoint tensor inventory (Hugging Face names and shapes).

Parity: these are the tensor names the reference's strict loader expects
(``nanovllm/utils/loader.py:52-151``; the official 0.8B audit lists 488 keys,
297 target params and 15 ``mtp.*`` keys, ``docs/qwen35-08b-validation-report.md:34-43``).
The names are fixed by the checkpoint format, so they are the same here.
"""

from __future__ import annotations

from typing import Any


def _g(cfg, name, default=None):
    return cfg.get(name, default) if isinstance(cfg, dict) else getattr(cfg, name, default)


def _attn_shapes(prefix: str, cfg, gated: bool) -> dict[str, tuple[tuple[int, ...], str]]:
    h = _g(cfg, "hidden_size")
    hq = _g(cfg, "num_attention_heads")
    hkv = _g(cfg, "num_key_value_heads")
    hd = _g(cfg, "head_dim")
    norm_kind = "zero_norm" if gated else "one_norm"
    return {
        f"{prefix}.q_proj.weight": ((hq * hd * (2 if gated else 1), h), "matrix"),
        f"{prefix}.k_proj.weight": ((hkv * hd, h), "matrix"),
        f"{prefix}.v_proj.weight": ((hkv * hd, h), "matrix"),
        f"{prefix}.o_proj.weight": ((h, hq * hd), "matrix"),
        f"{prefix}.q_norm.weight": ((hd,), norm_kind),
        f"{prefix}.k_norm.weight": ((hd,), norm_kind),
    }


def _mlp_shapes(prefix: str, cfg) -> dict[str, tuple[tuple[int, ...], str]]:
    h = _g(cfg, "hidden_size")
    i = _g(cfg, "intermediate_size")
    return {
        f"{prefix}.gate_proj.weight": ((i, h), "matrix"),
        f"{prefix}.up_proj.weight": ((i, h), "matrix"),
        f"{prefix}.down_proj.weight": ((h, i), "matrix"),
    }


def _gdn_shapes(prefix: str, cfg) -> dict[str, tuple[tuple[int, ...], str]]:
    h = _g(cfg, "hidden_size")
    hk = _g(cfg, "linear_num_key_heads")
    hv = _g(cfg, "linear_num_value_heads")
    dk = _g(cfg, "linear_key_head_dim")
    dv = _g(cfg, "linear_value_head_dim")
    kw = _g(cfg, "linear_conv_kernel_dim", 4)
    conv_dim = 2 * hk * dk + hv * dv
    return {
        f"{prefix}.in_proj_qkv.weight": ((conv_dim, h), "matrix"),
        f"{prefix}.in_proj_z.weight": ((hv * dv, h), "matrix"),
        f"{prefix}.in_proj_b.weight": ((hv, h), "matrix"),
        f"{prefix}.in_proj_a.weight": ((hv, h), "matrix"),
        f"{prefix}.conv1d.weight": ((conv_dim, 1, kw), "matrix"),
        f"{prefix}.A_log": ((hv,), "a_log"),
        f"{prefix}.dt_bias": ((hv,), "dt_bias"),
        f"{prefix}.norm.weight": ((dv,), "one_norm"),
        f"{prefix}.out_proj.weight": ((h, hv * dv), "matrix"),
    }


def hf_parameter_shapes(cfg: Any, include_mtp: bool = True) -> dict[str, tuple[tuple[int, ...], str]]:
    """``{hf_name: (shape, init_kind)}`` for the text model (+ MTP head)."""
    mt = _g(cfg, "model_type")
    h = _g(cfg, "hidden_size")
    v = _g(cfg, "vocab_size")
    hybrid = mt in ("qwen3_5_text", "qwen3_5")
    norm_kind = "zero_norm" if hybrid else "one_norm"
    out: dict[str, tuple[tuple[int, ...], str]] = {
        "model.embed_tokens.weight": ((v, h), "matrix"),
        "model.norm.weight": ((h,), norm_kind),
    }
    if not _g(cfg, "tie_word_embeddings", False):
        out["lm_head.weight"] = ((v, h), "matrix")
    layer_types = _g(cfg, "layer_types", None) or ["full_attention"] * _g(cfg, "num_hidden_layers")
    for i, kind in enumerate(layer_types):
        p = f"model.layers.{i}"
        out[f"{p}.input_layernorm.weight"] = ((h,), norm_kind)
        out[f"{p}.post_attention_layernorm.weight"] = ((h,), norm_kind)
        if kind == "linear_attention":
            out.update(_gdn_shapes(f"{p}.linear_attn", cfg))
        else:
            out.update(_attn_shapes(f"{p}.self_attn", cfg, gated=hybrid))
        out.update(_mlp_shapes(f"{p}.mlp", cfg))
    if hybrid and include_mtp and int(_g(cfg, "mtp_num_hidden_layers", 0) or 0) > 0:
        out["mtp.fc.weight"] = ((h, 2 * h), "matrix")
        out["mtp.pre_fc_norm_embedding.weight"] = ((h,), "zero_norm")
        out["mtp.pre_fc_norm_hidden.weight"] = ((h,), "zero_norm")
        out["mtp.norm.weight"] = ((h,), "zero_norm")
        out["mtp.layers.0.input_layernorm.weight"] = ((h,), "zero_norm")
        out["mtp.layers.0.post_attention_layernorm.weight"] = ((h,), "zero_norm")
        out.update(_attn_shapes("mtp.layers.0.self_attn", cfg, gated=True))
        out.update(_mlp_shapes("mtp.layers.0.mlp", cfg))
    return out
