"""Strict Hugging Face safetensors loading against the official Qwen3.5 checkpoint layout.

The official Qwen3.5-0.8B index has 488 tensors: 320 of the text model under
``model.language_model.``, 15 of the MTP head under ``mtp.`` and 153 of the vision tower under
``model.visual.`` (the reference's audit, ``tests/audit_qwen35_official_index.py``, reports 488 keys,
168 skipped = visual + MTP, 15 MTP keys).  These tests write a checkpoint with exactly that naming
and those counts -- the 24-layer 3:1 hybrid structure of the 0.8B model with small dimensions so the
file stays tiny -- and check the strict loader end to end: 0 missing / 0 unexpected for the target
and for the MTP head, visual / MTP / ``*_scale_inv`` tensors skipped, a dropped tensor or a stray
tensor failing the load by name, the tied-embedding alias, and the dense Qwen3 layout.  The loaded
parameters are checked against the checkpoint tensors they were packed from.
"""

import os

import pytest
import torch
from safetensors.torch import save_file

from inference_systems_b200.config import HFConfig, _text_defaults, load_hf_config
from inference_systems_b200.models.registry import create_model, normalize_hf_config
from inference_systems_b200.models.weights import hf_parameter_shapes
from inference_systems_b200.utils.loader import load_model

OFFICIAL_TEXT_KEYS, OFFICIAL_MTP_KEYS, OFFICIAL_VISUAL_KEYS = 320, 15, 153


def _cfg(tied=True):
    """The 0.8B layout (24 layers, every 4th full attention, MTP head) at small dimensions."""
    types = ["full_attention" if (i + 1) % 4 == 0 else "linear_attention" for i in range(24)]
    text = dict(model_type="qwen3_5_text", vocab_size=96, hidden_size=64, intermediate_size=128,
                num_hidden_layers=24, layer_types=types, num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                linear_num_key_heads=2, linear_num_value_heads=2, linear_key_head_dim=16, linear_value_head_dim=16,
                linear_conv_kernel_dim=4, rms_norm_eps=1e-6, max_position_embeddings=512,
                tie_word_embeddings=tied, mtp_num_hidden_layers=1, dtype="float32",
                rope_parameters={"rope_theta": 10_000_000, "partial_rotary_factor": 0.25})
    return {"model_type": "qwen3_5", "architectures": ["Qwen3_5ForConditionalGeneration"], "text_config": text,
            "tie_word_embeddings": tied}


def _official_tensors(cfg: dict, seed=0) -> dict[str, torch.Tensor]:
    """HF-named tensors with the official prefixes, plus the vision tower's and FP8 scale tensors."""
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name, (shape, _kind) in hf_parameter_shapes(cfg["text_config"], include_mtp=True).items():
        t = torch.randn(shape, generator=g)
        out[name if name.startswith("mtp.") or name == "lm_head.weight"
            else "model.language_model." + name[len("model."):]] = t
    for i in range(OFFICIAL_VISUAL_KEYS):  # stand-ins for the vision tower's tensors
        out[f"model.visual.blocks.{i // 9}.t{i % 9}.weight"] = torch.zeros(2)
    out["model.language_model.layers.0.mlp.down_proj.weight_scale_inv"] = torch.ones(1)
    return out


def _write(tmp_path, tensors, cfg):
    import json

    d = str(tmp_path)
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f)
    save_file({k: v.contiguous() for k, v in tensors.items()}, os.path.join(d, "model.safetensors"))
    return d


def _target(cfg):
    text, caps = normalize_hf_config(load_hf_config(cfg))
    text = HFConfig(text)  # the same steps as the engine's Config
    _text_defaults(text)
    return create_model(text, caps), text


def test_official_inventory_counts():
    cfg = _cfg()
    names = _official_tensors(cfg)
    text = [n for n in names if n.startswith("model.language_model.") and not n.endswith("_scale_inv")]
    mtp = [n for n in names if n.startswith("mtp.")]
    vis = [n for n in names if n.startswith("model.visual.")]
    assert (len(text), len(mtp), len(vis)) == (OFFICIAL_TEXT_KEYS, OFFICIAL_MTP_KEYS, OFFICIAL_VISUAL_KEYS)
    assert len(text) + len(mtp) + len(vis) == 488


def test_strict_load_of_the_official_layout(tmp_path):
    cfg = _cfg()
    tensors = _official_tensors(cfg)
    d = _write(tmp_path, tensors, cfg)
    model, text = _target(cfg)
    report = load_model(model, d, strict=True)
    assert report.missing_tensors == [] and report.unexpected_tensors == []
    assert len(report.consumed_tensors) == OFFICIAL_TEXT_KEYS
    skipped = set(report.skipped_tensors)
    assert sum(n.startswith("mtp.") for n in skipped) == OFFICIAL_MTP_KEYS
    assert sum(n.startswith("model.visual.") for n in skipped) == OFFICIAL_VISUAL_KEYS
    assert any(n.endswith("_scale_inv") for n in skipped)
    # packed parameters hold exactly the checkpoint tensors they were built from
    lay0 = model.layers[0].mixer
    qkv = tensors["model.language_model.layers.0.linear_attn.in_proj_qkv.weight"]
    assert torch.equal(lay0.in_proj[: qkv.shape[0]], qkv)
    att = model.layers[3].mixer
    q = tensors["model.language_model.layers.3.self_attn.q_proj.weight"]
    assert torch.equal(att.qkv_proj[: q.shape[0]], q)
    assert torch.equal(model.embed_tokens, tensors["model.language_model.embed_tokens.weight"])
    # the tied LM head is a view of the embedding table
    assert model.lm_head_weight().data_ptr() == model.embed_tokens.data_ptr()


def test_mtp_head_loads_only_its_fifteen_tensors(tmp_path):
    from inference_systems_b200.models.qwen3_5_mtp import Qwen3_5MTP

    cfg = _cfg()
    tensors = _official_tensors(cfg)
    d = _write(tmp_path, tensors, cfg)
    model, text = _target(cfg)
    mtp = Qwen3_5MTP(text, model)
    report = load_model(mtp, d, strict=True)
    assert report.missing_tensors == [] and report.unexpected_tensors == []
    assert len(report.consumed_tensors) == OFFICIAL_MTP_KEYS
    assert torch.equal(mtp.fc, tensors["mtp.fc.weight"])


def test_a_dropped_tensor_fails_the_strict_load_by_name(tmp_path):
    cfg = _cfg()
    tensors = _official_tensors(cfg)
    del tensors["model.language_model.layers.5.linear_attn.dt_bias"]
    d = _write(tmp_path, tensors, cfg)
    model, _ = _target(cfg)
    with pytest.raises(RuntimeError, match=r"model\.layers\.5\.linear_attn\.dt_bias"):
        load_model(model, d, strict=True)
    report = load_model(_target(cfg)[0], d, strict=False)
    assert report.missing_tensors == ["model.layers.5.linear_attn.dt_bias"]


def test_a_stray_tensor_fails_the_strict_load_by_name(tmp_path):
    cfg = _cfg()
    tensors = _official_tensors(cfg)
    tensors["model.language_model.typo.weight"] = torch.ones(1)
    d = _write(tmp_path, tensors, cfg)
    with pytest.raises(RuntimeError, match=r"model\.typo\.weight"):
        load_model(_target(cfg)[0], d, strict=True)


def test_tied_alias_and_untied_head(tmp_path):
    cfg = _cfg(tied=True)
    tensors = _official_tensors(cfg)
    tensors["lm_head.weight"] = tensors["model.language_model.embed_tokens.weight"].clone()
    report = load_model(_target(cfg)[0], _write(tmp_path, tensors, cfg), strict=True)
    assert "lm_head.weight" in report.consumed_tensors       # an alias of the tied embedding
    untied = _cfg(tied=False)
    t2 = _official_tensors(untied)
    assert "lm_head.weight" in t2
    (tmp_path / "u").mkdir()
    model, _ = _target(untied)
    load_model(model, _write(tmp_path / "u", t2, untied), strict=True)
    assert torch.equal(model.lm_head, t2["lm_head.weight"])
    del t2["lm_head.weight"]
    (tmp_path / "v").mkdir()
    with pytest.raises(RuntimeError, match="lm_head.weight"):
        load_model(_target(untied)[0], _write(tmp_path / "v", t2, untied), strict=True)


def test_dense_qwen3_layout(tmp_path):
    cfg = dict(model_type="qwen3", architectures=["Qwen3ForCausalLM"], vocab_size=64, hidden_size=32,
               intermediate_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=8,
               rms_norm_eps=1e-6, max_position_embeddings=256, tie_word_embeddings=True, dtype="float32",
               rope_theta=10000.0)
    g = torch.Generator().manual_seed(1)
    tensors = {n: torch.randn(s, generator=g) for n, (s, _) in hf_parameter_shapes(cfg).items()}
    d = _write(tmp_path, tensors, cfg)
    model, _ = _target(cfg)
    report = load_model(model, d, strict=True)
    assert report.missing_tensors == [] and report.unexpected_tensors == []
    assert len(report.consumed_tensors) == len(tensors) == 2 + 2 * 11
