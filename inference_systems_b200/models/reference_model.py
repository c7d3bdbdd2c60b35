"""Stand-alone fp32 Qwen3.5 / Qwen3 forward straight from checkpoint tensors.

This is the correctness oracle for the whole engine: it reads the Hugging
Face-named tensors directly (no packing, no TP sharding, no paged KV, no state
pools), recomputes every sequence from scratch, and runs the Gated DeltaNet
as an explicit token-by-token recurrence -- the same definition the
reference's fp32 oracle implements (``nanovllm/models/qwen35_reference.py:144-386``).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from inference_systems_b200.ops.reference import apply_rope, rope_cos_sin


def _g(cfg, k, d=None):
    return cfg.get(k, d) if isinstance(cfg, dict) else getattr(cfg, k, d)


def _norm(x, w, eps, zero_centered):
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return y * (1.0 + w.float()) if zero_centered else y * w.float()


def _attention(x, sd, p, cfg, hybrid, cos_sin):
    t = x.shape[0]
    hq, hkv, hd = _g(cfg, "num_attention_heads"), _g(cfg, "num_key_value_heads"), _g(cfg, "head_dim")
    eps = _g(cfg, "rms_norm_eps")
    qg = x @ sd[f"{p}.q_proj.weight"].float().t()
    if hybrid:
        qg = qg.view(t, hq, 2 * hd)
        q, gate = qg[..., :hd], qg[..., hd:]
    else:
        q, gate = qg.view(t, hq, hd), None
    k = (x @ sd[f"{p}.k_proj.weight"].float().t()).view(t, hkv, hd)
    v = (x @ sd[f"{p}.v_proj.weight"].float().t()).view(t, hkv, hd)
    q = _norm(q, sd[f"{p}.q_norm.weight"], eps, hybrid)
    k = _norm(k, sd[f"{p}.k_norm.weight"], eps, hybrid)
    pos = torch.arange(t)
    q, k = apply_rope(q, cos_sin, pos), apply_rope(k, cos_sin, pos)
    rep = hq // hkv
    kk, vv = k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1)
    s = torch.einsum("qhd,khd->hqk", q, kk) / math.sqrt(hd)
    s = s.masked_fill(torch.ones(t, t, dtype=torch.bool).triu(1), float("-inf"))
    o = torch.einsum("hqk,khd->qhd", s.softmax(-1), vv)
    if gate is not None:
        o = o * torch.sigmoid(gate)
    return o.reshape(t, hq * hd) @ sd[f"{p}.o_proj.weight"].float().t()


def _gdn(x, sd, p, cfg):
    t = x.shape[0]
    hk, hv = _g(cfg, "linear_num_key_heads"), _g(cfg, "linear_num_value_heads")
    dk, dv = _g(cfg, "linear_key_head_dim"), _g(cfg, "linear_value_head_dim")
    eps = _g(cfg, "rms_norm_eps")
    qkv = x @ sd[f"{p}.in_proj_qkv.weight"].float().t()
    z = (x @ sd[f"{p}.in_proj_z.weight"].float().t()).view(t, hv, dv)
    b = x @ sd[f"{p}.in_proj_b.weight"].float().t()
    a = x @ sd[f"{p}.in_proj_a.weight"].float().t()
    w = sd[f"{p}.conv1d.weight"].float().squeeze(1)  # [C, K]
    kw = w.shape[1]
    padded = torch.cat((torch.zeros(kw - 1, qkv.shape[1]), qkv), 0)
    conv = torch.stack([(padded[i:i + kw].t() * w).sum(-1) for i in range(t)])
    mixed = F.silu(conv)
    q = mixed[:, : hk * dk].view(t, hk, dk)
    k = mixed[:, hk * dk: 2 * hk * dk].view(t, hk, dk)
    v = mixed[:, 2 * hk * dk:].view(t, hv, dv)
    q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6)
    k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    rep = hv // hk
    q, k = q.repeat_interleave(rep, 1) / math.sqrt(dk), k.repeat_interleave(rep, 1)
    beta = torch.sigmoid(b)
    g = -sd[f"{p}.A_log"].float().exp() * F.softplus(a + sd[f"{p}.dt_bias"].float())
    state = torch.zeros(hv, dk, dv)
    outs = []
    for i in range(t):
        state = state * g[i].exp()[:, None, None]
        pred = torch.einsum("hd,hdv->hv", k[i], state)
        delta = (v[i] - pred) * beta[i][:, None]
        state = state + k[i][:, :, None] * delta[:, None, :]
        outs.append(torch.einsum("hd,hdv->hv", q[i], state))
    o = torch.stack(outs)
    o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + eps) * sd[f"{p}.norm.weight"].float()
    o = o * F.silu(z)
    return o.reshape(t, hv * dv) @ sd[f"{p}.out_proj.weight"].float().t()


def reference_logits(sd: dict[str, torch.Tensor], cfg, tokens: list[int]) -> torch.Tensor:
    """Logits ``[len(tokens), vocab]`` of the full causal forward in fp32."""
    hybrid = _g(cfg, "model_type") in ("qwen3_5_text", "qwen3_5")
    eps = _g(cfg, "rms_norm_eps")
    hd = _g(cfg, "head_dim")
    rope = _g(cfg, "rope_parameters", None) or {}
    theta = rope.get("rope_theta", _g(cfg, "rope_theta", 10000.0))
    rd = int(hd * rope.get("partial_rotary_factor", 1.0)) if rope else hd
    cos_sin = rope_cos_sin(len(tokens) + 1, rd, float(theta))
    x = sd["model.embed_tokens.weight"].float()[torch.tensor(tokens)]
    layer_types = _g(cfg, "layer_types", None) or ["full_attention"] * _g(cfg, "num_hidden_layers")
    for i, kind in enumerate(layer_types):
        p = f"model.layers.{i}"
        h = _norm(x, sd[f"{p}.input_layernorm.weight"], eps, hybrid)
        if kind == "linear_attention":
            x = x + _gdn(h, sd, f"{p}.linear_attn", cfg)
        else:
            x = x + _attention(h, sd, f"{p}.self_attn", cfg, hybrid, cos_sin)
        h = _norm(x, sd[f"{p}.post_attention_layernorm.weight"], eps, hybrid)
        gu_g = h @ sd[f"{p}.mlp.gate_proj.weight"].float().t()
        gu_u = h @ sd[f"{p}.mlp.up_proj.weight"].float().t()
        x = x + (F.silu(gu_g) * gu_u) @ sd[f"{p}.mlp.down_proj.weight"].float().t()
    h = _norm(x, sd["model.norm.weight"], eps, hybrid)
    head = sd.get("lm_head.weight", sd["model.embed_tokens.weight"]).float()
    return h @ head.t()


def reference_greedy(sd, cfg, prompt: list[int], steps: int) -> list[int]:
    toks = list(prompt)
    out = []
    for _ in range(steps):
        nxt = int(reference_logits(sd, cfg, toks)[-1].argmax())
        out.append(nxt)
        toks.append(nxt)
    return out
