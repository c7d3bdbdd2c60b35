"""Qwen3.5 one-layer multi-token-prediction (MTP) draft head.

Parity: ``nanovllm/models/qwen3_5_mtp.py:10-66`` -- ``fc([norm_e(embed(tok));
norm_h(h_target)])`` feeds one gated full-attention decoder layer (layer index
``num_hidden_layers``), then a final zero-centred RMSNorm.  The embedding and
LM head are the target model's (not registered here), so strict loading of
``mtp.*`` expects exactly the 15 checkpoint tensors.
"""

from __future__ import annotations

import torch
from torch import nn

from inference_systems_b200 import ops
from inference_systems_b200.models.qwen3_5 import DecoderLayer, HybridCausalLM, TPInfo
from inference_systems_b200.utils.context import ForwardBatch


class Qwen3_5MTP(nn.Module):
    checkpoint_prefix_mapping = (("model.language_model.", "model."),)
    checkpoint_included_prefixes = ("mtp.",)

    def __init__(self, cfg, target: HybridCausalLM):
        super().__init__()
        if int(getattr(cfg, "mtp_num_hidden_layers", 1) or 1) != 1:
            raise NotImplementedError("exactly one MTP layer is supported")
        object.__setattr__(self, "_target", target)
        self.tp = target.tp
        h = cfg.hidden_size
        self.eps = cfg.rms_norm_eps
        self.pre_fc_norm_embedding = nn.Parameter(torch.empty(h), requires_grad=False)
        self.pre_fc_norm_hidden = nn.Parameter(torch.empty(h), requires_grad=False)
        self.fc = nn.Parameter(torch.empty(h, 2 * h), requires_grad=False)
        self.norm = nn.Parameter(torch.empty(h), requires_grad=False)
        self.layer = DecoderLayer(cfg, self.tp, "full_attention", "mtp.layers.0", hybrid=True)

    def checkpoint_plan(self):
        plan = {
            "pre_fc_norm_embedding": (["mtp.pre_fc_norm_embedding.weight"], lambda g: g("mtp.pre_fc_norm_embedding.weight")),
            "pre_fc_norm_hidden": (["mtp.pre_fc_norm_hidden.weight"], lambda g: g("mtp.pre_fc_norm_hidden.weight")),
            "fc": (["mtp.fc.weight"], lambda g: g("mtp.fc.weight")),
            "norm": (["mtp.norm.weight"], lambda g: g("mtp.norm.weight")),
        }
        for k, v in self.layer.checkpoint_plan().items():
            plan[f"layer.{k}"] = v
        return plan

    def forward(self, batch: ForwardBatch, target_hidden: torch.Tensor, kv: tuple[torch.Tensor, torch.Tensor]) -> torch.Tensor:
        t = self._target
        e = ops.embed(batch.input_ids, t.embed_tokens, 0)
        e = ops.rmsnorm(e, self.pre_fc_norm_embedding, self.eps, True)
        hn = ops.rmsnorm(target_hidden, self.pre_fc_norm_hidden, self.eps, True)
        residual = ops.linear(torch.cat((e, hn), dim=-1), self.fc)
        x = ops.rmsnorm(residual, self.layer.input_layernorm, self.eps, True)
        y = self.layer.mixer(x, batch, kv, t.cos_sin(batch.input_ids.device))
        x = t._row_parallel(y, self.layer.mixer.o_proj, residual, self.layer.post_attention_layernorm)
        y = self.layer.mlp.forward_pre_down(x)
        return t._row_parallel(y, self.layer.mlp.down, residual, self.norm)
