"""Qwen3.5 hybrid (Gated DeltaNet + gated full attention) and dense Qwen3 causal LMs.

Parity (behaviour): ``nanovllm/models/qwen3_5.py:26-355`` and
``nanovllm/models/qwen3.py:14-216`` -- pre-norm residual decoder layers,
zero-centred RMSNorm, q-projection of width ``2*Hq*hd`` carrying an output
gate, per-head q/k RMSNorm, partial RoPE, GDN mixer with gated per-head
RMSNorm, SwiGLU MLP, tied LM head.

Design: parameters are stored in kernel-ready packed form per tensor-parallel
rank -- one projection GEMM per mixer (``q|gate|k|v`` for attention and
``qkv|z|b|a`` for GDN), gate/up rows interleaved in 64-row groups for the
fused SiLU*mul epilogue.  Each packed parameter knows which checkpoint
tensors it is built from (``checkpoint_plan``); the strict loader in
``utils/loader.py`` pulls from the checkpoint rather than pushing into
per-parameter callbacks.  When ``tp_size`` exceeds the KV-head count, KV heads
are replicated so every rank owns the KV head of its query heads (the
reference rejects that case, ``qwen3_5.py:33-34``).
"""

from __future__ import annotations

import math
import os
from typing import Callable

import torch
from torch import nn

from inference_systems_b200 import ops
from inference_systems_b200.models.registry import ModelCapabilities
from inference_systems_b200.ops.reference import pack_gate_up
from inference_systems_b200.utils.context import ForwardBatch

Getter = Callable[[str], torch.Tensor]


def _rows(t: torch.Tensor, rank: int, size: int, dim: int = 0) -> torch.Tensor:
    n = t.shape[dim] // size
    return t.narrow(dim, rank * n, n)


class TPInfo:
    def __init__(self, rank: int = 0, size: int = 1):
        self.rank, self.size = rank, size


class ColumnScratch:
    """Shared fp32 buffer for decode-sized column-parallel projections.

    For up to ``rows`` tokens the projection GEMM adds its split-K tiles into
    this buffer with vector atomics (so the split count only sets parallelism)
    and the single consumer (GDN scan, attention prepare, SiLU*mul) reads the
    fp32 values and re-zeroes them; the buffer is therefore all-zero between
    uses and one buffer serves every layer in turn.
    """

    def __init__(self):
        self.buf: torch.Tensor | None = None
        self.rows = 0

    def allocate(self, rows: int, width: int, device) -> None:
        self.rows = rows
        self.buf = torch.zeros(rows * width, dtype=torch.float32, device=device)

    def project(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor | None:
        t, n = x.shape[0], w.shape[0]
        if self.buf is None or not x.is_cuda or t > self.rows or t * n > self.buf.numel():
            return None
        acc = self.buf[: t * n].view(t, n)
        ops.linear_accumulate(x, w, acc)
        return acc


def _col_linear(x: torch.Tensor, w: torch.Tensor, silu_mul: bool = False) -> torch.Tensor:
    """Column-parallel projection of a replicated ``[T, H]`` activation."""
    return ops.linear_silu_mul(x, w) if silu_mul else ops.linear(x, w)


class AttentionMixer(nn.Module):
    def __init__(self, cfg, tp: TPInfo, gated: bool, zero_centered: bool, prefix: str):
        super().__init__()
        self.prefix = prefix
        self.tp = tp
        self.scratch: ColumnScratch | None = None
        self.gated = gated
        self.zero_centered = zero_centered
        self.total_heads = cfg.num_attention_heads
        self.total_kv_heads = cfg.num_key_value_heads
        if self.total_heads % tp.size:
            raise ValueError("query head count must be divisible by tensor parallel size")
        self.num_heads = self.total_heads // tp.size
        if self.total_kv_heads >= tp.size:
            if self.total_kv_heads % tp.size:
                raise ValueError("KV head count must be divisible by tensor parallel size")
            self.num_kv_heads = self.total_kv_heads // tp.size
            self.kv_head_start = tp.rank * self.num_kv_heads
        else:
            if tp.size % self.total_kv_heads:
                raise ValueError("tensor parallel size must be a multiple of the KV head count")
            self.num_kv_heads = 1
            group = self.total_heads // self.total_kv_heads
            self.kv_head_start = (tp.rank * self.num_heads) // group
        self.head_dim = cfg.head_dim
        self.scale = self.head_dim ** -0.5
        self.eps = cfg.rms_norm_eps
        h = cfg.hidden_size
        qw = self.num_heads * self.head_dim * (2 if gated else 1)
        kvw = self.num_kv_heads * self.head_dim
        self.q_width, self.kv_width = qw, kvw
        self.qkv_proj = nn.Parameter(torch.empty(qw + 2 * kvw, h), requires_grad=False)
        self.o_proj = nn.Parameter(torch.empty(h, self.num_heads * self.head_dim), requires_grad=False)
        self.q_norm = nn.Parameter(torch.empty(self.head_dim), requires_grad=False)
        self.k_norm = nn.Parameter(torch.empty(self.head_dim), requires_grad=False)
        rope = getattr(cfg, "rope_parameters", None) or {}
        theta = rope.get("rope_theta", getattr(cfg, "rope_theta", 10000.0)) if rope else getattr(cfg, "rope_theta", 10000.0)
        factor = rope.get("partial_rotary_factor", 1.0) if rope else 1.0
        self.rotary_dim = int(self.head_dim * factor)
        self.rope_theta = float(theta)

    def checkpoint_plan(self) -> dict[str, tuple[list[str], Callable[[Getter], torch.Tensor]]]:
        p, tp = self.prefix, self.tp
        hd = self.head_dim

        def kv_rows(t: torch.Tensor) -> torch.Tensor:
            return t.narrow(0, self.kv_head_start * hd, self.num_kv_heads * hd)

        def qkv(get: Getter) -> torch.Tensor:
            q = _rows(get(f"{p}.q_proj.weight"), tp.rank, tp.size)
            k = kv_rows(get(f"{p}.k_proj.weight"))
            v = kv_rows(get(f"{p}.v_proj.weight"))
            return torch.cat((q, k, v), 0)

        return {
            "qkv_proj": ([f"{p}.q_proj.weight", f"{p}.k_proj.weight", f"{p}.v_proj.weight"], qkv),
            "o_proj": ([f"{p}.o_proj.weight"], lambda g: _rows(g(f"{p}.o_proj.weight"), tp.rank, tp.size, 1)),
            "q_norm": ([f"{p}.q_norm.weight"], lambda g: g(f"{p}.q_norm.weight")),
            "k_norm": ([f"{p}.k_norm.weight"], lambda g: g(f"{p}.k_norm.weight")),
        }

    def forward(self, x: torch.Tensor, batch: ForwardBatch, kv: tuple[torch.Tensor, torch.Tensor],
                cos_sin: torch.Tensor) -> torch.Tensor:
        """Returns the rank-local pre-o_proj activation ``[T, Hq_local*hd]``."""
        qkv = self.scratch.project(x, self.qkv_proj) if self.scratch is not None else None
        if qkv is None:
            qkv = _col_linear(x, self.qkv_proj)
        k_cache, v_cache = kv
        return ops.attention_block(qkv, batch, self.q_norm, self.k_norm, cos_sin, k_cache, v_cache,
                                   num_heads=self.num_heads, num_kv_heads=self.num_kv_heads,
                                   head_dim=self.head_dim, eps=self.eps, gated=self.gated,
                                   zero_centered=self.zero_centered, scale=self.scale)


class GDNMixer(nn.Module):
    def __init__(self, cfg, tp: TPInfo, prefix: str):
        super().__init__()
        self.prefix = prefix
        self.tp = tp
        self.scratch: ColumnScratch | None = None
        thk, thv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
        if thk % tp.size or thv % tp.size:
            raise ValueError("GDN head counts must be divisible by tensor parallel size")
        if thv % thk:
            raise ValueError("linear_num_value_heads must divide by linear_num_key_heads")
        self.hk, self.hv = thk // tp.size, thv // tp.size
        self.total_hk, self.total_hv = thk, thv
        self.dk, self.dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
        self.kernel = cfg.linear_conv_kernel_dim
        self.eps = cfg.rms_norm_eps
        h = cfg.hidden_size
        self.key_dim, self.value_dim = self.hk * self.dk, self.hv * self.dv
        self.conv_dim = 2 * self.key_dim + self.value_dim
        self.proj_width = self.conv_dim + self.value_dim + 2 * self.hv
        # rows padded to a multiple of 64 so every projection row is 16-byte aligned for TMA
        self.proj_rows = (self.proj_width + 63) // 64 * 64
        self.in_proj = nn.Parameter(torch.empty(self.proj_rows, h), requires_grad=False)
        self.conv_w = nn.Parameter(torch.empty(self.conv_dim, self.kernel), requires_grad=False)
        self.A_log = nn.Parameter(torch.empty(self.hv, dtype=torch.float32), requires_grad=False)
        self.dt_bias = nn.Parameter(torch.empty(self.hv, dtype=torch.float32), requires_grad=False)
        self.norm_w = nn.Parameter(torch.empty(self.dv), requires_grad=False)
        self.out_proj = nn.Parameter(torch.empty(h, self.value_dim), requires_grad=False)

    def _qkv_rows(self, t: torch.Tensor) -> torch.Tensor:
        tkd = self.total_hk * self.dk
        r = self.tp.rank
        q = t.narrow(0, r * self.key_dim, self.key_dim)
        k = t.narrow(0, tkd + r * self.key_dim, self.key_dim)
        v = t.narrow(0, 2 * tkd + r * self.value_dim, self.value_dim)
        return torch.cat((q, k, v), 0)

    def checkpoint_plan(self):
        p, tp = self.prefix, self.tp
        keys = [f"{p}.in_proj_qkv.weight", f"{p}.in_proj_z.weight", f"{p}.in_proj_b.weight", f"{p}.in_proj_a.weight"]

        def in_proj(get: Getter) -> torch.Tensor:
            qkv = self._qkv_rows(get(keys[0]))
            z = _rows(get(keys[1]), tp.rank, tp.size)
            b = _rows(get(keys[2]), tp.rank, tp.size)
            a = _rows(get(keys[3]), tp.rank, tp.size)
            w = torch.cat((qkv, z, b, a), 0)
            pad = self.proj_rows - w.shape[0]
            return torch.cat((w, w.new_zeros(pad, w.shape[1])), 0) if pad else w

        return {
            "in_proj": (keys, in_proj),
            "conv_w": ([f"{p}.conv1d.weight"], lambda g: self._qkv_rows(g(f"{p}.conv1d.weight")).reshape(self.conv_dim, -1)),
            "A_log": ([f"{p}.A_log"], lambda g: _rows(g(f"{p}.A_log"), tp.rank, tp.size).float()),
            "dt_bias": ([f"{p}.dt_bias"], lambda g: _rows(g(f"{p}.dt_bias"), tp.rank, tp.size).float()),
            "norm_w": ([f"{p}.norm.weight"], lambda g: g(f"{p}.norm.weight")),
            "out_proj": ([f"{p}.out_proj.weight"], lambda g: _rows(g(f"{p}.out_proj.weight"), tp.rank, tp.size, 1)),
        }

    def forward(self, x: torch.Tensor, batch: ForwardBatch, pools: tuple[torch.Tensor, torch.Tensor],
                records: tuple | None = None, history: tuple | None = None) -> torch.Tensor:
        proj = self.scratch.project(x, self.in_proj) if self.scratch is not None else None
        if proj is None:
            proj = _col_linear(x, self.in_proj)
        rec_pool, conv_pool = pools
        if history is not None:
            return ops.gdn_with_history(proj, batch, self.conv_w, self.A_log, self.dt_bias, self.norm_w, rec_pool,
                                        conv_pool, *history, hk=self.hk, hv=self.hv, dk=self.dk, dv=self.dv,
                                        eps=self.eps)
        if records is not None:
            # (k, delta, log decay, conv window) replay records, or (state, conv window) snapshots
            verify = ops.gdn_verify if len(records) == 4 else ops.gdn_verify_snapshots
            return verify(proj, batch, self.conv_w, self.A_log, self.dt_bias, self.norm_w, rec_pool, conv_pool,
                          *records, hk=self.hk, hv=self.hv, dk=self.dk, dv=self.dv, eps=self.eps)
        return ops.gdn(proj, batch, self.conv_w, self.A_log, self.dt_bias, self.norm_w, rec_pool, conv_pool,
                       hk=self.hk, hv=self.hv, dk=self.dk, dv=self.dv, eps=self.eps)


class MLP(nn.Module):
    def __init__(self, cfg, tp: TPInfo, prefix: str):
        super().__init__()
        self.prefix, self.tp = prefix, tp
        self.scratch: ColumnScratch | None = None
        if cfg.intermediate_size % tp.size:
            raise ValueError("intermediate size must be divisible by tensor parallel size")
        self.inter = cfg.intermediate_size // tp.size
        h = cfg.hidden_size
        self.gate_up = nn.Parameter(torch.empty(2 * self.inter, h), requires_grad=False)
        self.down = nn.Parameter(torch.empty(h, self.inter), requires_grad=False)

    def checkpoint_plan(self):
        p, tp = self.prefix, self.tp
        return {
            "gate_up": ([f"{p}.gate_proj.weight", f"{p}.up_proj.weight"],
                        lambda g: pack_gate_up(_rows(g(f"{p}.gate_proj.weight"), tp.rank, tp.size),
                                               _rows(g(f"{p}.up_proj.weight"), tp.rank, tp.size))),
            "down": ([f"{p}.down_proj.weight"], lambda g: _rows(g(f"{p}.down_proj.weight"), tp.rank, tp.size, 1)),
        }

    def forward_pre_down(self, x: torch.Tensor) -> torch.Tensor:
        acc = self.scratch.project(x, self.gate_up) if self.scratch is not None else None
        if acc is not None:
            return ops.silu_mul_acc(acc, x.shape[0])
        return _col_linear(x, self.gate_up, silu_mul=True)


class DecoderLayer(nn.Module):
    def __init__(self, cfg, tp: TPInfo, layer_type: str, prefix: str, hybrid: bool):
        super().__init__()
        self.prefix = prefix
        self.is_linear = layer_type == "linear_attention"
        self.zero_centered = hybrid
        h = cfg.hidden_size
        self.eps = cfg.rms_norm_eps
        self.input_layernorm = nn.Parameter(torch.empty(h), requires_grad=False)
        self.post_attention_layernorm = nn.Parameter(torch.empty(h), requires_grad=False)
        if self.is_linear:
            self.mixer = GDNMixer(cfg, tp, f"{prefix}.linear_attn")
        else:
            self.mixer = AttentionMixer(cfg, tp, gated=hybrid, zero_centered=hybrid, prefix=f"{prefix}.self_attn")
        self.mlp = MLP(cfg, tp, f"{prefix}.mlp")

    def checkpoint_plan(self):
        p = self.prefix
        plan = {
            "input_layernorm": ([f"{p}.input_layernorm.weight"], lambda g: g(f"{p}.input_layernorm.weight")),
            "post_attention_layernorm": ([f"{p}.post_attention_layernorm.weight"],
                                         lambda g: g(f"{p}.post_attention_layernorm.weight")),
        }
        for sub_name, sub in (("mixer", self.mixer), ("mlp", self.mlp)):
            for k, v in sub.checkpoint_plan().items():
                plan[f"{sub_name}.{k}"] = v
        return plan

    def mixer_out_weight(self) -> torch.Tensor:
        return self.mixer.out_proj if self.is_linear else self.mixer.o_proj


class HybridCausalLM(nn.Module):
    """Shared body of Qwen3.5 (hybrid) and Qwen3 (dense) causal LMs."""

    hybrid = True
    checkpoint_prefix_mapping = (("model.language_model.", "model."), ("language_model.", "model."))
    explicitly_skipped_prefixes = ("model.visual.", "visual.", "mtp.")

    def __init__(self, cfg, caps: ModelCapabilities, tp_rank: int = 0, tp_size: int = 1):
        super().__init__()
        self.cfg = cfg
        self.caps = caps
        self.tp = TPInfo(tp_rank, tp_size)
        h, v = cfg.hidden_size, cfg.vocab_size
        self.hidden_size, self.vocab_size = h, v
        self.eps = cfg.rms_norm_eps
        if v % tp_size:
            raise ValueError("vocab size must be divisible by tensor parallel size")
        self.vocab_per_rank = v // tp_size
        self.vocab_start = tp_rank * self.vocab_per_rank
        self.tied = bool(cfg.tie_word_embeddings)
        # The embedding table is replicated on every rank (a lookup needs no
        # collective); the LM head is vocab-parallel.  With tied weights the
        # head is a row-slice view of the replicated table.
        self.embed_tokens = nn.Parameter(torch.empty(v, h), requires_grad=False)
        if not self.tied:
            self.lm_head = nn.Parameter(torch.empty(self.vocab_per_rank, h), requires_grad=False)
        self.norm = nn.Parameter(torch.empty(h), requires_grad=False)
        self.layers = nn.ModuleList(
            DecoderLayer(cfg, self.tp, t, f"model.layers.{i}", self.hybrid) for i, t in enumerate(caps.layer_types)
        )
        self.linear_layer_ids = [i for i, l in enumerate(self.layers) if l.is_linear]
        self.attn_layer_ids = [i for i, l in enumerate(self.layers) if not l.is_linear]
        self._cos_sin: torch.Tensor | None = None
        self.column_scratch = ColumnScratch()
        self.column_scratch_tokens = 0
        self.comm = None  # set by the runner (parallel.comm.TPComm) when tp_size > 1

    # ------------------------------------------------------------ weights
    def lm_head_weight(self) -> torch.Tensor:
        if self.tied:
            return self.embed_tokens.narrow(0, self.vocab_start, self.vocab_per_rank)
        return self.lm_head

    def checkpoint_plan(self):
        tp = self.tp
        plan = {
            "embed_tokens": (["model.embed_tokens.weight"], lambda g: g("model.embed_tokens.weight")),
            "norm": (["model.norm.weight"], lambda g: g("model.norm.weight")),
        }
        if not self.tied:
            plan["lm_head"] = (["lm_head.weight"], lambda g: _rows(g("lm_head.weight"), tp.rank, tp.size))
        for i, layer in enumerate(self.layers):
            for k, v in layer.checkpoint_plan().items():
                plan[f"layers.{i}.{k}"] = v
        return plan

    def attention_geometry(self) -> tuple[int, int, int]:
        if not self.attn_layer_ids:
            return 0, 0, 0
        m = self.layers[self.attn_layer_ids[0]].mixer
        return len(self.attn_layer_ids), m.num_kv_heads, m.head_dim

    def gdn_geometry(self):
        if not self.linear_layer_ids:
            return None
        m = self.layers[self.linear_layer_ids[0]].mixer
        return dict(num_layers=len(self.linear_layer_ids), hv=m.hv, hk=m.hk, dk=m.dk, dv=m.dv,
                    conv_dim=m.conv_dim, kernel=m.kernel)

    def cos_sin(self, device) -> torch.Tensor | None:
        if not self.attn_layer_ids:
            return None
        if self._cos_sin is None or self._cos_sin.device != torch.device(device):
            m = self.layers[self.attn_layer_ids[0]].mixer
            from inference_systems_b200.ops.reference import rope_cos_sin
            max_pos = int(min(self.cfg.max_position_embeddings, 1 << 20))
            self._cos_sin = rope_cos_sin(max_pos, m.rotary_dim, m.rope_theta, device)
        return self._cos_sin

    # ------------------------------------------------------------ forward
    def set_accumulator(self, max_tokens: int, device) -> None:
        """Persistent fp32 ``[max_tokens, hidden]`` buffer that row-parallel GEMMs add into.

        Every CTA of the output-projection GEMMs adds its (split-K) tile with
        vector atomics and the following add+RMSNorm kernel consumes and
        re-zeroes the rows it read, so the buffer is zero between uses.
        """
        self.acc = torch.zeros(max_tokens, self.hidden_size, dtype=torch.float32, device=device)
        # Column-parallel projections of at most this many tokens split K across enough CTAs to
        # cover every SM and add into an fp32 scratch consumed by the next kernel; above it the
        # atomics cost more than the extra parallelism gains (measured), so they store bf16.
        rows = min(max_tokens, int(os.environ.get("ISB_COLUMN_SCRATCH_TOKENS", str(self.column_scratch_tokens))))
        if rows > 0:
            widths = [m.shape[0] for m in self.parameters() if m.dim() == 2 and m.shape[1] == self.hidden_size
                      and m.shape[0] != self.vocab_size and m.shape[0] != self.vocab_per_rank]
            self.column_scratch.allocate(rows, max(widths), device)
            for mod in self.modules():
                if isinstance(mod, (AttentionMixer, GDNMixer, MLP)):
                    mod.scratch = self.column_scratch

    def _row_parallel(self, x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor, norm_w: torch.Tensor) -> torch.Tensor:
        """``residual += x @ w^T`` (summed over TP ranks); return RMSNorm(residual)."""
        if self.comm is not None and self.tp.size > 1:
            return self.comm.row_parallel_residual_norm(x, w, residual, norm_w, self.eps, self.hybrid)
        acc = getattr(self, "acc", None)
        if x.is_cuda and acc is not None and x.shape[0] <= acc.shape[0]:
            return ops.linear_add_rmsnorm(x, w, acc, residual, norm_w, self.eps, self.hybrid)
        y = ops.linear(x, w)
        return ops.add_rmsnorm(y, residual, norm_w, self.eps, self.hybrid)

    def forward(self, batch: ForwardBatch, kv_caches: list, state_pools: list | None) -> torch.Tensor:
        """Run all decoder layers; returns the final-normed hidden states ``[T, H]``.

        ``kv_caches[j] = (k_cache, v_cache)`` for the j-th attention layer and
        ``state_pools[j] = (recurrent_pool, conv_pool)`` for the j-th GDN layer.
        """
        cos_sin = self.cos_sin(batch.input_ids.device)
        layers = self.layers
        residual, x = ops.embed_rmsnorm(batch.input_ids, self.embed_tokens, layers[0].input_layernorm, self.eps,
                                        self.hybrid)
        attn_j = gdn_j = 0
        for i, layer in enumerate(layers):
            if layer.is_linear:
                rec = batch.gdn_verify[gdn_j] if batch.gdn_verify is not None else None
                hist = None
                if batch.gdn_history is not None:
                    h = batch.gdn_history
                    hist = (h["rows"], h["rec"][gdn_j], h["conv"][gdn_j])
                y = layer.mixer(x, batch, state_pools[gdn_j], rec, hist)
                gdn_j += 1
            else:
                y = layer.mixer(x, batch, kv_caches[attn_j], cos_sin)
                attn_j += 1
            x = self._row_parallel(y, layer.mixer_out_weight(), residual, layer.post_attention_layernorm)
            y = layer.mlp.forward_pre_down(x)
            next_norm = layers[i + 1].input_layernorm if i + 1 < len(layers) else self.norm
            x = self._row_parallel(y, layer.mlp.down, residual, next_norm)
        return x

    def sample(self, hidden: torch.Tensor, temperatures: torch.Tensor, rng: torch.Tensor) -> torch.Tensor:
        """Vocab-parallel LM head fused with greedy / Gumbel-max sampling -> token ids ``[B]`` int32."""
        if self.comm is not None and self.tp.size > 1:
            return self.comm.lm_head_sample(hidden, self.lm_head_weight(), temperatures, rng, self.vocab_start)
        _, idx = ops.lm_head_sample(hidden, self.lm_head_weight(), temperatures, rng, 0)
        return idx

    def compute_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """Full-vocabulary logits (rank-local shard when TP > 1)."""
        return ops.linear(hidden, self.lm_head_weight())


class Qwen3_5ForCausalLM(HybridCausalLM):
    hybrid = True


class Qwen3ForCausalLM(HybridCausalLM):
    hybrid = False
    explicitly_skipped_prefixes = ()
