"""Plain-PyTorch implementations of every kernel contract.

These run the engine on CPU and are the fp32 oracles that the CUDA kernels
are tested against.  The math follows the Qwen3.5 definitions the reference
implements in ``nanovllm/models/qwen35_reference.py:52-386`` (short causal
conv + SiLU, L2-normalised q/k, ``q / sqrt(Dk)``, gated delta rule with
``beta = sigmoid(b)``, ``g = -exp(A_log) * softplus(a + dt_bias)``),
``nanovllm/layers/layernorm.py:111-162`` (zero-centred RMSNorm, gated
RMSNorm) and ``nanovllm/layers/rotary_embedding.py:6-69`` (rotate-half
partial RoPE).  Layout contracts (shared with ``csrc/``):

* GDN projection row: ``[q (Hk*Dk) | k (Hk*Dk) | v (Hv*Dv) | z (Hv*Dv) | b (Hv) | a (Hv)]``;
  conv channels are the first ``2*Hk*Dk + Hv*Dv`` columns.
* Attention projection row: ``[per q-head (query hd | gate hd) | k (Hkv*hd) | v (Hkv*hd)]``.
* Paged KV cache: ``[num_blocks, Hkv, block_size, hd]`` per layer and per K/V;
  ``slot = block_id * block_size + offset``.
* gate/up packed weight: rows interleaved in groups of 64
  ``[g0..g63, u0..u63, g64..g127, u64..u127, ...]``.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

GATE_UP_GROUP = 64


# --------------------------------------------------------------------- norms
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, zero_centered: bool) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    scale = (1.0 + w.float()) if zero_centered else w.float()
    if zero_centered:
        return (y * scale).to(x.dtype)
    # Qwen3 dense RMSNorm: round the normalised value before the weight.
    return y.to(x.dtype) * w


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                zero_centered: bool) -> torch.Tensor:
    """``residual <- x + residual`` (rounded); return norm of the unrounded sum."""
    s = x.float() + residual.float()
    residual.copy_(s.to(residual.dtype))
    y = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + eps)
    if zero_centered:
        return (y * (1.0 + w.float())).to(x.dtype)
    return y.to(x.dtype) * w


def gated_rmsnorm(x: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    return (y * F.silu(z.float())).to(x.dtype)


# ---------------------------------------------------------------- embedding
def embed(ids: torch.Tensor, weight: torch.Tensor, vocab_start: int = 0) -> torch.Tensor:
    local = ids.long() - vocab_start
    valid = (local >= 0) & (local < weight.shape[0])
    out = F.embedding(local.clamp(0, weight.shape[0] - 1), weight)
    return out * valid.unsqueeze(-1).to(out.dtype)


# --------------------------------------------------------------------- gemm
def gemm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a[M,K] @ b[N,K]^T`` with fp32 accumulation, output in ``a.dtype``."""
    return (a.float() @ b.float().t()).to(a.dtype)


def pack_gate_up(gate: torch.Tensor, up: torch.Tensor, group: int = GATE_UP_GROUP) -> torch.Tensor:
    inter = gate.shape[0]
    assert inter % group == 0, f"intermediate size {inter} must be a multiple of {group}"
    g = gate.reshape(inter // group, group, -1)
    u = up.reshape(inter // group, group, -1)
    return torch.stack((g, u), dim=1).reshape(2 * inter, -1)


def silu_mul_packed(y: torch.Tensor, group: int = GATE_UP_GROUP) -> torch.Tensor:
    """Apply SiLU(gate)*up to the output of a packed gate/up GEMM."""
    t = y.shape[0]
    v = y.float().reshape(t, -1, 2, group)
    out = F.silu(v[:, :, 0]) * v[:, :, 1]
    return out.reshape(t, -1).to(y.dtype)


def gemm_silu_mul(a: torch.Tensor, b_packed: torch.Tensor) -> torch.Tensor:
    return silu_mul_packed((a.float() @ b_packed.float().t()), GATE_UP_GROUP).to(a.dtype)


# -------------------------------------------------------------------- rope
def rope_cos_sin(max_pos: int, rotary_dim: int, base: float, device=None) -> torch.Tensor:
    """``[max_pos, rotary_dim]`` table: cos (first half) then sin (second half)."""
    inv = 1.0 / (base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float64) / rotary_dim))
    t = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(t, inv)
    return torch.cat((f.cos(), f.sin()), dim=-1).float().to(device)


def apply_rope(x: torch.Tensor, cos_sin: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE on the first ``rotary_dim`` channels of ``x[T, H, D]``."""
    rd = cos_sin.shape[-1]
    cs = cos_sin[positions.long()]
    cos, sin = cs[:, None, : rd // 2], cs[:, None, rd // 2:]
    xf = x.float()
    x1, x2 = xf[..., : rd // 2], xf[..., rd // 2: rd]
    rot = torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1)
    return torch.cat((rot, xf[..., rd:]), dim=-1).to(x.dtype)


# ---------------------------------------------------------------- kv cache
def store_kv(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
             slot_mapping: torch.Tensor) -> None:
    """``k, v: [T, Hkv, hd]`` into ``[num_blocks, Hkv, bs, hd]`` caches (slot -1 skipped)."""
    bs = k_cache.shape[2]
    sm = slot_mapping.long()
    keep = sm >= 0
    if not bool(keep.any()):
        return
    sm = sm[keep]
    blk, off = sm // bs, sm % bs
    k_cache[blk, :, off] = k[keep].to(k_cache.dtype)
    v_cache[blk, :, off] = v[keep].to(v_cache.dtype)


def attn_qkv_prepare(qkv: torch.Tensor, positions: torch.Tensor, q_norm_w: torch.Tensor,
                     k_norm_w: torch.Tensor, cos_sin: torch.Tensor, num_heads: int, num_kv_heads: int,
                     head_dim: int, eps: float, gated: bool, zero_centered: bool):
    """Split the attention projection, q/k RMSNorm + partial RoPE.

    Returns ``(q [T,Hq,hd], gate [T,Hq,hd] | None, k [T,Hkv,hd], v [T,Hkv,hd])``.
    """
    t = qkv.shape[0]
    qw = num_heads * head_dim * (2 if gated else 1)
    kvw = num_kv_heads * head_dim
    qpart = qkv[:, :qw]
    if gated:
        qg = qpart.reshape(t, num_heads, 2 * head_dim)
        q, gate = qg[..., :head_dim], qg[..., head_dim:]
    else:
        q, gate = qpart.reshape(t, num_heads, head_dim), None
    k = qkv[:, qw:qw + kvw].reshape(t, num_kv_heads, head_dim)
    v = qkv[:, qw + kvw:qw + 2 * kvw].reshape(t, num_kv_heads, head_dim)
    q = rmsnorm(q, q_norm_w, eps, zero_centered)
    k = rmsnorm(k, k_norm_w, eps, zero_centered)
    q = apply_rope(q, cos_sin, positions)
    k = apply_rope(k, cos_sin, positions)
    return q, gate, k, v.contiguous()


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    cu_seqlens_q: torch.Tensor, context_lens: torch.Tensor, block_tables: torch.Tensor,
                    scale: float, gate: torch.Tensor | None = None) -> torch.Tensor:
    """Causal attention of packed queries over paged K/V.

    Query ``i`` of a sequence with ``n`` new tokens and ``ctx`` total tokens
    sits at position ``ctx - n + i`` and sees keys ``0 .. ctx - n + i``.
    Output ``[T, Hq*hd]``; multiplied by ``sigmoid(gate)`` when given.
    """
    t, hq, hd = q.shape
    hkv, bs = k_cache.shape[1], k_cache.shape[2]
    group = hq // hkv
    out = torch.empty(t, hq, hd, dtype=torch.float32, device=q.device)
    cu = cu_seqlens_q.tolist()
    ctx = context_lens.tolist()
    for i in range(len(cu) - 1):
        s, e = cu[i], cu[i + 1]
        n, c = e - s, ctx[i]
        if n == 0:
            continue
        nblk = (c + bs - 1) // bs
        blocks = block_tables[i, :nblk].long()
        kk = k_cache[blocks].permute(1, 0, 2, 3).reshape(hkv, nblk * bs, hd)[:, :c].float()
        vv = v_cache[blocks].permute(1, 0, 2, 3).reshape(hkv, nblk * bs, hd)[:, :c].float()
        kk = kk.repeat_interleave(group, 0)
        vv = vv.repeat_interleave(group, 0)
        qq = q[s:e].float().transpose(0, 1)  # [hq, n, hd]
        scores = (qq @ kk.transpose(1, 2)) * scale  # [hq, n, c]
        qpos = torch.arange(c - n, c, device=q.device)[:, None]
        kpos = torch.arange(c, device=q.device)[None, :]
        scores = scores.masked_fill(kpos > qpos, float("-inf"))
        p = torch.softmax(scores, dim=-1)
        out[s:e] = (p @ vv).transpose(0, 1)
    if gate is not None:
        out = out * torch.sigmoid(gate.float())
    return out.to(q.dtype).reshape(t, hq * hd)


# --------------------------------------------------------------------- GDN
def _l2n(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def gdn_split(proj: torch.Tensor, hk: int, hv: int, dk: int, dv: int):
    kd, vd = hk * dk, hv * dv
    conv_dim = 2 * kd + vd
    qkv = proj[:, :conv_dim]
    z = proj[:, conv_dim:conv_dim + vd]
    b = proj[:, conv_dim + vd:conv_dim + vd + hv]
    a = proj[:, conv_dim + vd + hv:conv_dim + vd + 2 * hv]
    return qkv, z, b, a


def gdn_step_fp32(state: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                  log_decay: torch.Tensor, beta: torch.Tensor):
    """One gated-delta step. ``state [..., Dk, Dv]``; q,k ``[..., Dk]``; v ``[..., Dv]``.

    Returns ``(out, new_state, delta)``.
    """
    state = state * log_decay.exp()[..., None, None]
    pred = torch.einsum("...d,...dv->...v", k, state)
    delta = (v - pred) * beta[..., None]
    state = state + k[..., :, None] * delta[..., None, :]
    out = torch.einsum("...d,...dv->...v", q, state)
    return out, state, delta


def gdn_sequence(proj: torch.Tensor, conv_w: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor,
                 norm_w: torch.Tensor, rec_state: torch.Tensor, conv_state: torch.Tensor, *,
                 hk: int, hv: int, dk: int, dv: int, eps: float, history_at: list[int] | None = None,
                 return_records: bool = False):
    """Run one sequence (``proj [n, P]``) from ``rec_state [Hv,Dk,Dv]`` / ``conv_state [C, K-1]``.

    Returns ``(out [n, Hv*Dv], new_rec, new_conv, rec_hist, conv_hist, records)`` where the
    histories hold the states *after* token ``i`` for each ``i`` in ``history_at`` and
    ``records`` is ``(k [n,Hv,Dk], delta [n,Hv,Dv], log_decay [n,Hv])`` when requested.
    """
    n = proj.shape[0]
    qkv, z, b, a = gdn_split(proj, hk, hv, dk, dv)
    kw = conv_w.shape[-1]
    x = qkv.float()
    window_state = conv_state.float().clone()  # [C, K-1]
    w = conv_w.float().reshape(conv_w.shape[0], kw)
    beta = torch.sigmoid(b.float())
    log_decay = -a_log.float().exp() * F.softplus(a.float() + dt_bias.float())
    state = rec_state.float().clone()
    rep = hv // hk
    outs = []
    rec_hist, conv_hist = [], []
    rk, rd, rl = [], [], []
    hist = set(history_at or [])
    for i in range(n):
        window = torch.cat((window_state, x[i][:, None]), dim=-1)  # [C, K]
        mixed = F.silu((window * w).sum(-1))
        window_state = window[:, 1:]
        q = mixed[: hk * dk].reshape(hk, dk)
        k = mixed[hk * dk: 2 * hk * dk].reshape(hk, dk)
        v = mixed[2 * hk * dk:].reshape(hv, dv)
        q = _l2n(q).repeat_interleave(rep, 0) / math.sqrt(dk)
        k = _l2n(k).repeat_interleave(rep, 0)
        o, state, delta = gdn_step_fp32(state, q, k, v, log_decay[i], beta[i])
        outs.append(o)
        if return_records:
            rk.append(k)
            rd.append(delta)
            rl.append(log_decay[i])
        if i in hist:
            rec_hist.append(state.clone())
            conv_hist.append(window_state.clone())
    core = torch.stack(outs) if outs else proj.new_zeros((0, hv, dv), dtype=torch.float32)
    core = core.to(proj.dtype)
    zz = z.reshape(n, hv, dv)
    y = gated_rmsnorm(core, zz, norm_w, eps).reshape(n, hv * dv)
    records = (torch.stack(rk), torch.stack(rd), torch.stack(rl)) if return_records and n else None
    return (y, state, window_state.to(conv_state.dtype),
            rec_hist, [c.to(conv_state.dtype) for c in conv_hist], records)


def gdn_forward(proj: torch.Tensor, cu_seqlens: list[int], slot_ids: list[int], conv_w, a_log, dt_bias,
                norm_w, rec_pool: torch.Tensor, conv_pool: torch.Tensor, *, hk, hv, dk, dv, eps) -> torch.Tensor:
    """Packed ragged batch; states read from and written back to the slot pools in place."""
    out = torch.empty(proj.shape[0], hv * dv, dtype=proj.dtype, device=proj.device)
    for i, slot in enumerate(slot_ids):
        s, e = cu_seqlens[i], cu_seqlens[i + 1]
        if e == s:
            continue
        y, rec, conv, *_ = gdn_sequence(proj[s:e], conv_w, a_log, dt_bias, norm_w, rec_pool[slot],
                                        conv_pool[slot], hk=hk, hv=hv, dk=dk, dv=dv, eps=eps)
        out[s:e] = y
        rec_pool[slot] = rec
        conv_pool[slot] = conv
    return out


# ------------------------------------------------------------- sampling
def sample_tokens(logits: torch.Tensor, temperatures: torch.Tensor, gumbel: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy where ``T <= 1e-10``; else Gumbel-max on ``logits / T``.

    ``argmax(softmax(l/T) / E)`` with ``E ~ Exp(1)`` (the reference sampler,
    ``nanovllm/layers/sampler.py:8-21``) equals ``argmax(l/T + G)`` with
    Gumbel noise ``G = -log E``, which needs no softmax and fuses into the
    LM-head GEMM epilogue.
    """
    lf = logits.float()
    greedy = temperatures <= 1e-10
    safe_t = torch.where(greedy, torch.ones_like(temperatures), temperatures).float()
    if gumbel is None:
        u = torch.rand_like(lf).clamp_(1e-20, 1.0)
        gumbel = -torch.log(-torch.log(u))
    sampled = (lf / safe_t[:, None] + gumbel).argmax(-1)
    return torch.where(greedy, lf.argmax(-1), sampled)
