"""Operator entry points used by the models and the runner.

CUDA tensors go to the sm_100a kernels of the ``inference_systems_b200._C``
extension (``torch.ops.isb.*``); a missing extension on a CUDA tensor is an
error, never a silent fallback.  CPU tensors run the plain-PyTorch contracts in
``ops/reference.py`` (the engine's CPU path and the kernels' test oracle).
"""

from __future__ import annotations

import os

import torch

from inference_systems_b200.ops import reference as ref
from inference_systems_b200.ops._ext import cuda_ops
from inference_systems_b200.utils.context import ForwardBatch


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, zero_centered: bool) -> torch.Tensor:
    if x.is_cuda:
        return cuda_ops().rmsnorm(x, w, eps, zero_centered)
    return ref.rmsnorm(x, w, eps, zero_centered)


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                zero_centered: bool) -> torch.Tensor:
    if x.is_cuda:
        return cuda_ops().add_rmsnorm(x, residual, w, eps, zero_centered)
    return ref.add_rmsnorm(x, residual, w, eps, zero_centered)


def embed(ids: torch.Tensor, weight: torch.Tensor, vocab_start: int = 0) -> torch.Tensor:
    if ids.is_cuda:
        return cuda_ops().embed(ids, weight, vocab_start)
    return ref.embed(ids, weight, vocab_start)


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    if x.is_cuda:
        return cuda_ops().gemm(x, w, 0)
    return ref.gemm(x, w)


def linear_accumulate(x: torch.Tensor, w: torch.Tensor, acc: torch.Tensor) -> None:
    """``acc[:T] += x @ w^T`` in fp32 (the consumer re-zeroes ``acc``)."""
    if x.is_cuda:
        cuda_ops().gemm_accum(x, w, acc, 0)
        return
    acc[: x.shape[0]] += x.float() @ w.float().t()


def add_rmsnorm_acc(acc: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                    zero_centered: bool) -> torch.Tensor:
    """``s = acc + residual``; ``residual <- s`` (rounded); return RMSNorm(s); ``acc <- 0``."""
    if residual.is_cuda:
        return cuda_ops().add_rmsnorm_acc(acc, residual, w, eps, zero_centered)
    t = residual.shape[0]
    out = ref.add_rmsnorm(acc[:t], residual, w, eps, zero_centered).to(residual.dtype)
    acc[:t].zero_()
    return out


def linear_add_rmsnorm(x: torch.Tensor, w: torch.Tensor, acc: torch.Tensor, residual: torch.Tensor,
                       norm_w: torch.Tensor, eps: float, zero_centered: bool) -> torch.Tensor:
    """``residual += x @ w^T``; return RMSNorm(residual).  On CUDA one kernel when its split-K grid
    fits on the SMs (the add + norm run behind an in-kernel grid barrier), else the accumulate GEMM
    and ``add_rmsnorm_acc``.  ``acc`` is the fp32 scratch, zero between uses."""
    if x.is_cuda:
        return cuda_ops().gemm_accum_norm(x, w, acc, residual, norm_w, eps, zero_centered)
    linear_accumulate(x, w, acc)
    return add_rmsnorm_acc(acc, residual, norm_w, eps, zero_centered)


def silu_mul_acc(acc: torch.Tensor, rows: int) -> torch.Tensor:
    """Consume a packed fp32 gate/up accumulator ``[>=rows, 2I]``: return ``SiLU(gate) * up`` (bf16), re-zero it."""
    if acc.is_cuda:
        return cuda_ops().silu_mul_acc(acc, rows)
    out = ref.silu_mul_packed(acc[:rows]).to(torch.bfloat16)
    acc[:rows].zero_()
    return out


def embed_rmsnorm(ids: torch.Tensor, table: torch.Tensor, w: torch.Tensor, eps: float,
                  zero_centered: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """First-layer fusion: ``residual = table[ids]``, ``out = RMSNorm(residual)``."""
    if ids.is_cuda:
        return cuda_ops().embed_rmsnorm(ids, table, w, eps, zero_centered)
    residual = ref.embed(ids, table, 0)
    return residual, ref.rmsnorm(residual, w, eps, zero_centered)


def linear_silu_mul(x: torch.Tensor, w_packed: torch.Tensor) -> torch.Tensor:
    if x.is_cuda:
        return cuda_ops().gemm(x, w_packed, 1)
    return ref.gemm_silu_mul(x, w_packed)


def attention_block(qkv: torch.Tensor, batch: ForwardBatch, q_norm: torch.Tensor, k_norm: torch.Tensor,
                    cos_sin: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, *, num_heads: int,
                    num_kv_heads: int, head_dim: int, eps: float, gated: bool, zero_centered: bool,
                    scale: float) -> torch.Tensor:
    """q/k norm + RoPE + KV store + paged causal attention (+ sigmoid output gate)."""
    if qkv.is_cuda:
        c = cuda_ops()
        q, gate = c.attn_prepare(qkv, batch.positions, batch.slot_mapping, q_norm, k_norm, cos_sin, k_cache,
                                 v_cache, num_heads, num_kv_heads, head_dim, eps, gated, zero_centered)
        if batch.is_prefill and batch.decode_rows is not None:
            row_ctx, row_bt = batch.decode_rows
            return c.attention_decode(q, gate, k_cache, v_cache, row_ctx, row_bt, scale, gated)
        if batch.is_prefill and _ATTN_TC and head_dim == 256 and num_heads // num_kv_heads in (1, 2, 3, 4, 6, 8):
            return c.attention_prefill_tc(q, gate, k_cache, v_cache, batch.cu_seqlens_q, batch.context_lens,
                                          batch.block_tables, scale, gated, batch.max_seqlen_q)
        if batch.is_prefill:
            return c.attention_prefill(q, gate, k_cache, v_cache, batch.cu_seqlens_q, batch.context_lens,
                                       batch.block_tables, scale, gated, batch.max_seqlen_q)
        return c.attention_decode(q, gate, k_cache, v_cache, batch.context_lens, batch.block_tables, scale, gated)
    q, gate, k, v = ref.attn_qkv_prepare(qkv, batch.positions, q_norm, k_norm, cos_sin, num_heads, num_kv_heads,
                                         head_dim, eps, gated, zero_centered)
    ref.store_kv(k, v, k_cache, v_cache, batch.slot_mapping)
    return ref.paged_attention(q, k_cache, v_cache, batch.cu_seqlens_q, batch.context_lens, batch.block_tables,
                               scale, gate)


_GDN_CHUNKED = os.environ.get("ISB_GDN_CHUNKED", "1") != "0"
_ATTN_TC = os.environ.get("ISB_ATTN_TC", "1") != "0"
GDN_CHUNK = 64


def gdn_chunk_table(batch: ForwardBatch) -> tuple[torch.Tensor, int]:
    """Device table ``[chunk_seq | chunk_t0 | chunk_n | cu_chunks]`` (int32) of 64-token chunks.

    Built once per forward from the host copy of ``cu_seqlens`` and shared by
    every GDN layer of that forward.
    """
    cached = getattr(batch, "_gdn_chunks", None)
    if cached is not None:
        return cached
    cu = batch.cu_seqlens_host
    seq, t0, n, cuc = [], [], [], [0]
    for i in range(len(cu) - 1):
        for s in range(cu[i], cu[i + 1], GDN_CHUNK):
            seq.append(i)
            t0.append(s)
            n.append(min(GDN_CHUNK, cu[i + 1] - s))
        cuc.append(len(seq))
    info = torch.tensor(seq + t0 + n + cuc, dtype=torch.int32).to(batch.cu_seqlens_q.device, non_blocking=True)
    batch._gdn_chunks = (info, len(seq))
    return batch._gdn_chunks


_SMS: int | None = None
_CHUNK_US = 10.0  # one 64-token chunk of the tensor-core chunked GDN prefill (B200)


def _chunked_is_faster(batch: ForwardBatch, hv: int) -> bool:
    """Pick the chunked prefill or the token scan for this batch from a cost model fitted on B200.

    Token scan: one CTA per (value head, sequence), two per SM, about 2.9 us per
    token step, so waves x longest length.  Chunked (tensor-core form): one CTA per
    (value head, sequence), one per SM, about ``_CHUNK_US`` per 64-token chunk in
    order, plus a fixed cost for the conv-window and norm kernels.
    """
    global _SMS
    if _SMS is None:
        _SMS = torch.cuda.get_device_properties(batch.cu_seqlens_q.device).multi_processor_count
    cu = batch.cu_seqlens_host
    b = len(cu) - 1
    lens = [cu[i + 1] - cu[i] for i in range(b)]
    lmax = max(lens, default=0)
    if lmax < 2:
        return False
    ceil = lambda x, y: -(-x // y)  # noqa: E731
    scan = ceil(b * hv, 2 * _SMS) * lmax * 2.9
    chunked = ceil(hv * b, _SMS) * ceil(lmax, GDN_CHUNK) * _CHUNK_US + 10.0
    return chunked < scan


def gdn(proj: torch.Tensor, batch: ForwardBatch, conv_w, a_log, dt_bias, norm_w, rec_pool, conv_pool, *,
        hk: int, hv: int, dk: int, dv: int, eps: float) -> torch.Tensor:
    """Gated DeltaNet mixer core (conv, norms, delta rule, gated norm); states updated in the pools."""
    if proj.is_cuda:
        c = cuda_ops()
        if batch.is_prefill and proj.dtype == torch.bfloat16 and _GDN_CHUNKED and _chunked_is_faster(batch, hv):
            info, nc = gdn_chunk_table(batch)
            return c.gdn_prefill_chunked(proj, batch.cu_seqlens_q, batch.state_slots, info, nc, conv_w, a_log,
                                         dt_bias, norm_w, rec_pool, conv_pool, hk, hv, eps)
        if batch.is_prefill:
            return c.gdn_prefill(proj, batch.cu_seqlens_q, batch.state_slots, conv_w, a_log, dt_bias, norm_w,
                                 rec_pool, conv_pool, hk, hv, dk, dv, eps, batch.max_seqlen_q)
        return c.gdn_decode(proj, batch.state_slots, conv_w, a_log, dt_bias, norm_w, rec_pool, conv_pool,
                            hk, hv, dk, dv, eps)
    return ref.gdn_forward(proj, batch.cu_seqlens_host, batch.slots_host, conv_w, a_log, dt_bias, norm_w,
                           rec_pool, conv_pool, hk=hk, hv=hv, dk=dk, dv=dv, eps=eps)


def gdn_verify(proj: torch.Tensor, batch: ForwardBatch, conv_w, a_log, dt_bias, norm_w, rec_pool, conv_pool,
               rec_k: torch.Tensor, rec_delta: torch.Tensor, rec_g: torch.Tensor, conv_hist: torch.Tensor, *,
               hk: int, hv: int, dk: int, dv: int, eps: float) -> torch.Tensor:
    """GDN mixer over speculative rows without touching the slot pools.

    Every token row ``t`` records its replay terms (``rec_k[t] = k_t``,
    ``rec_delta[t] = delta_t``, ``rec_g[t] = log decay_t``) and the conv window
    after it (``conv_hist[t]``), so the accepted prefix can later be folded into
    the pool state (``gdn_replay_commit``) and its conv window copied
    (``gdn_conv_commit``).  Parity: the reference's ReplaySSM verify
    (``nanovllm/engine/model_runner.py:1520-1569``).
    """
    if proj.is_cuda:
        rows = torch.arange(proj.shape[0], device=proj.device, dtype=torch.int32)
        return cuda_ops().gdn_scan_history(proj, batch.cu_seqlens_q, batch.state_slots, conv_w, a_log, dt_bias,
                                           norm_w, rec_pool, conv_pool, hk, hv, eps, False, rows, None, conv_hist,
                                           rec_k, rec_delta, rec_g)
    out = torch.empty(proj.shape[0], hv * dv, dtype=proj.dtype, device=proj.device)
    cu = batch.cu_seqlens_host
    for i, slot in enumerate(batch.slots_host):
        s, e = cu[i], cu[i + 1]
        if e == s:
            continue
        y, _, _, _, conv_h, (k, d, g) = ref.gdn_sequence(
            proj[s:e], conv_w, a_log, dt_bias, norm_w, rec_pool[slot], conv_pool[slot], hk=hk, hv=hv, dk=dk,
            dv=dv, eps=eps, history_at=list(range(e - s)), return_records=True)
        out[s:e] = y
        rec_k[s:e] = k
        rec_delta[s:e] = d
        rec_g[s:e] = g
        conv_hist[s:e] = torch.stack(conv_h)
    return out


def gdn_verify_snapshots(proj: torch.Tensor, batch: ForwardBatch, conv_w, a_log, dt_bias, norm_w, rec_pool,
                         conv_pool, hist_rec: torch.Tensor, conv_hist: torch.Tensor, *, hk: int, hv: int, dk: int,
                         dv: int, eps: float) -> torch.Tensor:
    """GDN mixer over speculative rows without touching the slot pools, keeping the full state after
    every row (``hist_rec[t]``, ``conv_hist[t]``): the accepted row's state is then copied into the
    pool.  The snapshot alternative to replay records (more memory, no fold at commit); parity: the
    reference's minimal-snapshot verify (``nanovllm/engine/model_runner.py:1570-1652``)."""
    if proj.is_cuda:
        rows = torch.arange(proj.shape[0], device=proj.device, dtype=torch.int32)
        return cuda_ops().gdn_scan_history(proj, batch.cu_seqlens_q, batch.state_slots, conv_w, a_log, dt_bias,
                                           norm_w, rec_pool, conv_pool, hk, hv, eps, False, rows, hist_rec, conv_hist,
                                           None, None, None)
    out = torch.empty(proj.shape[0], hv * dv, dtype=proj.dtype, device=proj.device)
    cu = batch.cu_seqlens_host
    for i, slot in enumerate(batch.slots_host):
        s, e = cu[i], cu[i + 1]
        if e == s:
            continue
        y, _, _, rh, ch, _ = ref.gdn_sequence(proj[s:e], conv_w, a_log, dt_bias, norm_w, rec_pool[slot],
                                              conv_pool[slot], hk=hk, hv=hv, dk=dk, dv=dv, eps=eps,
                                              history_at=list(range(e - s)))
        out[s:e] = y
        hist_rec[s:e] = torch.stack(rh)
        conv_hist[s:e] = torch.stack(ch)
    return out


def gdn_with_history(proj: torch.Tensor, batch: ForwardBatch, conv_w, a_log, dt_bias, norm_w, rec_pool, conv_pool,
                     rows: torch.Tensor, hist_rec: torch.Tensor, hist_conv: torch.Tensor, *, hk: int, hv: int, dk: int,
                     dv: int, eps: float) -> torch.Tensor:
    """GDN mixer that also records the state after selected tokens (token-recurrent scan).

    ``rows[t] >= 0`` marks token row ``t``: the recurrent / conv state right after
    it goes to ``hist_rec[rows[t]]`` / ``hist_conv[rows[t]]``; the final states are
    written back to the pools as usual.  Used for hybrid prefix checkpoints taken
    inside a prefill chunk (reference: ``capture_tensors`` of internal
    checkpoints, ``nanovllm/engine/state_manager.py:328-546``).
    """
    if proj.is_cuda:
        return cuda_ops().gdn_scan_history(proj, batch.cu_seqlens_q, batch.state_slots, conv_w, a_log, dt_bias,
                                           norm_w, rec_pool, conv_pool, hk, hv, eps, True, rows, hist_rec,
                                           hist_conv, None, None, None)
    out = torch.empty(proj.shape[0], hv * dv, dtype=proj.dtype, device=proj.device)
    cu = batch.cu_seqlens_host
    rows_h = rows.tolist()
    for i, slot in enumerate(batch.slots_host):
        s, e = cu[i], cu[i + 1]
        if e == s:
            continue
        marks = [t - s for t in range(s, e) if rows_h[t] >= 0]
        y, rec, conv, rh, ch, _ = ref.gdn_sequence(proj[s:e], conv_w, a_log, dt_bias, norm_w, rec_pool[slot],
                                                   conv_pool[slot], hk=hk, hv=hv, dk=dk, dv=dv, eps=eps,
                                                   history_at=marks)
        out[s:e] = y
        rec_pool[slot] = rec
        conv_pool[slot] = conv
        for local, r_state, c_state in zip(marks, rh, ch):
            hist_rec[rows_h[s + local]] = r_state
            hist_conv[rows_h[s + local]] = c_state
    return out


def lm_head_sample(hidden: torch.Tensor, weight: torch.Tensor, temperatures: torch.Tensor, rng: torch.Tensor,
                   vocab_offset: int) -> tuple[torch.Tensor, torch.Tensor]:
    """LM-head GEMM fused with greedy / Gumbel-max selection over this rank's vocab slice.

    ``rng`` is an int32 device tensor ``[seed, step]`` (read on the device, so a
    captured CUDA graph samples fresh noise every replay).  Returns
    ``(score [B] fp32, token [B] int32)`` where ``score`` is the winning
    (perturbed) logit, comparable across ranks for the cross-rank argmax.
    """
    if hidden.is_cuda:
        return cuda_ops().lm_head_sample(hidden, weight, temperatures, rng, vocab_offset)
    logits = ref.gemm(hidden, weight).float()
    seed, step = (int(v) for v in rng.tolist())
    val, idx = gumbel_select(logits, temperatures, seed, step, vocab_offset)
    return val, idx.to(torch.int32)


# ----------------------------------------------------------------- RNG
_M32 = 0xFFFFFFFF


def _fmix32(h: torch.Tensor) -> torch.Tensor:
    h = h & _M32
    h = h ^ (h >> 16)
    h = (h * 0x85EBCA6B) & _M32
    h = h ^ (h >> 13)
    h = (h * 0xC2B2AE35) & _M32
    h = h ^ (h >> 16)
    return h


def uniform_noise(seed: int, step: int, rows: torch.Tensor, cols: torch.Tensor) -> torch.Tensor:
    """Counter-based uniform(0,1) noise keyed by (seed, step, row, global vocab id).

    The same integer hash (MurmurHash3's 32-bit finaliser applied to a mixed
    key) runs in the CUDA sampling epilogue, so a token choice does not depend
    on the tensor-parallel split of the vocabulary.
    """
    key = (seed * 0x9E3779B1 + step * 0x85EBCA77) & _M32
    h = _fmix32(rows.long() * 0x27D4EB2F + key)
    h = _fmix32(h ^ (cols.long() * 0x165667B1 & _M32))
    return ((h >> 8).double() + 0.5) / float(1 << 24)


def gumbel_select(logits: torch.Tensor, temperatures: torch.Tensor, seed: int, step: int,
                  vocab_offset: int) -> tuple[torch.Tensor, torch.Tensor]:
    b, v = logits.shape
    greedy = temperatures.float() <= 1e-10
    rows = torch.arange(b, device=logits.device)[:, None]
    cols = torch.arange(v, device=logits.device)[None, :] + vocab_offset
    u = uniform_noise(seed, step, rows, cols)
    g = (-torch.log(-torch.log(u))).float()
    t = torch.where(greedy, torch.ones_like(temperatures.float()), temperatures.float())
    score = torch.where(greedy[:, None], logits, logits / t[:, None] + g)
    val, idx = score.max(dim=-1)
    return val, idx + vocab_offset


# ------------------------------------------------------- state maintenance
def gdn_replay_commit(rec_states: torch.Tensor, slot_ids: torch.Tensor, keys: torch.Tensor, deltas: torch.Tensor,
                      log_decays: torch.Tensor, commit_lengths: torch.Tensor, num_steps: int) -> None:
    """In place: ``S[l, slot_b] <- fold_{t < len_b} (exp(g_t) S + k_t delta_t^T)``."""
    if rec_states.is_cuda:
        cuda_ops().gdn_replay_commit(rec_states, slot_ids, keys, deltas, log_decays, commit_lengths, num_steps)
        return
    b = slot_ids.numel()
    idx = slot_ids.long()
    state = rec_states.index_select(1, idx)
    rows = b * num_steps  # records are [L, rows >= b*steps, ...]; the first b*steps rows are read
    k = keys[:, :rows].reshape(keys.shape[0], b, num_steps, *keys.shape[2:]).float()
    d = deltas[:, :rows].reshape(deltas.shape[0], b, num_steps, *deltas.shape[2:]).float()
    g = log_decays[:, :rows].reshape(log_decays.shape[0], b, num_steps, *log_decays.shape[2:]).float()
    lens = commit_lengths.long()
    for t in range(num_steps):
        upd = state * g[:, :, t].exp()[..., None, None] + torch.einsum("lbhd,lbhv->lbhdv", k[:, :, t], d[:, :, t])
        state = torch.where((lens > t).view(1, b, 1, 1, 1), upd, state)
    rec_states.index_copy_(1, idx, state)


def gdn_conv_commit(conv_states: torch.Tensor, conv_history: torch.Tensor, slot_ids: torch.Tensor,
                    boundaries: torch.Tensor, num_steps: int) -> None:
    """``conv[l, slot_b] <- conv_history[l, b * num_steps + boundaries[b]]``."""
    if conv_states.is_cuda:
        cuda_ops().gdn_conv_commit(conv_states, conv_history, slot_ids, boundaries, num_steps)
        return
    b = slot_ids.numel()
    rows = torch.arange(b) * num_steps + boundaries.long().cpu()
    conv_states.index_copy_(1, slot_ids.long(), conv_history.index_select(1, rows.to(conv_history.device)))


def quantize_state_int8(state: torch.Tensor, q_out: torch.Tensor, scale_out: torch.Tensor) -> None:
    """Symmetric int8 along the last (value) dim with an fp32 scale per row."""
    if state.is_cuda:
        cuda_ops().quantize_state_int8(state, q_out, scale_out)
        return
    s = state.float()
    scale = (s.abs().amax(dim=-1, keepdim=True) / 127.0).clamp(min=1e-8)
    q_out.copy_(torch.round(s / scale).clamp(-127, 127).to(torch.int8))
    scale_out.copy_(scale)


def dequantize_state_int8(q: torch.Tensor, scale: torch.Tensor, out: torch.Tensor) -> None:
    if q.is_cuda:
        cuda_ops().dequantize_state_int8(q, scale, out)
        return
    out.copy_(q.float() * scale)


def copy_kv_page(k_cache: torch.Tensor, v_cache: torch.Tensor, src_block: int, dst_block: int, num_tokens: int) -> None:
    """Copy-on-write of the first ``num_tokens`` rows of a page (all KV heads, K and V)."""
    if k_cache.is_cuda:
        cuda_ops().copy_kv_page(k_cache, v_cache, src_block, dst_block, num_tokens)
        return
    k_cache[dst_block, :, :num_tokens] = k_cache[src_block, :, :num_tokens]
    v_cache[dst_block, :, :num_tokens] = v_cache[src_block, :, :num_tokens]
