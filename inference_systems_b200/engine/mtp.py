"""Native multi-token-prediction (MTP) speculative decoding.

Parity (behaviour): ``nanovllm/engine/model_runner.py:1281-1792``
(``run_speculative``), ``:460-555`` (``_seed_mtp_prefill``), ``:604-666``
(``_mtp_step``) and ``nanovllm/engine/speculative.py:8-129`` -- greedy
drafting with the one-layer MTP head, parallel verification by the target,
longest-matching-prefix acceptance with the target's token at the first
mismatch, GDN state rolled back to the accepted boundary, shifted MTP KV
(the MTP entry at cache position ``q`` pairs token ``q+1`` with the target
hidden state of token ``q``).

Design (one target pass per round, everything on the device):

* A sequence enters a round with its pending token ``t_P`` (position ``P``,
  not yet run) and ``K`` drafts ``d_0..d_{K-1}`` kept on the device per state
  slot.  The target runs ONE varlen pass over ``[t_P, d_0, .., d_{K-1}]``
  (positions ``P..P+K``) -- the reference runs a separate target decode
  before its verify pass.  Its GDN layers leave the slot pools untouched and
  record compact replay terms ``(k_t, delta_t, log decay_t)`` plus the conv
  window after every row (``ops.gdn_verify``).
* The LM head picks ``v_j`` for every row; ``a`` = number of leading drafts
  equal to ``v_j``; the round emits ``v_0..v_a`` and ``v_a`` is the new
  pending token.  Acceptance is a few tensor ops: no host sync until the
  single device->host copy of ``(v, a)``.
* Commit folds the first ``a+1`` replay terms into the pool state in place
  (``gdn_replay_commit``) and copies the conv window after row ``a``
  (``gdn_conv_commit``).  Attention KV rows past the accepted boundary are
  simply overwritten later.
* The MTP head then catches up over the same ``K+1`` rows (token ``v_j``,
  hidden ``h_{P+j}``, cache position ``P+j``) -- the pairs for the accepted
  rows are exactly right and the rest are overwritten next round -- and its
  output at row ``a`` proposes the next round's first draft; ``K-1`` one-row
  MTP steps propose the rest.
* After a prefill chunk the same catch-up runs over the chunk's rows (the
  token after the chunk is the next prompt token or the sampled one), so no
  per-slot "previous hidden" buffer is needed across chunks.

``mtp_synthetic_acceptance = p`` (benchmark hook) makes the verifier agree
with each draft with probability ``p`` (a counter-based hash of the step
seed), so MTP throughput can be measured on random-weight models whose drafts
never match.  Emitted tokens then follow the drafts, and the state stays
consistent with what was emitted.
"""

from __future__ import annotations

from dataclasses import replace
from time import perf_counter_ns

import numpy as np
import torch

from inference_systems_b200 import ops
from inference_systems_b200.engine.sequence import Sequence
from inference_systems_b200.utils.context import ForwardBatch

_M32 = 0xFFFFFFFF


def _fmix32(h: torch.Tensor) -> torch.Tensor:
    h = h & _M32
    h = h ^ (h >> 16)
    h = (h * 0x85EBCA6B) & _M32
    h = h ^ (h >> 13)
    h = (h * 0xC2B2AE35) & _M32
    return h ^ (h >> 16)


def synthetic_uniform(rng: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """Uniform(0,1) ``[rows, cols]`` keyed by the device ``rng = [seed, step]`` (no host sync)."""
    r = rng.long()
    key = (r[0] * 0x9E3779B1 + r[1] * 0x85EBCA77 + 0x6A09E667) & _M32
    i = torch.arange(rows, device=rng.device, dtype=torch.int64)[:, None]
    j = torch.arange(cols, device=rng.device, dtype=torch.int64)[None, :]
    h = _fmix32(i * 0x27D4EB2F + key)
    h = _fmix32(h ^ ((j * 0x165667B1) & _M32))
    return ((h >> 8).float() + 0.5) / float(1 << 24)


def slot_of(block_tables: torch.Tensor, pos: torch.Tensor, block_size: int) -> torch.Tensor:
    """KV-cache slot of each (row, position); -1 where the page is not allocated."""
    page = (pos // block_size).long().clamp(max=block_tables.shape[1] - 1)
    blk = block_tables.gather(1, page if page.dim() == 2 else page[:, None])
    blk = blk if page.dim() == 2 else blk[:, 0]
    return torch.where(blk >= 0, blk * block_size + pos % block_size, torch.full_like(blk, -1)).to(torch.int32)


class MTPDriver:
    def __init__(self, runner):
        self.r = runner
        cfg = runner.config
        self.k = int(runner.num_speculative_tokens)
        self.synthetic = float(getattr(cfg, "mtp_synthetic_acceptance", None) or 0.0)
        dev = runner.device
        sm = runner.state_manager
        n_slots = (sm.max_num_seqs + 1) if sm is not None else cfg.max_num_seqs + 1
        self.drafts = torch.zeros(n_slots, self.k, dtype=torch.int32, device=dev)
        self.max_rows = cfg.max_num_seqs * (self.k + 1)
        geo = runner.model.gdn_geometry()
        # verify records: compact replay terms folded at commit (default), or full state snapshots
        # after every verify row copied at commit (``enable_mtp_replay_ssm=False``)
        self.replay = getattr(cfg, "enable_mtp_replay_ssm", None) is not False
        self.rec_k = self.hist_rec = None
        if geo is not None:
            L, hv, dk, dv = geo["num_layers"], geo["hv"], geo["dk"], geo["dv"]
            rows = self.max_rows
            if self.replay:
                self.rec_k = torch.zeros(L, rows, hv, dk, dtype=torch.float32, device=dev)
                self.rec_delta = torch.zeros(L, rows, hv, dv, dtype=torch.float32, device=dev)
                self.rec_g = torch.zeros(L, rows, hv, dtype=torch.float32, device=dev)
            else:
                need = L * rows * hv * dk * dv * 4
                if dev.type == "cuda" and need > torch.cuda.mem_get_info(dev)[0] // 4:
                    raise ValueError(f"MTP state snapshots need {need / 2**30:.1f} GiB for {rows} verify rows; "
                                     "use enable_mtp_replay_ssm=True or fewer max_num_seqs")
                self.hist_rec = torch.zeros(L, rows, hv, dk, dv, dtype=torch.float32, device=dev)
            self.conv_hist = torch.zeros(L, rows, geo["conv_dim"], geo["kernel"] - 1, dtype=runner.dtype, device=dev)
        n_attn = len(runner.model.attn_layer_ids)
        self.kv_index = n_attn  # the MTP layer is the last layer of the KV cache
        self.before_round = None  # test hook: callable(seqs, driver) run before each verify pass
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.graph_bufs: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        self.graph_replays = 0
        self.reset_metrics()

    # ------------------------------------------------------------ helpers
    def mtp_kv(self):
        kv = self.r.kv_cache
        return kv[self.kv_index, 0], kv[self.kv_index, 1]

    def reset_metrics(self) -> None:
        self.rounds = 0
        self.seq_rounds = 0
        self.draft_tokens = 0
        self.accepted_tokens = 0
        self.emitted_tokens = 0
        self.accept_hist = [0] * (self.k + 1)
        self.prefill_catchups = 0

    def metrics(self) -> dict:
        d = max(self.draft_tokens, 1)
        return {
            "rounds": self.rounds,
            "draft_tokens": self.draft_tokens,
            "accepted_tokens": self.accepted_tokens,
            "emitted_tokens": self.emitted_tokens,
            "acceptance_rate": self.accepted_tokens / d,
            "sequence_rounds": self.seq_rounds,
            "mean_emitted_per_round": self.emitted_tokens / max(self.seq_rounds, 1),
            "accepted_length_histogram": list(self.accept_hist),
            "prefill_catchups": self.prefill_catchups,
            "synthetic_acceptance": self.synthetic,
            "verify_records": "replay" if self.replay else "snapshot",
            "cudagraph_buckets": sorted(self.graphs),
            "cudagraph_replays": self.graph_replays,
        }

    def set_drafts(self, state_slot: int, tokens) -> None:
        self.drafts[state_slot] = torch.as_tensor(tokens, dtype=torch.int32, device=self.drafts.device)

    def _gdn_records(self, t: int):
        if self.rec_k is not None:
            return [(self.rec_k[j, :t], self.rec_delta[j, :t], self.rec_g[j, :t], self.conv_hist[j, :t])
                    for j in range(self.rec_k.shape[0])]
        if self.hist_rec is not None:
            return [(self.hist_rec[j, :t], self.conv_hist[j, :t]) for j in range(self.hist_rec.shape[0])]
        return None

    def _sample(self, hidden: torch.Tensor, rng: torch.Tensor) -> torch.Tensor:
        temps = torch.zeros(hidden.shape[0], dtype=torch.float32, device=hidden.device)
        return self.r.model.sample(hidden, temps, rng)

    def _draft_steps(self, tok: torch.Tensor, hid: torch.Tensor, base: torch.Tensor, block_tables: torch.Tensor,
                     caps: torch.Tensor, state_slots: torch.Tensor, rng: torch.Tensor, slots_host: list[int],
                     max_k: int) -> torch.Tensor:
        """K-1 one-row MTP steps from the first draft ``tok`` / MTP hidden ``hid``; returns ``[B, K]``."""
        b = tok.shape[0]
        out = [tok]
        dev = tok.device
        cu = torch.arange(b + 1, dtype=torch.int32, device=dev)
        for j in range(1, self.k):
            pos = base + j  # MTP cache position of this step's pair
            ctx = torch.minimum(pos + 1, caps).to(torch.int32)
            sm = torch.where(pos < caps, slot_of(block_tables, pos, self.r.block_size), torch.full_like(pos, -1))
            batch = ForwardBatch(
                is_prefill=False, input_ids=tok, positions=(pos + 1).to(torch.int32), cu_seqlens_q=cu,
                context_lens=ctx, block_tables=block_tables, slot_mapping=sm.to(torch.int32),
                state_slots=state_slots, logits_indices=cu[1:] - 1, max_seqlen_q=1, max_seqlen_k=max_k + j,
                cu_seqlens_host=list(range(b + 1)), slots_host=slots_host, num_seqs=b)
            hid = self.r.mtp(batch, hid, self.mtp_kv())
            tok = self._sample(hid, rng)
            out.append(tok)
        return torch.stack(out, dim=1)

    # ------------------------------------------------------------ prefill
    @torch.inference_mode()
    def after_prefill(self, seqs: list[Sequence], batch: ForwardBatch, hidden: torch.Tensor, sampled: torch.Tensor,
                      rng: torch.Tensor) -> None:
        """MTP catch-up over a prefill chunk; drafts for sequences whose prompt completed."""
        t0 = perf_counter_ns()
        nxt, done_rows, done_idx, base, caps = [], [], [], [], []
        row = 0
        for i, s in enumerate(seqs):
            start, n = s.num_cached_tokens, s.num_scheduled_tokens
            for p in range(start, start + n):
                nxt.append(s.token_ids[p + 1] if p + 1 < s.num_tokens else -1)
            row += n
            if start + n == s.num_tokens:
                done_rows.append(row - 1)
                done_idx.append(i)
                base.append(start + n - 1)
                caps.append(len(s.block_table) * self.r.block_size)
        dev = hidden.device
        ids = torch.as_tensor(np.asarray(nxt, np.int32), device=dev)
        if done_rows:
            r_t = torch.as_tensor(done_rows, dtype=torch.long, device=dev)
            ids[r_t] = sampled.index_select(0, torch.as_tensor(done_idx, dtype=torch.long, device=dev)).to(ids.dtype)
        cbatch = replace(batch, input_ids=ids, positions=batch.positions + 1, gdn_verify=None)
        m = self.r.mtp(cbatch, hidden, self.mtp_kv())
        self.prefill_catchups += 1
        if done_rows and self.k > 0:
            r_t = torch.as_tensor(done_rows, dtype=torch.long, device=dev)
            sel = torch.as_tensor(done_idx, dtype=torch.long, device=dev)
            m_sel = m.index_select(0, r_t)
            tok = self._sample(m_sel, rng)
            bt = batch.block_tables.index_select(0, sel)
            st = batch.state_slots.index_select(0, sel)
            drafts = self._draft_steps(tok, m_sel, torch.as_tensor(base, dtype=torch.int32, device=dev), bt,
                                       torch.as_tensor(caps, dtype=torch.int32, device=dev), st, rng,
                                       [batch.slots_host[i] for i in done_idx], max(base) + 1)
            self.drafts.index_copy_(0, st.long(), drafts)
        self.r.profiler.record_cpu("mtp.prefill_catchup", (perf_counter_ns() - t0) / 1e6)

    # -------------------------------------------------------------- round
    def _pack(self, seqs: list[Sequence], pad_to: int) -> np.ndarray:
        """``[pending | position | state slot | page capacity | rng(2) | block tables]`` int32.

        Rows past ``len(seqs)`` are padding: scratch state slot, no pages, zero
        capacity (so every kernel sees an empty context for them).
        """
        r = self.r
        b, mb = len(seqs), r.max_blocks_per_seq
        scratch = r.state_manager.scratch_slot_id if r.state_manager is not None else 0
        pend = np.zeros(pad_to, np.int32)
        pos0 = np.zeros(pad_to, np.int32)
        st = np.full(pad_to, scratch, np.int32)
        caps = np.zeros(pad_to, np.int32)
        bt = np.full((pad_to, mb), -1, dtype=np.int32)
        for i, s in enumerate(seqs):
            pend[i] = s.last_token
            pos0[i] = len(s) - 1
            st[i] = s.state_slot if s.state_slot is not None else scratch
            caps[i] = len(s.block_table) * r.block_size
            bt[i, :len(s.block_table)] = s.block_table
        rng = np.asarray([r.config.seed & 0x7FFFFFFF, r.sample_step & 0x7FFFFFFF], np.int32)
        return np.concatenate([pend, pos0, st, caps, rng, bt.reshape(-1)])

    def _round_device(self, meta: torch.Tensor, b: int, slots_host: list[int] | None,
                      max_k: int) -> torch.Tensor:
        """Device work of one round over ``b`` (possibly padded) rows; returns ``[v (b*(K+1)) | a (b)]`` int32.

        Host values are used only by the CPU reference path (``slots_host``,
        ``max_k``), so the body can be captured in a CUDA graph per batch bucket.
        """
        r = self.r
        k, bs = self.k, r.block_size
        mb = r.max_blocks_per_seq
        pend_d, pos_d, st_d, caps_d = (meta[i * b:(i + 1) * b] for i in range(4))
        rng_d = meta[4 * b:4 * b + 2]
        bt_d = meta[4 * b + 2:4 * b + 2 + b * mb].view(b, mb)
        dev = meta.device
        valid = caps_d > 0

        # ---- verify: one target pass over [pending, drafts]
        ar = torch.arange(k + 1, dtype=torch.int32, device=dev)
        drafts = self.drafts.index_select(0, st_d.long())                      # [B, K]
        ids = torch.cat((pend_d[:, None], drafts), dim=1).reshape(-1)
        pos2 = pos_d[:, None] + ar[None, :]                                    # [B, K+1]
        sm = slot_of(bt_d, pos2, bs).reshape(-1)
        t = b * (k + 1)
        cu = torch.arange(b + 1, dtype=torch.int32, device=dev) * (k + 1)
        ctx = torch.where(valid, pos_d + k + 1, torch.zeros_like(pos_d)).to(torch.int32)
        # every verify row attends as its own decode query: row j of a sequence sees positions <= P + j
        row_ctx = torch.where(valid[:, None], pos2 + 1, torch.zeros_like(pos2)).reshape(-1).to(torch.int32)
        row_bt = bt_d.repeat_interleave(k + 1, dim=0)
        vbatch = ForwardBatch(
            is_prefill=True, input_ids=ids, positions=pos2.reshape(-1).to(torch.int32), cu_seqlens_q=cu,
            context_lens=ctx, block_tables=bt_d, slot_mapping=sm, state_slots=st_d, logits_indices=cu[1:] - 1,
            max_seqlen_q=k + 1, max_seqlen_k=max_k, cu_seqlens_host=[i * (k + 1) for i in range(b + 1)],
            slots_host=slots_host or [], num_seqs=b, gdn_verify=self._gdn_records(t),
            decode_rows=(row_ctx, row_bt))
        hidden = r.model(vbatch, r.kv_layers(), r.state_layers())
        v = self._sample(hidden, rng_d).view(b, k + 1)
        if self.synthetic > 0.0 and k > 0:
            agree = synthetic_uniform(rng_d, b, k) < self.synthetic
            v = torch.cat((torch.where(agree, drafts, v[:, :k]), v[:, k:]), dim=1)
        if k > 0:
            acc = torch.cumprod((drafts == v[:, :k]).to(torch.int32), dim=1).sum(dim=1).to(torch.int32)
        else:
            acc = torch.zeros(b, dtype=torch.int32, device=dev)

        # ---- commit the accepted prefix of the GDN state
        sm_mgr = r.state_manager
        if sm_mgr is not None and self.rec_k is not None:
            ops.gdn_replay_commit(sm_mgr.recurrent_states, st_d, self.rec_k, self.rec_delta, self.rec_g, acc + 1, k + 1)
            ops.gdn_conv_commit(sm_mgr.conv_states, self.conv_hist, st_d, acc, k + 1)
        elif sm_mgr is not None and self.hist_rec is not None:
            # the snapshot after the last accepted row becomes the slot's state, in every GDN layer
            accepted_row = (torch.arange(b, device=dev) * (k + 1) + acc).long()
            sm_mgr.recurrent_states[:, st_d.long()] = self.hist_rec[:, accepted_row]
            ops.gdn_conv_commit(sm_mgr.conv_states, self.conv_hist, st_d, acc, k + 1)

        # ---- MTP catch-up over the verified rows, then the next drafts
        if k > 0:
            cbatch = replace(vbatch, input_ids=v.reshape(-1), positions=vbatch.positions + 1, gdn_verify=None)
            m = r.mtp(cbatch, hidden, self.mtp_kv())
            rows = torch.arange(b, dtype=torch.long, device=dev) * (k + 1) + acc.long()
            m_sel = m.index_select(0, rows)
            tok = self._sample(m_sel, rng_d)
            new = self._draft_steps(tok, m_sel, (pos_d + acc).to(torch.int32), bt_d, caps_d, st_d, rng_d,
                                    slots_host or [], max_k)
            self.drafts.index_copy_(0, st_d.long(), new)
        return r.with_status(torch.cat((v.reshape(-1).to(torch.int32), acc)))

    # ---------------------------------------------------------- graphs
    def _bucket(self, b: int) -> int | None:
        for s in sorted(self.graphs):
            if s >= b:
                return s
        return None

    @torch.inference_mode()
    def capture(self, sizes: list[int]) -> None:
        """One CUDA graph per batch bucket for the whole round (verify, accept, commit, drafts)."""
        r = self.r
        pool = None
        for b in sorted(sizes, reverse=True):
            flat = self._pack([], b)
            meta = torch.from_numpy(flat).to(r.device)
            big = int(r.config.max_model_len) + 2 * self.k + 1
            self._round_device(meta, b, None, big)  # warm-up outside the capture
            torch.cuda.synchronize(r.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                out = self._round_device(meta, b, None, big)
            if pool is None:
                pool = g.pool()
            self.graphs[b] = g
            self.graph_bufs[b] = (meta, out)
        torch.cuda.synchronize(r.device)
        if r.state_manager is not None:
            r.state_manager.reset_scratch()

    @torch.inference_mode()
    def run(self, seqs: list[Sequence]):
        """One speculative round for a decode batch; returns emitted token lists (rank 0)."""
        t0 = perf_counter_ns()
        r = self.r
        k = self.k
        b = len(seqs)
        if self.before_round is not None:
            self.before_round(seqs, self)
        bucket = self._bucket(b) if self.graphs else None
        if bucket is not None:
            flat = self._pack(seqs, bucket)
            meta, out_dev = self.graph_bufs[bucket]
            pinned = r._pinned(flat.shape[0])
            pinned[: flat.shape[0]].copy_(torch.from_numpy(flat))
            meta.copy_(pinned[: flat.shape[0]], non_blocking=True)
            r.h2d_bytes += flat.nbytes
            self.graphs[bucket].replay()
            self.graph_replays += 1
            tb = bucket * (k + 1)
            host = out_dev.to("cpu")
            r.d2h_bytes += host.numel() * 4
            r.check_status(host)
            vals = host[:tb].view(bucket, k + 1)[:b].tolist()
            accs = host[tb:tb + b].tolist()
        else:
            flat = self._pack(seqs, b)
            meta = r._upload(flat)
            slots_host = [s.state_slot if s.state_slot is not None else 0 for s in seqs]
            max_k = max(len(s) for s in seqs) + k
            host = self._round_device(meta, b, slots_host, max_k).to("cpu")
            r.d2h_bytes += host.numel() * 4
            r.check_status(host)
            t = b * (k + 1)
            vals = host[:t].view(b, k + 1).tolist()
            accs = host[t:t + b].tolist()  # the step's status word follows the accepted counts
        r.sample_step += 1
        out = [row[: a + 1] for row, a in zip(vals, accs)]
        self.rounds += 1
        self.seq_rounds += b
        self.draft_tokens += b * k
        self.accepted_tokens += int(sum(accs))
        self.emitted_tokens += int(sum(a + 1 for a in accs))
        for a in accs:
            self.accept_hist[a] += 1
        r.forward_calls += 1
        r.decode_tokens += int(sum(a + 1 for a in accs))
        r.profiler.record_cpu("mtp.round", (perf_counter_ns() - t0) / 1e6)
        return out if r.rank == 0 else None
