"""Continuous-batching scheduler.

Parity (behaviour): ``nanovllm/engine/scheduler.py:67-1784``.

* Policies: ``prefill_first`` (one prefill batch if any, else decode),
  ``decode_first`` (decode batch, then prefill with the leftover budget) and
  ``slo_aware`` (decode first; prefill budget bounded by the TPOT target from
  EWMA step-latency observations, deferred under KV pressure, widened under
  queue pressure) -- ``scheduler.py:640-776``.
* Chunked prefill up to ``max_num_batched_tokens``; with the hybrid prefix
  cache a chunk ends at the next retained checkpoint boundary so the GDN state
  can be captured there (``:1284-1419``).
* Admission: ``fcfs`` or ``hybrid_state_aware`` -- score = uncached tokens
  minus aging over a top-W window, overdue requests first, hysteresis against
  small wins, sticky recovery of requests that already hold resources
  (``:960-1142``).
* Preemption: ``lifo`` or ``recompute_aware`` (victim minimising recompute
  tokens per reclaimable block plus a repeat-preemption penalty,
  ``:1144-1282``); preempted requests free KV + state and recompute.
* Speculative decode reserves ``K + 1`` KV slots per step and trims the tail
  after commit (``:1421-1461``, ``:1731-1781``).
* Hybrid prefix capture transaction: prepare / reserve / publish / cancel
  (``:1527-1694``).

Design: counters live in one ``Counter`` (``self.stats``) instead of dozens of
attributes; ``get_metrics`` flattens it with the derived rates.
"""

from __future__ import annotations

from collections import Counter, deque
from dataclasses import dataclass
from time import perf_counter_ns

from inference_systems_b200.engine.block_manager import BlockManager
from inference_systems_b200.engine.hybrid_prefix_cache import (
    CheckpointBoundary,
    FullAttentionPrefixManager,
    GDNCheckpointManager,
    HybridCheckpointRetentionPolicy,
    HybridPrefixCoordinator,
    PendingHybridPrefixCapture,
    PrefixKVCandidate,
)
from inference_systems_b200.engine.profiler import PhaseProfiler
from inference_systems_b200.engine.sequence import Sequence, SequenceStatus


@dataclass
class ScheduledBatch:
    seqs: list[Sequence]
    is_prefill: bool

    @property
    def num_tokens(self) -> int:
        return sum(s.num_scheduled_tokens for s in self.seqs) if self.is_prefill else len(self.seqs)


@dataclass(frozen=True, slots=True)
class PrefixRecoveryProbe:
    kv_candidate_tokens: int
    gdn_checkpoint_tokens: int
    joint_recoverable_tokens: int
    scoring_reusable_tokens: int
    feasible: bool


@dataclass(frozen=True, slots=True)
class AdmissionProbe:
    sequence: Sequence
    queue_index: int
    reusable_tokens: int
    kv_candidate_tokens: int
    gdn_checkpoint_tokens: int
    joint_recoverable_tokens: int
    uncached_tokens: int
    age_ms: float
    score: float
    feasible: bool


@dataclass(frozen=True, slots=True)
class PreemptionProbe:
    sequence: Sequence
    computed_tokens: int
    logical_blocks: int
    reclaimable_blocks: int
    reusable_tokens: int
    recompute_tokens: int
    cost_per_block: float


def _cfg(config, name, default):
    return getattr(config, name, default)


def latency_summary(values) -> dict:
    if not values:
        return {"count": 0, "mean_us": 0.0, "p50_us": 0.0, "p95_us": 0.0, "p99_us": 0.0, "max_us": 0.0}
    s = sorted(values)

    def pct(p):
        return s[min(max(int(p * len(s) + 0.999999) - 1, 0), len(s) - 1)]

    return {"count": len(s), "mean_us": sum(s) / len(s), "p50_us": pct(0.5), "p95_us": pct(0.95),
            "p99_us": pct(0.99), "max_us": s[-1]}


class Scheduler:
    def __init__(self, config, state_manager=None, state_controller=None, prefix_checkpoint_pool=None):
        c = config
        self.max_num_seqs = c.max_num_seqs
        self.max_num_batched_tokens = c.max_num_batched_tokens
        self.eos = c.eos
        self.block_size = c.kvcache_block_size
        self.scheduling_policy = c.scheduling_policy
        self.waiting_admission_policy = _cfg(c, "waiting_admission_policy", "fcfs")
        self.preemption_policy = _cfg(c, "preemption_policy", "lifo")
        self.window = _cfg(c, "hybrid_scheduler_candidate_window", 8)
        self.aging_per_ms = _cfg(c, "hybrid_scheduler_aging_tokens_per_ms", 0.5)
        self.max_wait_ms = _cfg(c, "hybrid_scheduler_max_wait_ms", 200.0)
        self.min_saved_tokens = _cfg(c, "hybrid_scheduler_min_saved_tokens", 16)
        self.preemption_penalty = _cfg(c, "hybrid_scheduler_preemption_penalty", 128.0)
        self.score_source = _cfg(c, "hybrid_scheduler_score_source", "joint")
        self.enable_aging = _cfg(c, "hybrid_scheduler_enable_aging", True)
        self.enable_hysteresis = _cfg(c, "hybrid_scheduler_enable_hysteresis", True)
        self.enable_sticky = _cfg(c, "hybrid_scheduler_enable_sticky_recovery", True)
        self.enable_scheduler_profiling = _cfg(c, "enable_scheduler_profiling", False)
        hist = _cfg(c, "scheduler_decision_history_size", 4096)
        self.target_ttft_ms = _cfg(c, "scheduler_target_ttft_ms", 200.0)
        self.target_tpot_ms = _cfg(c, "scheduler_target_tpot_ms", 50.0)
        self.slo_prefill_priority_threshold = _cfg(c, "slo_prefill_priority_threshold", 0.8)
        self.slo_min_prefill_tokens = _cfg(c, "slo_min_prefill_tokens", 64)
        self.slo_kv_pressure_threshold = _cfg(c, "slo_kv_pressure_threshold", 0.9)
        self.slo_queue_pressure_threshold = _cfg(c, "slo_queue_pressure_threshold", 3)
        self.slo_latency_safety_margin_ms = _cfg(c, "slo_latency_safety_margin_ms", 5.0)
        self.ewma_alpha = _cfg(c, "scheduler_ewma_alpha", 0.2)
        self.state_manager = state_manager
        self.state_controller = state_controller
        self.enable_hybrid_prefix_cache = bool(_cfg(c, "enable_hybrid_prefix_cache", False) and state_manager is not None)
        self.enable_hybrid_internal_checkpoints = bool(
            self.enable_hybrid_prefix_cache and _cfg(c, "enable_hybrid_internal_checkpoints", False))
        self.hybrid_prefix_cache = None
        self.hybrid_prefix_coordinator = None
        self.hybrid_prefix_retention_policy = None
        self.hybrid_prefix_promotions: dict[int, tuple[CheckpointBoundary, int, PrefixKVCandidate, int]] = {}
        match_unit = _cfg(c, "prefix_match_unit", None) or c.kvcache_block_size
        if self.enable_hybrid_prefix_cache:
            if prefix_checkpoint_pool is None:
                raise ValueError("hybrid prefix cache requires a checkpoint pool")
            self.hybrid_prefix_cache = GDNCheckpointManager(
                prefix_checkpoint_pool.capacity, eviction_policy=_cfg(c, "hybrid_prefix_eviction_policy", "lru"))
            interval = (_cfg(c, "hybrid_prefix_checkpoint_interval_tokens", None)
                        or c.hybrid_prefix_checkpoint_interval_blocks * c.kvcache_block_size)
            self.hybrid_prefix_retention_policy = HybridCheckpointRetentionPolicy(
                block_size=match_unit, interval_tokens=interval,
                mode=_cfg(c, "hybrid_prefix_retention_policy", "periodic"))
        # A KV prefix hit alone is not a valid restart point for a model with
        # recurrent state; plain prefix caching is only on for stateless models.
        self.enable_prefix_cache = _cfg(c, "enable_prefix_cache", True) and (
            state_manager is None or self.enable_hybrid_prefix_cache)
        self.enable_chunked_prefill = _cfg(c, "enable_chunked_prefill", True)
        self.num_speculative_tokens = _cfg(c, "num_speculative_tokens", 0)
        self.block_manager = BlockManager(c.num_kvcache_blocks, c.kvcache_block_size, prefix_match_unit=match_unit)
        self.full_attention_prefix_manager = FullAttentionPrefixManager(self.block_manager)
        if self.hybrid_prefix_cache is not None:
            self.hybrid_prefix_coordinator = HybridPrefixCoordinator(
                self.full_attention_prefix_manager, self.hybrid_prefix_cache,
                promote_shared_junctions=_cfg(c, "hybrid_prefix_retention_policy", "periodic") == "adaptive",
                promotion_min_sightings=_cfg(c, "hybrid_prefix_promotion_min_sightings", 2),
                demand_capacity=max(prefix_checkpoint_pool.capacity * 16, 64))
        self.waiting: deque[Sequence] = deque()
        self.running: deque[Sequence] = deque()
        self.completed_request_metrics: deque[dict] = deque(maxlen=_cfg(c, "request_metrics_history_size", 1024))
        self.prefill_ms_per_token_ewma: float | None = None
        self.prefill_base_ms: float | None = None
        self.decode_step_ms_ewma: float | None = None
        self.mtp_phase_profiler = PhaseProfiler(_cfg(c, "enable_mtp_phase_profiling", False))
        self.admission_latency_us: deque[float] = deque(maxlen=hist)
        self.probe_latency_us: deque[float] = deque(maxlen=hist)
        self.preemption_latency_us: deque[float] = deque(maxlen=hist)
        self.decision_events: deque[dict] = deque(maxlen=hist)
        self.reset_metrics()

    # ------------------------------------------------------- state RPC
    def _allocate_state(self, seq: Sequence) -> None:
        if self.state_manager is None:
            return
        if self.state_controller is not None:
            self.state_controller.call("allocate_state_slot", seq)
        else:
            self.state_manager.allocate(seq)

    def _free_state(self, seq: Sequence) -> None:
        if self.state_manager is None or seq.state_slot is None:
            return
        if self.state_controller is not None:
            self.state_controller.call("free_state_slot", seq)
        else:
            self.state_manager.free(seq)

    def _state_available(self, seq: Sequence) -> bool:
        return self.state_manager is None or seq.state_slot is not None or self.state_manager.can_allocate

    # --------------------------------------------------------- metrics
    def reset_metrics(self) -> None:
        self.mtp_phase_profiler.reset()
        self.block_manager.reset_metrics()
        for d in (self.admission_latency_us, self.probe_latency_us, self.preemption_latency_us, self.decision_events):
            d.clear()
        self.completed_request_metrics.clear()
        self.stats: Counter = Counter()
        self.rank_histogram: Counter = Counter()
        self.max_observed_wait_ms = 0.0
        self.last_slo_decision: dict | None = None
        self.last_hybrid_scheduler_decision: dict | None = None
        if self.hybrid_prefix_coordinator is not None:
            self.hybrid_prefix_coordinator.reset_metrics()

    def get_scheduler_decision_events(self) -> list[dict]:
        return list(self.decision_events)

    def get_metrics(self) -> dict:
        s = self.stats
        eligible = s["prefix_cache_eligible_blocks"]
        decisions = s["hybrid_scheduler_admission_decisions"]
        m = {
            "prefix_cache_enabled": self.enable_prefix_cache,
            "prefix_cache_queries": s["prefix_cache_queries"],
            "prefix_cache_eligible_blocks": eligible,
            "prefix_cache_hit_blocks": s["prefix_cache_hit_blocks"],
            "prefix_cache_hit_rate": s["prefix_cache_hit_blocks"] / eligible if eligible else 0.0,
            "chunked_prefill_enabled": self.enable_chunked_prefill,
            "scheduling_policy": self.scheduling_policy,
            "waiting_admission_policy": self.waiting_admission_policy,
            "preemption_policy": self.preemption_policy,
            "num_waiting": len(self.waiting),
            "num_running": len(self.running),
            "kv_blocks_total": len(self.block_manager.blocks),
            "kv_blocks_used": len(self.block_manager.used_block_ids),
            "kv_pressure": self._kv_pressure(),
            "prefill_ms_per_token_ewma": self.prefill_ms_per_token_ewma,
            "prefill_base_ms": self.prefill_base_ms,
            "decode_step_ms_ewma": self.decode_step_ms_ewma,
            "last_slo_decision": self.last_slo_decision,
            "last_hybrid_scheduler_decision": self.last_hybrid_scheduler_decision,
            "hybrid_scheduler_selected_rank_histogram": dict(self.rank_histogram),
            "hybrid_scheduler_mean_selected_rank": (s["hybrid_scheduler_selected_original_rank_total"] / decisions
                                                    if decisions else 0.0),
            "hybrid_scheduler_max_observed_wait_ms": self.max_observed_wait_ms,
            "prefill_tokens_per_s": (s["prefill_observed_tokens"] / (s["prefill_observed_ms"] / 1e3)
                                     if s["prefill_observed_ms"] else 0.0),
            "decode_tokens_per_s": (s["decode_observed_tokens"] / (s["decode_observed_ms"] / 1e3)
                                    if s["decode_observed_ms"] else 0.0),
            "scheduler_admission_latency": latency_summary(self.admission_latency_us),
            "scheduler_probe_latency": latency_summary(self.probe_latency_us),
            "scheduler_preemption_latency": latency_summary(self.preemption_latency_us),
            "block_manager": {
                "prefix_cache_evictions": self.block_manager.prefix_cache_evictions,
                "cached_block_reassignments": self.block_manager.cached_block_reassignments,
                "duplicate_cache_registrations": self.block_manager.duplicate_cache_registrations,
                "partial_prefix_cow_allocations": self.block_manager.partial_prefix_cow_allocations,
                "cached_blocks": self.block_manager.num_cached_blocks,
            },
            "mtp_phase_profile": self.mtp_phase_profiler.metrics(),
        }
        for k, v in s.items():
            m.setdefault(k, v)
        for k in ("preemption_count", "aborted_request_count", "completed_request_count", "chunked_prefill_steps"):
            m.setdefault(k, 0)
        if self.hybrid_prefix_coordinator is not None:
            m.update(self.hybrid_prefix_coordinator.get_metrics())
        return m

    def get_request_metrics(self) -> list[dict]:
        return list(self.completed_request_metrics)

    # ---------------------------------------------------------- queue ops
    def is_finished(self) -> bool:
        return not self.waiting and not self.running

    def add(self, seq: Sequence) -> None:
        self.waiting.append(seq)

    def _retire(self, seq: Sequence, status: SequenceStatus, now_ns: int | None = None) -> None:
        seq.status = status
        seq.mark_finished(now_ns)
        if seq.block_table:
            self.block_manager.deallocate(seq)
        self._free_state(seq)
        self.stats["completed_request_count"] += 1
        self.completed_request_metrics.append(seq.lifecycle_metrics(now_ns))

    def abort(self, seq_id: int) -> bool:
        for q in (self.waiting, self.running):
            for seq in q:
                if seq.seq_id == seq_id:
                    q.remove(seq)
                    self._cancel_sequence_promotion(seq)
                    seq.num_scheduled_tokens = 0
                    self.stats["aborted_request_count"] += 1
                    self._retire(seq, SequenceStatus.ABORTED)
                    return True
        return False

    # ---------------------------------------------------------- policies
    def schedule(self) -> list[ScheduledBatch]:
        if self.scheduling_policy == "slo_aware":
            return self._schedule_slo_aware()
        if self.scheduling_policy == "prefill_first":
            prefill = self._schedule_prefill(self.max_num_batched_tokens, self.max_num_seqs)
            if prefill:
                return [ScheduledBatch(prefill, True)]
            decode = self._schedule_decode(self.max_num_seqs)
            assert decode, "scheduler made no progress"
            return [ScheduledBatch(decode, False)]
        decode = self._schedule_decode(self.max_num_seqs)
        prefill = self._schedule_prefill(self.max_num_batched_tokens - len(decode), self.max_num_seqs - len(decode))
        batches = ([ScheduledBatch(decode, False)] if decode else []) + ([ScheduledBatch(prefill, True)] if prefill else [])
        assert batches, "scheduler made no progress"
        return batches

    def _schedule_slo_aware(self, now_ns: int | None = None) -> list[ScheduledBatch]:
        now = now_ns if now_ns is not None else perf_counter_ns()
        if not self.running:
            wu = self._waiting_urgency(now)
            prefill = self._schedule_prefill(self.max_num_batched_tokens, self.max_num_seqs)
            assert prefill, "scheduler made no progress"
            self.stats["slo_prefill_priority_steps"] += 1
            self._record_slo_decision("prefill_only", 0.0, wu, self.max_num_batched_tokens)
            return [ScheduledBatch(prefill, True)]
        if not self.waiting:
            decode = self._schedule_decode(self.max_num_seqs)
            assert decode, "scheduler made no progress"
            self.stats["slo_decode_priority_steps"] += 1
            self._record_slo_decision("decode_only", self._decode_urgency(now), 0.0, 0)
            return [ScheduledBatch(decode, False)]
        du, wu = self._decode_urgency(now), self._waiting_urgency(now)
        decode = self._schedule_decode(self.max_num_seqs)
        rem_tok = self.max_num_batched_tokens - len(decode)
        rem_seq = self.max_num_seqs - len(decode)
        prefill: list[Sequence] = []
        budget = 0
        defer = self._kv_pressure() >= self.slo_kv_pressure_threshold and wu < self.slo_prefill_priority_threshold
        if len(self.waiting) >= self.slo_queue_pressure_threshold and rem_tok > 0 and rem_seq > 0:
            budget = rem_tok
            prefill = self._schedule_prefill(budget, rem_seq)
            self.stats["slo_dynamic_prefill_tokens"] += sum(s.num_scheduled_tokens for s in prefill)
            self.stats["slo_throughput_priority_steps"] += 1
        elif defer:
            self.stats["slo_admission_deferred_steps"] += 1
        elif rem_tok > 0 and rem_seq > 0:
            budget = self._latency_bounded_prefill_budget(rem_tok, wu)
            if budget:
                prefill = self._schedule_prefill(budget, rem_seq)
                self.stats["slo_dynamic_prefill_tokens"] += sum(s.num_scheduled_tokens for s in prefill)
            else:
                self.stats["slo_admission_deferred_steps"] += 1
        self.stats["slo_decode_priority_steps"] += 1
        self._record_slo_decision("decode_first" if prefill else "decode_only", du, wu, budget)
        batches = ([ScheduledBatch(decode, False)] if decode else []) + ([ScheduledBatch(prefill, True)] if prefill else [])
        assert batches, "scheduler made no progress"
        return batches

    def _latency_bounded_prefill_budget(self, remaining_tokens: int, waiting_urgency: float) -> int:
        """Tokens of prefill that fit in the decode step's TPOT slack (EWMA latency model)."""
        if self.prefill_ms_per_token_ewma is None or self.decode_step_ms_ewma is None:
            return remaining_tokens
        avail = max(self.target_tpot_ms - self.decode_step_ms_ewma - self.slo_latency_safety_margin_ms, 0.0)
        full = self.prefill_ms_per_token_ewma * self.max_num_batched_tokens
        if full <= avail or self.prefill_base_ms is None:
            return remaining_tokens
        if avail <= self.prefill_base_ms:
            self.stats["slo_infeasible_budget_steps"] += 1
            return remaining_tokens if waiting_urgency >= self.slo_prefill_priority_threshold else 0
        incr = full - self.prefill_base_ms
        budget = 0 if incr <= 0 else int((avail - self.prefill_base_ms) / (incr / self.max_num_batched_tokens))
        return min(remaining_tokens, max(min(self.slo_min_prefill_tokens, remaining_tokens), budget))

    def observe_batch(self, is_prefill: bool, num_tokens: int, duration_ms: float) -> None:
        if is_prefill:
            self.stats["prefill_observed_tokens"] += num_tokens
            self.stats["prefill_observed_ms"] += duration_ms
            self.prefill_base_ms = duration_ms if self.prefill_base_ms is None else min(self.prefill_base_ms, duration_ms)
            if num_tokens >= self.max_num_batched_tokens * 0.8:
                obs = duration_ms / num_tokens
                if self.prefill_ms_per_token_ewma is not None and obs > 2 * self.prefill_ms_per_token_ewma:
                    self.stats["slo_rejected_latency_observations"] += 1
                else:
                    self.prefill_ms_per_token_ewma = self._ewma(self.prefill_ms_per_token_ewma, obs)
        else:
            self.mtp_phase_profiler.record_cpu(
                "mtp.engine_model_runner_wall" if self.num_speculative_tokens else "target_only.engine_model_runner_wall",
                duration_ms)
            self.stats["decode_observed_tokens"] += num_tokens
            self.stats["decode_observed_ms"] += duration_ms
            self.decode_step_ms_ewma = self._ewma(self.decode_step_ms_ewma, duration_ms)

    def _ewma(self, prev: float | None, obs: float) -> float:
        return obs if prev is None else self.ewma_alpha * obs + (1 - self.ewma_alpha) * prev

    def _waiting_urgency(self, now_ns: int) -> float:
        if not self.waiting:
            return 0.0
        oldest = min(s.arrival_time_ns for s in self.waiting)
        return max((now_ns - oldest) / 1e6 / self.target_ttft_ms, 0.0)

    def _decode_urgency(self, now_ns: int) -> float:
        u = [max((now_ns - (s.last_token_time_ns or s.last_scheduled_time_ns or s.arrival_time_ns)) / 1e6
                 / self.target_tpot_ms, 0.0) for s in self.running]
        return max(u, default=0.0)

    def _kv_pressure(self) -> float:
        n = len(self.block_manager.blocks)
        return len(self.block_manager.used_block_ids) / n if n else 1.0

    def _record_slo_decision(self, decision: str, du: float, wu: float, budget: int) -> None:
        self.last_slo_decision = {"decision": decision, "decode_urgency": du, "waiting_urgency": wu,
                                  "prefill_budget": budget, "kv_pressure": self._kv_pressure()}

    # ---------------------------------------------------- prefix probes
    def _probe_prefix_details(self, seq: Sequence, *, durable_only: bool = False) -> PrefixRecoveryProbe:
        """Side-effect-free recoverability estimate for scoring."""
        if seq.block_table and not durable_only:
            t = seq.num_cached_tokens
            return PrefixRecoveryProbe(t, t, t, t, True)
        state_ok = self._state_available(seq)
        if self.enable_hybrid_prefix_cache:
            p = self.hybrid_prefix_coordinator.probe(seq)
            feasible = self.full_attention_prefix_manager.can_allocate(seq, p.candidate) and state_ok
            joint = p.boundary_tokens
            scoring = p.kv_candidate_tokens if self.score_source == "kv_only" else joint
            return PrefixRecoveryProbe(p.kv_candidate_tokens, joint, joint, scoring, feasible)
        if not self.enable_prefix_cache:
            return PrefixRecoveryProbe(0, 0, 0, 0, len(self.block_manager.free_block_ids) >= seq.num_blocks and state_ok)
        cands = self.block_manager.find_prefix_candidates(seq)
        cand = cands[0] if cands else None
        reuse = cand.boundary_tokens if cand else 0
        return PrefixRecoveryProbe(reuse, reuse, reuse, reuse,
                                   self.block_manager.can_allocate_candidate(seq, cand) and state_ok)

    def _probe_prefix(self, seq: Sequence, *, durable_only: bool = False) -> tuple[int, int, bool]:
        p = self._probe_prefix_details(seq, durable_only=durable_only)
        return p.scoring_reusable_tokens, p.kv_candidate_tokens, p.feasible

    def _admission_probe(self, seq: Sequence, index: int, now_ns: int) -> AdmissionProbe:
        p = self._probe_prefix_details(seq)
        uncached = max(seq.num_tokens - p.scoring_reusable_tokens, 0)
        age = max((now_ns - seq.arrival_time_ns) / 1e6, 0.0)
        score = uncached - (self.aging_per_ms * age if self.enable_aging else 0.0)
        return AdmissionProbe(seq, index, p.scoring_reusable_tokens, p.kv_candidate_tokens, p.gdn_checkpoint_tokens,
                              p.joint_recoverable_tokens, uncached, age, score, p.feasible)

    def _trace(self, event: dict, started_ns: int, sink: deque) -> None:
        if self.enable_scheduler_profiling:
            us = (perf_counter_ns() - started_ns) / 1e3
            sink.append(us)
            self.decision_events.append(event)

    def _select_waiting_candidate(self, now_ns: int | None = None) -> Sequence:
        if not self.waiting:
            raise RuntimeError("cannot select from an empty waiting queue")
        self.stats["scheduler_admission_decisions"] += 1
        t0 = perf_counter_ns()
        head = self.waiting[0]
        if self.waiting_admission_policy == "fcfs":
            self._trace({"type": "admission", "reason": "fcfs", "selected_request_id": head.seq_id,
                         "queue_index": 0}, t0, self.admission_latency_us)
            return head
        if self.enable_sticky and (head.block_table or head.preemption_count):
            self.stats["hybrid_scheduler_sticky_recovery_triggers"] += 1
            self._trace({"type": "admission", "reason": "sticky_recovery", "selected_request_id": head.seq_id,
                         "queue_index": 0}, t0, self.admission_latency_us)
            return head
        now = now_ns if now_ns is not None else perf_counter_ns()
        tp = perf_counter_ns()
        probes = [self._admission_probe(s, i, now) for i, s in enumerate(list(self.waiting)[: self.window])]
        if self.enable_scheduler_profiling:
            self.probe_latency_us.append((perf_counter_ns() - tp) / 1e3)
        self.stats["hybrid_scheduler_candidates_probed"] += len(probes)
        self.stats["hybrid_scheduler_admission_decisions"] += 1
        self.max_observed_wait_ms = max(self.max_observed_wait_ms, max(p.age_ms for p in probes))
        feasible = [p for p in probes if p.feasible]
        if not feasible:
            chosen, reason = probes[0], "no_feasible_candidate"
        else:
            best = min(feasible, key=lambda p: (p.score, p.sequence.arrival_time_ns, p.sequence.seq_id))
            overdue = [p for p in feasible if p.age_ms >= self.max_wait_ms] if self.enable_aging else []
            if overdue:
                chosen = min(overdue, key=lambda p: (p.sequence.arrival_time_ns, p.sequence.seq_id))
                reason = "aging_deadline"
                if chosen.sequence is not best.sequence:
                    self.stats["hybrid_scheduler_aging_overrides"] += 1
            else:
                chosen, reason = best, "minimum_effective_prefill"
                h = probes[0]
                if (self.enable_hysteresis and chosen.queue_index and h.feasible
                        and h.uncached_tokens - chosen.uncached_tokens < self.min_saved_tokens):
                    chosen, reason = h, "benefit_below_hysteresis"
                    self.stats["hybrid_scheduler_hysteresis_rejections"] += 1
        for p in probes:
            if p.queue_index < chosen.queue_index:
                p.sequence.mark_bypassed()
                if p.age_ms >= self.max_wait_ms:
                    self.stats["hybrid_scheduler_starvation_count"] += 1
        s = chosen.sequence
        s.last_scheduler_score = chosen.score
        s.last_reusable_tokens = chosen.reusable_tokens
        s.last_kv_candidate_tokens = chosen.kv_candidate_tokens
        s.last_gdn_checkpoint_tokens = chosen.gdn_checkpoint_tokens
        s.last_joint_recoverable_tokens = chosen.joint_recoverable_tokens
        if chosen.queue_index:
            self.waiting.remove(s)
            self.waiting.appendleft(s)
            self.stats["hybrid_scheduler_reorders"] += 1
        st = self.stats
        st["hybrid_scheduler_estimated_saved_prefill_tokens"] += max(probes[0].uncached_tokens - chosen.uncached_tokens, 0)
        st["hybrid_scheduler_selected_reusable_tokens"] += chosen.reusable_tokens
        st["hybrid_scheduler_selected_kv_candidate_tokens"] += chosen.kv_candidate_tokens
        st["hybrid_scheduler_selected_gdn_checkpoint_tokens"] += chosen.gdn_checkpoint_tokens
        st["hybrid_scheduler_selected_joint_recoverable_tokens"] += chosen.joint_recoverable_tokens
        st["hybrid_scheduler_estimated_remaining_prefill_tokens"] += chosen.uncached_tokens
        st["hybrid_scheduler_selected_original_rank_total"] += chosen.queue_index
        st["hybrid_scheduler_selected_original_rank_max"] = max(st["hybrid_scheduler_selected_original_rank_max"],
                                                                chosen.queue_index)
        self.rank_histogram[chosen.queue_index] += 1
        self.last_hybrid_scheduler_decision = {
            "reason": reason, "selected_request_id": s.seq_id, "queue_index": chosen.queue_index,
            "reusable_tokens": chosen.reusable_tokens, "kv_candidate_tokens": chosen.kv_candidate_tokens,
            "gdn_checkpoint_tokens": chosen.gdn_checkpoint_tokens,
            "joint_recoverable_tokens": chosen.joint_recoverable_tokens, "uncached_tokens": chosen.uncached_tokens,
            "age_ms": chosen.age_ms, "score": chosen.score, "window": len(probes)}
        self._trace({"type": "admission", **self.last_hybrid_scheduler_decision}, t0, self.admission_latency_us)
        return s

    # ---------------------------------------------------------- preemption
    def _preemption_probe(self, seq: Sequence) -> PreemptionProbe:
        p = self._probe_prefix_details(seq, durable_only=True)
        reclaim = self.block_manager.reclaimable_blocks(seq)
        recompute = max(seq.num_cached_tokens - p.scoring_reusable_tokens, 0)
        cost = (recompute / reclaim + self.preemption_penalty * seq.preemption_count) if reclaim else float("inf")
        return PreemptionProbe(seq, seq.num_cached_tokens, len(seq.block_table), reclaim, p.scoring_reusable_tokens,
                               recompute, cost)

    def _select_preemption_victim(self, current: Sequence) -> PreemptionProbe:
        self.stats["scheduler_preemption_decisions"] += 1
        t0 = perf_counter_ns()
        lifo = self.running[-1] if self.running else current
        if self.preemption_policy == "lifo":
            probe = (self._preemption_probe(lifo) if self.enable_scheduler_profiling else
                     PreemptionProbe(lifo, lifo.num_cached_tokens, len(lifo.block_table), 0, 0, 0, 0.0))
            lifo.estimated_recompute_tokens_lost += probe.recompute_tokens
            self._trace({"type": "preemption", "policy": "lifo", "selected_request_id": lifo.seq_id},
                        t0, self.preemption_latency_us)
            return probe
        probes = [self._preemption_probe(s) for s in [*self.running, current]]
        chosen = min(probes, key=lambda p: (p.cost_per_block, -p.reclaimable_blocks, p.sequence.seq_id))
        base = next(p for p in probes if p.sequence is lifo)
        st = self.stats
        st["recompute_aware_preemptions"] += 1
        st["recompute_aware_reclaimed_blocks"] += chosen.reclaimable_blocks
        st["recompute_aware_estimated_recompute_tokens"] += chosen.recompute_tokens
        st["recompute_aware_avoided_recompute_tokens"] += max(base.recompute_tokens - chosen.recompute_tokens, 0)
        chosen.sequence.estimated_recompute_tokens_lost += chosen.recompute_tokens
        self._trace({"type": "preemption", "policy": "recompute_aware", "selected_request_id": chosen.sequence.seq_id,
                     "lifo_request_id": lifo.seq_id}, t0, self.preemption_latency_us)
        return chosen

    def preempt(self, seq: Sequence) -> None:
        self.stats["preemption_count"] += 1
        seq.mark_preempted()
        seq.status = SequenceStatus.WAITING
        seq.is_prefill = True
        self._cancel_sequence_promotion(seq)
        self.block_manager.deallocate(seq)
        self._free_state(seq)
        self.waiting.appendleft(seq)

    # ------------------------------------------------------------- prefill
    def _admit(self, seq: Sequence, plan, num_cached_blocks: int) -> None:
        """Take KV pages + state slot for ``seq``; restore prefix state; roll back on any failure."""
        if plan is None:
            self.block_manager.allocate(seq, num_cached_blocks)
            self._allocate_state(seq)
            joint = num_cached_blocks * self.block_size
            kv_tokens = joint
        else:
            page_copy = None
            try:
                page_copy = self.full_attention_prefix_manager.allocate(seq, plan.candidate)
                self._allocate_state(seq)
                if page_copy is not None:
                    self.state_controller.call("copy_prefix_kv", page_copy.source_block_id,
                                               page_copy.destination_block_id, page_copy.num_tokens)
                if plan.hit is not None:
                    self.state_controller.call("restore_prefix_checkpoint", seq, plan.hit.checkpoint_slot)
                self.hybrid_prefix_coordinator.commit(plan)
                pc = plan.promotion_candidate
                if pc is not None:
                    self.hybrid_prefix_promotions[seq.seq_id] = (
                        CheckpointBoundary(pc.boundary_tokens, "shared_junction"),
                        pc.boundary_tokens - plan.boundary_tokens, pc,
                        self.hybrid_prefix_coordinator.demand_observations(pc))
            except Exception:
                self.hybrid_prefix_coordinator.cancel_promotion(plan.promotion_candidate)
                if page_copy is not None:
                    self.block_manager.release_cow_source(page_copy)
                if seq.state_slot is not None:
                    self._free_state(seq)
                if seq.block_table:
                    self.block_manager.deallocate(seq)
                raise
            if page_copy is not None:
                self.block_manager.release_cow_source(page_copy)
            joint, kv_tokens = plan.boundary_tokens, plan.kv_candidate_tokens
        seq.last_kv_candidate_tokens = kv_tokens
        seq.last_gdn_checkpoint_tokens = joint
        seq.last_joint_recoverable_tokens = joint
        seq.prefix_tokens_reused += joint
        self.stats["prefix_tokens_reused_actual"] += joint
        self.stats["prefix_cache_hit_blocks"] += num_cached_blocks
        seq.prefix_cache_hit_blocks += num_cached_blocks

    def _schedule_prefill(self, token_budget: int, sequence_budget: int) -> list[Sequence]:
        out: list[Sequence] = []
        used = 0
        while self.waiting and len(out) < sequence_budget:
            remaining = token_budget - used
            if remaining <= 0:
                break
            seq = self._select_waiting_candidate()
            plan = None
            num_cached_blocks = 0
            if not seq.block_table:
                if self.enable_hybrid_prefix_cache:
                    self.stats["prefix_cache_queries"] += 1
                    self.stats["prefix_cache_eligible_blocks"] += max(seq.num_blocks - 1, 0)
                    plan = self.hybrid_prefix_coordinator.plan(seq)
                    if plan is None:
                        break
                    num_cached_blocks = plan.num_cached_blocks
                else:
                    if self.enable_prefix_cache:
                        self.stats["prefix_cache_queries"] += 1
                        self.stats["prefix_cache_eligible_blocks"] += max(seq.num_blocks - 1, 0)
                    num_cached_blocks = self.block_manager.can_allocate(seq, use_prefix_cache=self.enable_prefix_cache)
                    if num_cached_blocks == -1:
                        break
                if not self._state_available(seq):
                    break
                todo = seq.num_tokens - (plan.boundary_tokens if plan is not None else num_cached_blocks * self.block_size)
            else:
                todo = seq.num_tokens - seq.num_cached_tokens
            if remaining < todo:
                if out:
                    break
                if not self.enable_chunked_prefill:
                    remaining = todo
            if not seq.block_table:
                self._admit(seq, plan, num_cached_blocks)
            seq.num_scheduled_tokens = min(todo, remaining)
            if self.enable_hybrid_prefix_cache and not self.enable_hybrid_internal_checkpoints:
                start = seq.num_cached_tokens
                nxt = self._next_retained_boundary(seq, start)
                if nxt is not None and 0 < nxt.boundary_tokens - start < seq.num_scheduled_tokens:
                    seq.num_scheduled_tokens = nxt.boundary_tokens - start
            seq.mark_scheduled()
            seq.prefill_tokens_executed += seq.num_scheduled_tokens
            self.stats["prefill_tokens_scheduled_total"] += seq.num_scheduled_tokens
            if seq.num_scheduled_tokens < todo:
                self.stats["chunked_prefill_steps"] += 1
            used += seq.num_scheduled_tokens
            if seq.num_cached_tokens + seq.num_scheduled_tokens == seq.num_tokens:
                # the MTP head drafts right after the last prefill chunk: pages for its cache rows
                k = self.num_speculative_tokens
                if k and self.block_manager.can_reserve_append(seq, k):
                    self.block_manager.reserve_append(seq, k)
                seq.status = SequenceStatus.RUNNING
                self.waiting.popleft()
                self.running.append(seq)
            out.append(seq)
        return out

    # -------------------------------------------------------------- decode
    def _schedule_decode(self, sequence_budget: int) -> list[Sequence]:
        t0 = perf_counter_ns()
        out: list[Sequence] = []
        # a speculative round writes target KV at pending..pending+K and MTP KV up to pending+2K-1
        reserve = 2 * self.num_speculative_tokens
        while self.running and len(out) < sequence_budget:
            seq = self.running.popleft()

            def fits() -> bool:
                if self.num_speculative_tokens:
                    return self.block_manager.can_reserve_append(seq, reserve)
                return self.block_manager.can_append(seq)

            while not fits():
                victim = self._select_preemption_victim(seq).sequence
                if victim is seq:
                    self.preempt(seq)
                    break
                self.running.remove(victim)
                self.preempt(victim)
            else:
                seq.num_scheduled_tokens = 1
                seq.is_prefill = False
                if self.num_speculative_tokens:
                    self.block_manager.reserve_append(seq, reserve)
                else:
                    self.block_manager.may_append(seq)
                seq.mark_scheduled()
                out.append(seq)
        self.running.extendleft(reversed(out))
        self.mtp_phase_profiler.record_cpu("scheduler.decode_admission", (perf_counter_ns() - t0) / 1e6)
        return out

    # --------------------------------------------------- hybrid captures
    def _cancel_sequence_promotion(self, seq: Sequence) -> None:
        promo = self.hybrid_prefix_promotions.pop(seq.seq_id, None)
        if promo is not None and self.hybrid_prefix_coordinator is not None:
            self.hybrid_prefix_coordinator.cancel_promotion(promo[2])

    def _next_retained_boundary(self, seq: Sequence, start_tokens: int) -> CheckpointBoundary | None:
        retained = self.hybrid_prefix_retention_policy.next_retained_boundary(start_tokens, seq.num_tokens)
        promo = self.hybrid_prefix_promotions.get(seq.seq_id)
        if promo is None or promo[0].boundary_tokens <= start_tokens:
            return retained
        if retained is None or promo[0].boundary_tokens <= retained.boundary_tokens:
            return promo[0]
        return retained

    def _classify_capture_boundary(self, seq: Sequence, boundary: int) -> CheckpointBoundary | None:
        promo = self.hybrid_prefix_promotions.get(seq.seq_id)
        if promo is not None and promo[0].boundary_tokens == boundary:
            return promo[0]
        return self.hybrid_prefix_retention_policy.classify(boundary, seq.num_tokens)

    def _internal_retained_boundaries(self, seq: Sequence, end_tokens: int) -> list[CheckpointBoundary]:
        kept = self.hybrid_prefix_retention_policy.retained_boundaries(seq.num_cached_tokens, end_tokens, seq.num_tokens)
        promo = self.hybrid_prefix_promotions.get(seq.seq_id)
        if promo is not None and seq.num_cached_tokens < promo[0].boundary_tokens <= end_tokens:
            kept = sorted([b for b in kept if b.boundary_tokens != promo[0].boundary_tokens] + [promo[0]],
                          key=lambda b: b.boundary_tokens)
        cap = self.hybrid_prefix_cache.capacity
        if len(kept) > cap:
            if promo is None:
                kept = kept[-cap:]
            else:
                others = [b for b in kept if b.boundary_tokens != promo[0].boundary_tokens]
                kept = sorted(others[-max(cap - 1, 0):] + [promo[0]], key=lambda b: b.boundary_tokens)
        return kept

    def internal_prefix_boundaries(self, seqs: list[Sequence], is_prefill: bool) -> dict[int, tuple[int, ...]]:
        if not is_prefill or not self.enable_hybrid_internal_checkpoints:
            return {}
        out = {}
        for seq in seqs:
            end = seq.num_cached_tokens + seq.num_scheduled_tokens
            inner = tuple(b.boundary_tokens for b in self._internal_retained_boundaries(seq, end)
                          if b.boundary_tokens < end)
            if inner:
                out[seq.seq_id] = inner
        return out

    def prepare_prefix_captures(self, seqs: list[Sequence], is_prefill: bool):
        """Plan GDN checkpoint captures at retained boundaries reached by this chunk.

        Returns ``(pending, blocks_hashed)``; block hashing happens here (before
        the capture needs the boundary's prefix hash) when anything is eligible.
        """
        if not is_prefill or not self.enable_hybrid_prefix_cache:
            return [], False
        retained_by = {}
        for seq in seqs:
            end = seq.num_cached_tokens + seq.num_scheduled_tokens
            if self.enable_hybrid_internal_checkpoints:
                kept = self._internal_retained_boundaries(seq, end)
            else:
                b = self._classify_capture_boundary(seq, end)
                kept = [b] if b is not None else []
            if kept and seq.num_scheduled_tokens > 0:
                retained_by[seq.seq_id] = (seq, kept)
        if not retained_by:
            return [], False
        for seq in seqs:
            self.block_manager.hash_blocks(seq)
        pending = []
        for seq, kept in retained_by.values():
            end = seq.num_cached_tokens + seq.num_scheduled_tokens
            for b in kept:
                meta = self.full_attention_prefix_manager.metadata_at_boundary(seq, b.boundary_tokens)
                promo = self.hybrid_prefix_promotions.get(seq.seq_id)
                junction = b.reason == "shared_junction" and promo is not None
                cap = PendingHybridPrefixCapture(
                    prefix_hash=meta.prefix_hash, boundary_tokens=b.boundary_tokens, tail_block_id=meta.tail_block_id,
                    state_slot=seq.state_slot, reason=b.reason, internal_state=b.boundary_tokens < end,
                    sequence_id=seq.seq_id, replay_saved_tokens=promo[1] if junction else b.boundary_tokens,
                    demand_count=promo[3] if junction else 0)
                if self.hybrid_prefix_coordinator.contains(meta.prefix_hash, b.boundary_tokens):
                    self._resolve_pending_promotion(cap, published=False)
                    continue
                pending.append(cap)
        return pending, True

    def reserve_prefix_capture(self, pending: PendingHybridPrefixCapture) -> bool:
        if self.hybrid_prefix_coordinator.contains(pending.prefix_hash, pending.boundary_tokens):
            self._resolve_pending_promotion(pending, published=False)
            return False
        for entry in self.hybrid_prefix_coordinator.reserve_capture(pending):
            self.state_controller.call("evict_prefix_checkpoint", entry.checkpoint_slot)
        return True

    def publish_prefix_capture(self, pending: PendingHybridPrefixCapture, checkpoint_slot: int) -> None:
        self.hybrid_prefix_coordinator.publish(pending, checkpoint_slot)
        if pending.reason == "shared_junction":
            self.hybrid_prefix_promotions.pop(pending.sequence_id, None)

    def cancel_prefix_capture(self, pending: PendingHybridPrefixCapture) -> None:
        self._resolve_pending_promotion(pending, published=False)

    def _resolve_pending_promotion(self, pending: PendingHybridPrefixCapture, *, published: bool) -> None:
        if pending.reason != "shared_junction":
            return
        self.hybrid_prefix_coordinator.resolve_capture(pending, published=published)
        self.hybrid_prefix_promotions.pop(pending.sequence_id, None)

    # --------------------------------------------------------- commit
    def _finished(self, seq: Sequence, token_id: int) -> bool:
        return (not seq.ignore_eos and token_id == self.eos) or seq.num_completion_tokens >= seq.max_tokens

    def postprocess(self, seqs: list[Sequence], token_ids: list[int], is_prefill: bool, *,
                    blocks_already_hashed: bool = False) -> None:
        t0 = perf_counter_ns()
        for seq, tok in zip(seqs, token_ids):
            if self.enable_prefix_cache and not blocks_already_hashed:
                self.block_manager.hash_blocks(seq)
            seq.num_cached_tokens += seq.num_scheduled_tokens
            seq.num_scheduled_tokens = 0
            if is_prefill and seq.num_cached_tokens < seq.num_tokens:
                continue
            seq.append_token(tok, t0)
            if self._finished(seq, tok):
                self.running.remove(seq)
                self._retire(seq, SequenceStatus.FINISHED, t0)
        if not is_prefill:
            self.mtp_phase_profiler.record_cpu("target_only.scheduler_commit", (perf_counter_ns() - t0) / 1e6)

    def postprocess_speculative(self, seqs: list[Sequence], output_token_ids: list[list[int]]) -> None:
        """Commit speculative outputs; the last emitted token stays pending (not yet run)."""
        t0 = perf_counter_ns()
        for seq, toks in zip(seqs, output_token_ids):
            if not toks:
                raise ValueError("speculative decode must emit at least one token")
            seq.num_cached_tokens += len(toks)
            seq.num_scheduled_tokens = 0
            for tok in toks:
                if seq.num_completion_tokens >= seq.max_tokens:
                    break
                seq.append_token(tok, t0)
                if not seq.ignore_eos and tok == self.eos:
                    break
            done = seq.num_completion_tokens >= seq.max_tokens or (
                not seq.ignore_eos and seq.completion_token_ids and seq.completion_token_ids[-1] == self.eos)
            if done:
                self.running.remove(seq)
                self._retire(seq, SequenceStatus.FINISHED, t0)
            else:
                seq.num_cached_tokens = len(seq) - 1
                self.block_manager.trim_to_sequence_length(seq)
        self.mtp_phase_profiler.record_cpu("scheduler.speculative_commit", (perf_counter_ns() - t0) / 1e6)
