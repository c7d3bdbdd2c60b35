"""Continuous-batching scheduler built from interchangeable policy objects.

Behavioural parity with ``nanovllm/engine/scheduler.py`` (batch composition
``:640-776``, admission ``:960-1142``, preemption ``:1144-1282``, chunked
prefill ``:1284-1419``, decode and speculative reservation ``:1421-1461``,
hybrid prefix captures ``:1527-1694``, commit ``:1696-1781``): the policy names,
their decisions and the metric keys are the same, so configurations,
dashboards and the reference's test scenarios carry over.

Structure (this module's own):
* One queue model: ``waiting`` and ``running`` deques of ``Sequence``.
* ``BatchPolicy`` (``PrefillFirst`` / ``DecodeFirst`` / ``SloAware``) decides
  what a step contains; ``AdmissionPolicy`` (``Fcfs`` / ``HybridStateAware``)
  decides which waiting request is admitted next; ``PreemptionPolicy``
  (``Lifo`` / ``RecomputeAware``) picks who gives up its pages when decode runs
  out of KV memory.  Each is a small object with one method, chosen once from the
  config.
* ``LatencyModel`` holds the EWMA step-latency estimates that the SLO policy
  turns into a prefill budget.
* ``PrefixOracle`` answers "how much of this request can be restored, and does
  it fit?" from the block manager (stateless models) or the hybrid prefix
  planner (KV + GDN checkpoints); admission and preemption both ask it.
* ``SchedulerTelemetry`` collects counters, latency samples and a bounded
  decision trace; ``get_metrics`` flattens it.
"""

from __future__ import annotations

from collections import Counter, deque
from dataclasses import dataclass
from time import perf_counter_ns

from inference_systems_b200.engine.block_manager import BlockManager, PrefixKVCandidate
from inference_systems_b200.engine.hybrid_prefix_cache import (
    AdmissionPlan,
    CaptureTicket,
    CheckpointIndex,
    HybridPrefixPlanner,
    RetainedBoundary,
    make_retention,
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


def latency_summary(values) -> dict:
    """count / mean / p50 / p95 / p99 / max of microsecond samples (nearest-rank percentiles)."""
    if not values:
        return {"count": 0, "mean_us": 0.0, "p50_us": 0.0, "p95_us": 0.0, "p99_us": 0.0, "max_us": 0.0}
    s = sorted(values)
    n = len(s)

    def rank(q: float) -> float:
        return s[min(max(-(-int(q * n * 1_000_000) // 1_000_000) - 1, 0), n - 1)]

    return {"count": n, "mean_us": sum(s) / n, "p50_us": rank(0.5), "p95_us": rank(0.95), "p99_us": rank(0.99),
            "max_us": s[-1]}


# ============================================================================ recoverability


@dataclass(frozen=True, slots=True)
class Recoverability:
    """How much of a request's prefix can be skipped, by source, and whether it can start now."""

    kv_tokens: int        # longest reusable KV prefix
    gdn_tokens: int       # longest boundary with a GDN checkpoint that matches it
    joint_tokens: int     # what admission would actually restore
    score_tokens: int     # what scheduling decisions count as reusable
    feasible: bool        # pages (and a state slot) are available


class PrefixOracle:
    """Read-only questions about prefix reuse, answered from the KV index (stateless models) or the
    hybrid planner (KV and GDN checkpoints must meet at one boundary)."""

    def __init__(self, sched: "Scheduler"):
        self.s = sched

    def assess(self, seq: Sequence, *, durable_only: bool = False) -> Recoverability:
        s = self.s
        if seq.block_table and not durable_only:
            t = seq.num_cached_tokens  # already admitted: what it holds is what it keeps
            return Recoverability(t, t, t, t, True)
        state_ok = s.state_available(seq)
        bm = s.block_manager
        if s.prefix_planner is not None:
            plan = s.prefix_planner.probe(seq)
            joint = plan.boundary_tokens
            score = plan.kv_candidate_tokens if s.score_source == "kv_only" else joint
            return Recoverability(plan.kv_candidate_tokens, joint, joint, score,
                                  bm.can_allocate_candidate(seq, plan.candidate) and state_ok)
        if not s.enable_prefix_cache:
            return Recoverability(0, 0, 0, 0, bm.num_free_blocks >= seq.num_blocks and state_ok)
        cands = bm.find_prefix_candidates(seq)
        best = cands[0] if cands else None
        t = best.boundary_tokens if best is not None else 0
        return Recoverability(t, t, t, t, bm.can_allocate_candidate(seq, best) and state_ok)


# ================================================================================ admission


@dataclass(frozen=True, slots=True)
class AdmissionCandidate:
    seq: Sequence
    position: int          # index in the waiting queue
    recover: Recoverability
    uncached_tokens: int
    age_ms: float
    score: float           # lower is better: uncached work minus aging credit


class FcfsAdmission:
    name = "fcfs"

    def select(self, sched: "Scheduler", now_ns: int) -> Sequence:
        head = sched.waiting[0]
        sched.telemetry.trace("admission", {"reason": "fcfs", "selected_request_id": head.seq_id, "queue_index": 0})
        return head


class HybridStateAwareAdmission:
    """Among the first ``window`` waiting requests, admit the one with the least prefill left after
    prefix restore; requests past ``max_wait_ms`` go first (aging), a small win does not overtake a
    feasible queue head (hysteresis), and a head that already holds pages or was preempted is
    resumed first (sticky recovery)."""

    name = "hybrid_state_aware"

    def select(self, sched: "Scheduler", now_ns: int) -> Sequence:
        cfg, tel = sched.policy_cfg, sched.telemetry
        head = sched.waiting[0]
        if cfg.sticky and (head.block_table or head.preemption_count):
            tel.count("hybrid_scheduler_sticky_recovery_triggers")
            tel.trace("admission", {"reason": "sticky_recovery", "selected_request_id": head.seq_id, "queue_index": 0})
            return head
        t_probe = perf_counter_ns()
        cands = []
        for i, seq in enumerate(list(sched.waiting)[: cfg.window]):
            rec = sched.oracle.assess(seq)
            uncached = max(seq.num_tokens - rec.score_tokens, 0)
            age = max((now_ns - seq.arrival_time_ns) / 1e6, 0.0)
            score = uncached - (cfg.aging_per_ms * age if cfg.aging else 0.0)
            cands.append(AdmissionCandidate(seq, i, rec, uncached, age, score))
        tel.sample_probe(t_probe)
        tel.count("hybrid_scheduler_candidates_probed", len(cands))
        tel.count("hybrid_scheduler_admission_decisions")
        tel.max_observed_wait_ms = max(tel.max_observed_wait_ms, max(c.age_ms for c in cands))
        chosen, reason = self._decide(cands, cfg, tel)
        for c in cands:
            if c.position < chosen.position:
                c.seq.mark_bypassed()
                if c.age_ms >= cfg.max_wait_ms:
                    tel.count("hybrid_scheduler_starvation_count")
        led, rec = chosen.seq.ledger, chosen.recover
        led.last_scheduler_score = chosen.score
        led.last_reusable_tokens = rec.score_tokens
        led.last_kv_candidate_tokens = rec.kv_tokens
        led.last_gdn_checkpoint_tokens = rec.gdn_tokens
        led.last_joint_recoverable_tokens = rec.joint_tokens
        if chosen.position:
            sched.waiting.remove(chosen.seq)
            sched.waiting.appendleft(chosen.seq)
            tel.count("hybrid_scheduler_reorders")
        tel.note_admission(cands[0], chosen)
        tel.last_hybrid_decision = {
            "reason": reason, "selected_request_id": chosen.seq.seq_id, "queue_index": chosen.position,
            "reusable_tokens": rec.score_tokens, "kv_candidate_tokens": rec.kv_tokens,
            "gdn_checkpoint_tokens": rec.gdn_tokens, "joint_recoverable_tokens": rec.joint_tokens,
            "uncached_tokens": chosen.uncached_tokens, "age_ms": chosen.age_ms, "score": chosen.score,
            "window": len(cands)}
        tel.trace("admission", tel.last_hybrid_decision)
        return chosen.seq

    @staticmethod
    def _decide(cands: list[AdmissionCandidate], cfg, tel) -> tuple[AdmissionCandidate, str]:
        feasible = [c for c in cands if c.recover.feasible]
        if not feasible:
            return cands[0], "no_feasible_candidate"
        best = min(feasible, key=lambda c: (c.score, c.seq.arrival_time_ns, c.seq.seq_id))
        if cfg.aging:
            overdue = [c for c in feasible if c.age_ms >= cfg.max_wait_ms]
            if overdue:
                oldest = min(overdue, key=lambda c: (c.seq.arrival_time_ns, c.seq.seq_id))
                if oldest.seq is not best.seq:
                    tel.count("hybrid_scheduler_aging_overrides")
                return oldest, "aging_deadline"
        head = cands[0]
        if (cfg.hysteresis and best.position and head.recover.feasible
                and head.uncached_tokens - best.uncached_tokens < cfg.min_saved_tokens):
            tel.count("hybrid_scheduler_hysteresis_rejections")
            return head, "benefit_below_hysteresis"
        return best, "minimum_effective_prefill"


# =============================================================================== preemption


@dataclass(frozen=True, slots=True)
class VictimCandidate:
    seq: Sequence
    reclaimable_blocks: int
    recompute_tokens: int
    cost_per_block: float


def _victim_candidate(sched: "Scheduler", seq: Sequence) -> VictimCandidate:
    rec = sched.oracle.assess(seq, durable_only=True)
    reclaim = sched.block_manager.reclaimable_blocks(seq)
    recompute = max(seq.num_cached_tokens - rec.score_tokens, 0)
    cost = (recompute / reclaim + sched.policy_cfg.preemption_penalty * seq.preemption_count
            if reclaim else float("inf"))
    return VictimCandidate(seq, reclaim, recompute, cost)


class LifoPreemption:
    """The most recently admitted running request gives way (the current one when none is left)."""

    name = "lifo"

    def victim(self, sched: "Scheduler", current: Sequence) -> Sequence:
        v = sched.running[-1] if sched.running else current
        if sched.telemetry.profiling:
            cand = _victim_candidate(sched, v)
            v.ledger.estimated_recompute_tokens_lost += cand.recompute_tokens
        else:
            cand = VictimCandidate(v, 0, 0, 0.0)
        sched.telemetry.note_victim(cand, "scheduler")
        sched.telemetry.trace("preemption", {"policy": "lifo", "selected_request_id": v.seq_id})
        return v


class RecomputeAwarePreemption:
    """The request whose preemption costs the least recompute per freed page gives way; each earlier
    preemption of a request adds a fixed penalty, so the same request is not picked every time."""

    name = "recompute_aware"

    def victim(self, sched: "Scheduler", current: Sequence) -> Sequence:
        cands = [_victim_candidate(sched, s) for s in [*sched.running, current]]
        chosen = min(cands, key=lambda c: (c.cost_per_block, -c.reclaimable_blocks, c.seq.seq_id))
        lifo_seq = sched.running[-1] if sched.running else current
        lifo = next(c for c in cands if c.seq is lifo_seq)
        tel = sched.telemetry
        tel.count("recompute_aware_preemptions")
        tel.count("recompute_aware_reclaimed_blocks", chosen.reclaimable_blocks)
        tel.count("recompute_aware_estimated_recompute_tokens", chosen.recompute_tokens)
        tel.count("recompute_aware_avoided_recompute_tokens", max(lifo.recompute_tokens - chosen.recompute_tokens, 0))
        chosen.seq.ledger.estimated_recompute_tokens_lost += chosen.recompute_tokens
        tel.note_victim(chosen, "scheduler")
        tel.note_victim(chosen, "recompute_aware")
        tel.trace("preemption", {"policy": "recompute_aware", "selected_request_id": chosen.seq.seq_id,
                                 "lifo_request_id": lifo_seq.seq_id})
        return chosen.seq


# ============================================================================ batch policies


class LatencyModel:
    """EWMA estimates of prefill cost per token (from near-full chunks), the cheapest prefill step
    seen, and the decode step time."""

    def __init__(self, alpha: float, max_batched_tokens: int):
        self.alpha, self.chunk = alpha, max_batched_tokens
        self.prefill_ms_per_token: float | None = None
        self.prefill_base_ms: float | None = None
        self.decode_step_ms: float | None = None

    def _blend(self, prev: float | None, x: float) -> float:
        return x if prev is None else self.alpha * x + (1.0 - self.alpha) * prev

    def observe_prefill(self, tokens: int, ms: float) -> bool:
        """Returns False when an outlier observation was rejected."""
        self.prefill_base_ms = ms if self.prefill_base_ms is None else min(self.prefill_base_ms, ms)
        if tokens < 0.8 * self.chunk:
            return True
        per = ms / tokens
        if self.prefill_ms_per_token is not None and per > 2.0 * self.prefill_ms_per_token:
            return False
        self.prefill_ms_per_token = self._blend(self.prefill_ms_per_token, per)
        return True

    def observe_decode(self, ms: float) -> None:
        self.decode_step_ms = self._blend(self.decode_step_ms, ms)


class PrefillFirst:
    name = "prefill_first"

    def compose(self, sched: "Scheduler", now_ns: int) -> list[ScheduledBatch]:
        prefill = sched.schedule_prefill(sched.max_num_batched_tokens, sched.max_num_seqs)
        if prefill:
            return [ScheduledBatch(prefill, True)]
        decode = sched.schedule_decode(sched.max_num_seqs)
        return [ScheduledBatch(decode, False)] if decode else []


class DecodeFirst:
    name = "decode_first"

    def compose(self, sched: "Scheduler", now_ns: int) -> list[ScheduledBatch]:
        decode = sched.schedule_decode(sched.max_num_seqs)
        prefill = sched.schedule_prefill(sched.max_num_batched_tokens - len(decode), sched.max_num_seqs - len(decode))
        return sched.batches(decode, prefill)


class SloAware:
    """Decode first; the prefill share of a step is sized so the step stays within the TPOT target
    (latency model), deferred under KV pressure unless the queue is urgent, and widened to the full
    budget when enough requests wait."""

    name = "slo_aware"

    def compose(self, sched: "Scheduler", now_ns: int) -> list[ScheduledBatch]:
        now = now_ns
        c, tel = sched.slo, sched.telemetry
        if not sched.running:
            wu = sched.waiting_urgency(now)
            prefill = sched.schedule_prefill(sched.max_num_batched_tokens, sched.max_num_seqs)
            tel.count("slo_prefill_priority_steps")
            tel.slo_decision("prefill_only", 0.0, wu, sched.max_num_batched_tokens, sched.kv_pressure())
            return sched.batches([], prefill)
        if not sched.waiting:
            du = sched.decode_urgency(now)
            decode = sched.schedule_decode(sched.max_num_seqs)
            tel.count("slo_decode_priority_steps")
            tel.slo_decision("decode_only", du, 0.0, 0, sched.kv_pressure())
            return sched.batches(decode, [])
        du, wu = sched.decode_urgency(now), sched.waiting_urgency(now)
        decode = sched.schedule_decode(sched.max_num_seqs)
        tokens_left = sched.max_num_batched_tokens - len(decode)
        seqs_left = sched.max_num_seqs - len(decode)
        room = tokens_left > 0 and seqs_left > 0
        budget, prefill = 0, []
        if len(sched.waiting) >= c["queue_pressure"] and room:
            budget = tokens_left
            prefill = sched.schedule_prefill(budget, seqs_left)
            tel.count("slo_dynamic_prefill_tokens", sum(s.num_scheduled_tokens for s in prefill))
            tel.count("slo_throughput_priority_steps")
        elif sched.kv_pressure() >= c["kv_pressure"] and wu < c["priority"]:
            tel.count("slo_admission_deferred_steps")
        elif room:
            budget = self.prefill_budget(sched, tokens_left, wu)
            if budget:
                prefill = sched.schedule_prefill(budget, seqs_left)
                tel.count("slo_dynamic_prefill_tokens", sum(s.num_scheduled_tokens for s in prefill))
            else:
                tel.count("slo_admission_deferred_steps")
        tel.count("slo_decode_priority_steps")
        tel.slo_decision("decode_first" if prefill else "decode_only", du, wu, budget, sched.kv_pressure())
        return sched.batches(decode, prefill)

    @staticmethod
    def prefill_budget(sched: "Scheduler", tokens_left: int, waiting_urgency: float) -> int:
        """Prefill tokens that fit in the TPOT slack next to the decode step (latency model)."""
        lat, c = sched.latency, sched.slo
        if lat.prefill_ms_per_token is None or lat.decode_step_ms is None:
            return tokens_left
        slack = max(c["target_tpot_ms"] - lat.decode_step_ms - c["margin_ms"], 0.0)
        full_chunk_ms = lat.prefill_ms_per_token * sched.max_num_batched_tokens
        if full_chunk_ms <= slack or lat.prefill_base_ms is None:
            return tokens_left
        if slack <= lat.prefill_base_ms:
            sched.telemetry.count("slo_infeasible_budget_steps")
            return tokens_left if waiting_urgency >= c["priority"] else 0
        per_token = (full_chunk_ms - lat.prefill_base_ms) / sched.max_num_batched_tokens
        fit = int((slack - lat.prefill_base_ms) / per_token) if per_token > 0 else 0
        return min(tokens_left, max(min(c["min_tokens"], tokens_left), fit))


# ================================================================================ telemetry


class SchedulerTelemetry:
    def __init__(self, profiling: bool, history: int):
        self.profiling = profiling
        self.admission_us: deque[float] = deque(maxlen=history)
        self.probe_us: deque[float] = deque(maxlen=history)
        self.preemption_us: deque[float] = deque(maxlen=history)
        self.bookkeeping_us: deque[float] = deque(maxlen=history)
        self.events: deque[dict] = deque(maxlen=history)
        self.reset()

    def reset(self) -> None:
        for d in (self.admission_us, self.probe_us, self.preemption_us, self.bookkeeping_us, self.events):
            d.clear()
        self.counters: Counter = Counter()
        self.rank_histogram: Counter = Counter()
        self.max_observed_wait_ms = 0.0
        self.last_slo_decision: dict | None = None
        self.last_hybrid_decision: dict | None = None
        self._t0 = 0

    def count(self, name: str, by: int = 1) -> None:
        self.counters[name] += by

    def begin(self) -> None:
        self._t0 = perf_counter_ns()

    def sample_probe(self, t0: int) -> None:
        us = (perf_counter_ns() - t0) / 1e3
        self.counters["hybrid_scheduler_probe_ms"] += us / 1e3
        if self.profiling:
            self.probe_us.append(us)

    def trace(self, kind: str, event: dict) -> None:
        """Close the decision opened by ``begin``: time it, and with profiling on keep a latency
        sample and a trace entry."""
        us = (perf_counter_ns() - self._t0) / 1e3
        self.counters["scheduler_admission_decision_ms" if kind == "admission" else
                      "scheduler_preemption_selection_ms"] += us / 1e3
        if kind == "preemption" and event.get("policy") == "recompute_aware":
            self.counters["recompute_aware_selection_ms"] += us / 1e3
        if not self.profiling:
            return
        (self.admission_us if kind == "admission" else self.preemption_us).append(us)
        self.events.append({"type": kind, **event})

    def note_victim(self, v: "VictimCandidate", prefix: str) -> None:
        t0 = perf_counter_ns()
        c = self.counters
        c[f"{prefix}_victim_computed_tokens"] += v.seq.num_cached_tokens
        c[f"{prefix}_victim_logical_blocks"] += len(v.seq.block_table)
        if prefix == "scheduler":
            c["scheduler_victim_reclaimable_blocks"] += v.reclaimable_blocks
            c["scheduler_victim_recompute_tokens"] += v.recompute_tokens
        if v.cost_per_block != float("inf"):
            c[f"{prefix}_cost_sum"] += v.cost_per_block
            c[f"{prefix}_cost_count"] += 1
        self._bookkeeping(t0)

    def _bookkeeping(self, t0: int) -> None:
        us = (perf_counter_ns() - t0) / 1e3
        self.counters["scheduler_metrics_bookkeeping_ms"] += us / 1e3
        if self.profiling:
            self.bookkeeping_us.append(us)

    def note_admission(self, head: AdmissionCandidate, chosen: AdmissionCandidate) -> None:
        t0 = perf_counter_ns()
        c, rec = self.counters, chosen.recover
        c["hybrid_scheduler_estimated_saved_prefill_tokens"] += max(head.uncached_tokens - chosen.uncached_tokens, 0)
        c["hybrid_scheduler_selected_reusable_tokens"] += rec.score_tokens
        c["hybrid_scheduler_selected_kv_candidate_tokens"] += rec.kv_tokens
        c["hybrid_scheduler_selected_gdn_checkpoint_tokens"] += rec.gdn_tokens
        c["hybrid_scheduler_selected_joint_recoverable_tokens"] += rec.joint_tokens
        c["hybrid_scheduler_estimated_remaining_prefill_tokens"] += chosen.uncached_tokens
        c["hybrid_scheduler_selected_original_rank_total"] += chosen.position
        c["hybrid_scheduler_selected_original_rank_max"] = max(c["hybrid_scheduler_selected_original_rank_max"],
                                                               chosen.position)
        self.rank_histogram[chosen.position] += 1
        self._bookkeeping(t0)

    def slo_decision(self, decision: str, du: float, wu: float, budget: int, kv_pressure: float) -> None:
        self.last_slo_decision = {"decision": decision, "decode_urgency": du, "waiting_urgency": wu,
                                  "prefill_budget": budget, "kv_pressure": kv_pressure}


class _PolicyConfig:
    """Knobs of the admission and preemption policies (from ``Config``)."""

    def __init__(self, c):
        g = lambda name, default: getattr(c, name, default)  # noqa: E731
        self.window = g("hybrid_scheduler_candidate_window", 8)
        self.aging_per_ms = g("hybrid_scheduler_aging_tokens_per_ms", 0.5)
        self.max_wait_ms = g("hybrid_scheduler_max_wait_ms", 200.0)
        self.min_saved_tokens = g("hybrid_scheduler_min_saved_tokens", 16)
        self.preemption_penalty = g("hybrid_scheduler_preemption_penalty", 128.0)
        self.aging = g("hybrid_scheduler_enable_aging", True)
        self.hysteresis = g("hybrid_scheduler_enable_hysteresis", True)
        self.sticky = g("hybrid_scheduler_enable_sticky_recovery", True)


_BATCH = {p.name: p for p in (PrefillFirst, DecodeFirst, SloAware)}
_ADMISSION = {p.name: p for p in (FcfsAdmission, HybridStateAwareAdmission)}
_PREEMPTION = {p.name: p for p in (LifoPreemption, RecomputeAwarePreemption)}


# ================================================================================ scheduler


class Scheduler:
    def __init__(self, config, state_manager=None, state_controller=None, prefix_checkpoint_pool=None):
        c = config
        g = lambda name, default: getattr(c, name, default)  # noqa: E731
        self.max_num_seqs = c.max_num_seqs
        self.max_num_batched_tokens = c.max_num_batched_tokens
        self.eos = c.eos
        self.block_size = c.kvcache_block_size
        self.scheduling_policy = c.scheduling_policy
        self.waiting_admission_policy = g("waiting_admission_policy", "fcfs")
        self.preemption_policy = g("preemption_policy", "lifo")
        for kind, table, name in (("scheduling", _BATCH, self.scheduling_policy),
                                  ("admission", _ADMISSION, self.waiting_admission_policy),
                                  ("preemption", _PREEMPTION, self.preemption_policy)):
            if name not in table:
                raise ValueError(f"unknown {kind} policy: {name}")
        self.batch_policy = _BATCH[self.scheduling_policy]()
        self.admission = _ADMISSION[self.waiting_admission_policy]()
        self.preemption = _PREEMPTION[self.preemption_policy]()
        self.policy_cfg = _PolicyConfig(c)
        self.score_source = g("hybrid_scheduler_score_source", "joint")
        self.slo = {"target_ttft_ms": g("scheduler_target_ttft_ms", 200.0),
                    "target_tpot_ms": g("scheduler_target_tpot_ms", 50.0),
                    "priority": g("slo_prefill_priority_threshold", 0.8),
                    "min_tokens": g("slo_min_prefill_tokens", 64),
                    "kv_pressure": g("slo_kv_pressure_threshold", 0.9),
                    "queue_pressure": g("slo_queue_pressure_threshold", 3),
                    "margin_ms": g("slo_latency_safety_margin_ms", 5.0)}
        self.latency = LatencyModel(g("scheduler_ewma_alpha", 0.2), self.max_num_batched_tokens)
        self.telemetry = SchedulerTelemetry(g("enable_scheduler_profiling", False),
                                            g("scheduler_decision_history_size", 4096))
        self.mtp_phase_profiler = PhaseProfiler(g("enable_mtp_phase_profiling", False))
        self.state_manager, self.state_controller = state_manager, state_controller
        self.num_speculative_tokens = g("num_speculative_tokens", 0)
        self.enable_chunked_prefill = g("enable_chunked_prefill", True)

        unit = g("prefix_match_unit", None) or self.block_size
        self.block_manager = BlockManager(c.num_kvcache_blocks, self.block_size, prefix_match_unit=unit)
        self.enable_hybrid_prefix_cache = bool(g("enable_hybrid_prefix_cache", False) and state_manager is not None)
        self.enable_hybrid_internal_checkpoints = bool(self.enable_hybrid_prefix_cache
                                                       and g("enable_hybrid_internal_checkpoints", False))
        self.prefix_planner: HybridPrefixPlanner | None = None
        self.retention = None
        if self.enable_hybrid_prefix_cache:
            if prefix_checkpoint_pool is None:
                raise ValueError("hybrid prefix cache requires a checkpoint pool")
            mode = g("hybrid_prefix_retention_policy", "periodic")
            interval = g("hybrid_prefix_checkpoint_interval_tokens", None) or (
                c.hybrid_prefix_checkpoint_interval_blocks * self.block_size)
            self.retention = make_retention(mode, unit, interval)
            index = CheckpointIndex(prefix_checkpoint_pool.capacity, g("hybrid_prefix_eviction_policy", "lru"))
            self.prefix_planner = HybridPrefixPlanner(
                self.block_manager, index, promote_shared_junctions=mode == "adaptive",
                promotion_min_sightings=g("hybrid_prefix_promotion_min_sightings", 2),
                demand_capacity=max(prefix_checkpoint_pool.capacity * 16, 64))
        # A KV hit alone is not a restart point for a model with recurrent state: plain prefix
        # caching is only on for stateless models (or together with GDN checkpoints).
        self.enable_prefix_cache = g("enable_prefix_cache", True) and (
            state_manager is None or self.enable_hybrid_prefix_cache)
        self.oracle = PrefixOracle(self)
        # time source of policy decisions (ages, urgencies); tests substitute a fixed clock
        self.clock = perf_counter_ns
        self.waiting: deque[Sequence] = deque()
        self.running: deque[Sequence] = deque()
        self.completed_request_metrics: deque[dict] = deque(maxlen=g("request_metrics_history_size", 1024))
        self.reset_metrics()

    # ------------------------------------------------------------- state slots
    def state_available(self, seq: Sequence) -> bool:
        return self.state_manager is None or seq.state_slot is not None or self.state_manager.can_allocate

    def _take_state(self, seq: Sequence) -> None:
        if self.state_manager is None:
            return
        if self.state_controller is not None:
            self.state_controller.call("allocate_state_slot", seq)
        else:
            self.state_manager.allocate(seq)

    def _release_state(self, seq: Sequence) -> None:
        if self.state_manager is None or seq.state_slot is None:
            return
        if self.state_controller is not None:
            self.state_controller.call("free_state_slot", seq)
        else:
            self.state_manager.free(seq)

    # ----------------------------------------------------------------- queues
    def is_finished(self) -> bool:
        return not self.waiting and not self.running

    def add(self, seq: Sequence) -> None:
        self.waiting.append(seq)

    def _retire(self, seq: Sequence, status: SequenceStatus, now_ns: int | None = None) -> None:
        seq.status = status
        seq.mark_finished(now_ns)
        if seq.block_table:
            self.block_manager.deallocate(seq)
        self._release_state(seq)
        self.telemetry.count("completed_request_count")
        self.completed_request_metrics.append(seq.lifecycle_metrics(now_ns))

    def abort(self, seq_id: int) -> bool:
        for q in (self.waiting, self.running):
            seq = next((s for s in q if s.seq_id == seq_id), None)
            if seq is not None:
                q.remove(seq)
                if self.prefix_planner is not None:
                    self.prefix_planner.forget(seq)
                seq.num_scheduled_tokens = 0
                self.telemetry.count("aborted_request_count")
                self._retire(seq, SequenceStatus.ABORTED)
                return True
        return False

    def kv_pressure(self) -> float:
        bm = self.block_manager
        return bm.num_used_blocks / bm.num_blocks

    def waiting_urgency(self, now_ns: int) -> float:
        if not self.waiting:
            return 0.0
        oldest = min(s.arrival_time_ns for s in self.waiting)
        return max((now_ns - oldest) / 1e6 / self.slo["target_ttft_ms"], 0.0)

    def decode_urgency(self, now_ns: int) -> float:
        def since(s: Sequence) -> int:
            t = s.timeline
            return t.last_token_ns or t.last_scheduled_ns or t.arrival_ns
        return max(((now_ns - since(s)) / 1e6 / self.slo["target_tpot_ms"] for s in self.running), default=0.0)

    @staticmethod
    def batches(decode: list[Sequence], prefill: list[Sequence]) -> list[ScheduledBatch]:
        out = [ScheduledBatch(decode, False)] if decode else []
        if prefill:
            out.append(ScheduledBatch(prefill, True))
        return out

    # -------------------------------------------------------------- schedule
    def schedule(self, now_ns: int | None = None) -> list[ScheduledBatch]:
        """The next step's batches (decode and/or prefill), by the configured batch policy."""
        batches = self.batch_policy.compose(self, now_ns if now_ns is not None else self.clock())
        if not batches:
            raise RuntimeError("scheduler made no progress")
        return batches

    def observe_batch(self, is_prefill: bool, num_tokens: int, duration_ms: float) -> None:
        tel = self.telemetry
        if is_prefill:
            tel.count("prefill_observed_tokens", num_tokens)
            tel.counters["prefill_observed_ms"] += duration_ms
            if not self.latency.observe_prefill(num_tokens, duration_ms):
                tel.count("slo_rejected_latency_observations")
            return
        self.mtp_phase_profiler.record_cpu(
            "mtp.engine_model_runner_wall" if self.num_speculative_tokens else "target_only.engine_model_runner_wall",
            duration_ms)
        tel.count("decode_observed_tokens", num_tokens)
        tel.counters["decode_observed_ms"] += duration_ms
        self.latency.observe_decode(duration_ms)

    def _next_waiting(self) -> Sequence:
        self.telemetry.count("scheduler_admission_decisions")
        self.telemetry.begin()
        return self.admission.select(self, self.clock())

    def _pick_victim(self, current: Sequence) -> Sequence:
        self.telemetry.count("scheduler_preemption_decisions")
        self.telemetry.begin()
        return self.preemption.victim(self, current)

    def preempt(self, seq: Sequence) -> None:
        self.telemetry.count("preemption_count")
        seq.mark_preempted()
        seq.status = SequenceStatus.WAITING
        seq.is_prefill = True
        if self.prefix_planner is not None:
            self.prefix_planner.forget(seq)
        self.block_manager.deallocate(seq)
        self._release_state(seq)
        self.waiting.appendleft(seq)

    # ---------------------------------------------------------------- prefill
    def _plan_admission(self, seq: Sequence) -> tuple[bool, AdmissionPlan | None, int]:
        """(fits, hybrid plan, whole cached pages) for a request without pages."""
        tel, bm = self.telemetry, self.block_manager
        if self.enable_prefix_cache:
            tel.count("prefix_cache_queries")
            tel.count("prefix_cache_eligible_blocks", max(seq.num_blocks - 1, 0))
        if self.prefix_planner is not None:
            plan = self.prefix_planner.plan(seq)
            return plan is not None, plan, plan.num_cached_blocks if plan is not None else 0
        cached = bm.can_allocate(seq, use_prefix_cache=self.enable_prefix_cache)
        return cached >= 0, None, max(cached, 0)

    def _admit(self, seq: Sequence, plan: AdmissionPlan | None, cached_pages: int) -> None:
        """Take pages and a state slot for ``seq`` and restore its prefix; undo everything on failure."""
        if plan is None:
            self.block_manager.allocate(seq, cached_pages)
            self._take_state(seq)
            kv_tokens = joint = cached_pages * self.block_size
        else:
            page_copy = None
            try:
                page_copy = self.block_manager.allocate_candidate(seq, plan.candidate)
                self._take_state(seq)
                if page_copy is not None:
                    self.state_controller.call("copy_prefix_kv", page_copy.source_block_id,
                                               page_copy.destination_block_id, page_copy.num_tokens)
                if plan.hit is not None:
                    self.state_controller.call("restore_prefix_checkpoint", seq, plan.hit.checkpoint_slot)
                self.prefix_planner.commit(seq, plan)
            except Exception:
                self.prefix_planner.abandon(plan)
                if page_copy is not None:
                    self.block_manager.release_cow_source(page_copy)
                if seq.state_slot is not None:
                    self._release_state(seq)
                if seq.block_table:
                    self.block_manager.deallocate(seq)
                raise
            if page_copy is not None:
                self.block_manager.release_cow_source(page_copy)
            joint, kv_tokens = plan.boundary_tokens, plan.kv_candidate_tokens
        led = seq.ledger
        led.last_kv_candidate_tokens = kv_tokens
        led.last_gdn_checkpoint_tokens = joint
        led.last_joint_recoverable_tokens = joint
        led.prefix_tokens_reused += joint
        led.prefix_cache_hit_blocks += cached_pages
        self.telemetry.count("prefix_tokens_reused_actual", joint)
        self.telemetry.count("prefix_cache_hit_blocks", cached_pages)

    def _chunk_end(self, seq: Sequence, start: int, todo: int, budget: int) -> int:
        """Tokens of ``seq`` to run this step: the budget (chunked prefill), cut at the next retained
        checkpoint boundary when the hybrid cache captures states between steps."""
        n = min(todo, budget)
        if self.prefix_planner is not None and not self.enable_hybrid_internal_checkpoints:
            nxt = self._next_retained(seq, start)
            if nxt is not None and 0 < nxt.boundary_tokens - start < n:
                n = nxt.boundary_tokens - start
        return n

    def schedule_prefill(self, token_budget: int, sequence_budget: int) -> list[Sequence]:
        out: list[Sequence] = []
        used = 0
        while self.waiting and len(out) < sequence_budget and token_budget - used > 0:
            remaining = token_budget - used
            seq = self._next_waiting()
            plan, cached_pages = None, 0
            if seq.block_table:  # a chunked prefill continues
                todo = seq.num_tokens - seq.num_cached_tokens
            else:
                fits, plan, cached_pages = self._plan_admission(seq)
                if not fits or not self.state_available(seq):
                    break
                start = plan.boundary_tokens if plan is not None else cached_pages * self.block_size
                todo = seq.num_tokens - start
            if remaining < todo:
                if out:
                    break  # do not split a prompt when others already fill the step
                if not self.enable_chunked_prefill:
                    remaining = todo
            if not seq.block_table:
                self._admit(seq, plan, cached_pages)
            seq.num_scheduled_tokens = self._chunk_end(seq, seq.num_cached_tokens, todo, remaining)
            seq.mark_scheduled()
            seq.ledger.prefill_tokens_executed += seq.num_scheduled_tokens
            self.telemetry.count("prefill_tokens_scheduled_total", seq.num_scheduled_tokens)
            if seq.num_scheduled_tokens < todo:
                self.telemetry.count("chunked_prefill_steps")
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

    # ----------------------------------------------------------------- decode
    def schedule_decode(self, sequence_budget: int) -> list[Sequence]:
        t0 = perf_counter_ns()
        out: list[Sequence] = []
        # a speculative round writes target KV at pending..pending+K and MTP KV up to pending+2K-1
        reserve = 2 * self.num_speculative_tokens
        bm = self.block_manager
        while self.running and len(out) < sequence_budget:
            seq = self.running.popleft()
            fits = (lambda s=seq: bm.can_reserve_append(s, reserve)) if reserve else (lambda s=seq: bm.can_append(s))
            while not fits():
                victim = self._pick_victim(seq)
                if victim is seq:
                    self.preempt(seq)
                    break
                self.running.remove(victim)
                self.preempt(victim)
            else:
                seq.num_scheduled_tokens = 1
                seq.is_prefill = False
                if reserve:
                    bm.reserve_append(seq, reserve)
                else:
                    bm.may_append(seq)
                seq.mark_scheduled()
                out.append(seq)
        self.running.extendleft(reversed(out))
        self.mtp_phase_profiler.record_cpu("scheduler.decode_admission", (perf_counter_ns() - t0) / 1e6)
        return out

    # reference-compatible names of the two building blocks
    _schedule_prefill = schedule_prefill
    _schedule_decode = schedule_decode

    # ------------------------------------------------------- hybrid captures
    def _next_retained(self, seq: Sequence, start: int) -> RetainedBoundary | None:
        found = self.retention.next_boundary(start, seq.num_tokens)
        promo = self.prefix_planner.promotion_for(seq)
        if promo is None or promo.boundary.boundary_tokens <= start:
            return found
        if found is None or promo.boundary.boundary_tokens <= found.boundary_tokens:
            return promo.boundary
        return found

    def _retained_in_chunk(self, seq: Sequence, end: int) -> list[RetainedBoundary]:
        """Boundaries inside ``(num_cached_tokens, end]`` that get a checkpoint this step, capped
        at the index capacity (the promoted junction always stays)."""
        start = seq.num_cached_tokens
        kept = self.retention.boundaries(start, end, seq.num_tokens)
        promo = self.prefix_planner.promotion_for(seq)
        j = promo.boundary if promo is not None and start < promo.boundary.boundary_tokens <= end else None
        if j is not None:
            kept = [b for b in kept if b.boundary_tokens != j.boundary_tokens] + [j]
        kept.sort(key=lambda b: b.boundary_tokens)
        cap = self.prefix_planner.index.capacity
        if len(kept) > cap:
            others = [b for b in kept if b is not j]
            keep = others[len(others) - (cap - (1 if j is not None else 0)):] if cap > (1 if j else 0) else []
            kept = sorted(keep + ([j] if j is not None else []), key=lambda b: b.boundary_tokens)
        return kept

    def _boundary_at_end(self, seq: Sequence, end: int) -> RetainedBoundary | None:
        promo = self.prefix_planner.promotion_for(seq)
        if promo is not None and promo.boundary.boundary_tokens == end:
            return promo.boundary
        return self.retention.classify(end, seq.num_tokens)

    def internal_prefix_boundaries(self, seqs: list[Sequence], is_prefill: bool) -> dict[int, tuple[int, ...]]:
        """Per request, retained boundaries strictly inside its scheduled chunk (internal checkpoints)."""
        if not is_prefill or not self.enable_hybrid_internal_checkpoints:
            return {}
        out = {}
        for seq in seqs:
            end = seq.num_cached_tokens + seq.num_scheduled_tokens
            inner = tuple(b.boundary_tokens for b in self._retained_in_chunk(seq, end) if b.boundary_tokens < end)
            if inner:
                out[seq.seq_id] = inner
        return out

    def prepare_prefix_captures(self, seqs: list[Sequence], is_prefill: bool):
        """Capture tickets for the retained boundaries this prefill step reaches.

        Returns ``(tickets, blocks_hashed)``: the step's pages are indexed here, before the tickets
        need their prefix hashes, whenever anything is eligible."""
        if not is_prefill or self.prefix_planner is None:
            return [], False
        wanted = []
        for seq in seqs:
            if seq.num_scheduled_tokens <= 0:
                continue
            end = seq.num_cached_tokens + seq.num_scheduled_tokens
            if self.enable_hybrid_internal_checkpoints:
                kept = self._retained_in_chunk(seq, end)
            else:
                b = self._boundary_at_end(seq, end)
                kept = [b] if b is not None else []
            if kept:
                wanted.append((seq, end, kept))
        if not wanted:
            return [], False
        for seq in seqs:
            self.block_manager.hash_blocks(seq)
        tickets = []
        planner = self.prefix_planner
        for seq, end, kept in wanted:
            promo = planner.promotion_for(seq)
            for b in kept:
                meta = self.block_manager.prefix_metadata_at_boundary(seq, b.boundary_tokens)
                junction = b.reason == "shared_junction" and promo is not None
                ticket = CaptureTicket(
                    prefix_hash=meta.prefix_hash, boundary_tokens=b.boundary_tokens, tail_block_id=meta.tail_block_id,
                    state_slot=seq.state_slot, reason=b.reason, internal_state=b.boundary_tokens < end,
                    sequence_id=seq.seq_id, replay_saved_tokens=promo.saved_replay_tokens if junction else b.boundary_tokens,
                    demand_count=promo.demand if junction else 0)
                if planner.contains(ticket.prefix_hash, ticket.boundary_tokens):
                    planner.settle(ticket, published=False)
                    continue
                tickets.append(ticket)
        return tickets, True

    def reserve_prefix_capture(self, ticket: CaptureTicket) -> bool:
        """Room in the index for ``ticket``; evicted checkpoints are freed on every rank."""
        evicted = self.prefix_planner.reserve(ticket)
        if evicted is None:
            return False
        for r in evicted:
            self.state_controller.call("evict_prefix_checkpoint", r.checkpoint_slot)
        return True

    def publish_prefix_capture(self, ticket: CaptureTicket, checkpoint_slot: int) -> None:
        self.prefix_planner.publish(ticket, checkpoint_slot)

    def cancel_prefix_capture(self, ticket: CaptureTicket) -> None:
        self.prefix_planner.settle(ticket, published=False)

    # ---------------------------------------------------------------- commit
    def _done(self, seq: Sequence, token_id: int) -> bool:
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
                continue  # a chunk in the middle of the prompt samples nothing
            seq.append_token(tok, t0)
            if self._done(seq, tok):
                self.running.remove(seq)
                self._retire(seq, SequenceStatus.FINISHED, t0)
        if not is_prefill:
            self.mtp_phase_profiler.record_cpu("target_only.scheduler_commit", (perf_counter_ns() - t0) / 1e6)

    def postprocess_speculative(self, seqs: list[Sequence], output_token_ids: list[list[int]]) -> None:
        """Commit a speculative round; the last emitted token stays pending (its KV is not written)."""
        t0 = perf_counter_ns()
        for seq, toks in zip(seqs, output_token_ids):
            if not toks:
                raise ValueError("speculative decode must emit at least one token")
            seq.num_cached_tokens += len(toks)
            seq.num_scheduled_tokens = 0
            finished = False
            for tok in toks:
                if seq.num_completion_tokens >= seq.max_tokens:
                    finished = True
                    break
                seq.append_token(tok, t0)
                if not seq.ignore_eos and tok == self.eos:
                    finished = True
                    break
            if finished or seq.num_completion_tokens >= seq.max_tokens:
                self.running.remove(seq)
                self._retire(seq, SequenceStatus.FINISHED, t0)
            else:
                seq.num_cached_tokens = len(seq) - 1
                self.block_manager.trim_to_sequence_length(seq)
        self.mtp_phase_profiler.record_cpu("scheduler.speculative_commit", (perf_counter_ns() - t0) / 1e6)

    # --------------------------------------------------------------- metrics
    def reset_metrics(self) -> None:
        self.mtp_phase_profiler.reset()
        self.block_manager.reset_metrics()
        self.telemetry.reset()
        self.completed_request_metrics.clear()
        if self.prefix_planner is not None:
            self.prefix_planner.reset_metrics()

    def get_scheduler_decision_events(self) -> list[dict]:
        return list(self.telemetry.events)

    def get_request_metrics(self) -> list[dict]:
        return list(self.completed_request_metrics)

    def get_metrics(self) -> dict:
        tel, c, bm = self.telemetry, self.telemetry.counters, self.block_manager
        eligible = c["prefix_cache_eligible_blocks"]
        decisions = c["hybrid_scheduler_admission_decisions"]
        cfg = self.policy_cfg

        def mean(total: str, count: str) -> float:
            return c[total] / c[count] if c[count] else 0.0

        m = {
            "prefix_cache_enabled": self.enable_prefix_cache,
            "prefix_cache_queries": c["prefix_cache_queries"],
            "prefix_cache_eligible_blocks": eligible,
            "prefix_cache_hit_blocks": c["prefix_cache_hit_blocks"],
            "prefix_cache_hit_rate": c["prefix_cache_hit_blocks"] / eligible if eligible else 0.0,
            "chunked_prefill_enabled": self.enable_chunked_prefill,
            "scheduling_policy": self.scheduling_policy,
            "waiting_admission_policy": self.waiting_admission_policy,
            "preemption_policy": self.preemption_policy,
            "hybrid_scheduler_score_source": self.score_source,
            "hybrid_scheduler_aging_enabled": cfg.aging,
            "hybrid_scheduler_hysteresis_enabled": cfg.hysteresis,
            "hybrid_scheduler_sticky_recovery_enabled": cfg.sticky,
            "scheduler_profiling_enabled": tel.profiling,
            "num_waiting": len(self.waiting),
            "num_running": len(self.running),
            "last_slo_decision": tel.last_slo_decision,
            "last_hybrid_scheduler_decision": tel.last_hybrid_decision,
            "hybrid_scheduler_reorder_rate": c["hybrid_scheduler_reorders"] / decisions if decisions else 0.0,
            "hybrid_scheduler_selected_original_rank_mean": mean("hybrid_scheduler_selected_original_rank_total",
                                                                 "hybrid_scheduler_admission_decisions"),
            "hybrid_scheduler_selected_rank_histogram": dict(sorted(tel.rank_histogram.items())),
            "hybrid_scheduler_max_observed_wait_ms": tel.max_observed_wait_ms,
            "hybrid_scheduler_admission_latency": latency_summary(tel.admission_us),
            "hybrid_scheduler_probe_latency": latency_summary(tel.probe_us),
            "recompute_aware_selection_latency": latency_summary(tel.preemption_us),
            "scheduler_metrics_bookkeeping_latency": latency_summary(tel.bookkeeping_us),
            "scheduler_victim_mean_cost_per_reclaimed_block": mean("scheduler_cost_sum", "scheduler_cost_count"),
            "recompute_aware_mean_cost_per_reclaimed_block": mean("recompute_aware_cost_sum",
                                                                  "recompute_aware_cost_count"),
            "prefill_ms_per_token_ewma": self.latency.prefill_ms_per_token,
            "prefill_base_ms": self.latency.prefill_base_ms,
            "decode_step_ms_ewma": self.latency.decode_step_ms,
            "prefill_tokens_per_s": (c["prefill_observed_tokens"] / (c["prefill_observed_ms"] / 1e3)
                                     if c["prefill_observed_ms"] else 0.0),
            "decode_tokens_per_s": (c["decode_observed_tokens"] / (c["decode_observed_ms"] / 1e3)
                                    if c["decode_observed_ms"] else 0.0),
            "kv_blocks_total": bm.num_blocks,
            "kv_blocks_used": bm.num_used_blocks,
            "kv_blocks_free": bm.num_free_blocks,
            "kv_blocks_cached": bm.num_cached_blocks,
            "kv_blocks_cached_reachable": bm.num_reachable_cached_blocks,
            "kv_pressure": self.kv_pressure(),
            "prefix_match_unit": bm.prefix_match_unit,
            "partial_prefix_cow_allocations": bm.partial_prefix_cow_allocations,
            "prefix_cache_evictions": bm.prefix_cache_evictions,
            "prefix_cache_cached_block_reassignments": bm.cached_block_reassignments,
            "prefix_cache_duplicate_registrations": bm.duplicate_cache_registrations,
            "block_manager": bm.metrics(),
            "mtp_phase_profile": self.mtp_phase_profiler.metrics(),
        }
        zero_keys = (
            "chunked_prefill_steps", "preemption_count", "aborted_request_count", "completed_request_count",
            "slo_prefill_priority_steps", "slo_decode_priority_steps", "slo_admission_deferred_steps",
            "slo_dynamic_prefill_tokens", "slo_rejected_latency_observations", "slo_infeasible_budget_steps",
            "slo_throughput_priority_steps", "scheduler_admission_decisions", "hybrid_scheduler_admission_decisions",
            "hybrid_scheduler_reorders", "hybrid_scheduler_aging_overrides", "hybrid_scheduler_candidates_probed",
            "hybrid_scheduler_estimated_saved_prefill_tokens", "hybrid_scheduler_selected_reusable_tokens",
            "hybrid_scheduler_selected_kv_candidate_tokens", "hybrid_scheduler_selected_gdn_checkpoint_tokens",
            "hybrid_scheduler_selected_joint_recoverable_tokens", "hybrid_scheduler_estimated_remaining_prefill_tokens",
            "hybrid_scheduler_selected_original_rank_max", "hybrid_scheduler_hysteresis_rejections",
            "hybrid_scheduler_sticky_recovery_triggers", "hybrid_scheduler_starvation_count",
            "hybrid_scheduler_probe_ms", "scheduler_admission_decision_ms", "recompute_aware_preemptions",
            "scheduler_preemption_decisions", "scheduler_victim_computed_tokens", "scheduler_victim_logical_blocks",
            "scheduler_victim_reclaimable_blocks", "scheduler_victim_recompute_tokens",
            "recompute_aware_reclaimed_blocks", "recompute_aware_estimated_recompute_tokens",
            "recompute_aware_avoided_recompute_tokens", "recompute_aware_selection_ms",
            "scheduler_preemption_selection_ms", "scheduler_metrics_bookkeeping_ms",
            "recompute_aware_victim_computed_tokens", "recompute_aware_victim_logical_blocks",
            "prefill_observed_tokens", "prefill_observed_ms", "prefill_tokens_scheduled_total",
            "prefix_tokens_reused_actual", "decode_observed_tokens", "decode_observed_ms")
        for k in zero_keys:
            m[k] = c[k]
        if self.prefix_planner is not None:
            m.update(self.prefix_planner.get_metrics())
        return m
