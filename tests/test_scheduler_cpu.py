"""Scheduler policies on the host: batch composition, chunked prefill, abort, prefix-cache metrics,
the SLO-aware prefill budget, hybrid-state-aware admission and preemption policies.

The scenarios follow the reference's scheduler tests (``tests/test_scheduler.py`` and
``tests/test_hybrid_state_aware_scheduler.py`` in ``ifeidepig/inference-systems``): the same
situations and the same expected decisions and metric values, driven through this package's
policy objects and a fixed scheduler clock.
"""

from types import SimpleNamespace

import pytest

from inference_systems_b200 import SamplingParams
from inference_systems_b200.engine.hybrid_prefix_cache import CaptureTicket
from inference_systems_b200.engine.scheduler import Scheduler
from inference_systems_b200.engine.sequence import Sequence, SequenceStatus

NOW = 10_000_000_000


@pytest.fixture(autouse=True)
def _page_size():
    old = Sequence.block_size
    Sequence.block_size = 256
    yield
    Sequence.block_size = old


def _cfg(**kw):
    base = dict(max_num_seqs=4, max_num_batched_tokens=256, eos=0, kvcache_block_size=256, num_kvcache_blocks=16,
                scheduling_policy="prefill_first", enable_prefix_cache=True, enable_chunked_prefill=True,
                scheduler_target_ttft_ms=200.0, scheduler_target_tpot_ms=50.0, slo_prefill_priority_threshold=0.8,
                slo_min_prefill_tokens=64, slo_kv_pressure_threshold=0.9, slo_queue_pressure_threshold=3)
    base.update(kw)
    return SimpleNamespace(**base)


def _sched(**kw) -> Scheduler:
    s = Scheduler(_cfg(**kw))
    s.clock = lambda: NOW
    return s


def _seq(tokens, *, age_ms=0.0, max_tokens=8):
    return Sequence(list(tokens), SamplingParams(temperature=0.1, max_tokens=max_tokens, ignore_eos=True),
                    arrival_time_ns=NOW - int(age_ms * 1e6))


def _running(s: Scheduler, token_gap_ms: float | None = None) -> Sequence:
    seq = _seq([1] * 64)
    s.block_manager.allocate(seq, 0)
    seq.status, seq.is_prefill = SequenceStatus.RUNNING, False
    if token_gap_ms is not None:
        seq.timeline.token(NOW - int(token_gap_ms * 1e6))
    s.running.append(seq)
    return seq


def _waiting(s: Scheduler, wait_ms: float = 0.0) -> Sequence:
    seq = _seq([2] * 300, age_ms=wait_ms)
    s.add(seq)
    return seq


# ----------------------------------------------------------------- batch composition
def test_prefill_first_runs_only_the_prefill():
    s = _sched()
    run, wait = _running(s), _waiting(s)
    batches = s.schedule()
    assert len(batches) == 1 and batches[0].is_prefill and batches[0].seqs == [wait]
    assert batches[0].num_tokens == 256 and run.num_scheduled_tokens == 0


def test_decode_first_fills_the_token_budget_with_both_phases():
    s = _sched(scheduling_policy="decode_first")
    run, wait = _running(s), _waiting(s)
    batches = s.schedule()
    assert [b.is_prefill for b in batches] == [False, True]
    assert batches[0].seqs == [run] and batches[1].seqs == [wait]
    assert sum(b.num_tokens for b in batches) == 256
    assert run.num_scheduled_tokens == 1 and wait.num_scheduled_tokens == 255


def test_abort_waiting_and_running_requests():
    s = _sched(scheduling_policy="decode_first")
    wait = _waiting(s)
    assert s.abort(wait.seq_id) and wait.is_finished and wait not in s.waiting
    assert s.get_metrics()["completed_request_count"] == 1
    assert s.get_request_metrics()[0]["status"] == "aborted"
    run = _running(s)
    free = s.block_manager.num_free_blocks
    assert s.abort(run.seq_id) and run.block_table == []
    assert s.block_manager.num_free_blocks == free + 1 and s.is_finished()
    assert not s.abort(999_999)


def test_chunked_prefill_off_schedules_the_whole_prompt():
    s = _sched(enable_chunked_prefill=False)
    wait = _waiting(s)
    assert s.schedule_prefill(256, 4) == [wait]
    assert wait.num_scheduled_tokens == 300 and len(wait.block_table) == 2
    assert s.get_metrics()["chunked_prefill_steps"] == 0


def test_chunked_prefill_metrics():
    s = _sched()
    _waiting(s)
    s.schedule()
    m = s.get_metrics()
    assert m["chunked_prefill_steps"] == 1 and m["kv_blocks_used"] == 2 and m["kv_blocks_free"] == 14


def test_prefix_cache_hit_is_observable():
    s = _sched()
    prompt = [3] * 300
    first = _seq(prompt, max_tokens=1)
    s.add(first)
    for _ in range(2):
        b = s.schedule()[0]
        s.postprocess(b.seqs, [9], is_prefill=True)
    again = _seq(prompt, max_tokens=1)
    s.add(again)
    b = s.schedule()[0]
    m = s.get_metrics()
    assert again.num_cached_tokens == 256 and b.num_tokens == 44
    assert m["prefix_cache_hit_blocks"] == 1 and m["prefix_cache_eligible_blocks"] == 2
    assert m["prefix_cache_hit_rate"] == 0.5


def test_prefix_cache_off_neither_hashes_nor_reuses():
    s = _sched(enable_prefix_cache=False)
    wait = _waiting(s)
    b = s.schedule()[0]
    s.postprocess(b.seqs, [9], is_prefill=True)
    m = s.get_metrics()
    assert wait.num_cached_tokens == 256
    assert m["prefix_cache_queries"] == 0 and m["prefix_cache_hit_blocks"] == 0 and m["kv_blocks_cached"] == 0


def test_metric_keys_cover_the_reference_dashboard_set():
    m = _sched().get_metrics()
    for k in ("hybrid_scheduler_admission_latency", "hybrid_scheduler_probe_latency",
              "recompute_aware_selection_latency", "hybrid_scheduler_selected_original_rank_mean",
              "scheduler_victim_mean_cost_per_reclaimed_block", "kv_blocks_cached_reachable",
              "prefix_cache_duplicate_registrations", "slo_throughput_priority_steps"):
        assert k in m


# ------------------------------------------------------------------------ SLO aware
def test_slo_urgent_prefill_does_not_skip_active_decode():
    s = _sched(scheduling_policy="slo_aware")
    run, wait = _running(s, token_gap_ms=10), _waiting(s, wait_ms=180)
    batches = s.schedule(NOW)
    assert [b.seqs for b in batches] == [[run], [wait]] and [b.is_prefill for b in batches] == [False, True]
    assert s.get_metrics()["last_slo_decision"]["decision"] == "decode_first"


def _latency(s, per_token=0.2, base=20.0, decode=6.0):
    s.latency.prefill_ms_per_token, s.latency.prefill_base_ms, s.latency.decode_step_ms = per_token, base, decode


def test_slo_budget_fits_the_tpot_slack():
    s = _sched(scheduling_policy="slo_aware")
    _latency(s)
    run, wait = _running(s, token_gap_ms=60), _waiting(s, wait_ms=100)
    batches = s.schedule(NOW)
    # slack 50 - 6 - 5 = 39 ms; (39 - 20) / ((0.2 * 256 - 20) / 256) = 155 tokens
    assert batches[0].seqs == [run] and batches[1].seqs == [wait] and batches[1].num_tokens == 155
    assert s.get_metrics()["last_slo_decision"]["prefill_budget"] == 155


def test_slo_kv_pressure_defers_nonurgent_prefill():
    s = _sched(scheduling_policy="slo_aware", slo_kv_pressure_threshold=0.05)
    run = _running(s, token_gap_ms=60)
    _waiting(s, wait_ms=20)
    batches = s.schedule(NOW)
    assert len(batches) == 1 and batches[0].seqs == [run] and not batches[0].is_prefill
    assert s.get_metrics()["slo_admission_deferred_steps"] == 1


def test_slo_infeasible_budget_waits_for_urgency():
    from inference_systems_b200.engine.scheduler import SloAware

    s = _sched(scheduling_policy="slo_aware", scheduler_target_tpot_ms=20.0)
    _latency(s)
    assert SloAware.prefill_budget(s, 255, 0.5) == 0
    assert SloAware.prefill_budget(s, 255, 0.9) == 255
    assert s.get_metrics()["slo_infeasible_budget_steps"] == 2


def test_slo_latency_observations():
    s = _sched(scheduling_policy="slo_aware")
    s.observe_batch(True, 256, 51.2)     # full chunk: 0.2 ms / token
    s.observe_batch(True, 32, 20.0)      # small chunk: only the base latency
    s.observe_batch(True, 256, 200.0)    # > 2x the estimate: rejected
    s.observe_batch(False, 4, 8.0)
    assert s.latency.prefill_ms_per_token == 0.2 and s.latency.prefill_base_ms == 20.0
    assert s.latency.decode_step_ms == 8.0
    assert s.get_metrics()["slo_rejected_latency_observations"] == 1


def test_slo_queue_pressure_restores_the_full_budget():
    s = _sched(scheduling_policy="slo_aware", slo_queue_pressure_threshold=3)
    _latency(s)
    _running(s, token_gap_ms=10)
    for w in (20, 15, 10):
        _waiting(s, wait_ms=w)
    batches = s.schedule(NOW)
    assert batches[1].num_tokens == 255
    assert s.get_metrics()["slo_throughput_priority_steps"] == 1


# ---------------------------------------------------------- hybrid-state-aware admission
def _hsa(**kw) -> Scheduler:
    base = dict(max_num_batched_tokens=1024, num_kvcache_blocks=32, prefix_match_unit=256,
                waiting_admission_policy="hybrid_state_aware", preemption_policy="recompute_aware",
                hybrid_scheduler_candidate_window=4, hybrid_scheduler_aging_tokens_per_ms=0.5,
                hybrid_scheduler_max_wait_ms=200.0, hybrid_scheduler_min_saved_tokens=16,
                hybrid_scheduler_preemption_penalty=0.0, num_speculative_tokens=0)
    base.update(kw)
    return _sched(**base)


def _seed(s: Scheduler, tokens, boundary=512):
    """Leave a finished request's first ``boundary`` tokens in the KV prefix cache."""
    src = _seq(tokens)
    s.block_manager.allocate(src, 0)
    src.num_scheduled_tokens = boundary
    s.block_manager.hash_blocks(src)
    s.block_manager.deallocate(src)


SHARED = list(range(512))


def _cold_warm(s, cold_age=10.0, warm_age=5.0):
    _seed(s, SHARED + [700] * 88)
    cold, warm = _seq([900] * 600, age_ms=cold_age), _seq(SHARED + [701] * 88, age_ms=warm_age)
    s.add(cold)
    s.add(warm)
    return cold, warm


def _select(s):
    return s._next_waiting()


def test_admission_prefers_reusable_work_within_the_window():
    s = _hsa()
    cold, warm = _cold_warm(s)
    assert _select(s) is warm and list(s.waiting) == [warm, cold]
    assert warm.ledger.last_reusable_tokens == 512 and cold.ledger.scheduler_bypass_count == 1
    m = s.get_metrics()
    assert m["hybrid_scheduler_reorders"] == 1 and m["hybrid_scheduler_estimated_saved_prefill_tokens"] == 512


def test_admission_window_bounds_queue_jumping():
    s = _hsa(hybrid_scheduler_candidate_window=1)
    cold, warm = _cold_warm(s)
    assert _select(s) is cold and list(s.waiting) == [cold, warm]


def test_zero_prefill_budget_probes_nothing():
    s = _hsa()
    a, b = _seq([900] * 600), _seq([901] * 600)
    s.add(a)
    s.add(b)
    assert s.schedule_prefill(0, 1) == [] and list(s.waiting) == [a, b]
    assert s.get_metrics()["hybrid_scheduler_admission_decisions"] == 0


@pytest.mark.parametrize("hysteresis", [True, False])
def test_hysteresis_keeps_the_feasible_head(hysteresis):
    s = _hsa(hybrid_scheduler_min_saved_tokens=600, hybrid_scheduler_enable_hysteresis=hysteresis)
    cold, warm = _cold_warm(s, cold_age=0.0, warm_age=0.0)
    if hysteresis:
        assert _select(s) is cold
        assert s.get_metrics()["last_hybrid_scheduler_decision"]["reason"] == "benefit_below_hysteresis"
    else:
        assert _select(s) is warm
        assert s.get_metrics()["hybrid_scheduler_hysteresis_rejections"] == 0


@pytest.mark.parametrize("aging", [True, False])
def test_aging_deadline_prevents_starvation(aging):
    s = _hsa(hybrid_scheduler_max_wait_ms=100.0, hybrid_scheduler_enable_aging=aging)
    overdue, warm = _cold_warm(s, cold_age=150.0, warm_age=5.0)
    if aging:
        assert _select(s) is overdue
        m = s.get_metrics()
        assert m["last_hybrid_scheduler_decision"]["reason"] == "aging_deadline"
        assert m["hybrid_scheduler_aging_overrides"] == 1
    else:
        assert _select(s) is warm and s.get_metrics()["hybrid_scheduler_aging_overrides"] == 0


def test_chunk_continuation_and_preempted_head_are_sticky():
    s = _hsa()
    cont = _seq([1] * 600)
    s.block_manager.allocate(cont, 0)
    cont.num_cached_tokens = 256
    s.add(cont)
    s.add(_seq([2] * 600))
    assert _select(s) is cont and s.get_metrics()["hybrid_scheduler_admission_decisions"] == 0
    s.block_manager.deallocate(cont)
    cont.ledger.preemption_count = 1
    assert _select(s) is cont


def test_sticky_recovery_can_be_switched_off():
    s = _hsa(hybrid_scheduler_enable_sticky_recovery=False)
    _seed(s, SHARED + [700] * 88)
    cont = _seq([900] * 600)
    s.block_manager.allocate(cont, 0)
    cont.num_cached_tokens = 256
    warm = _seq(SHARED + [701] * 88)
    s.add(cont)
    s.add(warm)
    assert _select(s) is warm and s.get_metrics()["hybrid_scheduler_sticky_recovery_triggers"] == 0


def test_reclaimable_blocks_exclude_shared_pages():
    s = _hsa()
    a = _seq([1] * 600)
    s.block_manager.allocate(a, 0)
    s.block_manager._share(a.block_table[0])   # another owner of the first page
    assert s.block_manager.reclaimable_blocks(a) == 2


# ---------------------------------------------------------------------- preemption
def _running_with_prefix(s, tokens, hashed=0):
    seq = _seq(tokens)
    s.block_manager.allocate(seq, 0)
    if hashed:
        seq.num_scheduled_tokens = hashed
        s.block_manager.hash_blocks(seq)
        seq.num_scheduled_tokens = 0
    seq.num_cached_tokens = len(tokens)
    seq.status = SequenceStatus.RUNNING
    return seq


def test_recompute_aware_victim_beats_lifo():
    s = _hsa()
    cheap = _running_with_prefix(s, list(range(512)) + [11] * 88, hashed=512)
    expensive = _running_with_prefix(s, [99] * 600)
    s.running.append(expensive)
    assert s._pick_victim(cheap) is cheap
    m = s.get_metrics()
    assert m["recompute_aware_estimated_recompute_tokens"] == 88
    assert m["recompute_aware_avoided_recompute_tokens"] == 512
    assert m["recompute_aware_reclaimed_blocks"] == 3
    assert cheap.ledger.estimated_recompute_tokens_lost == 88


def test_lifo_takes_the_newest_running_request():
    s = _hsa(preemption_policy="lifo")
    current, older, newest = (_running_with_prefix(s, [t] * 300) for t in (1, 2, 3))
    s.running.extend([older, newest])
    assert s._pick_victim(current) is newest and s.get_metrics()["recompute_aware_preemptions"] == 0


def test_decode_pressure_preempts_the_cheaper_request():
    s = _hsa(num_kvcache_blocks=4)
    current = _running_with_prefix(s, [90] * 257)
    current.num_cached_tokens = 256
    cheap = _running_with_prefix(s, list(range(256)) + [11] * 44, hashed=256)
    cheap.num_cached_tokens = 256
    s.running.extend([current, cheap])
    assert s.schedule_decode(1) == [current]
    assert current in s.running and cheap in s.waiting and cheap.preemption_count == 1
    assert len(current.block_table) == 3 and s.get_metrics()["preemption_count"] == 1


# ------------------------------------------------------- hybrid admission scoring
def _hybrid(score_source="joint"):
    """A 4-token-page hybrid scheduler whose checkpoint index holds the boundary at 4 tokens of a
    prefix whose KV is cached up to 8 tokens."""
    Sequence.block_size = 4
    s = Scheduler(_cfg(max_num_batched_tokens=1024, kvcache_block_size=4, prefix_match_unit=4, num_kvcache_blocks=12,
                       enable_hybrid_prefix_cache=True, hybrid_prefix_checkpoint_interval_blocks=1,
                       hybrid_scheduler_score_source=score_source, waiting_admission_policy="hybrid_state_aware"),
                  state_manager=SimpleNamespace(can_allocate=True), prefix_checkpoint_pool=SimpleNamespace(capacity=4))
    s.clock = lambda: NOW
    src = _seq(list(range(9)))
    s.block_manager.allocate(src, 0)
    src.num_scheduled_tokens = 8
    s.block_manager.hash_blocks(src)
    meta = s.block_manager.prefix_metadata_at_boundary(src, 4)
    s.block_manager.deallocate(src)
    s.prefix_planner.publish(CaptureTicket(meta.prefix_hash, 4, meta.tail_block_id, state_slot=0), checkpoint_slot=0)
    return s


def test_hybrid_admission_scores_the_kv_and_gdn_intersection():
    s = _hybrid()
    rec = s.oracle.assess(_seq(list(range(8)) + [99]))
    assert (rec.kv_tokens, rec.joint_tokens, rec.score_tokens) == (8, 4, 4)


def test_hybrid_kv_only_scoring_changes_ranking_not_restore():
    s = _hybrid("kv_only")
    rec = s.oracle.assess(_seq(list(range(8)) + [99]))
    assert (rec.kv_tokens, rec.gdn_tokens, rec.joint_tokens, rec.score_tokens) == (8, 4, 4, 8)


def test_profiling_exports_latency_and_decision_trace():
    s = _hsa(enable_scheduler_profiling=True)
    s.add(_seq([1] * 300))
    s.add(_seq([2] * 300))
    _select(s)
    m = s.get_metrics()
    assert m["hybrid_scheduler_admission_latency"]["count"] == 1
    assert m["hybrid_scheduler_probe_latency"]["count"] == 1
    assert s.get_scheduler_decision_events()[0]["type"] == "admission"
