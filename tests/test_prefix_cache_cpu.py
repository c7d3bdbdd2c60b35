"""Hybrid prefix cache control plane, KV block index and checkpoint pool on the host.

The scenarios follow the reference's ``tests/test_hybrid_prefix_cache.py`` and
``tests/test_block_manager.py`` (``ifeidepig/inference-systems``): joint KV + GDN restore
boundaries, the read-only probe, shared-junction promotion and its threshold, retention and
eviction policies, the sub-page (16-token) index with its copy-on-write plan and rollback, and the
checkpoint pool's storage formats.  They drive this package's planner / index / promoter objects.
"""

from types import SimpleNamespace

import pytest
import torch

from inference_systems_b200 import SamplingParams
from inference_systems_b200.engine.block_manager import BlockManager, PrefixKVCandidate
from inference_systems_b200.engine.hybrid_prefix_cache import (
    CaptureTicket,
    CheckpointIndex,
    HybridPrefixPlanner,
    make_retention,
)
from inference_systems_b200.engine.scheduler import Scheduler
from inference_systems_b200.engine.sequence import Sequence
from inference_systems_b200.engine.state_pool import HybridPrefixCheckpointPool, HybridStateManager


@pytest.fixture
def page4():
    old = Sequence.block_size
    Sequence.block_size = 4
    yield
    Sequence.block_size = old


@pytest.fixture
def page256():
    old = Sequence.block_size
    Sequence.block_size = 256
    yield
    Sequence.block_size = old


def _seq(tokens):
    return Sequence(list(tokens), SamplingParams(temperature=0.0, max_tokens=1))


def _cached_source(blocks, tokens, upto):
    """Run a request's first ``upto`` tokens through the index, then free its pages (they stay cached)."""
    src = _seq(tokens)
    blocks.allocate(src, 0)
    src.num_scheduled_tokens = upto
    blocks.hash_blocks(src)
    return src


def _ticket(c: PrefixKVCandidate, **kw):
    return CaptureTicket(c.prefix_hash, c.boundary_tokens, c.tail_block_id, state_slot=0, **kw)


# ------------------------------------------------------------------------------ KV index
def test_metadata_falls_back_to_the_shorter_checkpointed_boundary(page4):
    blocks = BlockManager(8, 4)
    src = _cached_source(blocks, range(9), 8)
    at4 = blocks.prefix_metadata_at_boundary(src, 4)
    blocks.deallocate(src)
    index = CheckpointIndex(capacity=1)
    index.insert(_ticket(at4), checkpoint_slot=0)
    cands = blocks.find_prefix_candidates(_seq(list(range(8)) + [99]))
    assert [c.boundary_tokens for c in cands] == [8, 4]
    hit = index.lookup(cands)
    assert hit is not None and hit.candidate.boundary_tokens == 4 and hit.checkpoint_slot == 0


def test_sub_page_index_finds_the_boundary_and_plans_copy_on_write(page256):
    blocks = BlockManager(12, 256, prefix_match_unit=16)
    shared = list(range(500))
    src = _cached_source(blocks, shared + [700 + i for i in range(64)], 564)
    blocks.deallocate(src)
    incoming = _seq(shared + [900 + i for i in range(64)])
    c = blocks.find_prefix_candidates(incoming)[0]
    assert (c.boundary_tokens, c.num_cached_blocks, c.tail_valid_tokens) == (496, 1, 240)
    assert blocks.can_allocate_candidate(incoming, c)
    cow = blocks.allocate_candidate(incoming, c)
    assert cow.source_block_id == c.tail_block_id and cow.destination_block_id == incoming.block_table[1]
    assert cow.destination_block_id != cow.source_block_id and cow.num_tokens == 240
    assert incoming.num_cached_tokens == 496
    blocks.release_cow_source(cow)
    blocks.deallocate(incoming)
    assert not blocks.used_block_ids


def test_sub_page_match_rounds_n_minus_one_n_n_plus_one(page256):
    blocks = BlockManager(12, 256, prefix_match_unit=16)
    tokens = list(range(240)) + [800 + i for i in range(80)]
    blocks.deallocate(_cached_source(blocks, tokens, 320))

    def longest(shared):
        return blocks.find_prefix_candidates(_seq(tokens[:shared] + [1200 + i for i in range(320 - shared)]))[0].boundary_tokens

    assert (longest(239), longest(240), longest(241)) == (224, 240, 240)


def test_reassigning_a_page_drops_its_sub_page_entries(page4):
    blocks = BlockManager(2, 8, prefix_match_unit=2)
    Sequence.block_size = 8
    src = _cached_source(blocks, range(9), 9)
    assert blocks.find_prefix_candidates(src)
    blocks.deallocate(src)
    blocks.allocate(_seq([50 + i for i in range(9)]), 0)
    assert blocks.find_prefix_candidates(src) == [] and blocks.prefix_cache_evictions > 0


def test_cached_page_reassignment_counts_an_eviction():
    Sequence.block_size = 2
    try:
        blocks = BlockManager(1, 2)
        src = _cached_source(blocks, [10, 20], 2)
        blocks.deallocate(src)
        assert blocks.num_cached_blocks == 1
        blocks.allocate(_seq([1, 2]), 0)
        assert blocks.cached_block_reassignments == 1 and blocks.prefix_cache_evictions == 1
        assert blocks.num_cached_blocks == 0 and blocks.num_reachable_cached_blocks == 0
    finally:
        Sequence.block_size = 256


def test_duplicate_registration_keeps_the_newest_page_reachable():
    Sequence.block_size = 2
    try:
        blocks = BlockManager(4, 2)
        a, b = _seq([1, 2, 90]), _seq([1, 2, 91])
        blocks.allocate(a, 0)
        blocks.allocate(b, 0)
        for s in (a, b):
            s.num_scheduled_tokens = 2
            blocks.hash_blocks(s)
        assert blocks.duplicate_cache_registrations == 1
        assert blocks.num_cached_blocks == 2 and blocks.num_reachable_cached_blocks == 1
        assert blocks.find_prefix_candidates(_seq([1, 2, 7]))[0].tail_block_id == b.block_table[0]
        blocks.reset_metrics()
        assert blocks.duplicate_cache_registrations == 0 and blocks.num_cached_blocks == 2
    finally:
        Sequence.block_size = 256


# ------------------------------------------------------------------------------ planner
def _planner(blocks, capacity=2, promote=False, sightings=2, policy="lru"):
    return HybridPrefixPlanner(blocks, CheckpointIndex(capacity, policy), promote_shared_junctions=promote,
                               promotion_min_sightings=sightings)


def test_plan_takes_the_longest_jointly_restorable_boundary(page4):
    blocks = BlockManager(8, 4)
    src = _cached_source(blocks, range(9), 8)
    at4 = blocks.prefix_metadata_at_boundary(src, 4)
    blocks.deallocate(src)
    p = _planner(blocks, capacity=1)
    p.index.insert(_ticket(at4), 0)
    plan = p.plan(_seq(list(range(8)) + [99]))
    assert plan.boundary_tokens == 4 and plan.num_cached_blocks == 1 and plan.hit.checkpoint_slot == 0


def test_probe_has_no_side_effects(page4):
    blocks = BlockManager(8, 4)
    src = _cached_source(blocks, range(9), 8)
    at4 = blocks.prefix_metadata_at_boundary(src, 4)
    blocks.deallocate(src)
    p = _planner(blocks, promote=True)
    p.index.insert(_ticket(at4), 0)
    before = (p.get_metrics(), dict(p.promoter.demand), list(p.index.records),
              p.index.records[(at4.prefix_hash, 4)].hits)
    probe = p.probe(_seq(list(range(8)) + [99]))
    assert probe.boundary_tokens == 4 and probe.kv_candidate_tokens == 8
    assert (p.get_metrics(), dict(p.promoter.demand), list(p.index.records),
            p.index.records[(at4.prefix_hash, 4)].hits) == before


def test_kv_only_match_gives_a_cold_plan(page4):
    blocks = BlockManager(8, 4)
    blocks.deallocate(_cached_source(blocks, range(9), 8))
    p = _planner(blocks, capacity=1)
    plan = p.plan(_seq(list(range(8)) + [99]))
    assert plan.hit is None and plan.boundary_tokens == 0 and plan.num_cached_blocks == 0
    assert p.get_metrics()["hybrid_prefix_fallback_count"] == 1


def test_adaptive_promotes_the_longest_kv_only_junction_once(page4):
    blocks = BlockManager(8, 4)
    blocks.deallocate(_cached_source(blocks, range(9), 8))
    p = _planner(blocks, promote=True)
    incoming = _seq(list(range(8)) + [99])
    plan = p.plan(incoming)
    assert plan.hit is None and plan.promotion_candidate.boundary_tokens == 8
    p.commit(incoming, plan)
    again = p.plan(incoming)
    assert again.promotion_candidate is None  # already pending
    m = p.get_metrics()
    assert m["hybrid_prefix_kv_only_miss_count"] == 2 and m["hybrid_prefix_alignment_lost_tokens"] == 16
    assert m["hybrid_prefix_shared_junction_promotions_planned"] == 1


def test_promotion_threshold_three_waits_for_the_third_sighting(page4):
    blocks = BlockManager(8, 4)
    blocks.deallocate(_cached_source(blocks, range(9), 8))
    p = _planner(blocks, promote=True, sightings=3)
    assert p.plan(_seq(list(range(8)) + [99])).promotion_candidate is None     # second sighting
    third = _seq(list(range(8)) + [100])
    plan = p.plan(third)
    assert plan.promotion_candidate is not None
    p.commit(third, plan)
    c = plan.promotion_candidate
    assert p.promoter.observations(c) == 2
    p.publish(CaptureTicket(c.prefix_hash, c.boundary_tokens, c.tail_block_id, state_slot=0,
                            reason="shared_junction", sequence_id=third.seq_id, replay_saved_tokens=8, demand_count=2),
              checkpoint_slot=0)
    fourth = _seq(list(range(8)) + [101])
    plan = p.plan(fourth)
    assert plan.hit is not None
    p.commit(fourth, plan)
    m = p.get_metrics()
    assert m["hybrid_prefix_promotion_min_sightings"] == 3 and m["hybrid_prefix_kv_only_miss_count"] == 2
    assert m["hybrid_prefix_useful_promotion_count"] == 1 and m["hybrid_prefix_useful_promotion_ratio"] == 1.0
    assert m["hybrid_prefix_promotions_not_yet_reused"] == 0
    assert m["hybrid_prefix_shared_junction_saved_replay_tokens"] == 8


def test_a_failed_junction_capture_can_be_promoted_again(page4):
    blocks = BlockManager(8, 4)
    blocks.deallocate(_cached_source(blocks, range(9), 8))
    p = _planner(blocks, promote=True)
    incoming = _seq(list(range(8)) + [99])
    first = p.plan(incoming)
    p.commit(incoming, first)
    c = first.promotion_candidate
    p.settle(CaptureTicket(c.prefix_hash, c.boundary_tokens, c.tail_block_id, state_slot=0, reason="shared_junction",
                           sequence_id=incoming.seq_id), published=False)
    assert p.plan(incoming).promotion_candidate is not None
    assert p.get_metrics()["hybrid_prefix_shared_junction_promotions_cancelled"] == 1


# ---------------------------------------------------------------- retention / eviction
def test_adaptive_retention_adds_the_prompt_tail_only():
    periodic, adaptive = make_retention("periodic", 4, 16), make_retention("adaptive", 4, 16)
    assert periodic.next_boundary(16, 27) is None
    b = adaptive.next_boundary(16, 27)
    assert (b.boundary_tokens, b.reason) == (24, "prompt_tail")
    assert adaptive.classify(20, 27) is None
    assert [x.boundary_tokens for x in adaptive.boundaries(0, 27, 27)] == [16, 24]


def test_cost_aware_eviction_keeps_a_reused_shorter_checkpoint():
    index = CheckpointIndex(2, "cost_aware")
    index.insert(CaptureTicket(11, 4, 1, 0), 0)
    index.insert(CaptureTicket(22, 8, 2, 1), 1)
    short = PrefixKVCandidate(1, 4, 11, 1)
    for _ in range(2):
        index.note_lookup(4, True, index.lookup([short]))
    evicted = index.make_room(CaptureTicket(33, 12, 3, 2))
    assert [r.prefix_hash for r in evicted] == [22] and (11, 4) in index
    assert index.metrics()["hybrid_prefix_evicted_retained_value"] == 8


def test_lru_eviction_is_bounded():
    index = CheckpointIndex(1)
    index.insert(CaptureTicket(11, 4, 2, 0), 0)
    evicted = index.make_room(CaptureTicket(22, 8, 3, 1))
    assert [r.prefix_hash for r in evicted] == [11] and not index.records
    index.insert(CaptureTicket(22, 8, 3, 1), 0)
    assert list(index.records) == [(22, 8)] and index.metrics()["hybrid_prefix_eviction_count"] == 1


def test_unused_junction_eviction_counts_as_pollution():
    index = CheckpointIndex(1)
    index.insert(CaptureTicket(11, 8, 1, 0, reason="shared_junction", replay_saved_tokens=8, demand_count=1), 0)
    assert len(index.make_room(CaptureTicket(22, 16, 2, 1, reason="prompt_tail"))) == 1
    m = index.metrics()
    assert m["hybrid_prefix_shared_junction_eviction_count"] == 1
    assert m["hybrid_prefix_unused_promotion_eviction_count"] == 1
    assert m["hybrid_prefix_entries_shared_junction"] == 0 and m["hybrid_prefix_peak_shared_junction_entries"] == 1


# -------------------------------------------------------------------- scheduler paths
class _Controller:
    def __init__(self, fail_on=None):
        self.next_slot, self.fail_on, self.calls = 0, fail_on, []

    def call(self, method, *args):
        self.calls.append(method)
        if method == self.fail_on:
            raise RuntimeError(f"injected {method} failure")
        if method == "allocate_state_slot":
            args[0].state_slot = self.next_slot
            self.next_slot += 1
            return args[0].state_slot
        if method == "free_state_slot":
            args[0].state_slot = None
        return None


def _hybrid_sched(controller, **kw):
    cfg = dict(max_num_seqs=4, max_num_batched_tokens=64, eos=-1, kvcache_block_size=4, prefix_match_unit=4,
               num_kvcache_blocks=16, scheduling_policy="prefill_first", enable_prefix_cache=True,
               enable_chunked_prefill=True, enable_hybrid_prefix_cache=True, hybrid_prefix_checkpoint_interval_blocks=4,
               hybrid_prefix_retention_policy="adaptive", hybrid_prefix_eviction_policy="cost_aware")
    cfg.update(kw)
    return Scheduler(SimpleNamespace(**cfg), state_manager=SimpleNamespace(can_allocate=True),
                     state_controller=controller, prefix_checkpoint_pool=SimpleNamespace(capacity=4))


def test_scheduler_promotes_a_shared_junction_for_the_next_request(page4):
    s = _hybrid_sched(_Controller())
    src = _seq([0, 1, 2, 3, 10, 11, 12, 13, 14])
    s.block_manager.allocate(src, 0)
    src.num_scheduled_tokens = 8
    s.block_manager.hash_blocks(src)
    tail = s.block_manager.prefix_metadata_at_boundary(src, 8)
    s.prefix_planner.publish(CaptureTicket(tail.prefix_hash, 8, tail.tail_block_id, 0, reason="prompt_tail"), 0)
    s.block_manager.deallocate(src)
    # B shares KV up to 4 tokens but has no GDN state there: it replays from 0 and captures at 4
    second = _seq([0, 1, 2, 3, 20, 21, 22, 23, 24])
    s.add(second)
    batch = s.schedule_prefill(64, 1)
    assert batch == [second] and second.num_cached_tokens == 0 and second.num_scheduled_tokens == 4
    pending, hashed = s.prepare_prefix_captures(batch, True)
    assert hashed and len(pending) == 1
    assert (pending[0].boundary_tokens, pending[0].reason, pending[0].replay_saved_tokens) == (4, "shared_junction", 4)
    s.publish_prefix_capture(pending[0], 1)
    s.postprocess(batch, [99], True, blocks_already_hashed=True)
    plan = s.prefix_planner.plan(_seq([0, 1, 2, 3, 30, 31, 32, 33, 34]))
    assert plan.hit is not None and plan.boundary_tokens == 4 and plan.promotion_candidate is None
    m = s.get_metrics()
    assert m["hybrid_prefix_shared_junction_promotions_published"] == 1 and m["hybrid_prefix_demand_entries"] == 0


def test_scheduler_splits_the_prefill_at_the_prompt_tail(page4):
    s = _hybrid_sched(_Controller(), hybrid_prefix_eviction_policy="lru", max_num_seqs=2)
    seq = _seq(range(27))
    s.add(seq)
    first = s.schedule_prefill(64, 1)
    assert first[0].num_scheduled_tokens == 16
    s.postprocess(first, [99], is_prefill=True)
    second = s.schedule_prefill(64, 1)
    assert second[0].num_scheduled_tokens == 8 and seq.num_cached_tokens + seq.num_scheduled_tokens == 24
    pending, hashed = s.prepare_prefix_captures(second, is_prefill=True)
    assert hashed and [(p.boundary_tokens, p.reason) for p in pending] == [(24, "prompt_tail")]


def test_internal_checkpoints_keep_one_prefill_and_list_its_boundaries(page4):
    s = _hybrid_sched(_Controller(), enable_hybrid_internal_checkpoints=True, hybrid_prefix_checkpoint_interval_blocks=1,
                      hybrid_prefix_retention_policy="periodic", max_num_seqs=2)
    seq = _seq(range(14))
    s.add(seq)
    batch = s.schedule_prefill(64, 1)
    assert batch[0].num_scheduled_tokens == 14          # no split at boundaries
    assert s.internal_prefix_boundaries(batch, True) == {seq.seq_id: (4, 8, 12)}
    pending, _ = s.prepare_prefix_captures(batch, True)
    assert [(p.boundary_tokens, p.internal_state) for p in pending] == [(4, True), (8, True), (12, True)]


def test_partial_page_cow_failure_rolls_back_pages_and_state(page4):
    Sequence.block_size = 8
    s = _hybrid_sched(_Controller(fail_on="copy_prefix_kv"), kvcache_block_size=8, prefix_match_unit=2,
                      num_kvcache_blocks=12, hybrid_prefix_checkpoint_interval_blocks=1,
                      hybrid_prefix_checkpoint_interval_tokens=2, hybrid_prefix_retention_policy="periodic",
                      hybrid_prefix_eviction_policy="lru", max_num_batched_tokens=32, max_num_seqs=2)
    src = _seq([0, 1, 2, 3, 4, 5, 80, 81, 82])
    s.block_manager.allocate(src, 0)
    src.num_scheduled_tokens = 8
    s.block_manager.hash_blocks(src)
    meta = s.block_manager.prefix_metadata_at_boundary(src, 6)
    s.prefix_planner.publish(CaptureTicket(meta.prefix_hash, 6, meta.tail_block_id, 0), 0)
    s.block_manager.deallocate(src)
    incoming = _seq([0, 1, 2, 3, 4, 5, 90, 91, 92])
    s.add(incoming)
    with pytest.raises(RuntimeError, match="injected copy_prefix_kv failure"):
        s.schedule_prefill(32, 1)
    assert incoming.block_table == [] and incoming.state_slot is None and incoming.num_cached_tokens == 0
    assert not s.block_manager.used_block_ids and int(s.block_manager.refs.sum()) == 0


# ------------------------------------------------------------------------ state pool
def _states(slots=2, dv=3, conv_dtype=torch.bfloat16):
    return HybridStateManager(max_num_seqs=slots, num_linear_layers=2, num_value_heads=2 if dv > 3 else 1,
                              key_head_dim=8 if dv > 3 else 2, value_head_dim=dv, conv_dim=4, conv_kernel_size=4,
                              conv_dtype=conv_dtype, device="cpu")


def test_checkpoint_capture_restore_free_isolation():
    sm = _states()
    pool = HybridPrefixCheckpointPool(sm, sm.bytes_per_slot() * 2)
    a, b = SimpleNamespace(state_slot=None), SimpleNamespace(state_slot=None)
    sa, sb = sm.allocate(a), sm.allocate(b)
    sm.recurrent_states[:, sa].fill_(3.5)
    sm.conv_states[:, sa].fill_(2.0)
    ck = pool.capture(sa)
    sm.recurrent_states[:, sb].fill_(99)
    sm.conv_states[:, sb].fill_(99)
    pool.restore(ck, sb)
    assert torch.equal(sm.recurrent_states[:, sb], sm.recurrent_states[:, sa])
    assert torch.equal(sm.conv_states[:, sb], sm.conv_states[:, sa])
    pool.free(ck)
    assert ck not in pool.used_checkpoint_slots
    assert not pool.recurrent.data[ck].any() and not pool.conv[ck].any()


@pytest.mark.parametrize("fmt", ["fp32", "bf16", "int8"])
def test_checkpoint_formats_round_trip(fmt):
    sm = _states(slots=1, dv=16)
    slot = sm.allocate(SimpleNamespace(state_slot=None))
    torch.manual_seed(7)
    rec = torch.randn_like(sm.recurrent_states[:, slot])
    conv = torch.randn_like(sm.conv_states[:, slot])
    sm.recurrent_states[:, slot] = rec
    sm.conv_states[:, slot] = conv
    pool = HybridPrefixCheckpointPool(sm, sm.bytes_per_slot() * 4, checkpoint_dtype=fmt)
    ck = pool.capture(slot)
    sm.clear_slot(slot)
    pool.restore(ck, slot)
    assert pool.recurrent.data.dtype == {"fp32": torch.float32, "bf16": torch.bfloat16, "int8": torch.int8}[fmt]
    assert pool.memory_bytes() == pool.capacity * pool.bytes_per_checkpoint
    assert torch.equal(sm.conv_states[:, slot], conv)
    got = sm.recurrent_states[:, slot]
    if fmt == "fp32":
        assert torch.equal(got, rec)
    elif fmt == "bf16":
        assert torch.equal(got, rec.to(torch.bfloat16).float())
    else:
        assert pool.recurrent.scales.shape[1:] == (2, 2, 8, 1)
        assert torch.all((got - rec).abs() <= pool.recurrent.scales[ck] / 2 + 1e-6)


def test_checkpoint_capacity_grows_as_the_format_shrinks():
    sm = _states(slots=1, dv=16)
    caps = {f: HybridPrefixCheckpointPool(sm, sm.bytes_per_slot() * 8, checkpoint_dtype=f).capacity
            for f in ("fp32", "bf16", "int8")}
    assert caps["fp32"] < caps["bf16"] < caps["int8"]


def test_int8_free_clears_values_scales_and_conv():
    sm = _states(slots=1)
    slot = sm.allocate(SimpleNamespace(state_slot=None))
    sm.conv_states[:, slot].fill_(3)
    pool = HybridPrefixCheckpointPool(sm, sm.bytes_per_slot(), checkpoint_dtype="int8")
    ck = pool.capture(slot)
    assert not pool.recurrent.data[ck].any() and torch.all(pool.recurrent.scales[ck] == 1e-8)
    pool.free(ck)
    assert not pool.recurrent.data[ck].any() and not pool.recurrent.scales[ck].any() and not pool.conv[ck].any()


def test_sparse_internal_states_are_captured_as_given():
    for fmt in ("fp32", "int8"):
        sm = _states(slots=1, dv=16)
        pool = HybridPrefixCheckpointPool(sm, sm.bytes_per_slot() * 2, checkpoint_dtype=fmt)
        rec = torch.randn(pool.recurrent_shape)
        conv = torch.randn(pool.conv_shape).to(torch.bfloat16)
        ck = pool.capture_tensors(rec, conv)
        slot = sm.allocate(SimpleNamespace(state_slot=None))
        pool.restore(ck, slot)
        assert torch.equal(sm.conv_states[:, slot], conv)
        tol = 0 if fmt == "fp32" else float(pool.recurrent.scales[ck].max())
        assert float((sm.recurrent_states[:, slot] - rec).abs().max()) <= tol
        with pytest.raises(ValueError):
            pool.capture_tensors(rec[:1], conv)
