"""Paged-KV allocator semantics (parity with the reference's tests/test_block_manager.py behaviour)."""

import pytest

from inference_systems_b200.engine.block_manager import BlockManager
from inference_systems_b200.engine.sequence import Sequence
from inference_systems_b200.sampling_params import SamplingParams


@pytest.fixture(autouse=True)
def _block_size():
    old = Sequence.block_size
    Sequence.block_size = 256
    yield
    Sequence.block_size = old


def seq(tokens):
    return Sequence(list(tokens), SamplingParams(max_tokens=4))


def finish_prefill(bm, s):
    s.num_scheduled_tokens = s.num_tokens - s.num_cached_tokens
    bm.hash_blocks(s)
    s.num_cached_tokens += s.num_scheduled_tokens
    s.num_scheduled_tokens = 0


def test_allocate_and_free_roundtrip():
    bm = BlockManager(8, 256)
    s = seq(range(600))
    assert bm.can_allocate(s) == 0
    bm.allocate(s, 0)
    assert len(s.block_table) == 3 and bm.num_free_blocks == 5
    bm.deallocate(s)
    assert bm.num_free_blocks == 8 and not s.block_table


def test_full_block_prefix_hit_reuses_pages():
    bm = BlockManager(8, 256)
    a = seq(list(range(600)))
    bm.allocate(a, 0)
    finish_prefill(bm, a)
    b = seq(list(range(512)) + [9999] * 40)
    cached = bm.can_allocate(b)
    assert cached == 2
    bm.allocate(b, cached)
    assert b.block_table[:2] == a.block_table[:2]
    assert b.num_cached_tokens == 512
    assert bm.ref_count(a.block_table[0]) == 2


def test_freed_cached_pages_stay_reusable_until_reassigned():
    bm = BlockManager(4, 256)
    a = seq(list(range(300)))
    bm.allocate(a, 0)
    finish_prefill(bm, a)
    first = a.block_table[0]
    bm.deallocate(a)
    b = seq(list(range(256)) + [7] * 10)
    assert bm.can_allocate(b) == 1
    bm.allocate(b, 1)
    assert b.block_table[0] == first


def test_fine_grained_candidates_and_partial_cow():
    bm = BlockManager(8, 256, prefix_match_unit=16)
    a = seq(list(range(300)))
    bm.allocate(a, 0)
    finish_prefill(bm, a)
    # shares 288 tokens (18 units) with a, then diverges
    b = seq(list(range(288)) + [5000 + i for i in range(50)])
    cands = bm.find_prefix_candidates(b)
    assert cands[0].boundary_tokens == 288
    assert cands[0].tail_valid_tokens == 288 - 256
    assert cands[-1].boundary_tokens == 16
    assert bm.can_allocate_candidate(b, cands[0])
    cow = bm.allocate_candidate(b, cands[0])
    assert cow is not None and cow.num_tokens == 32
    assert cow.source_block_id == a.block_table[1]
    assert cow.destination_block_id == b.block_table[1] != a.block_table[1]
    assert b.block_table[0] == a.block_table[0]
    assert b.num_cached_tokens == 288
    bm.release_cow_source(cow)


def test_fine_grained_keeps_one_unit_uncached():
    bm = BlockManager(8, 256, prefix_match_unit=16)
    a = seq(list(range(64)))
    bm.allocate(a, 0)
    finish_prefill(bm, a)
    same = seq(list(range(64)))
    # the final unit must be recomputed so prefill produces logits
    assert max(c.boundary_tokens for c in bm.find_prefix_candidates(same)) == 48


def test_reserve_append_and_trim():
    bm = BlockManager(8, 256)
    s = seq(range(255))
    bm.allocate(s, 0)
    assert bm.additional_blocks_for_append(s, 4) == 1
    bm.reserve_append(s, 4)
    assert len(s.block_table) == 2
    bm.trim_to_sequence_length(s)
    assert len(s.block_table) == 1


def test_can_append_boundary():
    bm = BlockManager(1, 256)
    s = seq(range(256))
    bm.allocate(s, 0)
    s.append_token(1)
    assert len(s) == 257 and not bm.can_append(s)


def test_reclaimable_blocks_counts_unshared():
    bm = BlockManager(8, 256)
    a = seq(range(600))
    bm.allocate(a, 0)
    finish_prefill(bm, a)
    b = seq(list(range(512)) + [1] * 5)
    bm.allocate(b, bm.can_allocate(b))
    assert bm.reclaimable_blocks(a) == 1
    assert bm.reclaimable_blocks(b) == 1
