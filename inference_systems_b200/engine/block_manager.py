"""Paged-KV block allocator with a chained-hash prefix index.

Parity: ``nanovllm/engine/block_manager.py:10-484`` -- ref-counted pages and a
free deque; xxhash64 chained block hashes; a fine-grained prefix index at
``prefix_match_unit`` granularity whose entries name the page that holds the
unit's last token (``tail_block_id``) and how many tokens of that page are
valid; partial-page copy-on-write plans (``KVPageCopy``); speculative
``reserve_append`` / ``trim_to_sequence_length``; ``reclaimable_blocks``.

The cached page of a freed block stays indexed until the block is handed out
again (lazy eviction), exactly like the reference, so a prefix can be reused
after its producer finished.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass

import numpy as np
import xxhash

from inference_systems_b200.engine.hybrid_prefix_cache import PrefixKVCandidate
from inference_systems_b200.engine.sequence import Sequence


@dataclass(frozen=True, slots=True)
class PrefixIndexEntry:
    prefix_hash: int
    unit_token_ids: tuple[int, ...]
    tail_block_id: int
    tail_valid_tokens: int


@dataclass(frozen=True, slots=True)
class KVPageCopy:
    source_block_id: int
    destination_block_id: int
    num_tokens: int


class Block:
    __slots__ = ("block_id", "ref_count", "hash", "token_ids", "prefix_hashes")

    def __init__(self, block_id: int):
        self.block_id = block_id
        self.ref_count = 0
        self.hash = -1
        self.token_ids: list[int] = []
        self.prefix_hashes: set[int] = set()

    def update(self, h: int, token_ids: list[int]) -> None:
        self.hash = h
        self.token_ids = list(token_ids)

    def reset(self) -> None:
        self.ref_count = 1
        self.hash = -1
        self.token_ids = []
        self.prefix_hashes.clear()


def chain_hash(token_ids, prefix: int = -1) -> int:
    h = xxhash.xxh64()
    if prefix != -1:
        h.update(prefix.to_bytes(8, "little"))
    h.update(np.asarray(list(token_ids), dtype=np.int64).tobytes())
    return h.intdigest()


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int, prefix_match_unit: int | None = None):
        self.block_size = block_size
        self.prefix_match_unit = prefix_match_unit or block_size
        if self.prefix_match_unit <= 0 or block_size % self.prefix_match_unit:
            raise ValueError("prefix_match_unit must divide block_size")
        self.blocks = [Block(i) for i in range(num_blocks)]
        self.hash_to_block_id: dict[int, int] = {}
        self.hash_to_prefix_entry: dict[int, PrefixIndexEntry] = {}
        self.free_block_ids: deque[int] = deque(range(num_blocks))
        self.used_block_ids: set[int] = set()
        self.reset_metrics()

    compute_hash = staticmethod(chain_hash)

    @property
    def fine_grained(self) -> bool:
        return self.prefix_match_unit < self.block_size

    def reset_metrics(self) -> None:
        self.prefix_cache_evictions = 0
        self.cached_block_reassignments = 0
        self.duplicate_cache_registrations = 0
        self.partial_prefix_cow_allocations = 0

    # ------------------------------------------------------- raw pages
    def _allocate_block(self) -> int:
        block_id = self.free_block_ids.popleft()
        block = self.blocks[block_id]
        assert block.ref_count == 0
        if block.hash != -1:
            self.cached_block_reassignments += 1
            if self.hash_to_block_id.get(block.hash) == block_id:
                del self.hash_to_block_id[block.hash]
                self.prefix_cache_evictions += 1
        for ph in tuple(block.prefix_hashes):
            entry = self.hash_to_prefix_entry.get(ph)
            if entry is not None and entry.tail_block_id == block_id:
                del self.hash_to_prefix_entry[ph]
                self.prefix_cache_evictions += 1
        block.reset()
        self.used_block_ids.add(block_id)
        return block_id

    def _deallocate_block(self, block_id: int) -> None:
        assert self.blocks[block_id].ref_count == 0
        self.used_block_ids.remove(block_id)
        self.free_block_ids.append(block_id)

    def _reference_block(self, block_id: int) -> None:
        block = self.blocks[block_id]
        if block_id in self.used_block_ids:
            block.ref_count += 1
        else:
            block.ref_count = 1
            self.free_block_ids.remove(block_id)
            self.used_block_ids.add(block_id)

    def _release_block(self, block_id: int) -> None:
        block = self.blocks[block_id]
        block.ref_count -= 1
        if block.ref_count == 0:
            self._deallocate_block(block_id)

    # ------------------------------------------------- prefix lookup
    def _full_block_prefix(self, seq: Sequence):
        """Yield ``(block_index, hash, block_id)`` along the cached full-block chain."""
        h = -1
        for i in range(seq.num_blocks - 1):
            tokens = seq.block(i)
            h = chain_hash(tokens, h)
            bid = self.hash_to_block_id.get(h, -1)
            if bid == -1 or self.blocks[bid].token_ids != tokens:
                return
            yield i, h, bid

    def can_allocate(self, seq: Sequence, use_prefix_cache: bool = True) -> int:
        """Cached full blocks reusable by ``seq`` or -1 if pages are short."""
        if not use_prefix_cache:
            return 0 if len(self.free_block_ids) >= seq.num_blocks else -1
        cached, new = 0, seq.num_blocks
        for _, _, bid in self._full_block_prefix(seq):
            cached += 1
            if bid in self.used_block_ids:
                new -= 1
        return cached if len(self.free_block_ids) >= new else -1

    def find_prefix_candidates(self, seq: Sequence) -> list[PrefixKVCandidate]:
        """All reusable prefix boundaries, longest first (one unit is always left to compute)."""
        if self.fine_grained:
            return self._find_fine_candidates(seq)
        out = [PrefixKVCandidate(num_cached_blocks=i + 1, boundary_tokens=(i + 1) * self.block_size,
                                 prefix_hash=h, tail_block_id=bid, tail_valid_tokens=self.block_size)
               for i, h, bid in self._full_block_prefix(seq)]
        out.reverse()
        return out

    def _find_fine_candidates(self, seq: Sequence) -> list[PrefixKVCandidate]:
        unit = self.prefix_match_unit
        limit = ((seq.num_tokens - 1) // unit) * unit
        h = -1
        out = []
        for start in range(0, limit, unit):
            end = start + unit
            toks = tuple(seq.token_ids[start:end])
            h = chain_hash(toks, h)
            entry = self.hash_to_prefix_entry.get(h)
            if entry is None or entry.unit_token_ids != toks:
                break
            out.append(PrefixKVCandidate(num_cached_blocks=end // self.block_size, boundary_tokens=end,
                                         prefix_hash=h, tail_block_id=entry.tail_block_id,
                                         tail_valid_tokens=end % self.block_size or self.block_size))
        out.reverse()
        return out

    def _full_prefix_block_ids(self, seq: Sequence, num_full_blocks: int) -> list[int]:
        if not self.fine_grained:
            ids, h = [], -1
            for i in range(num_full_blocks):
                h = chain_hash(seq.block(i), h)
                ids.append(self.hash_to_block_id[h])
            return ids
        unit = self.prefix_match_unit
        per_block = self.block_size // unit
        ids, h = [], -1
        for u in range(num_full_blocks * per_block):
            h = chain_hash(seq.token_ids[u * unit:(u + 1) * unit], h)
            if (u + 1) % per_block == 0:
                ids.append(self.hash_to_prefix_entry[h].tail_block_id)
        return ids

    def can_allocate_with_prefix(self, seq: Sequence, num_cached_blocks: int) -> bool:
        if num_cached_blocks < 0 or num_cached_blocks >= seq.num_blocks:
            raise ValueError("invalid cached block count")
        if num_cached_blocks and not any(c.num_cached_blocks == num_cached_blocks
                                         for c in self.find_prefix_candidates(seq)):
            return False
        need = seq.num_blocks
        h = -1
        for i in range(num_cached_blocks):
            h = chain_hash(seq.block(i), h)
            if self.hash_to_block_id[h] in self.used_block_ids:
                need -= 1
        return len(self.free_block_ids) >= need

    def can_allocate_candidate(self, seq: Sequence, candidate: PrefixKVCandidate | None) -> bool:
        if candidate is None:
            return len(self.free_block_ids) >= seq.num_blocks
        need = seq.num_blocks
        for bid in self._full_prefix_block_ids(seq, candidate.num_cached_blocks):
            if bid in self.used_block_ids:
                need -= 1
        partial = candidate.tail_valid_tokens != self.block_size
        if partial and candidate.tail_block_id not in self.used_block_ids:
            need += 1  # the COW source must stay pinned until its rows are copied
        return len(self.free_block_ids) >= need

    # ------------------------------------------------------ allocation
    def allocate_candidate(self, seq: Sequence, candidate: PrefixKVCandidate | None) -> KVPageCopy | None:
        """Allocate pages for ``seq``; pin and return a COW plan for a partial tail page."""
        assert not seq.block_table
        if candidate is None:
            self.allocate(seq, 0)
            return None
        full_ids = self._full_prefix_block_ids(seq, candidate.num_cached_blocks)
        partial = candidate.tail_valid_tokens != self.block_size
        pinned = False
        try:
            for bid in full_ids:
                self._reference_block(bid)
                seq.block_table.append(bid)
            if partial:
                self._reference_block(candidate.tail_block_id)
                pinned = True
            while len(seq.block_table) < seq.num_blocks:
                seq.block_table.append(self._allocate_block())
            seq.num_cached_tokens = candidate.boundary_tokens
            if not partial:
                return None
            self.partial_prefix_cow_allocations += 1
            return KVPageCopy(candidate.tail_block_id, seq.block_table[candidate.num_cached_blocks],
                              candidate.tail_valid_tokens)
        except Exception:
            if pinned:
                self._release_block(candidate.tail_block_id)
            self.deallocate(seq)
            raise

    def release_cow_source(self, page_copy: KVPageCopy) -> None:
        self._release_block(page_copy.source_block_id)

    def prefix_metadata_at_boundary(self, seq: Sequence, boundary_tokens: int) -> PrefixKVCandidate:
        if boundary_tokens <= 0 or boundary_tokens % self.prefix_match_unit:
            raise ValueError("prefix boundary must align to prefix_match_unit")
        bidx = (boundary_tokens - 1) // self.block_size
        if bidx >= len(seq.block_table):
            raise ValueError("prefix boundary has no allocated block")
        bid = seq.block_table[bidx]
        if self.fine_grained:
            h = -1
            for s in range(0, boundary_tokens, self.prefix_match_unit):
                h = chain_hash(seq.token_ids[s:s + self.prefix_match_unit], h)
            entry = self.hash_to_prefix_entry.get(h)
            if entry is None or entry.tail_block_id != bid:
                raise ValueError("prefix boundary has not been indexed")
            return PrefixKVCandidate(boundary_tokens // self.block_size, boundary_tokens, h, bid,
                                     boundary_tokens % self.block_size or self.block_size)
        block = self.blocks[bid]
        if block.hash == -1:
            raise ValueError("prefix boundary block has not been hashed")
        return PrefixKVCandidate(bidx + 1, boundary_tokens, block.hash, bid, self.block_size)

    def allocate(self, seq: Sequence, num_cached_blocks: int) -> None:
        assert not seq.block_table
        h = -1
        for i in range(num_cached_blocks):
            h = chain_hash(seq.block(i), h)
            bid = self.hash_to_block_id[h]
            self._reference_block(bid)
            seq.block_table.append(bid)
        for _ in range(num_cached_blocks, seq.num_blocks):
            seq.block_table.append(self._allocate_block())
        seq.num_cached_tokens = num_cached_blocks * self.block_size

    def deallocate(self, seq: Sequence) -> None:
        for bid in reversed(seq.block_table):
            self._release_block(bid)
        seq.num_cached_tokens = 0
        seq.block_table.clear()

    def reclaimable_blocks(self, seq: Sequence) -> int:
        return sum(self.blocks[b].ref_count == 1 for b in set(seq.block_table))

    def can_append(self, seq: Sequence) -> bool:
        return len(self.free_block_ids) >= (len(seq) % self.block_size == 1)

    def may_append(self, seq: Sequence) -> None:
        if len(seq) % self.block_size == 1:
            seq.block_table.append(self._allocate_block())

    def additional_blocks_for_append(self, seq: Sequence, num_tokens: int) -> int:
        if num_tokens < 0:
            raise ValueError("num_tokens must be non-negative")
        final = (len(seq) + num_tokens + self.block_size - 1) // self.block_size
        return max(final - len(seq.block_table), 0)

    def can_reserve_append(self, seq: Sequence, num_tokens: int) -> bool:
        return len(self.free_block_ids) >= self.additional_blocks_for_append(seq, num_tokens)

    def reserve_append(self, seq: Sequence, num_tokens: int) -> None:
        need = self.additional_blocks_for_append(seq, num_tokens)
        if len(self.free_block_ids) < need:
            raise RuntimeError("insufficient KV blocks for speculative append")
        for _ in range(need):
            seq.block_table.append(self._allocate_block())

    def trim_to_sequence_length(self, seq: Sequence) -> None:
        while len(seq.block_table) > seq.num_blocks:
            bid = seq.block_table.pop()
            block = self.blocks[bid]
            block.ref_count -= 1
            if block.ref_count != 0:
                raise RuntimeError("speculative tail block is unexpectedly shared")
            self._deallocate_block(bid)

    # --------------------------------------------------------- hashing
    def hash_blocks(self, seq: Sequence) -> None:
        """Index the pages completed by the scheduled chunk of ``seq``."""
        if self.fine_grained:
            self._hash_units(seq)
            return
        start = seq.num_cached_tokens // self.block_size
        end = (seq.num_cached_tokens + seq.num_scheduled_tokens) // self.block_size
        if start == end:
            return
        h = self.blocks[seq.block_table[start - 1]].hash if start > 0 else -1
        for i in range(start, end):
            block = self.blocks[seq.block_table[i]]
            tokens = seq.block(i)
            h = chain_hash(tokens, h)
            prev = self.hash_to_block_id.get(h)
            if prev is not None and prev != block.block_id and self.blocks[prev].token_ids == tokens:
                self.duplicate_cache_registrations += 1
            block.update(h, tokens)
            self.hash_to_block_id[h] = block.block_id

    def _hash_units(self, seq: Sequence) -> None:
        unit = self.prefix_match_unit
        done = (seq.num_cached_tokens + seq.num_scheduled_tokens) // unit
        first_new = seq.num_cached_tokens // unit
        h = -1
        for u in range(done):
            s, e = u * unit, (u + 1) * unit
            toks = tuple(seq.token_ids[s:e])
            h = chain_hash(toks, h)
            if u < first_new:
                continue
            bidx = (e - 1) // self.block_size
            bid = seq.block_table[bidx]
            entry = PrefixIndexEntry(h, toks, bid, e % self.block_size or self.block_size)
            prev = self.hash_to_prefix_entry.get(h)
            if prev is not None and prev.tail_block_id != bid:
                self.duplicate_cache_registrations += 1
            self.hash_to_prefix_entry[h] = entry
            self.blocks[bid].prefix_hashes.add(h)
            if e % self.block_size == 0:
                self.blocks[bid].update(h, seq.block(bidx))
                self.hash_to_block_id[h] = bid

    @property
    def num_cached_blocks(self) -> int:
        return sum(b.hash != -1 for b in self.blocks)

    @property
    def num_reachable_cached_blocks(self) -> int:
        if self.fine_grained:
            return len({e.tail_block_id for e in self.hash_to_prefix_entry.values()})
        return len(set(self.hash_to_block_id.values()))
