"""Paged KV allocator with a unit-granular prefix index.

Behavioural parity with ``nanovllm/engine/block_manager.py:10-484``:
reference-counted 256-token pages; a freed page keeps its cached contents
until it is handed out again (lazy eviction), so a prefix stays reusable after
its producer finished; prefix reuse at ``prefix_match_unit`` granularity with a
partial-page copy-on-write plan when the reusable prefix ends inside a page;
speculative ``reserve_append`` / ``trim_to_sequence_length``; metrics under the
same names.

Design:
* ONE index for both granularities.  Keys are chained hashes of consecutive
  ``prefix_match_unit``-token units (``unit == block_size`` is the page-level
  cache); an entry records the unit's tokens (collision guard), the page holding
  its last token and how many tokens of that page are valid.  Page-aligned
  entries double as full-page hits, so there is no separate page table.
* Per-request hash chains are cached on the ``Sequence`` (``unit_hashes``) and
  only extended as tokens arrive, so probing a waiting request again costs a
  dictionary lookup per unit, not a rehash of its prompt.
* Free pages live in an insertion-ordered map: handing out the oldest free page
  first keeps recently freed (cached) pages around longest, and a cached free
  page that is reused by a prefix hit leaves the free map in O(1).
* Reference counts are a numpy array; the pages each index entry points at are
  tracked per page, so reassigning a page drops exactly its entries.
* Hashes are xxh3-64 of the unit's int64 token bytes seeded with the previous
  unit's hash.
"""

from __future__ import annotations

from collections import Counter, OrderedDict
from dataclasses import dataclass

import numpy as np
import xxhash

from inference_systems_b200.engine.sequence import Sequence

_SEED_MASK = (1 << 64) - 1


def chain_hash(token_ids, prev: int | None = None) -> int:
    """Hash of one unit of tokens chained to the hash of everything before it."""
    data = np.asarray(list(token_ids), dtype=np.int64).tobytes()
    return xxhash.xxh3_64_intdigest(data, seed=0 if prev is None else (prev + 1) & _SEED_MASK)


@dataclass(frozen=True, slots=True)
class PrefixIndexEntry:
    """One indexed unit: its chained hash, its tokens, the page holding its last token and how
    many tokens of that page (from its start) are valid up to the unit's end."""

    prefix_hash: int
    unit_token_ids: tuple[int, ...]
    tail_block_id: int
    tail_valid_tokens: int


@dataclass(frozen=True, slots=True)
class KVPageCopy:
    """Copy-on-write plan: the first ``num_tokens`` rows of page ``source_block_id`` go to
    ``destination_block_id`` before the request writes the rest of that page."""

    source_block_id: int
    destination_block_id: int
    num_tokens: int


@dataclass(frozen=True, slots=True)
class PrefixKVCandidate:
    """A reusable KV prefix of a request: ``boundary_tokens`` tokens, of which the first
    ``num_cached_blocks`` pages are shared whole and, when ``tail_valid_tokens`` is less than a
    page, the rest comes from copying that many rows of ``tail_block_id``."""

    num_cached_blocks: int
    boundary_tokens: int
    prefix_hash: int
    tail_block_id: int
    tail_valid_tokens: int = 0


class _FreePages:
    """Free page ids in release order (oldest first), with O(1) removal of any page."""

    def __init__(self, n: int):
        self._order: OrderedDict[int, None] = OrderedDict((i, None) for i in range(n))

    def __len__(self) -> int:
        return len(self._order)

    def __contains__(self, page: int) -> bool:
        return page in self._order

    def pop_oldest(self) -> int:
        if not self._order:
            raise RuntimeError("no free KV blocks")
        return self._order.popitem(last=False)[0]

    def take(self, page: int) -> None:
        del self._order[page]

    def release(self, page: int) -> None:
        self._order[page] = None


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int, prefix_match_unit: int | None = None):
        if num_blocks <= 0 or block_size <= 0:
            raise ValueError("block count and size must be positive")
        self.block_size = block_size
        self.prefix_match_unit = prefix_match_unit or block_size
        if self.prefix_match_unit <= 0 or block_size % self.prefix_match_unit:
            raise ValueError("prefix_match_unit must divide block_size")
        self.num_blocks = num_blocks
        self.refs = np.zeros(num_blocks, dtype=np.int32)
        self.free = _FreePages(num_blocks)
        self.index: dict[int, PrefixIndexEntry] = {}
        # unit hashes whose entry was registered on each page (stale ones are skipped on reuse)
        self.page_units: list[set[int]] = [set() for _ in range(num_blocks)]
        # page-aligned unit hash last registered on each page: the page "holds a cached block"
        self.page_hash: list[int | None] = [None] * num_blocks
        self.reset_metrics()

    # ------------------------------------------------------------------ metrics
    def reset_metrics(self) -> None:
        self.stats: Counter = Counter()

    @property
    def prefix_cache_evictions(self) -> int:
        return self.stats["prefix_cache_evictions"]

    @property
    def cached_block_reassignments(self) -> int:
        return self.stats["cached_block_reassignments"]

    @property
    def duplicate_cache_registrations(self) -> int:
        return self.stats["duplicate_cache_registrations"]

    @property
    def partial_prefix_cow_allocations(self) -> int:
        return self.stats["partial_prefix_cow_allocations"]

    @property
    def fine_grained(self) -> bool:
        return self.prefix_match_unit < self.block_size

    @property
    def num_free_blocks(self) -> int:
        return len(self.free)

    @property
    def num_used_blocks(self) -> int:
        return self.num_blocks - len(self.free)

    @property
    def used_block_ids(self) -> frozenset[int]:
        return frozenset(int(i) for i in np.flatnonzero(self.refs > 0))

    def ref_count(self, page: int) -> int:
        return int(self.refs[page])

    @property
    def num_cached_blocks(self) -> int:
        """Pages (free or in use) that still hold a registered full-page unit."""
        return sum(h is not None for h in self.page_hash)

    @property
    def num_reachable_cached_blocks(self) -> int:
        """Pages that an index lookup can still reach."""
        if self.fine_grained:
            return len({e.tail_block_id for e in self.index.values()})
        return sum(1 for p, h in enumerate(self.page_hash)
                   if h is not None and (e := self.index.get(h)) is not None and e.tail_block_id == p)

    def metrics(self) -> dict:
        return {"prefix_cache_evictions": self.prefix_cache_evictions,
                "cached_block_reassignments": self.cached_block_reassignments,
                "duplicate_cache_registrations": self.duplicate_cache_registrations,
                "partial_prefix_cow_allocations": self.partial_prefix_cow_allocations,
                "cached_blocks": self.num_cached_blocks}

    # ------------------------------------------------------------------- pages
    def _fresh_page(self) -> int:
        """Hand out the oldest free page, dropping whatever the index still knew about it."""
        page = self.free.pop_oldest()
        if self.page_units[page] or self.page_hash[page] is not None:
            self.stats["cached_block_reassignments"] += 1
            for h in self.page_units[page]:
                e = self.index.get(h)
                if e is not None and e.tail_block_id == page:
                    del self.index[h]
                    self.stats["prefix_cache_evictions"] += 1
            self.page_units[page].clear()
            self.page_hash[page] = None
        self.refs[page] = 1
        return page

    def _share(self, page: int) -> None:
        """One more reference to a cached page (revived from the free map if unreferenced)."""
        if self.refs[page] == 0:
            self.free.take(page)
        self.refs[page] += 1

    def _drop(self, page: int) -> None:
        self.refs[page] -= 1
        if self.refs[page] == 0:
            self.free.release(page)
        elif self.refs[page] < 0:
            raise RuntimeError(f"page {page} released more often than referenced")

    # ----------------------------------------------------------------- hashing
    def _units(self, seq: Sequence, n_units: int) -> list[int]:
        """The first ``n_units`` chained unit hashes of ``seq`` (cached on the request)."""
        u = self.prefix_match_unit
        chain = seq.unit_hashes.setdefault(u, [])
        while len(chain) < n_units:
            k = len(chain)
            chain.append(chain_hash(seq.token_ids[k * u:(k + 1) * u], chain[-1] if chain else None))
        return chain[:n_units]

    def _lookup(self, seq: Sequence, k: int, h: int) -> PrefixIndexEntry | None:
        u = self.prefix_match_unit
        e = self.index.get(h)
        if e is None or list(e.unit_token_ids) != seq.token_ids[k * u:(k + 1) * u]:
            return None
        return e

    def _reusable_units(self, seq: Sequence) -> list[PrefixIndexEntry]:
        """Indexed units along ``seq``'s chain, leaving at least one token to compute."""
        u = self.prefix_match_unit
        limit = (seq.num_tokens - 1) // u
        out = []
        for k, h in enumerate(self._units(seq, limit)):
            e = self._lookup(seq, k, h)
            if e is None:
                break
            out.append(e)
        return out

    def _full_page_chain(self, seq: Sequence, pages: int) -> list[int]:
        """Page ids of the first ``pages`` whole pages along ``seq``'s indexed chain."""
        per = self.block_size // self.prefix_match_unit
        hashes = self._units(seq, pages * per)
        return [self.index[hashes[(p + 1) * per - 1]].tail_block_id for p in range(pages)]

    def hash_blocks(self, seq: Sequence) -> None:
        """Index the units completed by the scheduled chunk of ``seq``."""
        u, bs = self.prefix_match_unit, self.block_size
        first = seq.num_cached_tokens // u
        done = (seq.num_cached_tokens + seq.num_scheduled_tokens) // u
        if done <= first:
            return
        hashes = self._units(seq, done)
        for k in range(first, done):
            end = (k + 1) * u
            page = seq.block_table[(end - 1) // bs]
            h = hashes[k]
            prev = self.index.get(h)
            toks = tuple(seq.token_ids[k * u:end])
            if prev is not None and prev.tail_block_id != page and prev.unit_token_ids == toks:
                self.stats["duplicate_cache_registrations"] += 1
            self.index[h] = PrefixIndexEntry(h, toks, page, end % bs or bs)
            self.page_units[page].add(h)
            if end % bs == 0:
                self.page_hash[page] = h

    # ------------------------------------------------------------------ probes
    def can_allocate(self, seq: Sequence, use_prefix_cache: bool = True) -> int:
        """Whole cached pages ``seq`` would reuse, or -1 when free pages are short."""
        if not use_prefix_cache:
            return 0 if len(self.free) >= seq.num_blocks else -1
        per = self.block_size // self.prefix_match_unit
        pages = len(self._reusable_units(seq)) // per
        need = seq.num_blocks - sum(self.refs[p] > 0 for p in self._full_page_chain(seq, pages))
        return pages if len(self.free) >= need else -1

    def find_prefix_candidates(self, seq: Sequence) -> list[PrefixKVCandidate]:
        """Every reusable prefix boundary of ``seq``, longest first."""
        u, bs = self.prefix_match_unit, self.block_size
        out = []
        for k, e in enumerate(self._reusable_units(seq)):
            end = (k + 1) * u
            out.append(PrefixKVCandidate(end // bs, end, e.prefix_hash, e.tail_block_id, e.tail_valid_tokens))
        out.reverse()
        return out

    def _pages_needed(self, seq: Sequence, candidate: PrefixKVCandidate | None) -> int:
        if candidate is None:
            return seq.num_blocks
        need = seq.num_blocks - sum(self.refs[p] > 0 for p in self._full_page_chain(seq, candidate.num_cached_blocks))
        if candidate.tail_valid_tokens != self.block_size and self.refs[candidate.tail_block_id] == 0:
            need += 1  # the copy source must stay pinned (out of the free map) until it is copied
        return need

    def can_allocate_candidate(self, seq: Sequence, candidate: PrefixKVCandidate | None) -> bool:
        return len(self.free) >= self._pages_needed(seq, candidate)

    def can_allocate_with_prefix(self, seq: Sequence, num_cached_blocks: int) -> bool:
        if not 0 <= num_cached_blocks < seq.num_blocks:
            raise ValueError("invalid cached block count")
        cand = None
        if num_cached_blocks:
            cand = next((c for c in self.find_prefix_candidates(seq) if c.num_cached_blocks == num_cached_blocks
                         and c.tail_valid_tokens == self.block_size), None)
            if cand is None:
                return False
        return self.can_allocate_candidate(seq, cand)

    def prefix_metadata_at_boundary(self, seq: Sequence, boundary_tokens: int) -> PrefixKVCandidate:
        """The index entry of ``seq``'s prefix ending at ``boundary_tokens`` (must be indexed)."""
        u, bs = self.prefix_match_unit, self.block_size
        if boundary_tokens <= 0 or boundary_tokens % u:
            raise ValueError("prefix boundary must align to prefix_match_unit")
        page_idx = (boundary_tokens - 1) // bs
        if page_idx >= len(seq.block_table):
            raise ValueError("prefix boundary has no allocated block")
        page = seq.block_table[page_idx]
        k = boundary_tokens // u - 1
        h = self._units(seq, k + 1)[k]
        e = self._lookup(seq, k, h)
        if e is None or e.tail_block_id != page:
            raise ValueError("prefix boundary has not been indexed")
        return PrefixKVCandidate(boundary_tokens // bs, boundary_tokens, h, page, e.tail_valid_tokens)

    def reclaimable_blocks(self, seq: Sequence) -> int:
        """Pages that preempting ``seq`` would free (those it does not share)."""
        return sum(self.refs[p] == 1 for p in set(seq.block_table))

    # -------------------------------------------------------------- allocation
    def allocate(self, seq: Sequence, num_cached_blocks: int) -> None:
        if seq.block_table:
            raise RuntimeError("sequence already holds pages")
        shared = self._full_page_chain(seq, num_cached_blocks)
        for p in shared:
            self._share(p)
        seq.block_table.extend(shared)
        while len(seq.block_table) < seq.num_blocks:
            seq.block_table.append(self._fresh_page())
        seq.num_cached_tokens = num_cached_blocks * self.block_size

    def allocate_candidate(self, seq: Sequence, candidate: PrefixKVCandidate | None) -> KVPageCopy | None:
        """Pages for ``seq`` reusing ``candidate``; a boundary inside a page pins that page and
        returns the copy plan (release it with ``release_cow_source`` once copied)."""
        if candidate is None:
            self.allocate(seq, 0)
            return None
        if seq.block_table:
            raise RuntimeError("sequence already holds pages")
        partial = candidate.tail_valid_tokens != self.block_size
        pinned = False
        try:
            for p in self._full_page_chain(seq, candidate.num_cached_blocks):
                self._share(p)
                seq.block_table.append(p)
            if partial:
                self._share(candidate.tail_block_id)
                pinned = True
            while len(seq.block_table) < seq.num_blocks:
                seq.block_table.append(self._fresh_page())
        except Exception:
            if pinned:
                self._drop(candidate.tail_block_id)
            self.deallocate(seq)
            raise
        seq.num_cached_tokens = candidate.boundary_tokens
        if not partial:
            return None
        self.stats["partial_prefix_cow_allocations"] += 1
        return KVPageCopy(candidate.tail_block_id, seq.block_table[candidate.num_cached_blocks],
                          candidate.tail_valid_tokens)

    def release_cow_source(self, page_copy: KVPageCopy) -> None:
        self._drop(page_copy.source_block_id)

    def deallocate(self, seq: Sequence) -> None:
        for p in reversed(seq.block_table):
            self._drop(p)
        seq.block_table.clear()
        seq.num_cached_tokens = 0

    # ------------------------------------------------------------------ growth
    def can_append(self, seq: Sequence) -> bool:
        """Room for the token just appended (a new page when it starts one)."""
        return len(self.free) >= (1 if len(seq) % self.block_size == 1 else 0)

    def may_append(self, seq: Sequence) -> None:
        if len(seq) % self.block_size == 1:
            seq.block_table.append(self._fresh_page())

    def additional_blocks_for_append(self, seq: Sequence, num_tokens: int) -> int:
        if num_tokens < 0:
            raise ValueError("num_tokens must be non-negative")
        return max(-(-(len(seq) + num_tokens) // self.block_size) - len(seq.block_table), 0)

    def can_reserve_append(self, seq: Sequence, num_tokens: int) -> bool:
        return len(self.free) >= self.additional_blocks_for_append(seq, num_tokens)

    def reserve_append(self, seq: Sequence, num_tokens: int) -> None:
        need = self.additional_blocks_for_append(seq, num_tokens)
        if len(self.free) < need:
            raise RuntimeError("insufficient KV blocks for speculative append")
        for _ in range(need):
            seq.block_table.append(self._fresh_page())

    def trim_to_sequence_length(self, seq: Sequence) -> None:
        """Give back speculative pages beyond the sequence's committed length."""
        while len(seq.block_table) > seq.num_blocks:
            p = seq.block_table.pop()
            if self.refs[p] != 1:
                raise RuntimeError("speculative tail block is unexpectedly shared")
            self._drop(p)
