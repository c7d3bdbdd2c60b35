"""Control plane of the hybrid (KV + GDN-state) prefix cache.

A prefix of a hybrid model is only reusable where BOTH the paged KV of the
attention layers and a GDN recurrent/conv checkpoint exist at the same token
boundary.  Parity: ``nanovllm/engine/hybrid_prefix_cache.py:8-680``:

* ``HybridCheckpointRetentionPolicy`` -- which boundaries get a checkpoint
  (``periodic`` every ``interval_tokens``; ``adaptive`` also the last full unit
  before the prompt tail).
* ``GDNCheckpointManager`` -- bounded index ``(prefix_hash, boundary) -> slot``
  with LRU or cost-aware (``retained_value``) eviction and hit metrics.
* ``FullAttentionPrefixManager`` -- typed view over ``BlockManager``.
* ``HybridPrefixCoordinator`` -- longest boundary present in both; records
  KV-only misses and, in adaptive mode, promotes a "shared junction" after
  ``promotion_min_sightings`` sightings; ``probe`` is side-effect free.
"""

from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass
from time import perf_counter_ns


@dataclass(frozen=True, slots=True)
class PrefixKVCandidate:
    num_cached_blocks: int
    boundary_tokens: int
    prefix_hash: int
    tail_block_id: int
    tail_valid_tokens: int = 0


@dataclass(frozen=True, slots=True)
class HybridPrefixHit:
    candidate: PrefixKVCandidate
    checkpoint_slot: int


@dataclass(frozen=True, slots=True)
class HybridPrefixAllocationPlan:
    hit: HybridPrefixHit | None
    num_cached_blocks: int
    kv_candidate_tokens: int = 0
    promotion_candidate: PrefixKVCandidate | None = None

    @property
    def boundary_tokens(self) -> int:
        return self.hit.candidate.boundary_tokens if self.hit is not None else 0

    @property
    def candidate(self) -> PrefixKVCandidate | None:
        return self.hit.candidate if self.hit is not None else None


@dataclass(frozen=True, slots=True)
class PendingHybridPrefixCapture:
    prefix_hash: int
    boundary_tokens: int
    tail_block_id: int
    state_slot: int
    reason: str = "periodic"
    internal_state: bool = False
    sequence_id: int = -1
    replay_saved_tokens: int = 0
    demand_count: int = 0


@dataclass(slots=True)
class HybridPrefixEntry:
    prefix_hash: int
    boundary_tokens: int
    tail_block_id: int
    checkpoint_slot: int
    last_access_ns: int
    reason: str
    hit_count: int = 0
    replay_saved_tokens: int = 0
    demand_count: int = 0

    @property
    def retained_value(self) -> int:
        """Benefit proxy for cost-aware eviction: replay saved x (uses + 1)."""
        return (self.replay_saved_tokens or self.boundary_tokens) * (self.hit_count + self.demand_count + 1)


@dataclass(slots=True)
class PrefixDemandEntry:
    prefix_hash: int
    boundary_tokens: int
    observations: int
    last_seen_ns: int
    promotion_pending: bool = False


@dataclass(frozen=True, slots=True)
class CheckpointBoundary:
    boundary_tokens: int
    reason: str


class HybridCheckpointRetentionPolicy:
    def __init__(self, *, block_size: int, interval_tokens: int, mode: str = "periodic"):
        if block_size <= 0 or interval_tokens <= 0:
            raise ValueError("checkpoint boundary sizes must be positive")
        if interval_tokens % block_size:
            raise ValueError("checkpoint interval must align to KV blocks")
        if mode not in ("periodic", "adaptive"):
            raise ValueError(f"unsupported hybrid retention policy: {mode}")
        self.block_size, self.interval_tokens, self.mode = block_size, interval_tokens, mode

    def prompt_tail_boundary(self, prompt_tokens: int) -> int:
        return 0 if prompt_tokens <= 1 else ((prompt_tokens - 1) // self.block_size) * self.block_size

    def classify(self, boundary_tokens: int, prompt_tokens: int) -> CheckpointBoundary | None:
        if boundary_tokens <= 0 or boundary_tokens % self.block_size:
            return None
        if boundary_tokens % self.interval_tokens == 0:
            return CheckpointBoundary(boundary_tokens, "periodic")
        if self.mode == "adaptive" and boundary_tokens == self.prompt_tail_boundary(prompt_tokens):
            return CheckpointBoundary(boundary_tokens, "prompt_tail")
        return None

    def _walk(self, start_tokens: int, limit: int, prompt_tokens: int):
        b = (start_tokens // self.block_size + 1) * self.block_size
        while b <= limit:
            c = self.classify(b, prompt_tokens)
            if c is not None:
                yield c
            b += self.block_size

    def next_retained_boundary(self, start_tokens: int, prompt_tokens: int) -> CheckpointBoundary | None:
        return next(self._walk(start_tokens, self.prompt_tail_boundary(prompt_tokens), prompt_tokens), None)

    def retained_boundaries(self, start_tokens: int, end_tokens: int, prompt_tokens: int) -> list[CheckpointBoundary]:
        limit = min(end_tokens, self.prompt_tail_boundary(prompt_tokens))
        return list(self._walk(start_tokens, limit, prompt_tokens))


class GDNCheckpointManager:
    """Bounded checkpoint index; the tensors live in the runner's checkpoint pool."""

    def __init__(self, capacity: int, eviction_policy: str = "lru"):
        if capacity <= 0:
            raise ValueError("hybrid prefix cache capacity must be positive")
        if eviction_policy not in ("lru", "cost_aware"):
            raise ValueError(f"unsupported checkpoint eviction policy: {eviction_policy}")
        self.capacity = capacity
        self.eviction_policy = eviction_policy
        self.entries: dict[tuple[int, int], HybridPrefixEntry] = {}
        self.lru: OrderedDict[tuple[int, int], None] = OrderedDict()
        self.reset_metrics()

    def reset_metrics(self) -> None:
        self.queries = self.kv_candidate_tokens = self.committed_hit_tokens = 0
        self.captures = self.restores = self.evictions = self.evicted_retained_value = 0
        self.fallbacks = self.shared_junction_hits = self.useful_shared_junction_promotions = 0
        self.shared_junction_saved_replay_tokens = 0
        self.shared_junction_evictions = self.unused_shared_junction_evictions = 0
        self.peak_entries = len(self.entries)
        self.peak_shared_junction_entries = self._count("shared_junction")

    def _count(self, reason: str) -> int:
        return sum(e.reason == reason for e in self.entries.values())

    def find_hit(self, candidates: list[PrefixKVCandidate]) -> HybridPrefixHit | None:
        hit = self.peek_hit(candidates)
        self.record_lookup(candidates, hit)
        return hit

    def peek_hit(self, candidates: list[PrefixKVCandidate]) -> HybridPrefixHit | None:
        for c in candidates:
            e = self.entries.get((c.prefix_hash, c.boundary_tokens))
            if e is not None and e.tail_block_id == c.tail_block_id:
                return HybridPrefixHit(c, e.checkpoint_slot)
        return None

    def record_lookup(self, candidates: list[PrefixKVCandidate], hit: HybridPrefixHit | None) -> None:
        self.queries += 1
        if candidates:
            self.kv_candidate_tokens += candidates[0].boundary_tokens
        if hit is None:
            if candidates:
                self.fallbacks += 1
            return
        key = (hit.candidate.prefix_hash, hit.candidate.boundary_tokens)
        e = self.entries[key]
        e.last_access_ns = perf_counter_ns()
        if e.reason == "shared_junction":
            self.shared_junction_hits += 1
            self.shared_junction_saved_replay_tokens += e.replay_saved_tokens or e.boundary_tokens
            if e.hit_count == 0:
                self.useful_shared_junction_promotions += 1
        e.hit_count += 1
        self.lru.move_to_end(key)
        self.committed_hit_tokens += hit.candidate.boundary_tokens
        self.restores += 1

    def contains(self, prefix_hash: int, boundary_tokens: int) -> bool:
        return (prefix_hash, boundary_tokens) in self.entries

    def reserve_capture(self, pending: PendingHybridPrefixCapture) -> list[HybridPrefixEntry]:
        """Make room for one more entry; returns the evicted entries (their slots must be freed)."""
        if self.contains(pending.prefix_hash, pending.boundary_tokens):
            return []
        evicted = []
        while len(self.entries) >= self.capacity:
            if self.eviction_policy == "lru":
                key, _ = self.lru.popitem(last=False)
            else:
                key = min(self.entries, key=lambda k: (self.entries[k].retained_value, self.entries[k].last_access_ns))
                del self.lru[key]
            e = self.entries.pop(key)
            evicted.append(e)
            if e.reason == "shared_junction":
                self.shared_junction_evictions += 1
                if e.hit_count == 0:
                    self.unused_shared_junction_evictions += 1
            self.evicted_retained_value += e.retained_value
            self.evictions += 1
        return evicted

    def publish(self, pending: PendingHybridPrefixCapture, checkpoint_slot: int) -> None:
        key = (pending.prefix_hash, pending.boundary_tokens)
        if key in self.entries:
            raise ValueError("hybrid prefix checkpoint was already published")
        self.entries[key] = HybridPrefixEntry(pending.prefix_hash, pending.boundary_tokens, pending.tail_block_id,
                                              checkpoint_slot, perf_counter_ns(), pending.reason,
                                              replay_saved_tokens=pending.replay_saved_tokens,
                                              demand_count=pending.demand_count)
        self.lru[key] = None
        self.captures += 1
        self.peak_entries = max(self.peak_entries, len(self.entries))
        self.peak_shared_junction_entries = max(self.peak_shared_junction_entries, self._count("shared_junction"))

    def get_metrics(self) -> dict:
        unused_sj = sum(e.reason == "shared_junction" and e.hit_count == 0 for e in self.entries.values())
        return {
            "hybrid_prefix_cache_capacity": self.capacity,
            "hybrid_prefix_cache_entries": len(self.entries),
            "hybrid_prefix_cache_queries": self.queries,
            "hybrid_prefix_kv_candidate_tokens": self.kv_candidate_tokens,
            "hybrid_prefix_committed_hit_tokens": self.committed_hit_tokens,
            "hybrid_prefix_state_alignment_lost_tokens": self.kv_candidate_tokens - self.committed_hit_tokens,
            "hybrid_prefix_capture_count": self.captures,
            "hybrid_prefix_restore_count": self.restores,
            "hybrid_prefix_eviction_count": self.evictions,
            "hybrid_prefix_evicted_retained_value": self.evicted_retained_value,
            "hybrid_prefix_eviction_policy": self.eviction_policy,
            "hybrid_prefix_fallback_count": self.fallbacks,
            "hybrid_prefix_hit_rate": self.restores / self.queries if self.queries else 0.0,
            "hybrid_prefix_entries_periodic": self._count("periodic"),
            "hybrid_prefix_entries_prompt_tail": self._count("prompt_tail"),
            "hybrid_prefix_entries_shared_junction": self._count("shared_junction"),
            "hybrid_prefix_unused_shared_junction_entries": unused_sj,
            "hybrid_prefix_peak_entries": self.peak_entries,
            "hybrid_prefix_peak_shared_junction_entries": self.peak_shared_junction_entries,
            "hybrid_prefix_shared_junction_hit_count": self.shared_junction_hits,
            "hybrid_prefix_useful_promotion_count": self.useful_shared_junction_promotions,
            "hybrid_prefix_shared_junction_saved_replay_tokens": self.shared_junction_saved_replay_tokens,
            "hybrid_prefix_shared_junction_eviction_count": self.shared_junction_evictions,
            "hybrid_prefix_unused_promotion_eviction_count": self.unused_shared_junction_evictions,
        }


HybridPrefixCache = GDNCheckpointManager


class FullAttentionPrefixManager:
    def __init__(self, block_manager):
        self.block_manager = block_manager

    def find_candidates(self, sequence) -> list[PrefixKVCandidate]:
        return self.block_manager.find_prefix_candidates(sequence)

    def can_allocate(self, sequence, candidate: PrefixKVCandidate | None) -> bool:
        return self.block_manager.can_allocate_candidate(sequence, candidate)

    def allocate(self, sequence, candidate: PrefixKVCandidate | None):
        return self.block_manager.allocate_candidate(sequence, candidate)

    def metadata_at_boundary(self, sequence, boundary_tokens: int) -> PrefixKVCandidate:
        return self.block_manager.prefix_metadata_at_boundary(sequence, boundary_tokens)


class HybridPrefixCoordinator:
    def __init__(self, full_attention: FullAttentionPrefixManager, gdn_checkpoints: GDNCheckpointManager, *,
                 promote_shared_junctions: bool = False, promotion_min_sightings: int = 2,
                 demand_capacity: int = 1024):
        if demand_capacity <= 0:
            raise ValueError("prefix demand capacity must be positive")
        if promotion_min_sightings < 2:
            raise ValueError("demand-driven promotion requires at least two sightings")
        self.full_attention = full_attention
        self.gdn_checkpoints = gdn_checkpoints
        self.promote_shared_junctions = promote_shared_junctions
        self.promotion_min_sightings = promotion_min_sightings
        self.demand_capacity = demand_capacity
        self.demands: OrderedDict[tuple[int, int], PrefixDemandEntry] = OrderedDict()
        self.reset_promotion_metrics()

    def reset_promotion_metrics(self) -> None:
        self.kv_only_misses = self.alignment_lost_tokens = 0
        self.promotions_planned = self.promotions_published = self.promotions_cancelled = 0

    def _observe_alignment_gap(self, candidate: PrefixKVCandidate, committed: int) -> PrefixKVCandidate | None:
        lost = candidate.boundary_tokens - committed
        if lost <= 0:
            return None
        self.kv_only_misses += 1
        self.alignment_lost_tokens += lost
        if not self.promote_shared_junctions:
            return None
        key = (candidate.prefix_hash, candidate.boundary_tokens)
        now = perf_counter_ns()
        d = self.demands.get(key)
        if d is None:
            while len(self.demands) >= self.demand_capacity:
                victim = next((k for k, v in self.demands.items() if not v.promotion_pending), None)
                if victim is None:
                    return None
                self.demands.pop(victim)
            d = self.demands[key] = PrefixDemandEntry(candidate.prefix_hash, candidate.boundary_tokens, 0, now)
        d.observations += 1
        d.last_seen_ns = now
        self.demands.move_to_end(key)
        if d.promotion_pending or self.gdn_checkpoints.contains(*key):
            return None
        # A resident KV candidate proves one earlier producer, so this request
        # is sighting number ``1 + observations``.
        if 1 + d.observations < self.promotion_min_sightings:
            return None
        return candidate

    def _activate_promotion(self, candidate: PrefixKVCandidate | None) -> None:
        if candidate is None:
            return
        d = self.demands.get((candidate.prefix_hash, candidate.boundary_tokens))
        if d is None or d.promotion_pending:
            return
        d.promotion_pending = True
        self.promotions_planned += 1

    def cancel_promotion(self, candidate: PrefixKVCandidate | None) -> None:
        if candidate is None:
            return
        d = self.demands.get((candidate.prefix_hash, candidate.boundary_tokens))
        if d is not None and d.promotion_pending:
            d.promotion_pending = False
            self.promotions_cancelled += 1

    def demand_observations(self, candidate: PrefixKVCandidate) -> int:
        d = self.demands.get((candidate.prefix_hash, candidate.boundary_tokens))
        return d.observations if d is not None else 0

    def resolve_capture(self, pending: PendingHybridPrefixCapture, *, published: bool) -> None:
        if pending.reason != "shared_junction":
            return
        key = (pending.prefix_hash, pending.boundary_tokens)
        d = self.demands.get(key)
        if d is not None:
            d.promotion_pending = False
            if published:
                self.demands.pop(key, None)
        if published:
            self.promotions_published += 1
        else:
            self.promotions_cancelled += 1

    def _probe(self, candidates: list[PrefixKVCandidate]) -> HybridPrefixAllocationPlan:
        hit = self.gdn_checkpoints.peek_hit(candidates)
        return HybridPrefixAllocationPlan(hit, hit.candidate.num_cached_blocks if hit else 0,
                                          candidates[0].boundary_tokens if candidates else 0)

    def plan(self, sequence) -> HybridPrefixAllocationPlan | None:
        candidates = self.full_attention.find_candidates(sequence)
        p = self._probe(candidates)
        if not self.full_attention.can_allocate(sequence, p.candidate):
            return None
        promo = self._observe_alignment_gap(candidates[0], p.boundary_tokens) if candidates else None
        if p.hit is None:
            self.gdn_checkpoints.record_lookup(candidates, None)
        return HybridPrefixAllocationPlan(p.hit, p.num_cached_blocks, p.kv_candidate_tokens, promo)

    def probe(self, sequence) -> HybridPrefixAllocationPlan:
        return self._probe(self.full_attention.find_candidates(sequence))

    def commit(self, plan: HybridPrefixAllocationPlan) -> None:
        self._activate_promotion(plan.promotion_candidate)
        if plan.hit is not None:
            c = plan.hit.candidate
            view = PrefixKVCandidate(c.num_cached_blocks, plan.kv_candidate_tokens, c.prefix_hash,
                                     c.tail_block_id, c.tail_valid_tokens)
            self.gdn_checkpoints.record_lookup([view], plan.hit)

    def contains(self, prefix_hash: int, boundary_tokens: int) -> bool:
        return self.gdn_checkpoints.contains(prefix_hash, boundary_tokens)

    def reserve_capture(self, pending: PendingHybridPrefixCapture) -> list[HybridPrefixEntry]:
        return self.gdn_checkpoints.reserve_capture(pending)

    def publish(self, pending: PendingHybridPrefixCapture, checkpoint_slot: int) -> None:
        self.gdn_checkpoints.publish(pending, checkpoint_slot)
        self.resolve_capture(pending, published=True)

    def reset_metrics(self) -> None:
        self.gdn_checkpoints.reset_metrics()
        self.reset_promotion_metrics()

    def get_metrics(self) -> dict:
        m = self.gdn_checkpoints.get_metrics()
        m.update({
            "hybrid_prefix_kv_only_miss_count": self.kv_only_misses,
            "hybrid_prefix_alignment_lost_tokens": self.alignment_lost_tokens,
            "hybrid_prefix_shared_junction_promotions_planned": self.promotions_planned,
            "hybrid_prefix_shared_junction_promotions_published": self.promotions_published,
            "hybrid_prefix_shared_junction_promotions_cancelled": self.promotions_cancelled,
            "hybrid_prefix_demand_entries": len(self.demands),
            "hybrid_prefix_promotion_min_sightings": self.promotion_min_sightings,
            "hybrid_prefix_replay_due_to_missing_checkpoint_tokens": self.alignment_lost_tokens,
            "hybrid_prefix_useful_promotion_ratio": (
                self.gdn_checkpoints.useful_shared_junction_promotions / self.promotions_published
                if self.promotions_published else 0.0),
            "hybrid_prefix_promotions_not_yet_reused": sum(
                e.reason == "shared_junction" and e.hit_count == 0 for e in self.gdn_checkpoints.entries.values()),
        })
        return m
