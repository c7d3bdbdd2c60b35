"""Control plane of the hybrid (KV + GDN-state) prefix cache.

A prefix of a hybrid model can be skipped only where BOTH the paged KV of the
attention layers and a GDN recurrent/conv checkpoint exist at the same token
boundary.  Behavioural parity with ``nanovllm/engine/hybrid_prefix_cache.py``
(``:90-169`` retention, ``:172-376`` checkpoint index and eviction,
``:416-680`` coordination and shared-junction promotion): which boundaries get
a checkpoint, the longest jointly restorable boundary wins, a KV-only match
that is seen often enough is promoted to a checkpoint ("shared junction"), the
read-only ``probe`` used for scheduling scores, and the metric keys.

Design (this module's own):
* Retention is a strategy object that COMPUTES the retained boundaries of a
  range (multiples of the interval, plus the prompt tail in adaptive mode)
  instead of testing every unit boundary.
* ``CheckpointIndex`` keeps its records in recency order; eviction is a
  strategy object (``LruEviction`` / ``CostAwareEviction``) that picks the
  victim, and the cost model (replayed tokens saved x uses) lives there, not
  on the record.
* ``JunctionPromoter`` owns the demand ledger of KV-only matches and the
  promotion lifecycle (observed -> pending -> published | cancelled).
* ``HybridPrefixPlanner`` composes the block manager, the index and the
  promoter into admission plans and capture tickets; the scheduler drives it.
"""

from __future__ import annotations

from collections import Counter, OrderedDict
from dataclasses import dataclass, field
from time import perf_counter_ns

from inference_systems_b200.engine.block_manager import PrefixKVCandidate

# ----------------------------------------------------------------------------- boundaries


@dataclass(frozen=True, slots=True)
class RetainedBoundary:
    """A token boundary that gets a GDN checkpoint, and why: ``periodic`` (every interval),
    ``prompt_tail`` (last whole unit before the prompt's final token, adaptive mode) or
    ``shared_junction`` (promoted from repeated KV-only matches)."""

    boundary_tokens: int
    reason: str


class PeriodicRetention:
    """Retain a checkpoint every ``interval_tokens`` tokens (a multiple of the match unit)."""

    mode = "periodic"

    def __init__(self, unit: int, interval_tokens: int):
        if unit <= 0 or interval_tokens <= 0:
            raise ValueError("checkpoint boundary sizes must be positive")
        if interval_tokens % unit:
            raise ValueError("checkpoint interval must align to KV blocks")
        self.unit, self.interval = unit, interval_tokens

    def prompt_tail(self, prompt_tokens: int) -> int:
        """Last unit boundary strictly before the prompt's final token (0 if none)."""
        return ((prompt_tokens - 1) // self.unit) * self.unit if prompt_tokens > 1 else 0

    def classify(self, boundary: int, prompt_tokens: int) -> RetainedBoundary | None:
        if boundary <= 0 or boundary % self.unit:
            return None
        if boundary % self.interval == 0:
            return RetainedBoundary(boundary, "periodic")
        return None

    def boundaries(self, start: int, end: int, prompt_tokens: int) -> list[RetainedBoundary]:
        """Retained boundaries in ``(start, min(end, prompt tail)]``, ascending."""
        limit = min(end, self.prompt_tail(prompt_tokens))
        first = (start // self.interval + 1) * self.interval
        return [RetainedBoundary(b, "periodic") for b in range(first, limit + 1, self.interval)]

    def next_boundary(self, start: int, prompt_tokens: int) -> RetainedBoundary | None:
        found = self.boundaries(start, self.prompt_tail(prompt_tokens), prompt_tokens)
        return found[0] if found else None


class AdaptiveRetention(PeriodicRetention):
    """Periodic boundaries plus the prompt tail, so a repeated prompt restores almost all of it."""

    mode = "adaptive"

    def classify(self, boundary: int, prompt_tokens: int) -> RetainedBoundary | None:
        found = super().classify(boundary, prompt_tokens)
        if found is None and boundary > 0 and boundary == self.prompt_tail(prompt_tokens):
            return RetainedBoundary(boundary, "prompt_tail")
        return found

    def boundaries(self, start: int, end: int, prompt_tokens: int) -> list[RetainedBoundary]:
        out = super().boundaries(start, end, prompt_tokens)
        tail = self.prompt_tail(prompt_tokens)
        if start < tail <= end and tail % self.interval:
            out.append(RetainedBoundary(tail, "prompt_tail"))
        return out


def make_retention(mode: str, unit: int, interval_tokens: int) -> PeriodicRetention:
    if mode == "periodic":
        return PeriodicRetention(unit, interval_tokens)
    if mode == "adaptive":
        return AdaptiveRetention(unit, interval_tokens)
    raise ValueError(f"unsupported hybrid retention policy: {mode}")


# ------------------------------------------------------------------------- checkpoint index


@dataclass(frozen=True, slots=True)
class CaptureTicket:
    """A checkpoint to capture after the step that reached ``boundary_tokens`` of a request.

    ``internal_state``: the boundary lies inside the scheduled chunk, so the runner captures the
    state it recorded there instead of the slot's current state.  ``replay_saved_tokens`` /
    ``demand_count`` seed the cost model of a promoted shared junction."""

    prefix_hash: int
    boundary_tokens: int
    tail_block_id: int
    state_slot: int
    reason: str = "periodic"
    internal_state: bool = False
    sequence_id: int = -1
    replay_saved_tokens: int = 0
    demand_count: int = 0

    @property
    def key(self) -> tuple[int, int]:
        return (self.prefix_hash, self.boundary_tokens)


@dataclass(slots=True)
class CheckpointRecord:
    """A published GDN checkpoint: where its KV tail lives and which pool slot holds the state."""

    prefix_hash: int
    boundary_tokens: int
    tail_block_id: int
    checkpoint_slot: int
    reason: str
    last_used_ns: int
    hits: int = 0
    replay_saved_tokens: int = 0
    demand_count: int = 0


class LruEviction:
    name = "lru"

    def victim(self, records: "OrderedDict[tuple[int, int], CheckpointRecord]") -> tuple[int, int]:
        return next(iter(records))  # least recently used first


class CostAwareEviction:
    """Evict the record worth least: tokens of replay it saves per use x (uses + demand + 1)."""

    name = "cost_aware"

    @staticmethod
    def value(r: CheckpointRecord) -> int:
        return (r.replay_saved_tokens or r.boundary_tokens) * (r.hits + r.demand_count + 1)

    def victim(self, records: "OrderedDict[tuple[int, int], CheckpointRecord]") -> tuple[int, int]:
        return min(records, key=lambda k: (self.value(records[k]), records[k].last_used_ns))


@dataclass(frozen=True, slots=True)
class PrefixHit:
    candidate: PrefixKVCandidate
    checkpoint_slot: int


class CheckpointIndex:
    """Bounded map ``(prefix hash, boundary) -> checkpoint slot``; the states live in the runner's
    checkpoint pool, which frees the slots of the records this index evicts."""

    def __init__(self, capacity: int, eviction_policy: str = "lru"):
        if capacity <= 0:
            raise ValueError("hybrid prefix cache capacity must be positive")
        policies = {"lru": LruEviction, "cost_aware": CostAwareEviction}
        if eviction_policy not in policies:
            raise ValueError(f"unsupported checkpoint eviction policy: {eviction_policy}")
        self.capacity = capacity
        self.policy = policies[eviction_policy]()
        self.records: OrderedDict[tuple[int, int], CheckpointRecord] = OrderedDict()
        self.reset_metrics()

    @property
    def eviction_policy(self) -> str:
        return self.policy.name

    def reset_metrics(self) -> None:
        self.stats: Counter = Counter()
        self.peak_entries = len(self.records)
        self.peak_junctions = self._count("shared_junction")

    def _count(self, reason: str) -> int:
        return sum(r.reason == reason for r in self.records.values())

    def __contains__(self, key: tuple[int, int]) -> bool:
        return key in self.records

    def lookup(self, candidates: list[PrefixKVCandidate]) -> PrefixHit | None:
        """Longest candidate with a checkpoint whose KV tail is still the same page (no side effects)."""
        for c in candidates:
            r = self.records.get((c.prefix_hash, c.boundary_tokens))
            if r is not None and r.tail_block_id == c.tail_block_id:
                return PrefixHit(c, r.checkpoint_slot)
        return None

    def note_lookup(self, kv_tokens: int, had_candidates: bool, hit: PrefixHit | None) -> None:
        """Account one admission lookup; a hit refreshes its record."""
        st = self.stats
        st["queries"] += 1
        st["kv_candidate_tokens"] += kv_tokens
        if hit is None:
            if had_candidates:
                st["fallbacks"] += 1
            return
        key = (hit.candidate.prefix_hash, hit.candidate.boundary_tokens)
        r = self.records[key]
        r.last_used_ns = perf_counter_ns()
        if r.reason == "shared_junction":
            st["junction_hits"] += 1
            st["junction_saved_replay_tokens"] += r.replay_saved_tokens or r.boundary_tokens
            if r.hits == 0:
                st["useful_promotions"] += 1
        r.hits += 1
        self.records.move_to_end(key)
        st["committed_hit_tokens"] += hit.candidate.boundary_tokens
        st["restores"] += 1

    def make_room(self, ticket: CaptureTicket) -> list[CheckpointRecord]:
        """Evict until one more record fits; returns the evicted records (free their slots)."""
        if ticket.key in self.records:
            return []
        evicted = []
        while len(self.records) >= self.capacity:
            r = self.records.pop(self.policy.victim(self.records))
            evicted.append(r)
            self.stats["evictions"] += 1
            self.stats["evicted_retained_value"] += CostAwareEviction.value(r)
            if r.reason == "shared_junction":
                self.stats["junction_evictions"] += 1
                if r.hits == 0:
                    self.stats["unused_junction_evictions"] += 1
        return evicted

    def insert(self, ticket: CaptureTicket, checkpoint_slot: int) -> None:
        if ticket.key in self.records:
            raise ValueError("hybrid prefix checkpoint was already published")
        self.records[ticket.key] = CheckpointRecord(
            ticket.prefix_hash, ticket.boundary_tokens, ticket.tail_block_id, checkpoint_slot, ticket.reason,
            perf_counter_ns(), replay_saved_tokens=ticket.replay_saved_tokens, demand_count=ticket.demand_count)
        self.stats["captures"] += 1
        self.peak_entries = max(self.peak_entries, len(self.records))
        self.peak_junctions = max(self.peak_junctions, self._count("shared_junction"))

    def metrics(self) -> dict:
        st = self.stats
        unused = sum(r.reason == "shared_junction" and r.hits == 0 for r in self.records.values())
        return {
            "hybrid_prefix_cache_capacity": self.capacity,
            "hybrid_prefix_cache_entries": len(self.records),
            "hybrid_prefix_cache_queries": st["queries"],
            "hybrid_prefix_kv_candidate_tokens": st["kv_candidate_tokens"],
            "hybrid_prefix_committed_hit_tokens": st["committed_hit_tokens"],
            "hybrid_prefix_state_alignment_lost_tokens": st["kv_candidate_tokens"] - st["committed_hit_tokens"],
            "hybrid_prefix_capture_count": st["captures"],
            "hybrid_prefix_restore_count": st["restores"],
            "hybrid_prefix_eviction_count": st["evictions"],
            "hybrid_prefix_evicted_retained_value": st["evicted_retained_value"],
            "hybrid_prefix_eviction_policy": self.eviction_policy,
            "hybrid_prefix_fallback_count": st["fallbacks"],
            "hybrid_prefix_hit_rate": st["restores"] / st["queries"] if st["queries"] else 0.0,
            "hybrid_prefix_entries_periodic": self._count("periodic"),
            "hybrid_prefix_entries_prompt_tail": self._count("prompt_tail"),
            "hybrid_prefix_entries_shared_junction": self._count("shared_junction"),
            "hybrid_prefix_unused_shared_junction_entries": unused,
            "hybrid_prefix_peak_entries": self.peak_entries,
            "hybrid_prefix_peak_shared_junction_entries": self.peak_junctions,
            "hybrid_prefix_shared_junction_hit_count": st["junction_hits"],
            "hybrid_prefix_useful_promotion_count": st["useful_promotions"],
            "hybrid_prefix_shared_junction_saved_replay_tokens": st["junction_saved_replay_tokens"],
            "hybrid_prefix_shared_junction_eviction_count": st["junction_evictions"],
            "hybrid_prefix_unused_promotion_eviction_count": st["unused_junction_evictions"],
        }


# ------------------------------------------------------------------------ promotion


@dataclass(slots=True)
class _Demand:
    observations: int = 0
    last_seen_ns: int = 0
    pending: bool = False


class JunctionPromoter:
    """Counts KV-only matches per boundary; once a boundary has been reached by
    ``min_sightings`` requests in total (the producer that left the KV counts as one), the next
    request to reach it captures a checkpoint there."""

    def __init__(self, enabled: bool, min_sightings: int, capacity: int):
        if capacity <= 0:
            raise ValueError("prefix demand capacity must be positive")
        if min_sightings < 2:
            raise ValueError("demand-driven promotion requires at least two sightings")
        self.enabled, self.min_sightings, self.capacity = enabled, min_sightings, capacity
        self.demand: OrderedDict[tuple[int, int], _Demand] = OrderedDict()
        self.reset_metrics()

    def reset_metrics(self) -> None:
        self.stats: Counter = Counter()

    def _admit_key(self, key: tuple[int, int]) -> _Demand | None:
        d = self.demand.get(key)
        if d is not None:
            return d
        while len(self.demand) >= self.capacity:  # forget the stalest boundary that is not in flight
            stale = next((k for k, v in self.demand.items() if not v.pending), None)
            if stale is None:
                return None
            del self.demand[stale]
        d = self.demand[key] = _Demand()
        return d

    def observe(self, kv_best: PrefixKVCandidate, restored_tokens: int,
                index: CheckpointIndex) -> PrefixKVCandidate | None:
        """Record that the longest KV match ``kv_best`` went past the restorable boundary; returns it
        when it should be promoted now."""
        lost = kv_best.boundary_tokens - restored_tokens
        if lost <= 0:
            return None
        self.stats["kv_only_misses"] += 1
        self.stats["alignment_lost_tokens"] += lost
        if not self.enabled:
            return None
        key = (kv_best.prefix_hash, kv_best.boundary_tokens)
        d = self._admit_key(key)
        if d is None:
            return None
        d.observations += 1
        d.last_seen_ns = perf_counter_ns()
        self.demand.move_to_end(key)
        if d.pending or key in index or d.observations + 1 < self.min_sightings:
            return None
        return kv_best

    def activate(self, c: PrefixKVCandidate | None) -> None:
        d = self.demand.get((c.prefix_hash, c.boundary_tokens)) if c is not None else None
        if d is not None and not d.pending:
            d.pending = True
            self.stats["planned"] += 1

    def cancel(self, c: PrefixKVCandidate | None) -> None:
        d = self.demand.get((c.prefix_hash, c.boundary_tokens)) if c is not None else None
        if d is not None and d.pending:
            d.pending = False
            self.stats["cancelled"] += 1

    def observations(self, c: PrefixKVCandidate) -> int:
        d = self.demand.get((c.prefix_hash, c.boundary_tokens))
        return d.observations if d is not None else 0

    def resolve(self, ticket: CaptureTicket, published: bool) -> None:
        if ticket.reason != "shared_junction":
            return
        d = self.demand.get(ticket.key)
        if d is not None:
            d.pending = False
            if published:
                del self.demand[ticket.key]
        self.stats["published" if published else "cancelled"] += 1


# -------------------------------------------------------------------------- planner


@dataclass(frozen=True, slots=True)
class AdmissionPlan:
    """How a new request starts: from a restorable boundary (``hit``) or from scratch, how many
    KV tokens were matched, and the boundary to promote (if any)."""

    hit: PrefixHit | None
    num_cached_blocks: int
    kv_candidate_tokens: int = 0
    promotion_candidate: PrefixKVCandidate | None = None

    @property
    def boundary_tokens(self) -> int:
        return self.hit.candidate.boundary_tokens if self.hit is not None else 0

    @property
    def candidate(self) -> PrefixKVCandidate | None:
        return self.hit.candidate if self.hit is not None else None


@dataclass
class _Promotion:
    """A promoted boundary a request is on its way to, tracked until its checkpoint is captured."""

    boundary: RetainedBoundary
    saved_replay_tokens: int
    candidate: PrefixKVCandidate
    demand: int


class HybridPrefixPlanner:
    def __init__(self, block_manager, index: CheckpointIndex, *, promote_shared_junctions: bool = False,
                 promotion_min_sightings: int = 2, demand_capacity: int = 1024):
        self.blocks = block_manager
        self.index = index
        self.promoter = JunctionPromoter(promote_shared_junctions, promotion_min_sightings, demand_capacity)
        self.promotions: dict[int, _Promotion] = {}  # by sequence id

    @property
    def promotion_min_sightings(self) -> int:
        return self.promoter.min_sightings

    # ------------------------------------------------------------- admission
    def _assess(self, seq) -> tuple[list[PrefixKVCandidate], AdmissionPlan]:
        cands = self.blocks.find_prefix_candidates(seq)
        hit = self.index.lookup(cands)
        return cands, AdmissionPlan(hit, hit.candidate.num_cached_blocks if hit else 0,
                                    cands[0].boundary_tokens if cands else 0)

    def probe(self, seq) -> AdmissionPlan:
        """What admitting ``seq`` now would restore (no side effects)."""
        return self._assess(seq)[1]

    def plan(self, seq) -> AdmissionPlan | None:
        """The admission plan for ``seq``, or ``None`` when its pages do not fit."""
        cands, p = self._assess(seq)
        if not self.blocks.can_allocate_candidate(seq, p.candidate):
            return None
        promo = self.promoter.observe(cands[0], p.boundary_tokens, self.index) if cands else None
        if p.hit is None:
            self.index.note_lookup(p.kv_candidate_tokens, bool(cands), None)
        return AdmissionPlan(p.hit, p.num_cached_blocks, p.kv_candidate_tokens, promo)

    def commit(self, seq, plan: AdmissionPlan) -> None:
        """The plan was carried out for ``seq`` (pages taken, state restored)."""
        pc = plan.promotion_candidate
        self.promoter.activate(pc)
        if pc is not None:
            self.promotions[seq.seq_id] = _Promotion(RetainedBoundary(pc.boundary_tokens, "shared_junction"),
                                                     pc.boundary_tokens - plan.boundary_tokens, pc,
                                                     self.promoter.observations(pc))
        if plan.hit is not None:
            self.index.note_lookup(plan.kv_candidate_tokens, True, plan.hit)

    def abandon(self, plan: AdmissionPlan) -> None:
        """The plan failed part-way; a promotion it would have started is released."""
        self.promoter.cancel(plan.promotion_candidate)

    def forget(self, seq) -> None:
        """``seq`` left (preempted, aborted): its pending promotion is released."""
        p = self.promotions.pop(seq.seq_id, None)
        if p is not None:
            self.promoter.cancel(p.candidate)

    def promotion_for(self, seq) -> _Promotion | None:
        return self.promotions.get(seq.seq_id)

    # ---------------------------------------------------------------- capture
    def contains(self, prefix_hash: int, boundary_tokens: int) -> bool:
        return (prefix_hash, boundary_tokens) in self.index

    def reserve(self, ticket: CaptureTicket) -> list[CheckpointRecord] | None:
        """Room for ``ticket``'s record (evicted records returned), or ``None`` if already present."""
        if ticket.key in self.index:
            self.settle(ticket, published=False)
            return None
        return self.index.make_room(ticket)

    def publish(self, ticket: CaptureTicket, checkpoint_slot: int) -> None:
        self.index.insert(ticket, checkpoint_slot)
        self.settle(ticket, published=True)

    def settle(self, ticket: CaptureTicket, published: bool) -> None:
        """A shared-junction capture finished (published) or was dropped."""
        if ticket.reason != "shared_junction":
            return
        self.promoter.resolve(ticket, published)
        self.promotions.pop(ticket.sequence_id, None)

    # ---------------------------------------------------------------- metrics
    def reset_metrics(self) -> None:
        self.index.reset_metrics()
        self.promoter.reset_metrics()

    def get_metrics(self) -> dict:
        m = self.index.metrics()
        pst, ist = self.promoter.stats, self.index.stats
        m.update({
            "hybrid_prefix_kv_only_miss_count": pst["kv_only_misses"],
            "hybrid_prefix_alignment_lost_tokens": pst["alignment_lost_tokens"],
            "hybrid_prefix_shared_junction_promotions_planned": pst["planned"],
            "hybrid_prefix_shared_junction_promotions_published": pst["published"],
            "hybrid_prefix_shared_junction_promotions_cancelled": pst["cancelled"],
            "hybrid_prefix_demand_entries": len(self.promoter.demand),
            "hybrid_prefix_promotion_min_sightings": self.promoter.min_sightings,
            "hybrid_prefix_replay_due_to_missing_checkpoint_tokens": pst["alignment_lost_tokens"],
            "hybrid_prefix_useful_promotion_ratio": (ist["useful_promotions"] / pst["published"]
                                                     if pst["published"] else 0.0),
            "hybrid_prefix_promotions_not_yet_reused": sum(
                r.reason == "shared_junction" and r.hits == 0 for r in self.index.records.values()),
        })
        return m
