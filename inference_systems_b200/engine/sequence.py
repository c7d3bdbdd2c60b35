"""Request state: tokens, paging/slot ownership, a timeline and a scheduling ledger.

Behavioural parity with ``nanovllm/engine/sequence.py:9-240``: a request owns its
token ids, block table, GDN state slot and cached/scheduled token counters; its
lifecycle metrics use the same keys (TTFT, TPOT, gaps, queue time, ...), so
metrics consumers keep working.

Design:
* ``Sequence`` holds only what the scheduler, the block manager and the model
  runner need to place and run the request.
* ``RequestTimeline`` records time points (arrival, admission, scheduling,
  every emitted token, finish) in one int64 array that grows in place, and
  derives the latency metrics from it.
* ``SchedulingLedger`` holds the scheduler's per-request counters (how often it
  was scheduled, bypassed, preempted; what the last admission probe found).
* Worker ranks receive a compact tuple (``__getstate__``): metadata plus the last
  token for decode, the token list for prefill; the timeline and ledger stay on
  the host that schedules.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass
from enum import Enum, auto
from itertools import count
from time import perf_counter_ns

import numpy as np

from inference_systems_b200.sampling_params import SamplingParams


class SequenceStatus(Enum):
    WAITING = auto()
    RUNNING = auto()
    FINISHED = auto()
    ABORTED = auto()


def _ms(a: int | None, b: int | None) -> float | None:
    return None if a is None or b is None else (b - a) / 1e6


class RequestTimeline:
    """Monotonic time points of one request (``perf_counter_ns``)."""

    __slots__ = ("arrival_ns", "admitted_ns", "first_scheduled_ns", "last_scheduled_ns", "finished_ns",
                 "_tok", "_ntok")

    def __init__(self, arrival_ns: int, admitted_ns: int):
        self.arrival_ns = arrival_ns
        self.admitted_ns = admitted_ns
        self.first_scheduled_ns: int | None = None
        self.last_scheduled_ns: int | None = None
        self.finished_ns: int | None = None
        self._tok = np.empty(8, dtype=np.int64)
        self._ntok = 0

    def scheduled(self, t: int) -> None:
        if self.first_scheduled_ns is None:
            self.first_scheduled_ns = t
        self.last_scheduled_ns = t

    def token(self, t: int) -> None:
        if self._ntok == self._tok.shape[0]:
            self._tok = np.concatenate((self._tok, np.empty_like(self._tok)))
        self._tok[self._ntok] = t
        self._ntok += 1

    @property
    def token_times_ns(self) -> np.ndarray:
        return self._tok[: self._ntok]

    @property
    def first_token_ns(self) -> int | None:
        return int(self._tok[0]) if self._ntok else None

    @property
    def last_token_ns(self) -> int | None:
        return int(self._tok[self._ntok - 1]) if self._ntok else None

    def metrics(self, now_ns: int) -> dict:
        gaps = np.diff(self.token_times_ns) / 1e6
        end = self.finished_ns or now_ns
        return {
            "admission_delay_ms": _ms(self.arrival_ns, self.admitted_ns),
            "queue_ms": _ms(self.arrival_ns, self.first_scheduled_ns),
            "ttft_ms": _ms(self.arrival_ns, self.first_token_ns),
            "e2e_ms": _ms(self.arrival_ns, self.finished_ns),
            "tpot_ms": float(gaps.mean()) if gaps.size else None,
            "max_token_gap_ms": float(gaps.max()) if gaps.size else None,
            "time_since_last_token_ms": _ms(self.last_token_ns, end),
        }


@dataclass(slots=True)
class SchedulingLedger:
    """What the scheduler did with one request and what its last admission probe found."""

    schedule_count: int = 0
    preemption_count: int = 0
    scheduler_bypass_count: int = 0
    wait_rounds: int = 0
    max_wait_rounds: int = 0
    last_scheduler_score: float | None = None
    last_reusable_tokens: int = 0
    last_kv_candidate_tokens: int = 0
    last_gdn_checkpoint_tokens: int = 0
    last_joint_recoverable_tokens: int = 0
    estimated_recompute_tokens_lost: int = 0
    prefill_tokens_executed: int = 0
    prefix_tokens_reused: int = 0
    prefix_cache_hit_blocks: int = 0
    peak_kv_blocks: int = 0

    def bypassed(self) -> None:
        self.wait_rounds += 1
        self.max_wait_rounds = max(self.max_wait_rounds, self.wait_rounds)
        self.scheduler_bypass_count += 1

    def metrics(self) -> dict:
        d = asdict(self)
        del d["wait_rounds"], d["last_scheduler_score"]
        return d


_DEFAULT_PARAMS = SamplingParams()


class Sequence:
    block_size = 256
    _ids = count()

    def __init__(self, token_ids: list[int], sampling_params: SamplingParams = _DEFAULT_PARAMS,
                 arrival_time_ns: int | None = None, admitted_time_ns: int | None = None):
        if not token_ids:
            raise ValueError("prompt must contain at least one token")
        self.seq_id = next(Sequence._ids)
        self.status = SequenceStatus.WAITING
        self.token_ids = [int(t) for t in token_ids]
        self.num_tokens = len(self.token_ids)
        self.num_prompt_tokens = self.num_tokens
        self.last_token = self.token_ids[-1]
        self.num_cached_tokens = 0
        self.num_scheduled_tokens = 0
        self.is_prefill = True
        self.block_table: list[int] = []
        self.state_slot: int | None = None
        self.temperature = sampling_params.temperature
        self.max_tokens = sampling_params.max_tokens
        self.ignore_eos = sampling_params.ignore_eos
        now = perf_counter_ns()
        self.timeline = RequestTimeline(arrival_time_ns if arrival_time_ns is not None else now,
                                        admitted_time_ns if admitted_time_ns is not None else now)
        self.ledger = SchedulingLedger()
        # chained prefix hashes of this request's token units per unit size, extended lazily by the
        # block manager (tokens are only ever appended, so a computed hash never goes stale)
        self.unit_hashes: dict[int, list[int]] = {}

    # ---------------------------------------------------------------- views
    def __len__(self) -> int:
        return self.num_tokens

    def __getitem__(self, key):
        return self.token_ids[key]

    @property
    def is_finished(self) -> bool:
        return self.status is SequenceStatus.FINISHED or self.status is SequenceStatus.ABORTED

    @property
    def num_completion_tokens(self) -> int:
        return self.num_tokens - self.num_prompt_tokens

    @property
    def prompt_token_ids(self) -> list[int]:
        return self.token_ids[: self.num_prompt_tokens]

    @property
    def completion_token_ids(self) -> list[int]:
        return self.token_ids[self.num_prompt_tokens:]

    @property
    def num_blocks(self) -> int:
        return -(-self.num_tokens // self.block_size)

    @property
    def last_block_num_tokens(self) -> int:
        return self.num_tokens - (self.num_blocks - 1) * self.block_size

    def block(self, i: int) -> list[int]:
        if not 0 <= i < self.num_blocks:
            raise IndexError(f"block {i} of a {self.num_blocks}-block sequence")
        return self.token_ids[i * self.block_size:(i + 1) * self.block_size]

    # ------------------------------------------------------------ lifecycle
    @property
    def arrival_time_ns(self) -> int:
        return self.timeline.arrival_ns

    @property
    def preemption_count(self) -> int:
        return self.ledger.preemption_count

    def mark_scheduled(self, scheduled_at_ns: int | None = None) -> None:
        self.timeline.scheduled(scheduled_at_ns if scheduled_at_ns is not None else perf_counter_ns())
        led = self.ledger
        led.schedule_count += 1
        led.wait_rounds = 0
        led.peak_kv_blocks = max(led.peak_kv_blocks, len(self.block_table))

    def mark_preempted(self) -> None:
        self.ledger.preemption_count += 1

    def mark_bypassed(self) -> None:
        self.ledger.bypassed()

    def append_token(self, token_id: int, generated_at_ns: int | None = None) -> None:
        tok = int(token_id)
        self.token_ids.append(tok)
        self.last_token = tok
        self.num_tokens += 1
        self.timeline.token(generated_at_ns if generated_at_ns is not None else perf_counter_ns())

    def mark_finished(self, finished_at_ns: int | None = None) -> None:
        self.timeline.finished_ns = finished_at_ns if finished_at_ns is not None else perf_counter_ns()

    def lifecycle_metrics(self, now_ns: int | None = None) -> dict:
        now = now_ns if now_ns is not None else perf_counter_ns()
        return {"request_id": self.seq_id, "status": self.status.name.lower(),
                "prompt_tokens": self.num_prompt_tokens, "output_tokens": self.num_completion_tokens,
                **self.timeline.metrics(now), **self.ledger.metrics()}

    # ------------------------------------------------- transfer to worker ranks
    def __getstate__(self):
        payload = self.token_ids if self.is_prefill else self.last_token
        return (self.seq_id, self.num_tokens, self.num_prompt_tokens, self.num_cached_tokens,
                self.num_scheduled_tokens, self.block_table, self.state_slot, self.temperature,
                self.is_prefill, payload)

    def __setstate__(self, state):
        (self.seq_id, self.num_tokens, self.num_prompt_tokens, self.num_cached_tokens,
         self.num_scheduled_tokens, self.block_table, self.state_slot, self.temperature,
         self.is_prefill, payload) = state
        if isinstance(payload, list):
            self.token_ids, self.last_token = payload, payload[-1]
        else:
            self.token_ids, self.last_token = [], payload
