"""Request state.

Parity: ``nanovllm/engine/sequence.py:9-240`` -- token ids, block table,
state slot, cached / scheduled token counters, timestamps and the
lifecycle-metrics dictionary (same keys, so metrics consumers keep working).
Worker processes receive a compact copy (``__getstate__``): metadata plus the
last token for decode, the full token list for prefill.
"""

from __future__ import annotations

from enum import Enum, auto
from itertools import count
from time import perf_counter_ns

from inference_systems_b200.sampling_params import SamplingParams


class SequenceStatus(Enum):
    WAITING = auto()
    RUNNING = auto()
    FINISHED = auto()
    ABORTED = auto()


_DEFAULT_PARAMS = SamplingParams()


class Sequence:
    block_size = 256
    counter = count()

    def __init__(self, token_ids: list[int], sampling_params: SamplingParams = _DEFAULT_PARAMS,
                 arrival_time_ns: int | None = None, admitted_time_ns: int | None = None):
        if not token_ids:
            raise ValueError("prompt must contain at least one token")
        self.seq_id = next(Sequence.counter)
        self.status = SequenceStatus.WAITING
        self.token_ids = list(token_ids)
        self.last_token = self.token_ids[-1]
        self.num_tokens = len(self.token_ids)
        self.num_prompt_tokens = len(self.token_ids)
        self.num_cached_tokens = 0
        self.num_scheduled_tokens = 0
        self.is_prefill = True
        self.block_table: list[int] = []
        self.state_slot: int | None = None
        self.temperature = sampling_params.temperature
        self.max_tokens = sampling_params.max_tokens
        self.ignore_eos = sampling_params.ignore_eos
        now = perf_counter_ns()
        self.arrival_time_ns = arrival_time_ns if arrival_time_ns is not None else now
        self.admitted_time_ns = admitted_time_ns if admitted_time_ns is not None else now
        self.first_scheduled_time_ns: int | None = None
        self.last_scheduled_time_ns: int | None = None
        self.finished_time_ns: int | None = None
        self.token_timestamps_ns: list[int] = []
        self.schedule_count = 0
        self.preemption_count = 0
        self.wait_rounds = 0
        self.max_wait_rounds = 0
        self.scheduler_bypass_count = 0
        self.last_scheduler_score: float | None = None
        self.last_reusable_tokens = 0
        self.last_kv_candidate_tokens = 0
        self.last_gdn_checkpoint_tokens = 0
        self.last_joint_recoverable_tokens = 0
        self.estimated_recompute_tokens_lost = 0
        self.prefill_tokens_executed = 0
        self.prefix_tokens_reused = 0
        self.prefix_cache_hit_blocks = 0
        self.peak_kv_blocks = 0

    # ---- basic views ---------------------------------------------------
    def __len__(self):
        return self.num_tokens

    def __getitem__(self, key):
        return self.token_ids[key]

    @property
    def is_finished(self) -> bool:
        return self.status in (SequenceStatus.FINISHED, SequenceStatus.ABORTED)

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
        return (self.num_tokens + self.block_size - 1) // self.block_size

    @property
    def last_block_num_tokens(self) -> int:
        return self.num_tokens - (self.num_blocks - 1) * self.block_size

    def block(self, i: int) -> list[int]:
        assert 0 <= i < self.num_blocks
        return self.token_ids[i * self.block_size:(i + 1) * self.block_size]

    # ---- lifecycle -----------------------------------------------------
    def mark_scheduled(self, scheduled_at_ns: int | None = None) -> None:
        t = scheduled_at_ns if scheduled_at_ns is not None else perf_counter_ns()
        if self.first_scheduled_time_ns is None:
            self.first_scheduled_time_ns = t
        self.last_scheduled_time_ns = t
        self.schedule_count += 1
        self.wait_rounds = 0
        self.peak_kv_blocks = max(self.peak_kv_blocks, len(self.block_table))

    def mark_preempted(self) -> None:
        self.preemption_count += 1

    def mark_bypassed(self) -> None:
        self.wait_rounds += 1
        self.max_wait_rounds = max(self.max_wait_rounds, self.wait_rounds)
        self.scheduler_bypass_count += 1

    def append_token(self, token_id: int, generated_at_ns: int | None = None) -> None:
        self.token_ids.append(int(token_id))
        self.last_token = int(token_id)
        self.num_tokens += 1
        self.token_timestamps_ns.append(generated_at_ns if generated_at_ns is not None else perf_counter_ns())

    def mark_finished(self, finished_at_ns: int | None = None) -> None:
        self.finished_time_ns = finished_at_ns if finished_at_ns is not None else perf_counter_ns()

    @property
    def first_token_time_ns(self) -> int | None:
        return self.token_timestamps_ns[0] if self.token_timestamps_ns else None

    @property
    def last_token_time_ns(self) -> int | None:
        return self.token_timestamps_ns[-1] if self.token_timestamps_ns else None

    def lifecycle_metrics(self, now_ns: int | None = None) -> dict:
        now = now_ns if now_ns is not None else perf_counter_ns()
        ref = self.finished_time_ns or now

        def ms(a, b):
            return None if a is None or b is None else (b - a) / 1e6

        gaps = [(b - a) / 1e6 for a, b in zip(self.token_timestamps_ns, self.token_timestamps_ns[1:])]
        return {
            "request_id": self.seq_id,
            "status": self.status.name.lower(),
            "prompt_tokens": self.num_prompt_tokens,
            "output_tokens": self.num_completion_tokens,
            "admission_delay_ms": ms(self.arrival_time_ns, self.admitted_time_ns),
            "queue_ms": ms(self.arrival_time_ns, self.first_scheduled_time_ns),
            "ttft_ms": ms(self.arrival_time_ns, self.first_token_time_ns),
            "e2e_ms": ms(self.arrival_time_ns, self.finished_time_ns),
            "tpot_ms": sum(gaps) / len(gaps) if gaps else None,
            "max_token_gap_ms": max(gaps) if gaps else None,
            "time_since_last_token_ms": ms(self.last_token_time_ns, ref),
            "schedule_count": self.schedule_count,
            "preemption_count": self.preemption_count,
            "scheduler_bypass_count": self.scheduler_bypass_count,
            "max_wait_rounds": self.max_wait_rounds,
            "last_reusable_tokens": self.last_reusable_tokens,
            "last_kv_candidate_tokens": self.last_kv_candidate_tokens,
            "last_gdn_checkpoint_tokens": self.last_gdn_checkpoint_tokens,
            "last_joint_recoverable_tokens": self.last_joint_recoverable_tokens,
            "estimated_recompute_tokens_lost": self.estimated_recompute_tokens_lost,
            "prefill_tokens_executed": self.prefill_tokens_executed,
            "prefix_tokens_reused": self.prefix_tokens_reused,
            "prefix_cache_hit_blocks": self.prefix_cache_hit_blocks,
            "peak_kv_blocks": self.peak_kv_blocks,
        }

    # ---- compact transfer to worker ranks -------------------------------
    def __getstate__(self):
        tail = self.last_token if not self.is_prefill else self.token_ids
        return (self.seq_id, self.num_tokens, self.num_prompt_tokens, self.num_cached_tokens,
                self.num_scheduled_tokens, self.block_table, self.state_slot, self.temperature,
                self.is_prefill, tail)

    def __setstate__(self, state):
        (self.seq_id, self.num_tokens, self.num_prompt_tokens, self.num_cached_tokens,
         self.num_scheduled_tokens, self.block_table, self.state_slot, self.temperature,
         self.is_prefill, tail) = state
        if isinstance(tail, list):
            self.token_ids = tail
            self.last_token = tail[-1]
        else:
            self.token_ids = []
            self.last_token = tail
