"""Opt-in phase profiler: CPU wall time plus deferred CUDA-event timing.

Parity: ``nanovllm/engine/phase_profiler.py:40-138`` -- ``phase(name)``
context (NVTX range + ``record_function`` + CUDA events resolved later),
``record_cpu``, counters, one device synchronisation per ``flush``, summary
statistics per phase.  Disabled profilers cost one attribute test per phase.
"""

from __future__ import annotations

from contextlib import contextmanager
from statistics import median
from time import perf_counter_ns

import torch
from torch.profiler import record_function


def summarize(values: list[float]) -> dict:
    if not values:
        return {"count": 0, "total": 0.0, "mean": 0.0, "median": 0.0, "p95": 0.0, "q1": 0.0, "q3": 0.0}
    s = sorted(values)
    n = len(s)
    return {"count": n, "total": sum(s), "mean": sum(s) / n, "median": median(s),
            "p95": s[min(int(n * 0.95), n - 1)], "q1": s[n // 4], "q3": s[(3 * n) // 4]}


class PhaseProfiler:
    def __init__(self, enabled: bool = False):
        self.enabled = enabled
        self.reset()

    def reset(self) -> None:
        self.cpu_ms: dict[str, list[float]] = {}
        self.gpu_ms: dict[str, list[float]] = {}
        self.allocated_delta_bytes: dict[str, list[float]] = {}
        self.counters: dict[str, float] = {}
        self._pending: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []
        self.flush_count = 0
        self.flush_sync_ms = 0.0

    @contextmanager
    def phase(self, name: str, *, gpu: bool = True):
        if not self.enabled:
            yield
            return
        cuda = torch.cuda.is_available()
        timed = gpu and cuda
        if timed:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            mem0 = torch.cuda.memory_allocated()
            ev0.record()
        if cuda:
            torch.cuda.nvtx.range_push(name)
        rf = record_function(name)
        rf.__enter__()
        t0 = perf_counter_ns()
        try:
            yield
        finally:
            rf.__exit__(None, None, None)
            if cuda:
                torch.cuda.nvtx.range_pop()
            self.cpu_ms.setdefault(name, []).append((perf_counter_ns() - t0) / 1e6)
            if timed:
                ev1.record()
                self.allocated_delta_bytes.setdefault(name, []).append(float(torch.cuda.memory_allocated() - mem0))
                self._pending.append((name, ev0, ev1))

    def record_cpu(self, name: str, elapsed_ms: float) -> None:
        if self.enabled:
            self.cpu_ms.setdefault(name, []).append(float(elapsed_ms))

    def add_counter(self, name: str, value: float) -> None:
        if self.enabled:
            self.counters[name] = self.counters.get(name, 0.0) + float(value)

    def set_counter(self, name: str, value: float) -> None:
        if self.enabled:
            self.counters[name] = float(value)

    def flush(self) -> None:
        if not self.enabled or not self._pending:
            return
        t0 = perf_counter_ns()
        torch.cuda.synchronize()
        self.flush_sync_ms += (perf_counter_ns() - t0) / 1e6
        self.flush_count += 1
        for name, a, b in self._pending:
            self.gpu_ms.setdefault(name, []).append(float(a.elapsed_time(b)))
        self._pending.clear()

    def metrics(self) -> dict:
        names = sorted(set(self.cpu_ms) | set(self.gpu_ms))
        return {
            "enabled": self.enabled,
            "flush_count": self.flush_count,
            "flush_sync_ms": self.flush_sync_ms,
            "counters": dict(sorted(self.counters.items())),
            "phases": {n: {"cpu_ms": summarize(self.cpu_ms.get(n, [])),
                           "gpu_ms": summarize(self.gpu_ms.get(n, [])),
                           "allocated_delta_bytes": summarize(self.allocated_delta_bytes.get(n, []))}
                       for n in names},
        }
