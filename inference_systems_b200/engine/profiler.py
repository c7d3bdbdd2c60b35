"""Opt-in phase timing for the engine, and a kernel-time table for captured steps.

Behavioural parity with ``nanovllm/engine/phase_profiler.py:40-138``: named
phases timed on the host and (optionally) on the device, free-form counters,
one device synchronisation per ``flush``, per-phase summary statistics under
the same metric keys (``count, total, mean, median, p95, q1, q3``).

Design:
* Every phase name owns a ``Series`` (samples in a growable float64 array,
  summarised with numpy on demand).
* Device timing reuses CUDA events from a small free list instead of creating
  two events per phase; a span records its pair and the pair goes back to the
  free list when ``flush`` has read it.
* A disabled profiler returns a shared no-op context, so an instrumented call
  site costs one attribute test.
* ``kernel_time_table`` profiles replays of a captured step with CUPTI
  (``torch.profiler``) and renders per-kernel device time and share; the
  runner exposes it on every tensor-parallel rank at once.
"""

from __future__ import annotations

import contextlib
from time import perf_counter_ns

import numpy as np
import torch


class Series:
    """Samples of one quantity (ms or bytes)."""

    __slots__ = ("_v", "_n")

    def __init__(self):
        self._v = np.empty(16, dtype=np.float64)
        self._n = 0

    def add(self, x: float) -> None:
        if self._n == self._v.shape[0]:
            self._v = np.concatenate((self._v, np.empty_like(self._v)))
        self._v[self._n] = x
        self._n += 1

    def summary(self) -> dict:
        if self._n == 0:
            return {"count": 0, "total": 0.0, "mean": 0.0, "median": 0.0, "p95": 0.0, "q1": 0.0, "q3": 0.0}
        v = np.sort(self._v[: self._n])
        n = self._n
        # order statistics at fixed ranks (no interpolation): robust for a handful of samples
        return {"count": n, "total": float(v.sum()), "mean": float(v.mean()), "median": float(np.median(v)),
                "p95": float(v[min(int(n * 0.95), n - 1)]), "q1": float(v[n // 4]), "q3": float(v[(3 * n) // 4])}


class _Span:
    """One timed phase: host clock, optional CUDA event pair, NVTX / record_function ranges."""

    __slots__ = ("prof", "name", "gpu", "events", "t0", "mem0", "rf")

    def __init__(self, prof: "PhaseProfiler", name: str, gpu: bool):
        self.prof, self.name, self.gpu = prof, name, gpu

    def __enter__(self):
        p = self.prof
        self.events = p._take_events() if self.gpu else None
        if self.events is not None:
            self.mem0 = torch.cuda.memory_allocated()
            self.events[0].record()
        if p._cuda:
            torch.cuda.nvtx.range_push(self.name)
        self.rf = torch.profiler.record_function(self.name)
        self.rf.__enter__()
        self.t0 = perf_counter_ns()
        return self

    def __exit__(self, *exc):
        p = self.prof
        p._series(p.cpu_ms, self.name).add((perf_counter_ns() - self.t0) / 1e6)
        self.rf.__exit__(None, None, None)
        if p._cuda:
            torch.cuda.nvtx.range_pop()
        if self.events is not None:
            self.events[1].record()
            p._series(p.allocated_delta_bytes, self.name).add(float(torch.cuda.memory_allocated() - self.mem0))
            p._inflight.append((self.name, self.events))
        return False


_NOOP = contextlib.nullcontext()


class PhaseProfiler:
    def __init__(self, enabled: bool = False):
        self.enabled = bool(enabled)
        self._cuda = torch.cuda.is_available()
        self._free_events: list[tuple[torch.cuda.Event, torch.cuda.Event]] = []
        self.reset()

    def reset(self) -> None:
        self.cpu_ms: dict[str, Series] = {}
        self.gpu_ms: dict[str, Series] = {}
        self.allocated_delta_bytes: dict[str, Series] = {}
        self.counters: dict[str, float] = {}
        self._inflight: list[tuple[str, tuple]] = []
        self.flush_count = 0
        self.flush_sync_ms = 0.0

    @staticmethod
    def _series(table: dict, name: str) -> Series:
        s = table.get(name)
        if s is None:
            s = table[name] = Series()
        return s

    def _take_events(self):
        if not self._cuda:
            return None
        if self._free_events:
            return self._free_events.pop()
        return (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))

    def phase(self, name: str, *, gpu: bool = True):
        """Context manager timing ``name`` on the host and, with ``gpu``, on the current stream."""
        if not self.enabled:
            return _NOOP
        return _Span(self, name, gpu)

    def record_cpu(self, name: str, elapsed_ms: float) -> None:
        if self.enabled:
            self._series(self.cpu_ms, name).add(float(elapsed_ms))

    def add_counter(self, name: str, value: float) -> None:
        if self.enabled:
            self.counters[name] = self.counters.get(name, 0.0) + float(value)

    def set_counter(self, name: str, value: float) -> None:
        if self.enabled:
            self.counters[name] = float(value)

    def flush(self) -> None:
        """Resolve every recorded event pair with one device synchronisation."""
        if not self.enabled or not self._inflight:
            return
        t0 = perf_counter_ns()
        torch.cuda.synchronize()
        self.flush_sync_ms += (perf_counter_ns() - t0) / 1e6
        self.flush_count += 1
        for name, (a, b) in self._inflight:
            self._series(self.gpu_ms, name).add(float(a.elapsed_time(b)))
            self._free_events.append((a, b))
        self._inflight.clear()

    def metrics(self) -> dict:
        empty = Series()
        names = sorted(set(self.cpu_ms) | set(self.gpu_ms))
        return {
            "enabled": self.enabled,
            "flush_count": self.flush_count,
            "flush_sync_ms": self.flush_sync_ms,
            "counters": dict(sorted(self.counters.items())),
            "phases": {n: {"cpu_ms": self.cpu_ms.get(n, empty).summary(),
                           "gpu_ms": self.gpu_ms.get(n, empty).summary(),
                           "allocated_delta_bytes": self.allocated_delta_bytes.get(n, empty).summary()}
                       for n in names},
        }


def kernel_time_table(run, n: int = 3) -> str:
    """Per-kernel device time of ``n`` calls of ``run`` (CUPTI through torch.profiler), as text.

    Kernels launched with programmatic dependent launch start before their
    predecessor ends, so a kernel's span includes the time it waited inside
    ``griddepcontrol.wait``: read the shares as upper bounds per kernel.
    """
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(n):
            run()
        torch.cuda.synchronize()
    per_kernel: dict[str, list[float]] = {}
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            us = ev.device_time_total if hasattr(ev, "device_time_total") else ev.cuda_time_total
            per_kernel.setdefault(ev.name, []).append(us)
    total = sum(sum(v) for v in per_kernel.values()) or 1.0
    lines = [f"total device us per call: {total / n:.1f}"]
    for name, v in sorted(per_kernel.items(), key=lambda kv: -sum(kv[1])):
        lines.append(f"{sum(v) / n:10.1f} us  {100 * sum(v) / total:5.1f}%  x{len(v) // n:<4d} {name[:160]}")
    return "\n".join(lines) + "\n"
