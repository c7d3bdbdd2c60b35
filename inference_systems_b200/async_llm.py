"""Asynchronous streaming front end: ``AsyncLLMEngine``, ``RequestStream``, ``StreamOutput``.

Parity (behaviour): ``nanovllm/async_llm.py:11-199`` -- ``submit`` returns an
async iterator of outputs per request; each output carries the cumulative
completion token ids and text, so a bounded per-request queue may drop older
outputs without losing information; cancelling a stream aborts the request
and frees its KV pages and state slot; the first inference error fails every
open stream and rejects later submissions; ``close`` drains submitted work.

Design difference: the reference runs ``engine.step()`` on the event loop,
which blocks HTTP handling for the whole model step.  Here every engine call
(steps, admissions, aborts, metrics) runs on ONE dedicated engine thread, so
the event loop keeps parsing, tokenizing and streaming while the GPU works.
Requests are created (validated + tokenized) on the caller's thread and
handed to the engine thread through a lock-protected inbox that is drained
between steps; per-request snapshots are taken on the engine thread and
published to the streams on the event loop.
"""

from __future__ import annotations

import asyncio
import threading
from collections import deque
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from typing import Any

from inference_systems_b200.sampling_params import SamplingParams


@dataclass(frozen=True, slots=True)
class StreamOutput:
    request_id: int
    token_id: int                      # newest completion token (-1 before the first one)
    token_ids: tuple[int, ...]         # all completion tokens so far
    text: str                          # detokenized completion so far ("" without a tokenizer)
    finished: bool
    finish_reason: str | None = None   # "stop" | "length" | "abort"


@dataclass(frozen=True, slots=True)
class _StreamError:
    error: BaseException


class RequestStream:
    """Async iterator over one request's outputs."""

    def __init__(self, request_id: int, queue: asyncio.Queue, cancel_fn):
        self.request_id = request_id
        self._queue = queue
        self._cancel_fn = cancel_fn
        self._done = False

    def __aiter__(self):
        return self

    async def __anext__(self) -> StreamOutput:
        if self._done:
            raise StopAsyncIteration
        item = await self._queue.get()
        if item is None:
            self._done = True
            raise StopAsyncIteration
        if isinstance(item, _StreamError):
            self._done = True
            raise RuntimeError("the async engine failed while serving this request") from item.error
        if item.finished:
            self._done = True
        return item

    async def cancel(self) -> bool:
        if self._done:
            return False
        self._done = True
        return await self._cancel_fn(self.request_id)

    async def aclose(self) -> None:
        if not self._done:
            await self.cancel()


@dataclass
class _RequestState:
    queue: asyncio.Queue
    observed: int = 0


class AsyncLLMEngine:
    def __init__(self, model, stream_queue_size: int = 16, **kwargs):
        if stream_queue_size < 1:
            raise ValueError("stream_queue_size must be positive")
        from inference_systems_b200.llm import LLM

        self.engine = LLM(model, **kwargs)
        self.model_name = model if isinstance(model, str) else "model"
        self._queue_size = stream_queue_size
        self._requests: dict[int, _RequestState] = {}
        self._inbox: deque = deque()
        self._inbox_lock = threading.Lock()
        device = getattr(self.engine.model_runner, "device", None)

        def _bind_device():
            if device is not None and device.type == "cuda":
                import torch
                torch.cuda.set_device(device)

        self._executor = ThreadPoolExecutor(max_workers=1, thread_name_prefix="isb-engine", initializer=_bind_device)
        self._wakeup: asyncio.Event | None = None
        self._task: asyncio.Task | None = None
        self._closed = False
        self._failure: BaseException | None = None
        self._live: dict = {}  # engine thread only: request id -> Sequence

    @property
    def tokenizer(self):
        return self.engine.tokenizer

    # ------------------------------------------------------------ requests
    async def submit(self, prompt: str | list[int], sampling_params: SamplingParams) -> RequestStream:
        if self._closed:
            raise RuntimeError("the async engine is closed")
        if self._failure is not None:
            raise RuntimeError("the async engine has failed") from self._failure
        seq = self.engine.make_request(prompt, sampling_params)
        state = _RequestState(asyncio.Queue(maxsize=self._queue_size))
        self._requests[seq.seq_id] = state
        with self._inbox_lock:
            self._inbox.append(("add", seq))
        self._ensure_task()
        self._wakeup.set()
        return RequestStream(seq.seq_id, state.queue, self.cancel)

    async def cancel(self, request_id: int) -> bool:
        state = self._requests.pop(request_id, None)
        if state is None:
            return False
        with self._inbox_lock:
            self._inbox.append(("abort", request_id))
        if self._wakeup is not None:
            self._wakeup.set()
        self._clear(state.queue)
        state.queue.put_nowait(None)
        return True

    async def call(self, fn, *args) -> Any:
        """Run ``fn(*args)`` on the engine thread (serialised with the model steps)."""
        return await asyncio.get_running_loop().run_in_executor(self._executor, fn, *args)

    async def get_runtime_metrics(self) -> dict:
        return await self.call(self.engine.get_runtime_metrics)

    async def get_request_metrics(self) -> list[dict]:
        return await self.call(self.engine.get_request_metrics)

    async def close(self) -> None:
        """Reject new work, wait for submitted requests to finish, shut the engine down."""
        self._closed = True
        if self._wakeup is not None:
            self._wakeup.set()
        try:
            if self._task is not None:
                await self._task
        finally:
            await asyncio.get_running_loop().run_in_executor(self._executor, self.engine.exit)
            self._executor.shutdown(wait=True)
        if self._failure is not None:
            raise RuntimeError("the async engine stopped after an inference error") from self._failure

    # ---------------------------------------------------------- engine loop
    def _ensure_task(self) -> None:
        if self._wakeup is None:
            self._wakeup = asyncio.Event()
        if self._task is None:
            self._task = asyncio.get_running_loop().create_task(self._run())

    def _step_once(self) -> list[tuple]:
        """Engine thread: apply the inbox, run one step, snapshot every live request."""
        eng = self.engine
        with self._inbox_lock:
            ops = list(self._inbox)
            self._inbox.clear()
        live = {}
        for kind, arg in ops:
            if kind == "add":
                eng.scheduler.add(arg)
                live[arg.seq_id] = arg
            else:
                eng.abort_request(arg)
        self._live.update(live)
        for kind, arg in ops:
            if kind == "abort":
                self._live.pop(arg, None)
        if not eng.is_finished():
            eng.step()
        snaps = []
        eos = eng.config.eos
        for rid, seq in list(self._live.items()):
            toks = tuple(seq.completion_token_ids)
            reason = None
            if seq.is_finished:
                if seq.status.name == "ABORTED":
                    reason = "abort"
                elif toks and not seq.ignore_eos and toks[-1] == eos:
                    reason = "stop"
                else:
                    reason = "length"
                del self._live[rid]
            snaps.append((rid, toks, seq.is_finished, reason))
        return snaps

    async def _run(self) -> None:
        loop = asyncio.get_running_loop()
        try:
            while True:
                with self._inbox_lock:
                    pending = bool(self._inbox)
                if not pending and not self._live:
                    if self._closed:
                        return
                    self._wakeup.clear()
                    await self._wakeup.wait()
                    continue
                snaps = await loop.run_in_executor(self._executor, self._step_once)
                self._publish(snaps)
                await asyncio.sleep(0)
        except BaseException as e:  # noqa: BLE001 - every stream must learn about the failure
            self._failure = e
            for state in self._requests.values():
                self._clear(state.queue)
                state.queue.put_nowait(_StreamError(e))
            self._requests.clear()
            if not isinstance(e, Exception):
                raise

    def _publish(self, snaps) -> None:
        tok = self.engine.tokenizer
        for rid, toks, finished, reason in snaps:
            state = self._requests.get(rid)
            if state is None:
                continue
            if len(toks) == state.observed and not finished:
                continue
            state.observed = len(toks)
            text = tok.decode(list(toks)) if tok is not None else ""
            out = StreamOutput(rid, toks[-1] if toks else -1, toks, text, finished, reason)
            self._put_latest(state.queue, out)
            if finished:
                self._requests.pop(rid, None)

    @staticmethod
    def _clear(queue: asyncio.Queue) -> None:
        while True:
            try:
                queue.get_nowait()
            except asyncio.QueueEmpty:
                return

    @staticmethod
    def _put_latest(queue: asyncio.Queue, out: StreamOutput) -> None:
        """Outputs are cumulative, so the oldest queued one can be dropped when full."""
        while queue.full():
            queue.get_nowait()
        queue.put_nowait(out)
