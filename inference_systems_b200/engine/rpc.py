"""Rank-0 -> worker command channel over POSIX shared memory.

Parity: the reference ships pickled ``[method, *args]`` through a 1 MiB
``SharedMemory`` segment guarded by one event per worker plus an ack event
(``nanovllm/engine/model_runner.py:139-197``).  This channel works for both
spawned workers and independently launched ranks (``torchrun``): the header
holds a command sequence number and one ack counter per worker; workers poll
the sequence number with a short back-off, so no inherited ``mp.Event`` is
needed.  Payloads larger than the segment are rejected loudly.

Layout: ``[u64 seq][u64 nbytes][u64 ack * W][payload...]``.
"""

from __future__ import annotations

import pickle
import struct
import time
from multiprocessing import shared_memory

_HDR = 16


class CommandChannel:
    def __init__(self, name: str, world_size: int, rank: int, size: int = 1 << 22, create: bool | None = None):
        self.rank, self.workers = rank, world_size - 1
        self.size = size
        self.payload_off = _HDR + 8 * max(self.workers, 1)
        create = (rank == 0) if create is None else create
        if create:
            try:
                stale = shared_memory.SharedMemory(name=name)
                stale.close()
                stale.unlink()
            except FileNotFoundError:
                pass
            self.shm = shared_memory.SharedMemory(name=name, create=True, size=size)
            self.shm.buf[: self.payload_off] = bytes(self.payload_off)
        else:
            deadline = time.monotonic() + 120
            while True:
                try:
                    self.shm = shared_memory.SharedMemory(name=name)
                    break
                except FileNotFoundError:
                    if time.monotonic() > deadline:
                        raise
                    time.sleep(0.01)
            # Attaching registers the segment with this process's resource tracker, which would
            # unlink (or report as leaked) a segment that rank 0 owns and unlinks itself.  A worker
            # spawned by rank 0 shares rank 0's tracker (the registration is rank 0's own, which its
            # unlink removes); only an independently launched worker (torchrun) has a tracker of
            # its own to take the name out of.
            import multiprocessing as mp

            if mp.parent_process() is None:
                try:
                    from multiprocessing import resource_tracker
                    resource_tracker.unregister(self.shm._name, "shared_memory")
                except Exception:  # noqa: BLE001 - tracker internals differ across Python versions
                    pass
        self.owner = create
        self.seq = 0

    def _u64(self, off: int) -> int:
        return struct.unpack_from("<Q", self.shm.buf, off)[0]

    def _put_u64(self, off: int, v: int) -> None:
        struct.pack_into("<Q", self.shm.buf, off, v)

    def send(self, method: str, *args, timeout_s: float = 600.0) -> None:
        """Rank 0: wait until every worker consumed the previous command, then publish."""
        data = pickle.dumps((method, args), protocol=pickle.HIGHEST_PROTOCOL)
        if self.payload_off + len(data) > self.size:
            raise ValueError(f"RPC payload of {len(data)} bytes exceeds the {self.size}-byte channel")
        deadline = time.monotonic() + timeout_s
        spins = 0
        while any(self._u64(_HDR + 8 * w) != self.seq for w in range(self.workers)):
            spins += 1
            if spins > 1000:
                time.sleep(2e-5)
                if time.monotonic() > deadline:
                    raise TimeoutError("a worker rank stopped acknowledging commands")
        self.shm.buf[self.payload_off: self.payload_off + len(data)] = data
        self._put_u64(8, len(data))
        self.seq += 1
        self._put_u64(0, self.seq)

    def recv(self, timeout_s: float | None = None):
        """Worker: block until the next command; returns ``(method, args)``."""
        target = self.seq + 1
        deadline = None if timeout_s is None else time.monotonic() + timeout_s
        spins = 0
        while self._u64(0) != target:
            spins += 1
            if spins > 1000:
                time.sleep(2e-5)
                if deadline is not None and time.monotonic() > deadline:
                    raise TimeoutError("rank 0 sent no command in time")
        n = self._u64(8)
        method, args = pickle.loads(bytes(self.shm.buf[self.payload_off: self.payload_off + n]))
        self.seq = target
        self._put_u64(_HDR + 8 * (self.rank - 1), target)
        return method, args

    def close(self) -> None:
        try:
            self.shm.close()
            if self.owner:
                self.shm.unlink()
        except (FileNotFoundError, BufferError):
            pass
