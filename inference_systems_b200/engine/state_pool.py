"""GDN recurrent/conv state slots, prefix checkpoints and all-rank checkpoint transactions.

Behavioural parity with ``nanovllm/engine/state_manager.py``: a fixed pool of
per-request recurrent (fp32) and conv states with one extra scratch slot for
CUDA-graph padding rows (``:17-325``); a memory-budgeted pool of immutable
prefix checkpoints stored as fp32, bf16 or int8 with fp32 scales per
(layer, head, key channel) (``:328-546``); capture and restore as all-rank
transactions that either happen on every tensor-parallel rank or on none, with
only rank 0 raising (``:549-640``).

Design (this module's own):
* Kernels read and write the state pools in place by slot id; nothing is
  gathered into or scattered out of a batch tensor around a forward pass.
* ``SlotAllocator`` hands out the smallest free id (a heap), so every rank
  allocates the same ids in the same order and a rolled-back capture simply
  returns its id -- no queue order to restore.
* Checkpoint storage formats are codec objects (``Fp32Codec``, ``Bf16Codec``,
  ``Int8Codec``) that own their tensors; the pool only manages slots and budget.
* ``RankVote`` wraps the consensus collectives (all-reduce MIN for "everyone
  succeeded", MIN == MAX for "everyone chose the same slot"), on the NCCL group
  when it is the default, else on CPU tensors over gloo.
"""

from __future__ import annotations

import heapq

import torch
import torch.distributed as dist


class SlotAllocator:
    """Ids ``0..n-1``; allocation takes the smallest free id."""

    def __init__(self, n: int):
        self._free = list(range(n))
        self.used: set[int] = set()

    def __len__(self) -> int:
        return len(self._free)

    def take(self) -> int:
        if not self._free:
            raise RuntimeError("no free slots")
        slot = heapq.heappop(self._free)
        self.used.add(slot)
        return slot

    def give_back(self, slot: int) -> None:
        if slot not in self.used:
            raise ValueError(f"slot {slot} is not allocated")
        self.used.remove(slot)
        heapq.heappush(self._free, slot)


class HybridStateManager:
    """``recurrent [L_gdn, slots + 1, Hv, Dk, Dv]`` fp32 and ``conv [L_gdn, slots + 1, conv_dim, K - 1]``
    pools; slot ``slots`` is the scratch slot that padded rows of a captured batch point at."""

    def __init__(self, *, max_num_seqs: int, num_linear_layers: int, num_value_heads: int, key_head_dim: int,
                 value_head_dim: int, conv_dim: int, conv_kernel_size: int, conv_dtype: torch.dtype,
                 device: torch.device | str):
        if max_num_seqs <= 0 or num_linear_layers <= 0:
            raise ValueError("state pool dimensions must be positive")
        if conv_kernel_size < 2:
            raise ValueError("conv_kernel_size must be at least two")
        self.max_num_seqs = max_num_seqs
        self.num_linear_layers = num_linear_layers
        self.scratch_slot_id = max_num_seqs
        self.recurrent_states = torch.zeros(num_linear_layers, max_num_seqs + 1, num_value_heads, key_head_dim,
                                            value_head_dim, dtype=torch.float32, device=device)
        self.conv_states = torch.zeros(num_linear_layers, max_num_seqs + 1, conv_dim, conv_kernel_size - 1,
                                       dtype=conv_dtype, device=device)
        self.slots = SlotAllocator(max_num_seqs)

    @property
    def can_allocate(self) -> bool:
        return len(self.slots) > 0

    @property
    def used_slot_ids(self) -> set[int]:
        return self.slots.used

    def layer_pools(self, j: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.recurrent_states[j], self.conv_states[j]

    def clear_slot(self, slot: int) -> None:
        self.recurrent_states[:, slot].zero_()
        self.conv_states[:, slot].zero_()

    def allocate(self, sequence=None) -> int:
        """A zeroed slot (assigned to ``sequence.state_slot`` when given)."""
        if sequence is not None and getattr(sequence, "state_slot", None) is not None:
            raise ValueError("sequence already owns a state slot")
        if not self.can_allocate:
            raise RuntimeError("no free GDN state slots")
        slot = self.slots.take()
        self.clear_slot(slot)
        if sequence is not None:
            sequence.state_slot = slot
        return slot

    def free(self, sequence_or_slot) -> None:
        """Zero and release a slot (given directly or as ``sequence.state_slot``)."""
        seq = None if isinstance(sequence_or_slot, int) else sequence_or_slot
        slot = sequence_or_slot if seq is None else getattr(seq, "state_slot", None)
        if slot is None:
            return
        if slot not in self.slots.used:
            raise ValueError(f"state slot {slot} is not allocated")
        self.clear_slot(slot)
        self.slots.give_back(slot)
        if seq is not None:
            seq.state_slot = None

    def reset_scratch(self) -> None:
        self.clear_slot(self.scratch_slot_id)

    def memory_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.recurrent_states, self.conv_states))

    def bytes_per_slot(self) -> int:
        return sum(t[:, 0].numel() * t.element_size() for t in (self.recurrent_states, self.conv_states))


# -------------------------------------------------------------------- checkpoint codecs


class Fp32Codec:
    name, dtype = "fp32", torch.float32

    def __init__(self, capacity: int, shape: tuple[int, ...], device):
        self.data = torch.zeros(capacity, *shape, dtype=self.dtype, device=device)

    @classmethod
    def bytes_per(cls, shape: tuple[int, ...]) -> int:
        n = 1
        for d in shape:
            n *= d
        return n * torch.tensor([], dtype=cls.dtype).element_size()

    def encode(self, slot: int, state: torch.Tensor) -> None:
        self.data[slot].copy_(state)

    def decode(self, slot: int, out: torch.Tensor) -> None:
        out.copy_(self.data[slot])

    def clear(self, slot: int) -> None:
        self.data[slot].zero_()

    def nbytes(self) -> int:
        return self.data.numel() * self.data.element_size()


class Bf16Codec(Fp32Codec):
    name, dtype = "bf16", torch.bfloat16


class Int8Codec(Fp32Codec):
    """int8 values with one fp32 scale per (layer, head, key channel): quantised along Dv."""

    name, dtype = "int8", torch.int8

    def __init__(self, capacity: int, shape: tuple[int, ...], device):
        super().__init__(capacity, shape, device)
        self.scales = torch.zeros(capacity, *shape[:-1], 1, dtype=torch.float32, device=device)

    @classmethod
    def bytes_per(cls, shape: tuple[int, ...]) -> int:
        rows = 1
        for d in shape[:-1]:
            rows *= d
        return rows * shape[-1] + rows * 4

    def encode(self, slot: int, state: torch.Tensor) -> None:
        from inference_systems_b200 import ops
        ops.quantize_state_int8(state, self.data[slot], self.scales[slot])

    def decode(self, slot: int, out: torch.Tensor) -> None:
        from inference_systems_b200 import ops
        ops.dequantize_state_int8(self.data[slot], self.scales[slot], out)

    def clear(self, slot: int) -> None:
        super().clear(slot)
        self.scales[slot].zero_()

    def nbytes(self) -> int:
        return super().nbytes() + self.scales.numel() * 4


_CODECS = {c.name: c for c in (Fp32Codec, Bf16Codec, Int8Codec)}


class HybridPrefixCheckpointPool:
    """Immutable checkpoint copies of request states within a memory budget."""

    def __init__(self, state_manager: HybridStateManager, memory_budget_bytes: int, checkpoint_dtype: str = "fp32"):
        if checkpoint_dtype not in _CODECS:
            raise ValueError(f"checkpoint dtype must be one of {tuple(_CODECS)}, got {checkpoint_dtype}")
        sm = self.state_manager = state_manager
        self.checkpoint_dtype = checkpoint_dtype
        self.recurrent_shape = (sm.recurrent_states.shape[0], *sm.recurrent_states.shape[2:])
        self.conv_shape = (sm.conv_states.shape[0], *sm.conv_states.shape[2:])
        codec = _CODECS[checkpoint_dtype]
        conv_bytes = sm.conv_states[:, 0].numel() * sm.conv_states.element_size()
        self.bytes_per_checkpoint = codec.bytes_per(self.recurrent_shape) + conv_bytes
        self.capacity = memory_budget_bytes // self.bytes_per_checkpoint
        if self.capacity <= 0:
            raise ValueError("hybrid prefix checkpoint budget is smaller than one checkpoint: "
                             f"budget={memory_budget_bytes}, required={self.bytes_per_checkpoint}")
        dev = sm.recurrent_states.device
        self.recurrent = codec(self.capacity, self.recurrent_shape, dev)
        self.conv = torch.zeros(self.capacity, *self.conv_shape, dtype=sm.conv_states.dtype, device=dev)
        self.slots = SlotAllocator(self.capacity)

    @property
    def can_allocate(self) -> bool:
        return len(self.slots) > 0

    @property
    def used_checkpoint_slots(self) -> set[int]:
        return self.slots.used

    @property
    def free_checkpoint_slots(self) -> int:
        return len(self.slots)

    def capture(self, request_state_slot: int) -> int:
        """Checkpoint the current state of a request's slot; returns the checkpoint slot."""
        sm = self.state_manager
        if request_state_slot not in sm.used_slot_ids:
            raise ValueError("cannot checkpoint an unallocated request state slot")
        return self.capture_tensors(sm.recurrent_states[:, request_state_slot], sm.conv_states[:, request_state_slot])

    def capture_tensors(self, recurrent_state: torch.Tensor, conv_state: torch.Tensor) -> int:
        """Checkpoint explicit state tensors (states recorded inside a prefill chunk)."""
        if tuple(recurrent_state.shape) != self.recurrent_shape:
            raise ValueError(f"internal recurrent checkpoint must have shape {self.recurrent_shape}")
        if tuple(conv_state.shape) != self.conv_shape:
            raise ValueError(f"internal conv checkpoint must have shape {self.conv_shape}")
        if not self.can_allocate:
            raise RuntimeError("no free hybrid prefix checkpoint slots")
        ck = self.slots.take()
        try:
            self.recurrent.encode(ck, recurrent_state)
            self.conv[ck].copy_(conv_state)
        except Exception:
            self._clear(ck)
            self.slots.give_back(ck)
            raise
        return ck

    def restore(self, checkpoint_slot: int, request_state_slot: int) -> None:
        sm = self.state_manager
        if checkpoint_slot not in self.slots.used:
            raise ValueError("hybrid prefix checkpoint slot is not allocated")
        if request_state_slot not in sm.used_slot_ids:
            raise ValueError("request state slot is not allocated")
        self.recurrent.decode(checkpoint_slot, sm.recurrent_states[:, request_state_slot])
        sm.conv_states[:, request_state_slot].copy_(self.conv[checkpoint_slot])

    def _clear(self, ck: int) -> None:
        self.recurrent.clear(ck)
        self.conv[ck].zero_()

    def free(self, checkpoint_slot: int) -> None:
        if checkpoint_slot not in self.slots.used:
            raise ValueError("hybrid prefix checkpoint slot is not allocated")
        self._clear(checkpoint_slot)
        self.slots.give_back(checkpoint_slot)

    # an unpublished capture is undone exactly like an eviction (the allocator keeps the order)
    rollback_capture = free

    def memory_bytes(self) -> int:
        return self.recurrent.nbytes() + self.conv.numel() * self.conv.element_size()


# ------------------------------------------------------------------------ transactions


class RankVote:
    """Consensus over the default process group (a no-op with one rank)."""

    def __init__(self, like: torch.Tensor):
        self.active = dist.is_initialized() and dist.get_world_size() > 1
        nccl = self.active and dist.get_backend() == "nccl"
        self.device = like.device if nccl else torch.device("cpu")
        self.rank = dist.get_rank() if dist.is_initialized() else 0

    def all_ok(self, ok: bool) -> bool:
        if not self.active:
            return ok
        t = torch.tensor(int(ok), dtype=torch.int32, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        return bool(t.item())

    def all_equal(self, value: int) -> bool:
        if not self.active:
            return True
        lo = torch.tensor(value, dtype=torch.int64, device=self.device)
        hi = lo.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        return int(lo.item()) == int(hi.item())


def transactional_capture_prefix_checkpoint(pool: HybridPrefixCheckpointPool, request_state_slot: int, *,
                                            recurrent_state: torch.Tensor | None = None,
                                            conv_state: torch.Tensor | None = None) -> int:
    """Capture on every rank or on none.  Every rank votes before anyone raises; on failure every
    rank rolls back and rank 0 raises (other ranks return -1).  Ranks must agree on the slot id."""
    vote = RankVote(pool.conv)
    slot, error = None, None
    try:
        if (recurrent_state is None) != (conv_state is None):
            raise ValueError("both internal checkpoint tensors are required")
        slot = (pool.capture(request_state_slot) if recurrent_state is None
                else pool.capture_tensors(recurrent_state, conv_state))
    except Exception as exc:  # noqa: BLE001 - voted on below
        error = exc
    if not vote.active:
        if error is not None:
            raise error
        return slot
    if not vote.all_ok(error is None):
        if slot is not None:
            pool.rollback_capture(slot)
        if vote.rank == 0:
            raise RuntimeError("hybrid prefix capture rolled back on all ranks") from error
        return -1
    if not vote.all_equal(slot):
        pool.rollback_capture(slot)
        if vote.rank == 0:
            raise RuntimeError("hybrid prefix checkpoint slot IDs diverged across ranks")
        return -1
    return slot


def transactional_restore_prefix_checkpoint(pool: HybridPrefixCheckpointPool, checkpoint_slot: int,
                                            request_state_slot: int) -> None:
    """Restore on every rank, or put every rank's slot back as it was (rank 0 raises)."""
    sm = pool.state_manager
    vote = RankVote(pool.conv)
    saved = (sm.recurrent_states[:, request_state_slot].clone(), sm.conv_states[:, request_state_slot].clone())
    error = None
    try:
        pool.restore(checkpoint_slot, request_state_slot)
    except Exception as exc:  # noqa: BLE001 - voted on below
        error = exc
    if vote.all_ok(error is None):
        return
    sm.recurrent_states[:, request_state_slot].copy_(saved[0])
    sm.conv_states[:, request_state_slot].copy_(saved[1])
    if vote.rank == 0:
        raise RuntimeError("hybrid prefix restore rolled back on all ranks") from error
