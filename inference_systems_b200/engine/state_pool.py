"""GDN recurrent/conv state slots, prefix checkpoints and all-rank transactions.

Parity: ``nanovllm/engine/state_manager.py``:

* ``HybridStateManager`` (``:17-325``): fixed pools
  ``recurrent [L_gdn, slots+1, Hv, Dk, Dv] fp32`` and
  ``conv [L_gdn, slots+1, conv_dim, K-1]``; the extra slot is a scratch slot
  that padded CUDA-graph rows point at; allocate/free zero the slot;
  snapshot/restore; ReplaySSM commit.
* ``HybridPrefixCheckpointPool`` (``:328-546``): budgeted immutable copies in
  fp32 / bf16 / int8 (fp32 scale per (layer, head, key-channel)); capture,
  restore (dequantise once), free, rollback.
* ``transactional_capture/restore_prefix_checkpoint`` (``:549-640``): local
  prepare, all-reduce MIN of success, slot-id agreement (MIN == MAX), roll
  back everywhere on failure, only rank 0 raises.

Design difference: there is no gather/scatter around a forward pass -- the
kernels read and write the pools in place by slot id (the reference copies
the batch's states out and back every step, ``state_manager.py:99-143``).
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True, slots=True)
class HybridStateSnapshot:
    slot_ids: torch.Tensor
    recurrent_states: torch.Tensor
    conv_states: torch.Tensor


class HybridStateManager:
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
        n = max_num_seqs + 1
        self.recurrent_states = torch.zeros(num_linear_layers, n, num_value_heads, key_head_dim, value_head_dim,
                                            dtype=torch.float32, device=device)
        self.conv_states = torch.zeros(num_linear_layers, n, conv_dim, conv_kernel_size - 1, dtype=conv_dtype,
                                       device=device)
        self.free_slot_ids: deque[int] = deque(range(max_num_seqs))
        self.used_slot_ids: set[int] = set()

    @property
    def can_allocate(self) -> bool:
        return bool(self.free_slot_ids)

    def layer_pools(self, j: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.recurrent_states[j], self.conv_states[j]

    def _zero_slot(self, slot: int) -> None:
        self.recurrent_states[:, slot].zero_()
        self.conv_states[:, slot].zero_()

    def allocate(self, sequence=None) -> int:
        if not self.free_slot_ids:
            raise RuntimeError("no free GDN state slots")
        if sequence is not None and getattr(sequence, "state_slot", None) is not None:
            raise ValueError("sequence already owns a state slot")
        slot = self.free_slot_ids.popleft()
        self._zero_slot(slot)
        self.used_slot_ids.add(slot)
        if sequence is not None:
            sequence.state_slot = slot
        return slot

    def free(self, sequence_or_slot) -> None:
        if isinstance(sequence_or_slot, int):
            slot, seq = sequence_or_slot, None
        else:
            seq = sequence_or_slot
            slot = getattr(seq, "state_slot", None)
            if slot is None:
                return
        if slot not in self.used_slot_ids:
            raise ValueError(f"state slot {slot} is not allocated")
        self._zero_slot(slot)
        self.used_slot_ids.remove(slot)
        self.free_slot_ids.append(slot)
        if seq is not None:
            seq.state_slot = None

    def reset_scratch(self) -> None:
        self._zero_slot(self.scratch_slot_id)

    def snapshot(self, slot_ids: torch.Tensor) -> HybridStateSnapshot:
        idx = slot_ids.to(self.recurrent_states.device, torch.long)
        return HybridStateSnapshot(idx.clone(), self.recurrent_states.index_select(1, idx).clone(),
                                   self.conv_states.index_select(1, idx).clone())

    def restore(self, snap: HybridStateSnapshot) -> None:
        idx = snap.slot_ids.to(self.recurrent_states.device, torch.long)
        self.recurrent_states.index_copy_(1, idx, snap.recurrent_states.to(self.recurrent_states.dtype))
        self.conv_states.index_copy_(1, idx, snap.conv_states.to(self.conv_states.dtype))

    def restore_accepted_prefixes(self, snapshots: list[HybridStateSnapshot], accepted_lengths: torch.Tensor) -> None:
        """Row ``b`` gets ``snapshots[accepted_lengths[b]]`` (``snapshots[0]`` = pre-draft)."""
        if not snapshots:
            raise ValueError("at least the pre-draft snapshot is required")
        base = snapshots[0].slot_ids
        if accepted_lengths.numel() != base.numel():
            raise ValueError("accepted_lengths must have one value per snapshotted slot")
        for s in snapshots:
            if not torch.equal(s.slot_ids, base):
                raise ValueError("all speculative snapshots must use the same slot order")
        acc = accepted_lengths.to(torch.long).tolist()
        if any(a < 0 or a >= len(snapshots) for a in acc):
            raise ValueError("accepted length has no matching state snapshot")
        rec = torch.stack([snapshots[a].recurrent_states[:, b] for b, a in enumerate(acc)], dim=1)
        conv = torch.stack([snapshots[a].conv_states[:, b] for b, a in enumerate(acc)], dim=1)
        self.restore(HybridStateSnapshot(base, rec, conv))

    def replay_recurrent(self, slot_ids: torch.Tensor, keys: torch.Tensor, deltas: torch.Tensor,
                         log_decays: torch.Tensor, commit_lengths: torch.Tensor, *, num_steps: int) -> None:
        """Fold the accepted prefix of compact transitions into each slot's state.

        ``keys [L, B*steps, Hv, Dk]``, ``deltas [L, B*steps, Hv, Dv]``,
        ``log_decays [L, B*steps, Hv]``; row ``b`` folds its first
        ``commit_lengths[b]`` steps: ``S <- exp(g) S + k delta^T``.
        """
        from inference_systems_b200 import ops
        if num_steps <= 0:
            raise ValueError("replay requires at least one transition")
        b = slot_ids.numel()
        if commit_lengths.shape != (b,):
            raise ValueError("commit_lengths must have one value per slot")
        for t, name in ((keys, "key"), (deltas, "delta"), (log_decays, "decay")):
            if tuple(t.shape[:2]) != (self.num_linear_layers, b * num_steps):
                raise ValueError(f"replay {name} shape does not match layers x batch x steps")
        if not commit_lengths.is_cuda and bool(((commit_lengths < 1) | (commit_lengths > num_steps)).any()):
            raise ValueError("commit length is outside the replay window")
        ops.gdn_replay_commit(self.recurrent_states, slot_ids, keys, deltas, log_decays, commit_lengths, num_steps)

    def commit_conv_history(self, slot_ids: torch.Tensor, conv_history: torch.Tensor, boundaries: torch.Tensor, *,
                            num_steps: int) -> None:
        """``conv[l, slot_b] <- conv_history[l, b*steps + boundaries[b]]``."""
        from inference_systems_b200 import ops
        if conv_history.shape[0] != self.num_linear_layers:
            raise ValueError("conv history layer count does not match state pool")
        ops.gdn_conv_commit(self.conv_states, conv_history, slot_ids, boundaries, num_steps)

    def memory_bytes(self) -> int:
        return (self.recurrent_states.numel() * self.recurrent_states.element_size()
                + self.conv_states.numel() * self.conv_states.element_size())

    def bytes_per_slot(self) -> int:
        return (self.recurrent_states[:, 0].numel() * self.recurrent_states.element_size()
                + self.conv_states[:, 0].numel() * self.conv_states.element_size())


class HybridPrefixCheckpointPool:
    """Fixed-budget checkpoint copies of request states (fp32 / bf16 / int8)."""

    _DTYPES = ("fp32", "bf16", "int8")

    def __init__(self, state_manager: HybridStateManager, memory_budget_bytes: int, checkpoint_dtype: str = "fp32"):
        if checkpoint_dtype not in self._DTYPES:
            raise ValueError(f"checkpoint dtype must be one of {self._DTYPES}, got {checkpoint_dtype}")
        sm = state_manager
        self.state_manager = sm
        self.checkpoint_dtype = checkpoint_dtype
        rs, cs = sm.recurrent_states.shape, sm.conv_states.shape
        self.recurrent_shape = (rs[0], *rs[2:])
        self.conv_shape = (cs[0], *cs[2:])
        rec_elems = sm.recurrent_states[:, 0].numel()
        conv_bytes = sm.conv_states[:, 0].numel() * sm.conv_states.element_size()
        self.scale_shape = None
        scale_bytes = 0
        if checkpoint_dtype == "fp32":
            store, rec_bytes = torch.float32, rec_elems * 4
        elif checkpoint_dtype == "bf16":
            store, rec_bytes = torch.bfloat16, rec_elems * 2
        else:
            store, rec_bytes = torch.int8, rec_elems
            # one fp32 scale per (layer, head, key channel): quantise along Dv
            self.scale_shape = (*self.recurrent_shape[:3], 1)
            scale_bytes = self.scale_shape[0] * self.scale_shape[1] * self.scale_shape[2] * 4
        self.recurrent_bytes_per_checkpoint = rec_bytes
        self.scale_bytes_per_checkpoint = scale_bytes
        self.conv_bytes_per_checkpoint = conv_bytes
        self.bytes_per_checkpoint = rec_bytes + scale_bytes + conv_bytes
        self.capacity = memory_budget_bytes // self.bytes_per_checkpoint
        if self.capacity <= 0:
            raise ValueError("hybrid prefix checkpoint budget is smaller than one checkpoint: "
                             f"budget={memory_budget_bytes}, required={self.bytes_per_checkpoint}")
        dev = sm.recurrent_states.device
        self.recurrent_checkpoints = torch.zeros(self.capacity, *self.recurrent_shape, dtype=store, device=dev)
        self.recurrent_scales = (torch.zeros(self.capacity, *self.scale_shape, dtype=torch.float32, device=dev)
                                 if self.scale_shape is not None else None)
        self.conv_checkpoints = torch.zeros(self.capacity, *self.conv_shape, dtype=sm.conv_states.dtype, device=dev)
        self.free_checkpoint_slots: deque[int] = deque(range(self.capacity))
        self.used_checkpoint_slots: set[int] = set()

    @property
    def can_allocate(self) -> bool:
        return bool(self.free_checkpoint_slots)

    def _store(self, ck: int, rec: torch.Tensor, conv: torch.Tensor) -> None:
        from inference_systems_b200 import ops
        if self.checkpoint_dtype == "int8":
            ops.quantize_state_int8(rec, self.recurrent_checkpoints[ck], self.recurrent_scales[ck])
        else:
            self.recurrent_checkpoints[ck].copy_(rec)
        self.conv_checkpoints[ck].copy_(conv)

    def _zero(self, ck: int) -> None:
        self.recurrent_checkpoints[ck].zero_()
        if self.recurrent_scales is not None:
            self.recurrent_scales[ck].zero_()
        self.conv_checkpoints[ck].zero_()

    def _take(self) -> int:
        if not self.free_checkpoint_slots:
            raise RuntimeError("no free hybrid prefix checkpoint slots")
        return self.free_checkpoint_slots.popleft()

    def capture(self, request_state_slot: int) -> int:
        sm = self.state_manager
        if request_state_slot not in sm.used_slot_ids:
            raise ValueError("cannot checkpoint an unallocated request state slot")
        return self.capture_tensors(sm.recurrent_states[:, request_state_slot], sm.conv_states[:, request_state_slot])

    def capture_tensors(self, recurrent_state: torch.Tensor, conv_state: torch.Tensor) -> int:
        if tuple(recurrent_state.shape) != tuple(self.recurrent_shape):
            raise ValueError(f"internal recurrent checkpoint must have shape {self.recurrent_shape}")
        if tuple(conv_state.shape) != tuple(self.conv_shape):
            raise ValueError(f"internal conv checkpoint must have shape {self.conv_shape}")
        ck = self._take()
        try:
            self._store(ck, recurrent_state, conv_state)
        except Exception:
            self._zero(ck)
            self.free_checkpoint_slots.appendleft(ck)
            raise
        self.used_checkpoint_slots.add(ck)
        return ck

    def restore(self, checkpoint_slot: int, request_state_slot: int) -> None:
        from inference_systems_b200 import ops
        sm = self.state_manager
        if checkpoint_slot not in self.used_checkpoint_slots:
            raise ValueError("hybrid prefix checkpoint slot is not allocated")
        if request_state_slot not in sm.used_slot_ids:
            raise ValueError("request state slot is not allocated")
        dst = sm.recurrent_states[:, request_state_slot]
        if self.checkpoint_dtype == "int8":
            ops.dequantize_state_int8(self.recurrent_checkpoints[checkpoint_slot],
                                      self.recurrent_scales[checkpoint_slot], dst)
        else:
            dst.copy_(self.recurrent_checkpoints[checkpoint_slot])
        sm.conv_states[:, request_state_slot].copy_(self.conv_checkpoints[checkpoint_slot])

    def free(self, checkpoint_slot: int) -> None:
        if checkpoint_slot not in self.used_checkpoint_slots:
            raise ValueError("hybrid prefix checkpoint slot is not allocated")
        self._zero(checkpoint_slot)
        self.used_checkpoint_slots.remove(checkpoint_slot)
        self.free_checkpoint_slots.append(checkpoint_slot)

    def rollback_capture(self, checkpoint_slot: int) -> None:
        """Undo an unpublished capture and restore the deterministic free order."""
        if checkpoint_slot not in self.used_checkpoint_slots:
            raise ValueError("hybrid prefix checkpoint slot is not allocated")
        self._zero(checkpoint_slot)
        self.used_checkpoint_slots.remove(checkpoint_slot)
        self.free_checkpoint_slots = deque(sorted([*self.free_checkpoint_slots, checkpoint_slot]))

    def memory_bytes(self) -> int:
        n = self.recurrent_checkpoints.numel() * self.recurrent_checkpoints.element_size()
        if self.recurrent_scales is not None:
            n += self.recurrent_scales.numel() * 4
        return n + self.conv_checkpoints.numel() * self.conv_checkpoints.element_size()


# ------------------------------------------------------------ transactions
def _consensus_device(ref: torch.Tensor) -> torch.device:
    if dist.is_initialized() and dist.get_backend() == "nccl":
        return ref.device
    return torch.device("cpu")


def _multi_rank() -> bool:
    return dist.is_initialized() and dist.get_world_size() > 1


def _all_ok(ok: bool, ref: torch.Tensor) -> bool:
    flag = torch.tensor(1 if ok else 0, dtype=torch.int32, device=_consensus_device(ref))
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return int(flag.item()) == 1


def _same_everywhere(value: int, ref: torch.Tensor) -> bool:
    dev = _consensus_device(ref)
    lo = torch.tensor(value, dtype=torch.int64, device=dev)
    hi = lo.clone()
    dist.all_reduce(lo, op=dist.ReduceOp.MIN)
    dist.all_reduce(hi, op=dist.ReduceOp.MAX)
    return int(lo.item()) == int(hi.item())


def transactional_capture_prefix_checkpoint(pool: HybridPrefixCheckpointPool, request_state_slot: int, *,
                                            recurrent_state: torch.Tensor | None = None,
                                            conv_state: torch.Tensor | None = None) -> int:
    """Capture on every rank or on none; returns the agreed slot (-1 on non-zero ranks after failure)."""
    slot, err = None, None
    try:
        if recurrent_state is None and conv_state is None:
            slot = pool.capture(request_state_slot)
        elif recurrent_state is not None and conv_state is not None:
            slot = pool.capture_tensors(recurrent_state, conv_state)
        else:
            raise ValueError("both internal checkpoint tensors are required")
    except Exception as exc:  # join the vote before raising
        err = exc
    if not _multi_rank():
        if err is not None:
            raise err
        return slot
    ref = pool.recurrent_checkpoints
    if not _all_ok(err is None, ref):
        if slot is not None:
            pool.rollback_capture(slot)
        if dist.get_rank() == 0:
            raise RuntimeError("hybrid prefix capture rolled back on all ranks")
        return -1
    if not _same_everywhere(slot, ref):
        pool.rollback_capture(slot)
        if dist.get_rank() == 0:
            raise RuntimeError("hybrid prefix checkpoint slot IDs diverged across ranks")
        return -1
    return slot


def transactional_restore_prefix_checkpoint(pool: HybridPrefixCheckpointPool, checkpoint_slot: int,
                                            request_state_slot: int) -> None:
    """Restore on every rank or roll every rank back to the pre-restore state."""
    sm = pool.state_manager
    rec_backup = sm.recurrent_states[:, request_state_slot].clone()
    conv_backup = sm.conv_states[:, request_state_slot].clone()
    err = None
    try:
        pool.restore(checkpoint_slot, request_state_slot)
    except Exception as exc:
        err = exc
    ok = _all_ok(err is None, pool.recurrent_checkpoints) if _multi_rank() else err is None
    if not ok:
        sm.recurrent_states[:, request_state_slot].copy_(rec_backup)
        sm.conv_states[:, request_state_slot].copy_(conv_backup)
        if not dist.is_initialized() or dist.get_rank() == 0:
            raise RuntimeError("hybrid prefix restore rolled back on all ranks")
