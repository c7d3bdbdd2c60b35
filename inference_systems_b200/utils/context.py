"""Per-step batch metadata handed to every layer.

Parity: the reference keeps the same facts in a module-global ``Context``
(``nanovllm/utils/context.py:5-28``: ``is_prefill, cu_seqlens_q/k,
max_seqlen_q/k, slot_mapping, context_lens, block_tables, state_slot_ids``).
Here it is an explicit object passed down the forward call, so several
batches (target, MTP draft, verify) can be in flight without global state and
CUDA-graph captures own their static copies.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class ForwardBatch:
    is_prefill: bool
    input_ids: torch.Tensor            # [T] int64
    positions: torch.Tensor            # [T] int64
    cu_seqlens_q: torch.Tensor         # [B+1] int32 (device)
    context_lens: torch.Tensor         # [B] int32: tokens visible after this step
    block_tables: torch.Tensor         # [B, max_blocks] int32 (-1 padded)
    slot_mapping: torch.Tensor         # [T] int32 (-1 = do not store)
    state_slots: torch.Tensor          # [B] int32 GDN state-slot ids
    logits_indices: torch.Tensor       # [B] int64: row of each sequence's last token
    max_seqlen_q: int = 1
    max_seqlen_k: int = 1
    cu_seqlens_host: list[int] = field(default_factory=list)
    slots_host: list[int] = field(default_factory=list)
    num_seqs: int = 0
    # GDN states after selected tokens (hybrid prefix checkpoints inside a prefill chunk):
    # {"rows": [T] int32 (-1 = none), "rec": per-layer [R, Hv, Dk, Dv] fp32, "conv": per-layer [R, C, K-1]}
    gdn_history: dict | None = None
    # MTP verify: per GDN layer (rec_k, rec_delta, rec_g, conv_hist) record buffers; the
    # slot pools are then left untouched (see ops.gdn_verify)
    gdn_verify: list | None = None
    # Few query rows per sequence over a long cached context (MTP verify / catch-up): per-row
    # (context length [T] int32, block-table row [T, max_blocks] int32) so attention runs every
    # row as an independent split-KV decode query (causal by each row's own context length)
    decode_rows: tuple | None = None

    @property
    def num_tokens(self) -> int:
        return int(self.input_ids.shape[0])
