"""Greedy speculative-decoding verification helpers.

Parity: ``nanovllm/engine/speculative.py:8-129`` -- accept the longest
proposal prefix that matches the target's greedy tokens and emit the
target's token at the first mismatch (or the bonus token after a full
accept); the commit plan advances the context by the accepted length only.

On the device path the same rule runs as a few tensor ops
(``accept_lengths``) so the runner never syncs per scalar.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True, slots=True)
class GreedyVerificationResult:
    accepted_lengths: torch.Tensor
    output_tokens: list[list[int]]


@dataclass(frozen=True, slots=True)
class GreedyCommitPlan:
    accepted_lengths: torch.Tensor
    committed_context_lengths: torch.Tensor
    emitted_tokens: list[list[int]]
    replacement_tokens_require_decode: torch.Tensor


def accept_lengths(proposals: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Per row, the number of leading positions where ``proposals == targets`` (device op)."""
    match = (proposals == targets[:, : proposals.shape[1]]).to(torch.int32)
    return torch.cumprod(match, dim=1).sum(dim=1).to(torch.int32)


def greedy_verify_tokens(proposal_tokens: torch.Tensor, target_tokens: torch.Tensor) -> GreedyVerificationResult:
    if proposal_tokens.ndim != 2 or target_tokens.ndim != 2:
        raise ValueError("expected proposal and target tokens [batch, steps]")
    if proposal_tokens.shape != target_tokens.shape:
        raise ValueError("proposal and target token dimensions must match")
    acc = accept_lengths(proposal_tokens, target_tokens)
    p, t = proposal_tokens.tolist(), target_tokens.tolist()
    outs = []
    for row, a in enumerate(acc.tolist()):
        toks = p[row][:a]
        if a < len(p[row]):
            toks = toks + [t[row][a]]
        outs.append(toks)
    return GreedyVerificationResult(acc, outs)


def greedy_verify(proposal_tokens: torch.Tensor, target_logits: torch.Tensor) -> GreedyVerificationResult:
    if proposal_tokens.ndim != 2 or target_logits.ndim != 3:
        raise ValueError("expected proposals [batch, steps] and logits [batch, steps, vocab]")
    if proposal_tokens.shape != target_logits.shape[:2]:
        raise ValueError("proposal and target step dimensions must match")
    return greedy_verify_tokens(proposal_tokens, target_logits.argmax(dim=-1))


def build_greedy_commit_plan(base_context_lengths: torch.Tensor,
                             verification: GreedyVerificationResult) -> GreedyCommitPlan:
    if base_context_lengths.shape != verification.accepted_lengths.shape:
        raise ValueError("base_context_lengths must match accepted_lengths")
    committed = base_context_lengths + verification.accepted_lengths.to(base_context_lengths.dtype)
    need = torch.tensor([len(toks) > a for toks, a in zip(verification.output_tokens,
                                                            verification.accepted_lengths.tolist())],
                        dtype=torch.bool, device=base_context_lengths.device)
    return GreedyCommitPlan(verification.accepted_lengths, committed, verification.output_tokens, need)
