"""Tensor-parallel communication for the model's row-parallel layers and LM head.

Parity: the reference's tensor parallelism calls ``dist.all_reduce`` after
every row-parallel linear (``nanovllm/layers/linear.py:153-156``), after the GDN
out_proj (``nanovllm/layers/gated_delta_net.py:257,358``) and gathers the
vocab-parallel logits to rank 0 (``nanovllm/layers/embed_head.py:56-65``),
then broadcasts sampled tokens (``nanovllm/engine/model_runner.py:668-702``).

Here, on GPUs, one exchange per row-parallel layer, the same for decode and
prefill (every chunk up to ``max_tokens`` tokens; no NCCL on the data path):

* ``tp_gemm_rs`` = the row-parallel GEMM whose epilogue reduce-scatters by
  token: token rows are split into W contiguous shards; split-K CTAs first
  reduce their fp32 partial tiles in local memory, then each complete bf16 row
  owned by rank r is stored into rank r's slot for this rank (plain NVLink
  stores: a partial crosses the link once); the grid's last CTA bumps every
  rank's arrival counter.
* ``tp_norm_allgather`` = the owner side: once all W ranks arrived, it sums the
  W slots of each owned row in fp32, adds the residual, applies the next
  RMSNorm and pushes the normalised row into every rank's activation buffer
  (the all-gather, P2P stores), then releases every rank's gather counter; its
  last CTA waits until all owners' rows are in, so the next column-parallel
  GEMM reads a complete activation from local memory.  Per exchange a rank sends
  (W-1)/W * T * H bf16 partial sums and (W-1) * T/W * H bf16 activations, and
  every wait polls local memory.
* ``lm_head_sample`` = the LM-head GEMM with its fused greedy/Gumbel-max
  selection on this rank's vocab slice + ``xrank_argmax``, which exchanges 8
  bytes per row with every peer; every rank ends with the same token ids.

The residual stream stays replicated in shape, but each rank only reads and
updates the rows it owns (the rows it normalises); the activation buffers
alternate between two parities so an exchange's output survives the next one.

On CPU (gloo process groups, used by the tests) the same methods run with
``torch.distributed`` collectives.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from inference_systems_b200 import ops

_ALIGN = 256


def _align(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


def shard_rows(T: int, world: int) -> int:
    """Token rows owned by each rank for a ``T``-token exchange (contiguous shards)."""
    return max((T + world - 1) // world, 1)


# ISB_TP_FUSED_ONE_SHOT=0: one-shot exchanges run the GEMM and the owner-norm kernel separately
_FUSED_ONE_SHOT = os.environ.get("ISB_TP_FUSED_ONE_SHOT", "1") != "0"

class TPComm:
    def __init__(self, device: torch.device, rank: int, world: int, hidden: int, config=None,
                 max_tokens: int | None = None, max_sample_rows: int | None = None, group=None):
        self.device, self.rank, self.world, self.hidden = device, rank, world, hidden
        self.group = group
        spec = getattr(config, "num_speculative_tokens", 0) if config is not None else 0
        seqs = getattr(config, "max_num_seqs", 256) if config is not None else 256
        tokens = getattr(config, "max_num_batched_tokens", 8192) if config is not None else 8192
        self.max_tokens = int(os.environ.get("ISB_TP_MAX_TOKENS", max_tokens or max(tokens, seqs * (spec + 1), 256)))
        self.max_sample_rows = max_sample_rows or max(512, seqs * (spec + 1))
        # Exchanges of up to this many activation elements (T x H) run one-shot: every rank pushes
        # its whole bf16 partial to every rank and normalises every row itself -- one cross-GPU
        # hop instead of two, at W/2 times the bytes; larger ones (prefill) run two-shot.
        self.one_shot_elems = int(os.environ.get("ISB_TP_ONE_SHOT_ELEMS", 256 * 1024))
        self.xpar = 0
        self.fused = device.type == "cuda"
        self._peer_ptrs: list[int] = []
        if self.fused:
            self._setup_symmetric()

    # ----------------------------------------------------------- memory
    def _setup_symmetric(self) -> None:
        c = ops.cuda_ops()
        w, h, t = self.world, self.hidden, self.max_tokens
        off = 0
        layout = {}
        self.slot_rows = max(shard_rows(t, w), min(t, self.one_shot_elems // h))
        for name, nbytes in (("slots0", w * self.slot_rows * h * 2), ("slots1", w * self.slot_rows * h * 2),
                             ("x0", t * h * 2), ("x1", t * h * 2),
                             ("ctl", 32), ("xbuf", w * self.max_sample_rows * 8), ("xflag", w * 4)):
            layout[name] = off
            off += _align(nbytes)
        self.layout, self.nbytes = layout, off
        self.region, handle = c.symm_alloc(off)
        handles = [None] * w
        dist.all_gather_object(handles, handle.numpy().tobytes(), group=self.group)
        bases = []
        for r in range(w):
            if r == self.rank:
                bases.append(self.region.data_ptr())
            else:
                p = c.symm_open(torch.frombuffer(bytearray(handles[r]), dtype=torch.uint8))
                self._peer_ptrs.append(p)
                bases.append(p)
        self.bases = bases

        def table(name, extra=0):
            return torch.tensor([b + layout[name] + extra for b in bases], dtype=torch.int64, device=self.device)

        def local(name, dtype, count):
            o = layout[name]
            return self.region[o:o + count * torch.tensor([], dtype=dtype).element_size()].view(dtype)

        # slots and activation buffers alternate by exchange parity: in one-shot mode nothing makes a
        # rank wait for its peers to finish reading their slots, so a rank one exchange ahead must
        # push into the other buffer (it cannot get two ahead: its next owner kernel waits for
        # every peer's pushes of the exchange in between, which follow those peers' reads)
        self.slot_ptrs = [table("slots0"), table("slots1")]
        self.rs_ptrs = table("ctl", 0)      # ctl[0]: arrivals of row-parallel GEMMs
        self.ag_ptrs = table("ctl", 4)      # ctl[1]: arrivals of owners' activation rows
        self.x_ptrs = [table("x0"), table("x1")]
        self.slots_local = [local(f"slots{i}", torch.bfloat16, w * self.slot_rows * h).view(w, self.slot_rows, h)
                            for i in range(2)]
        # split-K partial tiles are reduced here before a row leaves this GPU (zero between uses)
        self.staging = torch.zeros(t, h, dtype=torch.float32, device=self.device)
        self.x_local = [local("x0", torch.bfloat16, t * h).view(t, h), local("x1", torch.bfloat16, t * h).view(t, h)]
        # arrivals of GEMM CTAs, arrivals of owner CTAs, both counters' targets after the last
        # exchange, the owner kernel's CTA-completion counter
        self.ctl = local("ctl", torch.int32, 8)
        self.xbuf_ptrs = table("xbuf")
        self.xflag_ptrs = table("xflag")
        self.xbuf_local = local("xbuf", torch.float32, w * self.max_sample_rows * 2)
        self.xflag_local = local("xflag", torch.int32, w)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def close(self) -> None:
        if self.fused and self._peer_ptrs:
            torch.cuda.synchronize(self.device)
            c = ops.cuda_ops()
            for p in self._peer_ptrs:
                c.symm_close(p)
            self._peer_ptrs = []

    # ------------------------------------------------------------ layers
    def owned_rows(self, T: int) -> tuple[int, int]:
        """``(lo, rows)``: the token rows this rank normalises in a ``T``-token exchange."""
        s = shard_rows(T, self.world)
        lo = min(self.rank * s, T)
        return lo, min(s, T - lo)

    def row_parallel_residual_norm(self, x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor,
                                   norm_w: torch.Tensor, eps: float, zero_centered: bool) -> torch.Tensor:
        """``residual += sum_ranks(x @ w^T)``; return RMSNorm(residual) (all rows, on every rank).

        On GPUs a two-shot exchange (large ``T``) updates only the rows this rank owns in
        ``residual``; a one-shot exchange updates all of them."""
        t = x.shape[0]
        if self.fused and t <= self.max_tokens:
            c = ops.cuda_ops()
            s = shard_rows(t, self.world)
            one = t * self.hidden <= self.one_shot_elems and t <= self.slot_rows
            p = self.xpar
            self.xpar ^= 1
            if one and t <= 128 and self.hidden <= 1024 and _FUSED_ONE_SHOT:
                # one kernel: GEMM, push to every rank, bounded wait for all ranks, residual + norm
                c.tp_gemm_rs_norm(x, w, self.slot_ptrs[p], self.slot_rows, self.rs_ptrs, self.rank,
                                  self.slots_local[p], residual, norm_w, self.x_local[p], self.ctl, eps, zero_centered)
                return self.x_local[p][:t]
            ctas = c.tp_gemm_rs(x, w, self.slot_ptrs[p], self.slot_rows, self.staging, self.rs_ptrs, self.rank, s, 0,
                                one)
            c.tp_norm_allgather(self.slots_local[p], residual, norm_w, self.x_ptrs[p], self.ag_ptrs, self.ctl, t, s,
                                self.rank, self.world * ctas, eps, zero_centered, True, one)
            return self.x_local[p][:t]
        y = ops.linear(x, w)
        dist.all_reduce(y, group=self.group)
        return ops.add_rmsnorm(y, residual, norm_w, eps, zero_centered)

    def lm_head_sample(self, hidden: torch.Tensor, w_local: torch.Tensor, temperatures: torch.Tensor,
                       rng: torch.Tensor, vocab_start: int) -> torch.Tensor:
        val, idx = ops.lm_head_sample(hidden, w_local, temperatures, rng, vocab_start)
        if self.fused:
            return ops.cuda_ops().xrank_argmax(val, idx, self.xbuf_ptrs, self.xflag_ptrs, self.xflag_local,
                                               self.xbuf_local, self.rank, self.max_sample_rows)
        vals = [torch.empty_like(val) for _ in range(self.world)]
        idxs = [torch.empty_like(idx) for _ in range(self.world)]
        dist.all_gather(vals, val, group=self.group)
        dist.all_gather(idxs, idx, group=self.group)
        v = torch.stack(vals)          # [W, B]
        i = torch.stack(idxs)
        best = v.max(dim=0).values
        cand = torch.where(v == best[None], i, torch.full_like(i, torch.iinfo(i.dtype).max))
        return cand.min(dim=0).values
