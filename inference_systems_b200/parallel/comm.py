"""Tensor-parallel communication for the model's row-parallel layers and LM head.

Parity: the reference's tensor parallelism calls ``dist.all_reduce`` after
every row-parallel linear (``nanovllm/layers/linear.py:153-156``), after the GDN
out_proj (``nanovllm/layers/gated_delta_net.py:257,358``) and gathers the
vocab-parallel logits to rank 0 (``nanovllm/layers/embed_head.py:56-65``),
then broadcasts sampled tokens (``nanovllm/engine/model_runner.py:668-702``).

Here, on GPUs:

* ``row_parallel_residual_norm`` = ONE GEMM kernel that reduces this rank's
  partial product into its own fp32 accumulator (split-K tiles added locally)
  and whose last CTA bumps this rank's completion counter
  (``tp_gemm_accum``) + ONE consumer kernel that waits until every peer's
  counter has caught up, sums all ranks' accumulators with NVLink P2P loads,
  adds the residual and applies the next RMSNorm (``add_rmsnorm_acc_tp``).
  Accumulators alternate between two parities per call; the consumer re-zeroes
  the previous call's buffer, which every peer has finished reading by then.
* ``lm_head_sample`` = the LM-head GEMM with its fused greedy/Gumbel-max
  selection on this rank's vocab slice + ``xrank_argmax``, which exchanges 8
  bytes per row with every peer; every rank ends with the same token ids.
* Prefill chunks larger than ``max_rows`` tokens run token-sharded (sequence
  parallel within the TP group) when ``sp_rows`` allows: the residual stream is
  split by tokens; each row-parallel GEMM stores its fp32 partial product and
  ``sp_rs_norm`` (reduce-scatter + residual + RMSNorm + all-gather) pulls only
  this rank's token rows from every peer, normalises them and pushes them into
  every rank's full activation buffer; the next column-parallel GEMM
  (``gemm_ag``) waits, per 128-row M tile, for the owning rank's counter and
  reads the tile from its own memory (a remote row crosses NVLink once, not
  once per column tile).  Per layer a rank pulls ``(W-1)/W * T/W * H`` fp32
  values and pushes ``(W-1) * T/W * H`` bf16 values, instead of all-reducing
  ``T * H``.  Otherwise larger chunks use NCCL all-reduce.

On CPU (gloo process groups, used by the tests) the same methods run with
``torch.distributed`` collectives.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.distributed as dist

from inference_systems_b200 import ops

_ALIGN = 256
_SP_TILE = 128  # shard rows are a multiple of the GEMM's M tile


def _align(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


@dataclass
class ShardedActivation:
    """A normalised activation ``[T, H]`` split by tokens over the TP group.

    Rank ``r`` holds rows ``[r*S, min((r+1)*S, T))`` in ``local`` (on GPUs: a
    view of its symmetric shard buffer of parity ``parity``).  Column-parallel
    layers consume it through ``TPComm.sp_linear``.
    """
    comm: "TPComm"
    local: torch.Tensor
    T: int
    S: int
    parity: int

    @property
    def shape(self):
        return (self.T, self.local.shape[1])

    @property
    def is_cuda(self) -> bool:
        return self.local.is_cuda


class TPComm:
    def __init__(self, device: torch.device, rank: int, world: int, hidden: int, config=None,
                 max_rows: int = 256, max_sample_rows: int | None = None, group=None):
        self.device, self.rank, self.world, self.hidden = device, rank, world, hidden
        self.group = group
        self.max_rows = int(os.environ.get("ISB_TP_MAX_ROWS", max_rows))
        spec = getattr(config, "num_speculative_tokens", 0) if config is not None else 0
        seqs = getattr(config, "max_num_seqs", 256) if config is not None else 256
        self.max_sample_rows = max_sample_rows or max(512, seqs * (spec + 1))
        self.set = 0
        self.fused = device.type == "cuda"
        # shard rows are a multiple of the GEMM's 128-row M tile on GPUs; CPU ranks split finer
        self.sp_tile = _SP_TILE if self.fused else 8
        self._peer_ptrs: list[int] = []
        # token-sharded prefill: ISB_TP_SP=1 enables it, for chunks of max_rows < T <= max_sp_rows
        self.sp = os.environ.get("ISB_TP_SP", "0") == "1" and world > 1
        tokens = getattr(config, "max_num_batched_tokens", 8192) if config is not None else 8192
        self.max_sp_rows = min(int(tokens), 16384) if self.sp else 0
        self.sp_set = 0
        if self.fused:
            self._setup_symmetric()

    # ----------------------------------------------------------- memory
    def _setup_symmetric(self) -> None:
        c = ops.cuda_ops()
        w, h = self.world, self.hidden
        off = 0
        layout = {}
        for name, nbytes in (("acc0", self.max_rows * h * 4), ("acc1", self.max_rows * h * 4),
                             ("accflag0", w * 4), ("accflag1", w * 4), ("gdone0", 4), ("gdone1", 4),
                             ("ndone0", 4), ("ndone1", 4), ("xbuf", w * self.max_sample_rows * 8), ("xflag", w * 4),
                             ("spacc0", self.max_sp_rows * h * 4), ("spacc1", self.max_sp_rows * h * 4),
                             ("xf0", self.max_sp_rows * h * 2), ("xf1", self.max_sp_rows * h * 2),
                             ("spgflag", 4), ("spgdone", 4), ("xsflag", 4), ("spdone", 4)):
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

        def table(name):
            return torch.tensor([b + layout[name] for b in bases], dtype=torch.int64, device=self.device)

        def local(name, dtype, count):
            o = layout[name]
            return self.region[o:o + count * torch.tensor([], dtype=dtype).element_size()].view(dtype)

        self.acc_ptrs = [table("acc0"), table("acc1")]
        self.accflag_ptrs = [table("accflag0"), table("accflag1")]
        self.acc_local = [local("acc0", torch.float32, self.max_rows * h).view(self.max_rows, h),
                          local("acc1", torch.float32, self.max_rows * h).view(self.max_rows, h)]
        self.accflag_local = [local("accflag0", torch.int32, w), local("accflag1", torch.int32, w)]
        self.rows_used = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.gdone = [local("gdone0", torch.int32, 1), local("gdone1", torch.int32, 1)]
        self.ndone = [local("ndone0", torch.int32, 1), local("ndone1", torch.int32, 1)]
        self.xbuf_ptrs = table("xbuf")
        self.xflag_ptrs = table("xflag")
        self.xbuf_local = local("xbuf", torch.float32, w * self.max_sample_rows * 2)
        self.xflag_local = local("xflag", torch.int32, w)
        if self.sp:
            self.spacc_ptrs = [table("spacc0"), table("spacc1")]
            self.spacc_local = [local(f"spacc{i}", torch.float32, self.max_sp_rows * h).view(self.max_sp_rows, h)
                                for i in range(2)]
            self.xf_local = [local(f"xf{i}", torch.bfloat16, self.max_sp_rows * h).view(self.max_sp_rows, h)
                             for i in range(2)]
            self.xf_ptrs = [table("xf0"), table("xf1")]
            self.no_maps = torch.empty(0, dtype=torch.uint8, device=self.device)  # gemm_ag: read local rows
            self.spgflag_ptrs, self.spgflag_local = table("spgflag"), local("spgflag", torch.int32, 1)
            self.spgdone = local("spgdone", torch.int32, 1)
            self.xsflag_ptrs, self.xsflag_local = table("xsflag"), local("xsflag", torch.int32, 1)
            self.spdone = local("spdone", torch.int32, 1)
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
    def row_parallel_residual_norm(self, x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor,
                                   norm_w: torch.Tensor, eps: float, zero_centered: bool) -> torch.Tensor:
        """``residual += sum_ranks(x @ w^T)``; return RMSNorm(residual)."""
        t = x.shape[0]
        if self.fused and t <= self.max_rows:
            c = ops.cuda_ops()
            s = self.set
            self.set ^= 1
            c.tp_gemm_accum(x, w, self.acc_local[s], self.accflag_local[s][:1], self.gdone[s], 0)
            return c.add_rmsnorm_acc_tp(self.acc_ptrs[s], self.acc_local[s ^ 1], residual, norm_w, eps,
                                        zero_centered, self.accflag_ptrs[s], self.accflag_local[s][:1],
                                        self.rows_used, s)
        y = ops.linear(x, w)
        dist.all_reduce(y, group=self.group)
        return ops.add_rmsnorm(y, residual, norm_w, eps, zero_centered)

    # ------------------------------------------------------------ token-sharded prefill
    def _shard_rows(self, T: int) -> int:
        per = (T + self.world - 1) // self.world
        return max(self.sp_tile, (per + self.sp_tile - 1) // self.sp_tile * self.sp_tile)

    def sp_rows(self, T: int) -> int:
        """Shard rows S for a ``T``-token forward, or 0 when it runs replicated."""
        if not self.sp or T <= self.max_rows or T > self.max_sp_rows:
            return 0
        return self._shard_rows(T)

    def sp_range(self, T: int, S: int) -> tuple[int, int]:
        lo = min(self.rank * S, T)
        return lo, min(lo + S, T)

    def sp_publish(self, x: torch.Tensor, T: int, S: int) -> ShardedActivation:
        """Make this rank's first normalised shard ``x`` ``[rows, H]`` visible to the group."""
        if not self.fused:
            return ShardedActivation(self, x, T, S, 0)
        q = self.sp_set
        self.sp_set ^= 1
        lo, hi = self.sp_range(T, S)
        ops.cuda_ops().sp_publish(x.contiguous(), self.xf_ptrs[q], lo, self.spdone, self.xsflag_local)
        return ShardedActivation(self, self.xf_local[q][lo:hi], T, S, q)

    def sp_linear(self, x: ShardedActivation, w: torch.Tensor, silu_mul: bool = False) -> torch.Tensor:
        """All-gather -> column-parallel GEMM: ``gather(x) @ w^T`` (SiLU-mul epilogue optional)."""
        if not self.fused:
            full = self._gather_cpu(x)
            return ops.linear_silu_mul(full, w) if silu_mul else ops.linear(full, w)
        c = ops.cuda_ops()
        return c.gemm_ag(self.xf_local[x.parity], self.no_maps, self.xsflag_ptrs, self.xsflag_local, x.S, x.T, w,
                         1 if silu_mul else 0)

    def sp_row_parallel_norm(self, y: torch.Tensor, w: torch.Tensor, residual: torch.Tensor, norm_w: torch.Tensor,
                             eps: float, zero_centered: bool, T: int, S: int) -> ShardedActivation:
        """Row-parallel GEMM -> reduce-scatter -> ``residual += ...`` -> RMSNorm, on this rank's token rows.

        ``y`` is ``[T, in/W]`` (all tokens), ``residual`` this rank's shard ``[rows, H]``.
        """
        lo, hi = self.sp_range(T, S)
        if not self.fused:
            full = ops.linear(y, w)
            dist.all_reduce(full, group=self.group)
            x = ops.add_rmsnorm(full[lo:hi].contiguous(), residual, norm_w, eps, zero_centered)
            return ShardedActivation(self, x, T, S, 0)
        c = ops.cuda_ops()
        s = self.sp_set
        self.sp_set ^= 1
        c.tp_gemm_accum(y, w, self.spacc_local[s], self.spgflag_local, self.spgdone, 1)
        c.sp_rs_norm(self.spacc_ptrs[s], self.spgflag_ptrs, self.spgflag_local, residual, norm_w, self.xf_ptrs[s],
                     lo, eps, zero_centered, self.spdone, self.xsflag_local)
        return ShardedActivation(self, self.xf_local[s][lo:hi], T, S, s)

    def sp_gather(self, x: ShardedActivation) -> torch.Tensor:
        """All rows ``[T, H]`` of a token-sharded activation on every rank."""
        if not self.fused:
            return self._gather_cpu(x)
        return ops.cuda_ops().sp_gather(self.xf_local[x.parity], self.xsflag_ptrs, self.xsflag_local, x.S, x.T)

    def _gather_cpu(self, x: ShardedActivation) -> torch.Tensor:
        h = x.local.shape[1]
        pad = torch.zeros(x.S, h, dtype=x.local.dtype, device=x.local.device)
        pad[: x.local.shape[0]] = x.local
        parts = [torch.empty_like(pad) for _ in range(self.world)]
        dist.all_gather(parts, pad, group=self.group)
        return torch.cat(parts)[: x.T].contiguous()

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
