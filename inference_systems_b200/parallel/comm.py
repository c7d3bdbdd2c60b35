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
* Prefill chunks larger than ``max_rows`` tokens use NCCL all-reduce.

On CPU (gloo process groups, used by the tests) the same methods run with
``torch.distributed`` collectives.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from inference_systems_b200 import ops

_ALIGN = 256


def _align(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


class TPComm:
    def __init__(self, device: torch.device, rank: int, world: int, hidden: int, config=None,
                 max_rows: int = 256, max_sample_rows: int | None = None, group=None):
        self.device, self.rank, self.world, self.hidden = device, rank, world, hidden
        self.group = group
        self.max_rows = max_rows
        spec = getattr(config, "num_speculative_tokens", 0) if config is not None else 0
        seqs = getattr(config, "max_num_seqs", 256) if config is not None else 256
        self.max_sample_rows = max_sample_rows or max(512, seqs * (spec + 1))
        self.set = 0
        self.fused = device.type == "cuda"
        self._peer_ptrs: list[int] = []
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
                             ("ndone0", 4), ("ndone1", 4), ("xbuf", w * self.max_sample_rows * 8), ("xflag", w * 4)):
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
