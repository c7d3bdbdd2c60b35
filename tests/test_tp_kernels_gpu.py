"""Tensor-parallel exchange kernels on one GPU: ``tp_gemm_rs`` + ``tp_norm_allgather``.

Both kernels address every rank's accumulator, activation buffer and counters through device
address tables, so W ranks can be laid out as W sets of local buffers on one GPU.  The W
row-parallel GEMMs run first (each reduce-scatters its partial product into the owners'
accumulators and bumps every rank's arrival counter); the W owner kernels then find their
arrival counters complete and run with the final all-gather wait switched off, so no launch ever
waits for a later one.  Results are compared with a plain PyTorch fp32 computation.

The bounded-wait test shortens the exchange's wait deadline, runs the owner kernel on a counter
that never advances, and checks that the kernel returns with the communication error word set.
"""

import pytest
import torch

from inference_systems_b200 import ops
from inference_systems_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def _addr_table(tensors, offset_bytes=0):
    return torch.tensor([t.data_ptr() + offset_bytes for t in tensors], dtype=torch.int64, device=DEV)


class EmulatedRanks:
    """W ranks' symmetric buffers as local tensors (NaN where nothing may be read)."""

    def __init__(self, w, t, h, one_shot=False):
        self.w, self.t, self.h, self.one_shot = w, t, h, one_shot
        self.slot_rows = t if one_shot else max((t + w - 1) // w, 1)
        self.slots = [torch.full((w, self.slot_rows, h), float("nan"), dtype=torch.bfloat16, device=DEV)
                      for _ in range(w)]
        self.staging = [torch.zeros(t, h, device=DEV) for _ in range(w)]
        self.x = [torch.full((t, h), float("nan"), dtype=torch.bfloat16, device=DEV) for _ in range(w)]
        self.ctl = [torch.zeros(8, dtype=torch.int32, device=DEV) for _ in range(w)]
        self.slot_ptrs = _addr_table(self.slots)
        self.rs_ptrs = _addr_table(self.ctl, 0)
        self.ag_ptrs = _addr_table(self.ctl, 4)
        self.x_ptrs = _addr_table(self.x)

    def owned(self, r, t):
        s = max((t + self.w - 1) // self.w, 1)
        if self.one_shot:  # every rank normalises every row
            return s, 0, t
        lo = min(r * s, t)
        return s, lo, min(s, t - lo)


def _exchange(ranks, xs, ws, res, nw, t, zc=True, splits=0):
    """One exchange on every emulated rank; returns (GEMM CTAs per rank, owner CTAs over all ranks)."""
    c = ops.cuda_ops()
    s = ranks.owned(0, t)[0]
    one = ranks.one_shot
    ctas = [c.tp_gemm_rs(xs[r], ws[r], ranks.slot_ptrs, ranks.slot_rows, ranks.staging[r], ranks.rs_ptrs, r, s, splits,
                         one) for r in range(ranks.w)]
    assert len(set(ctas)) == 1
    for r in range(ranks.w):
        c.tp_norm_allgather(ranks.slots[r], res[r], nw, ranks.x_ptrs, ranks.ag_ptrs, ranks.ctl[r], t, s, r,
                            ranks.w * ctas[0], 1e-6, zc, False, one)
    torch.cuda.synchronize()
    owners = 0 if one else sum(max(min(ranks.owned(r, t)[2], 296), 1) for r in range(ranks.w))
    return ctas[0], owners


@pytest.mark.parametrize("one_shot", [False, True])
@pytest.mark.parametrize("w,t,h,k,splits", [(2, 128, 1024, 1792, 0), (2, 128, 1024, 1792, 1), (4, 128, 1024, 512, 0),
                                            (8, 128, 1024, 256, 0), (8, 5, 1024, 448, 0), (2, 300, 5120, 1024, 0),
                                            (2, 300, 1024, 2048, 4), (4, 1, 1024, 512, 0)])
def test_reduce_scatter_norm_allgather(w, t, h, k, splits, one_shot):
    """Two-shot (reduce-scatter to the owner, owner normalises and pushes its rows to every rank)
    and one-shot (every rank pushes its whole partial to every rank and normalises every row)."""
    g = torch.Generator(device=DEV).manual_seed(w * 100 + t)
    ranks = EmulatedRanks(w, t, h, one_shot)
    xs = [torch.randn(t, k, device=DEV, generator=g).to(torch.bfloat16) for _ in range(w)]
    ws = [(torch.randn(h, k, device=DEV, generator=g) * 0.05).to(torch.bfloat16) for _ in range(w)]
    res0 = torch.randn(t, h, device=DEV, generator=g).to(torch.bfloat16)
    res = [res0.clone() for _ in range(w)]
    nw = (0.1 * torch.randn(h, device=DEV, generator=g)).to(torch.bfloat16)
    for step in range(2):  # two exchanges in a row: counters and sequence numbers move on
        summed = sum(x.float() @ wt.float().t() for x, wt in zip(xs, ws))
        want_res = res0.float() + summed
        want = ref.rmsnorm(want_res, nw, 1e-6, True)
        ctas, owners = _exchange(ranks, xs, ws, res, nw, t, splits=splits)
        assert torch.ops.isb.error_word() == 0
        for r in range(w):
            assert torch.isfinite(ranks.x[r].float()).all()
            assert _rel(ranks.x[r], want) < 1e-2                   # every rank holds every row
            _, lo, rows = ranks.owned(r, t)
            assert _rel(res[r][lo:lo + rows], want_res[lo:lo + rows]) < 1e-2 if rows else True
            assert torch.count_nonzero(ranks.staging[r]) == 0      # split-K staging re-zeroed
            rs, ag = w * ctas * (step + 1), owners * (step + 1)   # one-shot: no owner arrivals
            assert ranks.ctl[r].tolist() == [rs, ag, rs, ag, 0, 0, 0, 0]
        res0 = res[0].clone()
        for r in range(w):  # every rank's residual view, as the next layer would see its own rows
            _, lo, rows = ranks.owned(r, t)
            res0[lo:lo + rows] = res[r][lo:lo + rows]
        res = [res0.clone() for _ in range(w)]
        xs = [torch.randn(t, k, device=DEV, generator=g).to(torch.bfloat16) for _ in range(w)]


def test_owner_wait_runs_out_and_sets_the_error_word():
    """An arrival counter that never reaches its target: the owner kernel gives up after the
    (shortened) deadline, records the error and still returns; the GPU stays usable."""
    c = ops.cuda_ops()
    assert torch.ops.isb.error_word() == 0
    w, t, h = 2, 16, 1024
    ranks = EmulatedRanks(w, t, h)
    res = torch.randn(t, h, device=DEV).to(torch.bfloat16)
    nw = torch.zeros(h, device=DEV).to(torch.bfloat16)
    c.comm_set_wait_timeout(5_000_000)  # 5 ms
    try:
        c.tp_norm_allgather(ranks.slots[0], res, nw, ranks.x_ptrs, ranks.ag_ptrs, ranks.ctl[0], 16, 8, 0, 1, 1e-6,
                            True, True)
        torch.cuda.synchronize()
        word = torch.ops.isb.error_word()
    finally:
        c.comm_set_wait_timeout(2_000_000_000)
    assert (word >> 16) & 0x2, hex(word)   # communication module: arrival wait ran out
    assert torch.ops.isb.error_word() == 0  # read-and-clear
    # the device still runs kernels
    a = torch.randn(64, 64, device=DEV).to(torch.bfloat16)
    torch.testing.assert_close(ops.linear(a, a).float(), a.float() @ a.float().t(), atol=0.5, rtol=2e-2)
