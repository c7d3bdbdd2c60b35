"""Token-sharded tensor-parallel kernels on one GPU.

``gemm_ag``, ``sp_rs_norm``, ``sp_gather`` and ``sp_publish`` address every rank's buffers and
ready counters through device pointers, so W ranks can be laid out as W local buffers whose
counters are already published before the launch (nothing waits for another launch).  Each
kernel is compared with a plain PyTorch fp32 computation; rows that no rank writes hold NaN and
must not leak into any result.
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


def _counters(w, value=1):
    cnt = torch.full((w,), value, dtype=torch.int32, device=DEV)
    ptrs = torch.tensor([cnt.data_ptr() + 4 * r for r in range(w)], dtype=torch.int64, device=DEV)
    return cnt, ptrs


def _shards(w, s, t, h, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    full = torch.randn(t, h, device=DEV, generator=g).to(torch.bfloat16)
    bufs = []
    for r in range(w):
        b = torch.full((s, h), float("nan"), dtype=torch.bfloat16, device=DEV)
        rows = full[r * s: min((r + 1) * s, t)]
        b[: rows.shape[0]] = rows
        bufs.append(b)
    return full, bufs


@pytest.mark.parametrize("w,s,t,k,n,silu", [(2, 256, 300, 1024, 2048, False), (4, 128, 400, 1024, 768, False),
                                            (2, 256, 512, 1024, 1024, True), (3, 128, 257, 512, 384, False)])
@pytest.mark.parametrize("peer_maps", [True, False])
def test_gemm_allgather_operand(w, s, t, k, n, silu, peer_maps):
    """M tiles read from their owners' shard buffers (per-rank tensor maps) or from a local
    buffer into which every owner pushed its rows; either way each tile waits for its owner."""
    full, bufs = _shards(w, s, t, k, seed=w * 7 + t)
    g = torch.Generator(device=DEV).manual_seed(1)
    wt = (torch.randn(n, k, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    c = ops.cuda_ops()
    cnt, flags = _counters(w)
    if peer_maps:
        maps = c.ag_tensor_maps(torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64), s, k, bufs[0])
        out = c.gemm_ag(bufs[0], maps, flags, cnt[:1], s, t, wt, 1 if silu else 0)
    else:
        local = torch.full((w * s, k), float("nan"), dtype=torch.bfloat16, device=DEV)
        local[:t] = full
        out = c.gemm_ag(local, torch.empty(0, dtype=torch.uint8, device=DEV), flags, cnt[:1], s, t, wt,
                        1 if silu else 0)
    torch.cuda.synchronize()
    assert torch.ops.isb.error_word() == 0
    want = ops.linear_silu_mul(full, wt) if silu else ops.linear(full, wt)
    assert out.shape == want.shape
    assert torch.isfinite(out.float()).all()
    exp = full.float() @ wt.float().t()
    if silu:
        exp = ref.silu_mul_packed(exp)
    assert _rel(out, want) < 1e-2
    assert _rel(out, exp) < 2e-2


@pytest.mark.parametrize("w,s,t,h,rank", [(2, 256, 300, 1024, 1), (2, 256, 300, 1024, 0), (4, 128, 400, 5120, 2),
                                          (4, 128, 400, 1024, 3)])
def test_reduce_scatter_rmsnorm(w, s, t, h, rank):
    g = torch.Generator(device=DEV).manual_seed(t + rank)
    accs = [torch.randn(t, h, device=DEV, generator=g) * 0.5 for _ in range(w)]
    lo, hi = min(rank * s, t), min((rank + 1) * s, t)
    rows = hi - lo
    res = torch.randn(rows, h, device=DEV, generator=g).to(torch.bfloat16)
    nw = (0.1 * torch.randn(h, device=DEV, generator=g)).to(torch.bfloat16)
    xf = [torch.full((t, h), float("nan"), dtype=torch.bfloat16, device=DEV) for _ in range(w)]
    xf_ptrs = torch.tensor([x.data_ptr() for x in xf], dtype=torch.int64, device=DEV)
    acc_ptrs = torch.tensor([a.data_ptr() for a in accs], dtype=torch.int64, device=DEV)
    gcnt, gflags = _counters(w)
    done = torch.zeros(1, dtype=torch.int32, device=DEV)
    ready = torch.zeros(1, dtype=torch.int32, device=DEV)
    res_exp = res.clone()
    summed = sum(a[lo:hi] for a in accs)
    exp = ref.add_rmsnorm(summed, res_exp, nw, 1e-6, True)
    c = ops.cuda_ops()
    c.sp_rs_norm(acc_ptrs, gflags, gcnt[:1], res, nw, xf_ptrs, lo, 1e-6, True, done, ready)
    torch.cuda.synchronize()
    assert torch.ops.isb.error_word() == 0
    assert int(ready.item()) == 1 and int(done.item()) == 0
    for x in xf:  # the rows went to every rank's buffer, nothing else was written
        assert _rel(x[lo:hi], exp) < 1e-2
        assert torch.isnan(x[:lo].float()).all() and torch.isnan(x[hi:].float()).all()
    assert _rel(res, res_exp) < 1e-2


@pytest.mark.parametrize("w,s,t,h", [(2, 256, 300, 1024), (4, 128, 400, 640)])
def test_shard_publish_and_gather(w, s, t, h):
    g = torch.Generator(device=DEV).manual_seed(3)
    full = torch.randn(t, h, device=DEV, generator=g).to(torch.bfloat16)
    c = ops.cuda_ops()
    xf = [torch.full((t, h), float("nan"), dtype=torch.bfloat16, device=DEV) for _ in range(w)]
    xf_ptrs = torch.tensor([x.data_ptr() for x in xf], dtype=torch.int64, device=DEV)
    done = torch.zeros(1, dtype=torch.int32, device=DEV)
    ready = torch.zeros(1, dtype=torch.int32, device=DEV)
    for r in range(w):  # every "rank" pushes its rows into every buffer
        lo, hi = min(r * s, t), min((r + 1) * s, t)
        c.sp_publish(full[lo:hi].contiguous(), xf_ptrs, lo, done, ready)
    torch.cuda.synchronize()
    assert int(ready.item()) == w and int(done.item()) == 0
    for x in xf:
        assert torch.equal(x, full)
    cnt, flags = _counters(w)
    out = c.sp_gather(xf[1], flags, cnt[:1], s, t)
    torch.cuda.synchronize()
    assert torch.ops.isb.error_word() == 0
    assert torch.equal(out, full)
