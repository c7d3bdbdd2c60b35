"""Per-kernel microbenchmarks of the sm_100a ops at Qwen3.5-0.8B decode shapes.

    python bench_kernels.py [--batch 128] [--only gemm[,attention]] [--json out.json] [--once]
    python -m torch.distributed.run --nproc-per-node N ... bench_kernels.py --tp   (fused TP paths)

Method: every case builds R independent argument sets whose large operands
(weights, GDN state pool, KV cache) together exceed 2 x the 126 MB L2, captures
ONE CUDA graph that launches the op once per argument set, replays it after
warm-up and reports device time per launch (CUDA events around the replays).
Each launch therefore reads its big operand cold from HBM, with no host
launch overhead -- the same conditions as inside the decode-step graph.

Achieved bandwidth uses algorithmic bytes (operands read once, outputs
written once) against the measured HBM copy bandwidth in MEASURED_PEAKS.json
(fallback 6650 GB/s); GEMM FLOP rates against its measured bf16 peak
(fallback 1590 TFLOP/s).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from inference_systems_b200 import ops  # noqa: E402
from inference_systems_b200.ops._ext import load_extension  # noqa: E402
from inference_systems_b200.ops import reference as ref  # noqa: E402

L2_BYTES = 126 << 20


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def graph_time_us(fns, replays: int = 5) -> float:
    """Device time per launch of a CUDA graph that runs every fn in ``fns`` once."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for f in fns:
            f()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in fns:
            f()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(replays):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / (replays * len(fns))


def replicas(big_bytes: int) -> int:
    return max(2, math.ceil(2 * L2_BYTES / max(big_bytes, 1)))


def cases(b: int) -> dict:
    """name -> builder; a builder allocates its operands and returns (fns, algorithmic bytes, flops)."""
    dev, bf = "cuda", torch.bfloat16
    out = {}

    def gemm_case(name, n, k, mode, splits=0):
        def build():
            wbytes = n * k * 2
            r = replicas(wbytes)
            a = torch.randn(b, k, device=dev).to(bf)
            ws = [(torch.randn(n, k, device=dev) * 0.02).to(bf) for _ in range(r)]
            acc = torch.zeros(b, n, device=dev)
            if mode == "silu" and splits:
                fns = [lambda w=w: torch.ops.isb.gemm(a, w, 1, splits) for w in ws]
                ob = b * n // 2 * 2
            elif mode == "store" and splits:
                fns = [lambda w=w: torch.ops.isb.gemm(a, w, 0, splits) for w in ws]
                ob = b * n * 2
            elif mode == "silu":
                fns = [lambda w=w: ops.linear_silu_mul(a, w) for w in ws]
                ob = b * n // 2 * 2
            elif mode == "acc":
                fns = [lambda w=w: ops.linear_accumulate(a, w, acc) for w in ws]
                ob = b * n * 4 * 2
            else:
                fns = [lambda w=w: ops.linear(a, w) for w in ws]
                ob = b * n * 2
            return fns, wbytes + b * k * 2 + ob, 2 * b * n * k
        out[name] = build

    gemm_case("gemm_gdn_in_proj", 8224 + 32, 1024, "store")
    gemm_case("gemm_attn_qkv", 5120, 1024, "store")
    gemm_case("gemm_gate_up_silu", 7168, 1024, "silu")
    gemm_case("gemm_out_proj_accum", 1024, 2048, "acc")
    gemm_case("gemm_down_accum", 1024, 3584, "acc")
    gemm_case("gemm_out_proj_store", 1024, 2048, "store")
    for sp in (2, 4):  # split-K variants of the column-parallel GEMMs (workspace reduction)
        gemm_case(f"gemm_gdn_in_proj_split{sp}", 8224 + 32, 1024, "store", sp)
        gemm_case(f"gemm_gate_up_silu_split{sp}", 7168, 1024, "silu", sp)

    def lm_head():
        v = 248320
        w = (torch.randn(v, 1024, device=dev) * 0.02).to(bf)  # 508 MB: already > 2 x L2
        x = torch.randn(b, 1024, device=dev).to(bf)
        temps = torch.zeros(b, device=dev)
        rng = torch.zeros(2, dtype=torch.int32, device=dev)
        return [lambda: ops.lm_head_sample(x, w, temps, rng, 0)], (w.numel() + x.numel()) * 2, 2 * b * w.numel()
    out["lm_head_sample_greedy"] = lm_head

    def gdn():
        # GDN decode (16 key == 16 value heads, Dk = Dv = 128)
        hk = hv = 16
        d = 128
        c = 2 * hk * d + hv * d
        p = c + hv * d + 2 * hv
        state_bytes = b * hv * d * d * 4
        r = replicas(state_bytes)
        proj = torch.randn(b, p, device=dev).to(bf)
        conv_w = (torch.randn(c, 4, device=dev) * 0.5).to(bf)
        a_log, dt = torch.zeros(hv, device=dev), torch.ones(hv, device=dev)
        nw = torch.ones(d, device=dev).to(bf)
        slots = torch.arange(b, device=dev, dtype=torch.int32)
        pools = [(torch.randn(b + 1, hv, d, d, device=dev) * 0.01, torch.zeros(b + 1, c, 3, device=dev).to(bf))
                 for _ in range(r)]
        fns = [lambda rc=rc, cv=cv: torch.ops.isb.gdn_decode(proj, slots, conv_w, a_log, dt, nw, rc, cv, hk, hv, d,
                                                             d, 1e-6) for rc, cv in pools]
        return fns, 2 * state_bytes + proj.numel() * 2 + b * hv * d * 2, 0
    out["gdn_decode"] = gdn

    def attention():
        # attention decode: 8 q heads / 2 kv heads, hd 256, context 640
        ctx = 640
        kv_bytes = b * 2 * ctx * 256 * 2 * 2
        r = replicas(kv_bytes)
        q = torch.randn(b, 8, 256, device=dev).to(bf)
        gate = torch.randn(b, 8 * 256, device=dev).to(bf)
        bt = torch.arange(b * 3, device=dev, dtype=torch.int32).view(b, 3)
        bt = torch.cat((bt, torch.full((b, 2), -1, device=dev, dtype=torch.int32)), 1)
        cl = torch.full((b,), ctx, device=dev, dtype=torch.int32)
        caches = [(torch.randn(b * 3, 2, 256, 256, device=dev).to(bf), torch.randn(b * 3, 2, 256, 256, device=dev).to(bf))
                  for _ in range(r)]
        fns = [lambda kc=kc, vc=vc: torch.ops.isb.attention_decode(q, gate, kc, vc, cl, bt, 0.0625, True)
               for kc, vc in caches]
        return fns, kv_bytes + q.numel() * 2 * 2, 4 * b * 8 * ctx * 256
    out["attention_decode"] = attention

    def attention_prefill():
        # tensor-core causal prefill: 4 sequences x 2048 new tokens, 8 q / 2 kv heads, hd 256
        nseq, n = 4, 2048
        t = nseq * n
        q = (torch.randn(t, 8, 256, device=dev) * 0.5).to(bf)
        gate = torch.randn(t, 8 * 256, device=dev).to(bf)
        pages = n // 256
        kc = torch.randn(nseq * pages, 2, 256, 256, device=dev).to(bf)
        vc = torch.randn(nseq * pages, 2, 256, 256, device=dev).to(bf)
        bt = torch.arange(nseq * pages, device=dev, dtype=torch.int32).view(nseq, pages)
        cu = torch.arange(nseq + 1, device=dev, dtype=torch.int32) * n
        cl = torch.full((nseq,), n, device=dev, dtype=torch.int32)
        flops = 4 * nseq * 8 * 256 * (n * (n + 1) // 2)
        fn = lambda: torch.ops.isb.attention_prefill_tc(q, gate, kc, vc, cu, cl, bt, 0.0625, True, n)  # noqa: E731
        return [fn], (q.numel() * 2 * 3 + kc.numel() * 4), flops
    out["attention_prefill_tc"] = attention_prefill

    def gdn_chunked(nseq: int, n: int):
        # chunked GDN prefill: nseq sequences of n tokens, 16 key / 16 value heads (0.8B shape)
        hk = hv = 16
        d = 128
        c = 2 * hk * d + hv * d
        p = c + hv * d + 2 * hv
        t = nseq * n
        proj = torch.randn(t, p, device=dev).to(bf)
        conv_w = (torch.randn(c, 4, device=dev) * 0.5).to(bf)
        a_log, dt = torch.zeros(hv, device=dev), torch.ones(hv, device=dev)
        nw = torch.ones(d, device=dev).to(bf)
        slots = torch.arange(nseq, device=dev, dtype=torch.int32)
        rec = torch.zeros(nseq + 1, hv, d, d, device=dev)
        conv = torch.zeros(nseq + 1, c, 3, device=dev).to(bf)
        per = (n + 63) // 64
        seq, t0, nn = [], [], []
        for i in range(nseq):
            for st in range(0, n, 64):
                seq.append(i)
                t0.append(i * n + st)
                nn.append(min(64, n - st))
        nc = len(seq)
        info = torch.tensor(seq + t0 + nn + [i * per for i in range(nseq + 1)], dtype=torch.int32, device=dev)
        cu = torch.arange(nseq + 1, dtype=torch.int32, device=dev) * n
        fn = lambda: torch.ops.isb.gdn_prefill_chunked(proj, cu, slots, info, nc, conv_w, a_log, dt, nw, rec,  # noqa
                                                       conv, hk, hv, 1e-6)
        return [fn], proj.numel() * 2 + t * hv * d * 2, 0
    out["gdn_prefill_chunked"] = lambda: gdn_chunked(1, 8192)
    out["gdn_prefill_chunked_32x512"] = lambda: gdn_chunked(32, 512)

    def acc_norm():
        resid = torch.randn(b, 1024, device=dev).to(bf)
        nwh = torch.zeros(1024, device=dev).to(bf)
        acc = torch.zeros(b, 1024, device=dev)
        return [lambda: ops.add_rmsnorm_acc(acc, resid, nwh, 1e-6, True)], b * 1024 * (8 + 4 + 2), 0
    out["add_rmsnorm_acc"] = acc_norm
    return out


def tp_bench(batches=(1, 8, 128)) -> None:
    """Fused tensor-parallel paths vs the NCCL baseline; run under torch.distributed.run.

    * Row-parallel GEMM fused with the reduce-scatter (fp32 partial rows red.add'ed into their
      owner's accumulator over NVLink) + the owner's residual add + RMSNorm + all-gather push
      (``TPComm.row_parallel_residual_norm``), at the decode shape (0.8B MLP down, hidden 1024,
      intermediate 3584 / TP) for several batches, at the 27B MLP down shape (batch 64), and for a
      2048-token prefill chunk followed by the gate_up + SiLU GEMM.
    * Vocab-parallel LM head fused with the cross-rank argmax.
    Device time per call inside a CUDA graph (20 calls per graph, 5 replays), max over ranks.
    Roofline = max(FLOPs / measured bf16 peak, bytes this rank sends over NVLink / 770 GB/s,
    weight bytes / measured HBM).  The NCCL baseline is the same GEMM + ``dist.all_reduce`` of
    the bf16 product + the add+RMSNorm kernel.
    """
    import torch.distributed as dist

    from inference_systems_b200.parallel.comm import TPComm, shard_rows

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method="env://")
    hbm, tflops, src = peaks()
    nvlink = 770.0
    h, vocab = 1024, 248320 // world
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(rank)
    comms: dict[int, TPComm] = {}

    def comm_for(hh: int) -> TPComm:
        if hh not in comms:
            comms[hh] = TPComm(dev, rank, world, hh, None, max_tokens=2048)
        return comms[hh]

    rows = []

    def timed(fn, calls=20):
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(calls):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        dist.barrier()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for _ in range(calls):
                fn()
        gr.replay()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            gr.replay()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) * 1e3 / (5 * calls)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        del gr
        return float(t.item())

    def emit(row):
        rows.append(row)
        if rank == 0:
            print(json.dumps(row), flush=True)

    def link_bytes(T, hh):
        """Bytes this rank sends per exchange: partial sums of the other ranks' rows + its rows to every peer."""
        s = shard_rows(T, world)
        return (T - min(s, T)) * hh * 2 + (world - 1) * min(s, T) * hh * 2

    # decode: MLP down projection + exchange; 0.8B at several batches and the 27B shape at 64
    for hh, full_inter, b in [(1024, 3584, bb) for bb in batches] + [(5120, 17408, 64)]:
        ii = full_inter // world
        cm = comm_for(hh)
        wd = (torch.randn(hh, ii, device=dev, generator=g) * 0.02).to(bf)
        nwd = torch.zeros(hh, device=dev).to(bf)
        x = torch.randn(b, ii, device=dev, generator=g).to(bf)
        res = torch.randn(b, hh, device=dev, generator=g).to(bf)
        fused = timed(lambda: cm.row_parallel_residual_norm(x, wd, res, nwd, 1e-6, True))
        local_gemm = timed(lambda: ops.linear(x, wd))
        zero = torch.zeros(b, hh, device=dev, dtype=bf)
        local_norm = timed(lambda: ops.add_rmsnorm(zero, res, nwd, 1e-6, True))

        def nccl_path():
            y = ops.linear(x, wd)
            dist.all_reduce(y)
            return ops.add_rmsnorm(y, res, nwd, 1e-6, True)

        base = timed(nccl_path)
        flops = 2 * b * ii * hh
        roof = max(flops / (tflops * 1e12) * 1e6, link_bytes(b, hh) / (nvlink * 1e9) * 1e6,
                   (hh * ii * 2) / (hbm * 1e9) * 1e6)
        emit({"path": "row-parallel GEMM + reduce-scatter -> residual + RMSNorm + all-gather", "tp": world,
              "batch": b, "hidden": hh, "inter_per_rank": ii, "fused_us": round(fused, 2),
              "nccl_baseline_us": round(base, 2), "local_gemm_us": round(local_gemm, 2),
              "local_add_norm_us": round(local_norm, 2), "roofline_us": round(roof, 3),
              "fraction_of_roofline": round(roof / fused, 3)})
    # LM head + cross-rank argmax
    cm = comm_for(h)
    lm = (torch.randn(vocab, h, device=dev, generator=g) * 0.02).to(bf)
    for b in batches:
        hid = torch.randn(b, h, device=dev, generator=g).to(bf)
        temps = torch.zeros(b, device=dev)
        rng = torch.zeros(2, dtype=torch.int32, device=dev)
        fused = timed(lambda: cm.lm_head_sample(hid, lm, temps, rng, rank * vocab), calls=4)
        roof = max(2 * b * vocab * h / (tflops * 1e12) * 1e6, vocab * h * 2 / (hbm * 1e9) * 1e6,
                   (world - 1) * b * 8 / (nvlink * 1e9) * 1e6)
        emit({"path": "vocab-parallel LM head -> cross-rank argmax", "tp": world, "batch": b,
              "fused_us": round(fused, 2), "roofline_us": round(roof, 2), "fraction_of_roofline": round(roof / fused, 3)})
    # prefill chunk: row GEMM + reduce-scatter -> norm + all-gather -> gate_up + SiLU GEMM
    for hh, full_inter, T in ((1024, 3584, 2048), (5120, 17408, 2048)):
        ii = full_inter // world
        cm = comm_for(hh)
        wd = (torch.randn(hh, ii, device=dev, generator=g) * 0.02).to(bf)
        wgu = (torch.randn(2 * ii, hh, device=dev, generator=g) * 0.02).to(bf)
        nwd = torch.zeros(hh, device=dev).to(bf)
        y = torch.randn(T, ii, device=dev, generator=g).to(bf)
        res = torch.randn(T, hh, device=dev, generator=g).to(bf)

        def fused_path():
            x = cm.row_parallel_residual_norm(y, wd, res, nwd, 1e-6, True)
            return ops.linear_silu_mul(x, wgu)

        def nccl_path2():
            z = ops.linear(y, wd)
            dist.all_reduce(z)
            x = ops.add_rmsnorm(z, res, nwd, 1e-6, True)
            return ops.linear_silu_mul(x, wgu)

        fused = timed(fused_path, calls=4)
        base = timed(nccl_path2, calls=4)
        flops = 2 * T * ii * hh + 2 * T * hh * 2 * ii
        wbytes = (hh * ii + 2 * ii * hh) * 2
        roof = max(flops / (tflops * 1e12) * 1e6, link_bytes(T, hh) / (nvlink * 1e9) * 1e6, wbytes / (hbm * 1e9) * 1e6)
        emit({"path": "row GEMM + reduce-scatter -> residual + RMSNorm + all-gather -> gate_up GEMM",
              "tp": world, "tokens": T, "hidden": hh, "inter_per_rank": ii,
              "fused_us": round(fused, 2), "nccl_baseline_us": round(base, 2), "roofline_us": round(roof, 2),
              "fraction_of_roofline": round(roof / fused, 3)})
    torch.cuda.synchronize()
    err = torch.ops.isb.error_word()
    for cm in comms.values():
        cm.close()
    dist.barrier()
    dist.destroy_process_group()
    assert err == 0, f"device error word {err:#x}"


def tp_emulated_bench() -> None:
    """The tensor-parallel exchange kernels on ONE GPU with W ranks laid out as local buffers.

    Times, per launch inside a CUDA graph: the row-parallel GEMM with the reduce-scatter epilogue
    (``tp_gemm_rs``) next to the same GEMM accumulating locally (``gemm_accum``), and the owner
    kernel (``tp_norm_allgather``, final wait off: nothing on one GPU waits for a later launch).
    Isolates the kernels' own cost from cross-GPU latency."""
    from inference_systems_b200.parallel.comm import shard_rows

    c = ops.cuda_ops()
    dev, bf = "cuda", torch.bfloat16
    rows = []
    for world, b, hh, inter in ((2, 1, 1024, 3584), (2, 128, 1024, 3584), (8, 128, 1024, 3584),
                                (2, 64, 5120, 17408), (2, 2048, 1024, 3584)):
        k = inter // world
        s = shard_rows(b, world)
        one = b * hh <= 256 * 1024
        srows = b if one else s
        slots = [torch.zeros(world, srows, hh, dtype=bf, device=dev) for _ in range(world)]
        xs = [torch.zeros(b, hh, dtype=bf, device=dev) for _ in range(world)]
        ctl = [torch.zeros(8, dtype=torch.int32, device=dev) for _ in range(world)]
        staging = torch.zeros(b, hh, device=dev)
        tab = lambda ts, off=0: torch.tensor([t.data_ptr() + off for t in ts], dtype=torch.int64, device=dev)  # noqa: E731
        slot_ptrs, rs_ptrs, ag_ptrs, x_ptrs = tab(slots), tab(ctl), tab(ctl, 4), tab(xs)
        x = torch.randn(b, k, device=dev).to(bf)
        w = (torch.randn(hh, k, device=dev) * 0.02).to(bf)
        res = torch.randn(b, hh, device=dev).to(bf)
        nw = torch.zeros(hh, device=dev).to(bf)
        acc = torch.zeros(b, hh, device=dev)
        ctas = c.tp_gemm_rs(x, w, slot_ptrs, srows, staging, rs_ptrs, 0, s, 0, one)
        t_rs = graph_time_us([lambda: c.tp_gemm_rs(x, w, slot_ptrs, srows, staging, rs_ptrs, 0, s, 0, one)] * 20)
        t_acc = graph_time_us([lambda: c.gemm_accum(x, w, acc, 0)] * 20)
        t_norm = graph_time_us([lambda: c.tp_norm_allgather(slots[0], res, nw, x_ptrs, ag_ptrs, ctl[0], b, s, 0, 0,
                                                            1e-6, True, False, one)] * 20)
        t_accnorm = graph_time_us([lambda: ops.add_rmsnorm_acc(acc, res, nw, 1e-6, True)] * 20)
        torch.cuda.synchronize()
        row = {"path": "exchange kernels on one GPU (emulated ranks)", "one_shot": one, "tp": world, "tokens": b,
               "hidden": hh,
               "inter_per_rank": k, "gemm_ctas": ctas, "gemm_rs_us": round(t_rs, 2), "gemm_accum_us": round(t_acc, 2),
               "owner_norm_allgather_us": round(t_norm, 2), "local_add_norm_us": round(t_accnorm, 2)}
        rows.append(row)
        print(json.dumps(row), flush=True)
    assert torch.ops.isb.error_word() == 0


def split_sweep_bench() -> None:
    """Split-K factor of the accumulating decode GEMM (``gemm_accum``) and of the reduce-scatter
    GEMM (``tp_gemm_rs``, one-shot, 2 emulated ranks): time per launch with the weights cycled
    through enough copies to exceed L2, so each launch streams its weights from HBM."""
    c = ops.cuda_ops()
    dev, bf = "cuda", torch.bfloat16
    hh = 1024
    for k in (3584, 2048, 1792, 448):
        copies = max(2, (300 << 20) // (hh * k * 2))
        ws = [(torch.randn(hh, k, device=dev) * 0.02).to(bf) for _ in range(copies)]
        for b in (1, 128):
            x = torch.randn(b, k, device=dev).to(bf)
            acc = torch.zeros(b, hh, device=dev)
            slots = [torch.zeros(2, b, hh, dtype=bf, device=dev) for _ in range(2)]
            ctl = [torch.zeros(8, dtype=torch.int32, device=dev) for _ in range(2)]
            staging = torch.zeros(b, hh, device=dev)
            tab = lambda ts: torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=dev)  # noqa: E731
            slot_ptrs, rs_ptrs = tab(slots), tab(ctl)
            row = {"path": "split-K sweep (weights from HBM)", "tokens": b, "N": hh, "K": k,
                   "weight_mb": round(hh * k * 2 / 1e6, 2)}
            for sp in (1, 2, 4, 8, 16, 0):
                if sp > (k + 63) // 64:
                    continue
                t_acc = graph_time_us([lambda w=w: c.gemm_accum(x, w, acc, sp) for w in ws])
                t_rs = graph_time_us([lambda w=w: c.tp_gemm_rs(x, w, slot_ptrs, b, staging, rs_ptrs, 0, b, sp, True)
                                      for w in ws])
                key = "auto" if sp == 0 else str(sp)
                row[f"accum_us_s{key}"] = round(t_acc, 2)
                row[f"rs_us_s{key}"] = round(t_rs, 2)
            torch.cuda.synchronize()
            print(json.dumps(row), flush=True)
    assert torch.ops.isb.error_word() == 0


def main():
    if "--split-sweep" in sys.argv:
        load_extension()
        split_sweep_bench()
        return
    if "--tp-emulated" in sys.argv:
        load_extension()
        tp_emulated_bench()
        return
    if "--tp" in sys.argv:
        load_extension()
        tp_bench()
        return
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--only", default=None)
    ap.add_argument("--json", default=None)
    ap.add_argument("--once", action="store_true",
                    help="run each selected op twice (warm-up + one launch) with no graph: a small case for ncu -c 1")
    args = ap.parse_args()
    load_extension()
    hbm, tflops, src = peaks()
    rows = []
    for name, build in cases(args.batch).items():
        if args.only and not any(o in name for o in args.only.split(",")):
            continue
        fns, nbytes, flops = build()
        if args.once:
            fns[0]()
            fns[-1]()
            torch.cuda.synchronize()
            print(json.dumps({"op": name, "batch": args.batch, "launched": 2}), flush=True)
            continue
        us = graph_time_us(fns)
        gbs = nbytes / (us * 1e-6) / 1e9
        tf = flops / (us * 1e-6) / 1e12 if flops else 0.0
        rows.append({"op": name, "batch": args.batch, "us": round(us, 2), "GB/s": round(gbs, 1),
                     f"hbm_frac_of_{src}": round(gbs / hbm, 3), "TFLOP/s": round(tf, 1),
                     f"tc_frac_of_{src}": round(tf / tflops, 4) if flops else None})
        print(json.dumps(rows[-1]), flush=True)
    torch.cuda.synchronize()
    assert torch.ops.isb.error_word() == 0
    if args.json:
        with open(args.json, "w") as f:
            json.dump(rows, f, indent=1)


if __name__ == "__main__":
    main()
