"""Per-kernel microbenchmarks of the sm_100a ops at Qwen3.5 decode / prefill shapes.

    python bench_kernels.py [--batch 128] [--only gemm_in_proj] [--iters 20]

Each op is timed with CUDA events over ``--iters`` launches after warm-up,
with a 256 MiB L2-flush write between launches (the flush is excluded from
the timing by timing every launch separately).  Achieved bandwidth uses the
algorithmic bytes (operands read once, outputs written once) and is reported
against the measured HBM copy bandwidth in ``MEASURED_PEAKS.json`` (falls back
to 6650 GB/s); GEMM FLOP rates against its measured bf16 peak (fallback 1590 TFLOP/s).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from inference_systems_b200 import ops  # noqa: E402
from inference_systems_b200.ops._ext import load_extension  # noqa: E402
from inference_systems_b200.ops import reference as ref  # noqa: E402


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def timeit(fn, iters: int) -> float:
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(3):
        fn()
    times = []
    for _ in range(iters):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3)
    times.sort()
    return times[len(times) // 2]


def cases(b: int):
    dev = "cuda"
    bf = torch.bfloat16
    x = torch.randn(b, 1024, device=dev).to(bf)
    out = {}

    def gemm_case(name, n, k, silu=False):
        a = torch.randn(b, k, device=dev).to(bf)
        w = (torch.randn(n, k, device=dev) * 0.02).to(bf)
        fn = (lambda: ops.linear_silu_mul(a, w)) if silu else (lambda: ops.linear(a, w))
        out_cols = n // 2 if silu else n
        out[name] = (fn, (n * k + b * k + b * out_cols) * 2, 2 * b * n * k)

    gemm_case("gemm_gdn_in_proj", 8224, 1024)
    gemm_case("gemm_attn_qkv", 5120, 1024)
    gemm_case("gemm_out_proj", 1024, 2048)
    gemm_case("gemm_down", 1024, 3584)
    gemm_case("gemm_gate_up_silu", 7168, 1024, silu=True)
    w = (torch.randn(248320, 1024, device=dev) * 0.02).to(bf)
    temps = torch.zeros(b, device=dev)
    rng = torch.zeros(2, dtype=torch.int32, device=dev)
    out["lm_head_sample"] = (lambda: ops.lm_head_sample(x, w, temps, rng, 0), (w.numel() + x.numel()) * 2,
                             2 * b * w.numel())
    # GDN decode: 16 key/value heads, slot pool of 2b+1
    hk = hv = 16
    d = 128
    c = 2 * hk * d + hv * d
    p = c + hv * d + 2 * hv
    proj = torch.randn(b, p, device=dev).to(bf)
    conv_w = (torch.randn(c, 4, device=dev) * 0.5).to(bf)
    a_log = torch.zeros(hv, device=dev)
    dt = torch.ones(hv, device=dev)
    nw = torch.ones(d, device=dev).to(bf)
    rec = torch.randn(2 * b + 1, hv, d, d, device=dev) * 0.01
    conv = torch.zeros(2 * b + 1, c, 3, device=dev).to(bf)
    slots = torch.randperm(2 * b, device=dev)[:b].to(torch.int32)
    out["gdn_decode"] = (lambda: torch.ops.isb.gdn_decode(proj, slots, conv_w, a_log, dt, nw, rec, conv, hk, hv, d, d,
                                                          1e-6),
                         b * hv * d * d * 4 * 2 + proj.numel() * 2 + b * hv * d * 2, 0)
    # attention decode: 8 q heads / 2 kv heads, hd 256, context 640
    ctx = 640
    nblk = b * 3 + 4
    kc = torch.randn(nblk, 2, 256, 256, device=dev).to(bf)
    vc = torch.randn_like(kc)
    bt = torch.arange(b * 3, device=dev, dtype=torch.int32).view(b, 3)
    bt = torch.cat((bt, torch.full((b, 2), -1, device=dev, dtype=torch.int32)), 1)
    cl = torch.full((b,), ctx, device=dev, dtype=torch.int32)
    q = torch.randn(b, 8, 256, device=dev).to(bf)
    qkv = torch.randn(b, 5120, device=dev).to(bf)
    out["attention_decode"] = (lambda: torch.ops.isb.attention_decode(q, qkv, kc, vc, cl, bt, 0.0625, True),
                               b * 2 * ctx * 256 * 2 * 2 + q.numel() * 4, 4 * b * 8 * ctx * 256)
    r = torch.randn(b, 1024, device=dev).to(bf)
    nwh = torch.zeros(1024, device=dev).to(bf)
    out["add_rmsnorm"] = (lambda: ops.add_rmsnorm(x, r, nwh, 1e-6, True), b * 1024 * 2 * 4, 0)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--only", default=None)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--json", default=None)
    args = ap.parse_args()
    load_extension()
    hbm, tflops, src = peaks()
    rows = []
    for name, (fn, nbytes, flops) in cases(args.batch).items():
        if args.only and args.only not in name:
            continue
        us = timeit(fn, args.iters)
        gbs = nbytes / (us * 1e-6) / 1e9
        tf = flops / (us * 1e-6) / 1e12 if flops else 0.0
        rows.append({"op": name, "batch": args.batch, "us": round(us, 2), "GB/s": round(gbs, 1),
                     f"hbm_frac_of_{src}": round(gbs / hbm, 3), "TFLOP/s": round(tf, 1),
                     f"tc_frac_of_{src}": round(tf / tflops, 4) if flops else None})
    for r in rows:
        print(json.dumps(r))
    torch.cuda.synchronize()
    assert torch.ops.isb.error_word() == 0
    if args.json:
        with open(args.json, "w") as f:
            json.dump(rows, f, indent=1)


if __name__ == "__main__":
    main()
