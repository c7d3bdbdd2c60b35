"""Headline benchmark: Qwen3.5-0.8B-shape decode throughput (tokens/s, whole job).

    python bench.py --gpus N --steps K --warmup W [--batch 128] [--impl isb|reference]

For N > 1 the script is launched once per GPU by ``torch.distributed.run``;
rank 0 drives the engine, the other ranks serve it (tensor parallelism).

Workload: random-init Qwen3.5-0.8B-shape weights (bf16,
fp32 GDN state), ``--batch`` prompts of 512 uniform-random tokens, greedy
decoding with CUDA-graph decode steps.

Reported numbers:
* ``value``  -- device-timed decode throughput: K back-to-back replays of the
  decode-step CUDA graph (embedding -> 24 layers -> LM head + sampling for the
  whole batch), CUDA events on the launching stream with a barrier and
  synchronize on both sides, max over ranks.
* ``e2e``    -- the same metric through the public engine API: K
  ``LLMEngine.step()`` calls, each of which copies that step's packed inputs
  host->device from pinned memory and reads the sampled tokens back.
* ``ttft_p50_ms`` / ``tpot_p50_ms`` from the per-request lifecycle metrics.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (box, max over ranks) Qwen3.5 at TP 1/2/4/8; p50 TTFT & TPOT"
MODEL = "qwen3_5-0.8b"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=64)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--batch", type=int, default=128)
    p.add_argument("--prompt-len", type=int, default=512)
    p.add_argument("--output-len", type=int, default=256)
    p.add_argument("--impl", default="isb", choices=["isb", "reference"])
    p.add_argument("--model", default=MODEL)
    p.add_argument("--breakdown", action="store_true",
                   help="after timing, profile 3 decode-graph replays with torch.profiler (kernel-time shares)")
    return p.parse_args()


def kernel_breakdown(replay, path: str, n: int = 3) -> None:
    """Per-kernel device time of ``n`` replays (torch.profiler / CUPTI), written as a text table."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(n):
            replay()
        torch.cuda.synchronize()
    agg: dict[str, list[float]] = {}
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            agg.setdefault(ev.name, []).append(ev.device_time_total if hasattr(ev, "device_time_total") else ev.cuda_time_total)
    total = sum(sum(v) for v in agg.values())
    rows = sorted(agg.items(), key=lambda kv: -sum(kv[1]))
    with open(path, "w") as f:
        f.write(f"total device us per replay: {total / n:.1f}\n")
        for name, v in rows:
            f.write(f"{sum(v) / n:10.1f} us  {100 * sum(v) / total:5.1f}%  x{len(v) // n:<4d} {name[:160]}\n")


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.path = os.path.join(ROOT, "gpurun_out", f"clocks_gpu{gpu}.csv")

    def __enter__(self):
        os.makedirs(os.path.dirname(self.path), exist_ok=True)
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        rows = []
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]) if parts[3] not in ("[N/A]", "N/A") else 0.0,
                             parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        loaded = [r for r in rows if r[2] > 200.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(loaded)}


# --------------------------------------------------------------- own engine
def run_isb(args, rank: int, world: int) -> dict | None:
    import torch

    from inference_systems_b200 import SamplingParams
    from inference_systems_b200.engine.llm_engine import LLMEngine, serve_worker
    from inference_systems_b200.models.presets import preset

    cfg = preset(args.model)
    b = args.batch
    total_steps = args.steps + args.warmup
    kw = dict(load_format="dummy", device="cuda", tensor_parallel_size=world, max_num_seqs=b,
              max_num_state_slots=b, max_model_len=args.prompt_len + args.output_len + total_steps + 32,
              max_num_batched_tokens=16384, max_cudagraph_batch_size=b, enforce_eager=False,
              dist_port=int(os.environ.get("MASTER_PORT", "29500")) + 17, gpu_memory_utilization=0.85)
    if world > 1 and rank > 0:
        serve_worker(cfg, **kw)
        return None
    llm = LLMEngine(cfg, **kw)
    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, cfg["vocab_size"], (b, args.prompt_len), generator=g).tolist()
    sp = SamplingParams(temperature=0.0, max_tokens=args.output_len + total_steps + 8, ignore_eos=True)
    for p in prompts:
        llm.add_request(p, sp)
    # prefill until every request produced its first token
    t0 = time.perf_counter()
    while llm.scheduler.waiting or any(s.num_completion_tokens == 0 for s in llm.scheduler.running):
        llm.step()
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    runner = llm.model_runner
    for _ in range(args.warmup):
        llm.step()
    torch.cuda.synchronize()

    # ---------------- end-to-end: public engine API, K steps
    h2d0, d2h0 = runner.h2d_bytes, runner.d2h_bytes
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        torch.cuda.synchronize()
        ev0.record()
        wall0 = time.perf_counter()
        decoded = 0
        for _ in range(args.steps):
            _, stats = llm.step()
            decoded += stats.decode_tokens
        ev1.record()
        torch.cuda.synchronize()
        wall_e2e = time.perf_counter() - wall0
        e2e_ms = ev0.elapsed_time(ev1)
        h2d = (runner.h2d_bytes - h2d0) / args.steps
        d2h = (runner.d2h_bytes - d2h0) / args.steps
        # ---------------- device-timed: K decode-graph replays, max over ranks
        dev_ms = runner.call("bench_replay", b, args.warmup, args.steps)
    clocks = clk.summary()
    launches = runner.graph_kernel_count(b)
    if args.breakdown:
        g = runner.graphs[runner._graph_bucket(b)]
        kernel_breakdown(g.replay, os.path.join(ROOT, "gpurun_out", f"breakdown_tp{world}_b{b}.txt"))
    req = [s.lifecycle_metrics() for s in llm.scheduler.running]
    ttfts = sorted(m["ttft_ms"] for m in req if m["ttft_ms"] is not None)
    tpots = sorted(m["tpot_ms"] for m in req if m["tpot_ms"] is not None)
    value = b * args.steps / (dev_ms / 1e3)
    out = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dev_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (uniform-random token ids; random-init N(0,0.02) weights of the 0.8B architecture)",
        "config": {"model": "Qwen3.5-0.8B-shape hybrid (24 layers, 18 GDN + 6 gated attention, hidden 1024, vocab 248320)",
                   "global_batch": b, "seq_len": args.prompt_len, "parallelism": f"tp{world}",
                   "l2": "inputs larger than L2 (weights 1.5 GB + GDN state per step exceed the 126 MB L2)",
                   "cuda_graph_decode": True},
        "clocks": clocks,
        "e2e": {"value": round(decoded / (e2e_ms / 1e3), 1), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "wall_s": round(wall_e2e, 4),
                "api": "LLMEngine.step() (scheduler + packed pinned H2D + CUDA-graph step + token D2H)"},
        "gpu_launches": launches * args.steps,
        "gpu_launches_per_step": launches,
        "ttft_p50_ms": round(ttfts[len(ttfts) // 2], 2) if ttfts else None,
        "tpot_p50_ms": round(tpots[len(tpots) // 2], 3) if tpots else None,
        "prefill_s": round(prefill_s, 3),
        "impl": "isb",
    }
    llm.exit()
    return out


# --------------------------------------------------------------- reference
def run_reference(args, rank: int, world: int) -> dict | None:
    from bench_reference import run as ref_run
    return ref_run(args, rank, world, METRIC)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world != args.gpus:
        world = args.gpus
    if args.impl == "reference":
        out = run_reference(args, rank, world)
    else:
        out = run_isb(args, rank, world)
    if out is not None and rank == 0:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
