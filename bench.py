"""Headline benchmark: Qwen3.5-0.8B-shape decode throughput (tokens/s, whole job).

    python bench.py --gpus N --steps K --warmup W [--batch 128] [--impl isb|reference]

For N > 1 the script is launched once per GPU by ``torch.distributed.run``;
rank 0 drives the engine, the other ranks serve it (tensor parallelism).

Workload (the 0.8B decode configuration): random-init Qwen3.5-0.8B-shape weights (bf16,
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
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (box, max over ranks) Qwen3.5 at TP 1/2/4/8; p50 TTFT & TPOT"
MODEL = "qwen3_5-0.8b"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=128)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--batch", type=int, default=128)
    p.add_argument("--sweep", default=None, help="extra batch sizes, e.g. 1,8,32 (reported under 'sweep')")
    p.add_argument("--prompt-len", type=int, default=512)
    p.add_argument("--output-len", type=int, default=256)
    p.add_argument("--impl", default="isb", choices=["isb", "reference"])
    p.add_argument("--model", default=MODEL)
    p.add_argument("--mtp", type=int, default=0,
                   help="K > 0: MTP speculative decode with K drafts vs target-only")
    p.add_argument("--mtp-accept", type=float, default=0.6, help="seeded draft/target agreement probability")
    p.add_argument("--prefill-breakdown", action="store_true",
                   help="profile one prefill step of --batch prompts of --prompt-len tokens (kernel-time shares) and exit")
    p.add_argument("--breakdown", action="store_true",
                   help="after timing, profile 3 decode-graph replays with torch.profiler (kernel-time shares)")
    p.add_argument("--breakdown-dir", default="breakdowns",
                   help="folder (relative to the repository) for the --breakdown / --prefill-breakdown tables")
    return p.parse_args()


def kernel_breakdown(run, path: str, n: int = 3) -> None:
    """Per-kernel device time of ``n`` calls of ``run`` written as a text table (single process)."""
    from inference_systems_b200.engine.profiler import kernel_time_table

    os.makedirs(os.path.dirname(path), exist_ok=True)
    with open(path, "w") as f:
        f.write(kernel_time_table(run, n))


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock, power and clock-event reasons through NVML every ``period_s`` (read-only)."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, gpu: int, period_s: float = 0.01):
        self.gpu, self.period = gpu, period_s
        self.rows: list[tuple[float, float, int]] = []
        self.max_mhz = None
        self._stop = None

    def __enter__(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self._h = h
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception:  # noqa: BLE001 - no NVML: report unsampled
            self._nvml = None
            return self
        self._stop = threading.Event()

        def loop():
            n = self._nvml
            while not self._stop.is_set():
                try:
                    self.rows.append((float(n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM)),
                                      n.nvmlDeviceGetPowerUsage(self._h) / 1000.0,
                                      int(n.nvmlDeviceGetCurrentClocksEventReasons(self._h))))
                except Exception:  # noqa: BLE001
                    pass
                self._stop.wait(self.period)

        self._t = threading.Thread(target=loop, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        if self._stop is not None:
            self._stop.set()
            self._t.join(timeout=2)

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "samples": 0}
        loaded = [r for r in self.rows if r[1] > 200.0] or self.rows
        n = self._nvml
        reasons = sorted({name for name, attr in self.REASONS for r in loaded if r[2] & getattr(n, attr)})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(loaded), "power_w_median": round(statistics.median(r[1] for r in loaded), 1),
                "source": "NVML every 10 ms during the timed regions"}


# --------------------------------------------------------------- own engine
def model_desc(name: str) -> tuple[str, str]:
    """(config.model text, data text) for a preset, from its dimensions."""
    from inference_systems_b200.models.presets import preset

    c = preset(name)
    types = c.get("layer_types") or []
    n_lin = sum(t == "linear_attention" for t in types)
    size = {"qwen3_5-0.8b": "0.8B", "qwen3_5-9b": "9B", "qwen3_5-27b": "27B"}.get(name, name)
    model = (f"Qwen3.5-{size}-shape hybrid ({c['num_hidden_layers']} layers, {n_lin} GDN + "
             f"{len(types) - n_lin} gated attention, hidden {c['hidden_size']}, vocab {c['vocab_size']})")
    data = f"synthetic (uniform-random token ids; random-init N(0,0.02) weights of the {size} architecture)"
    return model, data


def _p50(xs):
    xs = sorted(x for x in xs if x is not None)
    return round(xs[len(xs) // 2], 3) if xs else None


def _serve_batch(llm, runner, cfg, b: int, args, clk) -> dict:
    """B requests (512-token prompts) generated to completion through ``LLMEngine.step``.

    Returns the end-to-end decode throughput over exactly ``steps`` decode
    steps (after ``warmup`` decode steps), per-request TTFT/TPOT p50, and the
    device-timed decode throughput of ``steps`` graph replays at this batch.
    """
    import torch

    from inference_systems_b200 import SamplingParams

    g = torch.Generator().manual_seed(b)
    prompts = torch.randint(0, cfg["vocab_size"], (b, args.prompt_len), generator=g).tolist()
    out_len = max(args.output_len, args.warmup + args.steps + 2)
    sp = SamplingParams(temperature=0.0, max_tokens=out_len, ignore_eos=True)
    llm.scheduler.reset_metrics()
    for p in prompts:
        llm.add_request(p, sp)
    t0 = time.perf_counter()
    while llm.scheduler.waiting or any(s.num_completion_tokens == 0 for s in llm.scheduler.running):
        llm.step()
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    first_tokens = sum(s.num_completion_tokens for s in llm.scheduler.running)
    gen0 = torch.cuda.Event(enable_timing=True)
    gen0.record()
    gen_steps = 0
    for _ in range(args.warmup):
        llm.step()
        gen_steps += 1
    torch.cuda.synchronize()
    h2d0, d2h0 = runner.h2d_bytes, runner.d2h_bytes
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk_on = clk.__enter__()
    ev0.record()
    wall0 = time.perf_counter()
    decoded = 0
    for _ in range(args.steps):
        _, stats = llm.step()
        decoded += stats.decode_tokens
    ev1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    e2e_ms = ev0.elapsed_time(ev1)
    h2d = (runner.h2d_bytes - h2d0) / args.steps
    d2h = (runner.d2h_bytes - d2h0) / args.steps
    gen_steps += args.steps
    while not llm.is_finished():  # finish the requests: TTFT / TPOT of complete requests
        llm.step()
        gen_steps += 1
    gen1 = torch.cuda.Event(enable_timing=True)
    gen1.record()
    torch.cuda.synchronize()
    gen_ms = gen0.elapsed_time(gen1)
    gen_tokens = b * out_len - first_tokens
    # device-timed: K decode-graph replays of this batch bucket, max over ranks
    dev_ms = runner.call("bench_replay", b, args.warmup, args.steps)
    clk_on.__exit__(None, None, None)
    req = llm.get_request_metrics()[-b:]
    return {
        "batch": b,
        "value": round(b * args.steps / (dev_ms / 1e3), 1),
        "ms_per_step": round(dev_ms / args.steps, 4),
        "e2e_value": round(decoded / (e2e_ms / 1e3), 1),
        "e2e_wall_s": round(wall, 4),
        "h2d_bytes_per_step": int(h2d),
        "d2h_bytes_per_step": int(d2h),
        "ttft_p50_ms": _p50(m.get("ttft_ms") for m in req),
        "tpot_p50_ms": _p50(m.get("tpot_ms") for m in req),
        "prefill_s": round(prefill_s, 3),
        "output_len": out_len,
        # the whole decode phase (context 513 .. 512 + output_len) through LLMEngine.step, not just
        # the timed window at its start
        "full_generation": {"decode_tokens": gen_tokens, "steps": gen_steps,
                            "e2e_tok_s": round(gen_tokens / (gen_ms / 1e3), 1),
                            "mean_step_ms": round(gen_ms / max(gen_steps, 1), 4)},
    }


def prefill_breakdown(args) -> None:
    """Kernel-time table of the first prefill step (no JSON line; diagnostics only)."""
    import torch

    from inference_systems_b200 import SamplingParams
    from inference_systems_b200.engine.llm_engine import LLMEngine
    from inference_systems_b200.models.presets import preset

    cfg = preset(args.model)
    b = args.batch
    llm = LLMEngine(cfg, load_format="dummy", device="cuda", max_num_seqs=b, max_num_state_slots=b,
                    max_model_len=args.prompt_len + 64, max_num_batched_tokens=max(16384, args.prompt_len),
                    enforce_eager=True, gpu_memory_utilization=0.85)
    g = torch.Generator().manual_seed(0)
    for _ in range(2):  # first pass warms up, second is profiled
        for p in torch.randint(0, cfg["vocab_size"], (b, args.prompt_len), generator=g).tolist():
            llm.add_request(p, SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True))
        if _ == 0:
            while not llm.is_finished():
                llm.step()
            continue
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        kernel_breakdown(lambda: llm.step(), os.path.join(ROOT, args.breakdown_dir, f"prefill_b{b}_len{args.prompt_len}.txt"), n=1)
        print(json.dumps({"prefill_step_s": round(time.perf_counter() - t0, 4), "batch": b,
                          "prompt_len": args.prompt_len}), flush=True)
        while not llm.is_finished():
            llm.step()
    llm.exit()


def run_isb(args, rank: int, world: int) -> dict | None:
    import torch

    from inference_systems_b200.engine.llm_engine import LLMEngine, serve_worker
    from inference_systems_b200.models.presets import preset

    cfg = preset(args.model)
    batches = sorted({args.batch, *([int(x) for x in args.sweep.split(",")] if args.sweep else [])})
    bmax = max(batches)
    out_len = max(args.output_len, args.warmup + args.steps + 2)
    kw = dict(load_format="dummy", device="cuda", tensor_parallel_size=world, max_num_seqs=bmax,
              max_num_state_slots=bmax, max_model_len=args.prompt_len + out_len + 32,
              max_num_batched_tokens=16384, max_cudagraph_batch_size=bmax, enforce_eager=False,
              dist_port=int(os.environ.get("MASTER_PORT", "29500")) + 17, gpu_memory_utilization=0.85)
    if world > 1 and rank > 0:
        serve_worker(cfg, **kw)
        return None
    llm = LLMEngine(cfg, **kw)
    runner = llm.model_runner
    clk = ClockSampler(torch.cuda.current_device())
    results = {b: _serve_batch(llm, runner, cfg, b, args, clk) for b in batches}
    head = results[args.batch]
    launches = runner.graph_kernel_count(args.batch)
    if args.breakdown:  # every rank replays and profiles (the exchanges need all ranks)
        runner.call("breakdown_replays", args.batch,
                    os.path.join(ROOT, args.breakdown_dir, f"breakdown_tp{world}_b{args.batch}.txt"))
    out = {
        "metric": METRIC,
        "value": head["value"],
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": head["ms_per_step"],
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": model_desc(args.model)[1],
        "config": {"model": model_desc(args.model)[0],
                   "global_batch": args.batch, "seq_len": args.prompt_len, "output_len": head["output_len"],
                   "parallelism": f"tp{world}",
                   "l2": "inputs larger than L2 (weights and GDN state read per step exceed the 126 MB L2)",
                   "cuda_graph_decode": True},
        "clocks": clk.summary(),
        "e2e": {"value": head["e2e_value"], "unit": "tokens/s", "h2d_bytes_per_step": head["h2d_bytes_per_step"],
                "d2h_bytes_per_step": head["d2h_bytes_per_step"], "wall_s": head["e2e_wall_s"],
                "api": "LLMEngine.step() (scheduler + packed pinned H2D + CUDA-graph step + token D2H)"},
        "gpu_launches": launches * args.steps,
        "gpu_launches_per_step": launches,
        "ttft_p50_ms": head["ttft_p50_ms"],
        "tpot_p50_ms": head["tpot_p50_ms"],
        "prefill_s": head["prefill_s"],
        "full_generation": head["full_generation"],
        "impl": "isb",
    }
    if len(batches) > 1:
        out["sweep"] = [results[b] for b in batches]
    llm.exit()
    return out


# ------------------------------------------------------------ MTP speculative decoding
def _decode_run(llm, cfg, b: int, args) -> dict:
    """B requests to completion; device-timed decode phase (after every first token)."""
    import torch

    from inference_systems_b200 import SamplingParams

    g = torch.Generator().manual_seed(1000 + b)
    prompts = torch.randint(0, cfg["vocab_size"], (b, args.prompt_len), generator=g).tolist()
    sp = SamplingParams(temperature=0.0, max_tokens=args.output_len, ignore_eos=True)
    llm.scheduler.reset_metrics()
    for p in prompts:
        llm.add_request(p, sp)
    while llm.scheduler.waiting or any(s.num_completion_tokens == 0 for s in llm.scheduler.running):
        llm.step()
    first = sum(s.num_completion_tokens for s in llm.scheduler.running)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    wall0 = time.perf_counter()
    steps = 0
    while not llm.is_finished():
        llm.step()
        steps += 1
    ev1.record()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    req = llm.get_request_metrics()[-b:]
    tokens = b * args.output_len - first
    return {"batch": b, "decode_tokens_per_s": round(tokens / (ms / 1e3), 1), "decode_steps": steps,
            "decode_ms": round(ms, 2), "wall_s": round(time.perf_counter() - wall0, 3),
            "tpot_p50_ms": _p50(m.get("tpot_ms") for m in req), "ttft_p50_ms": _p50(m.get("ttft_ms") for m in req)}


def run_mtp(args, rank: int, world: int) -> dict | None:
    """MTP speculative decoding (K drafts, seeded agreement p) vs target-only decoding, same workload."""
    import torch

    from inference_systems_b200.engine.llm_engine import LLMEngine, serve_worker
    from inference_systems_b200.models.presets import preset

    cfg = preset(args.model)
    batches = sorted({args.batch, *([int(x) for x in args.sweep.split(",")] if args.sweep else [])})
    bmax = max(batches)
    pages = (args.prompt_len + args.output_len + 2 * args.mtp + 255) // 256 + 1
    res = {}
    for mode in ("target", "mtp"):
        kw = dict(load_format="dummy", device="cuda", tensor_parallel_size=world, max_num_seqs=bmax,
                  max_num_state_slots=bmax, max_model_len=args.prompt_len + args.output_len + 32,
                  max_num_batched_tokens=16384, max_cudagraph_batch_size=bmax, enforce_eager=False,
                  num_kvcache_blocks=bmax * pages + 8,
                  dist_port=int(os.environ.get("MASTER_PORT", "29500")) + 19 + (mode == "mtp"))
        if mode == "mtp":
            kw.update(num_speculative_tokens=args.mtp, mtp_synthetic_acceptance=args.mtp_accept)
        if world > 1 and rank > 0:
            serve_worker(cfg, **kw)
            continue
        llm = LLMEngine(cfg, **kw)
        _decode_run(llm, cfg, min(batches), args)  # warm-up generation
        res[mode] = {b: _decode_run(llm, cfg, b, args) for b in batches}
        if mode == "mtp":
            res["mtp_metrics"] = llm.get_runtime_metrics()["model_runner"].get("mtp", {})
            if args.breakdown:
                drv = llm.model_runner.mtp_driver
                kernel_breakdown(drv.graphs[drv._bucket(args.batch)].replay,
                                 os.path.join(ROOT, args.breakdown_dir, f"breakdown_mtp{args.mtp}_b{args.batch}.txt"))
        llm.exit()
    if rank > 0:
        return None
    rows = []
    for b in batches:
        t, m = res["target"][b], res["mtp"][b]
        rows.append({"batch": b, "target_tok_s": t["decode_tokens_per_s"], "mtp_tok_s": m["decode_tokens_per_s"],
                     "speedup": round(m["decode_tokens_per_s"] / t["decode_tokens_per_s"], 3),
                     "target_tpot_p50_ms": t["tpot_p50_ms"], "mtp_tpot_p50_ms": m["tpot_p50_ms"]})
    head = next(r for r in rows if r["batch"] == args.batch)
    mm = res["mtp_metrics"]
    return {"metric": f"MTP speculative decode tok/s (K={args.mtp}, agreement p={args.mtp_accept}) vs target-only",
            "value": head["mtp_tok_s"], "unit": "tokens/s", "n_gpus": world, "higher_is_better": True,
            "dtype": "bf16", "data": "synthetic prompts; random-init 0.8B-shape target + 1-layer MTP head",
            "config": {"model": "Qwen3.5-0.8B-shape + MTP", "global_batch": args.batch, "seq_len": args.prompt_len,
                       "output_len": args.output_len, "parallelism": f"tp{world}", "num_speculative_tokens": args.mtp,
                       "synthetic_acceptance": args.mtp_accept, "cuda_graph": True},
            "vs_target_only": head["speedup"], "sweep": rows,
            "acceptance_rate": round(mm.get("acceptance_rate", 0.0), 4),
            "mean_emitted_per_round": round(mm.get("mean_emitted_per_round", 0.0), 3),
            "impl": "isb"}


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
    elif args.prefill_breakdown:
        prefill_breakdown(args)
        out = None
    elif args.mtp > 0:
        out = run_mtp(args, rank, world)
    else:
        out = run_isb(args, rank, world)
    if out is not None and rank == 0:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
