"""Online serving benchmark: Poisson arrivals through the engine's public API.

    python bench_serving.py --rate 16 --requests 256 [--gpus N] [--model qwen3_5-0.8b]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        --master-port 29600 bench_serving.py --gpus 8 --rate 32

Workload (the online serving configuration): arrivals are a Poisson process at ``--rate``
requests/s; prompt lengths are lognormal with median ``--prompt-median``
(clipped to ``--prompt-max``); output lengths are lognormal with median
``--output-median``; a ``--prefix-share`` fraction of the requests starts with
one shared random ``--prefix-len``-token hot prefix.  The engine runs chunked
prefill of ``--chunk`` tokens, 256-token KV pages with a 16-token prefix match
unit and (unless ``--no-prefix-cache``) the hybrid prefix cache, which restores
GDN recurrent/conv checkpoints for the shared prefix.

Requests are admitted between engine steps at their arrival times (wall
clock); TTFT counts from the arrival time.  Rank 0 prints one JSON line with
p50/p99 TTFT, TPOT and end-to-end latency, request throughput and output
token throughput.  Token ids are synthetic and weights are random-init.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--model", default="qwen3_5-0.8b")
    p.add_argument("--rate", type=float, default=16.0, help="Poisson arrival rate (requests/s)")
    p.add_argument("--requests", type=int, default=256)
    p.add_argument("--prompt-median", type=int, default=1024)
    p.add_argument("--prompt-max", type=int, default=8192)
    p.add_argument("--output-median", type=int, default=256)
    p.add_argument("--output-max", type=int, default=1024)
    p.add_argument("--prefix-share", type=float, default=0.3)
    p.add_argument("--prefix-len", type=int, default=2048)
    p.add_argument("--chunk", type=int, default=2048, help="max prefill tokens per step")
    p.add_argument("--max-num-seqs", type=int, default=256)
    p.add_argument("--no-prefix-cache", action="store_true")
    p.add_argument("--checkpoint-gib", type=int, default=4, help="GDN prefix-checkpoint pool budget (GiB)")
    p.add_argument("--seed", type=int, default=0)
    return p.parse_args()


def workload(args, vocab: int):
    import numpy as np

    rng = np.random.default_rng(args.seed)
    hot = rng.integers(0, vocab, args.prefix_len).tolist()
    reqs, t = [], 0.0
    for _ in range(args.requests):
        t += rng.exponential(1.0 / args.rate)
        n = int(min(args.prompt_max, max(16, round(rng.lognormal(math.log(args.prompt_median), 0.8)))))
        out = int(min(args.output_max, max(8, round(rng.lognormal(math.log(args.output_median), 0.6)))))
        if rng.random() < args.prefix_share:
            tail = max(16, n - args.prefix_len)
            prompt = hot + rng.integers(0, vocab, tail).tolist()
            prompt = prompt[: args.prompt_max]
            shared = True
        else:
            prompt = rng.integers(0, vocab, n).tolist()
            shared = False
        reqs.append((t, prompt, out, shared))
    return reqs


def pct(xs, q):
    xs = sorted(x for x in xs if x is not None)
    if not xs:
        return None
    return round(xs[min(len(xs) - 1, int(q * len(xs)))], 3)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    import torch

    from inference_systems_b200 import SamplingParams
    from inference_systems_b200.engine.llm_engine import LLMEngine, serve_worker
    from inference_systems_b200.models.presets import preset

    cfg = preset(args.model)
    kw = dict(load_format="dummy", device="cuda", tensor_parallel_size=world, max_num_seqs=args.max_num_seqs,
              max_num_state_slots=args.max_num_seqs, max_model_len=args.prompt_max + args.output_max + 64,
              max_num_batched_tokens=args.chunk, enable_chunked_prefill=True, scheduling_policy="decode_first",
              kvcache_block_size=256, prefix_match_unit=16, enable_prefix_cache=not args.no_prefix_cache,
              enable_hybrid_prefix_cache=not args.no_prefix_cache,
              hybrid_prefix_checkpoint_memory_bytes=args.checkpoint_gib << 30, gpu_memory_utilization=0.85,
              dist_port=int(os.environ.get("MASTER_PORT", "29500")) + 23)
    if world > 1 and rank > 0:
        serve_worker(cfg, **kw)
        return
    llm = LLMEngine(cfg, **kw)
    reqs = workload(args, cfg["vocab_size"])
    # warm-up: a few short requests through every path (prefill chunks, decode graphs)
    for p in [r[1][:512] for r in reqs[:4]]:
        llm.add_request(p, SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True))
    while not llm.is_finished():
        llm.step()
    llm.reset_runtime_metrics()

    t0 = time.perf_counter()
    t0_ns = time.perf_counter_ns()
    i, out_tokens = 0, 0
    while i < len(reqs) or not llm.is_finished():
        now = time.perf_counter() - t0
        while i < len(reqs) and reqs[i][0] <= now:
            arr, prompt, n_out, _ = reqs[i]
            llm.add_request(prompt, SamplingParams(temperature=0.0, max_tokens=n_out, ignore_eos=True),
                            arrival_time_ns=t0_ns + int(arr * 1e9))
            i += 1
        if llm.is_finished():
            time.sleep(min(0.002, max(0.0, reqs[i][0] - now)))
            continue
        _, stats = llm.step()
        out_tokens += stats.decode_tokens
    torch.cuda.synchronize()
    makespan = time.perf_counter() - t0
    req = llm.get_request_metrics()[-len(reqs):]
    sched = llm.get_runtime_metrics()["scheduler"]
    ttft = [m.get("ttft_ms") for m in req]
    tpot = [m.get("tpot_ms") for m in req]
    e2e = [m.get("e2e_ms") for m in req]
    total_out = sum(len_out for _, _, len_out, _ in reqs)
    res = {
        "metric": "online serving: p50/p99 TTFT and TPOT, request throughput (Poisson arrivals)",
        "value": round(len(req) / makespan, 3), "unit": "requests/s", "n_gpus": world, "higher_is_better": True,
        "dtype": "bf16", "data": "synthetic prompts (lognormal lengths, 30% share a hot prefix); random-init weights",
        "config": {"model": args.model, "parallelism": f"tp{world}", "rate_rps": args.rate, "requests": len(reqs),
                   "prompt_median": args.prompt_median, "prompt_max": args.prompt_max,
                   "output_median": args.output_median, "prefix_share": args.prefix_share,
                   "prefix_len": args.prefix_len, "chunked_prefill_tokens": args.chunk,
                   "prefix_cache": not args.no_prefix_cache},
        "ttft_ms": {"p50": pct(ttft, 0.5), "p99": pct(ttft, 0.99)},
        "tpot_ms": {"p50": pct(tpot, 0.5), "p99": pct(tpot, 0.99)},
        "e2e_ms": {"p50": pct(e2e, 0.5), "p99": pct(e2e, 0.99)},
        "output_tokens_per_s": round(total_out / makespan, 1),
        "makespan_s": round(makespan, 3),
        "prefix_cache": {k: v for k, v in sched.items() if "prefix" in k and isinstance(v, (int, float))},
        "impl": "isb",
    }
    llm.exit()
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
