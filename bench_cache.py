"""Hybrid prefix cache and scheduler studies (one GPU unless noted).

    python bench_cache.py checkpoints [--budget-mib 128]
    python bench_cache.py prefix [--prefix 496 --suffix 16]
    python bench_cache.py scheduler [--requests 24]

* ``checkpoints`` -- GDN checkpoint capture / restore time and pool capacity per storage format
  (fp32, bf16, int8 with per-row scales) for one request's state of the 0.8B shape (18 GDN layers,
  16 value heads, 128 x 128 fp32 state each).  The reference's study:
  ``benchmark_checkpoint_compression.py`` (published on an RTX 3060 Laptop:
  ``docs/checkpoint-compression.md:82-86``).
* ``prefix`` -- time to first token of a request whose first ``--prefix`` tokens were already
  served to an earlier request, with no prefix cache, with the page-level (256-token) hybrid cache
  and with the fine 16-token match unit (partial-page copy-on-write).  The reference's study:
  ``benchmark_fine_grained_prefix_cache.py`` (``docs/fine-grained-hybrid-prefix-cache-report.md``).
* ``scheduler`` -- a burst of requests where a third share a long prefix, under KV pressure:
  FCFS admission with LIFO preemption vs hybrid-state-aware admission with recompute-aware
  preemption; TTFT p50 / p99 and request throughput.  The reference's study:
  ``benchmark_hybrid_state_scheduler.py`` (``docs/serving-benchmark.md``).

Every result is printed as one JSON line.  Random-init weights of the 0.8B shape, synthetic tokens.
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


def _p(xs, q):
    xs = sorted(xs)
    return xs[min(int(q * len(xs)), len(xs) - 1)] if xs else None


def checkpoints(args) -> None:
    import torch

    from inference_systems_b200.engine.state_pool import HybridPrefixCheckpointPool, HybridStateManager

    for fmt in ("fp32", "bf16", "int8"):
        sm = HybridStateManager(max_num_seqs=1, num_linear_layers=18, num_value_heads=16, key_head_dim=128,
                                value_head_dim=128, conv_dim=6144, conv_kernel_size=4, conv_dtype=torch.bfloat16,
                                device="cuda")
        slot = sm.allocate()
        sm.recurrent_states[:, slot].normal_()
        sm.conv_states[:, slot].normal_()
        pool = HybridPrefixCheckpointPool(sm, args.budget_mib << 20, checkpoint_dtype=fmt)
        ref = sm.recurrent_states[:, slot].clone()
        cap, res = [], []
        for i in range(args.warmup + args.iters):
            e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            e[0].record()
            ck = pool.capture(slot)
            e[1].record()
            pool.restore(ck, slot)
            e[2].record()
            torch.cuda.synchronize()
            pool.free(ck)
            if i >= args.warmup:
                cap.append(e[0].elapsed_time(e[1]))
                res.append(e[1].elapsed_time(e[2]))
        err = float((sm.recurrent_states[:, slot] - ref).abs().max())
        print(json.dumps({"study": "checkpoint_formats", "format": fmt, "budget_mib": args.budget_mib,
                          "capacity": pool.capacity, "bytes_per_checkpoint": pool.bytes_per_checkpoint,
                          "capture_ms_p50": round(statistics.median(cap), 4),
                          "restore_ms_p50": round(statistics.median(res), 4),
                          "restore_max_abs_error": err}), flush=True)


DEVICE = "cuda"


def _engine(cfg, **kw):
    from inference_systems_b200.engine.llm_engine import LLMEngine

    base = dict(load_format="dummy", device=DEVICE, max_num_seqs=4, max_num_state_slots=4, max_model_len=4096,
                max_num_batched_tokens=4096, enforce_eager=DEVICE != "cuda", gpu_memory_utilization=0.5)
    base.update(kw)
    return LLMEngine(cfg, **base)


def _ttft(llm, prompt) -> float:
    from inference_systems_b200 import SamplingParams

    llm.add_request(prompt, SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True))
    t0 = time.perf_counter()
    while not llm.is_finished():
        llm.step()
    return (time.perf_counter() - t0) * 1e3


def prefix(args) -> None:
    import torch

    from inference_systems_b200.models.presets import preset

    cfg = preset(args.model)
    g = torch.Generator().manual_seed(0)
    shared = torch.randint(0, cfg["vocab_size"], (args.prefix,), generator=g).tolist()
    modes = {
        "no_cache": dict(enable_prefix_cache=False),
        "page_256": dict(enable_prefix_cache=True, enable_hybrid_prefix_cache=True, prefix_match_unit=256,
                         hybrid_prefix_checkpoint_interval_tokens=256, hybrid_prefix_retention_policy="adaptive",
                         hybrid_prefix_checkpoint_memory_bytes=1 << 30, max_num_seqs=1, max_num_state_slots=1,
                         enable_hybrid_internal_checkpoints=True),
        "fine_16": dict(enable_prefix_cache=True, enable_hybrid_prefix_cache=True, prefix_match_unit=16,
                        hybrid_prefix_checkpoint_interval_tokens=256, hybrid_prefix_retention_policy="adaptive",
                        hybrid_prefix_checkpoint_memory_bytes=1 << 30, max_num_seqs=1, max_num_state_slots=1,
                        enable_hybrid_internal_checkpoints=True),
    }
    for name, kw in modes.items():
        llm = _engine(cfg, **kw)
        warm = torch.randint(0, cfg["vocab_size"], (args.prefix + args.suffix,), generator=g).tolist()
        _ttft(llm, warm)  # compile / warm-up, unrelated tokens
        first = _ttft(llm, shared + torch.randint(0, cfg["vocab_size"], (args.suffix,), generator=g).tolist())
        second = [_ttft(llm, shared + torch.randint(0, cfg["vocab_size"], (args.suffix,), generator=g).tolist())
                  for _ in range(args.iters)]
        m = llm.get_runtime_metrics()["scheduler"]
        print(json.dumps({"study": "prefix_cache_ttft", "mode": name, "shared_prefix_tokens": args.prefix,
                          "suffix_tokens": args.suffix, "first_ttft_ms": round(first, 2),
                          "repeat_ttft_ms_p50": round(statistics.median(second), 2),
                          "restored_tokens": m.get("hybrid_prefix_committed_hit_tokens", 0),
                          "cow_allocations": m.get("partial_prefix_cow_allocations", 0)}), flush=True)
        llm.exit()


def scheduler(args) -> None:
    import torch

    from inference_systems_b200 import SamplingParams
    from inference_systems_b200.models.presets import preset

    cfg = preset(args.model)
    g = torch.Generator().manual_seed(1)
    hot = torch.randint(0, cfg["vocab_size"], (1024,), generator=g).tolist()
    prompts = []
    for i in range(args.requests):
        tail = torch.randint(0, cfg["vocab_size"], (256 + 64 * (i % 5),), generator=g).tolist()
        prompts.append(hot + tail if i % 3 == 0 else torch.randint(0, cfg["vocab_size"], (1024,), generator=g).tolist() + tail)
    policies = {"fcfs_lifo": dict(waiting_admission_policy="fcfs", preemption_policy="lifo"),
                "hybrid_state_aware": dict(waiting_admission_policy="hybrid_state_aware",
                                           preemption_policy="recompute_aware")}
    for name, kw in policies.items():
        llm = _engine(cfg, max_num_seqs=8, max_num_state_slots=8, num_kvcache_blocks=48, scheduling_policy="decode_first",
                      enable_prefix_cache=True, enable_hybrid_prefix_cache=True, prefix_match_unit=256,
                      hybrid_prefix_checkpoint_interval_tokens=256, hybrid_prefix_checkpoint_memory_bytes=2 << 30,
                      **kw)
        sp = SamplingParams(temperature=0.0, max_tokens=args.output, ignore_eos=True)
        t0 = time.perf_counter()
        for p in prompts:
            llm.add_request(p, sp)
        while not llm.is_finished():
            llm.step()
        wall = time.perf_counter() - t0
        req = llm.get_request_metrics()
        ttft = [r["ttft_ms"] for r in req if r.get("ttft_ms") is not None]
        m = llm.get_runtime_metrics()["scheduler"]
        print(json.dumps({"study": "hybrid_state_scheduler", "policy": name, "requests": len(prompts),
                          "ttft_p50_ms": round(_p(ttft, 0.5), 2), "ttft_p99_ms": round(_p(ttft, 0.99), 2),
                          "req_per_s": round(len(prompts) / wall, 3), "preemptions": m["preemption_count"],
                          "prefix_tokens_reused": m["prefix_tokens_reused_actual"]}), flush=True)
        llm.exit()


def main():
    p = argparse.ArgumentParser()
    p.add_argument("study", choices=["checkpoints", "prefix", "scheduler"])
    p.add_argument("--model", default="qwen3_5-0.8b")
    p.add_argument("--budget-mib", type=int, default=128)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--prefix", type=int, default=496)
    p.add_argument("--suffix", type=int, default=16)
    p.add_argument("--requests", type=int, default=24)
    p.add_argument("--output", type=int, default=32)
    p.add_argument("--device", default="cuda", help="cpu runs the same study on the PyTorch path (smoke test)")
    args = p.parse_args()
    global DEVICE
    DEVICE = args.device
    {"checkpoints": checkpoints, "prefix": prefix, "scheduler": scheduler}[args.study](args)


if __name__ == "__main__":
    main()
