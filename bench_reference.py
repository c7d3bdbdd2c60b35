"""Reference arm of ``bench.py``: the unmodified reference engine on the same workload.

The reference package is imported from ``baseline/_ref`` and driven only
through its public API (``nanovllm.LLM`` -> ``add_request`` / ``step``) with its
stock defaults, on a random-init checkpoint of the same Qwen3.5-0.8B shape
written to a temporary directory in Hugging Face layout (config.json,
model.safetensors, and a word-level tokenizer, because the reference engine
always loads a tokenizer).
"""

from __future__ import annotations

import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(ROOT, "baseline", "_ref")


def _unavailable(why: str) -> dict:
    return {"impl": "reference", "unavailable": why}


def _write_checkpoint(path: str, cfg: dict) -> None:
    from inference_systems_b200.models.presets import write_random_checkpoint

    if os.path.exists(os.path.join(path, "model.safetensors")):
        return
    os.makedirs(path, exist_ok=True)
    write_random_checkpoint(path, cfg, seed=0, include_mtp=True)
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    vocab = {f"t{i}": i for i in range(cfg["vocab_size"])}
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="t0"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    fast = PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="t0",
                                   eos_token=f"t{cfg['eos_token_id']}")
    fast.save_pretrained(path)


def run(args, rank: int, world: int, metric: str) -> dict | None:
    if not os.path.isdir(os.path.join(REF, "nanovllm")):
        return _unavailable("baseline/_ref/nanovllm is not installed")
    if world > 1 and rank > 0:
        return None  # the reference spawns its own tensor-parallel workers from rank 0
    from inference_systems_b200.models.presets import preset

    cfg = preset(args.model)
    if cfg["num_key_value_heads"] % world:
        return _unavailable(f"reference rejects TP={world}: Qwen3_5Attention requires num_key_value_heads "
                            f"({cfg['num_key_value_heads']}) divisible by TP (nanovllm/models/qwen3_5.py:33-34)")
    sys.path.insert(0, REF)
    try:
        import torch
        from nanovllm import LLM, SamplingParams
    except Exception as exc:  # noqa: BLE001
        return _unavailable(f"import failed: {type(exc).__name__}: {exc}")
    path = os.path.join("/tmp", f"isb_ref_ckpt_{args.model}")
    _write_checkpoint(path, cfg)
    b = args.batch
    total = args.steps + args.warmup
    try:
        llm = LLM(path, tensor_parallel_size=world, max_num_seqs=b, max_num_state_slots=b,
                  max_model_len=args.prompt_len + args.output_len + total + 32, enforce_eager=False)
    except Exception as exc:  # noqa: BLE001
        return _unavailable(f"engine construction failed: {type(exc).__name__}: {str(exc)[:300]}")
    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, cfg["vocab_size"], (b, args.prompt_len), generator=g).tolist()
    sp = SamplingParams(temperature=0.0, max_tokens=args.output_len + total + 8, ignore_eos=True)
    try:
        for p in prompts:
            llm.add_request(p, sp)
        t0 = time.perf_counter()
        sched = llm.scheduler
        while sched.waiting or any(s.num_completion_tokens == 0 for s in sched.running):
            llm.step()
        torch.cuda.synchronize()
        prefill_s = time.perf_counter() - t0
        for _ in range(args.warmup):
            llm.step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        decoded = 0
        for _ in range(args.steps):
            _, stats = llm.step()
            decoded += stats.decode_tokens
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        req = [s.lifecycle_metrics() for s in sched.running]
    except Exception as exc:  # noqa: BLE001
        llm.exit()
        return _unavailable(f"run failed: {type(exc).__name__}: {str(exc)[:300]}")
    ttfts = sorted(m["ttft_ms"] for m in req if m["ttft_ms"] is not None)
    tpots = sorted(m["tpot_ms"] for m in req if m["tpot_ms"] is not None)
    value = decoded / (ms / 1e3)
    llm.exit()
    return {
        "metric": metric, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform-random token ids; random-init N(0,0.02) weights of the 0.8B architecture)",
        "config": {"model": "Qwen3.5-0.8B-shape hybrid", "global_batch": b, "seq_len": args.prompt_len,
                   "parallelism": f"tp{world}", "l2": "inputs larger than L2"},
        "e2e": {"value": round(value, 1), "unit": "tokens/s", "note": "reference public API LLM.step()"},
        "ttft_p50_ms": round(ttfts[len(ttfts) // 2], 2) if ttfts else None,
        "tpot_p50_ms": round(tpots[len(tpots) // 2], 3) if tpots else None,
        "prefill_s": round(prefill_s, 3),
        "impl": "reference",
    }
