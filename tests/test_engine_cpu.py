"""CPU engine end to end against the stand-alone fp32 oracle (the tiny 4-layer shape and variants)."""

import os

import pytest
import torch
from safetensors.torch import save_file

from inference_systems_b200 import SamplingParams
from inference_systems_b200.llm import LLM
from inference_systems_b200.models.presets import preset, random_state_dict, write_config, write_random_checkpoint
from inference_systems_b200.models.reference_model import reference_greedy


def _ckpt(tmp_path, name="tiny", std=0.02, **over):
    cfg = preset(name, **over)
    sd = random_state_dict(cfg, seed=0, std=std)
    d = str(tmp_path)
    write_config(d, cfg)
    save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(d, "model.safetensors"))
    return d, cfg, sd


def _prompts(n, length, vocab, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (length,), generator=g).tolist() for _ in range(n)]


def test_baseline_config1_tiny_hybrid_matches_recurrence(tmp_path):
    """4 layers [GDN, GDN, GDN, attn], N(0, 0.02) seed 0, 2 x 32 prompts, 16 greedy steps."""
    d, cfg, sd = _ckpt(tmp_path)
    llm = LLM(d, device="cpu", max_num_seqs=2, max_num_state_slots=2, max_model_len=256)
    prompts = _prompts(2, 32, cfg["vocab_size"])
    out = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True), use_tqdm=False)
    llm.exit()
    for o, p in zip(out, prompts):
        assert o["token_ids"] == reference_greedy(sd, cfg, p, 16)


@pytest.mark.parametrize("chunk", [7, 40])
def test_chunked_prefill_and_batching_match_oracle(tmp_path, chunk):
    d, cfg, sd = _ckpt(tmp_path, std=0.25)
    llm = LLM(d, device="cpu", max_num_seqs=3, max_num_state_slots=3, max_model_len=256,
              max_num_batched_tokens=chunk, scheduling_policy="decode_first")
    prompts = _prompts(3, 30, cfg["vocab_size"], seed=chunk)
    out = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True), use_tqdm=False)
    metrics = llm.get_runtime_metrics()
    llm.exit()
    for o, p in zip(out, prompts):
        assert o["token_ids"] == reference_greedy(sd, cfg, p, 6)
    if chunk < 30:
        assert metrics["scheduler"]["chunked_prefill_steps"] > 0


def test_preemption_recompute_keeps_outputs(tmp_path):
    d, cfg, sd = _ckpt(tmp_path, std=0.25)
    # 2 KV pages for 3 sequences of ~260 tokens forces preemption and recompute
    llm = LLM(d, device="cpu", max_num_seqs=3, max_num_state_slots=3, max_model_len=512, num_kvcache_blocks=4,
              scheduling_policy="decode_first")
    prompts = _prompts(3, 250, cfg["vocab_size"], seed=3)
    out = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True), use_tqdm=False)
    pre = llm.get_runtime_metrics()["scheduler"]["preemption_count"]
    llm.exit()
    assert pre > 0
    for o, p in zip(out, prompts):
        assert o["token_ids"] == reference_greedy(sd, cfg, p, 10)


def test_abort_frees_resources(tmp_path):
    d, cfg, _ = _ckpt(tmp_path)
    llm = LLM(d, device="cpu", max_num_seqs=2, max_num_state_slots=2, max_model_len=256)
    rid = llm.add_request(_prompts(1, 20, cfg["vocab_size"])[0], SamplingParams(max_tokens=50, temperature=0.0))
    llm.step()
    assert llm.abort_request(rid)
    assert llm.is_finished()
    m = llm.get_runtime_metrics()
    assert m["scheduler"]["aborted_request_count"] == 1
    assert m["model_runner"]["state_slots_used"] == 0
    assert llm.get_request_metrics()[0]["status"] == "aborted"
    llm.exit()


def test_sampling_is_seeded_and_temperature_changes_tokens(tmp_path):
    d, cfg, _ = _ckpt(tmp_path, std=0.25)
    prompts = _prompts(2, 12, cfg["vocab_size"], seed=11)
    outs = []
    for _ in range(2):
        llm = LLM(d, device="cpu", max_num_seqs=2, max_num_state_slots=2, max_model_len=256, seed=5)
        outs.append([o["token_ids"] for o in llm.generate(prompts, SamplingParams(temperature=1.0, max_tokens=8),
                                                          use_tqdm=False)])
        llm.exit()
    assert outs[0] == outs[1]


def test_dense_qwen3_family(tmp_path):
    d, cfg, sd = _ckpt(tmp_path, name="qwen3-tiny", std=0.25)
    llm = LLM(d, device="cpu", max_num_seqs=2, max_model_len=256)
    prompts = _prompts(2, 20, cfg["vocab_size"], seed=2)
    out = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True), use_tqdm=False)
    llm.exit()
    for o, p in zip(out, prompts):
        assert o["token_ids"] == reference_greedy(sd, cfg, p, 5)


def test_dense_prefix_cache_hit(tmp_path):
    d, cfg, _ = _ckpt(tmp_path, name="qwen3-tiny", std=0.25)
    llm = LLM(d, device="cpu", max_num_seqs=2, max_model_len=1024)
    shared = _prompts(1, 300, cfg["vocab_size"], seed=4)[0]
    sp = SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True)
    a = llm.generate([shared + [1, 2]], sp, use_tqdm=False)
    b = llm.generate([shared + [1, 2]], sp, use_tqdm=False)
    m = llm.get_runtime_metrics()["scheduler"]
    llm.exit()
    assert a[0]["token_ids"] == b[0]["token_ids"]
    assert m["prefix_cache_hit_blocks"] >= 1


def test_eos_stops_generation(tmp_path):
    d, cfg, sd = _ckpt(tmp_path, std=0.25)
    prompt = _prompts(1, 10, cfg["vocab_size"], seed=9)[0]
    first = reference_greedy(sd, cfg, prompt, 1)[0]
    llm = LLM(d, device="cpu", max_num_seqs=1, max_num_state_slots=1, max_model_len=256, eos=first)
    out = llm.generate([prompt], SamplingParams(temperature=0.0, max_tokens=8), use_tqdm=False)
    llm.exit()
    assert out[0]["token_ids"] == [first]


def test_dummy_load_format_runs(tmp_path):
    llm = LLM(preset("tiny"), load_format="dummy", device="cpu", max_num_seqs=1, max_num_state_slots=1,
              max_model_len=128)
    out = llm.generate([[1, 2, 3]], SamplingParams(temperature=0.0, max_tokens=2, ignore_eos=True), use_tqdm=False)
    llm.exit()
    assert len(out[0]["token_ids"]) == 2


def test_random_checkpoint_writer_roundtrip(tmp_path):
    d = write_random_checkpoint(str(tmp_path), "tiny")
    assert os.path.exists(os.path.join(d, "config.json"))
    llm = LLM(d, device="cpu", max_num_seqs=1, max_num_state_slots=1, max_model_len=128)
    assert llm.model_runner.load_report.ok
    llm.exit()
