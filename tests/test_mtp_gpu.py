"""Native MTP speculative decoding on the sm_100a path.

The verify pass runs the prefill kernels over ``K+1`` rows per sequence while
target-only decoding runs the decode kernels, so bf16 rounding can break a
near-tie differently; agreement is therefore measured as matching prefixes.
"""

import os

import pytest
import torch
from safetensors.torch import save_file

from inference_systems_b200 import SamplingParams
from inference_systems_b200.models.presets import preset, random_state_dict, write_config

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    cfg = preset("tiny_hd")
    sd = random_state_dict(cfg, seed=0, std=0.05)
    d = str(tmp_path_factory.mktemp("tiny_hd_mtp"))
    write_config(d, cfg)
    save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(d, "model.safetensors"))
    return d, cfg


def _prompts(n, length, vocab, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (length,), generator=g).tolist() for _ in range(n)]


def _generate(d, prompts, n, hook=None, eager=True, **kw):
    from inference_systems_b200.llm import LLM

    llm = LLM(d, device="cuda", max_num_seqs=4, max_num_state_slots=4, max_model_len=1024, num_kvcache_blocks=32,
              max_num_batched_tokens=128, enforce_eager=eager, **kw)
    if hook is not None:
        llm.model_runner.mtp_driver.before_round = hook
    out = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=n,
                                                                        ignore_eos=True), use_tqdm=False)]
    m = llm.get_runtime_metrics()
    llm.exit()
    return out, m


def _prefix(a, b):
    n = 0
    for x, y in zip(a, b):
        if x != y:
            break
        n += 1
    return n


@pytest.mark.parametrize("k,eager,replay", [(1, True, None), (3, True, None), (2, False, None), (2, False, False)])
def test_mtp_oracle_drafts_match_target_only(ckpt, k, eager, replay):
    d, cfg = ckpt
    prompts = _prompts(3, 40, cfg["vocab_size"], seed=5)
    n = 12
    want, _ = _generate(d, prompts, n + 2 * k + 2)
    by_prompt = {tuple(p): w for p, w in zip(prompts, want)}
    rounds = [0]

    def hook(seqs, driver):
        for s in seqs:
            truth = by_prompt[tuple(s.prompt_token_ids)]
            done = s.num_completion_tokens
            drafts = list(truth[done:done + k])
            wrong = (rounds[0] + s.seq_id) % (k + 1)
            if wrong < k:
                drafts[wrong] = (drafts[wrong] + 1) % cfg["vocab_size"]
            driver.set_drafts(s.state_slot, drafts)
        rounds[0] += 1

    got, m = _generate(d, prompts, n, hook=hook, eager=eager, num_speculative_tokens=k, enable_mtp_replay_ssm=replay)
    prefixes = [_prefix(g, w) for g, w in zip(got, want)]
    assert sum(p == n for p in prefixes) >= 2 and min(prefixes) >= 4, (got, want)
    mtp = m["model_runner"]["mtp"]
    assert mtp["rounds"] > 0 and mtp["accepted_tokens"] > 0
    if not eager:
        assert mtp["cudagraph_replays"] == mtp["rounds"]
    assert torch.ops.isb.error_word() == 0


@pytest.mark.parametrize("eager", [True, False])
def test_mtp_synthetic_acceptance_runs_k_plus_one(ckpt, eager):
    d, cfg = ckpt
    prompts = _prompts(2, 30, cfg["vocab_size"], seed=6)
    got, m = _generate(d, prompts, 10, eager=eager, num_speculative_tokens=2, mtp_synthetic_acceptance=1.0)
    assert [len(g) for g in got] == [10, 10]
    mtp = m["model_runner"]["mtp"]
    assert mtp["acceptance_rate"] == 1.0
    assert mtp["mean_emitted_per_round"] == pytest.approx(3.0)
