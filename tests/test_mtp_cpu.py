"""Native MTP speculative decoding on the CPU path.

Greedy speculative decoding must be lossless: whatever the drafts are, the
emitted tokens equal target-only greedy decoding.  Random MTP weights almost
never agree with the target, so one test injects oracle drafts (the true
continuation with one wrong token at a rotating position) to drive every
accepted length through verify, rollback and commit.
"""

import os

import pytest
import torch
from safetensors.torch import save_file

from inference_systems_b200 import SamplingParams
from inference_systems_b200.llm import LLM
from inference_systems_b200.models.presets import preset, random_state_dict, write_config


def _ckpt(tmp_path, std=0.25):
    cfg = preset("tiny")
    sd = random_state_dict(cfg, seed=0, std=std)
    d = str(tmp_path)
    write_config(d, cfg)
    save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(d, "model.safetensors"))
    return d, cfg


def _prompts(n, length, vocab, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (length,), generator=g).tolist() for _ in range(n)]


def _generate(d, prompts, max_tokens, hook=None, **kw):
    llm = LLM(d, device="cpu", max_num_seqs=len(prompts), max_num_state_slots=len(prompts), max_model_len=256, **kw)
    if hook is not None:
        llm.model_runner.mtp_driver.before_round = hook
    out = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=max_tokens, ignore_eos=True),
                       use_tqdm=False)
    m = llm.get_runtime_metrics()
    llm.exit()
    return [o["token_ids"] for o in out], m


def test_mtp_with_model_drafts_is_lossless(tmp_path):
    d, cfg = _ckpt(tmp_path)
    prompts = _prompts(2, 20, cfg["vocab_size"], seed=1)
    want, _ = _generate(d, prompts, 10)
    got, m = _generate(d, prompts, 10, num_speculative_tokens=2)
    assert got == want
    mtp = m["model_runner"]["mtp"]
    assert mtp["rounds"] > 0 and mtp["prefill_catchups"] > 0


@pytest.mark.parametrize("k,replay", [(1, None), (3, None), (3, False)])
def test_mtp_oracle_drafts_cover_every_accept_length(tmp_path, k, replay):
    """Every accepted length 0..K occurs; with ``enable_mtp_replay_ssm=False`` the commit copies the
    state snapshot of the accepted row instead of folding replay records, with the same tokens."""
    d, cfg = _ckpt(tmp_path)
    prompts = _prompts(3, 17, cfg["vocab_size"], seed=2)
    n = 14
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

    got, m = _generate(d, prompts, n, hook=hook, num_speculative_tokens=k, max_num_batched_tokens=64,
                       enable_mtp_replay_ssm=replay)
    assert got == [w[:n] for w in want]
    hist = m["model_runner"]["mtp"]["accepted_length_histogram"]
    assert all(c > 0 for c in hist), hist
    assert m["model_runner"]["mtp"]["verify_records"] == ("snapshot" if replay is False else "replay")


def test_mtp_synthetic_full_acceptance_emits_k_plus_one(tmp_path):
    d, cfg = _ckpt(tmp_path)
    prompts = _prompts(2, 12, cfg["vocab_size"], seed=3)
    k = 2
    got, m = _generate(d, prompts, 9, num_speculative_tokens=k, mtp_synthetic_acceptance=1.0)
    assert [len(g) for g in got] == [9, 9]
    mtp = m["model_runner"]["mtp"]
    assert mtp["acceptance_rate"] == 1.0
    assert mtp["accepted_length_histogram"][k] == mtp["sequence_rounds"]
    assert mtp["mean_emitted_per_round"] == pytest.approx(k + 1)
