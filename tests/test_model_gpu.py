"""GPU model / engine integration: the sm_100a path against the fp32 CPU oracle."""

import os

import pytest
import torch
from safetensors.torch import save_file

from inference_systems_b200 import SamplingParams
from inference_systems_b200.models.presets import preset, random_state_dict, write_config
from inference_systems_b200.models.reference_model import reference_logits

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    cfg = preset("tiny_hd")
    sd = random_state_dict(cfg, seed=0, std=0.05)
    d = str(tmp_path_factory.mktemp("tiny_hd"))
    write_config(d, cfg)
    save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(d, "model.safetensors"))
    return d, cfg, sd


def _prompts(n, length, vocab, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (length,), generator=g).tolist() for _ in range(n)]


def test_prefill_logits_match_oracle(ckpt):
    from inference_systems_b200.config import Config
    from inference_systems_b200.engine.model_runner import ModelRunner
    from inference_systems_b200.engine.sequence import Sequence

    d, cfg, sd = ckpt
    config = Config(d, device="cuda", max_num_seqs=4, max_num_state_slots=4, max_model_len=1024, enforce_eager=True,
                    num_kvcache_blocks=32)
    runner = ModelRunner(config, 0)
    prompts = _prompts(2, 300, cfg["vocab_size"])
    seqs = [Sequence(p) for p in prompts]
    Sequence.block_size = 256
    for s, bt in zip(seqs, ([0, 1], [2, 3])):
        s.block_table = bt
        s.num_scheduled_tokens = len(s)
        runner.allocate_state_slot(s)
    runner.run(seqs, True)
    hidden = runner._last_hidden
    logits = runner.model.compute_logits(hidden).float().cpu()
    cu = [0, 300, 600]
    sdf = {k: v.float() for k, v in sd.items()}
    for i, p in enumerate(prompts):
        exp = reference_logits(sdf, cfg, p)
        got = logits[cu[i]:cu[i + 1]]
        cos = torch.nn.functional.cosine_similarity(got, exp, dim=-1)
        assert cos.min() > 0.99, cos.min()
    runner.exit()


@pytest.mark.parametrize("eager", [True, False])
def test_generate_matches_cpu_engine(ckpt, eager):
    from inference_systems_b200.llm import LLM

    d, cfg, _ = ckpt
    prompts = _prompts(3, 70, cfg["vocab_size"], seed=1)
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)
    gpu = LLM(d, device="cuda", max_num_seqs=4, max_num_state_slots=4, max_model_len=1024, enforce_eager=eager,
              num_kvcache_blocks=32, max_num_batched_tokens=100)
    out_g = [o["token_ids"] for o in gpu.generate(prompts, sp, use_tqdm=False)]
    metrics = gpu.get_runtime_metrics()
    gpu.exit()
    cpu = LLM(d, device="cpu", dtype="float32", max_num_seqs=4, max_num_state_slots=4, max_model_len=1024,
              num_kvcache_blocks=32, max_num_batched_tokens=100)
    out_c = [o["token_ids"] for o in cpu.generate(prompts, sp, use_tqdm=False)]
    cpu.exit()
    agree = sum(a == b for og, oc in zip(out_g, out_c) for a, b in zip(og[:4], oc[:4]))
    assert agree >= 10, (out_g, out_c)
    if not eager:
        assert metrics["model_runner"]["cudagraph_replays"] > 0
