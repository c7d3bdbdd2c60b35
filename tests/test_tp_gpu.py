"""Tensor parallelism on GPUs: fused GEMM -> peer-memory all-reduce -> RMSNorm and the cross-rank LM-head argmax."""

import os
import socket

import pytest
import torch
from safetensors.torch import save_file

from inference_systems_b200 import SamplingParams
from inference_systems_b200.models.presets import preset, random_state_dict, write_config

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cfg = preset("tiny_hd")
    sd = random_state_dict(cfg, seed=0, std=0.05)
    d = str(tmp_path_factory.mktemp("tp"))
    write_config(d, cfg)
    save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(d, "model.safetensors"))
    return d, cfg


@pytest.mark.parametrize("eager", [True, False])
def test_tp2_matches_tp1(ckpt, eager):
    from inference_systems_b200.llm import LLM

    d, cfg = ckpt
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg["vocab_size"], (60,), generator=g).tolist() for _ in range(3)]
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    outs = []
    for tp in (1, 2):
        llm = LLM(d, device="cuda", tensor_parallel_size=tp, max_num_seqs=4, max_num_state_slots=4,
                  max_model_len=512, num_kvcache_blocks=16, enforce_eager=eager, dist_port=_free_port())
        outs.append([o["token_ids"] for o in llm.generate(prompts, sp, use_tqdm=False)])
        llm.exit()
    agree = sum(a == b for x, y in zip(*outs) for a, b in zip(x[:4], y[:4]))
    assert agree >= 10, outs


def test_tp2_token_sharded_prefill(ckpt, monkeypatch):
    """Prefill chunks above the fused-row limit run token-sharded: reduce-scatter + residual +
    RMSNorm on each rank's rows (``sp_rs_norm``) and the all-gather fused into every
    column-parallel GEMM's operand loads (``gemm_ag``).  Tokens must agree with TP=1 and with
    the replicated TP=2 path."""
    from inference_systems_b200.llm import LLM

    d, cfg = ckpt
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg["vocab_size"], (n,), generator=g).tolist() for n in (300, 257, 333)]
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    outs = []
    for tp, sharded in ((1, "0"), (2, "0"), (2, "1")):
        monkeypatch.setenv("ISB_TP_SP", sharded)
        llm = LLM(d, device="cuda", tensor_parallel_size=tp, max_num_seqs=4, max_num_state_slots=4,
                  max_model_len=512, num_kvcache_blocks=16, enforce_eager=True, dist_port=_free_port())
        outs.append([o["token_ids"] for o in llm.generate(prompts, sp, use_tqdm=False)])
        llm.exit()
        assert torch.ops.isb.error_word() == 0
    agree_tp1 = sum(a == b for x, y in zip(outs[0], outs[2]) for a, b in zip(x[:4], y[:4]))
    agree_rep = sum(a == b for x, y in zip(outs[1], outs[2]) for a, b in zip(x[:4], y[:4]))
    assert agree_tp1 >= 10 and agree_rep >= 10, outs
