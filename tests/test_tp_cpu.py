"""Tensor parallelism on CPU ranks (gloo): TP=2 engine output == TP=1 output == fp32 oracle.

Parity with the reference's distributed-without-a-cluster tests
(``tests/test_qwen35_tp.py``): real multi-process ranks over gloo on CPU tensors.
"""

import os
import socket

import pytest
import torch
from safetensors.torch import save_file

from inference_systems_b200 import SamplingParams
from inference_systems_b200.llm import LLM
from inference_systems_b200.models.presets import preset, random_state_dict, write_config
from inference_systems_b200.models.reference_model import reference_greedy


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("name,tp", [("tiny", 2), ("tiny", 4)])
def test_tensor_parallel_engine_matches_oracle(tmp_path, name, tp):
    cfg = preset(name, linear_num_value_heads=4 if tp <= 4 else 8)
    sd = random_state_dict(cfg, seed=1, std=0.25)
    d = str(tmp_path)
    write_config(d, cfg)
    save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(d, "model.safetensors"))
    g = torch.Generator().manual_seed(7)
    prompts = [torch.randint(0, cfg["vocab_size"], (24,), generator=g).tolist() for _ in range(2)]
    llm = LLM(d, device="cpu", tensor_parallel_size=tp, max_num_seqs=2, max_num_state_slots=2, max_model_len=128,
              dist_port=_free_port(), max_num_batched_tokens=30)
    out = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True), use_tqdm=False)
    llm.exit()
    for o, p in zip(out, prompts):
        assert o["token_ids"] == reference_greedy(sd, cfg, p, 5)
