"""Hybrid (KV + GDN state) prefix cache end to end on the CPU engine.

A second request that shares a long prefix with the first must restore the
GDN recurrent/conv checkpoint captured by the first one and produce exactly the
tokens a cache-less engine produces.  Covered: periodic boundaries reached by
splitting prefill chunks, internal checkpoints recorded inside one prefill
chunk, and int8-compressed checkpoints.
"""

import os

import pytest
import torch
from safetensors.torch import save_file

from inference_systems_b200 import SamplingParams
from inference_systems_b200.llm import LLM
from inference_systems_b200.models.presets import preset, random_state_dict, write_config


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    cfg = preset("tiny")
    sd = random_state_dict(cfg, seed=0, std=0.25)
    d = str(tmp_path_factory.mktemp("tiny_hpc"))
    write_config(d, cfg)
    save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(d, "model.safetensors"))
    return d, cfg


def _prompts(vocab):
    g = torch.Generator().manual_seed(11)
    shared = torch.randint(0, vocab, (600,), generator=g).tolist()
    a = shared + torch.randint(0, vocab, (40,), generator=g).tolist()
    b = shared + torch.randint(0, vocab, (33,), generator=g).tolist()
    return a, b


def _run(d, prompts, **kw):
    llm = LLM(d, device="cpu", max_model_len=1024, **kw)
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    outs = [llm.generate([p], sp, use_tqdm=False)[0]["token_ids"] for p in prompts]  # one after the other
    m = llm.get_runtime_metrics()["scheduler"]
    llm.exit()
    return outs, m


@pytest.mark.parametrize("mode", ["periodic", "internal", "int8"])
def test_shared_prefix_restores_gdn_checkpoint(ckpt, mode):
    d, cfg = ckpt
    a, b = _prompts(cfg["vocab_size"])
    want, _ = _run(d, [a, b], max_num_seqs=1, max_num_state_slots=1, enable_prefix_cache=False)
    kw = dict(max_num_seqs=1, max_num_state_slots=1, enable_prefix_cache=True, enable_hybrid_prefix_cache=True,
              prefix_match_unit=16, hybrid_prefix_checkpoint_interval_tokens=256,
              hybrid_prefix_checkpoint_memory_bytes=64 << 20)
    if mode == "internal":
        kw.update(enable_hybrid_internal_checkpoints=True, max_num_batched_tokens=4096)
    if mode == "int8":
        kw.update(hybrid_prefix_checkpoint_dtype="int8")
    got, m = _run(d, [a, b], **kw)
    assert got[0] == want[0]
    if mode == "int8":  # lossy checkpoint: the continuation may drift, but the prefix is reused
        assert got[1][:2] == want[1][:2]
    else:
        assert got[1] == want[1]
    assert m["hybrid_prefix_restore_count"] >= 1
    assert m["hybrid_prefix_committed_hit_tokens"] >= 512
