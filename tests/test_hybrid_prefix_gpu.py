"""Hybrid prefix cache on the sm_100a path: checkpoint capture (including internal
checkpoints recorded by the scan kernel's history mode) and restore.

Run back to back, these also catch a kernel that reads a reallocated state slot
before the slot's zeroing is visible (the cache-less reference run would then
depend on timing)."""

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
    # std 0.25: logit margins large enough that bf16 rounding differences between chunkings
    # (cached prefix + short prefill vs one long prefill) do not flip greedy tokens
    sd = random_state_dict(cfg, seed=0, std=0.25)
    d = str(tmp_path_factory.mktemp("tiny_hd_hpc"))
    write_config(d, cfg)
    save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(d, "model.safetensors"))
    return d, cfg


def _run(d, prompts, **kw):
    from inference_systems_b200.llm import LLM

    llm = LLM(d, device="cuda", max_model_len=2048, num_kvcache_blocks=32, **kw)
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    outs = [llm.generate([p], sp, use_tqdm=False)[0]["token_ids"] for p in prompts]
    m = llm.get_runtime_metrics()["scheduler"]
    llm.exit()
    return outs, m


@pytest.mark.parametrize("internal", [False, True])
def test_shared_prefix_restores_on_gpu(ckpt, internal):
    d, cfg = ckpt
    g = torch.Generator().manual_seed(3)
    shared = torch.randint(0, cfg["vocab_size"], (700,), generator=g).tolist()
    a = shared + torch.randint(0, cfg["vocab_size"], (30,), generator=g).tolist()
    b = shared + torch.randint(0, cfg["vocab_size"], (21,), generator=g).tolist()
    want, _ = _run(d, [a, b], max_num_seqs=1, max_num_state_slots=1, enable_prefix_cache=False)
    kw = dict(max_num_seqs=1, max_num_state_slots=1, enable_prefix_cache=True, enable_hybrid_prefix_cache=True,
              prefix_match_unit=16, hybrid_prefix_checkpoint_interval_tokens=256,
              hybrid_prefix_checkpoint_memory_bytes=256 << 20)
    if internal:
        kw.update(enable_hybrid_internal_checkpoints=True, max_num_batched_tokens=4096)
    got, m = _run(d, [a, b], **kw)
    assert got[0] == want[0]
    assert got[1][:4] == want[1][:4]
    assert m["hybrid_prefix_restore_count"] >= 1
    assert torch.ops.isb.error_word() == 0
