"""A device wait that runs out surfaces as an engine-level error.

Every decode and prefill step appends the state of every kernel module's error word to the
sampled tokens it copies to the host; a nonzero word makes ``LLMEngine.step`` raise
``DeviceErrorStatus``.  The test shortens the cross-rank wait deadline to 5 ms, runs the
tensor-parallel owner kernel on an arrival counter that never advances (one GPU, buffers laid
out locally: nothing ever signals it), and checks that the engine's next step raises and names
the communication module.  The kernel returns after its deadline, so the GPU stays usable: the
test then clears the word and generates again.
"""

import os

import pytest
import torch
from safetensors.torch import save_file

from inference_systems_b200 import SamplingParams
from inference_systems_b200.models.presets import preset, random_state_dict, write_config

pytestmark = pytest.mark.gpu


def test_step_raises_after_a_device_wait_runs_out(tmp_path):
    from inference_systems_b200 import ops
    from inference_systems_b200.engine.model_runner import DeviceErrorStatus
    from inference_systems_b200.llm import LLM

    cfg = preset("tiny_hd")
    sd = random_state_dict(cfg, seed=0, std=0.05)
    d = str(tmp_path)
    write_config(d, cfg)
    save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(d, "model.safetensors"))
    llm = LLM(d, device="cuda", max_num_seqs=2, max_num_state_slots=2, max_model_len=512, num_kvcache_blocks=8,
              enforce_eager=False, max_cudagraph_batch_size=2)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg["vocab_size"], (30,), generator=g).tolist()
    sp = SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True)
    assert len(llm.generate([prompt], sp, use_tqdm=False)[0]["token_ids"]) == 4

    c = ops.cuda_ops()
    h = cfg["hidden_size"]
    slots = torch.zeros(2, 8, h, device="cuda", dtype=torch.bfloat16)
    res = torch.zeros(16, h, device="cuda", dtype=torch.bfloat16)
    x = torch.zeros(16, h, device="cuda", dtype=torch.bfloat16)
    ctl = torch.zeros(8, dtype=torch.int32, device="cuda")          # arrival counter stays at 0
    xs = torch.tensor([x.data_ptr()] * 2, dtype=torch.int64, device="cuda")
    ags = torch.tensor([ctl.data_ptr() + 4] * 2, dtype=torch.int64, device="cuda")
    c.comm_set_wait_timeout(5_000_000)
    try:
        c.tp_norm_allgather(slots, res, torch.zeros(h, device="cuda", dtype=torch.bfloat16), xs, ags, ctl, 16, 8, 0,
                            1, 1e-6, True, True)
        llm.add_request(prompt, sp)
        with pytest.raises(DeviceErrorStatus, match="tp-communication"):
            while not llm.is_finished():
                llm.step()
    finally:
        c.comm_set_wait_timeout(2_000_000_000)
    assert llm.model_runner.get_metrics()["device_errors"] == 1
    assert torch.ops.isb.error_word() == 0   # the engine read and cleared it
    # the GPU and the engine keep working once the word is clear
    for s in list(llm.scheduler.running) + list(llm.scheduler.waiting):
        llm.scheduler.abort(s.seq_id)
    assert len(llm.generate([prompt], sp, use_tqdm=False)[0]["token_ids"]) == 4
    llm.exit()
