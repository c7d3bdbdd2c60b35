"""AsyncLLMEngine and the OpenAI-compatible server on the CPU engine."""

import asyncio
import json
import os

import pytest
import torch
from safetensors.torch import save_file

from inference_systems_b200 import AsyncLLMEngine, SamplingParams
from inference_systems_b200.llm import LLM
from inference_systems_b200.models.presets import preset, random_state_dict, write_config


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    cfg = preset("tiny")
    sd = random_state_dict(cfg, seed=0, std=0.25)
    d = str(tmp_path_factory.mktemp("tiny_async"))
    write_config(d, cfg)
    save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(d, "model.safetensors"))
    return d, cfg


KW = dict(device="cpu", max_num_seqs=4, max_num_state_slots=4, max_model_len=256)


def _prompts(n, length, vocab, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (length,), generator=g).tolist() for _ in range(n)]


def test_async_streams_match_sync_generate(ckpt):
    d, cfg = ckpt
    prompts = _prompts(3, 15, cfg["vocab_size"], seed=1)
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    llm = LLM(d, **KW)
    want = [o["token_ids"] for o in llm.generate(prompts, sp, use_tqdm=False)]
    llm.exit()

    async def main():
        eng = AsyncLLMEngine(d, stream_queue_size=64, **KW)
        streams = [await eng.submit(p, sp) for p in prompts]

        async def collect(s):
            outs = [o async for o in s]
            return outs

        results = await asyncio.gather(*(collect(s) for s in streams))
        await eng.close()
        return results

    results = asyncio.run(main())
    for outs, w in zip(results, want):
        assert list(outs[-1].token_ids) == w
        assert outs[-1].finished and outs[-1].finish_reason == "length"
        # outputs are cumulative and grow one token per decode step
        assert [len(o.token_ids) for o in outs] == list(range(1, len(w) + 1))


def test_async_cancel_frees_request_and_small_queue_keeps_final(ckpt):
    d, cfg = ckpt
    prompts = _prompts(2, 10, cfg["vocab_size"], seed=2)

    async def main():
        eng = AsyncLLMEngine(d, stream_queue_size=1, **KW)
        s_cancel = await eng.submit(prompts[0], SamplingParams(temperature=0.0, max_tokens=50, ignore_eos=True))
        s_slow = await eng.submit(prompts[1], SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
        first = await s_cancel.__anext__()
        assert await s_cancel.cancel()
        rest = [o async for o in s_cancel]
        await asyncio.sleep(0.2)   # the slow consumer lets its bounded queue overflow
        outs = [o async for o in s_slow]
        m = await eng.get_runtime_metrics()
        await eng.close()
        return first, rest, outs, m

    first, rest, outs, m = asyncio.run(main())
    assert len(first.token_ids) >= 1 and rest == []
    assert outs[-1].finished and len(outs[-1].token_ids) == 8
    assert m["scheduler"]["aborted_request_count"] == 1


def test_async_failure_fails_streams_and_rejects_new(ckpt):
    d, cfg = ckpt
    prompts = _prompts(1, 10, cfg["vocab_size"], seed=3)

    async def main():
        eng = AsyncLLMEngine(d, **KW)

        def boom():
            raise RuntimeError("injected step failure")

        eng.engine.step = boom
        s = await eng.submit(prompts[0], SamplingParams(temperature=0.0, max_tokens=4))
        with pytest.raises(RuntimeError):
            async for _ in s:
                pass
        with pytest.raises(RuntimeError):
            await eng.submit(prompts[0], SamplingParams(temperature=0.0, max_tokens=4))
        with pytest.raises(RuntimeError):
            await eng.close()

    asyncio.run(main())


def test_device_error_status_fails_the_step_and_the_streams(ckpt):
    """A nonzero status word after a step (a kernel's bounded wait ran out) makes
    ``LLMEngine.step`` raise ``DeviceErrorStatus`` naming the module; the async engine's failure
    latch then fails every open stream with it.  The status word is faked on the CPU runner: the
    GPU test ``tests/test_engine_errors_gpu.py`` drives the same path from a real kernel."""
    from inference_systems_b200.engine.model_runner import DeviceErrorStatus

    d, cfg = ckpt
    prompts = _prompts(2, 10, cfg["vocab_size"], seed=4)

    def poison(runner):
        runner.error_addrs = "fake"   # any non-None value: the runner appends and checks a status word
        runner.with_status = lambda toks: torch.cat((toks.to(torch.int32), torch.tensor([1 << 2], dtype=torch.int32)))
        runner._read_error_words = lambda: 0x2 << 16

    llm = LLM(d, **KW)
    poison(llm.model_runner)
    llm.add_request(prompts[0], SamplingParams(temperature=0.0, max_tokens=4))
    with pytest.raises(DeviceErrorStatus, match="tp-communication=0x2"):
        llm.step()
    assert llm.model_runner.get_metrics()["device_errors"] == 1
    llm.exit()

    async def main():
        eng = AsyncLLMEngine(d, **KW)
        poison(eng.engine.model_runner)
        streams = [await eng.submit(p, SamplingParams(temperature=0.0, max_tokens=4)) for p in prompts]
        for s in streams:
            with pytest.raises(RuntimeError) as info:
                async for _ in s:
                    pass
            assert isinstance(info.value.__cause__, DeviceErrorStatus)
        with pytest.raises(RuntimeError):
            await eng.close()

    asyncio.run(main())


def test_server_completions_stream_and_metrics(ckpt):
    from fastapi.testclient import TestClient

    from inference_systems_b200.server import create_app

    d, cfg = ckpt
    prompt = _prompts(1, 12, cfg["vocab_size"], seed=4)[0]
    llm = LLM(d, **KW)
    want = llm.generate([prompt], SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True),
                        use_tqdm=False)[0]["token_ids"]
    llm.exit()
    eng = AsyncLLMEngine(d, **KW)
    with TestClient(create_app(eng)) as client:
        assert client.get("/health").json() == {"status": "ok"}
        assert client.get("/v1/models").json()["data"][0]["id"] == d
        r = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 5, "temperature": 0.0,
                                                 "ignore_eos": True})
        body = r.json()
        assert r.status_code == 200, body
        assert body["choices"][0]["token_ids"] == want
        assert body["usage"] == {"prompt_tokens": 12, "completion_tokens": 5, "total_tokens": 17}
        with client.stream("POST", "/v1/completions", json={"prompt": prompt, "max_tokens": 5, "temperature": 0.0,
                                                            "ignore_eos": True, "stream": True}) as resp:
            lines = [ln for ln in resp.iter_lines() if ln.startswith("data: ")]
        assert lines[-1] == "data: [DONE]"
        chunks = [json.loads(ln[6:]) for ln in lines[:-1]]
        assert chunks[-1]["choices"][0]["token_ids"] == want
        assert chunks[-1]["choices"][0]["finish_reason"] == "length"
        assert client.post("/v1/completions", json={"prompt": prompt, "bogus": 1}).status_code == 422
        assert client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}]}
                           ).status_code == 400
        m = client.get("/metrics").json()
        assert m["scheduler"]["completed_request_count"] >= 2
        assert len(client.get("/metrics/requests").json()) >= 2


def test_server_cli_maps_config_flags():
    from inference_systems_b200.server import parse_args

    args, kw = parse_args(["--model", "m", "--tensor-parallel-size", "2", "--disable-prefix-cache",
                           "--num-speculative-tokens", "2", "--hybrid-prefix-checkpoint-memory-mib", "64",
                           "--no-enforce-eager", "--scheduling-policy", "slo_aware",
                           "--mtp-synthetic-acceptance", "0.6"])
    assert args.model == "m"
    assert kw["tensor_parallel_size"] == 2 and kw["enable_prefix_cache"] is False
    assert kw["num_speculative_tokens"] == 2 and kw["enforce_eager"] is False
    assert kw["hybrid_prefix_checkpoint_memory_bytes"] == 64 << 20
    assert kw["scheduling_policy"] == "slo_aware" and kw["mtp_synthetic_acceptance"] == 0.6
