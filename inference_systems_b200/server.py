"""OpenAI-compatible HTTP server over ``AsyncLLMEngine``.

    python -m inference_systems_b200.server --model /path/to/qwen3.5 --tensor-parallel-size 2

Parity (behaviour): ``nanovllm/server.py:21-464`` -- ``/health``,
``/v1/models``, ``/metrics``, ``/metrics/requests``, ``/v1/completions`` and
``/v1/chat/completions`` (chat template), optional SSE streaming of text
deltas terminated by ``data: [DONE]``, usage counts, client disconnect
cancels the request.  Extensions: a completion prompt may also be a list of
token ids, and responses carry ``token_ids`` (useful for checkpoints without a
tokenizer).

The CLI is generated from ``Config``: every engine field ``foo_bar`` is the
flag ``--foo-bar`` (booleans as ``--foo-bar`` / ``--no-foo-bar``), plus the
reference's spellings (``--disable-prefix-cache``,
``--hybrid-prefix-checkpoint-memory-mib``, ...).
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import time
from contextlib import asynccontextmanager
from typing import Literal

from pydantic import BaseModel, ConfigDict, Field

from inference_systems_b200.async_llm import AsyncLLMEngine, RequestStream, StreamOutput
from inference_systems_b200.sampling_params import SamplingParams


class CompletionRequest(BaseModel):
    model_config = ConfigDict(extra="forbid")

    model: str | None = None
    prompt: str | list[int] = Field(min_length=1)
    max_tokens: int = Field(default=64, ge=1)
    temperature: float = Field(default=1.0, ge=0.0)
    stream: bool = False
    ignore_eos: bool = False


class ChatMessage(BaseModel):
    model_config = ConfigDict(extra="forbid")

    role: Literal["system", "user", "assistant"]
    content: str


class ChatCompletionRequest(BaseModel):
    model_config = ConfigDict(extra="forbid")

    model: str | None = None
    messages: list[ChatMessage] = Field(min_length=1)
    max_tokens: int = Field(default=64, ge=1)
    temperature: float = Field(default=1.0, ge=0.0)
    stream: bool = False
    ignore_eos: bool = False


def _sampling(req) -> SamplingParams:
    return SamplingParams(temperature=req.temperature, max_tokens=req.max_tokens, ignore_eos=req.ignore_eos)


def _sse(payload) -> str:
    return f"data: {payload if isinstance(payload, str) else json.dumps(payload)}\n\n"


def _delta(prev: str, cur: str) -> str:
    return cur[len(prev):] if cur.startswith(prev) else cur


async def _last(stream: RequestStream) -> StreamOutput | None:
    out = None
    async for out in stream:
        pass
    return out


def create_app(engine: AsyncLLMEngine, close_engine: bool = True):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import JSONResponse, StreamingResponse

    @asynccontextmanager
    async def lifespan(_app):
        yield
        if close_engine:
            await engine.close()

    app = FastAPI(title="inference_systems_b200", lifespan=lifespan)

    async def submit(prompt, req):
        try:
            return await engine.submit(prompt, _sampling(req))
        except ValueError as e:
            raise HTTPException(status_code=400, detail=str(e)) from e
        except RuntimeError as e:
            raise HTTPException(status_code=503, detail=str(e)) from e

    def n_prompt(prompt) -> int:
        if isinstance(prompt, list):
            return len(prompt)
        tok = engine.tokenizer
        return len(tok.encode(prompt)) if tok is not None else 0

    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": engine.model_name, "object": "model", "created": 0,
                                            "owned_by": "inference_systems_b200"}]}

    @app.get("/metrics")
    async def metrics():
        return JSONResponse(await engine.get_runtime_metrics())

    @app.get("/metrics/requests")
    async def request_metrics():
        return JSONResponse(await engine.get_request_metrics())

    async def run(prompt, req, chat: bool):
        stream = await submit(prompt, req)
        rid = f"{'chatcmpl' if chat else 'cmpl'}-{stream.request_id}"
        created = int(time.time())
        model = req.model or engine.model_name
        obj = "chat.completion" if chat else "text_completion"
        if not req.stream:
            try:
                out = await _last(stream)
            finally:
                await stream.aclose()
            text = out.text if out else ""
            toks = list(out.token_ids) if out else []
            choice = {"index": 0, "finish_reason": out.finish_reason if out else None, "token_ids": toks}
            if chat:
                choice["message"] = {"role": "assistant", "content": text}
            else:
                choice["text"] = text
            usage_p = n_prompt(prompt)
            return {"id": rid, "object": obj, "created": created, "model": model, "choices": [choice],
                    "usage": {"prompt_tokens": usage_p, "completion_tokens": len(toks),
                              "total_tokens": usage_p + len(toks)}}

        async def events():
            prev = ""
            chunk_obj = "chat.completion.chunk" if chat else "text_completion"
            try:
                if chat:
                    yield _sse({"id": rid, "object": chunk_obj, "created": created, "model": model,
                                "choices": [{"index": 0, "delta": {"role": "assistant"}, "finish_reason": None}]})
                async for out in stream:
                    d = _delta(prev, out.text)
                    prev = out.text
                    body = {"delta": {"content": d}} if chat else {"text": d}
                    body.update(index=0, finish_reason=out.finish_reason, token_ids=list(out.token_ids))
                    yield _sse({"id": rid, "object": chunk_obj, "created": created, "model": model,
                                "choices": [body]})
                yield _sse("[DONE]")
            finally:
                await stream.aclose()  # client went away (or done): abort frees KV + state

        return StreamingResponse(events(), media_type="text/event-stream")

    @app.post("/v1/completions")
    async def completions(req: CompletionRequest):
        return await run(req.prompt, req, chat=False)

    @app.post("/v1/chat/completions")
    async def chat_completions(req: ChatCompletionRequest):
        tok = engine.tokenizer
        if tok is None:
            raise HTTPException(status_code=400, detail="chat completions need a tokenizer with a chat template")
        prompt = tok.apply_chat_template([m.model_dump() for m in req.messages], tokenize=False,
                                         add_generation_prompt=True)
        return await run(prompt, req, chat=True)

    return app


# --------------------------------------------------------------------- CLI
_ALIASES = {
    # reference spelling -> (Config field, value transform)
    "--disable-prefix-cache": ("enable_prefix_cache", lambda v: not v),
    "--disable-chunked-prefill": ("enable_chunked_prefill", lambda v: not v),
    "--sequential-speculative-verify": ("speculative_parallel_verify", lambda v: not v),
    "--disable-hybrid-scheduler-aging": ("hybrid_scheduler_enable_aging", lambda v: not v),
    "--disable-hybrid-scheduler-hysteresis": ("hybrid_scheduler_enable_hysteresis", lambda v: not v),
    "--disable-hybrid-scheduler-sticky-recovery": ("hybrid_scheduler_enable_sticky_recovery", lambda v: not v),
}


def parse_args(argv=None) -> tuple[argparse.Namespace, dict]:
    from inference_systems_b200.config import Config

    p = argparse.ArgumentParser(description="OpenAI-compatible server for inference_systems_b200")
    p.add_argument("--model", required=True)
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=8000)
    p.add_argument("--stream-queue-size", type=int, default=16)
    p.add_argument("--hybrid-prefix-checkpoint-memory-mib", type=float, default=None)
    fields = {f.name: f for f in dataclasses.fields(Config) if f.init and f.name != "model"}
    for flag, (name, _) in _ALIASES.items():
        if name in fields:
            p.add_argument(flag, action="store_true", dest=f"alias_{name}")
    for name, f in fields.items():
        flag = "--" + name.replace("_", "-")
        default = f.default if f.default is not dataclasses.MISSING else None
        ann = str(f.type)
        if default is None:  # optional field: take the type from the annotation
            default = False if "bool" in ann else 0.0 if "float" in ann else 0 if "int" in ann else None
        if isinstance(default, bool):
            p.add_argument(flag, dest=name, action=argparse.BooleanOptionalAction, default=None)
        elif isinstance(default, int):
            p.add_argument(flag, dest=name, type=int, default=None)
        elif isinstance(default, float):
            p.add_argument(flag, dest=name, type=float, default=None)
        else:
            p.add_argument(flag, dest=name, type=str, default=None)
    args = p.parse_args(argv)
    kwargs = {name: getattr(args, name) for name in fields if getattr(args, name, None) is not None}
    for flag, (name, fn) in _ALIASES.items():
        if getattr(args, f"alias_{name}", False):
            kwargs[name] = fn(True)
    if args.hybrid_prefix_checkpoint_memory_mib is not None:
        kwargs["hybrid_prefix_checkpoint_memory_bytes"] = int(args.hybrid_prefix_checkpoint_memory_mib * (1 << 20))
    return args, kwargs


def main(argv=None) -> None:
    import uvicorn

    args, kwargs = parse_args(argv)
    engine = AsyncLLMEngine(args.model, stream_queue_size=args.stream_queue_size, **kwargs)
    uvicorn.run(create_app(engine), host=args.host, port=args.port)


if __name__ == "__main__":
    main()
