"""Synchronous serving engine (``LLM``).

Parity: ``nanovllm/engine/llm_engine.py:23-248`` -- build ``Config`` from
keyword arguments (unknown keys ignored), start tensor-parallel workers,
construct the rank-0 runner, tokenizer and scheduler; ``step`` executes every
scheduled batch and drives the hybrid-prefix capture transaction;
``generate`` loops until all requests finish and returns
``[{"text", "token_ids"}]`` in submission order.

Worker ranks are either spawned here (one process per GPU) or, when the
process was started by ``torch.distributed.run`` with ``WORLD_SIZE`` equal to
the TP size, already running: then ranks > 0 enter ``serve_worker`` and only
rank 0 constructs an ``LLMEngine``.
"""

from __future__ import annotations

import atexit
import gc
import os
from dataclasses import dataclass, fields
from time import perf_counter

import torch
import torch.multiprocessing as mp

from inference_systems_b200.config import Config
from inference_systems_b200.engine.model_runner import ModelRunner
from inference_systems_b200.engine.scheduler import Scheduler
from inference_systems_b200.engine.sequence import Sequence
from inference_systems_b200.sampling_params import SamplingParams


@dataclass(frozen=True)
class StepStats:
    prefill_tokens: int = 0
    decode_tokens: int = 0


def _config_from_kwargs(model, kwargs) -> Config:
    names = {f.name for f in fields(Config) if f.init}
    return Config(model, **{k: v for k, v in kwargs.items() if k in names})


def _worker_main(config: Config, rank: int) -> None:
    ModelRunner(config, rank)


def externally_launched(tp: int) -> bool:
    """True when this process is one rank of a ``torchrun`` job of exactly ``tp`` ranks."""
    return tp > 1 and int(os.environ.get("WORLD_SIZE", "1")) == tp and "RANK" in os.environ


def serve_worker(model, **kwargs) -> None:
    """Entry point for ranks > 0 of an externally launched job: run commands until ``exit``."""
    config = _config_from_kwargs(model, kwargs)
    ModelRunner(config, int(os.environ["RANK"]))


def _load_tokenizer(model):
    if isinstance(model, dict):
        return None
    names = ("tokenizer.json", "tokenizer_config.json", "vocab.json", "tokenizer.model")
    if not any(os.path.exists(os.path.join(model, n)) for n in names):
        return None
    from transformers import AutoTokenizer
    return AutoTokenizer.from_pretrained(model, use_fast=True)


class LLMEngine:
    def __init__(self, model, **kwargs):
        self._exited = False
        config = _config_from_kwargs(model, kwargs)
        self.config = config
        Sequence.block_size = config.kvcache_block_size
        self.ps = []
        if config.tensor_parallel_size > 1 and not externally_launched(config.tensor_parallel_size):
            ctx = mp.get_context("spawn")
            for r in range(1, config.tensor_parallel_size):
                p = ctx.Process(target=_worker_main, args=(config, r), daemon=False)
                p.start()
                self.ps.append(p)
        self.model_runner = ModelRunner(config, 0)
        self.tokenizer = _load_tokenizer(model)
        if self.tokenizer is not None and self.tokenizer.eos_token_id is not None and kwargs.get("eos") is None:
            config.eos = self.tokenizer.eos_token_id
        self.scheduler = Scheduler(config, state_manager=self.model_runner.state_manager,
                                   state_controller=self.model_runner,
                                   prefix_checkpoint_pool=self.model_runner.prefix_checkpoint_pool)
        atexit.register(self.exit)

    # ------------------------------------------------------------- lifecycle
    def exit(self) -> None:
        if self._exited:
            return
        self._exited = True
        atexit.unregister(self.exit)
        if hasattr(self, "scheduler"):
            self.scheduler.state_controller = None
            self.scheduler.state_manager = None
        runner = self.model_runner
        runner.call("exit")
        del self.model_runner
        del runner
        for p in self.ps:
            p.join()
        gc.collect()
        if torch.cuda.is_available():
            torch.cuda.empty_cache()

    # --------------------------------------------------------------- requests
    def add_request(self, prompt: str | list[int], sampling_params: SamplingParams,
                    arrival_time_ns: int | None = None) -> int:
        seq = self.make_request(prompt, sampling_params, arrival_time_ns)
        self.scheduler.add(seq)
        return seq.seq_id

    def make_request(self, prompt: str | list[int], sampling_params: SamplingParams,
                     arrival_time_ns: int | None = None) -> Sequence:
        """Validate and tokenize a request without touching the scheduler (any thread may call it)."""
        if isinstance(prompt, str):
            if self.tokenizer is None:
                raise ValueError("this model directory has no tokenizer; pass token ids")
            prompt = self.tokenizer.encode(prompt)
        if self.config.num_speculative_tokens and sampling_params.temperature > 1e-10:
            raise ValueError("native MTP speculative decoding currently supports greedy sampling only")
        if len(prompt) > self.config.max_model_len:
            raise ValueError("prompt exceeds max_model_len")
        if not prompt:
            raise ValueError("prompt must contain at least one token")
        return Sequence(prompt, sampling_params, arrival_time_ns=arrival_time_ns)

    def abort_request(self, request_id: int) -> bool:
        return self.scheduler.abort(request_id)

    def reset_runtime_metrics(self) -> None:
        self.scheduler.reset_metrics()
        self.model_runner.call("reset_metrics")

    def get_runtime_metrics(self) -> dict:
        return {"scheduler": self.scheduler.get_metrics(), "model_runner": self.model_runner.call("get_metrics")}

    def get_request_metrics(self) -> list[dict]:
        return self.scheduler.get_request_metrics()

    # ------------------------------------------------------------------ step
    def _run_captures(self, batch) -> bool:
        pending, hashed = self.scheduler.prepare_prefix_captures(batch.seqs, batch.is_prefill)
        try:
            for cap in pending:
                slot = None
                try:
                    if not self.scheduler.reserve_prefix_capture(cap):
                        continue
                    slot = self.model_runner.call("capture_prefix_checkpoint", cap.state_slot,
                                                  cap.boundary_tokens if cap.internal_state else None)
                    self.scheduler.publish_prefix_capture(cap, slot)
                except Exception:
                    if slot is not None:
                        self.model_runner.call("evict_prefix_checkpoint", slot)
                    self.scheduler.cancel_prefix_capture(cap)
                    raise
        finally:
            if batch.is_prefill and self.scheduler.enable_hybrid_internal_checkpoints:
                for seq in batch.seqs:
                    if seq.state_slot is not None:
                        self.model_runner.call("discard_internal_prefix_states", seq.state_slot)
        return hashed

    def step(self):
        outputs = []
        prefill_tokens = decode_tokens = 0
        for batch in self.scheduler.schedule():
            n = batch.num_tokens
            t0 = perf_counter()
            spec = self.config.num_speculative_tokens > 0 and not batch.is_prefill
            if spec:
                token_ids = self.model_runner.call("run_speculative", batch.seqs)
            else:
                inner = self.scheduler.internal_prefix_boundaries(batch.seqs, batch.is_prefill)
                token_ids = self.model_runner.call("run", batch.seqs, batch.is_prefill, inner)
            self.scheduler.observe_batch(batch.is_prefill, n, (perf_counter() - t0) * 1000)
            hashed = self._run_captures(batch)
            if spec:
                self.scheduler.postprocess_speculative(batch.seqs, token_ids)
            else:
                self.scheduler.postprocess(batch.seqs, token_ids, batch.is_prefill, blocks_already_hashed=hashed)
            outputs.extend((s.seq_id, s.completion_token_ids) for s in batch.seqs if s.is_finished)
            if batch.is_prefill:
                prefill_tokens += n
            else:
                decode_tokens += sum(len(t) for t in token_ids) if spec else n
        return outputs, StepStats(prefill_tokens, decode_tokens)

    def is_finished(self) -> bool:
        return self.scheduler.is_finished()

    def _decode_text(self, token_ids: list[int]) -> str:
        return self.tokenizer.decode(token_ids) if self.tokenizer is not None else ""

    def generate(self, prompts, sampling_params, use_tqdm: bool = True) -> list[dict]:
        from tqdm.auto import tqdm

        if not isinstance(sampling_params, list):
            sampling_params = [sampling_params] * len(prompts)
        ids = [self.add_request(p, sp) for p, sp in zip(prompts, sampling_params)]
        pbar = tqdm(total=len(prompts), desc="Generating", dynamic_ncols=True, disable=not use_tqdm)
        results: dict[int, list[int]] = {}
        prefill_tps = decode_tps = 0.0
        while not self.is_finished():
            t = perf_counter()
            out, stats = self.step()
            dt = perf_counter() - t
            if stats.prefill_tokens:
                prefill_tps = stats.prefill_tokens / dt
            if stats.decode_tokens:
                decode_tps = stats.decode_tokens / dt
            pbar.set_postfix({"Prefill": f"{int(prefill_tps)}tok/s", "Decode": f"{int(decode_tps)}tok/s"})
            for sid, toks in out:
                results[sid] = toks
                pbar.update(1)
        pbar.close()
        return [{"text": self._decode_text(results[i]), "token_ids": results[i]} for i in ids]
