"""Per-rank model executor.

Parity: ``nanovllm/engine/model_runner.py`` -- one runner per tensor-parallel
rank; rank 0 lives in the user process and forwards every call to the
workers (``call`` / ``loop``); KV cache sized from free memory; GDN state slot
pool; CUDA-graph decode buckets; sampling; partial-page KV copy with all-rank
consensus; hybrid prefix checkpoint capture/restore; metrics.

B200-first design:
* All per-step metadata (token ids, positions, slot mapping, cu_seqlens,
  context lengths, state slots, block tables, RNG counter, temperatures) is
  packed into ONE pinned int32 buffer and moved with ONE host->device copy.
* Kernels read/write the GDN pools in place by slot id; no gather/scatter.
* The LM head is fused with greedy/Gumbel-max selection and a cross-rank
  argmax, so every rank knows the sampled tokens (no logits gather, no token
  broadcast) and one device->host copy returns them.
* A decode step (embedding -> all layers -> LM head + sampling) is one CUDA
  graph per batch bucket.
"""

from __future__ import annotations

import os
from time import perf_counter_ns

import numpy as np
import torch
import torch.distributed as dist

from inference_systems_b200.engine.profiler import PhaseProfiler
from inference_systems_b200.engine.sequence import Sequence
from inference_systems_b200.engine.state_pool import (
    HybridPrefixCheckpointPool,
    HybridStateManager,
    transactional_capture_prefix_checkpoint,
    transactional_restore_prefix_checkpoint,
)
from inference_systems_b200.models.registry import create_model
from inference_systems_b200.utils.context import ForwardBatch
from inference_systems_b200.utils.loader import init_dummy, load_model


def count_graph_kernels(handle: int) -> int:
    """Number of kernel nodes in a captured CUDA graph (-1 if the bindings are unavailable)."""
    try:
        from cuda.bindings import runtime as rt

        graph = rt.cudaGraph_t(init_value=handle)
        err, _, n = rt.cudaGraphGetNodes(graph, 0)
        err, nodes, n = rt.cudaGraphGetNodes(graph, n)
        kernel = rt.cudaGraphNodeType.cudaGraphNodeTypeKernel
        return sum(1 for node in nodes if rt.cudaGraphNodeGetType(node)[1] == kernel)
    except Exception:  # pragma: no cover - depends on cuda-python
        return -1


class DeviceErrorStatus(RuntimeError):
    """A kernel of the last step reported an error (a bounded wait ran out or an index was out of
    range): its outputs, and possibly the state it wrote, are not valid."""


ERROR_WORD_MODULES = ("gemm", "attention", "tp-communication", "tensor-core attention", "gdn")


def describe_error_word(word: int) -> str:
    parts = [f"{name}={(word >> (8 * i)) & 0xFF:#x}" for i, name in enumerate(ERROR_WORD_MODULES)
             if (word >> (8 * i)) & 0xFF]
    return ", ".join(parts) or f"{word:#x}"


def _bucket_sizes(max_bs: int) -> list[int]:
    sizes = [1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256, 320, 384, 448, 512]
    out = [s for s in sizes if s < max_bs] + [max_bs]
    return sorted(set(out))


class ModelRunner:
    def __init__(self, config, rank: int = 0, channel_name: str | None = None, start_worker_loop: bool = True):
        self.config = config
        hf = config.hf_config
        self.rank = rank
        self.world_size = config.tensor_parallel_size
        self.block_size = config.kvcache_block_size
        self.enforce_eager = config.enforce_eager
        self.profiler = PhaseProfiler(getattr(config, "enable_mtp_phase_profiling", False))
        self.reset_metrics()
        use_cuda = config.device == "cuda"
        local_rank = int(os.environ.get("LOCAL_RANK", rank))
        self.device = torch.device("cuda", local_rank) if use_cuda else torch.device("cpu")
        if use_cuda:
            torch.cuda.set_device(self.device)
        if self.world_size > 1 and not dist.is_initialized():
            from datetime import timedelta
            from inference_systems_b200.engine.llm_engine import externally_launched
            # under torch.distributed.run the launcher owns the rendezvous store (env://)
            init = "env://" if externally_launched(self.world_size) else f"tcp://127.0.0.1:{config.dist_port}"
            dist.init_process_group("nccl" if use_cuda else "gloo", init_method=init,
                                    world_size=self.world_size, rank=rank,
                                    timeout=timedelta(seconds=config.dist_timeout_s))
        self.dtype = config.torch_dtype
        torch.manual_seed(config.seed)

        # ---------------------------------------------------------- model
        prev = torch.get_default_dtype()
        torch.set_default_dtype(self.dtype)
        try:
            with torch.device(self.device):
                self.model = create_model(hf, config.model_capabilities, tp_rank=rank, tp_size=self.world_size)
                self.mtp = None
                self.num_speculative_tokens = config.num_speculative_tokens
                if self.num_speculative_tokens:
                    from inference_systems_b200.models.qwen3_5_mtp import Qwen3_5MTP
                    self.mtp = Qwen3_5MTP(hf, self.model)
        finally:
            torch.set_default_dtype(prev)
        if config.load_format == "dummy":
            init_dummy(self.model, hf, seed=config.seed)
            if self.mtp is not None:
                init_dummy(self.mtp, hf, seed=config.seed)
        else:
            self.load_report = load_model(self.model, config.model, strict=True)
            if self.mtp is not None:
                load_model(self.mtp, config.model, strict=True)
        if self.world_size > 1:
            from inference_systems_b200.parallel.comm import TPComm
            self.comm = TPComm(self.device, rank, self.world_size, hf.hidden_size, config)
            self.model.comm = self.comm
        else:
            self.comm = None

        # Device addresses of every kernel module's error word: each step appends their state to
        # the sampled tokens (``step_status``), so the one device->host copy per step carries it.
        if self.device.type == "cuda":
            from inference_systems_b200 import ops
            self.error_addrs = ops.cuda_ops().error_word_addresses().to(self.device)
        else:
            self.error_addrs = None
        self.device_errors = 0
        if self.device.type == "cuda":
            spec_rows = config.max_num_seqs * (self.num_speculative_tokens + 1)
            self.model.set_accumulator(max(config.max_num_batched_tokens, config.max_num_seqs, spec_rows), self.device)

        # ------------------------------------------------------ GDN state
        self.state_manager = None
        geo = self.model.gdn_geometry()
        if geo is not None:
            slots = min(config.max_num_state_slots, config.max_num_seqs)
            self.state_manager = HybridStateManager(
                max_num_seqs=slots, num_linear_layers=geo["num_layers"], num_value_heads=geo["hv"],
                key_head_dim=geo["dk"], value_head_dim=geo["dv"], conv_dim=geo["conv_dim"],
                conv_kernel_size=geo["kernel"], conv_dtype=self.dtype, device=self.device)
        self.prefix_checkpoint_pool = None
        if getattr(config, "enable_hybrid_prefix_cache", False):
            self.prefix_checkpoint_pool = HybridPrefixCheckpointPool(
                self.state_manager, config.hybrid_prefix_checkpoint_memory_bytes,
                checkpoint_dtype=config.hybrid_prefix_checkpoint_dtype)
        self.internal_prefix_states: dict = {}

        # --------------------------------------------------------- KV cache
        self.allocate_kv_cache()
        # speculative rounds touch positions up to pending + 2K - 1 (target verify + MTP drafts)
        self.max_blocks_per_seq = (config.max_model_len + 2 * self.num_speculative_tokens + self.block_size) // self.block_size + 1
        self.sample_step = 0
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.graph_bufs: dict[int, dict] = {}
        self.graph_kernels: dict[int, int] = {}
        if self.mtp is not None:
            from inference_systems_b200.engine.mtp import MTPDriver
            self.mtp_driver = MTPDriver(self)
        if self.device.type == "cuda" and not self.enforce_eager:
            if self.mtp is not None:
                # decode batches run as speculative rounds: capture those instead of target-only steps
                self.mtp_driver.capture(_bucket_sizes(self._max_graph_batch()))
            else:
                self.capture_cudagraph()

        # ---------------------------------------------------------- RPC
        self.channel = None
        if self.world_size > 1:
            from inference_systems_b200.engine.rpc import CommandChannel
            name = channel_name or f"isb_rpc_{config.dist_port}"
            if rank == 0:
                self.channel = CommandChannel(name, self.world_size, 0)
                dist.barrier()
            else:
                dist.barrier()
                self.channel = CommandChannel(name, self.world_size, rank)
                if start_worker_loop:
                    self.loop()

    # ================================================================ RPC
    def call(self, method: str, *args):
        if self.world_size > 1 and self.rank == 0:
            self.channel.send(method, *args)
        return getattr(self, method)(*args)

    def loop(self) -> None:
        while True:
            method, args = self.channel.recv()
            getattr(self, method)(*args)
            if method == "exit":
                break

    def exit(self) -> None:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        self.graphs.clear()
        self.graph_bufs.clear()
        if self.mtp is not None:
            self.mtp_driver.graphs.clear()
            self.mtp_driver.graph_bufs.clear()
        if self.comm is not None:
            self.comm.close()
        if self.world_size > 1:
            dist.barrier()
            if self.channel is not None:
                self.channel.close()
            if dist.is_initialized():
                dist.destroy_process_group()

    # ========================================================== KV cache
    def allocate_kv_cache(self) -> None:
        cfg = self.config
        n_attn, hkv, hd = self.model.attention_geometry()
        n_layers = n_attn + (1 if self.mtp is not None else 0)
        self.num_kv_layers = n_layers
        if n_layers == 0:
            cfg.num_kvcache_blocks = max(cfg.num_kvcache_blocks, 1)
            self.kv_cache = None
            return
        block_bytes = 2 * n_layers * self.block_size * hkv * hd * self.dtype.itemsize
        if cfg.num_kvcache_blocks <= 0:
            if self.device.type == "cuda":
                free, total = torch.cuda.mem_get_info(self.device)
                reserve = 4 << 30
                budget = int(free - total * (1 - cfg.gpu_memory_utilization)) - reserve
                n = max(budget // block_bytes, 1)
            else:
                n = cfg.max_num_seqs * ((cfg.max_model_len + self.block_size - 1) // self.block_size + 1)
            if cfg.max_num_kvcache_blocks is not None:
                n = min(n, cfg.max_num_kvcache_blocks)
            cfg.num_kvcache_blocks = int(n)
        assert cfg.num_kvcache_blocks > 0
        self.kv_cache = torch.zeros(n_layers, 2, cfg.num_kvcache_blocks, hkv, self.block_size, hd,
                                    dtype=self.dtype, device=self.device)

    def kv_layers(self) -> list[tuple[torch.Tensor, torch.Tensor]]:
        n_attn = len(self.model.attn_layer_ids)
        return [(self.kv_cache[i, 0], self.kv_cache[i, 1]) for i in range(n_attn)]

    def state_layers(self):
        if self.state_manager is None:
            return None
        return [self.state_manager.layer_pools(j) for j in range(self.state_manager.num_linear_layers)]

    # ========================================================== metadata
    def _pack(self, seqs: list[Sequence], is_prefill: bool, pad_to: int | None = None):
        """Host-side metadata for one forward pass as one int32 array + its field slices."""
        if not is_prefill and seqs:
            return self._pack_decode(seqs, pad_to)
        return self._pack_general(seqs, is_prefill, pad_to)

    def _pack_decode(self, seqs: list[Sequence], pad_to: int | None = None):
        """``_pack`` for a decode batch (one token per sequence), built column-wise with numpy:
        this runs on the host between every two decode steps, so its cost adds to each step's
        end-to-end time (the general loop took about 150 us for 128 sequences)."""
        bs = self.block_size
        b = len(seqs)
        nb = pad_to or b
        mb = self.max_blocks_per_seq
        scratch = self.state_manager.scratch_slot_id if self.state_manager else 0
        # one pass over the sequences, then column arrays
        cols = list(zip(*[(s.num_tokens, s.last_token, s.state_slot, s.temperature, s.block_table) for s in seqs]))
        n = np.array(cols[0], np.int64)
        last_tok = np.array(cols[1], np.int64)
        st = np.array([scratch if x is None else x for x in cols[2]], np.int64)
        lens = [len(x) for x in cols[4]]
        bt = np.full((nb, mb), -1, dtype=np.int32)
        flat_bt = [blk for x in cols[4] for blk in x]
        if flat_bt:
            rows = np.repeat(np.arange(b), lens)
            cidx = np.arange(len(flat_bt)) - np.repeat(np.cumsum(lens) - lens, lens)
            bt[rows, cidx] = flat_bt
        pos = n - 1
        slots = bt[np.arange(b), pos // bs].astype(np.int64) * bs + pos % bs
        ids = np.zeros(nb, np.int32)
        ids[:b] = last_tok
        positions = np.zeros(nb, np.int32)
        positions[:b] = pos
        slot_mapping = np.full(nb, -1, np.int32)
        slot_mapping[:b] = slots
        cu = np.arange(nb + 1, dtype=np.int32)       # one token per row, padding rows included
        ctx = np.zeros(nb, np.int32)
        ctx[:b] = n
        state = np.full(nb, scratch, np.int32)
        state[:b] = st
        last = np.arange(nb, dtype=np.int32)
        temps = np.zeros(nb, dtype=np.float32)
        temps[:b] = cols[3]
        fields = [("input_ids", ids), ("positions", positions), ("slot_mapping", slot_mapping),
                  ("cu_seqlens_q", cu), ("context_lens", ctx), ("state_slots", state), ("logits_indices", last),
                  ("block_tables", bt.reshape(-1)),
                  ("rng", np.asarray([self.config.seed & 0x7FFFFFFF, self.sample_step & 0x7FFFFFFF], np.int32)),
                  ("temperatures", temps.view(np.int32))]
        flat = np.concatenate([f for _, f in fields])
        layout, off = {}, 0
        for name, f in fields:
            layout[name] = (off, f.shape[0])
            off += f.shape[0]
        meta = dict(num_seqs=b, max_q=1, max_k=int(n.max()), cu_host=list(range(b + 1)), slots_host=st.tolist(),
                    nb=nb, mb=mb)
        return flat, layout, meta

    def _pack_general(self, seqs: list[Sequence], is_prefill: bool, pad_to: int | None = None):
        bs = self.block_size
        b = len(seqs)
        nb = pad_to or b
        ids, pos, slots = [], [], []
        cu = [0]
        ctx, st, last = [], [], []
        for s in seqs:
            if is_prefill:
                start, n = s.num_cached_tokens, s.num_scheduled_tokens
                ids.extend(s.token_ids[start:start + n])
                pos.extend(range(start, start + n))
                bt = s.block_table
                if bt:
                    slots.extend(bt[p // bs] * bs + p % bs for p in range(start, start + n))
                else:
                    slots.extend([-1] * n)
                cu.append(cu[-1] + n)
                ctx.append(start + n)
            else:
                p = len(s) - 1
                ids.append(s.last_token)
                pos.append(p)
                slots.append(s.block_table[p // bs] * bs + p % bs)
                cu.append(cu[-1] + 1)
                ctx.append(len(s))
            st.append(s.state_slot if s.state_slot is not None else
                      (self.state_manager.scratch_slot_id if self.state_manager else 0))
            last.append(cu[-1] - 1)
        t = len(ids)
        nt = t if pad_to is None else pad_to
        scratch = self.state_manager.scratch_slot_id if self.state_manager else 0
        for _ in range(nb - b):
            cu.append(cu[-1] + (1 if not is_prefill else 0))
            ctx.append(0)
            st.append(scratch)
            last.append(max(cu[-1] - 1, 0))
        pad_t = nt - t
        ids.extend([0] * pad_t)
        pos.extend([0] * pad_t)
        slots.extend([-1] * pad_t)
        mb = self.max_blocks_per_seq
        bt = np.full((nb, mb), -1, dtype=np.int32)
        for i, s in enumerate(seqs):
            if s.block_table:
                bt[i, :len(s.block_table)] = s.block_table
        temps = np.zeros(nb, dtype=np.float32)
        temps[:b] = [s.temperature for s in seqs]
        fields = [("input_ids", np.asarray(ids, np.int32)), ("positions", np.asarray(pos, np.int32)),
                  ("slot_mapping", np.asarray(slots, np.int32)), ("cu_seqlens_q", np.asarray(cu, np.int32)),
                  ("context_lens", np.asarray(ctx, np.int32)), ("state_slots", np.asarray(st, np.int32)),
                  ("logits_indices", np.asarray(last, np.int32)), ("block_tables", bt.reshape(-1)),
                  ("rng", np.asarray([self.config.seed & 0x7FFFFFFF, self.sample_step & 0x7FFFFFFF], np.int32)),
                  ("temperatures", temps.view(np.int32))]
        flat = np.concatenate([f for _, f in fields])
        layout, off = {}, 0
        for name, f in fields:
            layout[name] = (off, f.shape[0])
            off += f.shape[0]
        meta = dict(num_seqs=b, max_q=max((s.num_scheduled_tokens for s in seqs), default=1) if is_prefill else 1,
                    max_k=max(ctx[:b], default=1), cu_host=cu[: b + 1], slots_host=st[:b], nb=nb, mb=mb)
        return flat, layout, meta

    def _batch_from(self, dev: torch.Tensor, layout, meta, is_prefill: bool) -> tuple[ForwardBatch, torch.Tensor, torch.Tensor]:
        def f(name):
            o, n = layout[name]
            return dev[o:o + n]

        batch = ForwardBatch(
            is_prefill=is_prefill, input_ids=f("input_ids"), positions=f("positions"),
            cu_seqlens_q=f("cu_seqlens_q"), context_lens=f("context_lens"),
            block_tables=f("block_tables").view(meta["nb"], meta["mb"]), slot_mapping=f("slot_mapping"),
            state_slots=f("state_slots"), logits_indices=f("logits_indices"), max_seqlen_q=meta["max_q"],
            max_seqlen_k=meta["max_k"], cu_seqlens_host=meta["cu_host"], slots_host=meta["slots_host"],
            num_seqs=meta["num_seqs"])
        temps = f("temperatures").view(torch.float32)
        return batch, f("rng"), temps

    def _upload(self, flat: np.ndarray) -> torch.Tensor:
        host = torch.from_numpy(flat)
        if self.device.type == "cpu":
            return host.clone()
        pinned = self._pinned(flat.shape[0])
        pinned[: flat.shape[0]].copy_(host)
        self.h2d_bytes += flat.nbytes
        return pinned[: flat.shape[0]].to(self.device, non_blocking=True)

    def _pinned(self, n: int) -> torch.Tensor:
        buf = getattr(self, "_pin_buf", None)
        if buf is None or buf.numel() < n:
            self._pin_buf = torch.empty(max(n, 1 << 16), dtype=torch.int32, pin_memory=True)
        return self._pin_buf

    # ========================================================= forward
    def _forward_sample(self, batch: ForwardBatch, rng: torch.Tensor, temps: torch.Tensor) -> torch.Tensor:
        hidden = self.model(batch, self.kv_layers(), self.state_layers())
        last = hidden.index_select(0, batch.logits_indices.long()) if batch.is_prefill else hidden
        self._last_hidden = hidden
        return self.model.sample(last, temps, rng)

    def with_status(self, toks: torch.Tensor) -> torch.Tensor:
        """``[toks | status]`` on GPUs: the last int32 has bit i set when kernel module i's error
        word is nonzero (``ERROR_WORD_MODULES`` order); unchanged on CPU."""
        if self.error_addrs is None:
            return toks
        from inference_systems_b200 import ops
        return ops.cuda_ops().step_status(toks.to(torch.int32).contiguous(), self.error_addrs)

    def check_status(self, host: torch.Tensor) -> None:
        """Raise ``DeviceErrorStatus`` (rank 0) when the step's status word is nonzero.  The detailed
        words are read (and cleared) first so the message names the failing kernels; workers only
        count the error, rank 0 fails the step for every request."""
        if self.error_addrs is None or int(host[-1]) == 0:
            return
        self.device_errors += 1
        word = self._read_error_words()
        if self.rank == 0:
            raise DeviceErrorStatus(f"device error in the last step ({describe_error_word(word)}); "
                                    "its outputs are not valid")

    def last_hidden_host(self) -> torch.Tensor | None:
        """Final-norm hidden states ``[T, H]`` (fp32, CPU) of the last eagerly run forward pass
        (prefill chunks always run eagerly); used by tests that score tokens against logits."""
        h = getattr(self, "_last_hidden", None)
        return None if h is None else h.float().cpu()

    @staticmethod
    def _read_error_words() -> int:
        """Every module's error word, packed 8 bits per module and cleared (synchronous)."""
        return int(torch.ops.isb.error_word())

    def _tokens_to_host(self, toks: torch.Tensor, n: int) -> list[int]:
        """Copy the sampled tokens (and, on GPUs, the status word after them) to the host."""
        host = toks.to("cpu", non_blocking=False)
        self.d2h_bytes += host.numel() * host.element_size()
        self.check_status(host)
        return host[:n].tolist()

    @torch.inference_mode()
    def run(self, seqs: list[Sequence], is_prefill: bool, internal_boundaries: dict | None = None):
        t0 = perf_counter_ns()
        b = len(seqs)
        bucket = self._graph_bucket(b) if not is_prefill else None
        if bucket is not None:
            flat, layout, meta = self._pack(seqs, False, pad_to=bucket)
            bufs = self.graph_bufs[bucket]
            host = torch.from_numpy(flat)
            pinned = self._pinned(flat.shape[0])
            pinned[: flat.shape[0]].copy_(host)
            bufs["meta"].copy_(pinned[: flat.shape[0]], non_blocking=True)
            self.h2d_bytes += flat.nbytes
            self.graphs[bucket].replay()
            toks = bufs["tokens"]
            self.graph_replays += 1
        else:
            flat, layout, meta = self._pack(seqs, is_prefill)
            dev = self._upload(flat)
            batch, rng, temps = self._batch_from(dev, layout, meta, is_prefill)
            marks = self._internal_history(seqs, batch, meta, internal_boundaries) if is_prefill else None
            toks = self._forward_sample(batch, rng, temps)
            if is_prefill and self.mtp is not None:
                self.mtp_driver.after_prefill(seqs, batch, self._last_hidden, toks, rng)
            if marks:
                self._capture_internal_states(batch, marks)
            toks = self.with_status(toks)
        self.sample_step += 1
        out = self._tokens_to_host(toks, b)
        self.forward_calls += 1
        if is_prefill:
            self.prefill_tokens += int(sum(s.num_scheduled_tokens for s in seqs))
        else:
            self.decode_tokens += b
        self.profiler.record_cpu("target_only.run", (perf_counter_ns() - t0) / 1e6)
        return out if self.rank == 0 else None

    def _internal_history(self, seqs, batch: ForwardBatch, meta, boundaries) -> list | None:
        """Attach GDN history buffers for checkpoint boundaries strictly inside this prefill chunk."""
        if not boundaries or self.state_manager is None:
            return None
        sm = self.state_manager
        cu = meta["cu_host"]
        rows = [-1] * batch.num_tokens
        marks = []  # (state slot, boundary tokens, history row)
        for i, s in enumerate(seqs):
            for b in boundaries.get(s.seq_id, ()):
                t = cu[i] + (b - 1 - s.num_cached_tokens)
                if cu[i] <= t < cu[i + 1]:
                    rows[t] = len(marks)
                    marks.append((s.state_slot, b, t))
        if not marks:
            return None
        r = len(marks)
        rs, cs = sm.recurrent_states.shape, sm.conv_states.shape
        batch.gdn_history = {
            "rows": torch.tensor(rows, dtype=torch.int32).to(self.device),
            "rec": [torch.empty(r, *rs[2:], dtype=torch.float32, device=self.device) for _ in range(rs[0])],
            "conv": [torch.empty(r, *cs[2:], dtype=sm.conv_states.dtype, device=self.device) for _ in range(cs[0])],
        }
        return marks

    def _capture_internal_states(self, batch: ForwardBatch, marks) -> None:
        """Keep the recorded (recurrent, conv) states until the engine publishes the checkpoints."""
        h = batch.gdn_history
        for k, (slot, boundary, _) in enumerate(marks):
            rec = torch.stack([layer[k] for layer in h["rec"]])
            conv = torch.stack([layer[k] for layer in h["conv"]])
            self.internal_prefix_states[(slot, boundary)] = (rec, conv)

    # ======================================================= CUDA graphs
    def _graph_bucket(self, b: int) -> int | None:
        if not self.graphs:
            return None
        for s in sorted(self.graphs):
            if s >= b:
                return s
        return None

    def _max_graph_batch(self) -> int:
        cfg = self.config
        return min(cfg.max_num_seqs, cfg.max_cudagraph_batch_size,
                   self.state_manager.max_num_seqs if self.state_manager else cfg.max_num_seqs)

    @torch.inference_mode()
    def capture_cudagraph(self) -> None:
        max_bs = self._max_graph_batch()
        pool = None
        dummy_seqs = []
        for bs_ in reversed(_bucket_sizes(max_bs)):
            flat, layout, meta = self._pack(dummy_seqs, False, pad_to=bs_)
            meta_dev = torch.from_numpy(flat).to(self.device)
            batch, rng, temps = self._batch_from(meta_dev, layout, meta, False)
            # warm up (kernel autotuning / lazy init) outside the capture
            self._forward_sample(batch, rng, temps)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph(keep_graph=True)
            with torch.cuda.graph(g, pool=pool):
                toks = self.with_status(self._forward_sample(batch, rng, temps))
            g.instantiate()
            if pool is None:
                pool = g.pool()
            self.graph_kernels[bs_] = count_graph_kernels(g.raw_cuda_graph())
            self.graphs[bs_] = g
            self.graph_bufs[bs_] = {"meta": meta_dev, "tokens": toks, "layout": layout}
        torch.cuda.synchronize(self.device)
        if self.state_manager is not None:
            self.state_manager.reset_scratch()

    # ======================================================= state RPCs
    def allocate_state_slot(self, seq: Sequence) -> int | None:
        if self.state_manager is None:
            return None
        return self.state_manager.allocate(seq)

    def free_state_slot(self, seq: Sequence) -> None:
        if self.state_manager is not None:
            self.state_manager.free(seq)

    def capture_prefix_checkpoint(self, state_slot: int, boundary_tokens: int | None = None) -> int:
        if boundary_tokens is not None:
            rec, conv = self.internal_prefix_states.pop((state_slot, boundary_tokens))
            return transactional_capture_prefix_checkpoint(self.prefix_checkpoint_pool, state_slot,
                                                           recurrent_state=rec, conv_state=conv)
        return transactional_capture_prefix_checkpoint(self.prefix_checkpoint_pool, state_slot)

    def restore_prefix_checkpoint(self, seq: Sequence, checkpoint_slot: int) -> None:
        transactional_restore_prefix_checkpoint(self.prefix_checkpoint_pool, checkpoint_slot, seq.state_slot)

    def evict_prefix_checkpoint(self, checkpoint_slot: int) -> None:
        self.prefix_checkpoint_pool.free(checkpoint_slot)

    def discard_internal_prefix_states(self, state_slot: int) -> None:
        for key in [k for k in self.internal_prefix_states if k[0] == state_slot]:
            del self.internal_prefix_states[key]

    def copy_prefix_kv(self, src_block: int, dst_block: int, num_tokens: int) -> None:
        """Partial-page copy-on-write on every rank, then an all-rank MIN consensus."""
        from inference_systems_b200 import ops
        ok = True
        try:
            if not (0 < num_tokens < self.block_size):
                raise ValueError("partial-page copy needs 0 < num_tokens < block_size")
            if self.kv_cache is not None:
                for layer in range(self.kv_cache.shape[0]):
                    ops.copy_kv_page(self.kv_cache[layer, 0], self.kv_cache[layer, 1], src_block, dst_block, num_tokens)
            self.cow_copies += 1
            self.cow_bytes += (2 * self.kv_cache.shape[0] * self.kv_cache.shape[3] * num_tokens
                               * self.kv_cache.shape[5] * self.kv_cache.element_size()) if self.kv_cache is not None else 0
        except Exception:
            ok = False
            if self.world_size == 1:
                raise
        if self.world_size > 1:
            flag = torch.tensor(1 if ok else 0, dtype=torch.int32,
                                device=self.device if dist.get_backend() == "nccl" else "cpu")
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            if int(flag.item()) == 0 and self.rank == 0:
                raise RuntimeError("partial-page KV copy failed on at least one rank")

    # ========================================================== metrics
    def reset_metrics(self) -> None:
        self.forward_calls = 0
        self.graph_replays = 0
        self.prefill_tokens = 0
        self.decode_tokens = 0
        self.cow_copies = 0
        self.cow_bytes = 0
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.profiler.reset()

    def get_metrics(self) -> dict:
        self.profiler.flush()
        m = {
            "forward_calls": self.forward_calls,
            "cudagraph_replays": self.graph_replays,
            "cudagraph_buckets": sorted(self.graphs),
            "prefill_tokens": self.prefill_tokens,
            "decode_tokens": self.decode_tokens,
            "kv_cow_copies": self.cow_copies,
            "kv_cow_bytes": self.cow_bytes,
            "h2d_bytes": self.h2d_bytes,
            "d2h_bytes": self.d2h_bytes,
            "device_errors": self.device_errors,
            "num_kvcache_blocks": self.config.num_kvcache_blocks,
            "phase_profile": self.profiler.metrics(),
        }
        if self.state_manager is not None:
            m["state_pool_bytes"] = self.state_manager.memory_bytes()
            m["state_slots_used"] = len(self.state_manager.used_slot_ids)
        if self.prefix_checkpoint_pool is not None:
            m["checkpoint_pool_bytes"] = self.prefix_checkpoint_pool.memory_bytes()
            m["checkpoint_slots_used"] = len(self.prefix_checkpoint_pool.used_checkpoint_slots)
        if self.mtp is not None:
            m["mtp"] = self.mtp_driver.metrics()
        return m

    # ============================================================ bench
    @torch.inference_mode()
    def bench_replay(self, batch_size: int, warmup: int, steps: int) -> float:
        """Device time (ms, max over ranks) of ``steps`` back-to-back decode-graph replays."""
        g = self.graphs[self._graph_bucket(batch_size)]
        for _ in range(warmup):
            g.replay()
        if self.world_size > 1:
            dist.barrier()
        torch.cuda.synchronize(self.device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize(self.device)
        if self.world_size > 1:
            dist.barrier()
        ms = e0.elapsed_time(e1)
        if self.world_size > 1:
            t = torch.tensor([ms], device=self.device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    @torch.inference_mode()
    def breakdown_replays(self, batch_size: int, path: str, n: int = 3) -> None:
        """Kernel-time table of ``n`` decode-graph replays, profiled on every rank at once (the
        tensor-parallel exchanges need every rank replaying); rank 0 writes ``path``."""
        from inference_systems_b200.engine.profiler import kernel_time_table
        g = self.graphs[self._graph_bucket(batch_size)]
        if self.world_size > 1:
            dist.barrier()
        text = kernel_time_table(g.replay, n)
        if self.rank == 0:
            os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
            with open(path, "w") as f:
                f.write(text)

    def graph_kernel_count(self, batch_size: int) -> int:
        return self.graph_kernels.get(self._graph_bucket(batch_size), -1)

    # ====================================================== speculative
    def run_speculative(self, seqs: list[Sequence]):
        return self.mtp_driver.run(seqs)
