"""Tensor parallelism on GPUs (TP 2, 4, 8) against TP 1 on the same checkpoint.

The exchange under test: the row-parallel GEMM reduce-scatters its fp32 partial product by
token over NVLink, the owner adds the residual, applies the next RMSNorm and pushes the row to
every rank (``parallel/comm.py``); the LM head samples through the cross-rank argmax.

bf16 activations make the TP=1 and TP=n sums round differently, so free-running greedy decoding
can legitimately part ways at a near-tie.  The checks therefore compare the models position by
position under teacher forcing: one prefill of the same token rows on both, then
(a) the final hidden states agree within a bf16 tolerance, and (b) the argmax of the logits
computed from them agrees at every position whose top-2 margin is not a near-tie.  Prefills of
120 and 420 tokens cover the swap-AB (decode-size) and the tiled (prefill-size) GEMM paths of the
exchange.  The CUDA-graph decode path is checked the same way: every token that TP=n emits must
be the teacher-forced argmax of TP=1's logits (or a near-tie).
"""

import os
import socket

import pytest
import torch
from safetensors.torch import load_file, save_file

from inference_systems_b200 import SamplingParams
from inference_systems_b200.models.presets import preset, random_state_dict, write_config

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
NEAR_TIE = 0.05  # logit margin below which either of the top two tokens is accepted


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    # 8 query / GDN heads so that every TP size up to 8 divides them (2 KV heads: replicated at TP 4, 8)
    cfg = preset("tiny_hd", num_attention_heads=8, linear_num_key_heads=8, linear_num_value_heads=8)
    sd = random_state_dict(cfg, seed=0, std=0.05)
    d = str(tmp_path_factory.mktemp("tp"))
    write_config(d, cfg)
    save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(d, "model.safetensors"))
    return d, cfg


def _llm(d, tp, **kw):
    from inference_systems_b200.llm import LLM

    return LLM(d, device="cuda", tensor_parallel_size=tp, max_num_seqs=4, max_num_state_slots=4, max_model_len=1024,
               num_kvcache_blocks=24, max_num_batched_tokens=1024, dist_port=_free_port(), **kw)


def _prefill_hidden(llm, prompts):
    llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True), use_tqdm=False)
    return llm.model_runner.last_hidden_host()


def _logits(hidden, emb):
    return hidden.float() @ emb.float().t()


def _argmax_agrees(a_logits, b_logits):
    """Fraction of rows whose argmax agrees, counting near-ties (in ``a``) as agreement."""
    top2 = a_logits.topk(2, dim=-1)
    margin = top2.values[:, 0] - top2.values[:, 1]
    same = a_logits.argmax(-1) == b_logits.argmax(-1)
    return ((same | (margin < NEAR_TIE)).float().mean().item(), int((margin < NEAR_TIE).sum()))


def _flips_are_within_logit_error(a_logits, b_logits):
    """Every row where the two argmaxes differ is a tie within the rows' own logit error: a's
    logit of b's choice is below a's maximum by at most twice the largest |a - b| of that row."""
    ia, ib = a_logits.argmax(-1), b_logits.argmax(-1)
    err = (a_logits - b_logits).abs().max(-1).values
    gap = a_logits.max(-1).values - a_logits.gather(-1, ib[:, None])[:, 0]
    flip = ia != ib
    return bool((gap[flip] <= 2 * err[flip] + 1e-4).all()), int(flip.sum())


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_tp_matches_tp1_teacher_forced(ckpt, tp):
    if torch.cuda.device_count() < tp:
        pytest.skip(f"needs {tp} GPUs")
    d, cfg = ckpt
    emb = load_file(os.path.join(d, "model.safetensors"))["model.embed_tokens.weight"]
    g = torch.Generator().manual_seed(11)
    v = cfg["vocab_size"]
    small = [torch.randint(0, v, (40,), generator=g).tolist() for _ in range(3)]                 # 120 rows
    large = [torch.randint(0, v, (n,), generator=g).tolist() for n in (300, 60, 60)]             # 420 rows
    hidden, gen = {}, {}
    for size in (1, tp):
        llm = _llm(d, size, enforce_eager=False)
        hidden[size] = [_prefill_hidden(llm, small), _prefill_hidden(llm, large)]
        gen[size] = [o["token_ids"] for o in llm.generate(small, SamplingParams(temperature=0.0, max_tokens=8,
                                                                                 ignore_eos=True), use_tqdm=False)]
        llm.exit()
        assert torch.ops.isb.error_word() == 0
    for h1, hn in zip(hidden[1], hidden[tp]):
        assert h1.shape == hn.shape
        rel = ((h1 - hn).norm() / h1.norm()).item()
        assert rel < 2e-2, rel
        l1, ln = _logits(h1, emb), _logits(hn, emb)
        frac, ties = _argmax_agrees(l1, ln)
        # fp32 sums over a different split of K round differently: at most 1 % of rows may pick a
        # different token, and only where TP=1's own two candidates are within the logit error
        assert frac >= 0.99, (frac, ties)
        bounded, flips = _flips_are_within_logit_error(l1, ln)
        assert bounded, flips
    # graph decode at TP=n: every emitted token is TP=1's teacher-forced argmax (or a near-tie)
    llm = _llm(d, 1, enforce_eager=True)
    for p, toks in zip(small, gen[tp]):
        h = _prefill_hidden(llm, [p + toks])
        lg = _logits(h[len(p) - 1: len(p) - 1 + len(toks)], emb)
        top2 = lg.topk(2, dim=-1)
        ok = (lg.argmax(-1) == torch.tensor(toks)) | (top2.values[:, 0] - top2.values[:, 1] < NEAR_TIE)
        assert bool(ok.all()), (toks, lg.argmax(-1).tolist())
    llm.exit()


def test_mtp_at_tp2_is_teacher_forced_greedy(ckpt):
    """MTP speculative decoding under TP=2 with the head's own drafts (verify pass, on-device
    accept, GDN replay commit, drafts through the cross-rank LM head, one CUDA graph per round):
    lossless greedy decoding means every emitted token is the target's greedy token given the
    tokens before it (TP=1 teacher-forced logits, near-ties accepted)."""
    d, cfg = ckpt
    emb = load_file(os.path.join(d, "model.safetensors"))["model.embed_tokens.weight"]
    g = torch.Generator().manual_seed(12)
    prompts = [torch.randint(0, cfg["vocab_size"], (50,), generator=g).tolist() for _ in range(3)]
    llm = _llm(d, 2, enforce_eager=False, num_speculative_tokens=2)
    out = [o["token_ids"] for o in llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=10,
                                                                         ignore_eos=True), use_tqdm=False)]
    mtp = llm.get_runtime_metrics()["model_runner"]["mtp"]
    llm.exit()
    assert mtp["rounds"] > 0 and mtp["cudagraph_replays"] == mtp["rounds"]
    assert [len(o) for o in out] == [10, 10, 10]
    ref = _llm(d, 1, enforce_eager=True)
    for p, toks in zip(prompts, out):
        h = _prefill_hidden(ref, [p + toks])
        lg = _logits(h[len(p) - 1: len(p) - 1 + len(toks)], emb)
        top2 = lg.topk(2, dim=-1)
        ok = (lg.argmax(-1) == torch.tensor(toks)) | (top2.values[:, 0] - top2.values[:, 1] < NEAR_TIE)
        assert bool(ok.all()), (toks, lg.argmax(-1).tolist())
    ref.exit()
    assert torch.ops.isb.error_word() == 0
