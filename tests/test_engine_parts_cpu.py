"""Request lifecycle metrics, the phase profiler and the model registry on the host.

Scenarios of the reference's ``tests/test_sequence.py``, ``tests/test_phase_profiler.py`` and
``tests/test_model_registry.py`` (``ifeidepig/inference-systems``), run against this package.
"""

from types import SimpleNamespace

import pytest

from inference_systems_b200 import SamplingParams
from inference_systems_b200.engine.profiler import PhaseProfiler
from inference_systems_b200.engine.sequence import Sequence, SequenceStatus
from inference_systems_b200.models.registry import create_model, normalize_hf_config


def test_lifecycle_metrics_from_the_request_timeline():
    s = Sequence([1, 2], SamplingParams(temperature=0.1, max_tokens=2, ignore_eos=True),
                 arrival_time_ns=1_000_000, admitted_time_ns=1_500_000)
    s.block_table = [3, 4]
    s.mark_scheduled(2_000_000)
    s.append_token(5, 3_000_000)
    s.mark_scheduled(4_000_000)
    s.append_token(6, 5_000_000)
    s.status = SequenceStatus.FINISHED
    s.mark_finished(6_000_000)
    m = s.lifecycle_metrics(now_ns=10_000_000)
    assert (m["queue_ms"], m["admission_delay_ms"], m["ttft_ms"], m["e2e_ms"]) == (1.0, 0.5, 2.0, 5.0)
    assert (m["tpot_ms"], m["max_token_gap_ms"], m["time_since_last_token_ms"]) == (2.0, 2.0, 1.0)
    assert (m["schedule_count"], m["peak_kv_blocks"], m["status"], m["output_tokens"]) == (2, 2, "finished", 2)


def test_empty_prompt_is_rejected():
    with pytest.raises(ValueError, match="at least one token"):
        Sequence([])


def test_worker_copy_carries_only_what_a_rank_needs():
    import pickle

    s = Sequence(list(range(10)))
    s.block_table = [7]
    copy = pickle.loads(pickle.dumps(s))
    assert copy.token_ids == list(range(10)) and copy.block_table == [7]
    s.is_prefill = False
    s.append_token(42)
    copy = pickle.loads(pickle.dumps(s))
    assert copy.token_ids == [] and copy.last_token == 42 and copy.num_tokens == 11


def test_disabled_profiler_records_nothing():
    p = PhaseProfiler(enabled=False)
    with p.phase("disabled", gpu=False):
        p.add_counter("ignored", 1)
    assert p.metrics() == {"enabled": False, "flush_count": 0, "flush_sync_ms": 0.0, "counters": {}, "phases": {}}


def test_cpu_profiler_summarises_samples_and_counters():
    p = PhaseProfiler(enabled=True)
    with p.phase("cpu", gpu=False):
        pass
    p.record_cpu("cpu", 2.0)
    p.add_counter("bytes", 10)
    p.add_counter("bytes", 5)
    m = p.metrics()
    assert m["phases"]["cpu"]["cpu_ms"]["count"] == 2 and m["phases"]["cpu"]["gpu_ms"]["count"] == 0
    assert m["counters"]["bytes"] == 15.0
    assert m["phases"]["cpu"]["cpu_ms"]["total"] >= 2.0


def _qwen3():
    return SimpleNamespace(model_type="qwen3", architectures=["Qwen3ForCausalLM"], vocab_size=32, hidden_size=8,
                           intermediate_size=16, num_hidden_layers=2, num_attention_heads=2, num_key_value_heads=1,
                           head_dim=4, hidden_act="silu", max_position_embeddings=32, rms_norm_eps=1e-6,
                           attention_bias=False, rope_theta=10_000, rope_scaling=None, tie_word_embeddings=True)


def _qwen35_wrapper():
    text = SimpleNamespace(
        model_type="qwen3_5_text", vocab_size=32, hidden_size=8, intermediate_size=16, num_hidden_layers=4,
        num_attention_heads=2, num_key_value_heads=1, head_dim=4, hidden_act="silu", max_position_embeddings=32,
        rms_norm_eps=1e-6, attention_bias=False, tie_word_embeddings=False, linear_num_key_heads=2,
        linear_num_value_heads=4, linear_key_head_dim=3, linear_value_head_dim=2, linear_conv_kernel_dim=4,
        layer_types=["linear_attention"] * 3 + ["full_attention"], mtp_num_hidden_layers=1,
        rope_parameters={"partial_rotary_factor": 0.5, "rope_theta": 10_000, "mrope_interleaved": True,
                         "mrope_section": [1, 0, 0]})
    return SimpleNamespace(model_type="qwen3_5", architectures=["Qwen3_5ForConditionalGeneration"], text_config=text)


def test_registry_keeps_qwen3_as_is():
    text, caps = normalize_hf_config(_qwen3())
    assert text.model_type == "qwen3" and caps.architecture == "Qwen3ForCausalLM"
    assert caps.full_attention_layer_indices == (0, 1) and caps.linear_attention_layer_indices == ()
    assert not caps.is_hybrid


def test_registry_maps_the_multimodal_wrapper_to_the_text_runtime():
    text, caps = normalize_hf_config(_qwen35_wrapper())
    assert text.model_type == "qwen3_5_text" and caps.architecture == "Qwen3_5ForCausalLM"
    assert caps.linear_attention_layer_indices == (0, 1, 2) and caps.full_attention_layer_indices == (3,)
    assert caps.is_hybrid and caps.supports_mrope and caps.mtp_num_hidden_layers == 1


def test_registry_rejects_unknown_models_and_layer_kinds():
    with pytest.raises(ValueError, match="unsupported model_type"):
        normalize_hf_config(SimpleNamespace(model_type="llama", num_hidden_layers=1))
    bad = _qwen35_wrapper()
    bad.text_config.layer_types = ["linear_attention", "mamba", "full_attention", "full_attention"]
    with pytest.raises(ValueError, match="unsupported layer types"):
        normalize_hf_config(bad)
    short = _qwen35_wrapper()
    short.text_config.layer_types = ["full_attention"]
    with pytest.raises(ValueError, match="entries for 4 layers"):
        normalize_hf_config(short)


def test_registry_builds_both_families():
    from inference_systems_b200.models.qwen3 import Qwen3ForCausalLM
    from inference_systems_b200.models.qwen3_5 import Qwen3_5ForCausalLM

    assert isinstance(create_model(*normalize_hf_config(_qwen3())), Qwen3ForCausalLM)
    m = create_model(*normalize_hf_config(_qwen35_wrapper()))
    assert isinstance(m, Qwen3_5ForCausalLM)
    assert [layer.is_linear for layer in m.layers] == [True, True, True, False]


def test_decode_metadata_fast_path_matches_the_general_packer():
    """The column-wise decode packer produces exactly the general packer's int32 array, layout
    and metadata (with graph padding, scratch-slot rows and mixed temperatures)."""
    import numpy as np

    from inference_systems_b200.engine.model_runner import ModelRunner

    seqs = []
    for i in range(37):
        s = Sequence(list(range(200 + 7 * i)), SamplingParams(temperature=0.1 * (i % 3), max_tokens=8))
        s.block_table = [i * 4 + j for j in range(-(-len(s) // 256))]
        s.state_slot = i if i % 5 else None
        s.is_prefill = False
        seqs.append(s)
    runner = SimpleNamespace(block_size=256, state_manager=SimpleNamespace(scratch_slot_id=99), max_blocks_per_seq=8,
                             config=SimpleNamespace(seed=3), sample_step=7)
    for pad in (None, 48):
        a = ModelRunner._pack_general(runner, seqs, False, pad)
        b = ModelRunner._pack_decode(runner, seqs, pad)
        assert np.array_equal(a[0], b[0]) and a[1] == b[1] and a[2] == b[2]
