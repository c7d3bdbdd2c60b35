"""All-rank hybrid-prefix transactions under injected failures (gloo ranks on CPU).

Parity with the reference's fault-injection tests
(``tests/test_hybrid_prefix_transaction.py``): failures are made on the host
(an exception raised by one rank's pool, a diverging slot id, a rank that
exits before a collective); no GPU is involved.  Every rank must end in the
same state, only rank 0 raises, and a dead peer surfaces as an error within
the process-group timeout instead of a hang.
"""

import json
import os
import socket
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from inference_systems_b200.engine.state_pool import (
    HybridPrefixCheckpointPool,
    HybridStateManager,
    transactional_capture_prefix_checkpoint,
    transactional_restore_prefix_checkpoint,
)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _pool(seed: int):
    sm = HybridStateManager(max_num_seqs=2, num_linear_layers=2, num_value_heads=2, key_head_dim=8, value_head_dim=8,
                            conv_dim=12, conv_kernel_size=4, conv_dtype=torch.float32, device=torch.device("cpu"))
    slot = sm.allocate()
    g = torch.Generator().manual_seed(seed)
    sm.recurrent_states[:, slot] = torch.randn(sm.recurrent_states[:, slot].shape, generator=g)
    sm.conv_states[:, slot] = torch.randn(sm.conv_states[:, slot].shape, generator=g)
    pool = HybridPrefixCheckpointPool(sm, 4 * 10**6, checkpoint_dtype="fp32")
    return sm, pool, slot


def _worker(rank: int, world: int, port: int, scenario: str, out_dir: str) -> None:
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=5))
    sm, pool, slot = _pool(100 + rank)
    res = {"rank": rank}
    try:
        if scenario == "capture_fails_on_rank1":
            if rank == 1:
                def boom(_slot):
                    raise RuntimeError("injected capture failure")
                pool.capture = boom
            try:
                res["slot"] = transactional_capture_prefix_checkpoint(pool, slot)
            except RuntimeError as e:
                res["raised"] = str(e)
            res["used"] = sorted(pool.used_checkpoint_slots)
        elif scenario == "slot_ids_diverge":
            if rank == 1:
                pool.slots.take()  # rank 1's next capture gets a different slot id
            try:
                res["slot"] = transactional_capture_prefix_checkpoint(pool, slot)
            except RuntimeError as e:
                res["raised"] = str(e)
            res["used"] = sorted(pool.used_checkpoint_slots)
            res["free"] = pool.free_checkpoint_slots
            res["capacity"] = pool.capacity
        elif scenario == "restore_fails_on_rank0":
            ck = transactional_capture_prefix_checkpoint(pool, slot)
            before = sm.recurrent_states[:, slot].clone()
            sm.recurrent_states[:, slot].add_(1.0)  # the request moved on after the capture
            moved = sm.recurrent_states[:, slot].clone()
            if rank == 0:
                def boom(_ck, _slot):
                    sm.recurrent_states[:, _slot].zero_()  # a partial write, then the failure
                    raise RuntimeError("injected restore failure")
                pool.restore = boom
            try:
                transactional_restore_prefix_checkpoint(pool, ck, slot)
            except RuntimeError as e:
                res["raised"] = str(e)
            res["rolled_back"] = bool(torch.equal(sm.recurrent_states[:, slot], moved))
            res["restored"] = bool(torch.equal(sm.recurrent_states[:, slot], before))
        elif scenario == "dead_peer":
            if rank == 1:
                os._exit(0)  # leaves between steps: no collective of its own in flight
            t0 = time.time()
            try:
                t = torch.ones(1)
                dist.all_reduce(t)
                res["error"] = None
            except Exception as e:  # noqa: BLE001 - any backend error is the detection signal
                res["error"] = type(e).__name__
            res["seconds"] = time.time() - t0
    finally:
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(res, f)
        if scenario != "dead_peer":
            dist.destroy_process_group()


def _run(scenario, tmp_path, world=2):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            pytest.fail(f"rank process hung in scenario {scenario}")
    out = {}
    for r in range(world):
        path = tmp_path / f"rank{r}.json"
        if path.exists():
            out[r] = json.loads(path.read_text())
    return out


def test_capture_failure_on_one_rank_rolls_back_everywhere(tmp_path):
    out = _run("capture_fails_on_rank1", tmp_path)
    assert "rolled back" in out[0]["raised"]
    assert out[1].get("slot") == -1 and "raised" not in out[1]   # only rank 0 raises
    assert out[0]["used"] == [] and out[1]["used"] == []


def test_diverging_slot_ids_roll_back(tmp_path):
    out = _run("slot_ids_diverge", tmp_path)
    assert "diverged" in out[0]["raised"]
    assert out[1].get("slot") == -1
    assert out[0]["used"] == [] and out[1]["used"] == [0]  # rank 1 keeps only the slot taken outside
    assert out[0]["free"] == out[0]["capacity"]
    assert out[1]["free"] == out[1]["capacity"] - 1  # only the slot taken before the transaction is gone


def test_restore_failure_restores_backup_on_all_ranks(tmp_path):
    out = _run("restore_fails_on_rank0", tmp_path)
    assert "rolled back" in out[0]["raised"]
    assert "raised" not in out[1]
    assert out[0]["rolled_back"] and out[1]["rolled_back"]
    assert not out[0]["restored"] and not out[1]["restored"]


def test_dead_peer_is_detected_not_hung(tmp_path):
    out = _run("dead_peer", tmp_path)
    assert out[0]["error"] is not None
    assert out[0]["seconds"] < 30
