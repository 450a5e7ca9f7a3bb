"""Failure detection without any GPU fault: host-side injected failures on gloo ranks."""

import os
import tempfile
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from afd_plugin_b200.runtime.launcher import LocalAFDSpec, launch_local
from afd_plugin_b200.runtime.watchdog import HeartbeatWatchdog


def _prompts(n=3, length=12):
    g = torch.Generator().manual_seed(0)
    return torch.randint(0, 1024, (n, length), generator=g).tolist()


def test_attention_rank_exception_surfaces_everywhere():
    spec = LocalAFDSpec(afd={"num_attention_ranks": 1, "num_ffn_ranks": 1}, prompts=_prompts(), max_tokens=8,
                        timeout_s=8, fault={"rank": 1, "kind": "raise", "at_step": 2})
    t0 = time.time()
    res = launch_local(spec, join_timeout_s=60)
    assert time.time() - t0 < 60
    assert "injected fault" in res[1]["error"]
    assert "error" in res[0]  # the FFN rank learns of it (timeout / closed peer), it does not hang


def test_ffn_rank_exit_surfaces_on_attention_side():
    spec = LocalAFDSpec(afd={"num_attention_ranks": 1, "num_ffn_ranks": 1}, prompts=_prompts(), max_tokens=4,
                        timeout_s=8, fault={"rank": 0, "kind": "exit_before_serve"})
    res = launch_local(spec, join_timeout_s=60)
    assert "error" in res[1]
    assert "error" in res[0]


def test_ffn_loop_error_reraised():
    from afd_plugin_b200.runtime.workers import AFDFFNWorker

    class Runner:
        def serve(self, stop=None, max_steps=None):
            raise ValueError("boom")

    w = AFDFFNWorker.__new__(AFDFFNWorker)
    w.device = torch.device("cpu")
    w.model_runner = Runner()
    w._thread = None
    w._stop = None
    w._error = None
    w.start_ffn_server_loop()
    w._thread.join(5)
    with pytest.raises(RuntimeError, match="FFN worker loop failed"):
        w.raise_ffn_loop_error_if_any()
    w.raise_ffn_loop_error_if_any()  # cleared after raising
    with pytest.raises(RuntimeError):
        w.execute_model()


def _hb_rank(rank, world, path, q):
    store = dist.FileStore(path, world)
    store.set_timeout(timedelta(seconds=20))
    # start together (process start-up times differ by seconds under load)
    store.add("ready", 1)
    while int(store.add("ready", 0)) < world:
        time.sleep(0.01)
    wd = HeartbeatWatchdog(store, rank, world, period_s=0.05, timeout_s=0.5).start()
    if rank == 1:
        time.sleep(0.3)
        wd.stop(clean=False)  # rank 1 "dies": stops beating but keeps the process alive for the store
        time.sleep(3.0)
        q.put((rank, []))
        return
    time.sleep(2.0)
    dead = sorted(wd.dead_peers())
    wd.stop()
    q.put((rank, dead))
    time.sleep(0.8)


def test_heartbeat_watchdog_detects_silent_peer():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    path = os.path.join(tempfile.mkdtemp(prefix="afd_hb_"), "store")
    ps = [ctx.Process(target=_hb_rank, args=(r, 3, path, q)) for r in range(3)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(30)
    got = dict(q.get(timeout=5) for _ in range(3))
    assert got[0] == [1] and got[2] == [1]


def test_health_check_runs_before_every_step_on_both_roles():
    """A peer that stopped heartbeating fails the next step on the host, before any wait on it."""
    from types import SimpleNamespace

    from afd_plugin_b200.engine_config import EngineConfig, ModelConfig
    from afd_plugin_b200.models import build_model, get_preset
    from afd_plugin_b200.runtime.engine import LLMEngine
    from afd_plugin_b200.runtime.ffn_runner import FFNModelRunner

    def dead():
        raise RuntimeError("AFD peer rank(s) [0] stopped heartbeating")

    arch = get_preset("tiny-dsv2")
    eng = LLMEngine(EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=64),
                                 max_num_seqs=2), build_model(arch, role="colocated", dtype=torch.float32))
    eng.add_request([1, 2, 3], 2)
    eng.health_check = dead
    with pytest.raises(RuntimeError, match="stopped heartbeating"):
        eng.step()
    assert eng.waiting  # nothing ran

    cp = SimpleNamespace(recv_dp_metadata_list=lambda: pytest.fail("must not wait for a payload"))
    conn = SimpleNamespace(control_plane=cp, attn_size=1, ffn_size=1)
    model = SimpleNamespace(device=torch.device("cpu"))
    cfg = SimpleNamespace(model_config=SimpleNamespace(enforce_eager=True))
    runner = FFNModelRunner(model, conn, cfg)
    runner.health_check = dead
    with pytest.raises(RuntimeError, match="stopped heartbeating"):
        runner.serve(max_steps=1)


def test_heartbeat_quiet_on_clean_runs(monkeypatch):
    monkeypatch.setenv("AFD_HEARTBEAT_TIMEOUT_S", "1.0")
    spec = LocalAFDSpec(afd={"num_attention_ranks": 2, "num_ffn_ranks": 1}, prompts=_prompts(n=4), max_tokens=6,
                        timeout_s=30)
    res = launch_local(spec, join_timeout_s=90)
    assert not any("error" in v for v in res.values()), res


@pytest.mark.parametrize("A", [1, 2])
def test_attention_rank_exception_with_async_scheduling(A):
    """A step launched ahead of its predecessor's read-back is in flight when the Attention rank raises:
    the error still surfaces on every rank within the process-group timeout (no hang)."""
    spec = LocalAFDSpec(afd={"num_attention_ranks": A, "num_ffn_ranks": 1}, prompts=_prompts(n=4), max_tokens=8,
                        timeout_s=8, fault={"rank": 1, "kind": "raise", "at_step": 3}, async_scheduling=True)
    t0 = time.time()
    res = launch_local(spec, join_timeout_s=60)
    assert time.time() - t0 < 60
    assert "injected fault" in res[1]["error"]
    assert all("error" in v for v in res.values())
