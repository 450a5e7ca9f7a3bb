"""End-to-end runner: scenario table, command lines, agreement gate, process-group teardown (CPU)."""

from __future__ import annotations

import json
import sys
import time

import pytest

from afd_plugin_b200.e2e import runner
from afd_plugin_b200.e2e.process_utils import group_alive, start_server, stop_server, wait_for_health
from afd_plugin_b200.e2e.scenarios import FUSED, NCCL, SCENARIOS, server_command


def test_scenario_table_covers_reference_topologies():
    for name, (graph, dbo, a, f) in {
        "afd-eager-2a1f": (False, False, 2, 1), "afd-graph-2a1f": (True, False, 2, 1),
        "afd-graph-dbo-2a1f": (True, True, 2, 1), "afd-eager-2a2f": (False, False, 2, 2),
        "afd-graph-2a2f": (True, False, 2, 2), "afd-graph-dbo-2a2f": (True, True, 2, 2),
    }.items():
        s = SCENARIOS[name]
        assert (s.graph, s.dbo, s.attention_ranks, s.ffn_ranks, s.connector) == (graph, dbo, a, f, NCCL)
    assert SCENARIOS["baseline-graph"].world_size == 1
    assert SCENARIOS["afd-fused-graph-6a2f"].world_size == 8 and SCENARIOS["afd-fused-graph-6a2f"].needs_cuda


def test_server_commands():
    base = server_command(SCENARIOS["baseline-graph"], python="py", preset="p", port=9, master_port=10,
                          max_num_seqs=4, capture_size=8)
    assert base[:3] == ["py", "-m", "afd_plugin_b200.serving"]
    assert base[base.index("--capture-sizes") + 1] == "4" and "--afd" not in base and "--eager" not in base
    afd = server_command(SCENARIOS["afd-graph-dbo-2a2f"], python="py", preset="p", port=9, master_port=10,
                         checkpoint="/ckpt")
    assert afd[1:4] == ["-m", "torch.distributed.run", "--nnodes"]
    assert afd[afd.index("--nproc-per-node") + 1] == "4" and afd[afd.index("--master-addr") + 1] == "127.0.0.1"
    assert "--dbo" in afd and afd[afd.index("--checkpoint") + 1] == "/ckpt"
    cfg = json.loads(afd[afd.index("--afd") + 1])
    assert cfg == {"num_attention_ranks": 2, "num_ffn_ranks": 2, "connector": NCCL}
    fused = server_command(SCENARIOS["afd-fused-graph-2a2f"], python="py", preset="p", port=9, master_port=10,
                           connector_extra={"fp8_dispatch": True})
    cfg = json.loads(fused[fused.index("--afd") + 1])
    assert cfg["connector"] == FUSED and cfg["connector_extra_config"] == {"fp8_dispatch": True}
    eager = server_command(SCENARIOS["afd-eager-2a1f"], python="py", preset="p", port=9, master_port=10)
    assert "--eager" in eager and "--capture-sizes" not in eager and "--tp" not in eager
    tp = server_command(SCENARIOS["afd-eager-tp2-1f"], python="py", preset="p", port=9, master_port=10)
    assert tp[tp.index("--tp") + 1] == "2" and tp[tp.index("--nproc-per-node") + 1] == "3"


def test_compare_and_gate():
    ref = [[1, 2, 3], [4, 5, 6], [7, 8, 9], [1, 1, 1]]
    out = [[1, 2, 3], [4, 5, 0], [0, 8, 9], [1, 1, 1]]
    m = runner.compare(out, ref)
    assert m["exact_match"] == 0.5 and m["first_token_match"] == 0.75
    assert m["mean_prefix_agreement"] == pytest.approx((1 + 2 / 3 + 0 + 1) / 4)
    assert runner.gate(m, min_exact=0.5, min_first=0.75) == []
    assert len(runner.gate(m, min_exact=0.9, min_first=0.9)) == 2
    with pytest.raises(ValueError):
        runner.compare(out[:2], ref)
    p1 = runner.make_prompts(5, 100, seed=3)
    assert p1 == runner.make_prompts(5, 100, seed=3) and all(0 <= t < 100 for p in p1 for t in p)


def _py(code: str) -> list[str]:
    return [sys.executable, "-c", code]


def test_stop_escalates_to_kill_and_reaps_the_group(tmp_path):
    # the leader ignores SIGTERM and has a child that also ignores it
    code = ("import signal, subprocess, sys, time; signal.signal(signal.SIGTERM, signal.SIG_IGN); "
            "subprocess.Popen([sys.executable, '-c', 'import signal, time; "
            "signal.signal(signal.SIGTERM, signal.SIG_IGN); time.sleep(120)']); time.sleep(120)")
    srv = start_server(_py(code), log_path=str(tmp_path / "log.txt"))
    time.sleep(1.0)
    assert group_alive(srv.pgid)
    assert stop_server(srv, term_timeout_s=1.0, kill_timeout_s=10.0) == "killed"
    assert not group_alive(srv.pgid)


def test_stop_terminates_cooperative_group_and_reports_exited():
    srv = start_server(_py("import time; time.sleep(120)"))
    time.sleep(0.3)
    assert stop_server(srv, term_timeout_s=10.0) == "terminated"
    done = start_server(_py("pass"))
    done.proc.wait(30)
    time.sleep(0.2)
    assert stop_server(done) == "exited"


def test_wait_for_health_reports_an_early_exit(tmp_path):
    srv = start_server(_py("print('boom'); raise SystemExit(3)"), log_path=str(tmp_path / "log.txt"))
    with pytest.raises(RuntimeError, match="code 3") as ei:
        wait_for_health(srv, "http://127.0.0.1:9", timeout_s=30, interval_s=0.05)
    assert "boom" in str(ei.value)
    stop_server(srv)


def test_runner_cpu_baseline_vs_afd(tmp_path):
    """Colocated engine, a 2A1F NCCL-connector deployment and attention TP2 (gloo on CPU) serve identical tokens."""
    out = tmp_path / "e2e.json"
    rc = runner.main(["--scenarios", "baseline-eager,afd-eager-2a1f,afd-eager-tp2-1f", "--preset", "tiny-dsv2",
                      "--dtype", "float32", "--device", "cpu", "--num-prompts", "4", "--max-tokens", "4", "--max-model-len", "128",
                      "--max-num-seqs", "4", "--min-exact-match", "1.0", "--startup-timeout", "240",
                      "--log-dir", str(tmp_path / "logs"), "--output", str(out)])
    assert rc == 0
    res = json.loads(out.read_text())["results"]
    for r in res[1:]:
        assert r["agreement"]["exact_match"] == 1.0 and r["gate"] == "pass", r["scenario"]
    assert all(t in ("terminated", "killed", "exited") for r in res for t in r["teardown"].split(","))


def test_scenario_restarts_on_a_taken_port(monkeypatch, tmp_path):
    calls = []

    def once(scn, args, prompts, *, log_dir):
        calls.append(1)
        if len(calls) < 3:
            raise RuntimeError("server exited with code 1 before it was healthy:\n[Errno 98] address already in use")
        return {"scenario": scn.name, "outputs": []}

    monkeypatch.setattr(runner, "_run_scenario_once", once)
    res = runner.run_scenario(SCENARIOS["afd-eager-2a1f"], None, [], log_dir=str(tmp_path))
    assert res["scenario"] == "afd-eager-2a1f" and len(calls) == 3
    calls.clear()

    def broken(scn, args, prompts, *, log_dir):
        calls.append(1)
        raise RuntimeError("server exited with code 1 before it was healthy:\nValueError: bad config")

    monkeypatch.setattr(runner, "_run_scenario_once", broken)
    with pytest.raises(RuntimeError, match="bad config"):
        runner.run_scenario(SCENARIOS["afd-eager-2a1f"], None, [], log_dir=str(tmp_path))
    assert len(calls) == 1


def test_pd_scenario_prefill_colocated_decode_afd(tmp_path):
    """Prefill on a colocated server, KV rows over HTTP, decode on a 2A1F AFD deployment behind the proxy."""
    scn = SCENARIOS["pd-baseline-to-afd-eager-2a1f"]
    assert scn.prefill.baseline and scn.world_size == 3 and scn.total_devices == 4
    out = tmp_path / "pd.json"
    rc = runner.main(["--scenarios", "baseline-eager,pd-baseline-to-afd-eager-2a1f", "--preset", "tiny-dsv2",
                      "--dtype", "float32", "--device", "cpu", "--num-prompts", "4", "--max-tokens", "4",
                      "--max-model-len", "128", "--max-num-seqs", "4", "--min-exact-match", "1.0",
                      "--startup-timeout", "240", "--log-dir", str(tmp_path / "logs"), "--output", str(out)])
    assert rc == 0
    res = json.loads(out.read_text())["results"]
    assert res[1]["agreement"]["exact_match"] == 1.0
    assert len(res[1]["teardown"].split(",")) == 3


def test_gsm8k_parsing_and_prompt():
    from afd_plugin_b200.e2e import gsm8k

    assert gsm8k.reference_answer("so 3 + 4 = 7.\n#### 7") == "7"
    assert gsm8k.reference_answer("#### 1,234") == "1234"
    assert gsm8k.extract_strict("The answer is #### $18.00") == "18"
    assert gsm8k.extract_strict("no marker 5") is None
    assert gsm8k.extract_flexible("first 3 then 4.50.") == "4.5"
    p = gsm8k.build_prompt([{"question": "1+1?", "answer": "#### 2"}], "2+2?")
    assert p == "Question: 1+1?\nAnswer: #### 2\n\nQuestion: 2+2?\nAnswer:"
    assert gsm8k._truncate(" #### 4\n\nQuestion: next") == " #### 4"


def test_gsm8k_against_a_fake_server(tmp_path):
    import threading

    import uvicorn
    from fastapi import FastAPI

    from afd_plugin_b200.e2e import gsm8k
    from afd_plugin_b200.runtime.launcher import free_port

    data = [{"question": f"What is {i} + {i}?", "answer": f"{i} + {i} = {2 * i}\n#### {2 * i}"} for i in range(12)]
    path = tmp_path / "gsm8k.jsonl"
    path.write_text("\n".join(json.dumps(d) for d in data))
    app = FastAPI()

    @app.post("/v1/completions")
    def complete(body: dict):
        q = body["prompt"].rsplit("Question: ", 1)[1]
        i = int(q.split()[2])
        text = f" {i} + {i} = {2 * i}\n#### {2 * i}\n\nQuestion: more" if i % 2 == 0 else f" it is {2 * i + 1}"
        return {"choices": [{"text": text, "token_ids": []}]}

    port = free_port()
    srv = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
    threading.Thread(target=srv.run, daemon=True).start()
    time.sleep(1.0)
    try:
        rc = gsm8k.main(["--url", f"http://127.0.0.1:{port}", "--data", str(path), "--shots", "2", "--limit", "8",
                         "--threshold", "0.4", "--output", str(tmp_path / "out.json")])
        res = json.loads((tmp_path / "out.json").read_text())
        # questions 2..9: the even ones are answered right
        assert res["n"] == 8 and res["exact_match_strict"] == 0.5 and res["exact_match_flexible"] == 0.5
        assert rc == 0 and res["gate"] == "pass"
    finally:
        srv.should_exit = True


def test_roles_launched_separately_join_one_afd_world(tmp_path):
    """An FFN server and an Attention server started on their own (the reference's deployment) form one world."""
    import os

    import requests

    from afd_plugin_b200.runtime.launcher import free_port

    afd_port, http = free_port(), free_port()
    base = {"num_attention_ranks": 1, "num_ffn_ranks": 1, "host": "127.0.0.1", "port": afd_port}
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, RANK="0", WORLD_SIZE="1", LOCAL_RANK="0", CUDA_VISIBLE_DEVICES="",
               PYTHONPATH=root + os.pathsep + os.environ.get("PYTHONPATH", ""))
    common = [sys.executable, "-m", "afd_plugin_b200.serving", "--preset", "tiny-dsv2", "--dtype", "float32",
              "--eager", "--max-model-len", "128", "--max-num-seqs", "4"]
    ffn_http = free_port()
    ffn = start_server(common + ["--port", str(ffn_http), "--afd", json.dumps(dict(base, role="ffn"))],
                       env=env, log_path=str(tmp_path / "ffn.log"))
    attn = start_server(common + ["--port", str(http), "--afd", json.dumps(dict(base, role="attention"))],
                        env=env, log_path=str(tmp_path / "attn.log"))
    try:
        url = f"http://127.0.0.1:{http}"
        wait_for_health(attn, url, timeout_s=240)
        prompts = runner.make_prompts(3, 1024, seed=2, min_len=6, max_len=12)
        got = runner.send_requests(url, prompts, 4, concurrency=3)
        import torch

        from afd_plugin_b200.engine_config import EngineConfig, ModelConfig
        from afd_plugin_b200.models import build_model, get_preset
        from afd_plugin_b200.runtime.engine import LLMEngine

        arch = get_preset("tiny-dsv2")
        eng = LLMEngine(EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=128),
                                     max_num_seqs=4),
                        build_model(arch, role="colocated", dtype=torch.float32, seed=0, max_positions=128))
        assert got == eng.generate(prompts, 4)
        assert requests.get(url + "/health", timeout=5).status_code == 200
        ffn_health = requests.get(f"http://127.0.0.1:{ffn_http}/health", timeout=5)
        assert ffn_health.status_code == 200 and ffn_health.json()["role"] == "ffn"
    finally:
        stop_server(attn)
        stop_server(ffn)


def test_async_scheduling_scenarios():
    """The async-scheduling rows pass the server flag; the others do not."""
    for name in ("baseline-graph-async", "afd-graph-2a2f-async", "afd-fused-graph-2a2f-async"):
        cmd = server_command(SCENARIOS[name], python="py", preset="p", port=9, master_port=10)
        assert "--async-scheduling" in cmd and SCENARIOS[name].async_scheduling
    plain = server_command(SCENARIOS["afd-graph-2a2f"], python="py", preset="p", port=9, master_port=10)
    assert "--async-scheduling" not in plain
