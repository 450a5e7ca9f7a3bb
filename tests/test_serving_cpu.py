"""HTTP completions server over a colocated engine (CPU)."""

import os
import tempfile
import threading
import time
from concurrent.futures import ThreadPoolExecutor

import pytest
import requests
import torch

from afd_plugin_b200.engine_config import EngineConfig, ModelConfig
from afd_plugin_b200.models import build_model, get_preset
from afd_plugin_b200.runtime.engine import LLMEngine
from afd_plugin_b200.runtime.launcher import free_port
from afd_plugin_b200.serving import EngineLoop, build_app, byte_detokenize, byte_tokenize


def _engine(async_scheduling=False):
    arch = get_preset("tiny-dsv2")
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=96), max_num_seqs=4,
                      async_scheduling=async_scheduling)
    return LLMEngine(ec, build_model(arch, role="colocated", dtype=torch.float32, seed=0, max_positions=96))


@pytest.fixture(params=[False, True], ids=["sync", "async"])
def any_server(request):
    yield from _serve_engine(request.param)


@pytest.fixture
def server():
    yield from _serve_engine(False)


def _serve_engine(async_scheduling):
    import uvicorn

    loop = EngineLoop(_engine(async_scheduling)).start()
    port = free_port()
    srv = uvicorn.Server(uvicorn.Config(build_app(loop), host="127.0.0.1", port=port, log_level="warning"))
    t = threading.Thread(target=srv.run, daemon=True)
    t.start()
    url = f"http://127.0.0.1:{port}"
    for _ in range(200):
        try:
            if requests.get(url + "/health", timeout=1).ok:
                break
        except requests.ConnectionError:
            time.sleep(0.05)
    yield url, loop
    srv.should_exit = True
    t.join(10)
    loop.stop()


def test_completions_match_engine_generate(any_server):
    url, loop = any_server
    prompts = [[5, 9, 100, 7, 3, 1], [42] * 10, [1, 2, 3], [900, 800, 700, 600]]
    want = _engine().generate(prompts, 6)
    with ThreadPoolExecutor(4) as ex:  # concurrent requests are batched by the engine loop
        resp = list(ex.map(lambda p: requests.post(url + "/v1/completions", json={"prompt": p, "max_tokens": 6},
                                                   timeout=60).json(), prompts))
    assert [r["choices"][0]["token_ids"] for r in resp] == want
    assert resp[0]["usage"] == {"prompt_tokens": 6, "completion_tokens": 6, "total_tokens": 12}
    m = requests.get(url + "/metrics", timeout=5).json()
    assert m["completed"] == 4 and m["generated_tokens"] == 24
    prom = requests.get(url + "/metrics/prometheus", timeout=5)
    assert prom.status_code == 200 and 'afd_completed_total{model="afd-b200"} 4.0' in prom.text
    assert "# TYPE afd_generated_tokens_total counter" in prom.text
    models = requests.get(url + "/v1/models", timeout=5).json()
    assert models["data"][0]["id"] == "afd-b200" and models["data"][0]["max_model_len"] == 96
    assert m["ttft_count"] == 4 and m["tpot_count"] == 4
    assert 0 < m["mean_ttft_s"] < 60 and 0 < m["mean_tpot_s"] < 60
    assert (loop.engine.num_async_steps > 0) == loop.engine.async_scheduling
    assert 0 < m["async_steps"] <= loop.engine.num_async_steps if loop.engine.async_scheduling else m["async_steps"] == 0


def test_text_prompt_and_validation(server):
    url, _ = server
    r = requests.post(url + "/v1/completions", json={"prompt": "hello", "max_tokens": 3}, timeout=60).json()
    assert len(r["choices"][0]["token_ids"]) == 3 and r["usage"]["prompt_tokens"] == 5
    assert requests.post(url + "/v1/completions", json={"prompt": [5000], "max_tokens": 3}, timeout=10).status_code == 400
    assert requests.post(url + "/v1/completions", json={"prompt": [1] * 95, "max_tokens": 8},
                         timeout=10).status_code == 400
    assert byte_detokenize(byte_tokenize("héllo", 1024)) == "héllo"


def _afd_serving_rank(world_rank, rendezvous, prompts, q):
    import os
    from datetime import timedelta

    import torch.distributed as dist

    from afd_plugin_b200.runtime.launcher import LocalAFDSpec, build_engine_config
    from afd_plugin_b200.parallel.topology import role_of_world_rank

    dist.init_process_group("gloo", init_method=rendezvous, rank=world_rank, world_size=3,
                            timeout=timedelta(seconds=60))
    role, role_rank = role_of_world_rank(world_rank, attention_size=2, ffn_size=1)
    spec = LocalAFDSpec(preset="tiny-dsv2", afd={"num_attention_ranks": 2, "num_ffn_ranks": 1, "role": role})
    ec = build_engine_config(spec)
    if role == "ffn":
        from afd_plugin_b200.runtime.workers import AFDFFNWorker

        w = AFDFFNWorker(ec)
        w.run_ffn_server_loop()
        w.shutdown()
        q.put((world_rank, None))
        return
    from afd_plugin_b200.runtime.workers import AFDAttentionWorker

    w = AFDAttentionWorker(ec)
    loop = EngineLoop(w.engine, group=w.groups.attention_group, world=2, rank=role_rank).start()
    outs = None
    if role_rank == 0:  # only the HTTP rank gets requests; rank 1 steps along with placeholder rows
        futs = [loop.submit(p, 5) for p in prompts]
        outs = [f.result(timeout=120) for f in futs]
        loop.stop()
    else:
        loop.join()  # ends when rank 0 stops
    w.shutdown()
    q.put((world_rank, outs))


def test_engine_loop_lockstep_across_attention_ranks():
    import torch.multiprocessing as mp

    prompts = [[5, 9, 100, 7, 3, 1], [42] * 10, [1, 2, 3]]
    want = _engine().generate(prompts, 5)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    rendezvous = "file://" + os.path.join(tempfile.mkdtemp(prefix="afd_rdv_"), "store")
    ps = [ctx.Process(target=_afd_serving_rank, args=(r, rendezvous, prompts, q)) for r in range(3)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=180) for _ in range(3))
    for p in ps:
        p.join(30)
    assert got[1] == want


def test_proxy_balances_over_two_servers():
    import uvicorn

    from afd_plugin_b200.serving.proxy import build_proxy_app

    servers, loops, urls = [], [], []
    for _ in range(2):
        loop = EngineLoop(_engine()).start()
        port = free_port()
        srv = uvicorn.Server(uvicorn.Config(build_app(loop), host="127.0.0.1", port=port, log_level="warning"))
        threading.Thread(target=srv.run, daemon=True).start()
        servers.append(srv)
        loops.append(loop)
        urls.append(f"http://127.0.0.1:{port}")
    pport = free_port()
    proxy = uvicorn.Server(uvicorn.Config(build_proxy_app(urls), host="127.0.0.1", port=pport, log_level="warning"))
    threading.Thread(target=proxy.run, daemon=True).start()
    purl = f"http://127.0.0.1:{pport}"
    for _ in range(200):
        try:
            if requests.get(purl + "/health", timeout=2).ok:
                break
        except requests.ConnectionError:
            time.sleep(0.05)
    prompts = [[5, 9, 100, 7], [42] * 6, [1, 2, 3], [900, 800]]
    want = _engine().generate(prompts, 4)
    with ThreadPoolExecutor(4) as ex:
        got = list(ex.map(lambda p: requests.post(purl + "/v1/completions", json={"prompt": p, "max_tokens": 4},
                                                  timeout=60).json()["choices"][0]["token_ids"], prompts))
    assert got == want
    h = requests.get(purl + "/health", timeout=10).json()
    assert all(h["backends"].values()) and sum(h["served"].values()) == 4 and min(h["served"].values()) >= 1
    for s in servers + [proxy]:
        s.should_exit = True
    for lp in loops:
        lp.stop()


def _serve(app):
    import uvicorn

    port = free_port()
    srv = uvicorn.Server(uvicorn.Config(app(port), host="127.0.0.1", port=port, log_level="warning"))
    threading.Thread(target=srv.run, daemon=True).start()
    url = f"http://127.0.0.1:{port}"
    for _ in range(400):
        try:
            if requests.get(url + "/health", timeout=2).ok:
                break
        except requests.ConnectionError:
            time.sleep(0.05)
    return srv, url


def test_disaggregated_prefill_decode_through_proxy():
    """Prefill server -> KV rows over HTTP -> decode server; tokens equal one engine's."""
    from afd_plugin_b200.serving.proxy import build_proxy_app

    pre_loop, dec_loop = EngineLoop(_engine()).start(), EngineLoop(_engine()).start()
    pre, pre_url = _serve(lambda port: build_app(pre_loop, advertise_port=port))
    dec, dec_url = _serve(lambda port: build_app(dec_loop, advertise_port=port))
    proxy, purl = _serve(lambda port: build_proxy_app(prefill=[pre_url], decode=[dec_url]))
    try:
        prompts = [[5, 9, 100, 7], [42] * 6, [1, 2, 3], [900, 800]]
        want = _engine().generate(prompts, 5)
        with ThreadPoolExecutor(4) as ex:
            got = list(ex.map(lambda p: requests.post(purl + "/v1/completions", json={"prompt": p, "max_tokens": 5},
                                                      timeout=120).json()["choices"][0]["token_ids"], prompts))
        assert got == want
        h = requests.get(purl + "/health", timeout=10).json()
        assert sum(h["prefill"]["served"].values()) == 4 and sum(h["decode"]["served"].values()) == 4
        # every held row was fetched: the prefill engine holds nothing
        assert pre_loop.call(lambda eng: len(eng.held)).result(timeout=30) == 0
        assert dec_loop.stats["completed"] == 4 and pre_loop.stats["completed"] == 4

        # a prefill leg answers with where to fetch the rows; a second fetch is a 404
        r = requests.post(pre_url + "/v1/completions", json={"prompt": [3, 4, 5], "max_tokens": 1,
                                                              "kv_transfer_params": {"do_remote_decode": True}},
                          timeout=60).json()
        params = r["kv_transfer_params"]
        assert params["do_remote_prefill"] and params["remote_port"] == int(pre_url.rsplit(":", 1)[1])
        bad = requests.post(dec_url + "/v1/completions", json={"prompt": [3, 4, 6], "max_tokens": 2,
                                                                "kv_transfer_params": params}, timeout=60)
        assert bad.status_code == 400 and "different prompt" in bad.json()["detail"]
        again = requests.post(dec_url + "/v1/completions", json={"prompt": [3, 4, 5], "max_tokens": 2,
                                                                  "kv_transfer_params": params}, timeout=60)
        assert again.status_code == 502
        assert requests.delete(f"{pre_url}/v1/kv/{params['remote_request_id']}", timeout=10).json() == \
            {"released": False}
    finally:
        for s in (pre, dec, proxy):
            s.should_exit = True
        pre_loop.stop()
        dec_loop.stop()


def _stream_tokens(url, body):
    import json as _json

    toks, usage, events = [], None, 0
    with requests.post(url + "/v1/completions", json=dict(body, stream=True), stream=True, timeout=60) as r:
        assert r.status_code == 200 and r.headers["content-type"].startswith("text/event-stream")
        for line in r.iter_lines():
            if not line or not line.startswith(b"data: "):
                continue
            data = line[len(b"data: "):]
            if data == b"[DONE]":
                break
            events += 1
            msg = _json.loads(data)
            toks += msg["choices"][0]["token_ids"]
            usage = msg.get("usage", usage)
    return toks, usage, events


def test_streaming_completions(any_server):
    url, _ = any_server
    prompt = [5, 9, 100, 7, 3, 1]
    want = _engine().generate([prompt], 6)[0]
    toks, usage, events = _stream_tokens(url, {"prompt": prompt, "max_tokens": 6})
    assert toks == want and events == 7  # one event per token plus the final one with usage
    assert usage == {"prompt_tokens": 6, "completion_tokens": 6, "total_tokens": 12}
    r = requests.post(url + "/v1/completions", json={"prompt": [1] * 95, "max_tokens": 8, "stream": True}, timeout=10)
    assert r.status_code == 400


def test_streaming_through_proxies_and_serve_bench():
    from afd_plugin_b200.bench import serve_bench
    from afd_plugin_b200.serving.proxy import build_proxy_app

    loops = [EngineLoop(_engine()).start() for _ in range(3)]
    a, a_url = _serve(lambda port: build_app(loops[0], advertise_port=port))
    pre, pre_url = _serve(lambda port: build_app(loops[1], advertise_port=port))
    dec, dec_url = _serve(lambda port: build_app(loops[2], advertise_port=port))
    plain, plain_url = _serve(lambda port: build_proxy_app([a_url]))
    pd, pd_url = _serve(lambda port: build_proxy_app(prefill=[pre_url], decode=[dec_url]))
    try:
        prompt = [42] * 7
        want = _engine().generate([prompt], 5)[0]
        assert _stream_tokens(plain_url, {"prompt": prompt, "max_tokens": 5})[0] == want
        assert _stream_tokens(pd_url, {"prompt": prompt, "max_tokens": 5})[0] == want
        summary = serve_bench.main(["--url", pd_url, "--num-prompts", "6", "--input-len", "9", "--output-len", "4",
                                    "--request-rate", "inf", "--max-concurrency", "3", "--vocab-size", "1024"])
        assert summary["completed"] == 6 and summary["failed"] == 0
        assert summary["total_output_tokens"] == 24 and summary["mean_ttft_ms"] > 0
        assert summary["mean_tpot_ms"] > 0 and summary["p99_e2el_ms"] >= summary["median_e2el_ms"]
        h = requests.get(pd_url + "/health", timeout=10).json()
        assert sum(h["decode"]["served"].values()) == 7 and all(v == 0 for v in h["decode"]["inflight"].values())
    finally:
        for s in (a, pre, dec, plain, pd):
            s.should_exit = True
        for lp in loops:
            lp.stop()


def test_chat_completions_direct_and_disaggregated():
    from afd_plugin_b200.serving import api_server
    from afd_plugin_b200.serving.proxy import build_proxy_app

    msgs = [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hi"}]
    ids = byte_tokenize(api_server.chat_prompt([api_server.ChatMessage(**m) for m in msgs]), 1024)
    want = _engine().generate([ids], 4)[0]
    loops = [EngineLoop(_engine()).start() for _ in range(2)]
    pre, pre_url = _serve(lambda port: build_app(loops[0], advertise_port=port))
    dec, dec_url = _serve(lambda port: build_app(loops[1], advertise_port=port))
    pd, pd_url = _serve(lambda port: build_proxy_app(prefill=[pre_url], decode=[dec_url]))
    try:
        r = requests.post(dec_url + "/v1/chat/completions", json={"messages": msgs, "max_completion_tokens": 4},
                          timeout=60).json()
        assert r["object"] == "chat.completion" and r["choices"][0]["token_ids"] == want
        assert r["choices"][0]["message"]["role"] == "assistant" and r["usage"]["prompt_tokens"] == len(ids)
        r = requests.post(pd_url + "/v1/chat/completions", json={"messages": msgs, "max_tokens": 4},
                          timeout=60).json()
        assert r["choices"][0]["token_ids"] == want
        toks = []
        with requests.post(pd_url + "/v1/chat/completions", json={"messages": msgs, "max_tokens": 4, "stream": True},
                           stream=True, timeout=60) as s:
            for line in s.iter_lines():
                if line.startswith(b"data: {"):
                    import json as _json

                    msg = _json.loads(line[6:])
                    assert msg["object"] == "chat.completion.chunk"
                    toks += msg["choices"][0]["token_ids"]
        assert toks == want
    finally:
        for s_ in (pre, dec, pd):
            s_.should_exit = True
        for lp in loops:
            lp.stop()


def test_client_disconnect_aborts_the_stream():
    eng = _engine()
    step = eng.step

    def slow_step():
        time.sleep(0.05)
        return step()

    eng.step = slow_step
    loop = EngineLoop(eng).start()
    srv, url = _serve(lambda port: build_app(loop, advertise_port=port))
    try:
        r = requests.post(url + "/v1/completions", json={"prompt": [1, 2, 3], "max_tokens": 80, "stream": True},
                          stream=True, timeout=60)
        it = r.iter_lines()
        got = 0
        for line in it:
            if line.startswith(b"data: {"):
                got += 1
                if got == 3:
                    break
        r.close()
        deadline = time.time() + 20
        while time.time() < deadline and loop.stats["aborted"] == 0:
            time.sleep(0.05)
        assert loop.stats["aborted"] == 1 and loop.stats["completed"] == 0
        assert not eng.running and not eng.waiting
        assert eng.kv.allocator.num_free == eng.kv.allocator.num_blocks - 1
    finally:
        srv.should_exit = True
        loop.stop()


def test_engine_abort_frees_a_waiting_or_running_request():
    eng = _engine()
    a = eng.add_request([1, 2, 3], 10)
    b = eng.add_request([4, 5], 10)
    eng.step()
    assert eng.abort(a) and eng.finished[a].aborted and len(eng.finished[a].output) == 1
    c = eng.add_request([6], 4)
    assert eng.abort(c) and eng.finished[c].output == []
    assert not eng.abort(12345)
    while eng.has_unfinished():
        eng.step()
    assert len(eng.finished[b].output) == 10 and not eng.finished[b].aborted
    assert eng.kv.allocator.num_free == eng.kv.allocator.num_blocks - 1


def test_client_disconnect_through_the_proxy_aborts_at_the_backend():
    from afd_plugin_b200.serving.proxy import build_proxy_app

    eng = _engine()
    step = eng.step

    def slow_step():
        time.sleep(0.05)
        return step()

    eng.step = slow_step
    loop = EngineLoop(eng).start()
    srv, url = _serve(lambda port: build_app(loop, advertise_port=port))
    proxy, purl = _serve(lambda port: build_proxy_app([url]))
    try:
        r = requests.post(purl + "/v1/completions", json={"prompt": [1, 2, 3], "max_tokens": 80, "stream": True},
                          stream=True, timeout=60)
        got = 0
        for line in r.iter_lines():
            if line.startswith(b"data: {"):
                got += 1
                if got == 3:
                    break
        r.close()
        deadline = time.time() + 20
        while time.time() < deadline and loop.stats["aborted"] == 0:
            time.sleep(0.05)
        assert loop.stats["aborted"] == 1
        h = requests.get(purl + "/health", timeout=10).json()
        assert all(v == 0 for v in h["inflight"].values())
    finally:
        for s_ in (srv, proxy):
            s_.should_exit = True
        loop.stop()


def test_balancer_add_remove_and_drain():
    from afd_plugin_b200.serving.proxy import Balancer

    bal = Balancer(["127.0.0.1:1", "http://127.0.0.1:2/"])
    assert bal.backends == ["http://127.0.0.1:1", "http://127.0.0.1:2"]
    a = bal.acquire(5.0)
    b = bal.acquire(1.0)
    assert {a, b} == set(bal.backends)
    assert bal.remove(a) == "isolated" and bal.acquire() == b  # isolated: no new requests
    bal.release(b)
    bal.release(a, 5.0)  # drained -> gone
    assert a not in bal.backends and bal.remove(a) == "unknown"
    assert bal.remove(b) == "isolated"
    bal.release(b)
    assert bal.backends == []
    with pytest.raises(RuntimeError):
        bal.acquire()
    assert bal.add("127.0.0.1:3") and not bal.add("http://127.0.0.1:3")


def test_proxy_instances_endpoints():
    from afd_plugin_b200.serving.proxy import build_proxy_app

    loops = [EngineLoop(_engine()).start() for _ in range(2)]
    a, a_url = _serve(lambda port: build_app(loops[0], advertise_port=port))
    b, b_url = _serve(lambda port: build_app(loops[1], advertise_port=port))
    proxy, purl = _serve(lambda port: build_proxy_app([a_url], instance_retry_s=0.2, max_retries=1))
    try:
        dead = f"127.0.0.1:{free_port()}"
        r = requests.post(purl + "/instances/add", json={"type": "backend", "instances": [b_url, dead]},
                          timeout=30).json()
        assert r["added"] == [b_url] and r["waiting_to_be_added"] == ["http://" + dead]
        assert set(r["current_backend_instances"]) == {a_url, b_url}
        r = requests.post(purl + "/instances/remove", json={"type": "backend", "instances": [a_url, dead]},
                          timeout=30).json()
        assert r["result"] == {a_url: "removed", "http://" + dead: "removed"}
        assert r["current_backend_instances"] == [b_url] and r["waiting_instances"] == []
        out = requests.post(purl + "/v1/completions", json={"prompt": [1, 2], "max_tokens": 2}, timeout=60)
        assert out.status_code == 200
        assert loops[1].stats["completed"] == 1 and loops[0].stats["completed"] == 0
        bad = requests.post(purl + "/instances/add", json={"type": "prefill", "instances": [a_url]}, timeout=30)
        assert bad.status_code == 400
        assert requests.get(purl + "/healthcheck", timeout=10).json()["backends"] == {b_url: True}
        assert requests.get(purl + "/v1/models", timeout=10).json()["data"][0]["object"] == "model"
        assert requests.post(purl + "/reset_prefix_cache", timeout=10).json()[b_url]["reset"] is False  # off
    finally:
        for s_ in (a, b, proxy):
            s_.should_exit = True
        for lp in loops:
            lp.stop()


def test_decode_bench_serving_skips_prefill():
    eng = _engine()
    eng.kv.fill_random_(seed=0)
    loop = EngineLoop(eng, decode_bench=True).start()
    srv, url = _serve(lambda port: build_app(loop, advertise_port=port))
    try:
        prompts = [[7] * 40, [3] * 25]
        outs = [requests.post(url + "/v1/completions", json={"prompt": p, "max_tokens": 5}, timeout=60).json()
                for p in prompts]
        assert [len(o["choices"][0]["token_ids"]) for o in outs] == [5, 5]
        toks, usage, _ = _stream_tokens(url, {"prompt": [9] * 30, "max_tokens": 4})
        assert len(toks) == 4 and usage["completion_tokens"] == 4
        m = requests.get(url + "/metrics", timeout=5).json()
        # every step was a decode step: no prefill ran
        assert m["steps"] == m["decode_steps"] and m["generated_tokens"] == 14
    finally:
        srv.should_exit = True
        loop.stop()


def test_failed_engine_answers_503():
    eng = _engine()

    def broken_step():
        raise RuntimeError("device lost")

    eng.step = broken_step
    loop = EngineLoop(eng).start()
    srv, url = _serve(lambda port: build_app(loop, advertise_port=port))
    try:
        first = requests.post(url + "/v1/completions", json={"prompt": [1, 2], "max_tokens": 2}, timeout=60)
        assert first.status_code == 503 and "device lost" in first.json()["detail"]
        assert requests.get(url + "/health", timeout=5).status_code == 503
        again = requests.post(url + "/v1/completions", json={"prompt": [1, 2], "max_tokens": 2}, timeout=60)
        assert again.status_code == 503
    finally:
        srv.should_exit = True
        loop.stop()


def _word_tokenizer(path):
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    words = ["[UNK]", "<s>", "</s>"] + [f"w{i}" for i in range(200)] + ["hello", "world", "user", "assistant", ":"]
    tok = Tokenizer(models.WordLevel({w: i for i, w in enumerate(words)}, unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    tok.decoder = decoders.WordPiece(prefix="##")
    fast = PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="[UNK]", bos_token="<s>", eos_token="</s>")
    fast.chat_template = "{% for m in messages %}{{ m['role'] }} : {{ m['content'] }} {% endfor %}assistant :"
    fast.save_pretrained(str(path))
    return fast


def test_hf_tokenizer_text_chat_and_stream(tmp_path):
    from afd_plugin_b200.serving.tokenizer import HFTokenizer, load_tokenizer

    fast = _word_tokenizer(tmp_path)
    tok = load_tokenizer(str(tmp_path), 1024)
    assert isinstance(tok, HFTokenizer) and tok.encode("hello world") == fast.encode("hello world")
    assert isinstance(load_tokenizer(None, 1024), type(load_tokenizer(str(tmp_path / "missing"), 1024)))
    loop = EngineLoop(_engine()).start()
    srv, url = _serve(lambda port: build_app(loop, advertise_port=port, tokenizer=tok))
    try:
        ids = fast.encode("hello world w5 w7")
        want = _engine().generate([ids], 5)[0]
        r = requests.post(url + "/v1/completions", json={"prompt": "hello world w5 w7", "max_tokens": 5},
                          timeout=60).json()
        assert r["choices"][0]["token_ids"] == want and r["choices"][0]["text"] == fast.decode(
            want, skip_special_tokens=True)
        msgs = [{"role": "user", "content": "hello w3"}]
        chat_ids = fast.apply_chat_template(msgs, tokenize=True, add_generation_prompt=True)
        chat_ids = list(chat_ids["input_ids"] if hasattr(chat_ids, "keys") else chat_ids)
        c = requests.post(url + "/v1/chat/completions", json={"messages": msgs, "max_tokens": 3}, timeout=60).json()
        assert c["usage"]["prompt_tokens"] == len(chat_ids)
        assert c["choices"][0]["token_ids"] == _engine().generate([chat_ids], 3)[0]
        text = ""
        with requests.post(url + "/v1/completions", json={"prompt": "hello world w5 w7", "max_tokens": 5,
                                                          "stream": True}, stream=True, timeout=60) as s:
            import json as _json

            for line in s.iter_lines():
                if line.startswith(b"data: {"):
                    text += _json.loads(line[6:])["choices"][0]["text"]
        assert text == r["choices"][0]["text"]
    finally:
        srv.should_exit = True
        loop.stop()


def test_server_cli_accepts_reference_recipe_flags():
    import json as _json

    from afd_plugin_b200.serving.__main__ import parse_args

    a = parse_args(["/models/dsv2-lite", "--additional-config",
                    '{"afd": {"role": "attention", "num_attention_ranks": 2, "num_ffn_ranks": 2}}',
                    "--compilation-config", '{"cudagraph_mode": "FULL_DECODE_ONLY", "cudagraph_capture_sizes": [64]}',
                    "--enable-dbo", "--dbo-decode-token-threshold", "2", "--dbo-prefill-token-threshold", "12",
                    "--enable-expert-parallel", "--tensor-parallel-size", "1", "--served-model-name", "dsv2"])
    assert a.checkpoint == "/models/dsv2-lite" and a.sizes == [64] and a.dbo and a.tp == 1 and not a.eager
    assert _json.loads(a.afd)["num_ffn_ranks"] == 2 and a.served_model_name == "dsv2"
    b = parse_args(["--compilation-config", '{"cudagraph_mode": "NONE"}', "--max-num-seqs", "8"])
    assert b.eager and b.sizes == [8] and b.checkpoint is None
    assert parse_args(["--enforce-eager", "--model", "/m"]).eager
    with pytest.raises(SystemExit):
        parse_args(["--compilation-config", '{"cudagraph_mode": "PIECEWISE"}'])
    with pytest.raises(SystemExit):
        parse_args(["--afd", "{}", "--additional-config", '{"afd": {}}'])


def test_text_stop_sequences(any_server):
    url, loop = any_server
    prompt = [5, 9, 100, 7, 3, 1]
    full = _engine().generate([prompt], 12)[0]
    text = byte_detokenize(full)
    stop = text[4:6]
    cut = text.find(stop)
    r = requests.post(url + "/v1/completions", json={"prompt": prompt, "max_tokens": 12, "stop": [stop, "\x00zz"]},
                      timeout=60).json()
    c = r["choices"][0]
    assert c["finish_reason"] == "stop" and c["text"] == text[:cut]
    assert c["token_ids"] == full[: len(c["token_ids"])] and len(c["token_ids"]) < 12
    plain = requests.post(url + "/v1/completions", json={"prompt": prompt, "max_tokens": 12, "stop": "\x00zz"},
                          timeout=60).json()["choices"][0]
    assert plain["finish_reason"] == "length" and plain["token_ids"] == full


def test_batch_of_prompts_in_one_request(server):
    url, _ = server
    prompts = [[5, 9, 100], [42] * 5, [1, 2, 3, 4]]
    want = _engine().generate(prompts, 3)
    r = requests.post(url + "/v1/completions", json={"prompt": prompts, "max_tokens": 3}, timeout=60).json()
    assert [c["token_ids"] for c in r["choices"]] == want and [c["index"] for c in r["choices"]] == [0, 1, 2]
    assert r["usage"]["prompt_tokens"] == 12 and r["usage"]["completion_tokens"] == 9
    t = requests.post(url + "/v1/completions", json={"prompt": ["ab", "cd"], "max_tokens": 2}, timeout=60).json()
    assert len(t["choices"]) == 2
    bad = requests.post(url + "/v1/completions", json={"prompt": prompts, "max_tokens": 2, "stream": True},
                        timeout=60)
    assert bad.status_code == 400


def test_openai_python_client_talks_to_the_server(server):
    """The official OpenAI client parses every response shape (completions, chat, streams)."""
    openai = pytest.importorskip("openai")
    url, _ = server
    client = openai.OpenAI(base_url=url + "/v1", api_key="unused")
    prompt = [5, 9, 100, 7, 3, 1]
    want = _engine().generate([prompt], 5)[0]
    c = client.completions.create(model="afd-b200", prompt=prompt, max_tokens=5)
    assert c.id.startswith("cmpl-") and c.choices[0].finish_reason == "length" and c.usage.completion_tokens == 5
    assert c.choices[0].text == byte_detokenize(want)
    chunks = list(client.completions.create(model="afd-b200", prompt=prompt, max_tokens=5, stream=True))
    assert "".join(ch.choices[0].text for ch in chunks) == byte_detokenize(want)
    chat = client.chat.completions.create(model="afd-b200", messages=[{"role": "user", "content": "hi"}],
                                          max_tokens=3, temperature=0.0)
    assert chat.id.startswith("chatcmpl-") and chat.choices[0].message.role == "assistant"
    stream = client.chat.completions.create(model="afd-b200", messages=[{"role": "user", "content": "hi"}],
                                            max_tokens=3, stream=True)
    text = "".join(ch.choices[0].delta.content or "" for ch in stream)
    assert text == chat.choices[0].message.content
    assert [m.id for m in client.models.list().data] == ["afd-b200"]


def test_completion_echo_and_penalty_fields(server):
    url, _ = server
    prompt = [5, 9, 100, 7]
    body = requests.post(url + "/v1/completions", json={"prompt": prompt, "max_tokens": 3, "echo": True},
                         timeout=60).json()
    want = _engine().generate([prompt], 3)[0]
    assert body["choices"][0]["text"] == byte_detokenize(prompt) + byte_detokenize(want)
    assert body["choices"][0]["token_ids"] == want
    bad = requests.post(url + "/v1/completions", json={"prompt": prompt, "max_tokens": 3, "echo": True,
                                                        "stream": True}, timeout=60)
    assert bad.status_code == 400
    forced = requests.post(url + "/v1/completions", json={"prompt": prompt, "max_tokens": 3,
                                                           "logit_bias": {"17": 100}}, timeout=60).json()
    assert forced["choices"][0]["token_ids"] == [17, 17, 17]
    bad = requests.post(url + "/v1/completions", json={"prompt": prompt, "max_tokens": 3,
                                                        "repetition_penalty": 0}, timeout=60)
    assert bad.status_code == 400


def test_chat_content_parts_equal_plain_text(server):
    url, _ = server
    plain = requests.post(url + "/v1/chat/completions", json={
        "messages": [{"role": "user", "content": "hello there"}], "max_tokens": 4}, timeout=60).json()
    parts = requests.post(url + "/v1/chat/completions", json={
        "messages": [{"role": "user", "content": [{"type": "text", "text": "hello "},
                                                  {"type": "text", "text": "there"}]}], "max_tokens": 4},
        timeout=60).json()
    assert parts["choices"][0]["token_ids"] == plain["choices"][0]["token_ids"]
    bad = requests.post(url + "/v1/chat/completions", json={
        "messages": [{"role": "user", "content": [{"type": "image_url", "image_url": {"url": "x"}}]}],
        "max_tokens": 4}, timeout=60)
    assert bad.status_code == 400
