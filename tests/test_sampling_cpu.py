"""Sampling: temperature / top-k / top-p masks, the exponential-race draw, seeds, engine and server wiring."""

from __future__ import annotations

import pytest
import torch

from afd_plugin_b200.engine_config import EngineConfig, ModelConfig
from afd_plugin_b200.models import build_model, get_preset
from afd_plugin_b200.runtime.engine import LLMEngine
from afd_plugin_b200.runtime.sampling import GREEDY, SamplingParams, filtered_probs, make_generator, sample


def _engine(seed=0):
    arch = get_preset("tiny-dsv2")
    ec = EngineConfig(ModelConfig(arch, dtype=torch.float32, enforce_eager=True, max_model_len=96, seed=seed),
                      max_num_seqs=4)
    return LLMEngine(ec, build_model(arch, role="colocated", dtype=torch.float32, seed=0, max_positions=96))


def test_greedy_rows_and_top_k_one_are_argmax():
    logits = torch.randn(4, 50, generator=torch.Generator().manual_seed(0))
    params = [GREEDY, SamplingParams(temperature=0.7, top_k=1), GREEDY, SamplingParams(temperature=2.0, top_k=1)]
    assert torch.equal(sample(logits, params, [None] * 4), logits.argmax(-1).int())


def test_draws_follow_the_distribution():
    base = torch.tensor([2.0, 1.0, 0.5, 0.0, -1.0])
    n = 20000
    logits = base.repeat(n, 1)
    toks = sample(logits, [SamplingParams(temperature=1.0)] * n, [None] * n, make_generator(1, "cpu"))
    freq = torch.bincount(toks.long(), minlength=5).float() / n
    assert torch.allclose(freq, torch.softmax(base, 0), atol=0.015)
    hot = sample(logits, [SamplingParams(temperature=0.5)] * n, [None] * n, make_generator(2, "cpu"))
    freq = torch.bincount(hot.long(), minlength=5).float() / n
    assert torch.allclose(freq, torch.softmax(base / 0.5, 0), atol=0.015)


def test_top_k_and_top_p_masks():
    logits = torch.log(torch.tensor([[0.5, 0.3, 0.15, 0.05]]))
    pk = filtered_probs(logits, [SamplingParams(temperature=1.0, top_k=2)])[0]
    assert torch.allclose(pk, torch.tensor([0.625, 0.375, 0.0, 0.0]), atol=1e-5)
    pp = filtered_probs(logits, [SamplingParams(temperature=1.0, top_p=0.7)])[0]
    assert torch.allclose(pp, torch.tensor([0.625, 0.375, 0.0, 0.0]), atol=1e-5)
    tiny = filtered_probs(logits, [SamplingParams(temperature=1.0, top_p=0.01)])[0]
    assert torch.allclose(tiny, torch.tensor([1.0, 0.0, 0.0, 0.0]))
    with pytest.raises(ValueError):
        SamplingParams(top_p=0.0)
    with pytest.raises(ValueError):
        SamplingParams(temperature=-1.0)


def test_seeded_rows_do_not_depend_on_the_batch():
    logits = torch.randn(3, 40, generator=torch.Generator().manual_seed(3))
    sp = SamplingParams(temperature=1.0, seed=11)
    alone = sample(logits[1:2], [sp], [make_generator(11, "cpu")])
    mixed = sample(logits, [SamplingParams(temperature=1.0), sp, GREEDY],
                   [None, make_generator(11, "cpu"), None], make_generator(99, "cpu"))
    assert int(alone[0]) == int(mixed[1]) and int(mixed[2]) == int(logits[2].argmax())


def test_engine_sampling_is_seeded_and_greedy_is_unchanged():
    prompt = [5, 9, 100, 7]
    greedy = _engine().generate([prompt], 6)[0]
    sp = SamplingParams(temperature=1.5, top_k=50, seed=123)

    def run(sampling, others=()):
        eng = _engine()
        rid = eng.add_request(prompt, 6, sampling=sampling)
        for o in others:
            eng.add_request(o, 6, sampling=SamplingParams(temperature=1.0))
        while eng.has_unfinished():
            eng.step()
        return eng.finished[rid].output

    a, b = run(sp), run(sp, others=([1, 2, 3], [4, 4, 4, 4]))
    assert a == b and len(a) == 6
    assert run(SamplingParams(temperature=1.5, top_k=50, seed=124)) != a
    assert run(None) == greedy


def test_kv_handoff_continues_a_seeded_stream():
    prompt = [3, 1, 4, 1, 5, 9, 2, 6]
    sp = SamplingParams(temperature=1.2, seed=7)
    ref = _engine()
    rid = ref.add_request(prompt, 6, sampling=sp)
    while ref.has_unfinished():
        ref.step()
    want = ref.finished[rid].output
    pre, dec = _engine(), _engine()
    r1 = pre.add_request(prompt, 1, hold_kv=True, sampling=sp)
    while pre.has_unfinished():
        pre.step()
    r2, _ = dec.add_prefilled_request(pre.export_kv(r1), 6, sampling=sp)
    while dec.has_unfinished():
        dec.step()
    assert dec.finished[r2].output == want


def test_server_sampling_fields():
    import threading
    import time

    import requests
    import uvicorn

    from afd_plugin_b200.runtime.launcher import free_port
    from afd_plugin_b200.serving import EngineLoop, build_app

    loop = EngineLoop(_engine()).start()
    port = free_port()
    srv = uvicorn.Server(uvicorn.Config(build_app(loop), host="127.0.0.1", port=port, log_level="warning"))
    threading.Thread(target=srv.run, daemon=True).start()
    url = f"http://127.0.0.1:{port}"
    for _ in range(200):
        try:
            if requests.get(url + "/health", timeout=2).ok:
                break
        except requests.ConnectionError:
            time.sleep(0.05)
    try:
        body = {"prompt": [5, 9, 100, 7], "max_tokens": 6, "temperature": 1.5, "top_k": 50, "seed": 123}
        a = requests.post(url + "/v1/completions", json=body, timeout=60).json()["choices"][0]["token_ids"]
        b = requests.post(url + "/v1/completions", json=body, timeout=60).json()["choices"][0]["token_ids"]
        assert a == b and len(a) == 6
        bad = requests.post(url + "/v1/completions", json=dict(body, top_p=1.5), timeout=60)
        assert bad.status_code == 400 and "top_p" in bad.json()["detail"]
    finally:
        srv.should_exit = True
        loop.stop()


def test_stop_tokens_and_eos():
    from dataclasses import replace

    prompt = [5, 9, 100, 7]
    full = _engine().generate([prompt], 8)[0]
    stop_at = full[3]
    eng = _engine()
    rid = eng.add_request(prompt, 8, sampling=SamplingParams(stop_token_ids=(stop_at,)))
    while eng.has_unfinished():
        eng.step()
    r = eng.finished[rid]
    cut = full.index(stop_at) + 1
    assert r.output == full[:cut] and r.finish_reason == "stop"
    # the model's EOS ends generation unless the request ignores it
    eos_eng = _engine()
    eos_eng.model.arch = replace(eos_eng.model.arch, eos_token_id=(stop_at,))
    a = eos_eng.add_request(prompt, 8)
    b = eos_eng.add_request(prompt, 8, sampling=SamplingParams(ignore_eos=True))
    while eos_eng.has_unfinished():
        eos_eng.step()
    assert eos_eng.finished[a].output == full[:cut] and eos_eng.finished[b].output == full
    assert eos_eng.finished[b].finish_reason == "length"


def test_hf_eos_parsing():
    from afd_plugin_b200.models.configs import ModelArchConfig

    hf = {"architectures": ["Qwen3MoeForCausalLM"], "model_type": "qwen3_moe", "hidden_size": 64,
          "num_hidden_layers": 2, "vocab_size": 100, "num_attention_heads": 4, "num_key_value_heads": 2,
          "head_dim": 16, "num_experts": 4, "num_experts_per_tok": 2, "moe_intermediate_size": 32,
          "eos_token_id": [7, 9]}
    assert ModelArchConfig.from_hf_config(hf).eos_token_id == (7, 9)
    hf["eos_token_id"] = 3
    assert ModelArchConfig.from_hf_config(hf).eos_token_id == (3,)


def test_engine_logprobs_match_log_softmax():
    eng = _engine()
    prompt = [5, 9, 100, 7]
    rid = eng.add_request(prompt, 4, sampling=SamplingParams(logprobs=3))
    while eng.has_unfinished():
        eng.step()
    r = eng.finished[rid]
    assert len(r.token_logprobs) == len(r.output) == 4 and all(len(t) == 3 for t in r.top_logprobs)
    # greedy: the chosen token is the most likely one
    for tok, lp, top in zip(r.output, r.token_logprobs, r.top_logprobs):
        assert top[0][0] == tok and abs(top[0][1] - lp) < 1e-6 and lp <= 0.0
    # recompute the first token's logprob from a fresh prefill
    ref = _engine()
    req = __import__("afd_plugin_b200.runtime.engine", fromlist=["Request"]).Request(0, prompt, 1)
    ref._ensure_blocks(req, len(prompt) + 1)
    ref.runner.prefill([prompt], [req.blocks], [0])
    want = torch.log_softmax(ref.runner.last_logits.float(), -1)[0, r.output[0]].item()
    assert abs(want - r.token_logprobs[0]) < 1e-5


def test_server_n_choices_and_logprobs():
    import threading
    import time

    import requests
    import uvicorn

    from afd_plugin_b200.runtime.launcher import free_port
    from afd_plugin_b200.serving import EngineLoop, build_app

    loop = EngineLoop(_engine()).start()
    port = free_port()
    srv = uvicorn.Server(uvicorn.Config(build_app(loop), host="127.0.0.1", port=port, log_level="warning"))
    threading.Thread(target=srv.run, daemon=True).start()
    url = f"http://127.0.0.1:{port}"
    for _ in range(200):
        try:
            if requests.get(url + "/health", timeout=2).ok:
                break
        except requests.ConnectionError:
            time.sleep(0.05)
    try:
        body = {"prompt": [5, 9, 100, 7], "max_tokens": 5, "temperature": 1.0, "seed": 5, "n": 3, "logprobs": 2}
        r = requests.post(url + "/v1/completions", json=body, timeout=60).json()
        assert [c["index"] for c in r["choices"]] == [0, 1, 2] and r["usage"]["completion_tokens"] == 15
        lp = r["choices"][0]["logprobs"]
        assert len(lp["tokens"]) == len(lp["token_logprobs"]) == len(lp["top_logprobs"]) == 5
        assert all(len(t) <= 2 for t in lp["top_logprobs"]) and lp["text_offset"][0] == 0
        again = requests.post(url + "/v1/completions", json=body, timeout=60).json()
        assert [c["token_ids"] for c in again["choices"]] == [c["token_ids"] for c in r["choices"]]
        chat = requests.post(url + "/v1/chat/completions", json={
            "messages": [{"role": "user", "content": "hi"}], "max_tokens": 3, "logprobs": True, "top_logprobs": 1},
            timeout=60).json()
        content = chat["choices"][0]["logprobs"]["content"]
        assert len(content) == 3 and len(content[0]["top_logprobs"]) == 1
        bad = requests.post(url + "/v1/completions", json=dict(body, stream=True), timeout=60)
        assert bad.status_code == 400
    finally:
        srv.should_exit = True
        loop.stop()


def test_penalties_follow_their_definitions():
    from afd_plugin_b200.runtime.sampling import apply_penalties

    logits = torch.tensor([[2.0, -1.0, 0.5, 3.0, 0.0]] * 3)
    prompts = [[0], [0], [0]]
    outputs = [[3, 3, 2], [3, 3, 2], [3, 3, 2]]
    params = [SamplingParams(presence_penalty=0.5), SamplingParams(frequency_penalty=0.25),
              SamplingParams(repetition_penalty=2.0)]
    x = apply_penalties(logits, params, prompts, outputs)
    assert torch.allclose(x[0], torch.tensor([2.0, -1.0, 0.0, 2.5, 0.0]))
    assert torch.allclose(x[1], torch.tensor([2.0, -1.0, 0.25, 2.5, 0.0]))
    assert torch.allclose(x[2], torch.tensor([1.0, -1.0, 0.25, 1.5, 0.0]))  # prompt token 0 too
    # no penalties: same values
    assert torch.equal(apply_penalties(logits, [GREEDY] * 3, prompts, outputs), logits)
    with pytest.raises(ValueError):
        SamplingParams(repetition_penalty=0.0)
    with pytest.raises(ValueError):
        SamplingParams(presence_penalty=3.0)


def test_engine_penalties_stop_greedy_repetition():
    """A strong presence penalty forbids repeating any generated token; greedy otherwise."""
    eng = _engine()
    prompt = [3, 1, 4, 1, 5]
    base = eng.generate([prompt], 24)[0]
    assert len(set(base)) < len(base), "the tiny model repeats itself greedily"
    eng2 = _engine()
    out = eng2.generate([prompt], 24, sampling=SamplingParams(presence_penalty=2.0, frequency_penalty=2.0,
                                                               repetition_penalty=50.0))[0]
    assert out[0] == base[0]  # nothing generated yet when the first token is chosen (prompt only matters)
    assert len(set(out)) > len(set(base))


def test_server_penalty_fields_and_vllm_top_k():
    from afd_plugin_b200.serving.api_server import CompletionRequest

    req = CompletionRequest(prompt="x", presence_penalty=0.5, top_k=-1)
    sp = req.sampling()
    assert sp.presence_penalty == 0.5 and sp.top_k == 0 and sp.penalized and sp.greedy
    assert CompletionRequest(prompt="x").sampling() is None


def test_min_tokens_holds_back_stop_tokens():
    eng = _engine()
    prompt = [2, 7, 1, 8]
    free = eng.generate([prompt], 12)[0]
    stop = free[1]  # the second greedy token: a stop token ends generation there
    eng2 = _engine()
    short = eng2.generate([prompt], 12, sampling=SamplingParams(stop_token_ids=(stop,)))[0]
    assert short == free[:2]
    eng3 = _engine()
    held = eng3.generate([prompt], 12, sampling=SamplingParams(stop_token_ids=(stop,), min_tokens=6))[0]
    assert stop not in held[:6] and len(held) >= 6
    assert held[0] == free[0]
    with pytest.raises(ValueError):
        SamplingParams(min_tokens=-1)


def test_logit_bias_forces_and_bans_tokens():
    from afd_plugin_b200.runtime.sampling import apply_penalties
    from afd_plugin_b200.serving.api_server import CompletionRequest

    logits = torch.tensor([[1.0, 2.0, 3.0]])
    x = apply_penalties(logits, [SamplingParams(logit_bias=((0, 5.0), (2, -100.0)))], [[]], [[]])
    assert torch.allclose(x, torch.tensor([[6.0, 2.0, -97.0]]))
    eng = _engine()
    out = eng.generate([[4, 4, 2]], 5, sampling=SamplingParams(logit_bias=((17, 100.0),)))[0]
    assert out == [17] * 5
    sp = CompletionRequest(prompt="x", logit_bias={"17": 100}).sampling()
    assert sp.logit_bias == ((17, 100.0),) and sp.greedy
    with pytest.raises(ValueError):
        SamplingParams(logit_bias=((1, 101.0),))
