"""Reference arm of ``bench.py`` (``python bench.py --impl reference``).

Runs the UNMODIFIED reference (``baseline/_ref``: the ``afd_plugin`` vLLM
plugin, installed with ``pip --target``) through its own stock code path on
the installed vLLM, for the same metric and workload as this framework's arm:
DeepSeek-V2-Lite architecture, bf16, random ("dummy") weights, 256 concurrent
requests with 1024 uniform-random prompt token ids and 256 output tokens,
ignore_eos, FULL_DECODE_ONLY CUDA graphs.  Nothing of ``afd_plugin_b200`` runs
on this path except the clock sampler (it only reads ``nvidia-smi``).

Scenarios, per the reference's own e2e scenario table
(``tests/e2e/runner.py:361-475``, ``build_baseline_command`` at ``:530-575``):

* N=1: the reference's "baseline" deployment -- native vLLM with the AFD
  plugin loaded through its ``vllm.general_plugins`` entry point and no AFD
  section in ``additional_config`` (one GPU cannot host an Attention and an
  FFN role).  It runs in-process through ``vllm.LLM`` /
  ``LLMEngine.step`` (``VLLM_ENABLE_V1_MULTIPROCESSING=0``), so the decode
  steps are timed with CUDA events on this process's stream.
* N>1: the reference's AFD deployment (``P2pNcclAFDConnector``; one
  ``vllm serve`` per role, as in
  ``recipe/gpu/P2pNcclAFDConnector/deepseek_v2_lite/prefill_decode_colocation/*.sh``).
  It is launched for real; when a role process exits or does not come up,
  the line reports ``unavailable`` with the tail of that process's log.

Timing: prefill (chunked, as vLLM schedules it) runs untimed until every
request has its first token; then W warm-up engine steps, then exactly K
engine steps bracketed by ``torch.cuda.synchronize()`` and CUDA events.
Each engine step is one decode iteration of every running request, host
scheduling and output processing included (the stock engine loop), so the
same number is also the end-to-end figure.
"""

from __future__ import annotations

import json
import os
import shutil
import signal
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")

# Public DeepSeek-V2-Lite config.json (architecture only; weights are dummy).
DSV2_LITE_HF = {
    "architectures": ["DeepseekV2ForCausalLM"],
    "model_type": "deepseek_v2",
    "vocab_size": 102400,
    "hidden_size": 2048,
    "intermediate_size": 10944,
    "moe_intermediate_size": 1408,
    "num_hidden_layers": 27,
    "num_attention_heads": 16,
    "num_key_value_heads": 16,
    "n_shared_experts": 2,
    "n_routed_experts": 64,
    "num_experts_per_tok": 6,
    "routed_scaling_factor": 1.0,
    "kv_lora_rank": 512,
    "q_lora_rank": None,
    "qk_rope_head_dim": 64,
    "qk_nope_head_dim": 128,
    "v_head_dim": 128,
    "topk_method": "greedy",
    "n_group": 1,
    "topk_group": 1,
    "norm_topk_prob": False,
    "scoring_func": "softmax",
    "first_k_dense_replace": 1,
    "moe_layer_freq": 1,
    "aux_loss_alpha": 0.001,
    "seq_aux": True,
    "hidden_act": "silu",
    "max_position_embeddings": 163840,
    "initializer_range": 0.02,
    "rms_norm_eps": 1e-6,
    "use_cache": True,
    "bos_token_id": 100000,
    "eos_token_id": 100001,
    "tie_word_embeddings": False,
    "rope_theta": 10000,
    "rope_scaling": {"type": "yarn", "factor": 40, "beta_fast": 32, "beta_slow": 1, "mscale": 0.707,
                     "mscale_all_dim": 0.707, "original_max_position_embeddings": 4096},
    "attention_bias": False,
    "attention_dropout": 0.0,
    "torch_dtype": "bfloat16",
}

MODELS = {"deepseek-v2-lite": DSV2_LITE_HF}
# N>1 role split of the AFD deployment (A, F), the same as this framework's arm.
AFD_TOPOLOGY = {2: (1, 1), 4: (2, 2), 8: (6, 2)}


def _emit(line: dict) -> None:
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(line), flush=True)


def _unavailable(reason: str) -> None:
    _emit({"impl": "reference", "unavailable": " ".join(reason.split())[:1500]})


def _write_model_dir(model: str) -> str:
    d = tempfile.mkdtemp(prefix="afd_ref_model_")
    with open(os.path.join(d, "config.json"), "w") as fh:
        json.dump(MODELS[model], fh, indent=1)
    with open(os.path.join(d, "generation_config.json"), "w") as fh:
        json.dump({"bos_token_id": 100000, "eos_token_id": 100001}, fh)
    return d


def _prompts(n: int, isl: int, vocab: int, seed: int = 0) -> list[list[int]]:
    import torch

    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n, isl), generator=g).tolist()


def _ref_env() -> dict:
    env = dict(os.environ)
    env["PYTHONPATH"] = REF_DIR + (os.pathsep + env["PYTHONPATH"] if env.get("PYTHONPATH") else "")
    return env


# ---------------------------------------------------------------- N = 1
def run_colocated(args, metric: str, model_desc: str) -> None:
    """The reference's baseline scenario on one GPU, timed in-process."""
    os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"
    os.environ.setdefault("VLLM_LOGGING_LEVEL", "WARNING")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import afd_plugin  # noqa: F401  (the installed reference; fails loudly if absent)
    import torch
    from vllm import LLM, SamplingParams
    from vllm.sampling_params import RequestOutputKind

    from afd_plugin_b200.utils.clocks import ClockSampler

    model_dir = _write_model_dir(args.model)
    hf = MODELS[args.model]
    batch, isl, osl = args.batch, args.isl, args.osl
    llm = LLM(
        model=model_dir,
        load_format="dummy",
        skip_tokenizer_init=True,
        dtype="bfloat16",
        seed=0,
        max_model_len=isl + osl + 64,
        max_num_seqs=batch,
        enable_prefix_caching=False,
        gpu_memory_utilization=0.85,
        compilation_config={"cudagraph_mode": "FULL_DECODE_ONLY", "cudagraph_capture_sizes": [batch]},
    )
    engine = llm.llm_engine
    params = SamplingParams(max_tokens=osl, ignore_eos=True, temperature=0.0, detokenize=False,
                            output_kind=RequestOutputKind.DELTA)
    for i, ids in enumerate(_prompts(batch, isl, hf["vocab_size"])):
        engine.add_request(f"r{i}", {"prompt_token_ids": ids}, params)
    got: dict[str, int] = {}
    guard = 0
    while len(got) < batch:  # prefill (untimed)
        for out in engine.step():
            got[out.request_id] = got.get(out.request_id, 0) + len(out.outputs[0].token_ids)
        guard += 1
        if guard > 10 * batch:
            raise RuntimeError("reference engine did not prefill every request")

    def step_tokens() -> int:
        return sum(len(o.outputs[0].token_ids) for o in engine.step())

    for _ in range(args.warmup):
        step_tokens()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    tokens = 0
    with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        ev[0].record()
        for i in range(args.steps):
            tokens += step_tokens()
            ev[i + 1].record()
        torch.cuda.synchronize()
    per_step = [ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps)]
    total_ms = ev[0].elapsed_time(ev[-1])
    if tokens < batch * args.steps * 0.95:
        raise RuntimeError(f"timed steps produced {tokens} tokens, expected about {batch * args.steps}")
    value = tokens / (total_ms / 1e3)
    c = clk.summary()
    import vllm

    _emit({
        "impl": "reference",
        "metric": metric,
        "value": round(value, 1),
        "unit": "tok/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 4),
        "p50_tpot_ms": round(statistics.median(per_step), 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (dummy-init weights; uniform-random prompt ids, prefilled untimed)",
        "config": {
            "model": model_desc,
            "global_batch": batch,
            "seq_len": isl + osl,
            "input_len": isl,
            "output_len": osl,
            "parallelism": "colocated-1gpu (reference baseline scenario: vLLM + afd_plugin, no AFD section)",
            "cuda_graphs": True,
            "dbo": False,
            "stack": f"afd_plugin (baseline/_ref) on vLLM {vllm.__version__}",
            "l2": "inputs larger than L2 (31 GB weights, ~10 GB KV per step); no flush",
        },
        "clocks": {"sm_mhz": c.get("sm_mhz"), "sm_max_mhz": c.get("sm_max_mhz"), "reasons": c.get("reasons", [])},
        "e2e": {"value": round(value, 1), "unit": "tok/s", "h2d_bytes_per_step": None, "d2h_bytes_per_step": None,
                "note": "the timed engine steps are the stock end-to-end loop"},
        "tokens_timed": tokens,
    })


# ---------------------------------------------------------------- N > 1
def _tail(path: str, n: int = 25) -> str:
    try:
        with open(path, errors="replace") as fh:
            lines = [ln.rstrip() for ln in fh.readlines() if ln.strip()]
    except OSError:
        return "(no log)"
    keep = [ln for ln in lines if "Error" in ln or "error" in ln or "Traceback" in ln or "raise" in ln]
    return " | ".join((keep[-6:] if keep else []) + lines[-n:][-6:])


def _vllm_serve_cmd(model_dir: str, role: str, a: int, f: int, port: int, api_port: int, per_rank: int) -> list:
    ranks = a if role == "attention" else f
    afd = {"afd": {"role": role, "connector": "P2pNcclAFDConnector", "host": "127.0.0.1", "port": port,
                   "num_attention_ranks": a, "num_ffn_ranks": f}}
    return [sys.executable, "-m", "vllm.entrypoints.cli.main", "serve", model_dir,
            "--load-format", "dummy", "--skip-tokenizer-init", "--dtype", "bfloat16",
            "--data-parallel-size", str(ranks), "--tensor-parallel-size", "1", "--enable-expert-parallel",
            "--additional-config", json.dumps(afd), "--max-num-seqs", str(per_rank),
            "--max-num-batched-tokens", str(max(per_rank, 64)), "--max-cudagraph-capture-size", str(per_rank),
            "--compilation-config", json.dumps({"cudagraph_mode": "FULL_DECODE_ONLY",
                                                "cudagraph_capture_sizes": [per_rank]}),
            "--host", "127.0.0.1", "--port", str(api_port)]


def run_afd(args, metric: str, model_desc: str) -> None:
    """Launch the reference's AFD deployment; report why it cannot be timed."""
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("gloo")
    reason = None
    if rank == 0:
        reason = _afd_launch_attempt(args)
    if world > 1:
        box = [reason]
        dist.broadcast_object_list(box, src=0)
        dist.destroy_process_group()
    if rank == 0:
        _unavailable(reason)


def _afd_launch_attempt(args) -> str:
    a, f = AFD_TOPOLOGY.get(args.gpus, (args.gpus - 1, 1))
    per_rank = -(-args.batch // a)
    model_dir = _write_model_dir(args.model)
    logdir = tempfile.mkdtemp(prefix="afd_ref_logs_")
    procs = []
    env = _ref_env()
    env["VLLM_USE_V2_MODEL_RUNNER"] = "0"
    gpus = list(range(args.gpus))
    roles = (("ffn", gpus[:f], 18400), ("attention", gpus[f:], 18401))  # FFN-first world order
    try:
        for role, devs, api in roles:
            e = dict(env)
            e["CUDA_VISIBLE_DEVICES"] = ",".join(str(d) for d in devs)
            log = os.path.join(logdir, f"{role}.log")
            fh = open(log, "w")
            procs.append((role, subprocess.Popen(_vllm_serve_cmd(model_dir, role, a, f, 16269, api, per_rank),
                                                 stdout=fh, stderr=subprocess.STDOUT, env=e,
                                                 start_new_session=True), log))
        deadline = time.time() + float(os.environ.get("AFD_REF_LAUNCH_TIMEOUT_S", "420"))
        while time.time() < deadline:
            for role, p, log in procs:
                if p.poll() is not None:
                    return (f"reference AFD {a}A{f}F launch (vllm serve, P2pNcclAFDConnector, "
                            f"{_vllm_version()}): {role} role exited with code {p.returncode}: {_tail(log)}")
            if _healthy(18401) and _healthy(18400):
                return (f"reference AFD {a}A{f}F came up on {_vllm_version()}, but its serving path has no "
                        "device-timed decode loop to drive from this process")
            time.sleep(3)
        return (f"reference AFD {a}A{f}F launch did not become healthy within the launch timeout; attention log: "
                f"{_tail(procs[-1][2])}")
    finally:
        for _, p, _ in procs:
            if p.poll() is None:
                try:
                    os.killpg(p.pid, signal.SIGTERM)
                    p.wait(timeout=20)
                except Exception:  # noqa: BLE001
                    try:
                        os.killpg(p.pid, signal.SIGKILL)
                    except Exception:  # noqa: BLE001
                        pass
        shutil.rmtree(model_dir, ignore_errors=True)


def _healthy(port: int) -> bool:
    import urllib.request

    try:
        with urllib.request.urlopen(f"http://127.0.0.1:{port}/health", timeout=2) as r:
            return r.status == 200
    except Exception:  # noqa: BLE001
        return False


def _vllm_version() -> str:
    from afd_plugin_b200.compat import installed_vllm_version

    return f"vLLM {installed_vllm_version() or '(not installed)'}"


def main(args, metric: str, model_desc: str) -> None:
    if not os.path.isdir(os.path.join(REF_DIR, "afd_plugin")):
        _unavailable("reference not installed under baseline/_ref (pip install --target baseline/_ref failed or "
                     "was not run)")
        return
    if args.model not in MODELS:
        _unavailable(f"reference arm has no config.json for model {args.model!r}")
        return
    if args.gpus == 1:
        try:
            run_colocated(args, metric, model_desc)
        except Exception as exc:  # noqa: BLE001
            import traceback

            tb = traceback.format_exc().strip().splitlines()
            from afd_plugin_b200.compat import reference_vllm_mismatch

            why = reference_vllm_mismatch()
            _unavailable(f"reference baseline run failed: {type(exc).__name__}: {exc} | " + " | ".join(tb[-4:])
                         + (f" | note: {why}" if why else ""))
        return
    run_afd(args, metric, model_desc)
