"""Run an AFD deployment as local processes (one per rank).

``launch_local`` spawns ``F + A`` processes in the FFN-first world order over
``127.0.0.1`` (gloo on CPU, NCCL on GPUs).  Attention ranks generate their
share of the prompts in lockstep; FFN ranks serve until the Attention side
sends the shutdown control payload.  Used by the CPU multi-rank tests and the
``python -m afd_plugin_b200.runtime.launcher`` CLI.
"""

from __future__ import annotations

import argparse
import json
import os
import socket
import traceback
from dataclasses import dataclass, field
from datetime import timedelta

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


@dataclass
class LocalAFDSpec:
    preset: str | None = "tiny-dsv2"
    arch: dict | None = None  # explicit ModelArchConfig fields (overrides preset)
    dtype: str = "float32"
    afd: dict = field(default_factory=dict)  # additional_config["afd"]
    prompts: list[list[int]] = field(default_factory=list)
    max_tokens: int = 16
    enforce_eager: bool = True
    use_ubatching: bool = False
    max_model_len: int = 128
    max_num_seqs: int = 8
    seed: int = 0
    backend: str = "gloo"
    capture_sizes: list[int] = field(default_factory=lambda: [8])
    timeout_s: int = 60
    # fault injection on the host (tests): {"rank": r, "kind": "raise"|"exit", "at_step": n}
    fault: dict | None = None
    # attention tensor parallelism: num_attention_ranks = DP x tp
    tp: int = 1
    # HF checkpoint directory: architecture from its config.json, role-filtered weights
    checkpoint: str | None = None
    # Attention ranks return the logits of their first N engine steps (fp32, CPU)
    record_logits_steps: int = 0
    # EngineConfig.async_scheduling on the Attention ranks
    async_scheduling: bool = False


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def build_engine_config(spec: LocalAFDSpec):
    from afd_plugin_b200.engine_config import CompilationConfig, EngineConfig, ModelConfig, ParallelConfig
    from afd_plugin_b200.models.configs import ModelArchConfig, get_preset

    if spec.checkpoint:
        from afd_plugin_b200.models.loader import read_hf_config

        arch = read_hf_config(spec.checkpoint)
    else:
        arch = ModelArchConfig(**spec.arch) if spec.arch else get_preset(spec.preset)
    dtype = getattr(torch, spec.dtype)
    A = int(spec.afd.get("num_attention_ranks", 1))
    return EngineConfig(
        model_config=ModelConfig(arch, dtype=dtype, enforce_eager=spec.enforce_eager,
                                 max_model_len=spec.max_model_len, seed=spec.seed, checkpoint=spec.checkpoint),
        parallel_config=ParallelConfig(data_parallel_size=A // spec.tp, tensor_parallel_size=spec.tp,
                                       use_ubatching=spec.use_ubatching, num_ubatches=2 if spec.use_ubatching else 1),
        compilation_config=CompilationConfig(cudagraph_capture_sizes=list(spec.capture_sizes)),
        additional_config={"afd": dict(spec.afd)},
        max_num_seqs=spec.max_num_seqs,
        async_scheduling=spec.async_scheduling,
    )


def split_prompts(prompts: list[list[int]], n: int) -> list[list[list[int]]]:
    """Contiguous, as-even-as-possible split (rank i gets a consecutive slice)."""
    base, extra = divmod(len(prompts), n)
    out, start = [], 0
    for i in range(n):
        k = base + (1 if i < extra else 0)
        out.append(prompts[start : start + k])
        start += k
    return out


def _rank_main(world_rank: int, world_size: int, rendezvous: str, spec: LocalAFDSpec, results) -> None:
    try:
        from afd_plugin_b200.parallel.topology import role_of_world_rank

        A = int(spec.afd.get("num_attention_ranks", 1))
        F = int(spec.afd.get("num_ffn_ranks", 1))
        role, role_rank = role_of_world_rank(world_rank, attention_size=A, ffn_size=F)
        backend = spec.backend
        local_rank = world_rank
        if backend == "nccl":
            torch.cuda.set_device(local_rank)
        dist.init_process_group(backend=backend, init_method=rendezvous, rank=world_rank, world_size=world_size,
                                timeout=timedelta(seconds=spec.timeout_s))
        afd = dict(spec.afd, role=role)
        spec_local = LocalAFDSpec(**{**spec.__dict__, "afd": afd})
        config = build_engine_config(spec_local)
        fault = spec.fault or {}
        if role == "ffn":
            from afd_plugin_b200.runtime.workers import AFDFFNWorker

            w = AFDFFNWorker(config, local_rank=local_rank)
            if fault.get("rank") == world_rank and fault.get("kind") == "exit_before_serve":
                os._exit(3)
            steps = w.run_ffn_server_loop()
            results.put((world_rank, {"role": role, "steps": steps}))
            w.shutdown()
        else:
            from afd_plugin_b200.runtime.workers import AFDAttentionWorker

            w = AFDAttentionWorker(config, local_rank=local_rank)
            # tensor-parallel peers serve the same requests (their data-parallel rank's share)
            mine = split_prompts(spec.prompts, A // spec.tp)[role_rank // spec.tp]
            ids = [w.engine.add_request(p, spec.max_tokens) for p in mine]
            if not spec.enforce_eager and backend == "nccl":
                w.engine.capture_graphs()
            group = w.groups.attention_group
            step = 0
            logits = []
            while True:
                flag = torch.tensor([int(w.engine.has_unfinished())])
                if A > 1:
                    dist.all_reduce(flag, group=group)
                if int(flag) == 0:
                    break
                if fault.get("rank") == world_rank and fault.get("at_step") == step:
                    if fault.get("kind") == "raise":
                        raise RuntimeError("injected fault")
                    os._exit(3)
                w.engine.step()
                if step < spec.record_logits_steps and w.engine.runner.last_logits is not None:
                    # numpy pickles by value (a tensor would travel as a shared-memory handle
                    # that dies with this process)
                    logits.append(w.engine.runner.last_logits[: len(ids)].float().cpu().numpy())
                step += 1
            outs = [w.engine.finished[i].output for i in ids] if role_rank % spec.tp == 0 else []
            if A > 1:
                dist.barrier(group=group)
            w.shutdown()
            results.put((world_rank, {"role": role, "outputs": outs, "steps": step, "logits": logits,
                                      "async_steps": w.engine.num_async_steps}))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:  # noqa: BLE001 - reported to the parent
        results.put((world_rank, {"error": f"{type(exc).__name__}: {exc}", "trace": traceback.format_exc()}))
        raise


def launch_local(spec: LocalAFDSpec, *, join_timeout_s: float = 180.0) -> dict[int, dict]:
    """Spawn the AFD world; returns ``{world_rank: result}`` (errors included)."""
    A = int(spec.afd.get("num_attention_ranks", 1))
    F = int(spec.afd.get("num_ffn_ranks", 1))
    world = A + F
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    # Rendezvous through a file of a fresh directory: no port to race for
    # (a port probed free can be taken again before rank 0 binds it).
    import shutil
    import tempfile
    import time

    rdv_dir = tempfile.mkdtemp(prefix="afd_rdv_")
    rendezvous = "file://" + os.path.join(rdv_dir, "store")
    procs = [ctx.Process(target=_rank_main, args=(r, world, rendezvous, spec, results), daemon=False)
             for r in range(world)]
    for p in procs:
        p.start()
    deadline = time.time() + join_timeout_s
    for p in procs:
        p.join(timeout=max(0.1, deadline - time.time()))
    out: dict[int, dict] = {}
    while not results.empty():
        r, v = results.get()
        out.setdefault(r, v)
    for r, p in enumerate(procs):
        if p.is_alive():
            p.kill()
            p.join(5)
            out.setdefault(r, {"error": "timeout: rank still running"})
        elif p.exitcode not in (0, None) and r not in out:
            out[r] = {"error": f"exit code {p.exitcode}"}
    shutil.rmtree(rdv_dir, ignore_errors=True)
    return out


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description="Run a local AFD deployment and print generated tokens.")
    ap.add_argument("--preset", default="tiny-dsv2")
    ap.add_argument("--additional-config", default='{"afd": {"num_attention_ranks": 1, "num_ffn_ranks": 1}}')
    ap.add_argument("--num-prompts", type=int, default=4)
    ap.add_argument("--prompt-len", type=int, default=32)
    ap.add_argument("--max-tokens", type=int, default=16)
    ap.add_argument("--backend", default="gloo")
    ap.add_argument("--dtype", default="float32")
    ap.add_argument("--checkpoint", default=None, help="HF checkpoint directory (else --preset, random init)")
    ap.add_argument("--tp", type=int, default=1, help="attention tensor parallelism")
    ap.add_argument("--dbo", action="store_true", help="two-ubatch overlap")
    ap.add_argument("--graphs", action="store_true", help="capture decode CUDA graphs (nccl backend)")
    ap.add_argument("--async-scheduling", action="store_true",
                    help="launch each decode step before the previous step's tokens are read back")
    args = ap.parse_args(argv)
    afd = json.loads(args.additional_config)["afd"]
    from afd_plugin_b200.models.configs import get_preset

    if args.checkpoint:
        from afd_plugin_b200.models.loader import read_hf_config

        vocab = read_hf_config(args.checkpoint).vocab_size
    else:
        vocab = get_preset(args.preset).vocab_size
    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, vocab, (args.num_prompts, args.prompt_len), generator=g).tolist()
    spec = LocalAFDSpec(preset=args.preset, afd=afd, prompts=prompts, max_tokens=args.max_tokens,
                        backend=args.backend, dtype=args.dtype, checkpoint=args.checkpoint, tp=args.tp,
                        use_ubatching=args.dbo, enforce_eager=not args.graphs,
                        async_scheduling=args.async_scheduling)
    res = launch_local(spec)
    print(json.dumps({str(k): v for k, v in sorted(res.items())}))
    return 0 if all("error" not in v for v in res.values()) else 1


if __name__ == "__main__":
    raise SystemExit(main())


__all__ = ["LocalAFDSpec", "build_engine_config", "free_port", "launch_local", "split_prompts"]
