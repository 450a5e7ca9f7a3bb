"""Fixed end-to-end serving scenarios.

The AFD rows keep the names and topologies of the reference's scenario table
(``tests/e2e/runner.py:361-395``: baseline, eager / graph / graph+DBO at 2A1F
and 2A2F, attention TP2); the ``afd-fused-*`` rows run the NVLink-fused
connector.  The baseline is one colocated engine (no AFD) rather than the
reference's DP4 vLLM deployment.
"""

from __future__ import annotations

import json
from dataclasses import dataclass

NCCL = "P2pNcclAFDConnector"
FUSED = "B200FusedAFDConnector"


@dataclass(frozen=True)
class Scenario:
    name: str
    baseline: bool
    graph: bool
    dbo: bool
    attention_ranks: int
    ffn_ranks: int
    connector: str = NCCL
    tp: int = 1  # attention tensor parallelism (attention_ranks = DP x tp)
    # Prefill/decode disaggregation: this scenario's server decodes behind the
    # proxy, and a server of the ``prefill`` scenario runs the prompts.
    prefill: "Scenario | None" = None
    # the server launches each decode step before the previous one's tokens are read back
    async_scheduling: bool = False

    @property
    def world_size(self) -> int:
        """Processes (GPUs) of this scenario's own server (the decode side of a PD scenario)."""
        return 1 if self.baseline else self.attention_ranks + self.ffn_ranks

    @property
    def total_devices(self) -> int:
        return self.world_size + (self.prefill.world_size if self.prefill is not None else 0)

    @property
    def needs_cuda(self) -> bool:
        return self.connector == FUSED or (self.prefill is not None and self.prefill.needs_cuda)

    def afd_config(self, extra: dict | None = None) -> dict:
        if self.baseline:
            return {}
        cfg = {"num_attention_ranks": self.attention_ranks, "num_ffn_ranks": self.ffn_ranks,
               "connector": self.connector}
        if extra:
            cfg["connector_extra_config"] = dict(extra)
        return cfg


def _s(name, baseline, graph, dbo, a, f, connector=NCCL, tp=1, async_scheduling=False) -> tuple[str, Scenario]:
    return name, Scenario(name, baseline, graph, dbo, a, f, connector, tp, async_scheduling=async_scheduling)


def _pd(name, decode: str, prefill: str) -> tuple[str, Scenario]:
    from dataclasses import replace

    return name, replace(_BASE[decode], name=name, prefill=_BASE[prefill])


_BASE: dict[str, Scenario] = dict([
    _s("baseline-eager", True, False, False, 1, 0),
    _s("baseline-graph", True, True, False, 1, 0),
    _s("afd-eager-1a1f", False, False, False, 1, 1),
    _s("afd-eager-2a1f", False, False, False, 2, 1),
    _s("afd-graph-2a1f", False, True, False, 2, 1),
    _s("afd-graph-dbo-2a1f", False, True, True, 2, 1),
    _s("afd-eager-2a2f", False, False, False, 2, 2),
    _s("afd-graph-2a2f", False, True, False, 2, 2),
    _s("afd-graph-dbo-2a2f", False, True, True, 2, 2),
    _s("afd-eager-tp2-1f", False, False, False, 2, 1, tp=2),
    _s("afd-graph-tp2-2f", False, True, False, 2, 2, tp=2),
    _s("afd-fused-graph-1a1f", False, True, False, 1, 1, FUSED),
    _s("afd-fused-graph-2a2f", False, True, False, 2, 2, FUSED),
    _s("afd-fused-graph-dbo-2a2f", False, True, True, 2, 2, FUSED),
    _s("afd-fused-graph-6a2f", False, True, False, 6, 2, FUSED),
    # async scheduling: greedy tokens must equal the synchronous rows'
    _s("baseline-graph-async", True, True, False, 1, 0, async_scheduling=True),
    _s("afd-graph-2a2f-async", False, True, False, 2, 2, async_scheduling=True),
    _s("afd-fused-graph-2a2f-async", False, True, False, 2, 2, FUSED, async_scheduling=True),
])

# Prefill on a colocated server, decode on an AFD deployment, the proxy in front.
SCENARIOS: dict[str, Scenario] = dict(_BASE, **dict([
    _pd("pd-baseline-to-afd-eager-1a1f", "afd-eager-1a1f", "baseline-eager"),
    _pd("pd-baseline-to-afd-eager-2a1f", "afd-eager-2a1f", "baseline-eager"),
    _pd("pd-baseline-to-afd-fused-graph-1a1f", "afd-fused-graph-1a1f", "baseline-graph"),
]))


def server_command(scn: Scenario, *, python: str, preset: str, port: int, master_port: int,
                   checkpoint: str | None = None, dtype: str = "bfloat16", max_num_seqs: int = 16,
                   max_model_len: int = 2048, capture_size: int = 8, seed: int = 0,
                   connector_extra: dict | None = None) -> list[str]:
    """The command line that serves ``scn`` on ``port`` (torchrun for AFD worlds)."""
    serve = ["-m", "afd_plugin_b200.serving", "--preset", preset, "--dtype", dtype, "--port", str(port),
             "--host", "127.0.0.1", "--max-num-seqs", str(max_num_seqs), "--max-model-len", str(max_model_len),
             "--seed", str(seed)]
    if checkpoint:
        serve += ["--checkpoint", checkpoint]
    if scn.graph:
        serve += ["--capture-sizes", str(min(capture_size, max_num_seqs))]
    else:
        serve += ["--eager"]
    if scn.dbo:
        serve += ["--dbo"]
    if scn.tp > 1:
        serve += ["--tp", str(scn.tp)]
    if scn.async_scheduling:
        serve += ["--async-scheduling"]
    if scn.baseline:
        return [python, *serve]
    serve += ["--afd", json.dumps(scn.afd_config(connector_extra), separators=(",", ":"))]
    return [python, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", str(scn.world_size),
            "--master-addr", "127.0.0.1", "--master-port", str(master_port), *serve]


__all__ = ["FUSED", "NCCL", "SCENARIOS", "Scenario", "server_command"]
